// GPTQ and SparseGPT column-block solve.
//
// Reference: GptqBlockQuantizer.Quantize (src/LLMCompressorSharp.Core/Algorithms/Gptq/
// GptqBlockQuantizer.cs:71-190), ComputeScaleZeroPoint (:196-234), FakeQuantizeColumn
// (:240-274); SparseGPT per the plan docs/superpowers/plans/2026-05-18-phase-4c-sparsegpt.md
// (:37-59, :1584-1656) in the same U-factor form.
//
// Rows are independent given U, so one thread owns one output row of the current block
// of <= 128 columns and keeps that row segment in registers.  The 128 sequential column
// steps (quantise, err = (w-q)/U[j][j], rank-1 update of the rest of the block) then run
// with no global traffic: U's diagonal block sits in shared memory and is read as
// broadcasts.  The block's W tile and its outputs move through shared memory so that
// every global access is coalesced.  The lazy tail update W[:, i2:] -= Err1 U[i1:i2, i2:]
// is a GEMM (gemm_f32) with Err1 stored transposed [cnt, m].
#include "ops.h"

namespace llmc {
namespace {

constexpr int BW = 128;     // columns per block held in registers
constexpr int ROWS = 64;    // rows (threads) per CTA
constexpr int WPAD = BW + 4;

struct BlockArgs {
    float* W; int64_t ldw;             // fp32 working copy; quantised values written back in place
    int64_t m, n;
    int64_t i1; int cnt;
    const float* U; int64_t ldu;
    // quantisation
    int bits, sym;
    const float* scales; const int32_t* zps;
    int64_t srow;   // scale entries per row (0 tensor, 1 channel, G group)
    int64_t gs;     // columns per scale entry along a row (n for tensor/channel)
    uint8_t* codes; int64_t crow;  // packed (bits<=4) or bytes; nullable
    float* err1t;   // [BW, m]
    // SparseGPT
    float sparsity; int mask_n, mask_m;
    uint8_t* mask; int64_t mrow;   // nullable, one byte per element
};

size_t block_smem_bytes() { return (size_t)BW * BW * 4 + (size_t)ROWS * WPAD * 4 + (size_t)ROWS * BW; }

// Keep mask of one row's block (SparseGPT): per-row top-k (unstructured) or N:M, ties to
// the lower column index.  sal points at the row's non-negative saliencies in shared
// memory (run-time indexed); the result is a 128-bit mask.
__device__ void select_keep(const float* sal, int cnt, float sparsity, int mask_n, int mask_m, unsigned (&bits)[BW / 32]) {
#pragma unroll
    for (int i = 0; i < BW / 32; i++) bits[i] = 0u;
    if (mask_m > 0) {
        for (int c = 0; c < cnt; c++) {
            const int g0 = (c / mask_m) * mask_m;
            const float sc = sal[c];
            int rank = 0;
            for (int o = g0; o < g0 + mask_m && o < cnt; o++) {
                const float so = sal[o];
                if (so > sc || (so == sc && o < c)) rank++;
            }
            if (rank < mask_n) bits[c / 32] |= 1u << (c % 32);
        }
        return;
    }
    const int k = (int)ceil((1.0 - (double)sparsity) * (double)cnt - 1e-9);
    if (k <= 0) return;
    // Largest threshold T (as ordered bits of a non-negative float) with #{sal >= T} >= k.
    unsigned prefix = 0;
    for (int bit = 31; bit >= 0; bit--) {
        const unsigned cand = prefix | (1u << bit);
        int count = 0;
        for (int c = 0; c < cnt; c++) count += (__float_as_uint(sal[c]) >= cand) ? 1 : 0;
        if (count >= k) prefix = cand;
    }
    int above = 0;
    for (int c = 0; c < cnt; c++) above += (__float_as_uint(sal[c]) > prefix) ? 1 : 0;
    int need = k - above;
    for (int c = 0; c < cnt; c++) {
        const unsigned b = __float_as_uint(sal[c]);
        bool kp = b > prefix;
        if (!kp && b == prefix && need > 0) {
            kp = true;
            need--;
        }
        if (kp) bits[c / 32] |= 1u << (c % 32);
    }
}

template <int MODE>  // 0 = GPTQ quantise, 1 = SparseGPT prune
__global__ void __launch_bounds__(ROWS) block_kernel(BlockArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    float* Us = reinterpret_cast<float*>(smem);                 // [BW][BW]
    float* Wt = Us + BW * BW;                                   // [ROWS][WPAD]
    uint8_t* Ct = reinterpret_cast<uint8_t*>(Wt + ROWS * WPAD); // [ROWS][BW]
    const int tid = threadIdx.x;
    const int64_t r0 = (int64_t)blockIdx.x * ROWS;
    const int cnt = a.cnt;

    for (int t = tid; t < BW * BW; t += ROWS) {
        const int j = t / BW, c = t % BW;
        Us[t] = (j < cnt && c < cnt) ? a.U[(a.i1 + j) * a.ldu + a.i1 + c] : 0.f;
    }
    for (int t = tid; t < ROWS * BW; t += ROWS) {
        const int rr = t / BW, c = t % BW;
        const int64_t R = r0 + rr;
        Wt[rr * WPAD + c] = (R < a.m && c < cnt) ? a.W[R * a.ldw + a.i1 + c] : 0.f;
    }
    __syncthreads();

    const int64_t R = r0 + tid;
    const bool row_ok = R < a.m;
    float w[BW];
#pragma unroll
    for (int c = 0; c < BW; c += 4) {
        float4 v = *reinterpret_cast<const float4*>(&Wt[tid * WPAD + c]);
        w[c] = v.x; w[c + 1] = v.y; w[c + 2] = v.z; w[c + 3] = v.w;
    }

    unsigned keep[BW / 32] = {0u, 0u, 0u, 0u};
    if constexpr (MODE == 1) {
        // Saliency w^2 / U[c][c]^2 from the block snapshot, staged in this thread's row of
        // the W tile (the original values already live in registers).
#pragma unroll
        for (int c = 0; c < BW; c++) {
            const float d = Us[c * BW + c];
            Wt[tid * WPAD + c] = __fdiv_rn(__fmul_rn(w[c], w[c]), fmaxf(__fmul_rn(d, d), 1e-10f));
        }
        select_keep(&Wt[tid * WPAD], cnt, a.sparsity, a.mask_n, a.mask_m, keep);
    }

    float qmin, qmax;
    qrange(a.bits, a.sym, &qmin, &qmax);
    // Scale entry of the current column: reloaded when the column crosses a group edge.
    int64_t g = a.i1 / a.gs;
    int64_t next_edge = (g + 1) * a.gs - a.i1;  // block-relative column where g changes
    float s = 1.f, zf = 0.f;
    int zi = 0;
    if constexpr (MODE == 0) {
        const int64_t si = row_ok ? R * a.srow + g : 0;
        s = a.scales[si];
        zi = a.zps[si];
        zf = (float)zi;
    }

#pragma unroll
    for (int j = 0; j < BW; j++) {
        if (j < cnt) {
            float q;
            uint8_t cb;
            if constexpr (MODE == 0) {
                if (j == next_edge) {
                    g++;
                    next_edge += a.gs;
                    const int64_t si = row_ok ? R * a.srow + g : 0;
                    s = a.scales[si];
                    zi = a.zps[si];
                    zf = (float)zi;
                }
                int code;
                q = fq_chain<float>(w[j], s, zf, qmin, qmax, &code);
                cb = a.bits <= 4 ? (uint8_t)((code - zi) & 0xF) : (uint8_t)code;
            } else {
                const bool kj = (keep[j / 32] >> (j % 32)) & 1u;
                q = kj ? w[j] : 0.f;
                cb = kj ? 1 : 0;
            }
            Wt[tid * WPAD + j] = q;
            Ct[tid * BW + j] = cb;
            const float piv = Us[j * BW + j];
            float err = 0.f;
            if (fabsf(piv) >= 1e-10f) {  // GptqBlockQuantizer.cs:146-150 (NumericEpsilon)
                err = __fdiv_rn(__fsub_rn(w[j], q), piv);
#pragma unroll
                for (int c4 = 0; c4 < BW / 4; c4++) {  // constant trip count: folds after unrolling
                    if (4 * c4 + 3 <= j) continue;
                    const float4 u = *reinterpret_cast<const float4*>(&Us[j * BW + 4 * c4]);
                    if (4 * c4 + 0 > j) w[4 * c4 + 0] = fmaf(-err, u.x, w[4 * c4 + 0]);
                    if (4 * c4 + 1 > j) w[4 * c4 + 1] = fmaf(-err, u.y, w[4 * c4 + 1]);
                    if (4 * c4 + 2 > j) w[4 * c4 + 2] = fmaf(-err, u.z, w[4 * c4 + 2]);
                    if (4 * c4 + 3 > j) w[4 * c4 + 3] = fmaf(-err, u.w, w[4 * c4 + 3]);
                }
            }
            if (row_ok) a.err1t[(int64_t)j * a.m + R] = err;
        }
    }
    __syncthreads();

    // Write back the quantised (or pruned) values in place.
    for (int t = tid; t < ROWS * BW; t += ROWS) {
        const int rr = t / BW, c = t % BW;
        const int64_t RR = r0 + rr;
        if (RR < a.m && c < cnt) a.W[RR * a.ldw + a.i1 + c] = Wt[rr * WPAD + c];
    }
    if (MODE == 0 && a.codes) {
        if (a.bits <= 4) {
            const int64_t b0 = a.i1 / 2, b1 = (a.i1 + cnt - 1) / 2;
            const int nb = (int)(b1 - b0 + 1);
            for (int t = tid; t < ROWS * nb; t += ROWS) {
                const int rr = t / nb;
                const int64_t b = b0 + t % nb;
                const int64_t RR = r0 + rr;
                if (RR >= a.m) continue;
                uint8_t* p = a.codes + RR * a.crow + b;
                const int64_t ch = 2 * b, cl = 2 * b + 1;
                const bool hi_in = ch >= a.i1 && ch < a.i1 + cnt;
                const bool lo_in = cl >= a.i1 && cl < a.i1 + cnt && cl < a.n;
                uint8_t v = (hi_in && (lo_in || cl >= a.n)) ? 0 : *p;
                if (hi_in) v = (uint8_t)((v & 0x0F) | (Ct[rr * BW + (ch - a.i1)] << 4));
                if (lo_in) v = (uint8_t)((v & 0xF0) | Ct[rr * BW + (cl - a.i1)]);
                *p = v;
            }
        } else {
            for (int t = tid; t < ROWS * BW; t += ROWS) {
                const int rr = t / BW, c = t % BW;
                const int64_t RR = r0 + rr;
                if (RR < a.m && c < cnt) a.codes[RR * a.crow + a.i1 + c] = Ct[rr * BW + c];
            }
        }
    }
    if (MODE == 1 && a.mask) {
        for (int t = tid; t < ROWS * BW; t += ROWS) {
            const int rr = t / BW, c = t % BW;
            const int64_t RR = r0 + rr;
            if (RR < a.m && c < cnt) a.mask[RR * a.mrow + a.i1 + c] = Ct[rr * BW + c];
        }
    }
}

template <int MODE>
llmc_status run_blocks(llmc_ctx* ctx, BlockArgs a, int block_size) {
    static bool attr_set = false;
    const size_t smem = block_smem_bytes();
    if (!attr_set) {
        LLMC_CUDA_TRY(cudaFuncSetAttribute(block_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr_set = true;
    }
    const int bs = block_size < 1 ? BW : (block_size > BW ? BW : block_size);
    const unsigned grid = (unsigned)((a.m + ROWS - 1) / ROWS);
    for (int64_t i1 = 0; i1 < a.n; i1 += bs) {
        const int cnt = (int)min((int64_t)bs, a.n - i1);
        a.i1 = i1;
        a.cnt = cnt;
        block_kernel<MODE><<<grid, ROWS, smem, ctx->stream>>>(a);
        LLMC_TRY(check_launch(ctx, "gptq_block"));
        const int64_t i2 = i1 + cnt;
        if (i2 < a.n) {
            // W[:, i2:] -= Err1 @ U[i1:i2, i2:]   (GptqBlockQuantizer.cs:173-180)
            GemmArgs g{a.m, a.n - i2, cnt, a.err1t, a.m, 1, LLMC_DTYPE_F32, a.U + i1 * a.ldu + i2, a.ldu, 0,
                       LLMC_DTYPE_F32, a.W + i2, a.ldw, -1.f, 1.f};
            LLMC_TRY(gemm_f32(ctx, g));
        }
    }
    return LLMC_OK;
}

}  // namespace

llmc_status gptq(llmc_ctx* ctx, const void* W, int dtype, int64_t m, int64_t n, int64_t ldw, const float* U, int64_t ldu,
                 const llmc_qconfig* cfg, float* wq_out, int64_t ldq, uint8_t* codes, float* scales_out,
                 int32_t* zps_out, int mode, uint8_t* mask_out) {
    const int strategy = cfg->strategy;
    const int64_t gs = strategy == LLMC_STRATEGY_GROUP ? cfg->group_size : n;
    const int64_t G = n_groups(strategy, n, gs);
    const int64_t nparams = strategy == LLMC_STRATEGY_TENSOR ? 1 : m * G;
    // Scratch: working copy (unless the caller's wq_out is used), Err1^T, params, reduction.
    const bool own_work = wq_out == nullptr;
    size_t need = 0;
    need += own_work ? (size_t)m * n * 4 + 256 : 0;
    need += (size_t)BW * m * 4 + 256;
    need += (size_t)nparams * 2 * 8 + 512;        // mins/maxs (+ scales/zps when not returned)
    need += (size_t)(2 * m + 128) * 4 + 256;      // per-tensor reduction scratch
    void* wsp;
    LLMC_TRY(workspace(ctx, need, &wsp));
    Carver cv{(char*)wsp};
    float* work = own_work ? cv.take<float>((size_t)m * n) : wq_out;
    const int64_t ldwork = own_work ? n : ldq;
    float* err1t = cv.take<float>((size_t)BW * m);
    float* mins = cv.take<float>(nparams);
    float* maxs = cv.take<float>(nparams);
    float* scales = scales_out ? scales_out : cv.take<float>(nparams);
    int32_t* zps = zps_out ? zps_out : cv.take<int32_t>(nparams);
    float* red = cv.take<float>(2 * m + 128);

    BlockArgs a{};
    a.W = work; a.ldw = ldwork; a.m = m; a.n = n;
    a.U = U; a.ldu = ldu;
    a.bits = cfg->num_bits; a.sym = cfg->symmetric;
    a.err1t = err1t;
    if (mode == 0) {
        // ComputeScaleZeroPoint from the ORIGINAL weight (GptqBlockQuantizer.cs:97, :196-234).
        LLMC_TRY(minmax(ctx, W, dtype, m, n, ldw, strategy, gs, mins, maxs, 0, red));
        LLMC_TRY(affine(ctx, mins, maxs, nparams, cfg->num_bits, cfg->symmetric, scales, zps));
        a.scales = scales; a.zps = zps;
        a.srow = strategy == LLMC_STRATEGY_TENSOR ? 0 : (strategy == LLMC_STRATEGY_CHANNEL ? 1 : G);
        a.gs = strategy == LLMC_STRATEGY_GROUP ? gs : n;
        a.codes = codes;
        a.crow = cfg->num_bits <= 4 ? (n + 1) / 2 : n;
    } else {
        a.srow = 0; a.gs = n;
        a.sparsity = cfg->sparsity; a.mask_n = cfg->mask_n; a.mask_m = cfg->mask_m;
        a.mask = mask_out; a.mrow = n;
    }
    LLMC_TRY(convert_to_f32(ctx, W, dtype, m, n, ldw, work, ldwork));
    if (mode == 0) return run_blocks<0>(ctx, a, cfg->block_size);
    return run_blocks<1>(ctx, a, cfg->block_size);
}

}  // namespace llmc
