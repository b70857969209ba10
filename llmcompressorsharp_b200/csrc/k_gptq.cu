// GPTQ and SparseGPT column-block solve.
//
// Reference: GptqBlockQuantizer.Quantize (src/LLMCompressorSharp.Core/Algorithms/Gptq/
// GptqBlockQuantizer.cs:71-190), ComputeScaleZeroPoint (:196-234), FakeQuantizeColumn
// (:240-274); SparseGPT per the plan docs/superpowers/plans/2026-05-18-phase-4c-sparsegpt.md
// (:37-59, :1584-1656) in the same U-factor form.
//
// Rows are independent given U, so one thread owns one output row of the current block of
// <= 128 columns.  The block is processed as four 32-column sub-blocks: a sub-block's row
// segment lives in registers and its 32 sequential column steps (quantise, err = (w-q)/U[j][j],
// rank-1 update of the rest of the sub-block) are fully unrolled; the sub-block's 32 errors
// then update the block's later columns, which wait in shared memory, in a rolled loop
// (U rows are shared-memory broadcasts).  This keeps the code small enough for the
// instruction cache.  The lazy tail update W[:, i2:] -= Err1 U[i1:i2, i2:] is a GEMM with
// Err1 stored transposed [cnt, m].
//
// Several weights that share one U (q/k/v, gate/up) are solved as one stacked matrix.
#include "ops.h"

namespace llmc {
namespace {

constexpr int BW = 128;      // columns per block
constexpr int SB = 32;       // columns per register sub-block
constexpr int ROWS = 64;     // rows (threads) per CTA
constexpr int WLD = ROWS + 1;  // column-major W tile: element (row r, col c) at c*WLD + r

struct BlockArgs {
    float* W; int64_t ldw;             // fp32 working copy; quantised values written back in place
    int64_t m, n;
    int64_t i1; int cnt;
    const float* U; int64_t ldu;
    // quantisation
    int bits, sym;
    const float* scales; const int32_t* zps;
    int64_t srow;   // scale entries per row (0 tensor, 1 channel / per-row, G group)
    int64_t gs;     // columns per scale entry along a row (n for tensor/channel)
    uint8_t* codes; int64_t crow;  // packed (bits<=4) or bytes; nullable
    int codes_bytes;               // 1: one byte per code even for bits <= 4 (act_order scatters them)
    const int32_t* col_group;      // act_order: scale entry (group) of each column; nullable
    float* err1t;   // [cnt, m] errors of the current block (inside the super-block's buffer)
    // SparseGPT
    float sparsity; int mask_n, mask_m;
    uint8_t* mask; int64_t mrow;   // nullable, one byte per element
};

template <int MODE>
constexpr size_t block_smem_bytes() {
    return (size_t)BW * BW * 4 + (size_t)BW * WLD * 4 + (size_t)BW * ROWS + (MODE == 1 ? (size_t)BW * WLD * 4 : 0) +
           (size_t)BW * 4;
}

// Keep mask of one row's block (SparseGPT): per-row top-k (unstructured) or N:M, ties to
// the lower column index.  sal[c * WLD] holds the row's non-negative saliencies.
__device__ void select_keep(const float* sal, int cnt, float sparsity, int mask_n, int mask_m, unsigned (&bits)[BW / 32]) {
#pragma unroll
    for (int i = 0; i < BW / 32; i++) bits[i] = 0u;
    if (mask_m > 0) {
        for (int c = 0; c < cnt; c++) {
            const int g0 = (c / mask_m) * mask_m;
            const float sc = sal[c * WLD];
            int rank = 0;
            for (int o = g0; o < g0 + mask_m && o < cnt; o++) {
                const float so = sal[o * WLD];
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
        for (int c = 0; c < cnt; c++) count += (__float_as_uint(sal[c * WLD]) >= cand) ? 1 : 0;
        if (count >= k) prefix = cand;
    }
    int above = 0;
    for (int c = 0; c < cnt; c++) above += (__float_as_uint(sal[c * WLD]) > prefix) ? 1 : 0;
    int need = k - above;
    for (int c = 0; c < cnt; c++) {
        const unsigned b = __float_as_uint(sal[c * WLD]);
        bool kp = b > prefix;
        if (!kp && b == prefix && need > 0) {
            kp = true;
            need--;
        }
        if (kp) bits[c / 32] |= 1u << (c % 32);
    }
}

__device__ __forceinline__ uint32_t smem_u32_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

template <int MODE>  // 0 = GPTQ quantise, 1 = SparseGPT prune
__global__ void __launch_bounds__(ROWS) block_kernel(BlockArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    float* Us = reinterpret_cast<float*>(smem);                  // [BW][BW] row-major
    float* Wt = Us + BW * BW;                                    // [BW][WLD] column-major tile
    uint8_t* Ct = reinterpret_cast<uint8_t*>(Wt + BW * WLD);     // [BW][ROWS] codes / mask bytes
    float* Sal = reinterpret_cast<float*>(Ct + BW * ROWS);       // MODE 1: [BW][WLD] saliencies
    float* Rp = Sal + (MODE == 1 ? BW * WLD : 0);                // [BW] reciprocals of U's diagonal
    const int tid = threadIdx.x;
    const int64_t r0 = (int64_t)blockIdx.x * ROWS;
    const int cnt = a.cnt;

    // U block: 16-byte asynchronous copies, all in flight at once (zero-filled past cnt).
    // W tile: 16-byte loads eight at a time, scattered into the column-major tile.
    const bool vec = ((reinterpret_cast<uintptr_t>(a.U) | reinterpret_cast<uintptr_t>(a.W)) % 16 == 0) &&
                     a.ldu % 4 == 0 && a.ldw % 4 == 0 && a.i1 % 4 == 0;
    if (vec) {
        for (int t = tid; t < BW * BW / 4; t += ROWS) {
            const int j = t / (BW / 4), c = (t % (BW / 4)) * 4;
            const int valid = (j < cnt) ? max(0, min(4, cnt - c)) : 0;
            const float* src = valid ? a.U + (a.i1 + j) * a.ldu + a.i1 + c : a.U;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32_addr(&Us[j * BW + c])),
                         "l"(src), "r"(valid * 4)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        constexpr int PER = ROWS * BW / 4 / ROWS;  // float4 per thread (32)
        constexpr int BATCH = 8;
#pragma unroll 1
        for (int b0 = 0; b0 < PER; b0 += BATCH) {
            float4 v[BATCH];
#pragma unroll
            for (int k = 0; k < BATCH; k++) {
                const int t = tid + (b0 + k) * ROWS;
                const int rr = t / (BW / 4), c = (t % (BW / 4)) * 4;
                const int64_t R = r0 + rr;
                if (R < a.m && c + 3 < cnt) {
                    v[k] = *reinterpret_cast<const float4*>(a.W + R * a.ldw + a.i1 + c);
                } else {
                    float e[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) e[i] = (R < a.m && c + i < cnt) ? a.W[R * a.ldw + a.i1 + c + i] : 0.f;
                    v[k] = make_float4(e[0], e[1], e[2], e[3]);
                }
            }
#pragma unroll
            for (int k = 0; k < BATCH; k++) {
                const int t = tid + (b0 + k) * ROWS;
                const int rr = t / (BW / 4), c = (t % (BW / 4)) * 4;
                Wt[(c + 0) * WLD + rr] = v[k].x;
                Wt[(c + 1) * WLD + rr] = v[k].y;
                Wt[(c + 2) * WLD + rr] = v[k].z;
                Wt[(c + 3) * WLD + rr] = v[k].w;
            }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else {
        for (int t = tid; t < BW * BW; t += ROWS) {
            const int j = t / BW, c = t % BW;
            Us[t] = (j < cnt && c < cnt) ? a.U[(a.i1 + j) * a.ldu + a.i1 + c] : 0.f;
        }
        for (int t = tid; t < ROWS * BW; t += ROWS) {
            const int rr = t / BW, c = t % BW;
            const int64_t R = r0 + rr;
            Wt[c * WLD + rr] = (R < a.m && c < cnt) ? a.W[R * a.ldw + a.i1 + c] : 0.f;
        }
    }
    __syncthreads();
    for (int c = tid; c < BW; c += ROWS) Rp[c] = __frcp_rn(Us[c * BW + c]);
    __syncthreads();

    const int64_t R = r0 + tid;
    const bool row_ok = R < a.m;

    unsigned keep[BW / 32] = {0u, 0u, 0u, 0u};
    if constexpr (MODE == 1) {
        // Saliency w^2 / U[c][c]^2 from the block snapshot (before any in-block update).
        for (int c = 0; c < BW; c++) {
            const float w = Wt[c * WLD + tid];
            const float d = Us[c * BW + c];
            Sal[c * WLD + tid] = __fdiv_rn(__fmul_rn(w, w), fmaxf(__fmul_rn(d, d), 1e-10f));
        }
        select_keep(&Sal[tid], cnt, a.sparsity, a.mask_n, a.mask_m, keep);
    }

    float qmin, qmax;
    qrange(a.bits, a.sym, &qmin, &qmax);
    // Scale entry of the current column: reloaded when the column crosses a group edge (or,
    // with a column-group map, when the map changes group).
    int64_t g = a.col_group ? a.col_group[a.i1] : a.i1 / a.gs;
    int64_t next_edge = (g + 1) * a.gs - a.i1;  // block-relative column where g changes
    // rs = rcp(s): x * rs stands in for x / s except within a few units in the last place of
    // a half-integer (where rint could differ) or when rs is not finite; those take the exact
    // op-by-op chain, so the code and the value equal the chain's.
    float s = 1.f, zf = 0.f, rs = 1.f;
    bool rs_ok = true;
    int zi = 0;
    if constexpr (MODE == 0) {
        const int64_t si = row_ok ? R * a.srow + g : 0;
        s = a.scales[si];
        zi = a.zps[si];
        zf = (float)zi;
        rs = __frcp_rn(s);
        rs_ok = fabsf(rs) <= 3.0e38f && rs != 0.f;
    }

    for (int c0 = 0; c0 < cnt; c0 += SB) {
        float w[SB], e[SB];
#pragma unroll
        for (int c = 0; c < SB; c++) w[c] = Wt[(c0 + c) * WLD + tid];
#pragma unroll
        for (int j = 0; j < SB; j++) {
            const int jj = c0 + j;
            e[j] = 0.f;
            if (jj < cnt) {
                float q;
                uint8_t cb;
                if constexpr (MODE == 0) {
                    bool reload = false;
                    if (a.col_group) {
                        const int64_t gc = a.col_group[a.i1 + jj];
                        reload = gc != g;
                        g = gc;
                    } else if (jj == next_edge) {
                        g++;
                        next_edge += a.gs;
                        reload = true;
                    }
                    if (reload) {
                        const int64_t si = row_ok ? R * a.srow + g : 0;
                        s = a.scales[si];
                        zi = a.zps[si];
                        zf = (float)zi;
                        rs = __frcp_rn(s);
                        rs_ok = fabsf(rs) <= 3.0e38f && rs != 0.f;
                    }
                    int code;
                    const float f = __fmul_rn(w[j], rs);
                    const float fr = rintf(f);
                    const float dd = fabsf(__fsub_rn(f, fr));
                    if (!rs_ok || fabsf(dd - 0.5f) <= fabsf(f) * 4.8e-7f + 1e-30f) {
                        q = fq_chain<float>(w[j], s, zf, qmin, qmax, &code);
                    } else {
                        float t = __fadd_rn(fr, zf);
                        t = (t < qmin) ? qmin : ((t > qmax) ? qmax : t);
                        code = (int)t;
                        q = __fmul_rn(__fsub_rn(t, zf), s);
                    }
                    cb = a.bits <= 4 ? (uint8_t)((code - zi) & 0xF) : (uint8_t)code;
                } else {
                    const bool kj = (keep[jj / 32] >> (jj % 32)) & 1u;
                    q = kj ? w[j] : 0.f;
                    cb = kj ? 1 : 0;
                }
                Wt[jj * WLD + tid] = q;
                Ct[jj * ROWS + tid] = cb;
                const float piv = Us[jj * BW + jj];
                if (fabsf(piv) >= 1e-10f) {  // GptqBlockQuantizer.cs:146-150 (NumericEpsilon)
                    // (w - q) / piv: reciprocal times the difference, then one residual correction
                    // (Markstein), within one unit in the last place of the IEEE quotient.
                    const float df = __fsub_rn(w[j], q);
                    const float rp = Rp[jj];
                    const float q0 = __fmul_rn(df, rp);
                    const float err = fmaf(fmaf(-q0, piv, df), rp, q0);
                    e[j] = err;
#pragma unroll
                    for (int c4 = 0; c4 < SB / 4; c4++) {  // constant trip count: folds after unrolling
                        if (4 * c4 + 3 <= j) continue;
                        const float4 u = *reinterpret_cast<const float4*>(&Us[jj * BW + c0 + 4 * c4]);
                        if (4 * c4 + 0 > j) w[4 * c4 + 0] = fmaf(-err, u.x, w[4 * c4 + 0]);
                        if (4 * c4 + 1 > j) w[4 * c4 + 1] = fmaf(-err, u.y, w[4 * c4 + 1]);
                        if (4 * c4 + 2 > j) w[4 * c4 + 2] = fmaf(-err, u.z, w[4 * c4 + 2]);
                        if (4 * c4 + 3 > j) w[4 * c4 + 3] = fmaf(-err, u.w, w[4 * c4 + 3]);
                    }
                }
                if (row_ok) a.err1t[(int64_t)jj * a.m + R] = e[j];
            }
        }
        // This sub-block's errors update the block's later columns (shared memory).
        for (int c = c0 + SB; c < cnt; c += 4) {
            float v0 = Wt[(c + 0) * WLD + tid], v1 = Wt[(c + 1) * WLD + tid];
            float v2 = Wt[(c + 2) * WLD + tid], v3 = Wt[(c + 3) * WLD + tid];
#pragma unroll
            for (int j = 0; j < SB; j++) {
                const float4 u = *reinterpret_cast<const float4*>(&Us[(c0 + j) * BW + c]);
                v0 = fmaf(-e[j], u.x, v0);
                v1 = fmaf(-e[j], u.y, v1);
                v2 = fmaf(-e[j], u.z, v2);
                v3 = fmaf(-e[j], u.w, v3);
            }
            Wt[(c + 0) * WLD + tid] = v0;
            Wt[(c + 1) * WLD + tid] = v1;
            Wt[(c + 2) * WLD + tid] = v2;
            Wt[(c + 3) * WLD + tid] = v3;
        }
    }
    __syncthreads();

    // Write back the quantised (or pruned) values in place.
    if (vec) {
        for (int t = tid; t < ROWS * BW / 4; t += ROWS) {
            const int rr = t / (BW / 4), c = (t % (BW / 4)) * 4;
            const int64_t RR = r0 + rr;
            if (RR >= a.m) continue;
            if (c + 3 < cnt) {
                *reinterpret_cast<float4*>(a.W + RR * a.ldw + a.i1 + c) =
                    make_float4(Wt[c * WLD + rr], Wt[(c + 1) * WLD + rr], Wt[(c + 2) * WLD + rr], Wt[(c + 3) * WLD + rr]);
            } else {
                for (int i = 0; i < 4 && c + i < cnt; i++) a.W[RR * a.ldw + a.i1 + c + i] = Wt[(c + i) * WLD + rr];
            }
        }
    } else {
        for (int t = tid; t < ROWS * BW; t += ROWS) {
            const int rr = t / BW, c = t % BW;
            const int64_t RR = r0 + rr;
            if (RR < a.m && c < cnt) a.W[RR * a.ldw + a.i1 + c] = Wt[c * WLD + rr];
        }
    }
    if (MODE == 0 && a.codes) {
        if (a.bits <= 4 && !a.codes_bytes) {
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
                if (hi_in) v = (uint8_t)((v & 0x0F) | (Ct[(ch - a.i1) * ROWS + rr] << 4));
                if (lo_in) v = (uint8_t)((v & 0xF0) | Ct[(cl - a.i1) * ROWS + rr]);
                *p = v;
            }
        } else {
            for (int t = tid; t < ROWS * BW; t += ROWS) {
                const int rr = t / BW, c = t % BW;
                const int64_t RR = r0 + rr;
                if (RR < a.m && c < cnt) a.codes[RR * a.crow + a.i1 + c] = Ct[c * ROWS + rr];
            }
        }
    }
    if (MODE == 1 && a.mask) {
        for (int t = tid; t < ROWS * BW; t += ROWS) {
            const int rr = t / BW, c = t % BW;
            const int64_t RR = r0 + rr;
            if (RR < a.m && c < cnt) a.mask[RR * a.mrow + a.i1 + c] = Ct[c * ROWS + rr];
        }
    }
}

// Per-tensor parameters of one weight replicated over its rows (batched per-tensor GPTQ).
__global__ void expand_rows_kernel(const float* s, const int32_t* z, int64_t rows, float* rs, int32_t* rz) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += (int64_t)gridDim.x * blockDim.x) {
        rs[i] = s[0];
        rz[i] = z[0];
    }
}

// Columns whose block errors are applied to the far tail in one GEMM: the tail update
// W[:, i2:] -= Err1 U[i1:i2, i2:] of GptqBlockQuantizer.cs:173-180 is split into a near part
// (inside the super-block, after every block) and a far part (after the super-block, one
// K = SUPER product).  The sum is the same; the fp32 tail of W is rewritten 4x less often.
constexpr int SUPER_BLOCKS = 4;

template <int MODE>
llmc_status run_blocks(llmc_ctx* ctx, BlockArgs a, int block_size) {
    static bool attr_set = false;
    const size_t smem = block_smem_bytes<MODE>();
    if (!attr_set) {
        LLMC_CUDA_TRY(cudaFuncSetAttribute(block_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr_set = true;
    }
    const int bs = block_size < 1 ? BW : (block_size > BW ? BW : block_size);
    const int64_t super = (int64_t)bs * SUPER_BLOCKS;
    const unsigned grid = (unsigned)((a.m + ROWS - 1) / ROWS);
    float* err_all = a.err1t;  // [super, m]: the super-block's errors, block after block
    for (int64_t s0 = 0; s0 < a.n; s0 += super) {
        const int64_t s1 = min(a.n, s0 + super);
        for (int64_t i1 = s0; i1 < s1; i1 += bs) {
            const int cnt = (int)min((int64_t)bs, s1 - i1);
            a.i1 = i1;
            a.cnt = cnt;
            a.err1t = err_all + (i1 - s0) * a.m;
            block_kernel<MODE><<<grid, ROWS, smem, ctx->stream>>>(a);
            LLMC_TRY(check_launch(ctx, "gptq_block"));
            const int64_t i2 = i1 + cnt;
            if (i2 < s1) {  // near: W[:, i2:s1] -= Err1 U[i1:i2, i2:s1]
                GemmArgs gm{a.m, s1 - i2, cnt, a.err1t, a.m, 1, LLMC_DTYPE_F32, a.U + i1 * a.ldu + i2, a.ldu, 0,
                            LLMC_DTYPE_F32, a.W + i2, a.ldw, -1.f, 1.f};
                LLMC_TRY(gemm_f32(ctx, gm));
            }
        }
        if (s1 < a.n) {  // far: W[:, s1:] -= Err[s0:s1] U[s0:s1, s1:]
            GemmArgs gm{a.m, a.n - s1, s1 - s0, err_all, a.m, 1, LLMC_DTYPE_F32, a.U + s0 * a.ldu + s1, a.ldu, 0,
                        LLMC_DTYPE_F32, a.W + s1, a.ldw, -1.f, 1.f};
            LLMC_TRY(gemm_f32(ctx, gm));
        }
    }
    return LLMC_OK;
}

}  // namespace

// count weights [m_k, n] sharing U; outputs are stacked in weight order (rows sum(m_k)).
// Per-tensor parameters come out one per weight; channel / group parameters per stacked row.
llmc_status gptq_batch(llmc_ctx* ctx, int count, const void* const* Ws, const int64_t* ms, const int64_t* ldws, int dtype,
                       int64_t n, const float* U, int64_t ldu, const llmc_qconfig* cfg, float* wq_out, int64_t ldq,
                       uint8_t* codes, float* scales_out, int32_t* zps_out, int mode, uint8_t* mask_out,
                       const int32_t* perm) {
    const int strategy = cfg->strategy;
    int64_t M = 0, mmax = 0;
    for (int k = 0; k < count; k++) {
        M += ms[k];
        mmax = ms[k] > mmax ? ms[k] : mmax;
    }
    const int64_t gs = strategy == LLMC_STRATEGY_GROUP ? cfg->group_size : n;
    const int64_t G = n_groups(strategy, n, gs);
    const bool tensor = strategy == LLMC_STRATEGY_TENSOR;
    const int64_t nrow_params = tensor ? M : M * G;  // what the block kernel indexes
    // Scratch: working copy (unless wq_out is used), Err1^T, params, reduction.
    const bool own_work = wq_out == nullptr;
    size_t need = 0;
    need += own_work ? (size_t)M * n * 4 + 256 : 0;
    need += (size_t)BW * SUPER_BLOCKS * M * 4 + 256;
    need += (size_t)(tensor ? 2 * count : M * G) * 2 * 4 + 1024;  // mins/maxs
    need += (size_t)nrow_params * 8 + 512;                          // per-row params (kernel side)
    need += (size_t)(tensor ? count : 0) * 8 + 512;                 // per-weight params if not returned
    need += (size_t)(2 * mmax + 128) * 4 + 256;                     // per-tensor reduction scratch
    if (perm) {                                                     // act_order
        need += (size_t)M * n * 4 + 256;                            // permuted working copy
        need += (size_t)2 * n * 4 + 512;                            // column-group map, inverse
        need += codes ? (size_t)M * n + 256 : 0;                    // codes in permuted order
    }
    void* wsp;
    LLMC_TRY(workspace(ctx, need, &wsp));
    Carver cv{(char*)wsp};
    float* work = own_work ? cv.take<float>((size_t)M * n) : wq_out;
    const int64_t ldwork = own_work ? n : ldq;
    float* err1t = cv.take<float>((size_t)BW * SUPER_BLOCKS * M);
    float* mins = cv.take<float>(tensor ? 2 * count : M * G);
    float* maxs = cv.take<float>(tensor ? 2 * count : M * G);
    float* krs = nullptr;
    int32_t* krz = nullptr;
    float* ts = nullptr;
    int32_t* tz = nullptr;
    if (tensor) {
        krs = cv.take<float>(M);
        krz = cv.take<int32_t>(M);
        ts = scales_out ? scales_out : cv.take<float>(count);
        tz = zps_out ? zps_out : cv.take<int32_t>(count);
    } else {
        krs = scales_out ? scales_out : cv.take<float>(M * G);
        krz = zps_out ? zps_out : cv.take<int32_t>(M * G);
    }
    float* red = cv.take<float>(2 * mmax + 128);
    float* workp = perm ? cv.take<float>((size_t)M * n) : nullptr;
    int32_t* col_group = perm ? cv.take<int32_t>(n) : nullptr;
    int32_t* inv = perm ? cv.take<int32_t>(n) : nullptr;
    uint8_t* codes_p = (perm && codes) ? cv.take<uint8_t>((size_t)M * n) : nullptr;

    // Stacked fp32 working copy of the ORIGINAL weights.
    int64_t off = 0;
    for (int k = 0; k < count; k++) {
        LLMC_TRY(convert_to_f32(ctx, Ws[k], dtype, ms[k], n, ldws[k], work + off * ldwork, ldwork));
        off += ms[k];
    }

    BlockArgs a{};
    a.W = work; a.ldw = ldwork; a.m = M; a.n = n;
    a.U = U; a.ldu = ldu;
    a.bits = cfg->num_bits; a.sym = cfg->symmetric;
    a.err1t = err1t;
    if (mode == 0) {
        // ComputeScaleZeroPoint from the ORIGINAL weight (GptqBlockQuantizer.cs:97, :196-234);
        // the fp32 copy holds exactly the original values.  Accumulate mode 2 is a new
        // MinMaxObserver per scale entry, as the reference creates one per tensor or row.
        if (tensor) {
            off = 0;
            for (int k = 0; k < count; k++) {
                LLMC_TRY(minmax(ctx, work + off * ldwork, LLMC_DTYPE_F32, ms[k], n, ldwork, LLMC_STRATEGY_TENSOR, n,
                                mins + k, maxs + k, 2, red));
                off += ms[k];
            }
            LLMC_TRY(affine(ctx, mins, maxs, count, cfg->num_bits, cfg->symmetric, ts, tz));
            off = 0;
            for (int k = 0; k < count; k++) {
                expand_rows_kernel<<<(unsigned)((ms[k] + 255) / 256), 256, 0, ctx->stream>>>(ts + k, tz + k, ms[k],
                                                                                              krs + off, krz + off);
                LLMC_TRY(check_launch(ctx, "expand_rows"));
                off += ms[k];
            }
            a.srow = 1;
            a.gs = n;
        } else {
            // One fresh MinMaxObserver per row (or per row and group): a NaN row gets +inf / -inf.
            LLMC_TRY(minmax(ctx, work, LLMC_DTYPE_F32, M, n, ldwork, strategy, gs, mins, maxs, 2, red));
            LLMC_TRY(affine(ctx, mins, maxs, M * G, cfg->num_bits, cfg->symmetric, krs, krz));
            a.srow = G;
            a.gs = strategy == LLMC_STRATEGY_GROUP ? gs : n;
        }
        a.scales = krs; a.zps = krz;
        a.codes = codes;
        a.crow = cfg->num_bits <= 4 ? (n + 1) / 2 : n;
        if (!perm) return run_blocks<0>(ctx, a, cfg->block_size);
        // act_order: the parameters above come from the original columns; the solve runs on the
        // permuted columns against the permuted Hessian's factor U, then everything is scattered
        // back to the original column order.
        LLMC_TRY(gather_cols(ctx, work, M, n, ldwork, perm, workp, n));
        LLMC_TRY(perm_maps(ctx, perm, n, a.gs, col_group, inv));
        a.W = workp;
        a.ldw = n;
        a.col_group = strategy == LLMC_STRATEGY_GROUP ? col_group : nullptr;
        a.codes = codes_p;
        a.codes_bytes = 1;
        a.crow = n;
        LLMC_TRY(run_blocks<0>(ctx, a, cfg->block_size));
        if (wq_out) LLMC_TRY(scatter_cols(ctx, workp, M, n, n, perm, wq_out, ldq));
        if (codes) LLMC_TRY(scatter_codes(ctx, codes_p, M, n, inv, cfg->num_bits, codes, cfg->num_bits <= 4 ? (n + 1) / 2 : n));
        return LLMC_OK;
    }
    a.srow = 0; a.gs = n;
    a.sparsity = cfg->sparsity; a.mask_n = cfg->mask_n; a.mask_m = cfg->mask_m;
    a.mask = mask_out; a.mrow = n;
    return run_blocks<1>(ctx, a, cfg->block_size);
}

llmc_status gptq(llmc_ctx* ctx, const void* W, int dtype, int64_t m, int64_t n, int64_t ldw, const float* U, int64_t ldu,
                 const llmc_qconfig* cfg, float* wq_out, int64_t ldq, uint8_t* codes, float* scales_out,
                 int32_t* zps_out, int mode, uint8_t* mask_out) {
    const void* ws[1] = {W};
    const int64_t mm[1] = {m}, ll[1] = {ldw};
    return gptq_batch(ctx, 1, ws, mm, ll, dtype, n, U, ldu, cfg, wq_out, ldq, codes, scales_out, zps_out, mode, mask_out,
                      nullptr);
}

}  // namespace llmc
