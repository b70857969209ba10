// Dynamic per-token activation quantisation (the "A" of W8A8).
//
// Extension.  QuantizationStrategy.PerToken exists in the reference
// (src/LLMCompressorSharp.TorchExtensions/Observers/QuantizationStrategy.cs:9-19), but
// RtnModifier.cs:69-70 rejects it for weights and nothing quantises activations.  The
// restatement: x [tokens, hidden] gets one min-max observer per token row (the per-channel
// observer of PerChannelMinMaxObserver.cs:38-76 on axis 0, so a row holding a NaN gets NaN
// parameters), Observer.ComputeAffineParams (Observer.cs:47-75), and the FakeQuantizeFunction
// op chain in x's dtype (FakeQuantizeFunction.cs:39-44).  Outputs: the integer code q =
// clamp(round(x / s) + zp) as one byte per element (two's complement for symmetric grids),
// the per-token scale and zero-point, and optionally the fake-quantised activations.
//
// One warp per token row, two passes over the row (the second pass re-reads it from L1/L2, so
// HBM sees the row once): 16-byte loads, NaN-propagating min / max with shuffles, then the
// quantisation.  For bf16 and fp32 inputs the codes come from x * rcp(s) when that provably
// equals the op-by-op chain (see quant_elem); other elements take fq_chain.
#include "ops.h"

#include <type_traits>

namespace llmc {
namespace {

constexpr int WARPS = 8;  // rows per 256-thread block

template <typename T>
struct VecOf {
    static constexpr int N = 16 / sizeof(T);
};

// Code and fake-quantised value of x under (s, z), identical to fq_chain<T>.  fast: every
// quotient of the row satisfies |x / s| + |z| <= 256 (checked from the row's min and max with a
// relative margin), so every intermediate of the chain is an integer of magnitude <= 256 once
// x / s is rounded to T, which T represents exactly.  Then the chain reduces to rint(T(x / s)),
// with T(x / s) taken from f = x * rcp(s) unless f lies within a few units in the last place of a
// T rounding midpoint (for fp32: of a half-integer), where the exact chain runs instead.
template <typename T>
__device__ __forceinline__ float quant_elem(float x, float s, float rcp, float zf, int z, float qmin, float qmax,
                                           int iqmin, int iqmax, bool fast, int* code) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        if (fast) {
            const float f = __fmul_rn(x, rcp);
            const uint32_t b = __float_as_uint(f);
            if (((b - 0x7FFCu) & 0xFFFFu) > 8u && fabsf(f) <= 3.0e38f) {
                // bf16 round-to-nearest-even on the bit pattern, then rint by the 1.5 * 2^23 trick
                const float t1 = __uint_as_float((b + 0x7FFFu + ((b >> 16) & 1u)) & 0xFFFF0000u);
                int t = __float_as_int(__fadd_rn(t1, 12582912.f)) - 0x4B400000 + z;
                t = t < iqmin ? iqmin : (t > iqmax ? iqmax : t);
                *code = t;
                return rnd<T>(__fmul_rn((float)(t - z), s));
            }
        }
    } else if constexpr (std::is_same<T, float>::value) {
        if (fast) {
            const float f = __fmul_rn(x, rcp);
            const float r = rintf(f);
            if (fabsf(fabsf(__fsub_rn(f, r)) - 0.5f) > fabsf(f) * 4.8e-7f + 1e-30f) {
                int t = (int)r + z;
                t = t < iqmin ? iqmin : (t > iqmax ? iqmax : t);
                *code = t;
                return __fmul_rn((float)(t - z), s);
            }
        }
    }
    return fq_chain<T>(x, s, zf, qmin, qmax, code);
}

template <typename T>
__global__ void __launch_bounds__(32 * WARPS) act_token_kernel(const T* x, int64_t rows, int64_t cols, int64_t ld,
                                                               int bits, int sym, int vec, uint8_t* codes, int64_t ldc,
                                                               float* scales, int32_t* zps, T* deq, int64_t ldd) {
    constexpr int V = VecOf<T>::N;
    const int lane = threadIdx.x & 31;
    float qmin, qmax;
    qrange(bits, sym, &qmin, &qmax);
    const int iqmin = (int)qmin, iqmax = (int)qmax;
    for (int64_t r = (int64_t)blockIdx.x * WARPS + threadIdx.x / 32; r < rows; r += (int64_t)gridDim.x * WARPS) {
        const T* row = x + r * ld;
        float mn = INFINITY, mx = -INFINITY;
        if (vec) {
            for (int64_t c = (int64_t)lane * V; c < cols; c += 32 * V) {
                const uint4 q = *reinterpret_cast<const uint4*>(row + c);
                const T* h = reinterpret_cast<const T*>(&q);
#pragma unroll
                for (int i = 0; i < V; i++) {
                    const float f = to_f<T>(h[i]);
                    mn = fmin_nan(mn, f);
                    mx = fmax_nan(mx, f);
                }
            }
        } else {
            for (int64_t c = lane; c < cols; c += 32) {
                const float f = to_f<T>(row[c]);
                mn = fmin_nan(mn, f);
                mx = fmax_nan(mx, f);
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            mn = fmin_nan(mn, __shfl_xor_sync(0xffffffffu, mn, off));
            mx = fmax_nan(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        }
        float s;
        int z;
        affine_params(mn, mx, bits, sym, &s, &z);
        if (lane == 0) {
            scales[r] = s;
            if (zps) zps[r] = z;
        }
        const float zf = (float)z;
        const float rcp = __frcp_rn(s);
        const float k = 1.f + 0x1p-20f;
        const float hi = fmaxf(mx, 0.f) * rcp * k + zf;  // NaN / Inf fail the test below
        const float lo = fminf(mn, 0.f) * rcp * k + zf;
        const bool fast = hi <= 256.f && lo >= -256.f && fabsf(rcp) <= 3.0e38f;
        uint8_t* crow = codes ? codes + r * ldc : nullptr;
        T* drow = deq ? deq + r * ldd : nullptr;
        if (vec) {
            for (int64_t c = (int64_t)lane * V; c < cols; c += 32 * V) {
                const uint4 q = *reinterpret_cast<const uint4*>(row + c);
                const T* h = reinterpret_cast<const T*>(&q);
                uint8_t cb[V];
                T ob[V];
#pragma unroll
                for (int i = 0; i < V; i++) {
                    int code;
                    const float o = quant_elem<T>(to_f<T>(h[i]), s, rcp, zf, z, qmin, qmax, iqmin, iqmax, fast, &code);
                    cb[i] = (uint8_t)code;
                    ob[i] = from_f<T>(o);
                }
                if (crow) {
                    if constexpr (V == 8) *reinterpret_cast<uint2*>(crow + c) = *reinterpret_cast<const uint2*>(cb);
                    else *reinterpret_cast<uint32_t*>(crow + c) = *reinterpret_cast<const uint32_t*>(cb);
                }
                if (drow) *reinterpret_cast<uint4*>(drow + c) = *reinterpret_cast<const uint4*>(ob);
            }
        } else {
            for (int64_t c = lane; c < cols; c += 32) {
                int code;
                const float o = quant_elem<T>(to_f<T>(row[c]), s, rcp, zf, z, qmin, qmax, iqmin, iqmax, fast, &code);
                if (crow) crow[c] = (uint8_t)code;
                if (drow) drow[c] = from_f<T>(o);
            }
        }
    }
}

// bf16 codes without fake-quantised values, rows of at most REG_NV * 256 columns (a multiple of
// 256): the row stays in registers (lane l holds vectors l, l + 32, ...), so it is loaded once
// with every load in flight, and the element loop is quant_elem's fast path on the paired fp32
// instructions of sm_100 (FMUL2 / FFMA2 / FADD2, each component rounded as its scalar form):
//   * f = x * rcp(s); a vector holding an f within 4 units in the last place of a bf16 rounding
//     midpoint (low 16 bits of f shifted up and offset, min-accumulated, one compare) takes
//     quant_elem element by element;
//   * bf16(f) by Veltkamp splitting, c = f * (2^16 + 1), bf16(f) = c - (c - f) (T. J. Dekker,
//     "A floating-point technique for extending the available precision", 1971), each
//     difference one fused multiply-add by -1; its tie-breaking can differ from round-to-even
//     only at the midpoints sent to quant_elem;
//   * rint by adding 1.5 * 2^23; the clamp to [qmin - zp, qmax - zp] on that float only in warps
//     whose row can reach the grid's ends; the code byte is the low byte of the sum's bit
//     pattern plus zp.
constexpr int REG_NV = 16;

// A vector holding an element near a bf16 rounding midpoint (or a row off the fast path): those
// elements take the op-by-op chain, the others token_codes8's arithmetic with the clamp; packed
// as token_codes8 packs.  One out-of-line copy, called from the batched rewrite below.
__device__ __noinline__ uint2 token_chain8(uint4 w, float s, float rcp, bool fast, int z, float qmin, float qmax,
                                           int iqmin, int iqmax) {
    constexpr float MAGIC = 12582912.f;  // 1.5 * 2^23
    const float zf = (float)z;
    const float cmin = MAGIC + (qmin - zf), cmax = MAGIC + (qmax - zf);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    uint32_t u[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float xv = (i & 1) ? __uint_as_float(ww[i / 2] & 0xFFFF0000u) : __uint_as_float(ww[i / 2] << 16);
        const float f = __fmul_rn(xv, rcp);
        if (!fast || (__float_as_uint(f) * 65536u - 0x7FFC0000u) <= 0x80000u) {
            int code;
            quant_elem<__nv_bfloat16>(xv, s, rcp, zf, z, qmin, qmax, iqmin, iqmax, false, &code);
            u[i] = (uint32_t)code;
        } else {
            const float c = __fmul_rn(f, 65537.f);
            const float b16 = __fsub_rn(c, __fsub_rn(c, f));
            u[i] = __float_as_uint(fminf(fmaxf(__fadd_rn(b16, MAGIC), cmin), cmax)) + (uint32_t)z;
        }
    }
    return make_uint2(__byte_perm(__byte_perm(u[0], u[1], 0x0040), __byte_perm(u[2], u[3], 0x0040), 0x5410),
                      __byte_perm(__byte_perm(u[4], u[5], 0x0040), __byte_perm(u[6], u[7], 0x0040), 0x5410));
}

// Vectors that need the chain are queued per warp in shared memory and rewritten in batches,
// one vector a lane: a branch to the chain costs the whole warp the chain's time whenever any
// lane takes it, and a 4,096-column row holds 512 vectors, of which a few percent hold an
// element near a midpoint.
constexpr int TOK_QCAP = 32;
struct TokQueue {
    uint4 w[TOK_QCAP];
    float s[TOK_QCAP], rcp[TOK_QCAP];
    int z[TOK_QCAP];
    int64_t off[TOK_QCAP];  // byte offset of the vector's codes; bit 62 set: the row is off the fast path
};

__device__ __forceinline__ void token_flush(TokQueue& q, int count, float qmin, float qmax, int iqmin, int iqmax,
                                            uint8_t* codes) {
    __syncwarp();  // the fast-path stores of these vectors came from other lanes of this warp
    const int lane = threadIdx.x & 31;
    if (lane < count) {
        const int64_t o = q.off[lane];
        const bool fast = (o & (int64_t(1) << 62)) == 0;
        *reinterpret_cast<uint2*>(codes + (o & ~(int64_t(1) << 62))) =
            token_chain8(q.w[lane], q.s[lane], q.rcp[lane], fast, q.z[lane], qmin, qmax, iqmin, iqmax);
    }
    __syncwarp();
}

template <bool CLAMP>
__device__ __forceinline__ uint2 token_codes8(const uint4& w, float rcp, float cmin, float cmax, int z, bool* near_mid) {
    constexpr float MAGIC = 12582912.f;  // 1.5 * 2^23
    const float2 rcp2 = make_float2(rcp, rcp), k2 = make_float2(65537.f, 65537.f);
    const float2 neg1 = make_float2(-1.f, -1.f), magic2 = make_float2(MAGIC, MAGIC);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    uint32_t u[8];
    uint32_t near = 0xFFFFFFFFu;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float2 xv = make_float2(__uint_as_float(ww[k] << 16), __uint_as_float(ww[k] & 0xFFFF0000u));
        const float2 f = __fmul2_rn(xv, rcp2);
        near = min(near, __float_as_uint(f.x) * 65536u - 0x7FFC0000u);
        near = min(near, __float_as_uint(f.y) * 65536u - 0x7FFC0000u);
        const float2 c = __fmul2_rn(f, k2);
        const float2 b16 = __ffma2_rn(__ffma2_rn(f, neg1, c), neg1, c);  // c - (c - f)
        float2 rf = __fadd2_rn(b16, magic2);
        if constexpr (CLAMP) {
            rf.x = fminf(fmaxf(rf.x, cmin), cmax);
            rf.y = fminf(fmaxf(rf.y, cmin), cmax);
        }
        u[2 * k] = __float_as_uint(rf.x) + (uint32_t)z;
        u[2 * k + 1] = __float_as_uint(rf.y) + (uint32_t)z;
    }
    *near_mid = near <= 0x80000u;
    return make_uint2(__byte_perm(__byte_perm(u[0], u[1], 0x0040), __byte_perm(u[2], u[3], 0x0040), 0x5410),
                      __byte_perm(__byte_perm(u[4], u[5], 0x0040), __byte_perm(u[6], u[7], 0x0040), 0x5410));
}

// The row kernel streams its rows through shared memory: while a warp quantises row r, row
// r + stride is already on its way (cp.async, 16 bytes a lane and vector) into the other half of
// the warp's double buffer, so each warp keeps a row of loads in flight through its compute.
// Each lane copies and later reads only its own 16-byte slots, so cp.async.wait_group alone
// orders the data for it; the buffer a copy overwrites was read one iteration earlier.  The
// loops over a row's vectors read the stage and are unrolled only a little: with the row held in
// registers and every loop fully unrolled (16 vectors x 2 clamp variants) the kernel's code no
// longer fit the instruction cache (ncu: "no instruction" the top stall, issue active 35 %).
constexpr int RWARPS = 4;                                   // warps (rows in flight) a block
constexpr int RSTAGE = REG_NV * 32;                         // uint4 slots of one row buffer
constexpr size_t REG_SMEM = (size_t)RWARPS * 2 * RSTAGE * 16 + RWARPS * sizeof(TokQueue);

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
                 "l"(gsrc)
                 : "memory");
}

template <bool CLAMP>
__device__ __forceinline__ void token_row_codes(const uint4* rowbuf, int nv, int lane, int64_t crow, float rcp,
                                                float cmin, float cmax, bool fast, float s, int z, float qmin,
                                                float qmax, int iqmin, int iqmax, uint8_t* codes, TokQueue& q,
                                                int& qn) {
#pragma unroll 2
    for (int j = 0; j < nv; j++) {  // nv is the same in every lane
        const uint4 w = rowbuf[j * 32 + lane];
        const int64_t off = crow + (int64_t)(j * 32 + lane) * 8;
        bool near_mid;
        *reinterpret_cast<uint2*>(codes + off) = token_codes8<CLAMP>(w, rcp, cmin, cmax, z, &near_mid);
        const bool slow = !fast || near_mid;
        const unsigned mask = __ballot_sync(0xffffffffu, slow);
        if (mask) {
            const int n = __popc(mask);
            if (qn + n > TOK_QCAP) {
                token_flush(q, qn, qmin, qmax, iqmin, iqmax, codes);
                qn = 0;
            }
            if (slow) {
                const int pos = qn + __popc(mask & ((1u << lane) - 1u));
                q.w[pos] = w;
                q.s[pos] = s;
                q.rcp[pos] = rcp;
                q.z[pos] = z;
                q.off[pos] = off | (fast ? int64_t(0) : (int64_t(1) << 62));
            }
            qn += n;
        }
    }
}

__global__ void __launch_bounds__(32 * RWARPS) act_token_bf16_reg_kernel(const __nv_bfloat16* x, int64_t rows,
                                                                         int64_t cols, int64_t ld, int bits, int sym,
                                                                         uint8_t* codes, int64_t ldc, float* scales,
                                                                         int32_t* zps) {
    constexpr float MAGIC = 12582912.f;
    const int lane = threadIdx.x & 31, warp = threadIdx.x / 32;
    const int nv = (int)(cols / 256);  // vectors per lane
    float qmin, qmax;
    qrange(bits, sym, &qmin, &qmax);
    const int iqmin = (int)qmin, iqmax = (int)qmax;
    const __nv_bfloat162 pinf = __float2bfloat162_rn(INFINITY), ninf = __float2bfloat162_rn(-INFINITY);
    extern __shared__ __align__(16) unsigned char tok_smem[];
    uint4* stage = reinterpret_cast<uint4*>(tok_smem) + (size_t)warp * 2 * RSTAGE;
    TokQueue* queues = reinterpret_cast<TokQueue*>(tok_smem + (size_t)RWARPS * 2 * RSTAGE * 16);
    TokQueue& q = queues[warp];
    int qn = 0;  // queued vectors of this warp (the same in every lane)
    const int64_t stride = (int64_t)gridDim.x * RWARPS;
    auto prefetch = [&](int64_t rr, int buf) {
        const __nv_bfloat16* src = x + rr * ld;
        uint4* dst = stage + buf * RSTAGE;
#pragma unroll 4
        for (int j = 0; j < nv; j++) cp_async16(dst + j * 32 + lane, src + (int64_t)(j * 32 + lane) * 8);
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    int64_t r = (int64_t)blockIdx.x * RWARPS + warp;
    if (r < rows) prefetch(r, 0);
    for (int it = 0; r < rows; r += stride, it++) {
        const uint4* rowbuf = stage + (it & 1) * RSTAGE;
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        if (r + stride < rows) prefetch(r + stride, (it & 1) ^ 1);
        __nv_bfloat162 mn2 = pinf, mx2 = ninf;
#pragma unroll 4
        for (int j = 0; j < nv; j++) {
            const uint4 w = rowbuf[j * 32 + lane];
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const __nv_bfloat162 p = *reinterpret_cast<const __nv_bfloat162*>(&ww[k]);
                mn2 = __hmin2_nan(mn2, p);
                mx2 = __hmax2_nan(mx2, p);
            }
        }
        float mn = fmin_nan(__low2float(mn2), __high2float(mn2));
        float mx = fmax_nan(__low2float(mx2), __high2float(mx2));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            mn = fmin_nan(mn, __shfl_xor_sync(0xffffffffu, mn, off));
            mx = fmax_nan(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        }
        float s;
        int z;
        affine_params(mn, mx, bits, sym, &s, &z);
        if (lane == 0) {
            scales[r] = s;
            if (zps) zps[r] = z;
        }
        const float zf = (float)z;
        const float rcp = __frcp_rn(s);
        const float k = 1.f + 0x1p-20f;
        const float hi = fmaxf(mx, 0.f) * rcp * k + zf;  // NaN / Inf fail the tests below
        const float lo = fminf(mn, 0.f) * rcp * k + zf;
        const bool fast = hi <= 256.f && lo >= -256.f && fabsf(rcp) <= 3.0e38f;
        // The clamp can act only if some quotient of the row rounds beyond the grid (the row's
        // parameters are the same in every lane, so the branch is uniform).
        const bool clamp = !(hi <= qmax + 0.25f && lo >= qmin - 0.25f);
        const float cmin = MAGIC + (qmin - zf), cmax = MAGIC + (qmax - zf);
        if (clamp)
            token_row_codes<true>(rowbuf, nv, lane, r * ldc, rcp, cmin, cmax, fast, s, z, qmin, qmax, iqmin, iqmax, codes,
                                  q, qn);
        else
            token_row_codes<false>(rowbuf, nv, lane, r * ldc, rcp, cmin, cmax, fast, s, z, qmin, qmax, iqmin, iqmax,
                                   codes, q, qn);
    }
    if (qn) token_flush(q, qn, qmin, qmax, iqmin, iqmax, codes);
}

template <typename T>
llmc_status launch(llmc_ctx* ctx, const void* x, int64_t rows, int64_t cols, int64_t ld, int bits, int sym,
                   uint8_t* codes, int64_t ldc, float* scales, int32_t* zps, void* deq, int64_t ldd) {
    constexpr int V = VecOf<T>::N;
    // 16-byte vectors need aligned rows for every input and output row start.
    const bool vec = (uintptr_t)x % 16 == 0 && ld % V == 0 && cols % V == 0 &&
                     (codes == nullptr || ((uintptr_t)codes % (size_t)V == 0 && ldc % V == 0)) &&
                     (deq == nullptr || ((uintptr_t)deq % 16 == 0 && ldd % V == 0));
    int64_t blocks = (rows + WARPS - 1) / WARPS;
    const int64_t cap = (int64_t)ctx->sm_count * 16;
    if (blocks > cap) blocks = cap;
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        if (vec && codes && !deq && cols % 256 == 0 && cols <= 256 * REG_NV && (uintptr_t)codes % 8 == 0 &&
            ldc % 8 == 0) {
            static bool attr[64];
            if (ctx->device < 0 || ctx->device >= 64) return fail(LLMC_ERR_UNSUPPORTED, "device index");
            if (!attr[ctx->device]) {
                LLMC_CUDA_TRY(cudaFuncSetAttribute(act_token_bf16_reg_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)REG_SMEM));
                attr[ctx->device] = true;
            }
            int64_t rblocks = (rows + RWARPS - 1) / RWARPS;
            const int64_t rcap = (int64_t)ctx->sm_count * 8;
            if (rblocks > rcap) rblocks = rcap;
            act_token_bf16_reg_kernel<<<(unsigned)rblocks, 32 * RWARPS, REG_SMEM, ctx->stream>>>(
                reinterpret_cast<const __nv_bfloat16*>(x), rows, cols, ld, bits, sym, codes, ldc, scales, zps);
            return check_launch(ctx, "act_token_bf16_reg");
        }
    }
    act_token_kernel<T><<<(unsigned)blocks, 32 * WARPS, 0, ctx->stream>>>(
        reinterpret_cast<const T*>(x), rows, cols, ld, bits, sym, vec ? 1 : 0, codes, ldc, scales, zps,
        reinterpret_cast<T*>(deq), ldd);
    return check_launch(ctx, "act_token");
}

}  // namespace

llmc_status act_quant_per_token(llmc_ctx* ctx, const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld,
                                int bits, int sym, uint8_t* codes, int64_t ldc, float* scales, int32_t* zps, void* deq,
                                int64_t ldd) {
    switch (dtype) {
        case LLMC_DTYPE_F32: return launch<float>(ctx, x, rows, cols, ld, bits, sym, codes, ldc, scales, zps, deq, ldd);
        case LLMC_DTYPE_BF16:
            return launch<__nv_bfloat16>(ctx, x, rows, cols, ld, bits, sym, codes, ldc, scales, zps, deq, ldd);
        case LLMC_DTYPE_F16: return launch<__half>(ctx, x, rows, cols, ld, bits, sym, codes, ldc, scales, zps, deq, ldd);
    }
    return fail(LLMC_ERR_INVALID_ARG, "bad dtype %d", dtype);
}

}  // namespace llmc
