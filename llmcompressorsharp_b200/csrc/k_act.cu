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
