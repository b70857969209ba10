// Shared internals of libllmc_b200: context, error state, workspace, dtype helpers.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdarg.h>
#include <stdio.h>
#include <string>

#include "../../include/llmc_b200.h"

namespace llmc {

// ---- error state (thread-local message behind llmc_last_error) ------------------------
void set_error(const char* fmt, ...);
llmc_status fail(llmc_status st, const char* fmt, ...);

#define LLMC_CUDA_TRY(expr)                                                                    \
    do {                                                                                       \
        cudaError_t _e = (expr);                                                               \
        if (_e != cudaSuccess)                                                                 \
            return ::llmc::fail(LLMC_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,                \
                                cudaGetErrorString(_e), __FILE__, __LINE__);                   \
    } while (0)

#define LLMC_TRY(expr)                                                                         \
    do {                                                                                       \
        llmc_status _s = (expr);                                                               \
        if (_s != LLMC_OK) return _s;                                                          \
    } while (0)

// ---- entry-point guard ----------------------------------------------------------------
// Every llmc_status entry point opens with LLMC_ENTRY():
//  - an NVTX range named after the function (seen by nsys / ncu --nvtx, a no-op without a
//    tool attached);
//  - host-side fault injection for failure-path tests, read once from the environment:
//    LLMC_FAULT="<function>:<status>[:<k>][,...]" makes <function> return <status> with the
//    message "injected fault in <function>" on every call, or on its k-th call only (k >= 1).
//    An injected call touches neither its arguments nor the GPU.
struct NvtxScope {
    explicit NvtxScope(const char* name);
    ~NvtxScope();
};
llmc_status injected_fault(const char* fn);

#define LLMC_ENTRY()                                        \
    ::llmc::NvtxScope _llmc_nvtx(__func__);                 \
    do {                                                    \
        llmc_status _f = ::llmc::injected_fault(__func__);  \
        if (_f != LLMC_OK) return _f;                       \
    } while (0)

}  // namespace llmc

// ---- context ---------------------------------------------------------------------------
struct llmc_ctx {
    int device = 0;
    int sm_count = 148;
    // SMs this context's persistent kernels may occupy (0 = all); see llmc_set_sm_limit.
    int sm_limit = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    int64_t launches = 0;
    // Growable scratch owned by the context (stream-ordered reuse: one op at a time).
    void* ws = nullptr;
    size_t ws_bytes = 0;
    // Second scratch area for operand copies made by routines called while ws is in use.
    void* ws2 = nullptr;
    size_t ws2_bytes = 0;
    // Device status words (flags written by kernels, e.g. a non-positive pivot).
    int* dflags = nullptr;
    int* hflags = nullptr;  // pinned mirror
    // try_wait attempts each bounded wait of the tensor-core kernels makes before it gives up
    // (llmc_set_wait_limit); 0 gives up at the first wait.
    uint32_t wait_limit = 1u << 26;
    // llmc_set_deferred_errors: decide device-side failures (a non-PD Hessian) without a host
    // wait and report them at the next llmc_sync.
    int deferred_errors = 0;
};

struct llmc_hessian {
    llmc_ctx* ctx = nullptr;
    int64_t d = 0;
    float* h = nullptr;  // [d, d] fp32, upper triangle authoritative
    int64_t samples = 0;
};

namespace llmc {

// Returns scratch of at least `bytes`, valid until the next workspace() call on ctx.
llmc_status workspace(llmc_ctx* ctx, size_t bytes, void** out);
// Same for the second scratch area (used by the tensor-core GEMM's operand split).
llmc_status workspace2(llmc_ctx* ctx, size_t bytes, void** out);

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Bump allocator over one workspace block.
struct Carver {
    char* base;
    size_t off = 0;
    template <typename T>
    T* take(size_t count) {
        off = align_up(off, 256);
        T* p = reinterpret_cast<T*>(base + off);
        off += count * sizeof(T);
        return p;
    }
};

inline llmc_status check_launch(llmc_ctx* ctx, const char* what) {
    ctx->launches++;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(LLMC_ERR_CUDA, "launch of %s failed: %s", what, cudaGetErrorString(e));
    return LLMC_OK;
}

// Grid size for a persistent kernel of this context: the SM count, capped by llmc_set_sm_limit.
inline int persistent_sms(const llmc_ctx* ctx) {
    return (ctx->sm_limit > 0 && ctx->sm_limit < ctx->sm_count) ? ctx->sm_limit : ctx->sm_count;
}

inline int dtype_size(int32_t dt) { return dt == LLMC_DTYPE_F32 ? 4 : 2; }
inline bool dtype_ok(int32_t dt) { return dt == LLMC_DTYPE_F32 || dt == LLMC_DTYPE_BF16 || dt == LLMC_DTYPE_F16; }

// ---- device dtype helpers ----------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// Round an fp32 value to T and back: one LibTorch reduced-precision op = fp32 op + this.
template <typename T> __device__ __forceinline__ float rnd(float v) { return to_f<T>(from_f<T>(v)); }

// FakeQuantizeFunction.forward op chain (FakeQuantizeFunction.cs:39-44) in dtype T:
// div -> round(half-even) -> add zp -> clamp -> [code] -> sub zp -> mul scale, each op
// rounded to T.  x must already be T-representable.  IEEE intrinsics keep the compiler
// from contracting or reassociating any step.
template <typename T>
__device__ __forceinline__ float fq_chain(float x, float s, float zpf, float qmin, float qmax, int* code) {
    float t = rnd<T>(__fdiv_rn(x, s));
    t = rnd<T>(rintf(t));
    t = rnd<T>(__fadd_rn(t, zpf));
    t = (t < qmin) ? qmin : ((t > qmax) ? qmax : t);  // NaN passes through like torch.clamp
    t = rnd<T>(t);
    *code = (int)t;
    t = rnd<T>(__fsub_rn(t, zpf));
    return rnd<T>(__fmul_rn(t, s));
}

// min / max that return NaN when either operand is NaN (torch.amin / amax / minimum /
// maximum, .NET MathF.Min / MathF.Max); fminf / fmaxf would drop the NaN instead.
__device__ __forceinline__ float fmin_nan(float a, float b) {
    float r;
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float fmax_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// How a segment's min / max is folded into the stored value (k_quant.cu's observer kernels):
//   FOLD_NONE      store the batch value (torch x.min(): NaN when any element is NaN);
//   FOLD_MINIMUM   torch.minimum / maximum with the stored value, NaN propagating
//                  (PerChannelMinMaxObserver.cs:64-74);
//   FOLD_OBSERVER  MinMaxObserver's `if (bMin < _min) _min = bMin` (MinMaxObserver.cs:34-42):
//                  the stored value changes only where the batch value is strictly beyond it,
//                  so a NaN batch changes nothing;
//   FOLD_FRESH     FOLD_OBSERVER against a new observer's +inf / -inf.
enum { FOLD_NONE = 0, FOLD_MINIMUM = 1, FOLD_OBSERVER = 2, FOLD_FRESH = 3 };
__device__ __forceinline__ float fold_min(float b, const float* stored, int mode) {
    if (mode == FOLD_NONE) return b;
    if (mode == FOLD_MINIMUM) return fmin_nan(b, *stored);
    const float o = mode == FOLD_OBSERVER ? *stored : INFINITY;
    return b < o ? b : o;
}
__device__ __forceinline__ float fold_max(float b, const float* stored, int mode) {
    if (mode == FOLD_NONE) return b;
    if (mode == FOLD_MINIMUM) return fmax_nan(b, *stored);
    const float o = mode == FOLD_OBSERVER ? *stored : -INFINITY;
    return b > o ? b : o;
}

// Observer.ComputeAffineParams (Observer.cs:47-75) with IEEE single ops; the zero-point
// conversion saturates like .NET's (long) cast before Math.Clamp.  MathF.Max returns NaN for a
// NaN operand, so a NaN min or max gives a NaN scale (and zero-point 0) as in the reference.
__device__ __forceinline__ void affine_params(float mn, float mx, int bits, int sym, float* scale, int* zp) {
    if (sym) {
        float am = fmax_nan(fabsf(mn), fabsf(mx));
        float qmax = (float)((1 << (bits - 1)) - 1);
        *scale = (am == 0.f) ? 1.f : __fdiv_rn(am, qmax);
        *zp = 0;
    } else {
        float qmax = (float)((1 << bits) - 1);
        float range = __fsub_rn(mx, mn);
        float s = (range == 0.f) ? 1.f : __fdiv_rn(range, qmax);
        float v = rintf(__fsub_rn(0.f, __fdiv_rn(mn, s)));
        int z;
        if (v != v) z = 0;
        else z = (int)fminf(fmaxf(v, 0.f), qmax);
        *scale = s;
        *zp = z;
    }
}

__host__ __device__ inline void qrange(int bits, int sym, float* qmin, float* qmax) {
    if (sym) {
        *qmax = (float)((1 << (bits - 1)) - 1);
        *qmin = -*qmax;
    } else {
        *qmin = 0.f;
        *qmax = (float)((1 << bits) - 1);
    }
}

}  // namespace llmc
