// MSEObserver grid search (src/LLMCompressorSharp.TorchExtensions/Observers/MSEObserver.cs:50-93):
// absMax = max |x|; candidate i = 1..G takes the symmetric range +-absMax*i/G through
// ComputeAffineParams; its error is mean((x - FQ(x))^2) with FQ the FakeQuantize op chain in x's
// dtype; the first minimum wins.  One kernel pass adds the squared errors of every candidate
// (a thread holds a few elements in registers and loops over the candidates); the candidate
// parameters and the choice are scalar host math, as in the reference.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>
#include <cstring>
#include <vector>

#include "common.cuh"

namespace llmc {
namespace {

constexpr int MSE_NT = 256;
constexpr int MSE_PER = 4;          // elements per thread per tile
constexpr int MSE_MAX_GRID = 4096;  // candidates (shared memory: 8 bytes each)

template <typename T>
__global__ void __launch_bounds__(MSE_NT) absmax_kernel(const T* x, int64_t n, unsigned int* out) {
    float m = 0.f;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(to_f<T>(x[i])));
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // |x| >= 0, so the float order is the order of the bit patterns
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

// sums[g] += sum over x of (x - FQ_g(x))^2, each difference and square rounded to T like the
// reference's tensor ops, accumulated in fp64.
template <typename T>
__global__ void __launch_bounds__(MSE_NT) mse_grid_kernel(const T* x, int64_t n, const float* scales, const float* zps,
                                                          int G, float qmin, float qmax, double* sums) {
    extern __shared__ double ssum[];
    for (int g = threadIdx.x; g < G; g += blockDim.x) ssum[g] = 0.0;
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t tile = (int64_t)blockDim.x * MSE_PER;
    // base depends on the block only, so every warp runs the same iterations (full-mask shuffles)
    for (int64_t base = (int64_t)blockIdx.x * tile; base < n; base += (int64_t)gridDim.x * tile) {
        float v[MSE_PER];
        bool ok[MSE_PER];
#pragma unroll
        for (int k = 0; k < MSE_PER; k++) {
            const int64_t idx = base + threadIdx.x + (int64_t)k * blockDim.x;
            ok[k] = idx < n;
            v[k] = ok[k] ? to_f<T>(x[idx]) : 0.f;
        }
        for (int g = 0; g < G; g++) {
            const float s = scales[g], z = zps[g];
            double acc = 0.0;
#pragma unroll
            for (int k = 0; k < MSE_PER; k++) {
                if (!ok[k]) continue;
                int code;
                const float fq = fq_chain<T>(v[k], s, z, qmin, qmax, &code);
                const float e = rnd<T>(__fsub_rn(v[k], fq));
                acc += (double)rnd<T>(__fmul_rn(e, e));
            }
            for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (lane == 0) atomicAdd(&ssum[g], acc);
        }
    }
    __syncthreads();
    for (int g = threadIdx.x; g < G; g += blockDim.x) atomicAdd(&sums[g], ssum[g]);
}

// Observer.ComputeAffineParams (Observer.cs:47-75) in IEEE single on the host (the reference's
// C# float math); MathF.Round is round half to even.
void affine_host(float mn, float mx, int bits, int sym, float* scale, int* zp) {
    volatile float vmn = mn, vmx = mx;  // keep each operation in single precision
    if (sym) {
        const float am = std::fmax(std::fabs(vmn), std::fabs(vmx));
        const float qmax = (float)((1 << (bits - 1)) - 1);
        volatile float s = am / qmax;
        *scale = (am == 0.f) ? 1.f : (float)s;
        *zp = 0;
    } else {
        const float qmax = (float)((1 << bits) - 1);
        volatile float range = vmx - vmn;
        volatile float s = (range == 0.f) ? 1.f : range / qmax;
        volatile float q = vmn / s;
        volatile float neg = 0.f - q;
        const float v = std::nearbyint((float)neg);
        *scale = s;
        *zp = (v != v) ? 0 : (int)std::fmin(std::fmax(v, 0.f), qmax);
    }
}

// The reference's `.mean()` result in x's dtype, read as a float.
float mean_in_dtype(double sum, int64_t n, int dtype) {
    const float m = (float)(sum / (double)n);
    if (dtype == LLMC_DTYPE_BF16) return __bfloat162float(__float2bfloat16_rn(m));
    if (dtype == LLMC_DTYPE_F16) return __half2float(__float2half_rn(m));
    return m;
}

template <typename T>
llmc_status launch_mse(llmc_ctx* ctx, const void* x, int64_t n, unsigned int* dmax, const float* dsc, const float* dzp,
                       int G, int bits, int sym, double* dsums, bool pass) {
    const int64_t want = (n + MSE_NT - 1) / MSE_NT;
    const int blocks_max = (int)(want < (int64_t)ctx->sm_count * 8 ? (want < 1 ? 1 : want) : (int64_t)ctx->sm_count * 8);
    if (!pass) {
        absmax_kernel<T><<<blocks_max, MSE_NT, 0, ctx->stream>>>(static_cast<const T*>(x), n, dmax);
        return check_launch(ctx, "mse_absmax");
    }
    float qmin, qmax;
    qrange(bits, sym, &qmin, &qmax);
    const int64_t tiles = (n + (int64_t)MSE_NT * MSE_PER - 1) / ((int64_t)MSE_NT * MSE_PER);
    const int blocks = (int)(tiles < (int64_t)ctx->sm_count * 4 ? (tiles < 1 ? 1 : tiles) : (int64_t)ctx->sm_count * 4);
    mse_grid_kernel<T><<<blocks, MSE_NT, (size_t)G * sizeof(double), ctx->stream>>>(static_cast<const T*>(x), n, dsc, dzp, G,
                                                                                    qmin, qmax, dsums);
    return check_launch(ctx, "mse_grid");
}

llmc_status dispatch_mse(llmc_ctx* ctx, int dtype, const void* x, int64_t n, unsigned int* dmax, const float* dsc,
                         const float* dzp, int G, int bits, int sym, double* dsums, bool pass) {
    switch (dtype) {
        case LLMC_DTYPE_F32: return launch_mse<float>(ctx, x, n, dmax, dsc, dzp, G, bits, sym, dsums, pass);
        case LLMC_DTYPE_BF16: return launch_mse<__nv_bfloat16>(ctx, x, n, dmax, dsc, dzp, G, bits, sym, dsums, pass);
        case LLMC_DTYPE_F16: return launch_mse<__half>(ctx, x, n, dmax, dsc, dzp, G, bits, sym, dsums, pass);
    }
    return fail(LLMC_ERR_INVALID_ARG, "unsupported dtype %d", dtype);
}

}  // namespace
}  // namespace llmc

using namespace llmc;

extern "C" llmc_status llmc_observer_mse(llmc_ctx* ctx, const void* x, int32_t dtype, int64_t count,
                                         int32_t grid_points, int32_t num_bits, int32_t symmetric, float* scale_out,
                                         int32_t* zp_out, double* mse_out) {
    LLMC_ENTRY();
    if (!ctx) return fail(LLMC_ERR_INVALID_ARG, "context must not be null");
    if (!x || !scale_out || !zp_out) return fail(LLMC_ERR_INVALID_ARG, "x, scale_out and zp_out must not be null");
    if (!dtype_ok(dtype)) return fail(LLMC_ERR_INVALID_ARG, "unsupported dtype %d", dtype);
    if (grid_points < 2 || grid_points > MSE_MAX_GRID)
        return fail(LLMC_ERR_OUT_OF_RANGE, "gridPoints must be >= 2 (and <= %d here).", MSE_MAX_GRID);
    if (num_bits < 2 || num_bits > 16) return fail(LLMC_ERR_OUT_OF_RANGE, "numBits must be between 2 and 16 inclusive.");
    if (count <= 0) return fail(LLMC_ERR_NO_SAMPLES, "MSEObserver has no calibration samples. Call Update before GetQuantParams.");
    LLMC_CUDA_TRY(cudaSetDevice(ctx->device));
    const int G = grid_points;
    void* wsp;
    LLMC_TRY(workspace(ctx, 256 + (size_t)G * (4 + 4 + 8) + 1024, &wsp));
    Carver cv{(char*)wsp};
    unsigned int* dmax = cv.take<unsigned int>(4);
    float* dsc = cv.take<float>(G);
    float* dzp = cv.take<float>(G);
    double* dsums = cv.take<double>(G);
    LLMC_CUDA_TRY(cudaMemsetAsync(dmax, 0, sizeof(unsigned int), ctx->stream));
    LLMC_TRY(dispatch_mse(ctx, dtype, x, count, dmax, nullptr, nullptr, 0, num_bits, symmetric, nullptr, false));
    unsigned int bits_max = 0;
    LLMC_CUDA_TRY(cudaMemcpyAsync(&bits_max, dmax, sizeof(bits_max), cudaMemcpyDeviceToHost, ctx->stream));
    LLMC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    float abs_max;
    std::memcpy(&abs_max, &bits_max, sizeof(abs_max));
    if (mse_out)
        for (int i = 0; i < G; i++) mse_out[i] = NAN;
    if (abs_max == 0.f) {  // MSEObserver.cs:64-67
        *scale_out = 1.f;
        *zp_out = 0;
        return LLMC_OK;
    }
    // candidates i = 1..G (MSEObserver.cs:72-78); a zero scale is skipped
    std::vector<float> sc, zf;
    std::vector<int> zi, idx;
    for (int i = 1; i <= G; i++) {
        volatile float frac = (float)i / (float)G;
        volatile float cmax = abs_max * frac;
        float s;
        int z;
        affine_host(-cmax, cmax, num_bits, symmetric, &s, &z);
        if (s == 0.f) continue;
        sc.push_back(s);
        zf.push_back((float)z);
        zi.push_back(z);
        idx.push_back(i - 1);
    }
    volatile float qs = (float)((1 << (num_bits - 1)) - 1);
    float best_scale = abs_max / qs;  // MSEObserver.cs:69
    int best_zp = 0;
    if (!sc.empty()) {
        const int Gv = (int)sc.size();
        LLMC_CUDA_TRY(cudaMemcpyAsync(dsc, sc.data(), Gv * sizeof(float), cudaMemcpyHostToDevice, ctx->stream));
        LLMC_CUDA_TRY(cudaMemcpyAsync(dzp, zf.data(), Gv * sizeof(float), cudaMemcpyHostToDevice, ctx->stream));
        LLMC_CUDA_TRY(cudaMemsetAsync(dsums, 0, Gv * sizeof(double), ctx->stream));
        LLMC_TRY(dispatch_mse(ctx, dtype, x, count, nullptr, dsc, dzp, Gv, num_bits, symmetric, dsums, true));
        std::vector<double> sums(Gv);
        LLMC_CUDA_TRY(cudaMemcpyAsync(sums.data(), dsums, Gv * sizeof(double), cudaMemcpyDeviceToHost, ctx->stream));
        LLMC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
        float best_mse = INFINITY;
        for (int k = 0; k < Gv; k++) {
            const float mse = mean_in_dtype(sums[k], count, dtype);
            if (mse_out) mse_out[idx[k]] = mse;
            if (mse < best_mse) {  // the first minimum wins (MSEObserver.cs:83-88)
                best_mse = mse;
                best_scale = sc[k];
                best_zp = zi[k];
            }
        }
    }
    *scale_out = best_scale;
    *zp_out = best_zp;
    return LLMC_OK;
}
