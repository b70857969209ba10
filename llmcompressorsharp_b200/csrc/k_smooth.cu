// SmoothQuant activation statistics / smoothing and the AWQ scale grid search.
//
// Reference: SmoothQuantModifier.UpdateActivationMax (src/LLMCompressorSharp.Core/Algorithms/
// SmoothQuant/SmoothQuantModifier.cs:71-115), ApplyMapping (:117-182); AWQ per the design
// sketch docs/llmcompressorsharp/algorithm-mapping.md:214-249.
#include "ops.h"

namespace llmc {
namespace {

constexpr int NT = 256;

// Column-wise max |x| over rows, folded into out with an integer atomicMax on the float
// bits (valid because every value is >= 0).  Each thread owns VEC consecutive columns
// and a slice of rows, so a warp reads 32*16 contiguous bytes per row.
template <typename T, int VEC>
__global__ void __launch_bounds__(NT) col_absmax_kernel(const T* x, int64_t rows, int64_t cols, int64_t ld,
                                                        int64_t rows_per_block, float* out) {
    const int64_t c0 = ((int64_t)blockIdx.x * NT + threadIdx.x) * VEC;
    if (c0 >= cols) return;
    const int64_t r0 = (int64_t)blockIdx.y * rows_per_block;
    const int64_t r1 = min(rows, r0 + rows_per_block);
    float mx[VEC];
#pragma unroll
    for (int i = 0; i < VEC; i++) mx[i] = 0.f;
    const bool full = c0 + VEC <= cols;
    for (int64_t r = r0; r < r1; r++) {
        const T* p = x + r * ld + c0;
        if (VEC > 1 && full) {
            uint4 q = *reinterpret_cast<const uint4*>(p);
            const T* h = reinterpret_cast<const T*>(&q);
#pragma unroll
            for (int i = 0; i < VEC; i++) mx[i] = fmaxf(mx[i], fabsf(to_f<T>(h[i])));
        } else {
            for (int i = 0; i < VEC && c0 + i < cols; i++) mx[i] = fmaxf(mx[i], fabsf(to_f<T>(p[i])));
        }
    }
    for (int i = 0; i < VEC && c0 + i < cols; i++)
        atomicMax(reinterpret_cast<int*>(out + c0 + i), __float_as_int(mx[i]));
}

// MathF.Pow result taken as the correctly rounded single-precision power: pow evaluated in
// double and rounded once to float.  The host C library's powf usually returns the same value
// but does not guarantee it, so agreement with the reference is exact only where it does.
__device__ __forceinline__ float powf_cr(float a, float b) { return (float)pow((double)a, (double)b); }

__global__ void smooth_scales_kernel(const float* act, const float* wmax, int64_t n, float alpha, float* s) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float num = powf_cr(fmaxf(act[i], 1e-5f), alpha);
        const float den = powf_cr(fmaxf(wmax[i], 1e-5f), __fsub_rn(1.f, alpha));
        s[i] = fmaxf(__fdiv_rn(num, den), 1e-5f);  // SmoothQuantModifier.cs:165-172
    }
}

// smooth /= s ; balance *= s, with s first rounded to the smooth weight's dtype
// (tensor(s).to(smoothW.dtype), SmoothQuantModifier.cs:174-178).
template <typename TS, typename TB>
__global__ void scale_apply_kernel(const float* s, TS* smooth, TB* balance, int64_t m, int64_t hidden) {
    const int64_t total = m * hidden;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total + hidden;
         t += (int64_t)gridDim.x * blockDim.x) {
        if (t < total) {
            const int64_t c = t % hidden;
            const float sc = rnd<TS>(s[c]);
            balance[t] = from_f<TB>(__fmul_rn(to_f<TB>(balance[t]), sc));
        } else if (smooth) {
            const int64_t c = t - total;
            const float sc = rnd<TS>(s[c]);
            smooth[c] = from_f<TS>(__fdiv_rn(to_f<TS>(smooth[c]), sc));
        }
    }
}

// AWQ: s_k[c] = max(a_c^(k/G) / wmax_c^(1-k/G), 1e-4) for k = 1..G (torch fp32 pow).
__global__ void awq_scales_kernel(const float* act, const float* wmax, int64_t n, int grid_pts, float* sk) {
    const int64_t total = (int64_t)grid_pts * n;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int k = (int)(t / n) + 1;
        const int64_t c = t % n;
        const float alpha = __fdiv_rn((float)k, (float)grid_pts);
        const float v = __fdiv_rn(powf_cr(act[c], alpha), powf_cr(wmax[c], __fsub_rn(1.f, alpha)));
        sk[t] = fmaxf(v, 1e-4f);
    }
}

// One pass per grid point over W: segment (row, group) min/max of W*s, affine params,
// fake-quant in fp32, squared error of FQ(W*s)/s - W accumulated in double.
// One warp per segment; lanes stride over the segment's columns.
template <typename T>
__global__ void __launch_bounds__(NT) awq_err_kernel(const T* W, int64_t m, int64_t n, int64_t ldw, int64_t gs,
                                                     const float* s, int bits, int sym, double* mse_acc) {
    const int64_t nseg = (n + gs - 1) / gs;
    const int64_t total = m * nseg;
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * NT + threadIdx.x) / 32;
    const int64_t nwarps = (int64_t)gridDim.x * NT / 32;
    float qmin, qmax;
    qrange(bits, sym, &qmin, &qmax);
    double acc = 0.0;
    for (int64_t seg = warp; seg < total; seg += nwarps) {
        const int64_t r = seg / nseg, c0 = (seg % nseg) * gs, c1 = min(n, c0 + gs);
        float mn = INFINITY, mx = -INFINITY;
        for (int64_t c = c0 + lane; c < c1; c += 32) {
            const float v = __fmul_rn(to_f<T>(W[r * ldw + c]), s[c]);
            mn = fminf(mn, v);
            mx = fmaxf(mx, v);
        }
        for (int o = 16; o > 0; o >>= 1) {
            mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        }
        float sc;
        int z;
        affine_params(mn, mx, bits, sym, &sc, &z);
        for (int64_t c = c0 + lane; c < c1; c += 32) {
            const float w = to_f<T>(W[r * ldw + c]);
            const float v = __fmul_rn(w, s[c]);
            int code;
            const float fq = fq_chain<float>(v, sc, (float)z, qmin, qmax, &code);
            const float e = __fsub_rn(__fdiv_rn(fq, s[c]), w);
            acc += (double)e * (double)e;
        }
    }
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) atomicAdd(mse_acc, acc);
}

// reciprocals of the grid's scales, for the error term FQ(W*s)/s of the one-pass search
__global__ void recip_kernel(const float* x, int64_t n, float* out) {
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x)
        out[t] = __frcp_rn(x[t]);
}

// One pass over W for every grid point (group strategy, group <= 256 columns).  A block owns one
// column group: it stages that group's columns of every s_k and 1 / s_k in shared memory, and its
// warps take rows.  A warp holds its (row, group) segment in registers (8 columns per lane) and,
// per grid point, takes the min / max of W * s_k with shuffles, the affine parameters, the
// fake-quantised value (x * rcp(scale) where that provably equals the op-by-op chain, the chain
// itself elsewhere, as in the GPTQ block kernel) and the squared error of FQ(W * s_k) / s_k - W,
// summed per lane in double in shared memory (a lane's PER squared errors of one grid point are
// added in fp32 first, then once in double).  W is read from memory once instead of twice per
// grid point.  The error divides by multiplying with 1 / s_k (within one unit in the last place of
// the quotient), so the sums differ from the per-point kernel's by about 1e-7 relative.
// Squared error of one (row, group) segment held by a warp (PER columns a lane) for one grid
// point: min / max of W * s_k, the affine parameters, the fake-quantised value and
// (FQ / s_k - W)^2 summed over the lane's columns in fp32.
template <int PER>
__device__ __forceinline__ float awq_seg_err(const float (&w)[PER], const float* sv, const float* rv, int lane, int L,
                                             int bits, int sym, float qmin, float qmax) {
    float v[PER];
    float mn = INFINITY, mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int col = lane + 32 * i;
        v[i] = col < L ? __fmul_rn(w[i], sv[col]) : 0.f;
        if (col < L) {
            mn = fmin_nan(mn, v[i]);
            mx = fmax_nan(mx, v[i]);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mn = fmin_nan(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmax_nan(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    float sc;
    int z;
    affine_params(mn, mx, bits, sym, &sc, &z);
    const float zf = (float)z;
    const float rsc = __frcp_rn(sc);
    const bool rs_ok = fabsf(rsc) <= 3.0e38f && rsc != 0.f;
    float part = 0.f;
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int col = lane + 32 * i;
        if (col >= L) continue;
        float fq;
        const float f = __fmul_rn(v[i], rsc);
        const float fr = rintf(f);
        if (!rs_ok || fabsf(fabsf(__fsub_rn(f, fr)) - 0.5f) <= fabsf(f) * 4.8e-7f + 1e-30f) {
            int code;
            fq = fq_chain<float>(v[i], sc, zf, qmin, qmax, &code);
        } else {
            float t = __fadd_rn(fr, zf);
            t = (t < qmin) ? qmin : ((t > qmax) ? qmax : t);
            fq = __fmul_rn(__fsub_rn(t, zf), sc);
        }
        const float e = __fsub_rn(__fmul_rn(fq, rv[col]), w[i]);
        part = __fmaf_rn(e, e, part);
    }
    return part;
}

constexpr int AWQ_WARPS = NT / 32;
constexpr int AWQ_PER = 8;  // columns per lane: groups of up to 256

template <typename T, int PER>
__global__ void __launch_bounds__(NT) awq_err_group_kernel(const T* W, int64_t m, int64_t n, int64_t ldw, int gs,
                                                           const float* sk, const float* rsk, int grid_pts, int bits,
                                                           int sym, double* sums) {
    extern __shared__ __align__(16) unsigned char awq_smem[];
    double* accs = reinterpret_cast<double*>(awq_smem);           // [warps][grid_pts][32]
    float* ss = reinterpret_cast<float*>(accs + (size_t)AWQ_WARPS * grid_pts * 32);  // [grid_pts][gs]
    float* rs = ss + (size_t)grid_pts * gs;                        // [grid_pts][gs]
    const int64_t c0 = (int64_t)blockIdx.x * gs;
    const int L = (int)min((int64_t)gs, n - c0);
    for (int t = threadIdx.x; t < grid_pts * gs; t += NT) {
        const int k = t / gs, i = t % gs;
        ss[t] = i < L ? sk[(int64_t)k * n + c0 + i] : 1.f;
        rs[t] = i < L ? rsk[(int64_t)k * n + c0 + i] : 1.f;
    }
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    double* acc = accs + (size_t)warp * grid_pts * 32 + lane;
    for (int k = 0; k < grid_pts; k++) acc[k * 32] = 0.0;
    __syncthreads();
    float qmin, qmax;
    qrange(bits, sym, &qmin, &qmax);
    // Two rows per pass (r and r + stride; a missing second row is all zeros, whose error is 0):
    // the two rows' chains per grid point (shuffles, affine parameters, reciprocal, elements) are
    // independent, so their latencies overlap.
    const int64_t stride = (int64_t)gridDim.y * AWQ_WARPS;
    for (int64_t r = (int64_t)blockIdx.y * AWQ_WARPS + warp; r < m; r += 2 * stride) {
        const int64_t r2 = r + stride;
        float w[PER], w2[PER];
#pragma unroll
        for (int i = 0; i < PER; i++) {
            const int col = lane + 32 * i;
            w[i] = col < L ? to_f<T>(W[r * ldw + c0 + col]) : 0.f;
            w2[i] = (col < L && r2 < m) ? to_f<T>(W[r2 * ldw + c0 + col]) : 0.f;
        }
#pragma unroll 1
        for (int k = 0; k < grid_pts; k++) {
            const float* sv = ss + k * gs;
            const float* rv = rs + k * gs;
            const float p1 = awq_seg_err<PER>(w, sv, rv, lane, L, bits, sym, qmin, qmax);
            const float p2 = awq_seg_err<PER>(w2, sv, rv, lane, L, bits, sym, qmin, qmax);
            acc[k * 32] += (double)p1 + (double)p2;
        }
    }
    __syncthreads();
    // sum over warps and lanes: one thread per grid point
    for (int k = threadIdx.x; k < grid_pts; k += NT) {
        double t = 0.0;
        for (int wq = 0; wq < AWQ_WARPS; wq++)
            for (int l = 0; l < 32; l++) t += accs[((size_t)wq * grid_pts + k) * 32 + l];
        atomicAdd(sums + k, t);
    }
}

// Squared errors of a lane's PER columns for one grid point, pairs of columns on the paired fp32
// instructions (each component rounded as its scalar form): f = v * rcp(s), rint(f) as
// (f + 1.5 * 2^23) - 1.5 * 2^23, fq = (clamp(rint(f) + zp) - zp) * s, e = fq * (1 / s_k) - w.
// The chain replaces fq where the quotient may round otherwise than v / s: within 4.8e-7 |f| of a
// half-integer, |f| >= 2^22 (where the rint trick no longer holds; caught by the same bound), a
// NaN, or a scale without a finite reciprocal.  The clamp runs only in warps that need it.
template <int PER, bool CLAMP>
__device__ __forceinline__ float2 awq_pairs(const float (&v)[PER], const float (&w)[PER], const float4* rv, float rsc,
                                            float sc, float zf, float qmin, float qmax, bool rs_ok) {
    const float2 rsc2 = make_float2(rsc, rsc), sc2 = make_float2(sc, sc);
    const float2 zf2 = make_float2(zf, zf), nzf2 = make_float2(-zf, -zf);
    const float2 mg2 = make_float2(12582912.f, 12582912.f), nmg2 = make_float2(-12582912.f, -12582912.f);
    const float2 neg1 = make_float2(-1.f, -1.f);
    float2 part2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int q = 0; q < PER / 4; q++) {
        const float4 r4 = rv[q];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int e0 = 4 * q + 2 * h;
            const float2 f = __fmul2_rn(make_float2(v[e0], v[e0 + 1]), rsc2);
            const float2 fr = __fadd2_rn(__fadd2_rn(f, mg2), nmg2);
            const float2 d = __ffma2_rn(fr, neg1, f);  // f - fr
            float2 t = __fadd2_rn(fr, zf2);
            if constexpr (CLAMP) {
                t.x = fminf(fmaxf(t.x, qmin), qmax);
                t.y = fminf(fmaxf(t.y, qmin), qmax);
            }
            float2 fq = __fmul2_rn(__fadd2_rn(t, nzf2), sc2);
            // |d| <= 0.5, so "within 4.8e-7 |f| of a half-integer" is |d| + 4.8e-7 |f| >= 0.5
            if (!rs_ok || !(fmaf(fabsf(f.x), 4.8e-7f, fabsf(d.x)) < 0.5f)) {
                int code;
                fq.x = fq_chain<float>(v[e0], sc, zf, qmin, qmax, &code);
            }
            if (!rs_ok || !(fmaf(fabsf(f.y), 4.8e-7f, fabsf(d.y)) < 0.5f)) {
                int code;
                fq.y = fq_chain<float>(v[e0 + 1], sc, zf, qmin, qmax, &code);
            }
            const float2 pr = __fmul2_rn(fq, h ? make_float2(r4.z, r4.w) : make_float2(r4.x, r4.y));
            const float2 e = __ffma2_rn(make_float2(w[e0], w[e0 + 1]), neg1, pr);  // fq / s_k - w
            part2 = __ffma2_rn(e, e, part2);
        }
    }
    return part2;
}

// The one-pass search with several rows a warp (2-byte weights; group width a multiple of PER
// and a divisor of n): a (row, group) segment takes L = gs / PER lanes holding PER consecutive
// columns each, so a warp covers 32 / L rows at once and one instruction stream serves all of
// them.  Per grid point and lane that shares the min / max shuffles (log2 L rounds), the affine
// parameters and the reciprocal among PER elements instead of gs / 32, and reads s_k and 1 / s_k
// as 16-byte vectors.  Rows past m are all zeros (error 0).  The arithmetic per element is
// awq_seg_err's.
template <typename T, int PER>
__global__ void __launch_bounds__(NT) awq_err_rows_kernel(const T* W, int64_t m, int64_t n, int64_t ldw, int gs,
                                                          const float* sk, const float* rsk, int grid_pts, int bits,
                                                          int sym, double* sums) {
    extern __shared__ __align__(16) unsigned char awq_smem[];
    double* accs = reinterpret_cast<double*>(awq_smem);           // [warps][grid_pts][32]
    float* ss = reinterpret_cast<float*>(accs + (size_t)AWQ_WARPS * grid_pts * 32);  // [grid_pts][gs]
    float* rs = ss + (size_t)grid_pts * gs;                        // [grid_pts][gs]
    const int64_t c0 = (int64_t)blockIdx.x * gs;
    for (int t = threadIdx.x; t < grid_pts * gs; t += NT) {
        const int k = t / gs, i = t % gs;
        ss[t] = sk[(int64_t)k * n + c0 + i];
        rs[t] = rsk[(int64_t)k * n + c0 + i];
    }
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int L = gs / PER;        // lanes a segment (power of two)
    const int rpw = 32 / L;        // rows a warp
    const int sub = lane % L, rsub = lane / L;
    double* acc = accs + (size_t)warp * grid_pts * 32 + lane;
    for (int k = 0; k < grid_pts; k++) acc[k * 32] = 0.0;
    __syncthreads();
    float qmin, qmax;
    qrange(bits, sym, &qmin, &qmax);
    const int64_t stride = (int64_t)gridDim.y * AWQ_WARPS * rpw;
    for (int64_t rb = ((int64_t)blockIdx.y * AWQ_WARPS + warp) * rpw; rb < m; rb += stride) {
        const int64_t r = rb + rsub;
        float w[PER];
        if (r < m) {
            const uint4* src = reinterpret_cast<const uint4*>(W + r * ldw + c0 + (int64_t)sub * PER);
#pragma unroll
            for (int q = 0; q < PER / 8; q++) {
                const uint4 u = src[q];
                const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
                for (int i = 0; i < 8; i++) w[q * 8 + i] = to_f<T>(h[i]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < PER; i++) w[i] = 0.f;
        }
#pragma unroll 1
        for (int k = 0; k < grid_pts; k++) {
            const float4* sv = reinterpret_cast<const float4*>(ss + k * gs + sub * PER);
            const float4* rv = reinterpret_cast<const float4*>(rs + k * gs + sub * PER);
            float v[PER];
            float mn = INFINITY, mx = -INFINITY;
#pragma unroll
            for (int q = 0; q < PER / 4; q++) {
                const float4 s4 = sv[q];
                const float2 a = __fmul2_rn(make_float2(w[4 * q + 0], w[4 * q + 1]), make_float2(s4.x, s4.y));
                const float2 c = __fmul2_rn(make_float2(w[4 * q + 2], w[4 * q + 3]), make_float2(s4.z, s4.w));
                v[4 * q + 0] = a.x;
                v[4 * q + 1] = a.y;
                v[4 * q + 2] = c.x;
                v[4 * q + 3] = c.y;
            }
#pragma unroll
            for (int i = 0; i < PER; i++) {
                mn = fmin_nan(mn, v[i]);
                mx = fmax_nan(mx, v[i]);
            }
            for (int o = L / 2; o > 0; o >>= 1) {
                mn = fmin_nan(mn, __shfl_xor_sync(0xffffffffu, mn, o));
                mx = fmax_nan(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            }
            float sc;
            int z;
            affine_params(mn, mx, bits, sym, &sc, &z);
            const float zf = (float)z;
            const float rsc = __frcp_rn(sc);
            const bool rs_ok = fabsf(rsc) <= 3.0e38f && rsc != 0.f;
            // The clamp to [qmin, qmax] can act only if an extreme's code leaves the grid: on the
            // fast path v -> rint(v * rcp(s)) is monotone, so the segment's extremes bound every
            // element; an extreme near a half-integer (or off the fast path) counts as leaving.
            bool clamp_need = true;
            if (rs_ok) {
                const float fx = __fmul_rn(mx, rsc), fn = __fmul_rn(mn, rsc);
                const float rx = __fsub_rn(__fadd_rn(fx, 12582912.f), 12582912.f);
                const float rn = __fsub_rn(__fadd_rn(fn, 12582912.f), 12582912.f);
                const bool tie = !(fmaf(fabsf(fx), 4.8e-7f, fabsf(__fsub_rn(fx, rx))) < 0.5f) ||
                                 !(fmaf(fabsf(fn), 4.8e-7f, fabsf(__fsub_rn(fn, rn))) < 0.5f);
                clamp_need = tie || __fadd_rn(rx, zf) > qmax || __fadd_rn(rn, zf) < qmin;
            }
            const float2 pr2 = __any_sync(0xffffffffu, clamp_need)
                                   ? awq_pairs<PER, true>(v, w, rv, rsc, sc, zf, qmin, qmax, rs_ok)
                                   : awq_pairs<PER, false>(v, w, rv, rsc, sc, zf, qmin, qmax, rs_ok);
            const float2 part2 = pr2;
            const float part = __fadd_rn(part2.x, part2.y);
            acc[k * 32] += (double)part;
        }
    }
    __syncthreads();
    for (int k = threadIdx.x; k < grid_pts; k += NT) {
        double t = 0.0;
        for (int wq = 0; wq < AWQ_WARPS; wq++)
            for (int l = 0; l < 32; l++) t += accs[((size_t)wq * grid_pts + k) * 32 + l];
        atomicAdd(sums + k, t);
    }
}

__global__ void awq_pick_kernel(const double* sums, int grid_pts, double denom, const float* sk, int64_t n, double* mse_out,
                                float* best_s, int* best_k) {
    __shared__ int kbest;
    if (threadIdx.x == 0) {
        double best = INFINITY;
        int kb = 1;
        for (int k = 0; k < grid_pts; k++) {
            const double v = sums[k] / denom;
            if (mse_out) mse_out[k] = v;
            if (v < best) {
                best = v;
                kb = k + 1;
            }
        }
        kbest = kb;
        best_k[0] = kb;
    }
    __syncthreads();
    for (int64_t c = threadIdx.x; c < n; c += blockDim.x) best_s[c] = sk[(int64_t)(kbest - 1) * n + c];
}

int grid_for(llmc_ctx* ctx, int64_t items) {
    int64_t b = (items + NT - 1) / NT;
    int64_t cap = (int64_t)ctx->sm_count * 8;
    return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

template <typename T>
llmc_status launch_col_absmax(llmc_ctx* ctx, const void* x, int64_t rows, int64_t cols, int64_t ld, float* out) {
    constexpr int V = 16 / sizeof(T);
    const bool vec = ((uintptr_t)x % 16 == 0) && (ld % V == 0);
    const int vv = vec ? V : 1;
    const int64_t col_threads = (cols + vv - 1) / vv;
    const unsigned gx = (unsigned)((col_threads + NT - 1) / NT);
    int64_t want_blocks = (int64_t)ctx->sm_count * 8;
    int64_t gy = want_blocks / gx;
    if (gy < 1) gy = 1;
    if (gy > rows) gy = rows > 0 ? rows : 1;
    if (gy > 65535) gy = 65535;
    const int64_t rpb = (rows + gy - 1) / gy;
    gy = (rows + rpb - 1) / rpb;
    if (gy < 1) gy = 1;
    dim3 grid(gx, (unsigned)gy);
    if (vec) col_absmax_kernel<T, V><<<grid, NT, 0, ctx->stream>>>((const T*)x, rows, cols, ld, rpb, out);
    else col_absmax_kernel<T, 1><<<grid, NT, 0, ctx->stream>>>((const T*)x, rows, cols, ld, rpb, out);
    return check_launch(ctx, "col_absmax");
}

}  // namespace

llmc_status col_absmax(llmc_ctx* ctx, const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, float* out,
                       int accumulate) {
    if (!accumulate) LLMC_CUDA_TRY(cudaMemsetAsync(out, 0, (size_t)cols * sizeof(float), ctx->stream));
    if (rows <= 0) return LLMC_OK;
    switch (dtype) {
        case LLMC_DTYPE_F32: return launch_col_absmax<float>(ctx, x, rows, cols, ld, out);
        case LLMC_DTYPE_BF16: return launch_col_absmax<__nv_bfloat16>(ctx, x, rows, cols, ld, out);
        case LLMC_DTYPE_F16: return launch_col_absmax<__half>(ctx, x, rows, cols, ld, out);
    }
    return fail(LLMC_ERR_INVALID_ARG, "bad dtype");
}

llmc_status scale_apply(llmc_ctx* ctx, const float* s, void* smooth, int sdt, void* balance, int bdt, int64_t m,
                        int64_t hidden) {
    const int g = grid_for(ctx, m * hidden + hidden);
#define LLMC_SA(TS, TB) \
    scale_apply_kernel<TS, TB><<<g, NT, 0, ctx->stream>>>(s, (TS*)smooth, (TB*)balance, m, hidden)
    if (sdt == LLMC_DTYPE_F32 && bdt == LLMC_DTYPE_F32) LLMC_SA(float, float);
    else if (sdt == LLMC_DTYPE_BF16 && bdt == LLMC_DTYPE_BF16) LLMC_SA(__nv_bfloat16, __nv_bfloat16);
    else if (sdt == LLMC_DTYPE_F16 && bdt == LLMC_DTYPE_F16) LLMC_SA(__half, __half);
    else if (sdt == LLMC_DTYPE_F32 && bdt == LLMC_DTYPE_BF16) LLMC_SA(float, __nv_bfloat16);
    else if (sdt == LLMC_DTYPE_BF16 && bdt == LLMC_DTYPE_F32) LLMC_SA(__nv_bfloat16, float);
    else return fail(LLMC_ERR_UNSUPPORTED, "scale_apply: dtype pair (%d, %d) not supported", sdt, bdt);
#undef LLMC_SA
    return check_launch(ctx, "scale_apply");
}

llmc_status smooth_apply(llmc_ctx* ctx, const float* act_max, void* smooth, int sdt, void* balance, int bdt, int64_t m,
                         int64_t hidden, float alpha, float* s_out) {
    void* wsp;
    LLMC_TRY(workspace(ctx, (size_t)hidden * 8 + 1024, &wsp));
    Carver cv{(char*)wsp};
    float* wmax = cv.take<float>(hidden);
    float* s = s_out ? s_out : cv.take<float>(hidden);
    LLMC_TRY(col_absmax(ctx, balance, bdt, m, hidden, hidden, wmax, 0));
    smooth_scales_kernel<<<grid_for(ctx, hidden), NT, 0, ctx->stream>>>(act_max, wmax, hidden, alpha, s);
    LLMC_TRY(check_launch(ctx, "smooth_scales"));
    return scale_apply(ctx, s, smooth, sdt, balance, bdt, m, hidden);
}

llmc_status awq_search(llmc_ctx* ctx, const void* W, int dtype, int64_t m, int64_t n, int64_t ldw, const float* act_max,
                       int grid_pts, const llmc_qconfig* cfg, float* best_s, double* mse_out, int32_t* best_k) {
    void* wsp;
    LLMC_TRY(workspace(ctx, (size_t)n * 4 + (size_t)grid_pts * n * 4 + (size_t)grid_pts * 8 + 2048, &wsp));
    Carver cv{(char*)wsp};
    float* wmax = cv.take<float>(n);
    float* sk = cv.take<float>((size_t)grid_pts * n);
    double* sums = cv.take<double>(grid_pts);
    int* kdev = cv.take<int>(4);
    LLMC_TRY(col_absmax(ctx, W, dtype, m, n, ldw, wmax, 0));
    awq_scales_kernel<<<grid_for(ctx, (int64_t)grid_pts * n), NT, 0, ctx->stream>>>(act_max, wmax, n, grid_pts, sk);
    LLMC_TRY(check_launch(ctx, "awq_scales"));
    LLMC_CUDA_TRY(cudaMemsetAsync(sums, 0, (size_t)grid_pts * sizeof(double), ctx->stream));
    const int64_t gs = cfg->strategy == LLMC_STRATEGY_GROUP ? cfg->group_size : n;
    const int64_t segs = m * ((n + gs - 1) / gs);
    int64_t nb = (segs + 7) / 8;
    if (nb > (int64_t)ctx->sm_count * 8) nb = (int64_t)ctx->sm_count * 8;
    int blocks = (int)nb;
    if (blocks < 1) blocks = 1;
    const size_t smem = (size_t)AWQ_WARPS * grid_pts * 32 * 8 + (size_t)2 * grid_pts * gs * 4;
    if (cfg->strategy == LLMC_STRATEGY_GROUP && gs <= 32 * AWQ_PER && smem <= 200 * 1024 && ctx->device >= 0 &&
        ctx->device < 64) {
        float* rsk = nullptr;
        void* wsp2;
        LLMC_TRY(workspace2(ctx, (size_t)grid_pts * n * 4 + 256, &wsp2));
        rsk = static_cast<float*>(wsp2);
        recip_kernel<<<grid_for(ctx, (int64_t)grid_pts * n), NT, 0, ctx->stream>>>(sk, (int64_t)grid_pts * n, rsk);
        LLMC_TRY(check_launch(ctx, "recip"));
        const int64_t ngroups = (n + gs - 1) / gs;
        // Several rows a warp: 2-byte weights in 16-byte rows, whole groups of 16 (or 8) * 2^j
        // columns.
        auto pow2 = [](int64_t v) { return v >= 1 && (v & (v - 1)) == 0; };
        int rper = 0;
        if ((dtype == LLMC_DTYPE_BF16 || dtype == LLMC_DTYPE_F16) && n % gs == 0 && (uintptr_t)W % 16 == 0 &&
            ldw % 8 == 0) {
            if (gs % 16 == 0 && pow2(gs / 16) && gs / 16 <= 32) rper = 16;
            else if (gs % 8 == 0 && pow2(gs / 8) && gs / 8 <= 32) rper = 8;
        }
        if (rper) {
            static bool rattr[64][2][2];
            const int di = dtype == LLMC_DTYPE_BF16 ? 0 : 1, qi = rper == 16 ? 0 : 1;
            const int64_t rows_per_block = (int64_t)AWQ_WARPS * (32 / (gs / rper));
            const int64_t rmax = (m + rows_per_block - 1) / rows_per_block;
#define LLMC_AWQR(T, PER)                                                                                         \
    do {                                                                                                          \
        auto kern = awq_err_rows_kernel<T, PER>;                                                                  \
        if (!rattr[ctx->device][di][qi]) {                                                                        \
            LLMC_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));    \
            rattr[ctx->device][di][qi] = true;                                                                    \
        }                                                                                                         \
        int per_sm = 0;                                                                                           \
        LLMC_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NT, smem));                    \
        const int64_t slots = (int64_t)ctx->sm_count * (per_sm > 0 ? per_sm : 1);                                \
        int64_t ry = slots / ngroups;                                                                             \
        if (ry > rmax) ry = rmax;                                                                                 \
        if (ry < 1) ry = 1;                                                                                       \
        if (ry > 65535) ry = 65535;                                                                               \
        kern<<<dim3((unsigned)ngroups, (unsigned)ry), NT, smem, ctx->stream>>>((const T*)W, m, n, ldw, (int)gs, sk, \
                                                                              rsk, grid_pts, cfg->num_bits,       \
                                                                              cfg->symmetric, sums);              \
    } while (0)
            if (dtype == LLMC_DTYPE_BF16) {
                if (rper == 16) LLMC_AWQR(__nv_bfloat16, 16);
                else LLMC_AWQR(__nv_bfloat16, 8);
            } else {
                if (rper == 16) LLMC_AWQR(__half, 16);
                else LLMC_AWQR(__half, 8);
            }
#undef LLMC_AWQR
            LLMC_TRY(check_launch(ctx, "awq_err_rows"));
            goto picked;
        }
        {
        const int64_t ry_max = (m + AWQ_WARPS - 1) / AWQ_WARPS;
        static bool attr[64][3][2];
        const int ti = dtype == LLMC_DTYPE_F32 ? 0 : (dtype == LLMC_DTYPE_BF16 ? 1 : 2);
        const int pi = gs <= 128 ? 0 : 1;
        // Rows per group column: as many blocks as fit on the GPU at once (one wave), so no
        // second, partly filled wave doubles the time of the last blocks.
#define LLMC_AWQ1(T)                                                                                              \
    do {                                                                                                          \
        auto kern = pi == 0 ? awq_err_group_kernel<T, 4> : awq_err_group_kernel<T, AWQ_PER>;                       \
        if (!attr[ctx->device][ti][pi]) {                                                                         \
            LLMC_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));    \
            attr[ctx->device][ti][pi] = true;                                                                     \
        }                                                                                                         \
        int per_sm = 0;                                                                                           \
        LLMC_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NT, smem));                    \
        const int64_t slots = (int64_t)ctx->sm_count * (per_sm > 0 ? per_sm : 1);                                \
        int64_t ry = slots / ngroups;                                                                             \
        if (ry > ry_max) ry = ry_max;                                                                             \
        if (ry < 1) ry = 1;                                                                                       \
        if (ry > 65535) ry = 65535;                                                                               \
        kern<<<dim3((unsigned)ngroups, (unsigned)ry), NT, smem, ctx->stream>>>((const T*)W, m, n, ldw, (int)gs, sk, \
                                                                              rsk, grid_pts, cfg->num_bits,       \
                                                                              cfg->symmetric, sums);              \
    } while (0)
        switch (dtype) {
            case LLMC_DTYPE_F32: LLMC_AWQ1(float); break;
            case LLMC_DTYPE_BF16: LLMC_AWQ1(__nv_bfloat16); break;
            case LLMC_DTYPE_F16: LLMC_AWQ1(__half); break;
            default: return fail(LLMC_ERR_INVALID_ARG, "bad dtype");
        }
#undef LLMC_AWQ1
        LLMC_TRY(check_launch(ctx, "awq_err_group"));
        }
    } else {
        for (int k = 0; k < grid_pts; k++) {
            const float* s = sk + (int64_t)k * n;
            switch (dtype) {
                case LLMC_DTYPE_F32:
                    awq_err_kernel<float><<<blocks, NT, 0, ctx->stream>>>((const float*)W, m, n, ldw, gs, s, cfg->num_bits,
                                                                          cfg->symmetric, sums + k);
                    break;
                case LLMC_DTYPE_BF16:
                    awq_err_kernel<__nv_bfloat16><<<blocks, NT, 0, ctx->stream>>>((const __nv_bfloat16*)W, m, n, ldw, gs, s,
                                                                                  cfg->num_bits, cfg->symmetric, sums + k);
                    break;
                case LLMC_DTYPE_F16:
                    awq_err_kernel<__half><<<blocks, NT, 0, ctx->stream>>>((const __half*)W, m, n, ldw, gs, s, cfg->num_bits,
                                                                           cfg->symmetric, sums + k);
                    break;
                default: return fail(LLMC_ERR_INVALID_ARG, "bad dtype");
            }
            LLMC_TRY(check_launch(ctx, "awq_err"));
        }
    }
picked:
    awq_pick_kernel<<<1, NT, 0, ctx->stream>>>(sums, grid_pts, (double)m * (double)n, sk, n, mse_out, best_s, kdev);
    LLMC_TRY(check_launch(ctx, "awq_pick"));
    if (!best_k) return LLMC_OK;  // best_s and mse_out are written in stream order
    LLMC_CUDA_TRY(cudaMemcpyAsync(ctx->hflags, kdev, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
    LLMC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    *best_k = ctx->hflags[0];
    return LLMC_OK;
}

}  // namespace llmc
