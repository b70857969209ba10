// Observers, affine parameters, fake quantisation, RTN quantise+pack, int4 packing.
//
// Reference: MinMaxObserver.cs:24-45, PerChannelMinMaxObserver.cs:38-76, Observer.cs:47-75,
// FakeQuantizeFunction.cs:30-47, RtnModifier.cs:44-122, Int4PackedTensor.cs:47-161.
//
// These are HBM-bound streams.  A "segment" is the set of elements that share one
// (scale, zero-point): a whole row (per-channel), a (row, group) slice (group) or a row as
// the first level of a per-tensor reduction.  A group of L lanes (L a power of two <= 32)
// owns one segment and walks it with 16-byte vector loads, so a warp covers 32*16 bytes
// of consecutive columns per step; the segment's min/max is combined with xor shuffles
// inside the lane group.
#include "ops.h"

#include <type_traits>

namespace llmc {
namespace {

constexpr int NT = 256;

template <typename T, int VEC>
struct Vec {
    float v[VEC];
    __device__ __forceinline__ void load(const T* p) {
        if constexpr (VEC == 1) {
            v[0] = to_f<T>(p[0]);
        } else {
            static_assert(VEC * sizeof(T) == 16, "16-byte vectors");
            uint4 q = *reinterpret_cast<const uint4*>(p);
            const T* h = reinterpret_cast<const T*>(&q);
#pragma unroll
            for (int i = 0; i < VEC; i++) v[i] = to_f<T>(h[i]);
        }
    }
};

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

// Segment geometry shared by the min/max and the fused RTN kernels.
struct SegGeom {
    int64_t rows, cols, ld, gs, nseg;  // nseg = segments per row
    int L;                              // lanes per segment
};

template <typename T, int VEC>
__device__ __forceinline__ void seg_reduce(const T* x, const SegGeom& g, int64_t seg, bool active, float& mn,
                                           float& mx) {
    mn = INFINITY;
    mx = -INFINITY;
    const int sub = lane_id() % g.L;
    int64_t r = 0, c0 = 0, c1 = 0;
    if (active) {
        r = seg / g.nseg;
        const int64_t s = seg % g.nseg;
        c0 = s * g.gs;
        c1 = min(g.cols, c0 + g.gs);
    }
    const T* row = x + r * g.ld;
    for (int64_t c = c0 + (int64_t)sub * VEC; c < c1; c += (int64_t)g.L * VEC) {
        if (c + VEC <= c1) {
            Vec<T, VEC> v;
            v.load(row + c);
#pragma unroll
            for (int i = 0; i < VEC; i++) {
                mn = fmin_nan(mn, v.v[i]);
                mx = fmax_nan(mx, v.v[i]);
            }
        } else {
            for (int64_t i = c; i < c1; i++) {
                float f = to_f<T>(row[i]);
                mn = fmin_nan(mn, f);
                mx = fmax_nan(mx, f);
            }
        }
    }
    for (int off = g.L / 2; off > 0; off >>= 1) {
        mn = fmin_nan(mn, __shfl_xor_sync(0xffffffffu, mn, off));
        mx = fmax_nan(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(NT) seg_minmax_kernel(const T* x, SegGeom g, float* mins, float* maxs, int fold) {
    const int64_t groups_per_block = NT / g.L;
    const int64_t total = g.rows * g.nseg;
    const int64_t lg = threadIdx.x / g.L;
    for (int64_t base = (int64_t)blockIdx.x * groups_per_block; base < total;
         base += (int64_t)gridDim.x * groups_per_block) {
        // Loop bound is uniform across the block, so every lane reaches the shuffles.
        const int64_t seg = base + lg;
        const bool active = seg < total;
        float mn, mx;
        seg_reduce<T, VEC>(x, g, seg, active, mn, mx);
        if (active && (lane_id() % g.L) == 0) {
            mn = fold_min(mn, mins + seg, fold);
            mx = fold_max(mx, maxs + seg, fold);
            mins[seg] = mn;
            maxs[seg] = mx;
        }
    }
}

// Division of a segment index by the (runtime) number of segments per row with one
// multiply-high, add and shift (Granlund and Montgomery, "Division by invariant integers
// using multiplication", 1994): for 1 <= d < 2^31, l = ceil(log2 d), m = floor(2^32 (2^l - d)
// / d) + 1, n / d = (mulhi(n, m) + n) >> l for every n < 2^31.
struct FastDiv {
    uint32_t m, l;
};

FastDiv make_fastdiv(uint32_t d) {
    uint32_t l = 0;
    while ((1ull << l) < d) l++;
    const uint64_t m = ((1ull << 32) * ((1ull << l) - d)) / d + 1;
    return FastDiv{(uint32_t)m, l};
}

__device__ __forceinline__ uint32_t fastdiv(uint32_t n, FastDiv f) { return (__umulhi(n, f.m) + n) >> f.l; }

// Lanes of one segment load RV vectors each per step (segments of RV * L * VEC elements take
// one step; longer ones loop), with one min/max pair per vector slot to keep the dependency
// chains short.  Segment s of the launch is row s / nseg, columns (s % nseg) * seglen ...
constexpr int RV = 4;

template <typename T, int VEC>
__global__ void __launch_bounds__(NT) seg_minmax_reg_kernel(const T* x, SegGeom g, FastDiv fd, float* mins,
                                                            float* maxs, int fold) {
    const int L = g.L;
    const uint32_t gpb = NT / L;
    const uint32_t total = (uint32_t)(g.rows * g.nseg);
    const uint32_t lg = threadIdx.x / L;
    const int sub = lane_id() % L;
    const int64_t seglen = g.gs < g.cols ? g.gs : g.cols;
    for (uint32_t base = blockIdx.x * gpb; base < total; base += gridDim.x * gpb) {
        const uint32_t seg = base + lg;
        const bool active = seg < total;
        const uint32_t sg = active ? seg : 0;
        const uint32_t r = fastdiv(sg, fd);
        const T* row = x + (int64_t)r * g.ld + (int64_t)(sg - r * (uint32_t)g.nseg) * seglen;
        float mn[RV], mx[RV];
#pragma unroll
        for (int j = 0; j < RV; j++) {
            mn[j] = INFINITY;
            mx[j] = -INFINITY;
        }
        if (active) {
            for (int64_t c = (int64_t)sub * VEC; c < seglen; c += (int64_t)L * VEC * RV) {
                Vec<T, VEC> v[RV];
#pragma unroll
                for (int j = 0; j < RV; j++) v[j].load(row + c + (int64_t)j * L * VEC);
#pragma unroll
                for (int j = 0; j < RV; j++)
#pragma unroll
                    for (int i = 0; i < VEC; i++) {
                        mn[j] = fmin_nan(mn[j], v[j].v[i]);
                        mx[j] = fmax_nan(mx[j], v[j].v[i]);
                    }
            }
        }
        float a = fmin_nan(fmin_nan(mn[0], mn[1]), fmin_nan(mn[2], mn[3]));
        float b = fmax_nan(fmax_nan(mx[0], mx[1]), fmax_nan(mx[2], mx[3]));
        for (int off = L / 2; off > 0; off >>= 1) {
            a = fmin_nan(a, __shfl_xor_sync(0xffffffffu, a, off));
            b = fmax_nan(b, __shfl_xor_sync(0xffffffffu, b, off));
        }
        if (active && sub == 0) {
            mins[seg] = fold_min(a, mins + seg, fold);
            maxs[seg] = fold_max(b, maxs + seg, fold);
        }
    }
}

// Lanes per segment for the register kernels: segments of RV * L * VEC elements (L a power of
// two <= 32), or L = 32 for segments that are a multiple of 32 * RV * VEC; 0 = not eligible.
int reg_lanes(int64_t seglen, int vec) {
    if (seglen % ((int64_t)RV * vec) != 0) return 0;
    if (seglen % ((int64_t)32 * RV * vec) == 0) return 32;
    const int64_t l = seglen / ((int64_t)RV * vec);
    return (l >= 1 && l <= 32 && (l & (l - 1)) == 0) ? (int)l : 0;
}

__global__ void affine_kernel(const float* mins, const float* maxs, int64_t count, int bits, int sym, float* scales,
                              int32_t* zps) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
        float s;
        int z;
        affine_params(mins[i], maxs[i], bits, sym, &s, &z);
        scales[i] = s;
        zps[i] = z;
    }
}

// Writes VEC codes of one row starting at column c (c even when packing nibbles).
template <int VEC>
__device__ __forceinline__ void store_codes(uint8_t* row_codes, int64_t c, const int* q, int zp, int bits, int n_valid) {
    if (bits <= 4) {
        if (n_valid == VEC && (VEC % 2) == 0) {
            uint8_t b[VEC / 2 > 0 ? VEC / 2 : 1];
#pragma unroll
            for (int i = 0; i < VEC / 2; i++)
                b[i] = (uint8_t)((((q[2 * i] - zp) & 0xF) << 4) | ((q[2 * i + 1] - zp) & 0xF));
            uint8_t* p = row_codes + c / 2;
            if constexpr (VEC == 8) *reinterpret_cast<uint32_t*>(p) = *reinterpret_cast<uint32_t*>(b);
            else if constexpr (VEC == 4) *reinterpret_cast<uint16_t*>(p) = *reinterpret_cast<uint16_t*>(b);
            else
#pragma unroll
                for (int i = 0; i < VEC / 2; i++) p[i] = b[i];
        } else {
            for (int i = 0; i < n_valid; i++) {
                const int64_t col = c + i;
                uint8_t nib = (uint8_t)((q[i] - zp) & 0xF);
                uint8_t* p = row_codes + col / 2;
                if (col % 2 == 0) *p = (uint8_t)((*p & 0x0F) | (nib << 4));
                else *p = (uint8_t)((*p & 0xF0) | nib);
            }
        }
    } else {
        for (int i = 0; i < n_valid; i++) row_codes[c + i] = (uint8_t)q[i];
    }
}

__host__ __device__ inline int64_t code_row_bytes(int bits, int64_t n) { return bits <= 4 ? (n + 1) / 2 : n; }

// Fused observer + fake-quant for CHANNEL / GROUP, or fake-quant with one scale (TENSOR,
// params precomputed into scales[0]/zps[0]).
template <typename T, int VEC>
__global__ void __launch_bounds__(NT) rtn_kernel(const T* x, SegGeom g, int bits, int sym, int tensor_mode,
                                                  float* scales, int32_t* zps, uint8_t* codes, T* deq, int64_t ld_deq) {
    const int64_t groups_per_block = NT / g.L;
    const int64_t total = g.rows * g.nseg;
    const int64_t lg = threadIdx.x / g.L;
    const int sub = lane_id() % g.L;
    float qmin, qmax;
    qrange(bits, sym, &qmin, &qmax);
    const int64_t crow = code_row_bytes(bits, g.cols);
    for (int64_t base = (int64_t)blockIdx.x * groups_per_block; base < total;
         base += (int64_t)gridDim.x * groups_per_block) {
        const int64_t seg = base + lg;
        const bool active = seg < total;
        float s;
        int z;
        if (tensor_mode) {
            s = scales[0];
            z = zps[0];
        } else {
            float mn, mx;
            seg_reduce<T, VEC>(x, g, seg, active, mn, mx);
            affine_params(mn, mx, bits, sym, &s, &z);
            if (active && sub == 0) {
                scales[seg] = s;
                zps[seg] = z;
            }
        }
        if (!active) continue;
        const float zf = (float)z;
        const int64_t r = seg / g.nseg;
        const int64_t c0 = (seg % g.nseg) * g.gs, c1 = min(g.cols, c0 + g.gs);
        const T* row = x + r * g.ld;
        for (int64_t c = c0 + (int64_t)sub * VEC; c < c1; c += (int64_t)g.L * VEC) {
            const int nv = (int)min((int64_t)VEC, c1 - c);
            float v[VEC];
            if (nv == VEC) {
                Vec<T, VEC> vv;
                vv.load(row + c);
#pragma unroll
                for (int i = 0; i < VEC; i++) v[i] = vv.v[i];
            } else {
                for (int i = 0; i < VEC; i++) v[i] = i < nv ? to_f<T>(row[c + i]) : 0.f;
            }
            int q[VEC];
            float o[VEC];
#pragma unroll
            for (int i = 0; i < VEC; i++) o[i] = fq_chain<T>(v[i], s, zf, qmin, qmax, &q[i]);
            if (codes) store_codes<VEC>(codes + r * crow, c, q, z, bits, nv);
            if (deq) {
                T* d = deq + r * ld_deq + c;
                if (nv == VEC && VEC * sizeof(T) == 16) {
                    uint4 pk;
                    T* h = reinterpret_cast<T*>(&pk);
#pragma unroll
                    for (int i = 0; i < VEC; i++) h[i] = from_f<T>(o[i]);
                    *reinterpret_cast<uint4*>(d) = pk;
                } else {
                    for (int i = 0; i < nv; i++) d[i] = from_f<T>(o[i]);
                }
            }
        }
    }
}

// The op-by-op FakeQuantizeFunction chain, out of line (the register RTN kernel calls it
// only for the rare elements its integer path does not cover).
struct FqOut {
    float value;
    int code;
};

template <typename T>
__device__ __noinline__ FqOut fq_chain_call(float x, float s, float zpf, float qmin, float qmax) {
    FqOut r;
    r.value = fq_chain<T>(x, s, zpf, qmin, qmax, &r.code);
    return r;
}

// RTN with every segment held in registers: each lane loads RV vectors of its segment
// (segment length = RV * L * VEC), so a thread keeps RV loads in flight and the per-segment
// parameter math is shared by RV * VEC elements.  Elements follow the op-by-op chain (the
// bf16 kernel below has the integer path).
template <typename T, int VEC>
__global__ void __launch_bounds__(NT) rtn_reg_kernel(const T* x, SegGeom g, FastDiv fd, int bits, int sym,
                                                     int tensor_mode, float* scales, int32_t* zps, uint8_t* codes,
                                                     T* deq, int64_t ld_deq) {
    const int L = g.L;
    const uint32_t gpb = NT / L;
    const uint32_t total = (uint32_t)(g.rows * g.nseg);
    const uint32_t lg = threadIdx.x / L;
    const int sub = lane_id() % L;
    const int64_t seglen = g.gs < g.cols ? g.gs : g.cols;
    float qmin, qmax;
    qrange(bits, sym, &qmin, &qmax);
    const int64_t crow = code_row_bytes(bits, g.cols);
    for (uint32_t base = blockIdx.x * gpb; base < total; base += gridDim.x * gpb) {
        const uint32_t seg = base + lg;
        const bool active = seg < total;
        const uint32_t sg = active ? seg : 0;
        const uint32_t r = fastdiv(sg, fd);
        const int64_t c0 = (int64_t)(sg - r * (uint32_t)g.nseg) * seglen;
        const T* row = x + (int64_t)r * g.ld + c0;
        Vec<T, VEC> v[RV];
        float mn[RV], mx[RV];
#pragma unroll
        for (int j = 0; j < RV; j++) {
            mn[j] = INFINITY;
            mx[j] = -INFINITY;
        }
        if (active) {
#pragma unroll
            for (int j = 0; j < RV; j++) v[j].load(row + (int64_t)(j * L + sub) * VEC);
#pragma unroll
            for (int j = 0; j < RV; j++)
#pragma unroll
                for (int i = 0; i < VEC; i++) {
                    mn[j] = fmin_nan(mn[j], v[j].v[i]);
                    mx[j] = fmax_nan(mx[j], v[j].v[i]);
                }
        }
        float smin = fmin_nan(fmin_nan(mn[0], mn[1]), fmin_nan(mn[2], mn[3]));
        float smax = fmax_nan(fmax_nan(mx[0], mx[1]), fmax_nan(mx[2], mx[3]));
        for (int off = L / 2; off > 0; off >>= 1) {
            smin = fmin_nan(smin, __shfl_xor_sync(0xffffffffu, smin, off));
            smax = fmax_nan(smax, __shfl_xor_sync(0xffffffffu, smax, off));
        }
        if (!active) continue;
        float s;
        int z;
        if (tensor_mode) {
            s = scales[0];
            z = zps[0];
        } else {
            affine_params(smin, smax, bits, sym, &s, &z);
            if (sub == 0) {
                scales[seg] = s;
                zps[seg] = z;
            }
        }
        const float zf = (float)z;
        uint8_t* crow_p = codes ? codes + (int64_t)r * crow : nullptr;
#pragma unroll
        for (int j = 0; j < RV; j++) {
            const int64_t c = c0 + (int64_t)(j * L + sub) * VEC;
            int q[VEC];
            float o[VEC];
#pragma unroll
            for (int i = 0; i < VEC; i++) o[i] = fq_chain<T>(v[j].v[i], s, zf, qmin, qmax, &q[i]);
            if (crow_p) store_codes<VEC>(crow_p, c, q, z, bits, VEC);
            if (deq) {
                T* d = deq + (int64_t)r * ld_deq + c;
                uint4 pk;
                T* h = reinterpret_cast<T*>(&pk);
#pragma unroll
                for (int i = 0; i < VEC; i++) h[i] = from_f<T>(o[i]);
                *reinterpret_cast<uint4*>(d) = pk;
            }
        }
    }
}

// bf16 RTN, register-resident like rtn_reg_kernel, with an integer path that is exact by
// construction.  With r = rcp_rn(s), f = x * r is within 3 units in the last place of
// fl(x / s), so bf16(f) == bf16(fl(x / s)) unless the low 16 bits of f lie within 4 of the
// bf16 rounding midpoint 0x8000 (those elements, and NaN / Inf, take the op-by-op chain).  If
// every quotient of the segment satisfies -256 <= x / s + zp <= 256 (checked from its min and
// max with a 2^-20 relative margin), every intermediate of FakeQuantizeFunction's chain (rint,
// + zp, clamp, - zp) is an integer of magnitude <= 256, which bf16 represents exactly, so
// the chain reduces to integer arithmetic on rint(bf16(x / s)) and the dequantised value to
// bf16((q - zp) * s).  The bf16 rounding of f is done on its bit pattern (round to nearest
// even at bit 16) and rint by adding 1.5 * 2^23 (ties to even, exact for |v| < 2^22), so the
// path needs no conversion instructions.
template <bool DEQ>
__global__ void __launch_bounds__(NT) rtn_bf16_kernel(const __nv_bfloat16* x, SegGeom g, FastDiv fd, int bits, int sym,
                                                      int tensor_mode, float* scales, int32_t* zps, uint8_t* codes,
                                                      __nv_bfloat16* deq, int64_t ld_deq) {
    constexpr int VEC = 8;
    const int L = g.L;
    const uint32_t gpb = NT / L;
    const uint32_t total = (uint32_t)(g.rows * g.nseg);
    const uint32_t lg = threadIdx.x / L;
    const int sub = lane_id() % L;
    const int64_t seglen = g.gs < g.cols ? g.gs : g.cols;
    float qmin, qmax;
    qrange(bits, sym, &qmin, &qmax);
    const int iqmin = (int)qmin, iqmax = (int)qmax;
    const int64_t crow = code_row_bytes(bits, g.cols);
    const __nv_bfloat162 pinf = __float2bfloat162_rn(INFINITY), ninf = __float2bfloat162_rn(-INFINITY);
    for (uint32_t base = blockIdx.x * gpb; base < total; base += gridDim.x * gpb) {
        const uint32_t seg = base + lg;
        const bool active = seg < total;
        const uint32_t sg = active ? seg : 0;
        const uint32_t r = fastdiv(sg, fd);
        const int64_t c0 = (int64_t)(sg - r * (uint32_t)g.nseg) * seglen;
        const __nv_bfloat16* row = x + (int64_t)r * g.ld + c0;
        uint4 w[RV];
        __nv_bfloat162 mn2[2] = {pinf, pinf}, mx2[2] = {ninf, ninf};
        if (active) {
#pragma unroll
            for (int j = 0; j < RV; j++) w[j] = *reinterpret_cast<const uint4*>(row + (int64_t)(j * L + sub) * VEC);
#pragma unroll
            for (int j = 0; j < RV; j++) {
                const uint32_t ww[4] = {w[j].x, w[j].y, w[j].z, w[j].w};
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const __nv_bfloat162 p = *reinterpret_cast<const __nv_bfloat162*>(&ww[k]);
                    mn2[k & 1] = __hmin2_nan(mn2[k & 1], p);
                    mx2[k & 1] = __hmax2_nan(mx2[k & 1], p);
                }
            }
        }
        const __nv_bfloat162 mnp = __hmin2_nan(mn2[0], mn2[1]), mxp = __hmax2_nan(mx2[0], mx2[1]);
        float smin = fmin_nan(__low2float(mnp), __high2float(mnp));
        float smax = fmax_nan(__low2float(mxp), __high2float(mxp));
        for (int off = L / 2; off > 0; off >>= 1) {
            smin = fmin_nan(smin, __shfl_xor_sync(0xffffffffu, smin, off));
            smax = fmax_nan(smax, __shfl_xor_sync(0xffffffffu, smax, off));
        }
        if (!active) continue;
        float s;
        int z;
        if (tensor_mode) {
            s = scales[0];
            z = zps[0];
        } else {
            affine_params(smin, smax, bits, sym, &s, &z);
            if (sub == 0) {
                scales[seg] = s;
                zps[seg] = z;
            }
        }
        const float zf = (float)z;
        const float rcp = __frcp_rn(s);
        const float k = 1.f + 0x1p-20f;
        const float hi = fmaxf(smax, 0.f) * rcp * k + zf;  // NaN / Inf fail the tests below
        const float lo = fminf(smin, 0.f) * rcp * k + zf;
        const bool fast = bits <= 8 && hi <= 256.f && lo >= -256.f;
        uint8_t* crow_p = codes ? codes + (int64_t)r * crow : nullptr;
#pragma unroll
        for (int j = 0; j < RV; j++) {
            const int64_t c = c0 + (int64_t)(j * L + sub) * VEC;
            const uint32_t ww[4] = {w[j].x, w[j].y, w[j].z, w[j].w};
            int q[VEC];
            float o[VEC];
            uint32_t slow = fast ? 0u : (1u << VEC) - 1u;
#pragma unroll
            for (int i = 0; i < VEC; i++) {
                const float xv = (i & 1) ? __uint_as_float(ww[i / 2] & 0xFFFF0000u) : __uint_as_float(ww[i / 2] << 16);
                const float f = __fmul_rn(xv, rcp);
                const uint32_t b = __float_as_uint(f);
                if (((b - 0x7FFCu) & 0xFFFFu) <= 8u || !(fabsf(f) <= 3.0e38f)) slow |= 1u << i;
                const float t1 = __uint_as_float((b + 0x7FFFu + ((b >> 16) & 1u)) & 0xFFFF0000u);
                int t = __float_as_int(__fadd_rn(t1, 12582912.f)) - 0x4B400000 + z;
                t = t < iqmin ? iqmin : (t > iqmax ? iqmax : t);
                q[i] = t;
                if (DEQ) o[i] = __fmul_rn(__int_as_float(0x4B400000 + (t - z)) - 12582912.f, s);
            }
            if (slow) {
#pragma unroll
                for (int i = 0; i < VEC; i++)
                    if ((slow >> i) & 1u) {
                        const float xv =
                            (i & 1) ? __uint_as_float(ww[i / 2] & 0xFFFF0000u) : __uint_as_float(ww[i / 2] << 16);
                        const FqOut e = fq_chain_call<__nv_bfloat16>(xv, s, zf, qmin, qmax);
                        o[i] = e.value;
                        q[i] = e.code;
                    }
            }
            if (crow_p) store_codes<VEC>(crow_p, c, q, z, bits, VEC);
            if (DEQ) {
                uint4 pk;
                __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(&pk);
#pragma unroll
                for (int i = 0; i < VEC; i++) h[i] = __float2bfloat16_rn(o[i]);
                *reinterpret_cast<uint4*>(deq + (int64_t)r * ld_deq + c) = pk;
            }
        }
    }
}

// bf16 RTN to packed nibbles (num_bits <= 4, no dequantised output): rtn_bf16_kernel's exact
// integer path with fewer instructions per element.  Each 32-bit word holds two bf16 columns,
// and the two are carried through the paired fp32 instructions of sm_100 (FMUL2 / FFMA2 /
// FADD2, each component rounded exactly as its scalar form).
//   * f = x * rcp(s); an element whose f lies within 4 units in the last place of a bf16
//     rounding midpoint takes the op-by-op chain (as in rtn_bf16_kernel).  The test takes the
//     low 16 bits of f, shifted up and offset, min-accumulated over a vector's eight elements
//     and compared once.
//   * bf16(f) by Veltkamp splitting, c = f * (2^16 + 1), bf16(f) = c - (c - f): rounding to
//     nearest on 8 significant bits on the floating-point pipe (T. J. Dekker, "A floating-point
//     technique for extending the available precision", 1971).  Each difference is one fused
//     multiply-add by -1 (the product is exact, so the one rounding is the subtraction's).  Its
//     tie-breaking may differ from round-to-even, but ties are exactly the midpoint elements
//     sent to the chain.
//   * rint by adding 1.5 * 2^23, then the clamp to [qmin - zp, qmax - zp] on that float (only in
//     warps whose segments can reach the grid's ends: a separate instantiation of the element
//     loop); the code nibble (q - zp) & 0xF is the low nibble of the sum's bit pattern.
//   * Nibbles are gathered with byte permutes, two 32-bit words per eight columns.
// A lane holds NRV 8-column vectors of one segment, so the segment's L = length / (8 NRV) lanes
// each repeat its parameter math (min / max, scale, zero-point, reciprocal) once per 8 NRV
// elements.  The launch bound follows the registers that holds: four 256-thread blocks per SM
// at NRV = 4 (64 registers; on 224 Llama-3-8B weights that ran 4 % faster than the unbounded
// 72-register build), three at 8, two at 16.  On those weights (g128, so L = 4, 2, 1 lanes a
// group) NRV = 4 ran at 2,426 GB/s, 8 at 1,890 and 16 at 1,144: with fewer lanes a group, one
// load instruction of a warp covers fewer whole 32-byte sectors and fewer warps are resident,
// which costs more than the repeated parameter math saves.
// Largest NRV the launch picks.
#ifndef NIB_RV_MAX
#define NIB_RV_MAX 4
#endif

// A vector holding an element near a bf16 rounding midpoint (or a segment off the fast path):
// those elements take the op-by-op chain, the others nib_vector's arithmetic with the clamp;
// packed as nib_vector packs.  One out-of-line copy, so the unrolled element loops that call it
// stay small.
__device__ __noinline__ uint32_t nib_chain8(uint4 w, float rcp, bool fast, float s, float zf, int z, float qmin,
                                            float qmax) {
    constexpr float MAGIC = 12582912.f;  // 1.5 * 2^23
    const float cmin = MAGIC + (qmin - zf), cmax = MAGIC + (qmax - zf);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    uint32_t u[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float xv = (i & 1) ? __uint_as_float(ww[i / 2] & 0xFFFF0000u) : __uint_as_float(ww[i / 2] << 16);
        const float f = __fmul_rn(xv, rcp);
        if (!fast || (__float_as_uint(f) * 65536u - 0x7FFC0000u) <= 0x80000u) {
            int code;
            fq_chain<__nv_bfloat16>(xv, s, zf, qmin, qmax, &code);
            u[i] = (uint32_t)((code - z) & 0xF);
        } else {
            const float c = __fmul_rn(f, 65537.f);
            const float b16 = __fsub_rn(c, __fsub_rn(c, f));
            u[i] = __float_as_uint(fminf(fmaxf(__fadd_rn(b16, MAGIC), cmin), cmax));
        }
    }
    const uint32_t ev = __byte_perm(__byte_perm(u[0], u[2], 0x0040), __byte_perm(u[4], u[6], 0x0040), 0x5410);
    const uint32_t od = __byte_perm(__byte_perm(u[1], u[3], 0x0040), __byte_perm(u[5], u[7], 0x0040), 0x5410);
    return ((ev << 4) & 0xF0F0F0F0u) | (od & 0x0F0F0F0Fu);
}

template <bool CLAMP>
__device__ __forceinline__ bool nib_vector(const uint4& w, float rcp, float cmin, float cmax, bool fast, uint8_t* dst) {
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
        // low 16 bits of f within 4 of 0x8000  <=>  (bits(f) - 0x7FFC) * 2^16 <= 8 * 2^16 (mod 2^32)
        near = min(near, __float_as_uint(f.x) * 65536u - 0x7FFC0000u);
        near = min(near, __float_as_uint(f.y) * 65536u - 0x7FFC0000u);
        const float2 c = __fmul2_rn(f, k2);
        const float2 b16 = __ffma2_rn(__ffma2_rn(f, neg1, c), neg1, c);  // c - (c - f)
        float2 rf = __fadd2_rn(b16, magic2);
        if constexpr (CLAMP) {
            rf.x = fminf(fmaxf(rf.x, cmin), cmax);
            rf.y = fminf(fmaxf(rf.y, cmin), cmax);
        }
        u[2 * k] = __float_as_uint(rf.x);
        u[2 * k + 1] = __float_as_uint(rf.y);
    }
    // byte b of the output holds columns 2b (high nibble) and 2b + 1 (low nibble)
    const uint32_t ev = __byte_perm(__byte_perm(u[0], u[2], 0x0040), __byte_perm(u[4], u[6], 0x0040), 0x5410);
    const uint32_t od = __byte_perm(__byte_perm(u[1], u[3], 0x0040), __byte_perm(u[5], u[7], 0x0040), 0x5410);
    *reinterpret_cast<uint32_t*>(dst) = ((ev << 4) & 0xF0F0F0F0u) | (od & 0x0F0F0F0Fu);
    // a vector near a midpoint (or off the fast path) is rewritten later by nib_chain8
    return !fast || near <= 0x80000u;
}

// Vectors that need the exact chain are queued per warp in shared memory and rewritten in
// batches, one vector a lane: in SIMT a branch to the chain costs the whole warp the chain's
// time whenever any lane takes it, and on 4-bit weights about 1 % of 8-column vectors (so most
// warp iterations of 128 vectors) hold an element near a bf16 rounding midpoint.
constexpr int NIB_QCAP = 32;  // queued vectors a warp
struct NibQueue {
    uint4 w[NIB_QCAP];
    float s[NIB_QCAP], rcp[NIB_QCAP];
    int z[NIB_QCAP];
    int64_t off[NIB_QCAP];  // byte offset of the vector's codes; bit 62 set: the segment is off the fast path
};

// Rewrites the queue's count vectors (lane i takes entry i) and empties it.  The fast-path
// stores of those vectors came from other lanes of this warp: __syncwarp orders them first.
__device__ __forceinline__ void nib_flush(NibQueue& q, int count, float qmin, float qmax, uint8_t* codes) {
    __syncwarp();
    const int lane = lane_id();
    if (lane < count) {
        const int64_t o = q.off[lane];
        const bool fast = (o & (int64_t(1) << 62)) == 0;
        const int z = q.z[lane];
        *reinterpret_cast<uint32_t*>(codes + (o & ~(int64_t(1) << 62))) =
            nib_chain8(q.w[lane], q.rcp[lane], fast, q.s[lane], (float)z, z, qmin, qmax);
    }
    __syncwarp();
}

template <int NRV>
__global__ void __launch_bounds__(NT, NRV <= 4 ? 4 : (NRV <= 8 ? 3 : 2))
    rtn_bf16_nib_kernel(const __nv_bfloat16* x, SegGeom g, FastDiv fd, int bits, int sym, int tensor_mode,
                        float* scales, int32_t* zps, uint8_t* codes) {
    constexpr int VEC = 8;
    const int L = g.L;
    const uint32_t gpb = NT / L;
    const uint32_t total = (uint32_t)(g.rows * g.nseg);
    const uint32_t lg = threadIdx.x / L;
    const int sub = lane_id() % L;
    const int64_t seglen = g.gs < g.cols ? g.gs : g.cols;
    float qmin, qmax;
    qrange(bits, sym, &qmin, &qmax);
    const int64_t crow = code_row_bytes(bits, g.cols);
    const __nv_bfloat162 pinf = __float2bfloat162_rn(INFINITY), ninf = __float2bfloat162_rn(-INFINITY);
    constexpr float MAGIC = 12582912.f;  // 1.5 * 2^23
    __shared__ NibQueue queues[NT / 32];
    NibQueue& q = queues[threadIdx.x / 32];
    int qn = 0;  // queued vectors of this warp (the same in every lane)
    for (uint32_t base = blockIdx.x * gpb; base < total; base += gridDim.x * gpb) {
        const uint32_t seg = base + lg;
        const bool active = seg < total;
        const uint32_t sg = active ? seg : 0;
        const uint32_t r = fastdiv(sg, fd);
        const int64_t c0 = (int64_t)(sg - r * (uint32_t)g.nseg) * seglen;
        const __nv_bfloat16* row = x + (int64_t)r * g.ld + c0;
        uint4 w[NRV];
        __nv_bfloat162 mn2[2] = {pinf, pinf}, mx2[2] = {ninf, ninf};
        if (active) {
#pragma unroll
            for (int j = 0; j < NRV; j++) w[j] = *reinterpret_cast<const uint4*>(row + (int64_t)(j * L + sub) * VEC);
#pragma unroll
            for (int j = 0; j < NRV; j++) {
                const uint32_t ww[4] = {w[j].x, w[j].y, w[j].z, w[j].w};
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const __nv_bfloat162 p = *reinterpret_cast<const __nv_bfloat162*>(&ww[k]);
                    mn2[k & 1] = __hmin2_nan(mn2[k & 1], p);
                    mx2[k & 1] = __hmax2_nan(mx2[k & 1], p);
                }
            }
        }
        const __nv_bfloat162 mnp = __hmin2_nan(mn2[0], mn2[1]), mxp = __hmax2_nan(mx2[0], mx2[1]);
        float smin = fmin_nan(__low2float(mnp), __high2float(mnp));
        float smax = fmax_nan(__low2float(mxp), __high2float(mxp));
        for (int off = L / 2; off > 0; off >>= 1) {
            smin = fmin_nan(smin, __shfl_xor_sync(0xffffffffu, smin, off));
            smax = fmax_nan(smax, __shfl_xor_sync(0xffffffffu, smax, off));
        }
        float s;
        int z;
        if (tensor_mode) {
            s = scales[0];
            z = zps[0];
        } else {
            affine_params(smin, smax, bits, sym, &s, &z);
            if (active && sub == 0) {
                scales[seg] = s;
                zps[seg] = z;
            }
        }
        const float zf = (float)z;
        const float rcp = __frcp_rn(s);
        const float k = 1.f + 0x1p-20f;
        const float hi = fmaxf(smax, 0.f) * rcp * k + zf;  // NaN / Inf fail the tests below
        const float lo = fminf(smin, 0.f) * rcp * k + zf;
        const bool fast = hi <= 256.f && lo >= -256.f;
        // The clamp can act only if some element's rounded quotient lies beyond the grid.  On
        // the fast path x -> rint(bf16(x * rcp)) is monotone (rounded products with rcp > 0,
        // round to nearest, rint), so the segment's extremes bound every element's code; an
        // extreme near a bf16 rounding midpoint (where the split's tie-breaking may differ)
        // counts as reaching the grid's end.  Elements near a midpoint take the exact chain,
        // which clamps by itself.
        bool clamp = true;
        if (fast) {
            const float fx = __fmul_rn(smax, rcp), fn = __fmul_rn(smin, rcp);
            const bool mid = (__float_as_uint(fx) * 65536u - 0x7FFC0000u) <= 0x80000u ||
                             (__float_as_uint(fn) * 65536u - 0x7FFC0000u) <= 0x80000u;
            const float cx = __fmul_rn(fx, 65537.f), cn = __fmul_rn(fn, 65537.f);
            const float qx = __fsub_rn(__fadd_rn(__fsub_rn(cx, __fsub_rn(cx, fx)), MAGIC), MAGIC);
            const float qn = __fsub_rn(__fadd_rn(__fsub_rn(cn, __fsub_rn(cn, fn)), MAGIC), MAGIC);
            clamp = mid || __fadd_rn(qx, zf) > qmax || __fadd_rn(qn, zf) < qmin;
        }
        const bool warp_clamp = __any_sync(0xffffffffu, active && clamp);
        const float cmin = MAGIC + (qmin - zf), cmax = MAGIC + (qmax - zf);
        const int64_t crow_off = (int64_t)r * crow;
        // every lane reaches the votes (inactive lanes store nothing and queue nothing)
        unsigned slow_bits = 0;  // bit j: vector j needs the chain
        if (active) {
#pragma unroll
            for (int j = 0; j < NRV; j++) {
                uint8_t* dst = codes + crow_off + (c0 + (int64_t)(j * L + sub) * VEC) / 2;
                const bool slow = warp_clamp ? nib_vector<true>(w[j], rcp, cmin, cmax, fast, dst)
                                             : nib_vector<false>(w[j], rcp, cmin, cmax, fast, dst);
                slow_bits |= slow ? (1u << j) : 0u;
            }
        }
        if (!__any_sync(0xffffffffu, slow_bits != 0)) continue;  // the common case: one vote
#pragma unroll
        for (int j = 0; j < NRV; j++) {
            const int64_t off = crow_off + (c0 + (int64_t)(j * L + sub) * VEC) / 2;
            const bool slow = (slow_bits >> j) & 1u;
            const unsigned mask = __ballot_sync(0xffffffffu, slow);
            if (mask) {
                const int n = __popc(mask);
                if (qn + n > NIB_QCAP) {
                    nib_flush(q, qn, qmin, qmax, codes);
                    qn = 0;
                }
                if (slow) {
                    const int pos = qn + __popc(mask & ((1u << lane_id()) - 1u));
                    q.w[pos] = w[j];
                    q.s[pos] = s;
                    q.rcp[pos] = rcp;
                    q.z[pos] = z;
                    q.off[pos] = off | (fast ? int64_t(0) : (int64_t(1) << 62));
                }
                qn += n;
            }
        }
    }
    if (qn) nib_flush(q, qn, qmin, qmax, codes);
}

template <typename T>
__global__ void fake_quant_flat_kernel(const T* x, int64_t n, float s, float zf, float qmin, float qmax, T* out,
                                       int32_t* codes) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int q;
        const float v = fq_chain<T>(to_f<T>(x[i]), s, zf, qmin, qmax, &q);
        if (out) out[i] = from_f<T>(v);
        if (codes) codes[i] = q;
    }
}

__global__ void int4_pack_kernel(const int32_t* q, int64_t n, int zp, uint8_t* out) {
    const int64_t nb = (n + 1) / 2;
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nb; b += (int64_t)gridDim.x * blockDim.x) {
        const int hi = (q[2 * b] - zp) & 0xF;
        const int lo = (2 * b + 1 < n) ? ((q[2 * b + 1] - zp) & 0xF) : 0;
        out[b] = (uint8_t)((hi << 4) | lo);
    }
}

__global__ void int4_unpack_kernel(const uint8_t* p, int64_t n, float s, int sym, float* out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint8_t b = p[i / 2];
        int nib = (i % 2 == 0) ? (b >> 4) : (b & 0xF);
        if (sym && (nib & 0x8)) nib -= 16;  // Int4PackedTensor.cs:132-136: sign-extend only if symmetric
        out[i] = __fmul_rn((float)nib, s);
    }
}

template <typename T>
__global__ void convert_kernel(const T* src, int64_t rows, int64_t cols, int64_t lds, float* dst, int64_t ldd) {
    const int64_t total = rows * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / cols, c = i % cols;
        dst[r * ldd + c] = to_f<T>(src[r * lds + c]);
    }
}

__global__ void symmetrize_kernel(const float* src, int64_t d, int64_t lds, float* dst, int64_t ldd) {
    const int64_t total = d * d;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / d, c = i % d;
        dst[r * ldd + c] = (r <= c) ? src[r * lds + c] : src[c * lds + r];
    }
}

int grid_for(llmc_ctx* ctx, int64_t items, int per_block) {
    int64_t b = (items + per_block - 1) / per_block;
    int64_t cap = (int64_t)ctx->sm_count * 16;
    if (b > cap) b = cap;
    if (b < 1) b = 1;
    return (int)b;
}

// Lanes per segment: the power of two <= 32 closest to (segment length / VEC) from below.
int lanes_for(int64_t seglen, int vec) {
    int64_t chunks = (seglen + vec - 1) / vec;
    int L = 1;
    while (L < 32 && L * 2 <= chunks) L *= 2;
    return L;
}

template <typename T>
bool vec_ok(const void* x, int64_t ld, int64_t gs, int64_t cols) {
    constexpr int V = 16 / sizeof(T);
    return ((uintptr_t)x % 16 == 0) && (ld % V == 0) && (gs % V == 0) && (cols % V == 0 || gs >= cols);
}

template <typename T>
llmc_status launch_minmax(llmc_ctx* ctx, const void* x, int64_t rows, int64_t cols, int64_t ld, int64_t gs,
                          float* mins, float* maxs, int fold) {
    constexpr int V = 16 / sizeof(T);
    SegGeom g{rows, cols, ld, gs, (cols + gs - 1) / gs, 1};
    const int64_t total = rows * g.nseg;
    if (vec_ok<T>(x, ld, gs, cols)) {
        const int64_t seglen = gs < cols ? gs : cols;
        g.L = lanes_for(seglen, V);
        const int rl = reg_lanes(seglen, V);
        if (cols % seglen == 0 && rl > 0 && total < (int64_t(1) << 31) && g.nseg < (int64_t(1) << 31)) {
            g.L = rl;
            seg_minmax_reg_kernel<T, V><<<grid_for(ctx, total, NT / g.L), NT, 0, ctx->stream>>>(
                reinterpret_cast<const T*>(x), g, make_fastdiv((uint32_t)g.nseg), mins, maxs, fold);
        } else {
            seg_minmax_kernel<T, V><<<grid_for(ctx, total, NT / g.L), NT, 0, ctx->stream>>>(
                reinterpret_cast<const T*>(x), g, mins, maxs, fold);
        }
    } else {
        g.L = lanes_for(gs < cols ? gs : cols, 1);
        seg_minmax_kernel<T, 1><<<grid_for(ctx, total, NT / g.L), NT, 0, ctx->stream>>>(
            reinterpret_cast<const T*>(x), g, mins, maxs, fold);
    }
    return check_launch(ctx, "seg_minmax");
}

llmc_status dispatch_minmax(llmc_ctx* ctx, const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, int64_t gs,
                            float* mins, float* maxs, int fold) {
    switch (dtype) {
        case LLMC_DTYPE_F32: return launch_minmax<float>(ctx, x, rows, cols, ld, gs, mins, maxs, fold);
        case LLMC_DTYPE_BF16: return launch_minmax<__nv_bfloat16>(ctx, x, rows, cols, ld, gs, mins, maxs, fold);
        case LLMC_DTYPE_F16: return launch_minmax<__half>(ctx, x, rows, cols, ld, gs, mins, maxs, fold);
    }
    return fail(LLMC_ERR_INVALID_ARG, "bad dtype %d", dtype);
}

template <typename T>
llmc_status launch_rtn(llmc_ctx* ctx, const void* x, int64_t m, int64_t n, int64_t ldw, int64_t gs, int bits, int sym,
                       int tensor_mode, float* scales, int32_t* zps, uint8_t* codes, void* deq) {
    constexpr int V = 16 / sizeof(T);
    SegGeom g{m, n, ldw, gs, (n + gs - 1) / gs, 1};
    const int64_t total = m * g.nseg;
    // Vector path also needs whole code bytes per lane (even column starts) and aligned output.
    const bool deq_ok = deq == nullptr || ((uintptr_t)deq % 16 == 0);
    const bool codes_ok = codes == nullptr || bits > 4 || (n % 2 == 0);
    // The vector paths store a vector's packed codes with one 4-byte store.
    const bool codes_al = codes == nullptr || (uintptr_t)codes % 4 == 0;
    const int64_t seglen = gs < n ? gs : n;
    const int64_t lanes = seglen / (RV * V);
    const bool reg_ok = seglen % (RV * V) == 0 && lanes >= 1 && lanes <= 32 && (lanes & (lanes - 1)) == 0 &&
                        n % seglen == 0 && total < (int64_t(1) << 31) && g.nseg < (int64_t(1) << 31);
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        if (vec_ok<T>(x, ldw, gs, n) && deq_ok && codes_ok && codes_al && reg_ok) {
            g.L = (int)lanes;
            const FastDiv fd = make_fastdiv((uint32_t)g.nseg);
            if (!deq && codes && bits <= 4) {
                // Vectors per lane: as many as a segment holds, up to NIB_RV_MAX, so fewer lanes
                // share (and repeat) a segment's parameter math.
                int nrv = NIB_RV_MAX;
                while (nrv > RV && seglen % ((int64_t)nrv * V) != 0) nrv /= 2;
                g.L = (int)(seglen / ((int64_t)nrv * V));
#define LLMC_NIB(NRV)                                                                                  \
    rtn_bf16_nib_kernel<NRV><<<grid_for(ctx, total, NT / g.L), NT, 0, ctx->stream>>>(                  \
        reinterpret_cast<const T*>(x), g, fd, bits, sym, tensor_mode, scales, zps, codes)
                if (nrv == 16) LLMC_NIB(16);
                else if (nrv == 8) LLMC_NIB(8);
                else LLMC_NIB(RV);
#undef LLMC_NIB
                return check_launch(ctx, "rtn_bf16_nib");
            }
            if (deq)
                rtn_bf16_kernel<true><<<grid_for(ctx, total, NT / g.L), NT, 0, ctx->stream>>>(
                    reinterpret_cast<const T*>(x), g, fd, bits, sym, tensor_mode, scales, zps, codes,
                    reinterpret_cast<T*>(deq), n);
            else
                rtn_bf16_kernel<false><<<grid_for(ctx, total, NT / g.L), NT, 0, ctx->stream>>>(
                    reinterpret_cast<const T*>(x), g, fd, bits, sym, tensor_mode, scales, zps, codes, nullptr, n);
            return check_launch(ctx, "rtn_bf16");
        }
    }
    if (vec_ok<T>(x, ldw, gs, n) && deq_ok && codes_ok && codes_al && reg_ok) {
        g.L = (int)lanes;
        rtn_reg_kernel<T, V><<<grid_for(ctx, total, NT / g.L), NT, 0, ctx->stream>>>(
            reinterpret_cast<const T*>(x), g, make_fastdiv((uint32_t)g.nseg), bits, sym, tensor_mode, scales, zps, codes,
            reinterpret_cast<T*>(deq), n);
    } else if (vec_ok<T>(x, ldw, gs, n) && deq_ok && codes_ok && codes_al) {
        g.L = lanes_for(gs < n ? gs : n, V);
        rtn_kernel<T, V><<<grid_for(ctx, total, NT / g.L), NT, 0, ctx->stream>>>(
            reinterpret_cast<const T*>(x), g, bits, sym, tensor_mode, scales, zps, codes, reinterpret_cast<T*>(deq), n);
    } else {
        g.L = lanes_for(gs < n ? gs : n, 1);
        // The scalar path packs nibbles one at a time (read-modify-write of a byte), so
        // one lane owns each segment's codes; segments start on even columns (odd group
        // sizes with packed codes are rejected by the caller), so no byte is shared.
        if (codes && bits <= 4) g.L = 1;
        rtn_kernel<T, 1><<<grid_for(ctx, total, NT / g.L), NT, 0, ctx->stream>>>(
            reinterpret_cast<const T*>(x), g, bits, sym, tensor_mode, scales, zps, codes, reinterpret_cast<T*>(deq), n);
    }
    return check_launch(ctx, "rtn");
}

}  // namespace

size_t minmax_scratch_floats(int strategy, int64_t rows) {
    return strategy == LLMC_STRATEGY_TENSOR ? (size_t)(2 * rows + 64) : 0;
}

llmc_status minmax(llmc_ctx* ctx, const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, int strategy,
                   int64_t group_size, float* mins, float* maxs, int accumulate, float* scratch) {
    if (strategy == LLMC_STRATEGY_TENSOR) {
        // Level 1: per-row min/max into scratch; level 2: min over the row minima and max
        // over the row maxima (each level-2 call also produces one unused value).  Both levels
        // propagate NaN, so the batch value is torch's x.min() / x.max(); the fold into the
        // running value is MinMaxObserver's.
        const int fold = accumulate == 0 ? FOLD_NONE : (accumulate == 1 ? FOLD_OBSERVER : FOLD_FRESH);
        float* rmin = scratch;
        float* rmax = scratch + rows;
        float* unused = scratch + 2 * rows + 32;
        LLMC_TRY(dispatch_minmax(ctx, x, dtype, rows, cols, ld, cols, rmin, rmax, FOLD_NONE));
        LLMC_TRY(dispatch_minmax(ctx, rmin, LLMC_DTYPE_F32, 1, rows, rows, rows, mins, unused, fold));
        LLMC_TRY(dispatch_minmax(ctx, rmax, LLMC_DTYPE_F32, 1, rows, rows, rows, unused, maxs, fold));
        return LLMC_OK;
    }
    const int64_t gs = strategy == LLMC_STRATEGY_GROUP ? group_size : cols;
    const int fold = accumulate == 0 ? FOLD_NONE : (accumulate == 1 ? FOLD_MINIMUM : FOLD_FRESH);
    return dispatch_minmax(ctx, x, dtype, rows, cols, ld, gs, mins, maxs, fold);
}

llmc_status affine(llmc_ctx* ctx, const float* mins, const float* maxs, int64_t count, int bits, int sym, float* scales,
                   int32_t* zps) {
    affine_kernel<<<grid_for(ctx, count, NT), NT, 0, ctx->stream>>>(mins, maxs, count, bits, sym, scales, zps);
    return check_launch(ctx, "affine");
}

llmc_status rtn(llmc_ctx* ctx, const void* W, int dtype, int64_t m, int64_t n, int64_t ldw, const llmc_qconfig* cfg,
                uint8_t* codes, float* scales, int32_t* zps, void* deq, float* scratch) {
    const int bits = cfg->num_bits, sym = cfg->symmetric;
    int tensor_mode = 0;
    int64_t gs = n;
    if (cfg->strategy == LLMC_STRATEGY_TENSOR) {
        // scratch: [2m + 64] for the two-level reduction, then 2 device scalars.
        float* mn = scratch + 2 * m + 64;
        float* mx = mn + 1;
        LLMC_TRY(minmax(ctx, W, dtype, m, n, ldw, LLMC_STRATEGY_TENSOR, n, mn, mx, 2, scratch));  // fresh observer
        LLMC_TRY(affine(ctx, mn, mx, 1, bits, sym, scales, zps));
        tensor_mode = 1;
    } else if (cfg->strategy == LLMC_STRATEGY_GROUP) {
        gs = cfg->group_size;
    }
    switch (dtype) {
        case LLMC_DTYPE_F32: return launch_rtn<float>(ctx, W, m, n, ldw, gs, bits, sym, tensor_mode, scales, zps, codes, deq);
        case LLMC_DTYPE_BF16: return launch_rtn<__nv_bfloat16>(ctx, W, m, n, ldw, gs, bits, sym, tensor_mode, scales, zps, codes, deq);
        case LLMC_DTYPE_F16: return launch_rtn<__half>(ctx, W, m, n, ldw, gs, bits, sym, tensor_mode, scales, zps, codes, deq);
    }
    return fail(LLMC_ERR_INVALID_ARG, "bad dtype");
}

llmc_status fake_quant_flat(llmc_ctx* ctx, const void* x, int dtype, int64_t count, float s, int zp, int bits, int sym,
                            void* out, int32_t* codes) {
    float qmin, qmax;
    qrange(bits, sym, &qmin, &qmax);
    const int g = grid_for(ctx, count, NT);
    switch (dtype) {
        case LLMC_DTYPE_F32:
            fake_quant_flat_kernel<float><<<g, NT, 0, ctx->stream>>>((const float*)x, count, s, (float)zp, qmin, qmax,
                                                                     (float*)out, codes);
            break;
        case LLMC_DTYPE_BF16:
            fake_quant_flat_kernel<__nv_bfloat16><<<g, NT, 0, ctx->stream>>>((const __nv_bfloat16*)x, count, s, (float)zp,
                                                                             qmin, qmax, (__nv_bfloat16*)out, codes);
            break;
        case LLMC_DTYPE_F16:
            fake_quant_flat_kernel<__half><<<g, NT, 0, ctx->stream>>>((const __half*)x, count, s, (float)zp, qmin, qmax,
                                                                      (__half*)out, codes);
            break;
        default: return fail(LLMC_ERR_INVALID_ARG, "bad dtype");
    }
    return check_launch(ctx, "fake_quant");
}

llmc_status int4_pack(llmc_ctx* ctx, const int32_t* q, int64_t n, int zp, uint8_t* out) {
    int4_pack_kernel<<<grid_for(ctx, (n + 1) / 2, NT), NT, 0, ctx->stream>>>(q, n, zp, out);
    return check_launch(ctx, "int4_pack");
}

llmc_status int4_unpack(llmc_ctx* ctx, const uint8_t* p, int64_t n, float s, int sym, float* out) {
    int4_unpack_kernel<<<grid_for(ctx, n, NT), NT, 0, ctx->stream>>>(p, n, s, sym, out);
    return check_launch(ctx, "int4_unpack");
}

llmc_status convert_to_f32(llmc_ctx* ctx, const void* src, int dtype, int64_t rows, int64_t cols, int64_t lds, float* dst,
                           int64_t ldd) {
    const int g = grid_for(ctx, rows * cols, NT);
    switch (dtype) {
        case LLMC_DTYPE_F32: convert_kernel<float><<<g, NT, 0, ctx->stream>>>((const float*)src, rows, cols, lds, dst, ldd); break;
        case LLMC_DTYPE_BF16:
            convert_kernel<__nv_bfloat16><<<g, NT, 0, ctx->stream>>>((const __nv_bfloat16*)src, rows, cols, lds, dst, ldd);
            break;
        case LLMC_DTYPE_F16: convert_kernel<__half><<<g, NT, 0, ctx->stream>>>((const __half*)src, rows, cols, lds, dst, ldd); break;
        default: return fail(LLMC_ERR_INVALID_ARG, "bad dtype");
    }
    return check_launch(ctx, "convert_to_f32");
}

llmc_status symmetrize_from_upper(llmc_ctx* ctx, const float* src, int64_t d, int64_t lds, float* dst, int64_t ldd) {
    symmetrize_kernel<<<grid_for(ctx, d * d, NT), NT, 0, ctx->stream>>>(src, d, lds, dst, ldd);
    return check_launch(ctx, "symmetrize");
}

}  // namespace llmc
