// fp32 SIMT GEMM with triangular K-range hints, lower/upper-block output masks and split-K.
//
// Serves the fp32 parts of the hot path: the Cholesky/inverse recursion
// (HessianInverseSolver.cs:62-90), the GPTQ lazy tail update W[:, i2:] -= Err1 U[i1:i2, i2:]
// (GptqBlockQuantizer.cs:173-180) and the fp32-input Hessian H += X^T X
// (HessianAccumulator.cs:59-64).  128x128x8 tiles, 256 threads, 8x8 outputs per thread,
// double-buffered shared memory.
#include "ops.h"

namespace llmc {
namespace {

constexpr int BM = 128, BN = 128, BK = 8, NT = 256;

template <typename T>
__device__ __forceinline__ float ldg_f(const T* p) { return to_f<T>(p[0]); }

// Loads 4 consecutive elements of a row (contiguous dim) starting at (r, c).
template <typename T>
__device__ __forceinline__ void load4(const T* base, int64_t ld, int64_t r, int64_t c, int64_t R, int64_t Cc,
                                      bool vec, float v[4]) {
    if (r < R && vec && c + 3 < Cc) {
        const T* p = base + r * ld + c;
        if constexpr (sizeof(T) == 4) {
            float4 q = *reinterpret_cast<const float4*>(p);
            v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
        } else {
            uint2 q = *reinterpret_cast<const uint2*>(p);
            const T* h = reinterpret_cast<const T*>(&q);
            v[0] = to_f<T>(h[0]); v[1] = to_f<T>(h[1]); v[2] = to_f<T>(h[2]); v[3] = to_f<T>(h[3]);
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] = (r < R && c + i < Cc) ? ldg_f(base + r * ld + c + i) : 0.f;
}

template <typename TA, typename TB>
__global__ void __launch_bounds__(NT) gemm_kernel(GemmArgs g, int a_vec, int b_vec, int64_t kchunk) {
    const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
    if (g.c_mode == 1 && m0 + BM - 1 < n0) return;  // tile entirely above the diagonal
    if (g.c_mode == 2 && m0 > n0 + BN - 1) return;  // tile entirely below the diagonal

    int64_t kb = 0, ke = g.K;
    if (g.a_tri == TRI_KLE) ke = min(ke, m0 + BM);
    if (g.a_tri == TRI_KGE) kb = max(kb, m0);
    if (g.b_tri == TRI_KLE) ke = min(ke, n0 + BN);
    if (g.b_tri == TRI_KGE) kb = max(kb, n0);
    kb = kb / BK * BK;
    if (g.split_k > 1) {
        int64_t s0 = kb + (int64_t)blockIdx.z * kchunk;
        int64_t s1 = min(ke, s0 + kchunk);
        kb = s0;
        ke = s1;
    }
    const bool has_work = ke > kb;

    __shared__ __align__(16) float As[2][BK][BM];
    __shared__ __align__(16) float Bs[2][BK][BN];

    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;
    const TA* A = reinterpret_cast<const TA*>(g.A);
    const TB* B = reinterpret_cast<const TB*>(g.B);

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.f;

    float ra[4], rb[4];
    // Thread -> load coordinates.
    // "row-contiguous along k" loads (A no-trans / B trans): r = tid/2, k = (tid%2)*4.
    // "row-contiguous along m/n" loads (A trans / B no-trans): k = tid/32, c = (tid%32)*4.
    auto load_tiles = [&](int64_t k0) {
        if (!g.a_trans) load4<TA>(A, g.lda, m0 + tid / 2, k0 + (tid % 2) * 4, g.M, ke, a_vec, ra);
        else load4<TA>(A, g.lda, k0 + tid / 32, m0 + (tid % 32) * 4, ke, g.M, a_vec, ra);
        if (g.b_trans) load4<TB>(B, g.ldb, n0 + tid / 2, k0 + (tid % 2) * 4, g.N, ke, b_vec, rb);
        else load4<TB>(B, g.ldb, k0 + tid / 32, n0 + (tid % 32) * 4, ke, g.N, b_vec, rb);
    };
    auto store_tiles = [&](int buf) {
        if (!g.a_trans) {
#pragma unroll
            for (int i = 0; i < 4; i++) As[buf][(tid % 2) * 4 + i][tid / 2] = ra[i];
        } else {
            *reinterpret_cast<float4*>(&As[buf][tid / 32][(tid % 32) * 4]) = make_float4(ra[0], ra[1], ra[2], ra[3]);
        }
        if (g.b_trans) {
#pragma unroll
            for (int i = 0; i < 4; i++) Bs[buf][(tid % 2) * 4 + i][tid / 2] = rb[i];
        } else {
            *reinterpret_cast<float4*>(&Bs[buf][tid / 32][(tid % 32) * 4]) = make_float4(rb[0], rb[1], rb[2], rb[3]);
        }
    };

    if (has_work) {
        load_tiles(kb);
        store_tiles(0);
        __syncthreads();
        int buf = 0;
        for (int64_t k0 = kb; k0 < ke; k0 += BK) {
            const bool more = k0 + BK < ke;
            if (more) load_tiles(k0 + BK);
#pragma unroll
            for (int k = 0; k < BK; k++) {
                float a[8], b[8];
                float4 a0 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
                float4 a1 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4 + 64]);
                float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4]);
                float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4 + 64]);
                a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
                a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
                b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
                b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
                for (int i = 0; i < 8; i++)
#pragma unroll
                    for (int j = 0; j < 8; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
            }
            if (more) {
                store_tiles(buf ^ 1);
                __syncthreads();
                buf ^= 1;
            }
        }
    }

    // Epilogue.
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int64_t r = m0 + ty * 4 + (i % 4) + (i / 4) * 64;
        if (r >= g.M) continue;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int64_t c = n0 + tx * 4 + (j % 4) + (j / 4) * 64;
            if (c >= g.N) continue;
            if (g.c_mode == 1 && r < c) continue;
            float* p = g.C + r * g.ldc + c;
            const float v = g.alpha * acc[i][j];
            if (g.split_k > 1) {
                if (has_work) atomicAdd(p, v);
            } else {
                *p = (g.beta == 0.f) ? v : fmaf(g.beta, *p, v);
            }
        }
    }
}

// ---- small GEMMs: 32 x 32 tiles, K split over the CTA's 8 warps ----------------------------
// The lower levels of the Cholesky recursion and the GPTQ near-block updates of short weights
// produce GEMMs of a few 128 x 128 tiles, which the kernel above runs on a handful of SMs.
// Here every 32 x 32 output tile is its own CTA; the CTA stages KC-deep slabs of A and B in
// shared memory, each warp accumulates a 32 x 32 partial over its KC/8 slice of the slab
// (lane: 4 rows x 8 columns), and the 8 partials are summed through shared memory.
constexpr int ST = 32, SKC = 128, SNT = 256;

template <typename T>
__device__ __forceinline__ float ld_el(const T* base, int64_t ld, int64_t r, int64_t c, int64_t R, int64_t Cc) {
    return (r < R && c < Cc) ? to_f<T>(base[r * ld + c]) : 0.f;
}

template <typename T>
__global__ void __launch_bounds__(SNT) gemm_small_kernel(GemmArgs g) {
    const int64_t m0 = (int64_t)blockIdx.y * ST, n0 = (int64_t)blockIdx.x * ST;
    if (g.c_mode == 1 && m0 + ST - 1 < n0) return;
    if (g.c_mode == 2 && m0 > n0 + ST - 1) return;
    int64_t kb = 0, ke = g.K;
    if (g.a_tri == TRI_KLE) ke = min(ke, m0 + ST);
    if (g.a_tri == TRI_KGE) kb = max(kb, m0);
    if (g.b_tri == TRI_KLE) ke = min(ke, n0 + ST);
    if (g.b_tri == TRI_KGE) kb = max(kb, n0);

    __shared__ __align__(16) float As[SKC][ST];  // As[k][m]
    __shared__ __align__(16) float Bs[SKC][ST];  // Bs[k][n]
    const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
    const int rg = lane / 4, cg = lane % 4;  // rows rg*4 .. +3, columns cg*8 .. +7
    const T* A = reinterpret_cast<const T*>(g.A);
    const T* B = reinterpret_cast<const T*>(g.B);
    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.f;

    for (int64_t k0 = kb; k0 < ke; k0 += SKC) {
        const int64_t kc = min((int64_t)SKC, ke - k0);
        // stage A[m0 .. +32, k0 .. +kc] as As[k][m] and B[k0 .. +kc, n0 .. +32] as Bs[k][n]
        for (int e = tid; e < SKC * ST; e += SNT) {
            int k, mm;
            if (!g.a_trans) { mm = e / SKC; k = e % SKC; }  // contiguous along k
            else { k = e / ST; mm = e % ST; }              // contiguous along m
            float v = 0.f;
            if (k < kc) v = g.a_trans ? ld_el(A, g.lda, k0 + k, m0 + mm, ke, g.M) : ld_el(A, g.lda, m0 + mm, k0 + k, g.M, ke);
            As[k][mm] = v;
            int nn;
            if (g.b_trans) { nn = e / SKC; k = e % SKC; }  // B stored [n][k]
            else { k = e / ST; nn = e % ST; }
            v = 0.f;
            if (k < kc) v = g.b_trans ? ld_el(B, g.ldb, n0 + nn, k0 + k, g.N, ke) : ld_el(B, g.ldb, k0 + k, n0 + nn, ke, g.N);
            Bs[k][nn] = v;
        }
        __syncthreads();
        const int ks = warp * (SKC / 8);
#pragma unroll 4
        for (int k = ks; k < ks + SKC / 8; k++) {
            const float4 a = *reinterpret_cast<const float4*>(&As[k][rg * 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[k][cg * 8]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[k][cg * 8 + 4]);
            const float av[4] = {a.x, a.y, a.z, a.w};
            const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
    // Sum the 8 warps' partials: red[w][r][c] reuses As/Bs (8 x 32 x 32 floats = 32 KB).
    float* red = &As[0][0];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) red[(warp * ST + rg * 4 + i) * ST + cg * 8 + j] = acc[i][j];
    __syncthreads();
    for (int e = tid; e < ST * ST; e += SNT) {
        const int r = e / ST, c = e % ST;
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) s += red[(w * ST + r) * ST + c];
        const int64_t gr = m0 + r, gc = n0 + c;
        if (gr >= g.M || gc >= g.N) continue;
        if (g.c_mode == 1 && gr < gc) continue;
        if (g.c_mode == 2 && gr > gc) continue;
        float* p = g.C + gr * g.ldc + gc;
        const float v = g.alpha * s;
        *p = (g.beta == 0.f) ? v : fmaf(g.beta, *p, v);
    }
}

template <typename TA, typename TB>
llmc_status launch(llmc_ctx* ctx, const GemmArgs& g) {
    auto aligned = [](const void* p, int64_t ld, int es) {
        return ((uintptr_t)p % (4 * es) == 0) && (ld % 4 == 0);
    };
    const int a_vec = aligned(g.A, g.lda, sizeof(TA));
    const int b_vec = aligned(g.B, g.ldb, sizeof(TB));
    int64_t kb_span = g.K;
    int split = g.split_k < 1 ? 1 : g.split_k;
    int64_t kchunk = (kb_span + split - 1) / split;
    kchunk = (kchunk + BK - 1) / BK * BK;
    if (split > 1) split = (int)((kb_span + kchunk - 1) / kchunk);
    GemmArgs a = g;
    a.split_k = split;
    dim3 grid((unsigned)((g.N + BN - 1) / BN), (unsigned)((g.M + BM - 1) / BM), (unsigned)split);
    if (grid.y > 65535) return fail(LLMC_ERR_UNSUPPORTED, "gemm: M=%lld too large", (long long)g.M);
    gemm_kernel<TA, TB><<<grid, NT, 0, ctx->stream>>>(a, a_vec, b_vec, kchunk);
    return check_launch(ctx, "gemm_f32");
}

}  // namespace

llmc_status gemm_f32(llmc_ctx* ctx, const GemmArgs& g) {
    if (g.M <= 0 || g.N <= 0) return LLMC_OK;
    if (g.split_k > 1 && g.beta != 1.f) return fail(LLMC_ERR_INTERNAL, "gemm: split-K needs beta == 1");
    if (g.K <= 0) {
        if (g.beta == 1.f) return LLMC_OK;
        // C = beta * C: run with an empty K range (all accumulators zero).
    }
    if (g.a_dtype != g.b_dtype) return fail(LLMC_ERR_INTERNAL, "gemm: mixed operand dtypes");
    // Large fp32 products go to the tensor cores (3 x TF32); small ones stay on the SIMT kernel.
    if (g.a_dtype == LLMC_DTYPE_F32 && g.K > 0 && (double)g.M * (double)g.N * (double)g.K >= (double)(1 << 26)) {
        llmc_status st = gemm_tc(ctx, g);
        if (st != LLMC_ERR_UNSUPPORTED) return st;
    }
    // Few 128 x 128 tiles and no split-K: 32 x 32 tiles spread the product over more SMs.
    const int64_t tiles128 = ((g.M + BM - 1) / BM) * ((g.N + BN - 1) / BN);
    if (g.a_dtype == LLMC_DTYPE_F32 && g.split_k <= 1 && tiles128 < ctx->sm_count && g.M <= 65535LL * ST) {
        dim3 grid((unsigned)((g.N + ST - 1) / ST), (unsigned)((g.M + ST - 1) / ST));
        gemm_small_kernel<float><<<grid, SNT, 0, ctx->stream>>>(g);
        return check_launch(ctx, "gemm_small");
    }
    switch (g.a_dtype) {
        case LLMC_DTYPE_F32: return launch<float, float>(ctx, g);
        case LLMC_DTYPE_BF16: return launch<__nv_bfloat16, __nv_bfloat16>(ctx, g);
        case LLMC_DTYPE_F16: return launch<__half, __half>(ctx, g);
    }
    return fail(LLMC_ERR_INVALID_ARG, "gemm: bad dtype");
}

}  // namespace llmc
