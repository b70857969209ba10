// Damped Cholesky inverse and the GPTQ upper factor.
//
// Reference: HessianInverseSolver.Compute (src/LLMCompressorSharp.TorchExtensions/Hessian/
// HessianInverseSolver.cs:44-92) and the factor U = chol(Hinv)^T of GptqBlockQuantizer.cs:105-118.
//
// Recursive blocked factorisation that produces L and L^-1 together:
//   chol_inv([[A11, .], [A21, A22]]):
//     (L11, L11^-1) = chol_inv(A11)
//     L21   = A21 L11^-T                       (GEMM, triangular operand)
//     A22  -= L21 L21^T                        (GEMM, lower output only)
//     (L22, L22^-1) = chol_inv(A22)
//     (L^-1)21 = -L22^-1 (L21 L11^-1)          (two GEMMs)
// with a one-CTA shared-memory kernel for blocks of <= 128.  All O(d^3) work is GEMM.
//
// U directly: with P the index-reversal permutation and L' = chol(P H' P), the matrix
// U = P L'^-1 P is upper triangular and U^T U = H'^-1, i.e. U is exactly the upper
// Cholesky factor of H'^-1 that GptqBlockQuantizer computes through Hinv.  One
// factorisation + inverse replaces the reference's four O(d^3) steps.
#include "ops.h"

namespace llmc {
namespace {

constexpr int NB = 128;  // diagonal block size of the recursion's base case

__global__ void diag_lambda_kernel(const float* H, int64_t d, int64_t ldh, float damp, float* lam) {
    // mean(diag H) read back as a float, times the damping fraction as C# float math
    // (HessianInverseSolver.cs:64-65).  The sum is taken in double, then rounded.
    __shared__ double part[256];
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < d; i += blockDim.x) s += (double)H[i * ldh + i];
    part[threadIdx.x] = s;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
        if ((int)threadIdx.x < w) part[threadIdx.x] += part[threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const float mean = (float)(part[0] / (double)d);
        lam[0] = damp > 0.f ? __fmul_rn(damp, mean) : 0.f;
    }
}

// A[i][j] = H'[p(i)][p(j)] for i >= j, 0 above the diagonal; p flips when `flip`.
__global__ void prep_kernel(const float* H, int64_t d, int64_t ldh, int upper_only, int flip, const float* lam,
                            float* A, int64_t lda) {
    const int64_t total = d * d;
    const float l = lam[0];
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / d, j = t % d;
        float v = 0.f;
        if (i >= j) {
            int64_t pi = flip ? d - 1 - i : i, pj = flip ? d - 1 - j : j;
            if (upper_only && pi > pj) {
                int64_t tmp = pi;
                pi = pj;
                pj = tmp;
            }
            v = H[pi * ldh + pj];
            if (i == j) v = __fadd_rn(v, l);
        }
        A[i * lda + j] = v;
    }
}

// Cholesky + triangular inverse of one n x n (n <= NB) diagonal block in shared memory,
// blocked in 32-column panels.  A's lower triangle is read; L (zeros above) goes back to A
// and L^-1 to I.  A pivot that is not > 0 (or NaN) raises flags[0] and the block continues
// with a unit pivot, so the kernel always terminates; the host reports the failure.
//
// Per panel p (columns c0 = 32p .. c0+31):
//   1. warp 0 factors the 32 x 32 diagonal block in registers (lane i holds row i; column k
//      of the factor is broadcast with shuffles) and then inverts it (lane j builds column j
//      of L11^-1 by forward substitution against the shared-memory copy of L11);
//   2. all warps form the panel below, L21 = A21 L11^-T, from the explicit inverse;
//   3. all warps apply the trailing update A22 -= L21 L21^T (lower triangle).
// The off-diagonal blocks of L^-1 follow block row by block row:
//   X_ij = -X_ii (sum_{k=j..i-1} L_ik X_kj).
// Rows and columns in [n, round_up(n, 32)) are identity padding and are never stored.
constexpr int BASE_THREADS = 512;  // 16 warps; 128 registers per thread for the register-resident factor
constexpr int BW = BASE_THREADS / 32;
constexpr int BLD = NB + 1;
constexpr unsigned FULL = 0xffffffffu;

size_t base_smem_bytes() { return (size_t)2 * NB * BLD * sizeof(float); }

// Unblocked Cholesky of the 32 x 32 lower block of sL at (c0, c0) by one warp: lane i keeps
// row i in registers; step K broadcasts the pivot and column K of the factor with shuffles.
template <int K>
__device__ __forceinline__ void chol32_step(float (&r)[32], int lane, int& bad) {
    float piv = __shfl_sync(FULL, r[K], K);
    if (!(piv > 0.f)) {
        bad = 1;
        piv = 1.f;
    }
    // 1 / sqrt(piv) from the SFU (within 2 ulp) and sqrt(piv) as piv times it: this step is on
    // the block's critical path, and the correctly rounded square root and reciprocal each cost
    // several times the latency; the factor's error bars (1e-4 relative on U) are far wider.
    const float inv_s = rsqrtf(piv);
    const float s = __fmul_rn(piv, inv_s);
    r[K] = (lane == K) ? s : ((lane > K) ? __fmul_rn(r[K], inv_s) : 0.f);
#pragma unroll
    for (int j = K + 1; j < 32; j++) {
        const float ljk = __shfl_sync(FULL, r[K], j);
        r[j] = (lane >= j) ? fmaf(-r[K], ljk, r[j]) : r[j];
    }
    if constexpr (K + 1 < 32) chol32_step<K + 1>(r, lane, bad);
}

__device__ __forceinline__ void factor_diag32(float* sL, int c0, int lane, int* flags) {
    float r[32];
#pragma unroll
    for (int j = 0; j < 32; j++) r[j] = (j <= lane) ? sL[(c0 + lane) * BLD + c0 + j] : 0.f;
    int bad = 0;
    chol32_step<0>(r, lane, bad);
    if (bad && lane == 0) atomicOr(flags, 1);
#pragma unroll
    for (int j = 0; j < 32; j++) sL[(c0 + lane) * BLD + c0 + j] = (j <= lane) ? r[j] : 0.f;
}

// Column `lane` of the inverse of the 32 x 32 lower block of sL at (c0, c0), into sX.
__device__ __forceinline__ void invert_diag32(const float* sL, float* sX, int c0, int lane) {
    float x[32];
#pragma unroll
    for (int i = 0; i < 32; i++) {
        const float* Li = sL + (c0 + i) * BLD + c0;
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < i; k++) acc = fmaf(Li[k], x[k], acc);  // x[k] = 0 for k < lane
        const float rii = __frcp_rn(Li[i]);  // independent of acc: off the substitution chain
        x[i] = (i < lane) ? 0.f : ((i == lane) ? rii : __fmul_rn(-acc, rii));
    }
#pragma unroll
    for (int i = 0; i < 32; i++) sX[(c0 + i) * BLD + c0 + lane] = x[i];
}

__global__ void __launch_bounds__(BASE_THREADS) chol_inv_base_kernel(float* A, float* I, int64_t ld, int n, int* flags) {
    extern __shared__ float sm[];
    float* sL = sm;             // [NB][BLD]
    float* sX = sm + NB * BLD;  // [NB][BLD]
    const int tid = threadIdx.x;
    const int lane = tid % 32, warp = tid / 32;
    const int np = (n + 31) / 32 * 32;
    const int P = np / 32;
    for (int i = warp; i < np; i += BW)
        for (int j = lane; j < np; j += 32) {
            float v;
            if (i < n && j < n) v = (j <= i) ? A[i * ld + j] : 0.f;
            else v = (i == j) ? 1.f : 0.f;
            sL[i * BLD + j] = v;
            sX[i * BLD + j] = 0.f;
        }
    __syncthreads();

    constexpr int RPW = (NB - 32) / BW;  // panel rows per warp (6)
    for (int p = 0; p < P; p++) {
        const int c0 = 32 * p;
        if (warp == 0) {
            factor_diag32(sL, c0, lane, flags);
            __syncwarp();
            invert_diag32(sL, sX, c0, lane);
        }
        __syncthreads();
        const int r0 = c0 + 32;
        if (r0 >= np) break;
        // Panel: L21[r][j] = sum_{k <= j} A21[r][k] X11[j][k]; warp -> rows, lane -> column.
        float pv[RPW];
        const float* Xj = sX + (c0 + lane) * BLD + c0;
#pragma unroll
        for (int a = 0; a < RPW; a++) {
            const int r = r0 + warp + BW * a;
            float acc = 0.f;
            if (r < np) {
                const float* Ar = sL + r * BLD + c0;
#pragma unroll
                for (int k = 0; k < 32; k++) acc = fmaf(Ar[k], Xj[k], acc);  // Xj[k] = 0 for k > lane
            }
            pv[a] = acc;
        }
        __syncthreads();
#pragma unroll
        for (int a = 0; a < RPW; a++) {
            const int r = r0 + warp + BW * a;
            if (r < np) sL[r * BLD + c0 + lane] = pv[a];
        }
        __syncthreads();
        // Trailing update of the lower triangle: A22[r][s] -= sum_k L21[r][k] L21[s][k].
#pragma unroll
        for (int a = 0; a < RPW; a++) {
            const int r = r0 + warp + BW * a;
            if (r >= np) continue;
            const float* Lr = sL + r * BLD + c0;
#pragma unroll
            for (int b = 0; b < 3; b++) {
                const int s2 = r0 + lane + 32 * b;
                if (s2 > r) continue;
                const float* Ls = sL + s2 * BLD + c0;
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < 32; k++) acc = fmaf(Lr[k], Ls[k], acc);
                sL[r * BLD + s2] = __fsub_rn(sL[r * BLD + s2], acc);
            }
        }
        __syncthreads();
    }

    // Off-diagonal blocks of L^-1, block row by block row.
    for (int bi = 1; bi < P; bi++) {
        const int i0 = 32 * bi;
        // T_j[a][b] = sum_{m = 32 j .. i0-1} L[i0+a][m] X[m][32 j + b], for every block j < bi.
        float tv[2][3];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const float* La = sL + (i0 + warp + BW * h) * BLD;
#pragma unroll
            for (int bj = 0; bj < 3; bj++) {
                float acc = 0.f;
                if (bj < bi) {
                    const int col = 32 * bj + lane;
                    for (int m = 32 * bj; m < i0; m++) acc = fmaf(La[m], sX[m * BLD + col], acc);
                }
                tv[h][bj] = acc;
            }
        }
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int bj = 0; bj < 3; bj++)
                if (bj < bi) sX[(i0 + warp + BW * h) * BLD + 32 * bj + lane] = tv[h][bj];
        __syncthreads();
        // X_ij[a][b] = -sum_{c <= a} X_ii[a][c] T_j[c][b]
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int ar = warp + BW * h;
            const float* Xa = sX + (i0 + ar) * BLD + i0;
#pragma unroll
            for (int bj = 0; bj < 3; bj++) {
                float acc = 0.f;
                if (bj < bi) {
                    const int col = 32 * bj + lane;
                    for (int c = 0; c <= ar; c++) acc = fmaf(Xa[c], sX[(i0 + c) * BLD + col], acc);
                }
                tv[h][bj] = -acc;
            }
        }
        __syncthreads();
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int bj = 0; bj < 3; bj++)
                if (bj < bi) sX[(i0 + warp + BW * h) * BLD + 32 * bj + lane] = tv[h][bj];
        __syncthreads();
    }

    for (int i = warp; i < n; i += BW)
        for (int j = lane; j < n; j += 32) {
            A[i * ld + j] = sL[i * BLD + j];
            I[i * ld + j] = sX[i * BLD + j];
        }
}

// out[i][j] = src[d-1-i][d-1-j] (flip) or src[j][i] (transpose); src lower -> out upper.
__global__ void remap_kernel(const float* src, int64_t d, int64_t lds, int mode, float* out, int64_t ldo) {
    const int64_t total = d * d;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / d, j = t % d;
        float v;
        if (mode == 0) v = src[(d - 1 - i) * lds + (d - 1 - j)];
        else v = (j >= i) ? src[j * lds + i] : 0.f;
        out[i * ldo + j] = v;
    }
}

__global__ void copy2d_kernel(const float* src, int64_t rows, int64_t cols, int64_t lds, float* dst, int64_t ldd) {
    const int64_t total = rows * cols;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / cols, j = t % cols;
        dst[i * ldd + j] = src[i * lds + j];
    }
}

// flags[1] = 1 when any element of the (symmetric) input is nonzero.  With only_if_failed
// the kernel does nothing unless flags[0] (a non-positive pivot) is set.
__global__ void nonzero_kernel(const float* H, int64_t d, int64_t ldh, int upper_only, int* flags, int only_if_failed) {
    if (only_if_failed && *(volatile int*)flags == 0) return;
    const int64_t total = d * d;
    int any = 0;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / d, j = t % d;
        if ((!upper_only || i <= j) && H[i * ldh + j] != 0.f) any = 1;
    }
    if (__syncthreads_or(any) && threadIdx.x == 0) atomicOr(flags + 1, 1);
}

// Deferred end of llmc_chol_inverse(want_upper = 1): the flipped factor (as remap_kernel mode 0)
// when the factorisation succeeded; otherwise zeros (pinv of the all-zero matrix, the
// reference's fallback, HessianInverseSolver.cs:85-91), and for a nonzero matrix also the
// deferred NOT_PD word flags[3], reported by the next llmc_sync.
__global__ void finish_upper_kernel(const float* src, int64_t d, int64_t lds, float* out, int64_t ldo, int* flags) {
    const int failed = *(volatile int*)flags;
    if (failed && blockIdx.x == 0 && threadIdx.x == 0 && *(volatile int*)(flags + 1)) atomicOr(flags + 3, 1);
    const int64_t total = d * d;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / d, j = t % d;
        out[i * ldo + j] = failed ? 0.f : src[(d - 1 - i) * lds + (d - 1 - j)];
    }
}

// Deferred end of llmc_upper_factor: U = L^T (remap_kernel mode 1) when chol(Hinv) succeeded,
// else Hinv itself (GptqBlockQuantizer.cs:112-118).
__global__ void finish_factor_kernel(const float* L, const float* hinv, int64_t d, int64_t ldl, int64_t ldh, float* out,
                                     int64_t ldo, const int* flags) {
    const int failed = *(volatile const int*)flags;
    const int64_t total = d * d;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / d, j = t % d;
        out[i * ldo + j] = failed ? hinv[i * ldh + j] : ((j >= i) ? L[j * ldl + i] : 0.f);
    }
}

int grid_for(llmc_ctx* ctx, int64_t items) {
    int64_t b = (items + 255) / 256;
    int64_t cap = (int64_t)ctx->sm_count * 8;
    return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

struct CholWs {
    float* A;
    float* I;
    float* tmp;  // n2 x n1 scratch when L must be kept
    int64_t ld;
};

llmc_status rec(llmc_ctx* ctx, const CholWs& w, int64_t off, int64_t n, int keep_L) {
    float* A = w.A + off * w.ld + off;
    float* I = w.I + off * w.ld + off;
    if (n <= NB) {
        static bool attr = false;
        if (!attr) {
            LLMC_CUDA_TRY(cudaFuncSetAttribute(chol_inv_base_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)base_smem_bytes()));
            attr = true;
        }
        chol_inv_base_kernel<<<1, BASE_THREADS, base_smem_bytes(), ctx->stream>>>(A, I, w.ld, (int)n, ctx->dflags);
        return check_launch(ctx, "chol_inv_base");
    }
    int64_t n1 = ((n / 2 + NB - 1) / NB) * NB;
    if (n1 >= n) n1 = n - NB;
    const int64_t n2 = n - n1;
    float* A21 = A + n1 * w.ld;
    float* I11 = I;
    float* I21 = I + n1 * w.ld;
    float* I22 = I21 + n1;

    LLMC_TRY(rec(ctx, w, off, n1, keep_L));
    GemmArgs g{};
    // L21 = A21 L11^-T  -> held in I21 (free until the end of this frame)
    g = GemmArgs{n2, n1, n1, A21, w.ld, 0, LLMC_DTYPE_F32, I11, w.ld, 1, LLMC_DTYPE_F32, I21, w.ld, 1.f, 0.f};
    g.b_tri = TRI_KLE;
    LLMC_TRY(gemm_f32(ctx, g));
    // A22 -= L21 L21^T (lower triangle)
    g = GemmArgs{n2, n2, n1, I21, w.ld, 0, LLMC_DTYPE_F32, I21, w.ld, 1, LLMC_DTYPE_F32, A21 + n1, w.ld, -1.f, 1.f};
    g.c_mode = 1;
    LLMC_TRY(gemm_f32(ctx, g));
    float* T = A21;  // A21 is dead once L21 lives in I21 ...
    if (keep_L) {    // ... unless the caller wants L back, then A21 <- L21 and T is scratch.
        copy2d_kernel<<<grid_for(ctx, n2 * n1), 256, 0, ctx->stream>>>(I21, n2, n1, w.ld, A21, w.ld);
        LLMC_TRY(check_launch(ctx, "copy2d"));
        T = w.tmp;
    }
    LLMC_TRY(rec(ctx, w, off + n1, n2, keep_L));
    const int64_t ldt = keep_L ? n1 : w.ld;
    // T = L21 L11^-1
    g = GemmArgs{n2, n1, n1, I21, w.ld, 0, LLMC_DTYPE_F32, I11, w.ld, 0, LLMC_DTYPE_F32, T, ldt, 1.f, 0.f};
    g.b_tri = TRI_KGE;
    LLMC_TRY(gemm_f32(ctx, g));
    // (L^-1)21 = -L22^-1 T
    g = GemmArgs{n2, n1, n2, I22, w.ld, 0, LLMC_DTYPE_F32, T, ldt, 0, LLMC_DTYPE_F32, I21, w.ld, -1.f, 0.f};
    g.a_tri = TRI_KLE;
    return gemm_f32(ctx, g);
}

llmc_status read_flags(llmc_ctx* ctx, int* f0, int* f1) {
    LLMC_TRY(device_error_check(ctx));
    LLMC_CUDA_TRY(cudaMemcpyAsync(ctx->hflags, ctx->dflags, 2 * sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
    LLMC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    *f0 = ctx->hflags[0];
    *f1 = ctx->hflags[1];
    return LLMC_OK;
}

// Factor the prepared lower matrix in w.A.  Unless the context defers errors, wait for it and
// report a non-positive pivot in *not_pd (the caller then decides between the all-zero case,
// pinv(0) = 0, and a genuine failure); with deferred errors *not_pd is 0 and the decision is
// left to the device (flags[0]).
llmc_status factor(llmc_ctx* ctx, const CholWs& w, int64_t d, int keep_L, int* not_pd) {
    LLMC_CUDA_TRY(cudaMemsetAsync(ctx->dflags, 0, 2 * sizeof(int), ctx->stream));
    LLMC_CUDA_TRY(cudaMemsetAsync(w.I, 0, (size_t)d * w.ld * sizeof(float), ctx->stream));
    LLMC_TRY(rec(ctx, w, 0, d, keep_L));
    *not_pd = 0;
    if (ctx->deferred_errors) return LLMC_OK;
    int f0, f1;
    LLMC_TRY(read_flags(ctx, &f0, &f1));
    *not_pd = f0 != 0;
    return LLMC_OK;
}

}  // namespace

llmc_status chol_inverse(llmc_ctx* ctx, const float* H, int64_t d, int64_t ldh, float damp, int upper_only, float* out,
                         int64_t ldo, int want_upper) {
    void* wsp;
    const size_t dd = (size_t)d * d;
    LLMC_TRY(workspace(ctx, 2 * dd * sizeof(float) + 4096, &wsp));
    Carver cv{(char*)wsp};
    CholWs w{cv.take<float>(dd), cv.take<float>(dd), nullptr, d};
    float* lam = cv.take<float>(4);
    diag_lambda_kernel<<<1, 256, 0, ctx->stream>>>(H, d, ldh, damp, lam);
    LLMC_TRY(check_launch(ctx, "diag_lambda"));
    prep_kernel<<<grid_for(ctx, dd), 256, 0, ctx->stream>>>(H, d, ldh, upper_only, want_upper ? 1 : 0, lam, w.A, d);
    LLMC_TRY(check_launch(ctx, "prep"));
    int not_pd = 0;
    LLMC_TRY(factor(ctx, w, d, 0, &not_pd));
    if (ctx->deferred_errors && want_upper) {
        // No host wait: the zero test and the output choice run on the device.
        nonzero_kernel<<<grid_for(ctx, dd), 256, 0, ctx->stream>>>(H, d, ldh, upper_only, ctx->dflags, 1);
        LLMC_TRY(check_launch(ctx, "nonzero"));
        finish_upper_kernel<<<grid_for(ctx, dd), 256, 0, ctx->stream>>>(w.I, d, d, out, ldo, ctx->dflags);
        return check_launch(ctx, "finish_upper");
    }
    if (ctx->deferred_errors) {
        // Hinv needs the host's decision below; take it synchronously.
        int f0, f1;
        LLMC_TRY(read_flags(ctx, &f0, &f1));
        not_pd = f0 != 0;
    }
    if (not_pd) {
        // HessianInverseSolver.cs:85-91 falls back to pinv(H').  pinv of the zero matrix is
        // zero (the no-calibration-data case, answered without the eigensolver).
        LLMC_CUDA_TRY(cudaMemsetAsync(ctx->dflags, 0, 2 * sizeof(int), ctx->stream));
        prep_kernel<<<grid_for(ctx, dd), 256, 0, ctx->stream>>>(H, d, ldh, upper_only, 0, lam, w.A, d);
        LLMC_TRY(check_launch(ctx, "prep"));
        nonzero_kernel<<<grid_for(ctx, dd), 256, 0, ctx->stream>>>(w.A, d, d, 0, ctx->dflags, 0);
        LLMC_TRY(check_launch(ctx, "nonzero"));
        int f0, f1;
        LLMC_TRY(read_flags(ctx, &f0, &f1));
        if (f1 == 0) {
            LLMC_CUDA_TRY(cudaMemset2DAsync(out, ldo * sizeof(float), 0, d * sizeof(float), d, ctx->stream));
            return LLMC_OK;
        }
        LLMC_TRY(pinv_symmetric(ctx, w.A, w.I, d, out, ldo));
        if (!want_upper) return LLMC_OK;
        // GPTQ's factor of that Hinv (GptqBlockQuantizer.cs:105-118): chol(Hinv)^T, or Hinv itself
        // when it has no Cholesky factor (the usual case for a pseudo-inverse).  In place: the
        // factorisation reads its input into the workspace first.
        return upper_factor(ctx, out, d, ldo, out, ldo);
    }
    if (want_upper) {
        remap_kernel<<<grid_for(ctx, dd), 256, 0, ctx->stream>>>(w.I, d, d, 0, out, ldo);
        return check_launch(ctx, "remap_flip");
    }
    // Hinv = L^-T L^-1 (HessianInverseSolver.cs:83)
    GemmArgs g{d, d, d, w.I, d, 1, LLMC_DTYPE_F32, w.I, d, 0, LLMC_DTYPE_F32, out, ldo, 1.f, 0.f};
    g.a_tri = TRI_KGE;
    g.b_tri = TRI_KGE;
    return gemm_f32(ctx, g);
}

llmc_status upper_factor(llmc_ctx* ctx, const float* hinv, int64_t d, int64_t ldh, float* out, int64_t ldo) {
    void* wsp;
    const size_t dd = (size_t)d * d;
    const int64_t half = (d + 1) / 2 + NB;
    LLMC_TRY(workspace(ctx, (2 * dd + (size_t)half * half) * sizeof(float) + 4096, &wsp));
    Carver cv{(char*)wsp};
    CholWs w{cv.take<float>(dd), cv.take<float>(dd), cv.take<float>((size_t)half * half), d};
    float* lam = cv.take<float>(4);
    diag_lambda_kernel<<<1, 256, 0, ctx->stream>>>(hinv, d, ldh, 0.f, lam);
    LLMC_TRY(check_launch(ctx, "diag_lambda"));
    prep_kernel<<<grid_for(ctx, dd), 256, 0, ctx->stream>>>(hinv, d, ldh, 0, 0, lam, w.A, d);
    LLMC_TRY(check_launch(ctx, "prep"));
    int not_pd = 0;
    LLMC_TRY(factor(ctx, w, d, 1, &not_pd));
    if (ctx->deferred_errors) {
        finish_factor_kernel<<<grid_for(ctx, dd), 256, 0, ctx->stream>>>(w.A, hinv, d, d, ldh, out, ldo, ctx->dflags);
        return check_launch(ctx, "finish_factor");
    }
    if (not_pd) {
        // GptqBlockQuantizer.cs:112-118: fall back to Hinv itself.
        copy2d_kernel<<<grid_for(ctx, dd), 256, 0, ctx->stream>>>(hinv, d, d, ldh, out, ldo);
        return check_launch(ctx, "copy2d");
    }
    remap_kernel<<<grid_for(ctx, dd), 256, 0, ctx->stream>>>(w.A, d, d, 1, out, ldo);
    return check_launch(ctx, "remap_transpose");
}

}  // namespace llmc
