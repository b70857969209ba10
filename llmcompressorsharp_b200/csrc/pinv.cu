// Pseudo-inverse of a symmetric matrix: the reference's fallback when the damped Hessian has no
// Cholesky factor (HessianInverseSolver.cs:85-91 returns linalg.pinv(H')).
//
// torch.linalg.pinv(A) (hermitian = false, no tolerances given) keeps the singular values
// s > rtol * max(s) with rtol = eps(fp32) * max(m, n) and returns V diag(1/s) U^T.  For a
// symmetric A the singular values are the |lambda| of its eigenvalues and the result is
//   pinv(A) = sum_k [|lambda_k| > tol] v_k v_k^T / lambda_k,
// which is what this computes: eigenvalues and eigenvectors from cuSOLVER's symmetric
// eigensolver (syevd), then one scaling kernel and one 3xTF32 GEMM (V^T (D V)).  Rows and
// columns of an exactly zero row of the matrix (a dead input channel) are set to exactly zero,
// their value in exact arithmetic (the eigensolver, like an SVD, leaves rounding residue there),
// so that GPTQ's later Cholesky of the result meets a zero pivot at that channel and takes the
// U = Hinv fallback, as exact arithmetic does.  cuSOLVER is
// opened with dlopen at the first call, so the library has no link-time dependency on it;
// cusolverDn.h supplies the types only.  A rare, synchronous path: it waits for the eigensolver's
// status and allocates its own scratch.
#include <cusolverDn.h>
#include <dlfcn.h>

#include <algorithm>
#include <cfloat>
#include <climits>
#include <cstring>
#include <mutex>

#include "ops.h"

namespace llmc {
namespace {

struct SolverApi {
    cusolverStatus_t (*create)(cusolverDnHandle_t*);
    cusolverStatus_t (*destroy)(cusolverDnHandle_t);
    cusolverStatus_t (*set_stream)(cusolverDnHandle_t, cudaStream_t);
    cusolverStatus_t (*syevd_buffer)(cusolverDnHandle_t, cusolverEigMode_t, cublasFillMode_t, int, const float*, int,
                                     const float*, int*);
    cusolverStatus_t (*syevd)(cusolverDnHandle_t, cusolverEigMode_t, cublasFillMode_t, int, float*, int, float*, float*,
                              int, int*);
};

const SolverApi* solver_api() {
    static std::once_flag once;
    static SolverApi api;
    static bool ok = false;
    std::call_once(once, [] {
        void* lib = dlopen("libcusolver.so.11", RTLD_NOW | RTLD_LOCAL);
        if (!lib) lib = dlopen("libcusolver.so", RTLD_NOW | RTLD_LOCAL);
        if (!lib) return;
        bool all = true;
        auto sym = [&](auto& fn, const char* name) {
            void* p = dlsym(lib, name);
            all &= p != nullptr;
            std::memcpy(&fn, &p, sizeof(p));
        };
        sym(api.create, "cusolverDnCreate");
        sym(api.destroy, "cusolverDnDestroy");
        sym(api.set_stream, "cusolverDnSetStream");
        sym(api.syevd_buffer, "cusolverDnSsyevd_bufferSize");
        sym(api.syevd, "cusolverDnSsyevd");
        ok = all;
    });
    return ok ? &api : nullptr;
}

// B[k][:] = V[k][:] / lambda_k when |lambda_k| > tol, else 0.  Row k of V is the k-th
// eigenvector (syevd's column-major output read row-major); w holds the eigenvalues in
// ascending order, so max |lambda| is at one of its ends.  A NaN spectrum (a NaN input) gives
// a NaN result rather than zeros.
__global__ void pinv_scale_kernel(const float* V, const float* w, int64_t d, float rtol, float* B) {
    const float lo = w[0], hi = w[d - 1];
    const bool nan = lo != lo || hi != hi;
    const float tol = __fmul_rn(rtol, fmaxf(fabsf(lo), fabsf(hi)));
    const int64_t total = d * d;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const float lam = w[t / d];
        B[t] = nan ? __int_as_float(0x7fc00000) : (fabsf(lam) > tol ? __fmul_rn(V[t], __frcp_rn(lam)) : 0.f);
    }
}

// nz[i] = 1 when row i of the symmetric matrix (its lower triangle in A) holds a non-zero entry.
__global__ void pinv_nonzero_rows_kernel(const float* A, int64_t d, int* nz) {
    const int64_t total = d * d;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / d, j = t % d;
        if (j <= i && A[t] != 0.f) {
            nz[i] = 1;
            nz[j] = 1;
        }
    }
}

// A row (and column) that is exactly zero in the matrix is an exact null direction, so it is
// exactly zero in the pseudo-inverse; the eigensolver leaves rounding residue there instead.
__global__ void pinv_zero_dead_kernel(const int* nz, int64_t d, float* out, int64_t ldo) {
    const int64_t total = d * d;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / d, j = t % d;
        if (!nz[i] || !nz[j]) out[i * ldo + j] = 0.f;
    }
}

struct SolverHandle {
    const SolverApi* api = nullptr;
    cusolverDnHandle_t h = nullptr;
    ~SolverHandle() {
        if (h) api->destroy(h);
    }
};

struct DeviceScratch {
    void* p = nullptr;
    ~DeviceScratch() {
        if (p) cudaFree(p);
    }
};

}  // namespace

// A: d x d row-major, its lower triangle holding the symmetric matrix (destroyed: it receives
// the eigenvectors).  B: d x d scratch.  out (ldo) = pinv of the matrix.
llmc_status pinv_symmetric(llmc_ctx* ctx, float* A, float* B, int64_t d, float* out, int64_t ldo) {
    if (d < 1 || d > INT_MAX / 2) return fail(LLMC_ERR_INVALID_ARG, "pinv: unsupported size d=%lld", (long long)d);
    SolverHandle sh;
    sh.api = solver_api();
    if (!sh.api) return fail(LLMC_ERR_UNSUPPORTED, "pinv fallback needs cuSOLVER (libcusolver.so.11), which could not "
                             "be loaded");
    if (sh.api->create(&sh.h) != CUSOLVER_STATUS_SUCCESS) {
        sh.h = nullptr;
        return fail(LLMC_ERR_CUDA, "pinv: cusolverDnCreate failed");
    }
    if (sh.api->set_stream(sh.h, ctx->stream) != CUSOLVER_STATUS_SUCCESS)
        return fail(LLMC_ERR_CUDA, "pinv: cusolverDnSetStream failed");
    const int n = (int)d;
    // The row-major lower triangle is the column-major upper triangle.
    const cublasFillMode_t uplo = CUBLAS_FILL_MODE_UPPER;
    DeviceScratch wbuf, wsp;
    const size_t w_floats = ((size_t)d + 63) / 64 * 64;
    LLMC_CUDA_TRY(cudaMalloc(&wbuf.p, 2 * w_floats * sizeof(float) + 64));
    float* w = static_cast<float*>(wbuf.p);
    int* nz = reinterpret_cast<int*>(w + w_floats);
    int* info = nz + w_floats;
    const int64_t blocks = std::max<int64_t>(
        std::min<int64_t>(((int64_t)d * d + 255) / 256, (int64_t)ctx->sm_count * 8), 1);
    LLMC_CUDA_TRY(cudaMemsetAsync(nz, 0, (size_t)d * sizeof(int), ctx->stream));
    pinv_nonzero_rows_kernel<<<(int)blocks, 256, 0, ctx->stream>>>(A, d, nz);
    LLMC_TRY(check_launch(ctx, "pinv_nonzero_rows"));
    int lwork = 0;
    if (sh.api->syevd_buffer(sh.h, CUSOLVER_EIG_MODE_VECTOR, uplo, n, A, n, w, &lwork) != CUSOLVER_STATUS_SUCCESS)
        return fail(LLMC_ERR_CUDA, "pinv: cusolverDnSsyevd_bufferSize failed");
    LLMC_CUDA_TRY(cudaMalloc(&wsp.p, (size_t)std::max(lwork, 1) * sizeof(float)));
    float* work = static_cast<float*>(wsp.p);
    if (sh.api->syevd(sh.h, CUSOLVER_EIG_MODE_VECTOR, uplo, n, A, n, w, work, lwork, info) != CUSOLVER_STATUS_SUCCESS)
        return fail(LLMC_ERR_CUDA, "pinv: cusolverDnSsyevd failed");
    int hinfo = 0;
    LLMC_CUDA_TRY(cudaMemcpyAsync(&hinfo, info, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
    LLMC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    if (hinfo != 0)
        return fail(LLMC_ERR_NOT_PD, "damped Hessian (d=%lld) is not positive definite and its pseudo-inverse "
                    "failed: the symmetric eigensolver did not converge (info %d)", (long long)d, hinfo);
    const float rtol = (float)((double)FLT_EPSILON * (double)d);
    pinv_scale_kernel<<<(int)blocks, 256, 0, ctx->stream>>>(A, w, d, rtol, B);
    LLMC_TRY(check_launch(ctx, "pinv_scale"));
    // out = V^T (D V), V with the eigenvectors as rows.
    GemmArgs g{d, d, d, A, d, 1, LLMC_DTYPE_F32, B, d, 0, LLMC_DTYPE_F32, out, ldo, 1.f, 0.f};
    LLMC_TRY(gemm_f32(ctx, g));
    pinv_zero_dead_kernel<<<(int)blocks, 256, 0, ctx->stream>>>(nz, d, out, ldo);
    LLMC_TRY(check_launch(ctx, "pinv_zero_dead"));
    // The kernels read the eigenvalues and the row flags from wbuf, freed on return.
    LLMC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    return LLMC_OK;
}

}  // namespace llmc
