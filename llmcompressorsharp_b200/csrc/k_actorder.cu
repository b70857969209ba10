// GPTQ activation order ("act_order"): columns quantised in decreasing order of the Hessian
// diagonal.
//
// Extension.  The reference rejects GPTQConfig.ActOrder (GPTQModifier.cs:47-56,
// GptqBlockQuantizer.cs:77-82).  The restatement follows the published GPTQ activation-order
// heuristic with static groups:
//   perm   = stable argsort of diag(H), descending (NaN first, ties by column index);
//   H_p    = H[perm][:, perm], factor U_p of H_p as for any Hessian;
//   params = ComputeScaleZeroPoint of the ORIGINAL weight, per original column group
//            (GptqBlockQuantizer.cs:97 computes them before the loop);
//   loop   = the column-block solve over W[:, perm] against U_p, column a using the
//            parameters of original column perm[a]'s group;
//   output = the fake-quantised weight and codes scattered back to the original columns.
//
// Kernels here: the permutation, the permuted Hessian, the column gather of the working copy,
// the per-column group map and the scatter of the results.
#include "ops.h"

namespace llmc {
namespace {

constexpr int RANK_TILE = 1024;

// a (at index i) comes before b (at index j) in the descending order with NaN first.
__device__ __forceinline__ bool before(float a, int i, float b, int j) {
    const bool na = a != a, nb = b != b;
    if (na != nb) return na;
    if (!na && a != b) return a > b;
    return i < j;
}

// perm[rank(i)] = i with rank(i) = number of diagonal entries that come before entry i.
__global__ void diag_rank_kernel(const float* H, int64_t d, int64_t ldh, int32_t* perm) {
    __shared__ float keys[RANK_TILE];
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const float ki = i < d ? H[i * ldh + i] : 0.f;
    int64_t rank = 0;
    for (int64_t t0 = 0; t0 < d; t0 += RANK_TILE) {
        const int64_t cnt = min((int64_t)RANK_TILE, d - t0);
        __syncthreads();
        for (int64_t k = threadIdx.x; k < cnt; k += blockDim.x) keys[k] = H[(t0 + k) * ldh + t0 + k];
        __syncthreads();
        if (i < d)
            for (int64_t k = 0; k < cnt; k++) rank += before(keys[k], (int)(t0 + k), ki, (int)i) ? 1 : 0;
    }
    if (i < d) perm[rank] = (int32_t)i;
}

// out[a][b] = H[perm[a]][perm[b]] (the upper triangle of H is read when upper_only).
__global__ void permute_sym_kernel(const float* H, int64_t d, int64_t ldh, int upper_only, const int32_t* perm,
                                   float* out, int64_t ldo) {
    const int64_t total = d * d;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t a = t / d, b = t % d;
        int64_t i = perm[a], j = perm[b];
        if (upper_only && i > j) {
            const int64_t x = i;
            i = j;
            j = x;
        }
        out[a * ldo + b] = H[i * ldh + j];
    }
}

// dst[r][a] = src[r][perm[a]]
__global__ void gather_cols_kernel(const float* src, int64_t rows, int64_t n, int64_t lds, const int32_t* perm, float* dst,
                                   int64_t ldd) {
    const int64_t total = rows * n;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / n, a = t % n;
        dst[r * ldd + a] = src[r * lds + perm[a]];
    }
}

// dst[r][perm[a]] = src[r][a]
__global__ void scatter_cols_kernel(const float* src, int64_t rows, int64_t n, int64_t lds, const int32_t* perm,
                                    float* dst, int64_t ldd) {
    const int64_t total = rows * n;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / n, a = t % n;
        dst[r * ldd + perm[a]] = src[r * lds + a];
    }
}

// col_group[a] = perm[a] / gs; inv[perm[a]] = a.
__global__ void perm_maps_kernel(const int32_t* perm, int64_t n, int64_t gs, int32_t* col_group, int32_t* inv) {
    for (int64_t a = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; a < n; a += (int64_t)gridDim.x * blockDim.x) {
        const int32_t p = perm[a];
        col_group[a] = (int32_t)(p / gs);
        inv[p] = (int32_t)a;
    }
}

// Codes, one byte per element in permuted column order ([rows, n], row stride n), back to the
// original columns: packed nibbles (bits <= 4; even column in the high nibble) or bytes.
__global__ void scatter_codes_kernel(const uint8_t* src, int64_t rows, int64_t n, const int32_t* inv, int bits,
                                     uint8_t* dst, int64_t crow) {
    const int64_t per_row = bits <= 4 ? (n + 1) / 2 : n;
    const int64_t total = rows * per_row;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / per_row, c = t % per_row;
        const uint8_t* s = src + r * n;
        if (bits <= 4) {
            const int64_t c0 = 2 * c, c1 = 2 * c + 1;
            const uint8_t hi = s[inv[c0]] & 0xF;
            const uint8_t lo = c1 < n ? (uint8_t)(s[inv[c1]] & 0xF) : (uint8_t)0;
            dst[r * crow + c] = (uint8_t)((hi << 4) | lo);
        } else {
            dst[r * crow + c] = s[inv[c]];
        }
    }
}

int grid_n(llmc_ctx* ctx, int64_t items) {
    int64_t b = (items + 255) / 256;
    const int64_t cap = (int64_t)ctx->sm_count * 8;
    return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace

llmc_status act_order_perm(llmc_ctx* ctx, const float* H, int64_t d, int64_t ldh, int32_t* perm) {
    diag_rank_kernel<<<(unsigned)((d + 255) / 256), 256, 0, ctx->stream>>>(H, d, ldh, perm);
    return check_launch(ctx, "diag_rank");
}

llmc_status permute_hessian(llmc_ctx* ctx, const float* H, int64_t d, int64_t ldh, int upper_only, const int32_t* perm,
                            float* out, int64_t ldo) {
    permute_sym_kernel<<<grid_n(ctx, d * d), 256, 0, ctx->stream>>>(H, d, ldh, upper_only, perm, out, ldo);
    return check_launch(ctx, "permute_sym");
}

llmc_status gather_cols(llmc_ctx* ctx, const float* src, int64_t rows, int64_t n, int64_t lds, const int32_t* perm,
                        float* dst, int64_t ldd) {
    gather_cols_kernel<<<grid_n(ctx, rows * n), 256, 0, ctx->stream>>>(src, rows, n, lds, perm, dst, ldd);
    return check_launch(ctx, "gather_cols");
}

llmc_status scatter_cols(llmc_ctx* ctx, const float* src, int64_t rows, int64_t n, int64_t lds, const int32_t* perm,
                         float* dst, int64_t ldd) {
    scatter_cols_kernel<<<grid_n(ctx, rows * n), 256, 0, ctx->stream>>>(src, rows, n, lds, perm, dst, ldd);
    return check_launch(ctx, "scatter_cols");
}

llmc_status perm_maps(llmc_ctx* ctx, const int32_t* perm, int64_t n, int64_t gs, int32_t* col_group, int32_t* inv) {
    perm_maps_kernel<<<grid_n(ctx, n), 256, 0, ctx->stream>>>(perm, n, gs, col_group, inv);
    return check_launch(ctx, "perm_maps");
}

llmc_status scatter_codes(llmc_ctx* ctx, const uint8_t* src, int64_t rows, int64_t n, const int32_t* inv, int bits,
                          uint8_t* dst, int64_t crow) {
    const int64_t per_row = bits <= 4 ? (n + 1) / 2 : n;
    scatter_codes_kernel<<<grid_n(ctx, rows * per_row), 256, 0, ctx->stream>>>(src, rows, n, inv, bits, dst, crow);
    return check_launch(ctx, "scatter_codes");
}

}  // namespace llmc
