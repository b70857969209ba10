// Internal launchers shared between the translation units of libllmc_b200.
#pragma once
#include "common.cuh"

namespace llmc {

// ---- fp32 SIMT GEMM (k_gemm.cu) --------------------------------------------------------
// C[M,N] = alpha * op(A) @ op(B) + beta * C, row-major, op(X) = X or X^T.
// Triangular hints restrict each tile's K range (the skipped region must hold zeros):
//   a_tri: 0 none, 1 op(A)[i][k] == 0 for k > i, 2 op(A)[i][k] == 0 for k < i
//   b_tri: 0 none, 1 op(B)[k][j] == 0 for k > j, 2 op(B)[k][j] == 0 for k < j
// c_mode: 0 full, 1 only i >= j is written (lower), 2 only tiles with i-tile <= j-tile (upper
// blocks of a symmetric product; diagonal tiles written in full).
// split_k > 1 partitions K; partial products are added with atomics (beta must be 1).
enum { TRI_NONE = 0, TRI_KLE = 1, TRI_KGE = 2 };
struct GemmArgs {
    int64_t M, N, K;
    const void* A; int64_t lda; int a_trans; int a_dtype;
    const void* B; int64_t ldb; int b_trans; int b_dtype;
    float* C; int64_t ldc;
    float alpha, beta;
    int a_tri = 0, b_tri = 0, c_mode = 0, split_k = 1;
};
llmc_status gemm_f32(llmc_ctx* ctx, const GemmArgs& g);
// Tensor-core (3 x TF32) path of gemm_f32; LLMC_ERR_UNSUPPORTED when the shape does not fit it.
llmc_status gemm_tc(llmc_ctx* ctx, const GemmArgs& g);

// ---- tcgen05 symmetric rank-k update (k_hessian_tc.cu) ------------------------------------
// H[upper tiles] += X^T X for bf16/f16 X [rows, d] (row stride ld).  Returns
// LLMC_ERR_UNSUPPORTED when the shape/alignment is outside the kernel's contract.
llmc_status syrk_tc(llmc_ctx* ctx, const void* x, int dtype, int64_t rows, int64_t d, int64_t ld, float* H, int64_t ldh);

// ---- observers / quantisation (k_quant.cu) -----------------------------------------------
// scratch: minmax_scratch_floats(strategy, rows) floats (only the per-tensor reduction uses it).
// Element reductions propagate NaN (torch.amin / amax).  accumulate: 0 stores the batch values;
// 1 folds them into mins / maxs (TENSOR: MinMaxObserver's strict-less rule, a NaN batch changes
// nothing; CHANNEL / GROUP: torch.minimum / maximum); 2 folds them into a new MinMaxObserver
// (+inf / -inf) per entry.
llmc_status minmax(llmc_ctx* ctx, const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld,
                   int strategy, int64_t group_size, float* mins, float* maxs, int accumulate, float* scratch);
size_t minmax_scratch_floats(int strategy, int64_t rows);
llmc_status affine(llmc_ctx* ctx, const float* mins, const float* maxs, int64_t count, int bits, int sym,
                   float* scales, int32_t* zps);
// Number of (scale, zp) entries per row and per-row stride for a strategy over n columns.
inline int64_t n_groups(int strategy, int64_t n, int64_t gs) {
    return strategy == LLMC_STRATEGY_GROUP ? (n + gs - 1) / gs : 1;
}

// ---- Cholesky / inverse (k_chol.cu) -------------------------------------------------------
llmc_status chol_inverse(llmc_ctx* ctx, const float* H, int64_t d, int64_t ldh, float damp, int upper_only,
                         float* out, int64_t ldo, int want_upper);
llmc_status upper_factor(llmc_ctx* ctx, const float* hinv, int64_t d, int64_t ldh, float* out, int64_t ldo);
// pinv of a symmetric matrix given by the lower triangle of A (d x d row-major, overwritten),
// torch.linalg.pinv's default cutoff; B is d x d scratch (pinv.cu).  Synchronises the stream.
llmc_status pinv_symmetric(llmc_ctx* ctx, float* A, float* B, int64_t d, float* out, int64_t ldo);

// ---- per-token activation quantisation (k_act.cu) ------------------------------------------
llmc_status act_quant_per_token(llmc_ctx* ctx, const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld,
                                int bits, int sym, uint8_t* codes, int64_t ldc, float* scales, int32_t* zps, void* deq,
                                int64_t ldd);

// ---- compressed-tensors packing (k_pack.cu) --------------------------------------------------
// zrow: zero-point entries per row (0: one shared entry, tensor strategy); zp_out (nullable)
// receives the row-packed zero-points [ceil(m / (32 / bits)), zrow] (zrow >= 1).
llmc_status ct_pack(llmc_ctx* ctx, const uint8_t* codes, int64_t m, int64_t n, int64_t crow, const int32_t* zps,
                    int64_t zrow, int64_t gs, int bits, int sym, int32_t* out, int64_t ldo, int32_t* zp_out);

// ---- GPTQ activation order (k_actorder.cu) --------------------------------------------------
llmc_status act_order_perm(llmc_ctx* ctx, const float* H, int64_t d, int64_t ldh, int32_t* perm);
llmc_status permute_hessian(llmc_ctx* ctx, const float* H, int64_t d, int64_t ldh, int upper_only, const int32_t* perm,
                            float* out, int64_t ldo);
llmc_status gather_cols(llmc_ctx* ctx, const float* src, int64_t rows, int64_t n, int64_t lds, const int32_t* perm,
                        float* dst, int64_t ldd);
llmc_status scatter_cols(llmc_ctx* ctx, const float* src, int64_t rows, int64_t n, int64_t lds, const int32_t* perm,
                         float* dst, int64_t ldd);
llmc_status perm_maps(llmc_ctx* ctx, const int32_t* perm, int64_t n, int64_t gs, int32_t* col_group, int32_t* inv);
llmc_status scatter_codes(llmc_ctx* ctx, const uint8_t* src, int64_t rows, int64_t n, const int32_t* inv, int bits,
                          uint8_t* dst, int64_t crow);

// ---- misc ----------------------------------------------------------------------------------
// Drops the no-allocation observer's cached device address of its static row buffer on
// `device` (noalloc.cu); llmc_init calls it so that a reset device gets a fresh lookup.
void noalloc_forget(int device);
llmc_status device_error_check(llmc_ctx* ctx);
llmc_status symmetrize_from_upper(llmc_ctx* ctx, const float* src, int64_t d, int64_t lds, float* dst, int64_t ldd);
llmc_status convert_to_f32(llmc_ctx* ctx, const void* src, int dtype, int64_t rows, int64_t cols, int64_t lds,
                           float* dst, int64_t ldd);

}  // namespace llmc
