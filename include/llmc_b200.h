/*
 * llmc_b200.h — C ABI of the B200 (sm_100a) one-shot compression library.
 *
 * Every entry point replaces one LibTorch call chain of LLMCompressorSharp's hot path;
 * the comment on each cites the reference interface (path:line, relative to the
 * LLMCompressorSharp repository root) whose behaviour it reproduces.
 *
 * Conventions
 *  - All tensor arguments are caller-owned DEVICE pointers on the context's device
 *    (TorchSharp / PyTorch CUDA tensor data pointers), row-major, with an explicit
 *    leading dimension in elements where one is taken.  The library keeps no caller
 *    pointer after a call returns.
 *  - Work is stream-ordered on the context's stream (llmc_set_stream; by default a
 *    stream the context creates).  A call returns when its work is enqueued, except
 *    where a result is read back to the host (documented per call).
 *  - Every function returns an llmc_status; nothing throws or aborts across the ABI.
 *    llmc_last_error() gives the calling thread's message for the last failure.
 *  - Handles (llmc_ctx, llmc_hessian) are not thread-safe: one context per device and
 *    host thread.
 */
#ifndef LLMC_B200_H
#define LLMC_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define LLMC_ABI_VERSION 1

typedef enum {
    LLMC_OK = 0,
    LLMC_ERR_INVALID_ARG = 1,  /* null pointer / bad enum  -> ArgumentNullException, ArgumentException */
    LLMC_ERR_SHAPE = 2,        /* "last dim", "square"     -> ArgumentException */
    LLMC_ERR_UNSUPPORTED = 3,  /* ActOrder, strategy        -> NotSupportedException */
    LLMC_ERR_NOT_PD = 4,       /* Cholesky failed and no device fallback applies */
    LLMC_ERR_CUDA = 5,
    LLMC_ERR_NCCL = 6,
    LLMC_ERR_TIMEOUT = 7,      /* a bounded device wait gave up */
    LLMC_ERR_INTERNAL = 8,
    LLMC_ERR_NO_SAMPLES = 9,   /* observer without samples -> InvalidOperationException */
    LLMC_ERR_OUT_OF_RANGE = 10 /* numBits, inFeatures       -> ArgumentOutOfRangeException */
} llmc_status;

typedef enum { LLMC_DTYPE_F32 = 0, LLMC_DTYPE_BF16 = 1, LLMC_DTYPE_F16 = 2 } llmc_dtype;

/* QuantizationStrategy (src/LLMCompressorSharp.TorchExtensions/Observers/QuantizationStrategy.cs:9-19)
 * plus GROUP, one (scale, zero-point) per (output row, group_size input columns). */
typedef enum {
    LLMC_STRATEGY_TENSOR = 0,
    LLMC_STRATEGY_CHANNEL = 1,
    LLMC_STRATEGY_TOKEN = 2,
    LLMC_STRATEGY_GROUP = 3
} llmc_strategy;

/* GPTQConfig / RtnConfig fields (src/LLMCompressorSharp.Core/Algorithms/Configs/GPTQConfig.cs:22-59,
 * RtnConfig.cs:17-26), plus group_size and the SparseGPT mask fields. */
typedef struct {
    int32_t num_bits;      /* 2..16 */
    int32_t symmetric;     /* 1: grid [-(2^(b-1)-1), 2^(b-1)-1]; 0: [0, 2^b-1] with zero-point */
    int32_t strategy;      /* llmc_strategy */
    int32_t channel_axis;  /* must be 0 (output channels of a Linear weight) */
    int32_t group_size;    /* columns per group for LLMC_STRATEGY_GROUP */
    int32_t block_size;    /* GPTQ / SparseGPT column block (columns are processed <=128 at a time) */
    float damp;            /* DampeningFrac */
    int32_t act_order;     /* must be 0 (the reference rejects ActOrder) */
    float sparsity;        /* SparseGPT unstructured sparsity in [0,1) */
    int32_t mask_n;        /* SparseGPT N:M structure (keep N of every M); 0 = unstructured */
    int32_t mask_m;
} llmc_qconfig;

typedef struct llmc_ctx llmc_ctx;
typedef struct llmc_hessian llmc_hessian;

/* ---- library / context ------------------------------------------------------------ */
const char* llmc_last_error(void);
int32_t llmc_abi_version(void);
llmc_status llmc_init(int32_t device, llmc_ctx** out);
llmc_status llmc_destroy(llmc_ctx* ctx);
/* Use the caller's cudaStream_t (passed as void*); NULL restores the context's own
 * (non-blocking) stream.  To run on the legacy default stream pass cudaStreamLegacy
 * ((void*)0x1), not NULL. */
llmc_status llmc_set_stream(llmc_ctx* ctx, void* stream);
/* Share the device with another context (0 = this context has it to itself).  sms > 0 caps
 * the persistent Hessian kernel at `sms` SMs, and makes the tensor-core GEMMs of the factor and
 * the GPTQ tail launch one CTA per tile (instead of one persistent CTA per SM) so that they
 * start wherever SMs free up.  No reference counterpart: two contexts on one device, one
 * accumulating the next layer's Hessians while the other solves the previous layer on another
 * stream. */
llmc_status llmc_set_sm_limit(llmc_ctx* ctx, int32_t sms);
/* Bound of every wait inside this context's tensor-core kernels (the Hessian and the 3xTF32
 * GEMMs), in try_wait attempts; tries < 0 restores the default (2^26).  A wait that runs out
 * stops its kernel: the kernel raises an error word, waits (bounded) for the copies and MMAs
 * it issued, frees its tensor memory and returns; the next llmc_sync (or any call that reads
 * results) reports LLMC_ERR_TIMEOUT, clears the word, and the context stays usable.  tries = 0
 * makes the first wait of the next such kernel give up at once, before it has issued any copy.
 * No reference counterpart (the reference has no device waits). */
llmc_status llmc_set_wait_limit(llmc_ctx* ctx, int64_t tries);
/* on = 1: llmc_chol_inverse with want_upper = 1 and llmc_upper_factor no longer wait for the
 * factorisation.  A non-positive-definite input is then decided on the device: the all-zero
 * matrix still gives the zero factor (pinv(0) = 0, HessianInverseSolver.cs:85-91) and
 * llmc_upper_factor still falls back to U = Hinv (GptqBlockQuantizer.cs:112-118), while any
 * other non-PD input gets a zero factor and LLMC_ERR_NOT_PD from the next llmc_sync (or from
 * any call that reads results back) instead of from the call itself; the pseudo-inverse
 * fallback needs the synchronous path, so a host factors such a Hessian again with deferred
 * errors off.  on = 0 (the default) restores the synchronous reporting.  No reference counterpart: it lets one host thread
 * enqueue a layer's solve while other streams keep running. */
llmc_status llmc_set_deferred_errors(llmc_ctx* ctx, int32_t on);
llmc_status llmc_sync(llmc_ctx* ctx);
/* Number of kernels this context has launched since creation (diagnostics / bench). */
llmc_status llmc_launch_count(llmc_ctx* ctx, int64_t* out);

/* ---- Hessian accumulation: HessianAccumulator ---------------------------------------
 * src/LLMCompressorSharp.TorchExtensions/Hessian/HessianAccumulator.cs:16-99.
 * The handle owns an fp32 [d,d] device matrix; updates accumulate the upper triangle,
 * reads return the full symmetric matrix. */
/* ctor, HessianAccumulator.cs:26-35 (in_features <= 0 -> OUT_OF_RANGE) */
llmc_status llmc_hessian_create(llmc_ctx* ctx, int64_t in_features, llmc_hessian** out);
/* Update(x), HessianAccumulator.cs:47-67: H += X^T X for X = [rows, in_features] with row
 * stride ld (elements); dtype F32/BF16/F16.  bf16/f16 run on tcgen05 tensor cores with
 * fp32 accumulation (products are exact); f32 runs 3xTF32 on the tensor cores (in_features
 * >= 512 and rows >= 1024) or an fp32 SIMT kernel (smaller calls). */
llmc_status llmc_hessian_update(llmc_hessian* h, const void* x, int32_t dtype, int64_t rows, int64_t ld);
/* GetHessian(), HessianAccumulator.cs:71-75: writes the full symmetric [d,d] fp32 to out. */
llmc_status llmc_hessian_get(llmc_hessian* h, float* out);
/* Raw device pointer of the accumulator (upper triangle authoritative), for zero-copy use
 * by llmc_chol_inverse (pass upper_only=1) and for collectives. */
llmc_status llmc_hessian_data(llmc_hessian* h, float** out);
/* Reset(), HessianAccumulator.cs:78-83 */
llmc_status llmc_hessian_reset(llmc_hessian* h);
/* SampleCount, HessianAccumulator.cs:38 */
llmc_status llmc_hessian_sample_count(llmc_hessian* h, int64_t* out);
/* Add rows to the sample count without data (after an external reduction of H). */
llmc_status llmc_hessian_add_samples(llmc_hessian* h, int64_t rows);
/* Dispose(), HessianAccumulator.cs:86-93 */
llmc_status llmc_hessian_destroy(llmc_hessian* h);

/* ---- Hessian collectives over NCCL (multi-GPU: one process or thread per GPU) -------------
 * Calibration tokens are split across ranks; the partial Hessians sum exactly
 * (HessianAccumulator.cs:59-64 is a sum over rows).  NCCL is loaded from libnccl.so.2 at the
 * first call (the library does not link it; a process that already loaded it shares that
 * copy); without it these calls return LLMC_ERR_UNSUPPORTED.  `comm` is an ncclComm_t: the
 * caller's own, or one made by llmc_nccl_comm_init.  Every rank must make the same calls in
 * the same order. */
#define LLMC_NCCL_UNIQUE_ID_BYTES 128
/* ncclGetUniqueId on the root rank; the caller sends the bytes to the other ranks. */
llmc_status llmc_nccl_unique_id(uint8_t* out, int64_t size);
/* ncclCommInitRank on the context's device. */
llmc_status llmc_nccl_comm_init(llmc_ctx* ctx, int32_t world, int32_t rank, const uint8_t* unique_id, int64_t size,
                                void** comm_out);
llmc_status llmc_nccl_comm_destroy(void* comm);
/* H and the sample count summed over all ranks, in place on every rank (ncclAllReduce of the
 * [d,d] fp32 matrix on the context's stream).  Synchronises the stream (the count is read back). */
llmc_status llmc_hessian_allreduce(llmc_hessian* h, void* comm);
/* H and the sample count summed onto `root` only (ncclReduce); other ranks keep their partial
 * H and count.  Synchronises the stream. */
llmc_status llmc_hessian_reduce(llmc_hessian* h, void* comm, int32_t root);

/* ---- damped Cholesky inverse: HessianInverseSolver.Compute ------------------------------
 * src/LLMCompressorSharp.TorchExtensions/Hessian/HessianInverseSolver.cs:44-92 and the U
 * factor of GptqBlockQuantizer.cs:105-118.
 *   H' = H + damp * mean(diag H) * I (damp > 0 only)
 *   want_upper = 0: out = Hinv = L^-T L^-1 with L = chol(H')           (the solver's return)
 *   want_upper = 1: out = U, upper triangular with U^T U = H'^-1          (GPTQ's factor; computed
 *                   directly as the inverse of the reversed-order Cholesky factor of H')
 * upper_only = 1 reads only the upper triangle of H (as llmc_hessian_data leaves it).
 * Non-positive-definite H' (no Cholesky factor): the reference's fallback Hinv = pinv(H')
 * (HessianInverseSolver.cs:85-91), computed from the symmetric eigendecomposition of H' with
 * torch.linalg.pinv's default cutoff (|lambda| > eps(fp32) * d * max |lambda| kept); cuSOLVER
 * is opened at the first such call.  The all-zero matrix gives 0 without the eigensolver.  With
 * want_upper = 1 the result is then GPTQ's factor of that Hinv: chol(Hinv)^T, or Hinv itself
 * when it has no Cholesky factor (GptqBlockQuantizer.cs:105-118).  LLMC_ERR_NOT_PD only if the
 * eigensolver does not converge.  Reads one flag back to the host (synchronises the stream). */
llmc_status llmc_chol_inverse(llmc_ctx* ctx, const float* H, int64_t d, int64_t ldh, float damp,
                              int32_t upper_only, float* out, int64_t ldo, int32_t want_upper);
/* U = chol(Hinv)^T with the reference's fallback U = Hinv when Hinv is not PD
 * (GptqBlockQuantizer.cs:105-118).  Synchronises the stream. */
llmc_status llmc_upper_factor(llmc_ctx* ctx, const float* hinv, int64_t d, int64_t ldh, float* out, int64_t ldo);

/* ---- GPTQ column-block solve: GptqBlockQuantizer.Quantize --------------------------------
 * src/LLMCompressorSharp.Core/Algorithms/Gptq/GptqBlockQuantizer.cs:71-274.
 * W [m,n] (dtype, row stride ldw) is not modified.  U is the upper factor (llmc_chol_inverse
 * want_upper=1 or llmc_upper_factor).  Scales / zero-points come from the ORIGINAL W
 * (ComputeScaleZeroPoint, :196-234) with the strategy's shape: TENSOR [1], CHANNEL [m],
 * GROUP [m, ceil(n/group_size)].
 * Outputs (each optional, NULL to skip):
 *   wq_out    fp32 [m,n] (row stride ldq) fake-quantised weight — the reference's return value
 *   codes_out integer codes q = clamp(round(w/s)+zp): bits <= 4 packed two per byte, row-major
 *             ceil(n/2) bytes per row, even column in the HIGH nibble, nibble = (q - zp) & 0xF
 *             (Int4PackedTensor.cs:47-69); 4 < bits <= 8 one byte (uint8)q per element
 *   scales_out fp32, zps_out int32 (shapes above). */
llmc_status llmc_gptq_quantize(llmc_ctx* ctx, const void* W, int32_t dtype, int64_t m, int64_t n, int64_t ldw,
                               const float* U, int64_t ldu, const llmc_qconfig* cfg,
                               float* wq_out, int64_t ldq, uint8_t* codes_out, float* scales_out, int32_t* zps_out);

/* Several weights that share one Hessian (q/k/v read the attention input, gate/up the MLP
 * input) solved in one call as a stacked matrix: weight k is W[k] [m[k], n] (row stride
 * ldw[k]); every output is stacked in weight order over sum(m) rows (wq_out row stride ldq,
 * codes/scales/zero-points as llmc_gptq_quantize for the stacked matrix), except that the
 * TENSOR strategy returns one scale / zero-point per weight.  Results equal `count` separate
 * llmc_gptq_quantize calls (GptqBlockQuantizer.Quantize per weight, GPTQModifier.cs:119-136).
 * W, m and ldw are host arrays of `count` entries; W[k] are device pointers. */
llmc_status llmc_gptq_quantize_batch(llmc_ctx* ctx, int32_t count, const void* const* W, const int64_t* m,
                                     const int64_t* ldw, int32_t dtype, int64_t n, const float* U, int64_t ldu,
                                     const llmc_qconfig* cfg, float* wq_out, int64_t ldq, uint8_t* codes_out,
                                     float* scales_out, int32_t* zps_out);

/* ---- GPTQ activation order (extension) -----------------------------------------------------
 * No reference counterpart: the reference rejects GPTQConfig.ActOrder (GPTQModifier.cs:47-56,
 * GptqBlockQuantizer.cs:77-82; llmc_gptq_quantize keeps that rejection).  Flow: perm from
 * llmc_gptq_act_order_perm(H); H_p from llmc_permute_hessian(H, perm); U_p from
 * llmc_chol_inverse(H_p, want_upper = 1); then llmc_gptq_quantize_batch_perm(W, U_p, perm).
 * Scales / zero-points come from the original weight per original column group (static
 * groups, as GptqBlockQuantizer.cs:97 computes them before the loop); outputs are in the
 * original column order. */
/* perm_out[k] = column with the k-th largest H[k][k] (stable: equal values by index; NaN first). */
llmc_status llmc_gptq_act_order_perm(llmc_ctx* ctx, const float* H, int64_t d, int64_t ldh, int32_t* perm_out);
/* out[a][b] = H[perm[a]][perm[b]], full matrix; upper_only reads H's upper triangle. */
llmc_status llmc_permute_hessian(llmc_ctx* ctx, const float* H, int64_t d, int64_t ldh, int32_t upper_only,
                                 const int32_t* perm, float* out, int64_t ldo);
/* llmc_gptq_quantize_batch with U the factor of the permuted Hessian and perm its column order;
 * cfg->act_order is not checked.  Arguments otherwise as llmc_gptq_quantize_batch. */
llmc_status llmc_gptq_quantize_batch_perm(llmc_ctx* ctx, int32_t count, const void* const* W, const int64_t* m,
                                          const int64_t* ldw, int32_t dtype, int64_t n, const float* U, int64_t ldu,
                                          const int32_t* perm, const llmc_qconfig* cfg, float* wq_out, int64_t ldq,
                                          uint8_t* codes_out, float* scales_out, int32_t* zps_out);

/* ---- SparseGPT (plan docs/superpowers/plans/2026-05-18-phase-4c-sparsegpt.md:37-59,1584-1656,
 * in the U-factor form of GptqBlockQuantizer.cs:124-181).  out fp32 [m,n] pruned weight,
 * mask_out (optional) one byte per element, 1 = kept. */
llmc_status llmc_sparsegpt_prune(llmc_ctx* ctx, const void* W, int32_t dtype, int64_t m, int64_t n, int64_t ldw,
                                 const float* U, int64_t ldu, const llmc_qconfig* cfg,
                                 float* out, int64_t ldo, uint8_t* mask_out);

/* ---- observers -----------------------------------------------------------------------
 * MinMaxObserver.Update (MinMaxObserver.cs:24-45), PerChannelMinMaxObserver.Update
 * (PerChannelMinMaxObserver.cs:38-76, channel axis 0 of a 2-D view) and the group extension.
 * x is [rows, cols] (row stride ld).  Output count: TENSOR 1, CHANNEL rows, GROUP
 * rows*ceil(cols/group_size).  accumulate = 1 folds into the existing min/max (running
 * observer), 0 overwrites. */
llmc_status llmc_observer_minmax(llmc_ctx* ctx, const void* x, int32_t dtype, int64_t rows, int64_t cols, int64_t ld,
                                 int32_t strategy, int64_t group_size, float* min_io, float* max_io, int32_t accumulate);

/* Per-tensor llmc_observer_minmax that allocates no device memory when called.  It has no
 * counterpart in the reference: it serves callers that may not allocate or free device
 * memory mid-run (an activation hook on a model's stream, where cudaFree's device-wide wait
 * would stall the forward; a host whose caching allocator owns a fixed memory budget).
 * Its row buffer is a fixed array in the library, so rows <= LLMC_NOALLOC_MINMAX_MAX_ROWS
 * (larger: LLMC_ERR_SHAPE, nothing launched).  The first call on a device looks up that
 * array's address; make it before any stream capture.  llmc_init drops the looked-up address
 * of its device, so after a device reset create a new context before calling again.  All
 * calls on a device share the array, so calls that can overlap (two streams, two threads)
 * race: order them on one stream.  The calling thread's current device is the same after the
 * call as before it.  Arguments as llmc_observer_minmax with strategy TENSOR; output count 1. */
#define LLMC_NOALLOC_MINMAX_MAX_ROWS 65536
llmc_status llmc_observer_minmax_tensor_noalloc(llmc_ctx* ctx, const void* x, int32_t dtype, int64_t rows,
                                                int64_t cols, int64_t ld, float* min_io, float* max_io,
                                                int32_t accumulate);
/* Observer.ComputeAffineParams (Observer.cs:47-75), element-wise over count pairs. */
llmc_status llmc_affine_params(llmc_ctx* ctx, const float* mins, const float* maxs, int64_t count, int32_t num_bits,
                               int32_t symmetric, float* scale_out, int32_t* zp_out);

/* ---- fake quantisation / RTN / packing -------------------------------------------------
 * FakeQuantize.Apply (FakeQuantize.cs:22-38 -> FakeQuantizeFunction.cs:30-47) with scalar
 * parameters, computed in x's dtype op by op; out (optional) has x's dtype.  codes_out
 * (optional, int32) receives the clamped integer q = clamp(round(x/s)+zp) of the same chain
 * (Int4PackedTensor.FromFloat, Int4PackedTensor.cs:79-100, before the zero-point shift). */
llmc_status llmc_fake_quantize(llmc_ctx* ctx, const void* x, int32_t dtype, int64_t count, float scale, int32_t zp,
                               int32_t num_bits, int32_t symmetric, void* out, int32_t* codes_out);
/* MSEObserver.GetQuantParams (MSEObserver.cs:50-93) over `count` elements of x: absMax = max|x|;
 * for i = 1..grid_points the symmetric range +-absMax*i/grid_points gives (scale, zp) through
 * ComputeAffineParams, and mse_i = mean((x - FQ(x))^2) with the FakeQuantize op chain in x's dtype;
 * the first minimum wins (absMax == 0: scale 1, zp 0).  scale_out, zp_out and mse_out (optional,
 * [grid_points], NaN for a skipped candidate) are HOST pointers; synchronises the stream.
 * grid_points < 2 -> OUT_OF_RANGE; count == 0 -> NO_SAMPLES. */
llmc_status llmc_observer_mse(llmc_ctx* ctx, const void* x, int32_t dtype, int64_t count, int32_t grid_points,
                              int32_t num_bits, int32_t symmetric, float* scale_out, int32_t* zp_out, double* mse_out);
/* RtnModifier.OnEndCore (RtnModifier.cs:44-122) for one weight [m,n]: observer -> params ->
 * fake-quant, one pass over W for CHANNEL/GROUP (TENSOR adds one reduction pass).  Outputs as
 * llmc_gptq_quantize; deq_out (optional) has W's dtype like the reference's result. */
llmc_status llmc_rtn_quantize(llmc_ctx* ctx, const void* W, int32_t dtype, int64_t m, int64_t n, int64_t ldw,
                              const llmc_qconfig* cfg, uint8_t* codes_out, float* scales_out, int32_t* zps_out,
                              void* deq_out);
/* Int4PackedTensor.PackedBytes / FromPackedBytes+Dequantize (Int4PackedTensor.cs:47-161) over
 * a flat vector with one (scale, zero-point): pack stores (q - zp) & 0xF, even index high. */
llmc_status llmc_int4_pack(llmc_ctx* ctx, const int32_t* q, int64_t count, int32_t zero_point, uint8_t* packed);
llmc_status llmc_int4_unpack_dequant(llmc_ctx* ctx, const uint8_t* packed, int64_t count, float scale,
                                     int32_t zero_point, int32_t symmetric, float* out);

/* ---- compressed-tensors "pack-quantized" words --------------------------------------------
 * SafetensorsWriter.cs:25-35 writes dense fp32 weights only; the checkpoint the reference's
 * documentation names (docs/llm-compressor/deployment.md:124-132) is compressed-tensors'
 * pack-quantized layout.  From one weight's codes as the GPTQ / RTN entry points write them
 * ((q - zp) & 0xF nibbles, even column high, for num_bits <= 4; the byte q otherwise; crow bytes
 * per row) and its int32 zero-points (one per scale entry of `strategy`):
 *   packed_out [m, ldp] int32: q' + 2^(bits-1) in bits-wide fields, first column in the low
 *     bits, q' = q (symmetric) or q - 2^(bits-1) (asymmetric), last word zero-padded;
 *   zp_packed_out (optional; asymmetric channel / group only) [ceil(m / (32 / bits)), G] int32:
 *     zp packed the same way along the rows.
 * num_bits must divide 32. */
llmc_status llmc_pack_compressed_tensors(llmc_ctx* ctx, const uint8_t* codes, int64_t m, int64_t n, int64_t crow,
                                         const int32_t* zps, int32_t strategy, int64_t group_size, int32_t num_bits,
                                         int32_t symmetric, int32_t* packed_out, int64_t ldp, int32_t* zp_packed_out);

/* ---- per-token activation quantisation (extension) -------------------------------------------
 * No reference counterpart: QuantizationStrategy.PerToken exists (QuantizationStrategy.cs:9-19)
 * but RtnModifier.cs:69-70 rejects it for weights and the reference has no activation quantiser.
 * Dynamic W8A8-style quantisation of activations x [rows = tokens, cols = hidden] (row stride ld):
 * one min-max observer per token row (PerChannelMinMaxObserver.cs:38-76 on axis 0; NaN propagates
 * to the row's parameters), Observer.ComputeAffineParams (Observer.cs:47-75), and the
 * FakeQuantizeFunction op chain in x's dtype (FakeQuantizeFunction.cs:39-44).
 *   codes_out (optional) [rows, ldc] bytes: q = clamp(round(x / s) + zp), two's complement for a
 *     symmetric grid (int8 view), unsigned for an asymmetric one; a NaN element's code is 0;
 *   scales_out [rows] fp32; zps_out (optional) [rows] int32;
 *   deq_out (optional) [rows, ldd] in x's dtype: the fake-quantised activations.
 * num_bits in [2, 8]. */
llmc_status llmc_act_quant_per_token(llmc_ctx* ctx, const void* x, int32_t dtype, int64_t rows, int64_t cols, int64_t ld,
                                     int32_t num_bits, int32_t symmetric, uint8_t* codes_out, int64_t ldc,
                                     float* scales_out, int32_t* zps_out, void* deq_out, int64_t ldd);

/* ---- SmoothQuant / AWQ ------------------------------------------------------------------
 * UpdateActivationMax (SmoothQuantModifier.cs:71-115): running_max[cols] = max(running_max,
 * max_rows |x|) (accumulate = 0 overwrites). */
llmc_status llmc_act_absmax(llmc_ctx* ctx, const void* x, int32_t dtype, int64_t rows, int64_t cols, int64_t ld,
                            float* running_max, int32_t accumulate);
/* ApplyMapping (SmoothQuantModifier.cs:117-182): wmax = |balance|.amax(0); s_i = max(max(a_i,1e-5)^alpha /
 * max(wmax_i,1e-5)^(1-alpha), 1e-5); smooth /= s, balance *= s, in the weights' dtype.
 * s_out (optional, fp32 [hidden]). */
llmc_status llmc_smooth_apply(llmc_ctx* ctx, const float* act_max, void* smooth_w, int32_t smooth_dtype,
                              void* balance_w, int32_t balance_dtype, int64_t m, int64_t hidden, float alpha,
                              float* s_out);
/* The apply step alone with a given s (AWQ's chosen scale, algorithm-mapping.md:243-248):
 * smooth /= s (skipped when smooth_w is NULL), balance *= s, s rounded to the smooth dtype. */
llmc_status llmc_scale_apply(llmc_ctx* ctx, const float* s, void* smooth_w, int32_t smooth_dtype, void* balance_w,
                             int32_t balance_dtype, int64_t m, int64_t hidden);
/* AWQ grid search (docs/llmcompressorsharp/algorithm-mapping.md:214-249): for k=1..n_grid,
 * s = act_max^(k/n) / wmax^(1-k/n) (>= 1e-4), mse_k = mean((FQ(W*s)/s - W)^2) with FQ the RTN
 * of cfg.  Writes the best s (fp32 [n]) and mse per grid point (fp64 [n_grid]) on the device;
 * best_k (1-based) is read back to the host, which synchronises the stream.  With best_k NULL
 * nothing is read back and the call only enqueues work (extension: the reference's search
 * returns the chosen point; a caller that applies best_s on the device does not need it). */
llmc_status llmc_awq_search(llmc_ctx* ctx, const void* W, int32_t dtype, int64_t m, int64_t n, int64_t ldw,
                            const float* act_max, int32_t n_grid, const llmc_qconfig* cfg, float* best_s,
                            double* mse_out, int32_t* best_k);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* LLMC_B200_H */
