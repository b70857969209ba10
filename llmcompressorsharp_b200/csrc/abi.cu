// extern "C" entry points of libllmc_b200 (declared in include/llmc_b200.h).
//
// Argument validation mirrors the reference's exceptions (listed per entry point in the
// header); each maps to an llmc_status and a thread-local message.
#include "ops.h"

#include <nvtx3/nvToolsExt.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

namespace llmc {

static thread_local std::string g_err;

void set_error(const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
}

llmc_status fail(llmc_status st, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return st;
}

NvtxScope::NvtxScope(const char* name) { nvtxRangePushA(name); }
NvtxScope::~NvtxScope() { nvtxRangePop(); }

namespace {

struct Fault {
    std::string fn;
    llmc_status status;
    long long nth;  // 0: every call
    std::atomic<long long> calls{0};
};

std::vector<Fault*>& faults() {
    static std::vector<Fault*> list;
    static std::once_flag once;
    std::call_once(once, [] {
        const char* env = std::getenv("LLMC_FAULT");
        if (!env) return;
        std::string spec(env);
        size_t pos = 0;
        while (pos <= spec.size()) {
            size_t end = spec.find(',', pos);
            if (end == std::string::npos) end = spec.size();
            std::string item = spec.substr(pos, end - pos);
            pos = end + 1;
            size_t c1 = item.find(':');
            if (c1 == std::string::npos || c1 == 0) continue;
            size_t c2 = item.find(':', c1 + 1);
            const long st = std::strtol(item.substr(c1 + 1, c2 == std::string::npos ? std::string::npos : c2 - c1 - 1).c_str(),
                                        nullptr, 10);
            const long long k = c2 == std::string::npos ? 0 : std::strtoll(item.substr(c2 + 1).c_str(), nullptr, 10);
            if (st <= 0 || st > LLMC_ERR_OUT_OF_RANGE || k < 0) continue;
            Fault* f = new Fault();
            f->fn = item.substr(0, c1);
            f->status = (llmc_status)st;
            f->nth = k;
            list.push_back(f);
        }
    });
    return list;
}

}  // namespace

llmc_status injected_fault(const char* fn) {
    for (Fault* f : faults()) {
        if (f->fn != fn) continue;
        const long long n = ++f->calls;
        if (f->nth == 0 || n == f->nth) return fail(f->status, "injected fault in %s (call %lld)", fn, n);
    }
    return LLMC_OK;
}

// Synchronises the stream and reports the device error words, clearing them: word 2, a bounded
// device wait that gave up (written by the tensor-core kernels), as LLMC_ERR_TIMEOUT; word 3, a
// Hessian that was not positive definite in a factorisation run with deferred errors, as
// LLMC_ERR_NOT_PD.
llmc_status device_error_check(llmc_ctx* ctx) {
    LLMC_CUDA_TRY(cudaMemcpyAsync(ctx->hflags + 2, ctx->dflags + 2, 2 * sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
    LLMC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    const int timeout = ctx->hflags[2], not_pd = ctx->hflags[3];
    if (timeout || not_pd) {
        ctx->hflags[2] = ctx->hflags[3] = 0;
        LLMC_CUDA_TRY(cudaMemsetAsync(ctx->dflags + 2, 0, 2 * sizeof(int), ctx->stream));
    }
    if (timeout)
        return fail(LLMC_ERR_TIMEOUT, "a bounded wait inside a tensor-core kernel gave up; results of the "
                    "affected calls are incomplete");
    if (not_pd)
        return fail(LLMC_ERR_NOT_PD, "a damped Hessian factorised with deferred errors was not positive definite "
                    "(its factor was written as zeros); the pseudo-inverse fallback runs on the synchronous "
                    "path: factor it again with deferred errors off");
    return LLMC_OK;
}

static llmc_status grow(llmc_ctx* ctx, void** buf, size_t* cap, size_t bytes, void** out) {
    if (bytes > *cap) {
        if (*buf) {
            // The old block may still be in use by queued work on this stream.
            LLMC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
            LLMC_CUDA_TRY(cudaFree(*buf));
            *buf = nullptr;
            *cap = 0;
        }
        size_t want = align_up(bytes, (size_t)1 << 20);
        cudaError_t e = cudaMalloc(buf, want);
        if (e != cudaSuccess) {
            *buf = nullptr;
            return fail(LLMC_ERR_CUDA, "workspace allocation of %zu bytes failed: %s", want, cudaGetErrorString(e));
        }
        *cap = want;
    }
    *out = *buf;
    return LLMC_OK;
}

llmc_status workspace(llmc_ctx* ctx, size_t bytes, void** out) { return grow(ctx, &ctx->ws, &ctx->ws_bytes, bytes, out); }
llmc_status workspace2(llmc_ctx* ctx, size_t bytes, void** out) {
    return grow(ctx, &ctx->ws2, &ctx->ws2_bytes, bytes, out);
}

// Internal launchers implemented in the kernel translation units.
llmc_status rtn(llmc_ctx*, const void*, int, int64_t, int64_t, int64_t, const llmc_qconfig*, uint8_t*, float*, int32_t*,
                void*, float*);
llmc_status fake_quant_flat(llmc_ctx*, const void*, int, int64_t, float, int, int, int, void*, int32_t*);
llmc_status int4_pack(llmc_ctx*, const int32_t*, int64_t, int, uint8_t*);
llmc_status int4_unpack(llmc_ctx*, const uint8_t*, int64_t, float, int, float*);
llmc_status gptq(llmc_ctx*, const void*, int, int64_t, int64_t, int64_t, const float*, int64_t, const llmc_qconfig*,
                 float*, int64_t, uint8_t*, float*, int32_t*, int, uint8_t*);
llmc_status gptq_batch(llmc_ctx*, int, const void* const*, const int64_t*, const int64_t*, int, int64_t, const float*,
                       int64_t, const llmc_qconfig*, float*, int64_t, uint8_t*, float*, int32_t*, int, uint8_t*,
                       const int32_t*);
llmc_status col_absmax(llmc_ctx*, const void*, int, int64_t, int64_t, int64_t, float*, int);
llmc_status smooth_apply(llmc_ctx*, const float*, void*, int, void*, int, int64_t, int64_t, float, float*);
llmc_status scale_apply(llmc_ctx*, const float*, void*, int, void*, int, int64_t, int64_t);
llmc_status awq_search(llmc_ctx*, const void*, int, int64_t, int64_t, int64_t, const float*, int, const llmc_qconfig*,
                       float*, double*, int32_t*);
size_t minmax_scratch_floats(int strategy, int64_t rows);

static llmc_status check_bits(int bits) {
    if (bits < 2 || bits > 16) return fail(LLMC_ERR_OUT_OF_RANGE, "numBits must be between 2 and 16 inclusive (got %d).", bits);
    return LLMC_OK;
}

static llmc_status check_qconfig(const llmc_qconfig* c, int for_gptq) {
    if (!c) return fail(LLMC_ERR_INVALID_ARG, "config must not be null");
    LLMC_TRY(check_bits(c->num_bits));
    if (for_gptq && c->act_order)
        return fail(LLMC_ERR_UNSUPPORTED,
                    "GPTQConfig.ActOrder=true is not yet implemented. Column reordering by Hessian diagonal is deferred.");
    if (c->strategy == LLMC_STRATEGY_TOKEN)
        return fail(LLMC_ERR_UNSUPPORTED, "PerToken strategy applies to activations, not weights.");
    if (c->strategy != LLMC_STRATEGY_TENSOR && c->strategy != LLMC_STRATEGY_CHANNEL && c->strategy != LLMC_STRATEGY_GROUP)
        return fail(LLMC_ERR_UNSUPPORTED, "Quantization strategy %d is not supported.", c->strategy);
    if (c->strategy == LLMC_STRATEGY_CHANNEL && c->channel_axis != 0)
        return fail(LLMC_ERR_UNSUPPORTED, "per-channel quantisation of a 2-D weight uses channel axis 0");
    if (c->strategy == LLMC_STRATEGY_GROUP && c->group_size <= 0)
        return fail(LLMC_ERR_INVALID_ARG, "group_size must be positive for the group strategy");
    return LLMC_OK;
}

}  // namespace llmc

using namespace llmc;

#define CTX_CHECK(ctx)                                                                        \
    do {                                                                                      \
        if (!(ctx)) return fail(LLMC_ERR_INVALID_ARG, "context must not be null");            \
        cudaError_t _e = cudaSetDevice((ctx)->device);                                        \
        if (_e != cudaSuccess) return fail(LLMC_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(_e)); \
    } while (0)

#define NULL_CHECK(p, name) \
    do { if (!(p)) return fail(LLMC_ERR_INVALID_ARG, "%s must not be null", name); } while (0)

extern "C" {

const char* llmc_last_error(void) { return g_err.c_str(); }
int32_t llmc_abi_version(void) { return LLMC_ABI_VERSION; }

llmc_status llmc_init(int32_t device, llmc_ctx** out) {
    LLMC_ENTRY();
    NULL_CHECK(out, "out");
    *out = nullptr;
    int n = 0;
    LLMC_CUDA_TRY(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return fail(LLMC_ERR_INVALID_ARG, "device %d out of range (have %d)", device, n);
    LLMC_CUDA_TRY(cudaSetDevice(device));
    cudaDeviceProp prop;
    LLMC_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) return fail(LLMC_ERR_UNSUPPORTED, "this library is built for sm_100a (B200); device is sm_%d%d",
                                      prop.major, prop.minor);
    llmc_ctx* c = new (std::nothrow) llmc_ctx();
    if (!c) return fail(LLMC_ERR_INTERNAL, "out of host memory");
    c->device = device;
    c->sm_count = prop.multiProcessorCount;
    cudaError_t e = cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&c->dflags, 16 * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(c->dflags, 0, 16 * sizeof(int));
    if (e == cudaSuccess) e = cudaMallocHost(&c->hflags, 16 * sizeof(int));
    if (e != cudaSuccess) {
        if (c->own_stream) cudaStreamDestroy(c->own_stream);
        if (c->dflags) cudaFree(c->dflags);
        delete c;
        return fail(LLMC_ERR_CUDA, "context setup failed: %s", cudaGetErrorString(e));
    }
    c->stream = c->own_stream;
    noalloc_forget(device);
    *out = c;
    return LLMC_OK;
}

llmc_status llmc_destroy(llmc_ctx* ctx) {
    LLMC_ENTRY();
    if (!ctx) return LLMC_OK;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->ws) cudaFree(ctx->ws);
    if (ctx->ws2) cudaFree(ctx->ws2);
    if (ctx->dflags) cudaFree(ctx->dflags);
    if (ctx->hflags) cudaFreeHost(ctx->hflags);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return LLMC_OK;
}

llmc_status llmc_set_stream(llmc_ctx* ctx, void* stream) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    ctx->stream = stream ? (cudaStream_t)stream : ctx->own_stream;
    return LLMC_OK;
}

llmc_status llmc_set_sm_limit(llmc_ctx* ctx, int32_t sms) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    if (sms < 0) return fail(LLMC_ERR_INVALID_ARG, "sm limit must be >= 0 (0 = no limit)");
    ctx->sm_limit = sms;
    return LLMC_OK;
}

llmc_status llmc_set_wait_limit(llmc_ctx* ctx, int64_t tries) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    if (tries > (int64_t)UINT32_MAX) return fail(LLMC_ERR_OUT_OF_RANGE, "wait limit above 2^32 - 1");
    ctx->wait_limit = tries < 0 ? (uint32_t)(1u << 26) : (uint32_t)tries;
    return LLMC_OK;
}

llmc_status llmc_set_deferred_errors(llmc_ctx* ctx, int32_t on) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    ctx->deferred_errors = on ? 1 : 0;
    return LLMC_OK;
}

llmc_status llmc_sync(llmc_ctx* ctx) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    return device_error_check(ctx);
}

llmc_status llmc_launch_count(llmc_ctx* ctx, int64_t* out) {
    LLMC_ENTRY();
    NULL_CHECK(ctx, "ctx");
    NULL_CHECK(out, "out");
    *out = ctx->launches;
    return LLMC_OK;
}

// ---- Hessian ------------------------------------------------------------------------------
llmc_status llmc_hessian_create(llmc_ctx* ctx, int64_t in_features, llmc_hessian** out) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(out, "out");
    *out = nullptr;
    if (in_features <= 0) return fail(LLMC_ERR_OUT_OF_RANGE, "inFeatures must be positive (got %lld).", (long long)in_features);
    llmc_hessian* h = new (std::nothrow) llmc_hessian();
    if (!h) return fail(LLMC_ERR_INTERNAL, "out of host memory");
    h->ctx = ctx;
    h->d = in_features;
    const size_t bytes = (size_t)in_features * in_features * sizeof(float);
    cudaError_t e = cudaMalloc(&h->h, bytes);
    if (e == cudaSuccess) e = cudaMemsetAsync(h->h, 0, bytes, ctx->stream);
    if (e != cudaSuccess) {
        if (h->h) cudaFree(h->h);
        delete h;
        return fail(LLMC_ERR_CUDA, "Hessian allocation (%zu bytes): %s", bytes, cudaGetErrorString(e));
    }
    *out = h;
    return LLMC_OK;
}

llmc_status llmc_hessian_update(llmc_hessian* h, const void* x, int32_t dtype, int64_t rows, int64_t ld) {
    LLMC_ENTRY();
    NULL_CHECK(h, "hessian");
    llmc_ctx* ctx = h->ctx;
    CTX_CHECK(ctx);
    NULL_CHECK(x, "x");
    if (!dtype_ok(dtype)) return fail(LLMC_ERR_INVALID_ARG, "unsupported dtype %d", dtype);
    if (rows < 0) return fail(LLMC_ERR_SHAPE, "rows must be non-negative");
    if (ld < h->d)
        return fail(LLMC_ERR_SHAPE, "Input last dim (ld=%lld) must equal inFeatures (%lld).", (long long)ld, (long long)h->d);
    if (rows > 0) {
        llmc_status st = LLMC_ERR_UNSUPPORTED;
        if (dtype != LLMC_DTYPE_F32) st = syrk_tc(ctx, x, dtype, rows, h->d, ld, h->h, h->d);
        if (dtype == LLMC_DTYPE_F32 && h->d >= 512 && rows >= 1024) {
            // fp32 input: 3xTF32 on the tensor cores (hi/lo split of X once, CTA pairs on 256 x 256
            // upper tiles), the token range split so that the units fill the pairs, with at least
            // 1024 tokens per split.
            const int64_t t = (h->d + 255) / 256;
            const int64_t upper = t * (t + 1) / 2;
            int64_t split = ((int64_t)persistent_sms(ctx) / 2 + upper - 1) / upper;
            if (split > rows / 1024) split = rows / 1024;
            if (split < 1) split = 1;
            GemmArgs g{h->d, h->d, rows, x, ld, 1, dtype, x, ld, 0, dtype, h->h, h->d, 1.f, 1.f};
            g.c_mode = 2;
            g.split_k = (int)split;
            st = gemm_tc(ctx, g);
        }
        if (st == LLMC_ERR_UNSUPPORTED) {
            // fp32 input (or a shape outside the tensor-core kernel's contract): fp32 SIMT.
            const int64_t tiles = (h->d + 127) / 128;
            const int64_t upper = tiles * (tiles + 1) / 2;
            int64_t split = (2 * (int64_t)ctx->sm_count + upper - 1) / upper;
            const int64_t max_split = (rows + 1023) / 1024;
            if (split > max_split) split = max_split;
            // Each split sums <= 2048 products sequentially in fp32 before one atomic add,
            // which keeps the accumulated rounding near the oracle's blocked sgemm.
            const int64_t min_split = (rows + 2047) / 2048;
            if (split < min_split) split = min_split;
            if (split < 1) split = 1;
            GemmArgs g{h->d, h->d, rows, x, ld, 1, dtype, x, ld, 0, dtype, h->h, h->d, 1.f, 1.f};
            g.c_mode = 2;
            g.split_k = (int)split;
            st = gemm_f32(ctx, g);
        }
        if (st != LLMC_OK) return st;
    }
    h->samples += rows;
    return LLMC_OK;
}

llmc_status llmc_hessian_get(llmc_hessian* h, float* out) {
    LLMC_ENTRY();
    NULL_CHECK(h, "hessian");
    CTX_CHECK(h->ctx);
    NULL_CHECK(out, "out");
    LLMC_TRY(device_error_check(h->ctx));
    return symmetrize_from_upper(h->ctx, h->h, h->d, h->d, out, h->d);
}

llmc_status llmc_hessian_data(llmc_hessian* h, float** out) {
    LLMC_ENTRY();
    NULL_CHECK(h, "hessian");
    NULL_CHECK(out, "out");
    *out = h->h;
    return LLMC_OK;
}

llmc_status llmc_hessian_reset(llmc_hessian* h) {
    LLMC_ENTRY();
    NULL_CHECK(h, "hessian");
    CTX_CHECK(h->ctx);
    LLMC_CUDA_TRY(cudaMemsetAsync(h->h, 0, (size_t)h->d * h->d * sizeof(float), h->ctx->stream));
    h->samples = 0;
    return LLMC_OK;
}

llmc_status llmc_hessian_sample_count(llmc_hessian* h, int64_t* out) {
    LLMC_ENTRY();
    NULL_CHECK(h, "hessian");
    NULL_CHECK(out, "out");
    *out = h->samples;
    return LLMC_OK;
}

llmc_status llmc_hessian_add_samples(llmc_hessian* h, int64_t rows) {
    LLMC_ENTRY();
    NULL_CHECK(h, "hessian");
    h->samples += rows;
    return LLMC_OK;
}

llmc_status llmc_hessian_destroy(llmc_hessian* h) {
    LLMC_ENTRY();
    if (!h) return LLMC_OK;
    cudaSetDevice(h->ctx->device);
    cudaStreamSynchronize(h->ctx->stream);
    cudaFree(h->h);
    delete h;
    return LLMC_OK;
}

// ---- inverse ----------------------------------------------------------------------------------
llmc_status llmc_chol_inverse(llmc_ctx* ctx, const float* H, int64_t d, int64_t ldh, float damp, int32_t upper_only,
                              float* out, int64_t ldo, int32_t want_upper) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(H, "hessian");
    NULL_CHECK(out, "out");
    if (d <= 0 || ldh < d || ldo < d) return fail(LLMC_ERR_SHAPE, "Hessian must be a square 2-D tensor (d=%lld).", (long long)d);
    return chol_inverse(ctx, H, d, ldh, damp, upper_only, out, ldo, want_upper);
}

llmc_status llmc_upper_factor(llmc_ctx* ctx, const float* hinv, int64_t d, int64_t ldh, float* out, int64_t ldo) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(hinv, "hinv");
    NULL_CHECK(out, "out");
    if (d <= 0 || ldh < d || ldo < d) return fail(LLMC_ERR_SHAPE, "Hinv must be square (d=%lld).", (long long)d);
    return upper_factor(ctx, hinv, d, ldh, out, ldo);
}

// ---- GPTQ / SparseGPT ------------------------------------------------------------------------
llmc_status llmc_gptq_quantize(llmc_ctx* ctx, const void* W, int32_t dtype, int64_t m, int64_t n, int64_t ldw,
                               const float* U, int64_t ldu, const llmc_qconfig* cfg, float* wq_out, int64_t ldq,
                               uint8_t* codes_out, float* scales_out, int32_t* zps_out) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(W, "weight");
    NULL_CHECK(U, "hinv");
    LLMC_TRY(check_qconfig(cfg, 1));
    if (!dtype_ok(dtype)) return fail(LLMC_ERR_INVALID_ARG, "unsupported dtype %d", dtype);
    if (m <= 0 || n <= 0 || ldw < n || ldu < n) return fail(LLMC_ERR_SHAPE, "bad weight/U shape");
    if (wq_out && ldq < n) return fail(LLMC_ERR_SHAPE, "ldq < n");
    if (codes_out && cfg->num_bits > 8) return fail(LLMC_ERR_UNSUPPORTED, "integer codes are produced for num_bits <= 8");
    if (codes_out && cfg->num_bits <= 4 && cfg->strategy == LLMC_STRATEGY_GROUP && (cfg->group_size % 2))
        return fail(LLMC_ERR_UNSUPPORTED, "packed int4 codes need an even group size");
    return gptq(ctx, W, dtype, m, n, ldw, U, ldu, cfg, wq_out, ldq, codes_out, scales_out, zps_out, 0, nullptr);
}

llmc_status llmc_gptq_quantize_batch(llmc_ctx* ctx, int32_t count, const void* const* W, const int64_t* m,
                                     const int64_t* ldw, int32_t dtype, int64_t n, const float* U, int64_t ldu,
                                     const llmc_qconfig* cfg, float* wq_out, int64_t ldq, uint8_t* codes_out,
                                     float* scales_out, int32_t* zps_out) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(W, "weights");
    NULL_CHECK(m, "m");
    NULL_CHECK(ldw, "ldw");
    NULL_CHECK(U, "hinv");
    LLMC_TRY(check_qconfig(cfg, 1));
    if (count < 1 || count > 64) return fail(LLMC_ERR_INVALID_ARG, "count must be in [1, 64]");
    if (!dtype_ok(dtype)) return fail(LLMC_ERR_INVALID_ARG, "unsupported dtype %d", dtype);
    if (n <= 0 || ldu < n) return fail(LLMC_ERR_SHAPE, "bad U shape");
    for (int k = 0; k < count; k++) {
        NULL_CHECK(W[k], "weight");
        if (m[k] <= 0 || ldw[k] < n) return fail(LLMC_ERR_SHAPE, "bad shape of weight %d", k);
    }
    if (wq_out && ldq < n) return fail(LLMC_ERR_SHAPE, "ldq < n");
    if (codes_out && cfg->num_bits > 8) return fail(LLMC_ERR_UNSUPPORTED, "integer codes are produced for num_bits <= 8");
    if (codes_out && cfg->num_bits <= 4 && cfg->strategy == LLMC_STRATEGY_GROUP && (cfg->group_size % 2))
        return fail(LLMC_ERR_UNSUPPORTED, "packed int4 codes need an even group size");
    return gptq_batch(ctx, count, W, m, ldw, dtype, n, U, ldu, cfg, wq_out, ldq, codes_out, scales_out, zps_out, 0,
                      nullptr, nullptr);
}

// ---- GPTQ activation order (extension) ---------------------------------------------------------
llmc_status llmc_gptq_act_order_perm(llmc_ctx* ctx, const float* H, int64_t d, int64_t ldh, int32_t* perm_out) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(H, "hessian");
    NULL_CHECK(perm_out, "perm_out");
    if (d <= 0 || ldh < d || d > (int64_t)INT32_MAX)
        return fail(LLMC_ERR_SHAPE, "Hessian must be a square 2-D tensor (d=%lld).", (long long)d);
    return act_order_perm(ctx, H, d, ldh, perm_out);
}

llmc_status llmc_permute_hessian(llmc_ctx* ctx, const float* H, int64_t d, int64_t ldh, int32_t upper_only,
                                 const int32_t* perm, float* out, int64_t ldo) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(H, "hessian");
    NULL_CHECK(perm, "perm");
    NULL_CHECK(out, "out");
    if (d <= 0 || ldh < d || ldo < d) return fail(LLMC_ERR_SHAPE, "Hessian must be a square 2-D tensor (d=%lld).", (long long)d);
    if (out == H) return fail(LLMC_ERR_INVALID_ARG, "out must not alias the Hessian");
    return permute_hessian(ctx, H, d, ldh, upper_only, perm, out, ldo);
}

llmc_status llmc_gptq_quantize_batch_perm(llmc_ctx* ctx, int32_t count, const void* const* W, const int64_t* m,
                                          const int64_t* ldw, int32_t dtype, int64_t n, const float* U, int64_t ldu,
                                          const int32_t* perm, const llmc_qconfig* cfg, float* wq_out, int64_t ldq,
                                          uint8_t* codes_out, float* scales_out, int32_t* zps_out) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(W, "weights");
    NULL_CHECK(m, "m");
    NULL_CHECK(ldw, "ldw");
    NULL_CHECK(U, "hinv");
    NULL_CHECK(perm, "perm");
    LLMC_TRY(check_qconfig(cfg, 0));
    if (count < 1 || count > 64) return fail(LLMC_ERR_INVALID_ARG, "count must be in [1, 64]");
    if (!dtype_ok(dtype)) return fail(LLMC_ERR_INVALID_ARG, "unsupported dtype %d", dtype);
    if (n <= 0 || ldu < n || n > (int64_t)INT32_MAX) return fail(LLMC_ERR_SHAPE, "bad U shape");
    for (int k = 0; k < count; k++) {
        NULL_CHECK(W[k], "weight");
        if (m[k] <= 0 || ldw[k] < n) return fail(LLMC_ERR_SHAPE, "bad shape of weight %d", k);
    }
    if (wq_out && ldq < n) return fail(LLMC_ERR_SHAPE, "ldq < n");
    if (codes_out && cfg->num_bits > 8) return fail(LLMC_ERR_UNSUPPORTED, "integer codes are produced for num_bits <= 8");
    return gptq_batch(ctx, count, W, m, ldw, dtype, n, U, ldu, cfg, wq_out, ldq, codes_out, scales_out, zps_out, 0,
                      nullptr, perm);
}

llmc_status llmc_sparsegpt_prune(llmc_ctx* ctx, const void* W, int32_t dtype, int64_t m, int64_t n, int64_t ldw,
                                 const float* U, int64_t ldu, const llmc_qconfig* cfg, float* out, int64_t ldo,
                                 uint8_t* mask_out) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(W, "weight");
    NULL_CHECK(U, "hinv");
    NULL_CHECK(cfg, "config");
    NULL_CHECK(out, "out");
    if (!dtype_ok(dtype)) return fail(LLMC_ERR_INVALID_ARG, "unsupported dtype %d", dtype);
    if (m <= 0 || n <= 0 || ldw < n || ldu < n || ldo < n) return fail(LLMC_ERR_SHAPE, "bad weight/U shape");
    if (cfg->mask_m > 0 && (cfg->mask_n < 0 || cfg->mask_n > cfg->mask_m || cfg->mask_m > 128))
        return fail(LLMC_ERR_INVALID_ARG, "bad N:M mask (%d:%d)", cfg->mask_n, cfg->mask_m);
    if (cfg->mask_m <= 0 && !(cfg->sparsity >= 0.f && cfg->sparsity < 1.f))
        return fail(LLMC_ERR_OUT_OF_RANGE, "sparsity must be in [0, 1)");
    llmc_qconfig c = *cfg;
    if (c.mask_m > 0 && (c.block_size % c.mask_m) && c.block_size < 128)
        return fail(LLMC_ERR_INVALID_ARG, "block_size must be a multiple of the N:M group");
    return gptq(ctx, W, dtype, m, n, ldw, U, ldu, &c, out, ldo, nullptr, nullptr, nullptr, 1, mask_out);
}

// ---- observers ------------------------------------------------------------------------------
llmc_status llmc_observer_minmax(llmc_ctx* ctx, const void* x, int32_t dtype, int64_t rows, int64_t cols, int64_t ld,
                                 int32_t strategy, int64_t group_size, float* min_io, float* max_io, int32_t accumulate) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(x, "x");
    NULL_CHECK(min_io, "min");
    NULL_CHECK(max_io, "max");
    if (!dtype_ok(dtype)) return fail(LLMC_ERR_INVALID_ARG, "unsupported dtype %d", dtype);
    if (rows <= 0 || cols <= 0 || ld < cols) return fail(LLMC_ERR_SHAPE, "bad shape");
    if (strategy == LLMC_STRATEGY_GROUP && group_size <= 0) return fail(LLMC_ERR_INVALID_ARG, "group_size must be positive");
    if (strategy != LLMC_STRATEGY_TENSOR && strategy != LLMC_STRATEGY_CHANNEL && strategy != LLMC_STRATEGY_GROUP)
        return fail(LLMC_ERR_UNSUPPORTED, "strategy %d", strategy);
    float* scratch = nullptr;
    if (strategy == LLMC_STRATEGY_TENSOR) {
        void* w;
        LLMC_TRY(workspace(ctx, minmax_scratch_floats(strategy, rows) * sizeof(float), &w));
        scratch = (float*)w;
    }
    return minmax(ctx, x, dtype, rows, cols, ld, strategy, group_size, min_io, max_io, accumulate, scratch);
}

llmc_status llmc_affine_params(llmc_ctx* ctx, const float* mins, const float* maxs, int64_t count, int32_t num_bits,
                               int32_t symmetric, float* scale_out, int32_t* zp_out) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    LLMC_TRY(check_bits(num_bits));
    NULL_CHECK(mins, "mins");
    NULL_CHECK(maxs, "maxs");
    NULL_CHECK(scale_out, "scale_out");
    NULL_CHECK(zp_out, "zp_out");
    if (count <= 0) return LLMC_OK;
    return affine(ctx, mins, maxs, count, num_bits, symmetric, scale_out, zp_out);
}

// ---- fake quant / RTN / packing ---------------------------------------------------------------
llmc_status llmc_fake_quantize(llmc_ctx* ctx, const void* x, int32_t dtype, int64_t count, float scale, int32_t zp,
                               int32_t num_bits, int32_t symmetric, void* out, int32_t* codes_out) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(x, "x");
    if (!out && !codes_out) return fail(LLMC_ERR_INVALID_ARG, "out and codes_out must not both be null");
    LLMC_TRY(check_bits(num_bits));
    if (!dtype_ok(dtype)) return fail(LLMC_ERR_INVALID_ARG, "unsupported dtype %d", dtype);
    if (count <= 0) return LLMC_OK;
    return fake_quant_flat(ctx, x, dtype, count, scale, zp, num_bits, symmetric, out, codes_out);
}

llmc_status llmc_rtn_quantize(llmc_ctx* ctx, const void* W, int32_t dtype, int64_t m, int64_t n, int64_t ldw,
                              const llmc_qconfig* cfg, uint8_t* codes_out, float* scales_out, int32_t* zps_out,
                              void* deq_out) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(W, "weight");
    LLMC_TRY(check_qconfig(cfg, 0));
    NULL_CHECK(scales_out, "scales_out");
    NULL_CHECK(zps_out, "zps_out");
    if (!dtype_ok(dtype)) return fail(LLMC_ERR_INVALID_ARG, "unsupported dtype %d", dtype);
    if (m <= 0 || n <= 0 || ldw < n) return fail(LLMC_ERR_SHAPE, "bad weight shape");
    if (codes_out && cfg->num_bits > 8) return fail(LLMC_ERR_UNSUPPORTED, "integer codes are produced for num_bits <= 8");
    if (codes_out && cfg->num_bits <= 4 && cfg->strategy == LLMC_STRATEGY_GROUP && (cfg->group_size % 2))
        return fail(LLMC_ERR_UNSUPPORTED, "packed int4 codes need an even group size");
    float* scratch = nullptr;
    if (cfg->strategy == LLMC_STRATEGY_TENSOR) {
        void* w;
        LLMC_TRY(workspace(ctx, (minmax_scratch_floats(LLMC_STRATEGY_TENSOR, m) + 64) * sizeof(float), &w));
        scratch = (float*)w;
    }
    return rtn(ctx, W, dtype, m, n, ldw, cfg, codes_out, scales_out, zps_out, deq_out, scratch);
}

llmc_status llmc_int4_pack(llmc_ctx* ctx, const int32_t* q, int64_t count, int32_t zero_point, uint8_t* packed) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(q, "q");
    NULL_CHECK(packed, "packed");
    if (count <= 0) return LLMC_OK;
    return int4_pack(ctx, q, count, zero_point, packed);
}

llmc_status llmc_int4_unpack_dequant(llmc_ctx* ctx, const uint8_t* packed, int64_t count, float scale, int32_t zero_point,
                                     int32_t symmetric, float* out) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(packed, "packed");
    NULL_CHECK(out, "out");
    (void)zero_point;  // Dequantize() multiplies the stored (q - zp) value by the scale.
    if (count <= 0) return LLMC_OK;
    return int4_unpack(ctx, packed, count, scale, symmetric, out);
}

// ---- compressed-tensors packing ---------------------------------------------------------------------
llmc_status llmc_pack_compressed_tensors(llmc_ctx* ctx, const uint8_t* codes, int64_t m, int64_t n, int64_t crow,
                                         const int32_t* zps, int32_t strategy, int64_t group_size, int32_t num_bits,
                                         int32_t symmetric, int32_t* packed_out, int64_t ldp, int32_t* zp_packed_out) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(codes, "codes");
    NULL_CHECK(packed_out, "packed_out");
    LLMC_TRY(check_bits(num_bits));
    if (num_bits > 8) return fail(LLMC_ERR_UNSUPPORTED, "codes are produced for num_bits <= 8");
    if (32 % num_bits) return fail(LLMC_ERR_UNSUPPORTED, "pack-quantized needs 32 / num_bits fields per word");
    if (m <= 0 || n <= 0) return fail(LLMC_ERR_SHAPE, "bad weight shape");
    if (crow < (num_bits <= 4 ? (n + 1) / 2 : n)) return fail(LLMC_ERR_SHAPE, "crow shorter than a row of codes");
    const int64_t per = 32 / num_bits;
    if (ldp < (n + per - 1) / per) return fail(LLMC_ERR_SHAPE, "ldp shorter than a row of packed words");
    if (strategy != LLMC_STRATEGY_TENSOR && strategy != LLMC_STRATEGY_CHANNEL && strategy != LLMC_STRATEGY_GROUP)
        return fail(LLMC_ERR_UNSUPPORTED, "strategy %d", strategy);
    if (strategy == LLMC_STRATEGY_GROUP && group_size <= 0) return fail(LLMC_ERR_INVALID_ARG, "group_size must be positive");
    if (!symmetric && num_bits <= 4) NULL_CHECK(zps, "zero_points");
    if (zp_packed_out && (symmetric || strategy == LLMC_STRATEGY_TENSOR))
        return fail(LLMC_ERR_INVALID_ARG, "packed zero-points exist for asymmetric channel / group weights only");
    if (zp_packed_out) NULL_CHECK(zps, "zero_points");
    const int64_t gs = strategy == LLMC_STRATEGY_GROUP ? group_size : n;
    const int64_t zrow = strategy == LLMC_STRATEGY_TENSOR ? 0 : n_groups(strategy, n, gs);
    return ct_pack(ctx, codes, m, n, crow, zps, zrow, gs, num_bits, symmetric, packed_out, ldp, zp_packed_out);
}

// ---- per-token activation quantisation (extension) ------------------------------------------------
llmc_status llmc_act_quant_per_token(llmc_ctx* ctx, const void* x, int32_t dtype, int64_t rows, int64_t cols, int64_t ld,
                                     int32_t num_bits, int32_t symmetric, uint8_t* codes_out, int64_t ldc,
                                     float* scales_out, int32_t* zps_out, void* deq_out, int64_t ldd) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(x, "x");
    NULL_CHECK(scales_out, "scales_out");
    LLMC_TRY(check_bits(num_bits));
    if (num_bits > 8) return fail(LLMC_ERR_UNSUPPORTED, "per-token codes are bytes: num_bits must be <= 8");
    if (!dtype_ok(dtype)) return fail(LLMC_ERR_INVALID_ARG, "unsupported dtype %d", dtype);
    if (rows < 0 || cols <= 0 || ld < cols) return fail(LLMC_ERR_SHAPE, "bad activation shape");
    if (codes_out && ldc < cols) return fail(LLMC_ERR_SHAPE, "ldc < cols");
    if (deq_out && ldd < cols) return fail(LLMC_ERR_SHAPE, "ldd < cols");
    if (rows == 0) return LLMC_OK;
    return act_quant_per_token(ctx, x, dtype, rows, cols, ld, num_bits, symmetric, codes_out, ldc, scales_out, zps_out,
                               deq_out, ldd);
}

// ---- SmoothQuant / AWQ --------------------------------------------------------------------------
llmc_status llmc_act_absmax(llmc_ctx* ctx, const void* x, int32_t dtype, int64_t rows, int64_t cols, int64_t ld,
                            float* running_max, int32_t accumulate) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(x, "x");
    NULL_CHECK(running_max, "running_max");
    if (!dtype_ok(dtype)) return fail(LLMC_ERR_INVALID_ARG, "unsupported dtype %d", dtype);
    if (rows < 0 || cols <= 0 || ld < cols) return fail(LLMC_ERR_SHAPE, "bad activation shape");
    return col_absmax(ctx, x, dtype, rows, cols, ld, running_max, accumulate);
}

llmc_status llmc_smooth_apply(llmc_ctx* ctx, const float* act_max, void* smooth_w, int32_t smooth_dtype, void* balance_w,
                              int32_t balance_dtype, int64_t m, int64_t hidden, float alpha, float* s_out) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(act_max, "act_max");
    NULL_CHECK(smooth_w, "smooth weight");
    NULL_CHECK(balance_w, "balance weight");
    if (!(alpha >= 0.f && alpha <= 1.f)) return fail(LLMC_ERR_OUT_OF_RANGE, "SmoothingStrength (alpha) must be in [0, 1].");
    if (m <= 0 || hidden <= 0) return fail(LLMC_ERR_SHAPE, "bad balance weight shape");
    return smooth_apply(ctx, act_max, smooth_w, smooth_dtype, balance_w, balance_dtype, m, hidden, alpha, s_out);
}

llmc_status llmc_scale_apply(llmc_ctx* ctx, const float* s, void* smooth_w, int32_t smooth_dtype, void* balance_w,
                             int32_t balance_dtype, int64_t m, int64_t hidden) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(s, "s");
    NULL_CHECK(balance_w, "balance weight");
    if (m <= 0 || hidden <= 0) return fail(LLMC_ERR_SHAPE, "bad balance weight shape");
    return scale_apply(ctx, s, smooth_w, smooth_w ? smooth_dtype : balance_dtype, balance_w, balance_dtype, m, hidden);
}

llmc_status llmc_awq_search(llmc_ctx* ctx, const void* W, int32_t dtype, int64_t m, int64_t n, int64_t ldw,
                            const float* act_max, int32_t n_grid, const llmc_qconfig* cfg, float* best_s,
                            double* mse_out, int32_t* best_k) {
    LLMC_ENTRY();
    CTX_CHECK(ctx);
    NULL_CHECK(W, "weight");
    NULL_CHECK(act_max, "act_max");
    NULL_CHECK(best_s, "best_s");
    LLMC_TRY(check_qconfig(cfg, 0));
    if (cfg->strategy == LLMC_STRATEGY_TENSOR) return fail(LLMC_ERR_UNSUPPORTED, "AWQ search needs channel or group scales");
    if (n_grid < 1) return fail(LLMC_ERR_OUT_OF_RANGE, "n_grid must be >= 1");
    if (m <= 0 || n <= 0 || ldw < n) return fail(LLMC_ERR_SHAPE, "bad weight shape");
    return awq_search(ctx, W, dtype, m, n, ldw, act_max, n_grid, cfg, best_s, mse_out, best_k);
}

}  // extern "C"
