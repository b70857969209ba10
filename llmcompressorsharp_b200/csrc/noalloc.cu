// Per-tensor min/max observer that makes no device allocation when it is called.
//
// llmc_observer_minmax with the per-tensor strategy reduces in two levels: per-row minima
// and maxima go to a row buffer, then one more pass reduces that buffer.  The row buffer
// comes from the context's growable workspace, and growing it means cudaFree + cudaMalloc.
// cudaFree waits for the whole device, and cudaMalloc can fail when another allocator owns
// the memory.  Two kinds of caller cannot accept either:
//   * an activation hook that runs between two layers of a model on the model's stream,
//     where a device-wide wait stalls every other stream of the process mid-forward;
//   * a host whose device memory belongs to its own caching allocator under a fixed budget
//     (a .NET/TorchSharp process, for one), where a stray cudaMalloc can fail with
//     out-of-memory or split the pool.
// This variant keeps the row buffer in a fixed array in the library's device data instead,
// so a call only launches kernels.
//
// Limits and rules:
//   * rows <= LLMC_NOALLOC_MINMAX_MAX_ROWS (65536); larger inputs are rejected with
//     LLMC_ERR_SHAPE before anything is launched.  cols and ld are not limited.
//   * The first call on a device does set-up: it looks up the array's device address with
//     cudaGetSymbolAddress (which may load the module).  Make that first call before any
//     stream capture begins.  llmc_init forgets the looked-up address of its device, so a
//     host that resets the device (cudaDeviceReset, which unloads the module and may place
//     the array elsewhere) and then creates a new context gets a fresh lookup.
//   * The call makes its context's device current for its own work and gives the calling
//     thread its previous current device back before it returns.
//   * Every call on one device shares the one array.  Calls whose kernels can overlap
//     (different streams, or different host threads without ordering) race on it and give
//     wrong results; order them on one stream.
//   * Nothing in the array has to start at zero: the first pass writes every row slot that
//     the second pass reads, so the array is never cleared.
#include <mutex>

#include "ops.h"

namespace llmc {
namespace {

constexpr int64_t kMaxRows = LLMC_NOALLOC_MINMAX_MAX_ROWS;
constexpr int kMaxDevices = 64;

// 2 * kMaxRows + 64 floats (minmax_scratch_floats for the per-tensor strategy): 512.25 KiB.
__device__ __align__(256) float g_minmax_rows[2 * kMaxRows + 64];

std::mutex g_setup_mu;
float* g_rows_addr[kMaxDevices] = {};

// Device address of g_minmax_rows on `device` (which must be current), looked up once.
llmc_status rows_buffer(int device, float** out) {
    if (device < 0 || device >= kMaxDevices) return fail(LLMC_ERR_UNSUPPORTED, "device index %d too large", device);
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_rows_addr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_minmax_rows);
        if (e != cudaSuccess || !p)
            return fail(LLMC_ERR_CUDA, "cudaGetSymbolAddress of the static row buffer failed: %s",
                        cudaGetErrorString(e));
        g_rows_addr[device] = static_cast<float*>(p);
    }
    *out = g_rows_addr[device];
    return LLMC_OK;
}

}  // namespace

void noalloc_forget(int device) {
    if (device < 0 || device >= kMaxDevices) return;
    std::lock_guard<std::mutex> lock(g_setup_mu);
    g_rows_addr[device] = nullptr;
}

}  // namespace llmc

using namespace llmc;

extern "C" llmc_status llmc_observer_minmax_tensor_noalloc(llmc_ctx* ctx, const void* x, int32_t dtype, int64_t rows,
                                                          int64_t cols, int64_t ld, float* min_io, float* max_io,
                                                          int32_t accumulate) {
    LLMC_ENTRY();
    if (!ctx) return fail(LLMC_ERR_INVALID_ARG, "context must not be null");
    if (!x) return fail(LLMC_ERR_INVALID_ARG, "x must not be null");
    if (!min_io) return fail(LLMC_ERR_INVALID_ARG, "min must not be null");
    if (!max_io) return fail(LLMC_ERR_INVALID_ARG, "max must not be null");
    if (!dtype_ok(dtype)) return fail(LLMC_ERR_INVALID_ARG, "unsupported dtype %d", dtype);
    if (rows <= 0 || cols <= 0 || ld < cols) return fail(LLMC_ERR_SHAPE, "bad shape");
    if (rows > kMaxRows)
        return fail(LLMC_ERR_SHAPE,
                    "rows=%lld exceeds the static row buffer of the no-allocation observer (at most %lld rows); "
                    "use llmc_observer_minmax",
                    (long long)rows, (long long)kMaxRows);
    int prev = -1;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return fail(LLMC_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (prev != ctx->device) {
        e = cudaSetDevice(ctx->device);
        if (e != cudaSuccess) return fail(LLMC_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
    }
    float* scratch = nullptr;
    llmc_status st = rows_buffer(ctx->device, &scratch);
    if (st == LLMC_OK)
        st = minmax(ctx, x, dtype, rows, cols, ld, LLMC_STRATEGY_TENSOR, cols, min_io, max_io, accumulate, scratch);
    if (prev != ctx->device) {
        e = cudaSetDevice(prev);
        if (e != cudaSuccess && st == LLMC_OK)
            return fail(LLMC_ERR_CUDA, "restoring the caller's device: %s", cudaGetErrorString(e));
    }
    return st;
}
