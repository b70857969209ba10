// Hessian collectives over NCCL for multi-GPU jobs driven through the C ABI (one process or
// thread per GPU): llmc_hessian_allreduce / llmc_hessian_reduce sum the partial Hessians of a
// token-sharded calibration set, plus helpers that make a communicator so a host without its
// own NCCL binding (the C# one) can use them.  NCCL is opened with dlopen at the first call,
// so the library has no link-time dependency on it; nccl.h supplies the types only.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

namespace llmc {
namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*);
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*group_start)();
    ncclResult_t (*group_end)();
    const char* (*error_string)(ncclResult_t);
};

const NcclApi* nccl_api() {
    static std::once_flag once;
    static NcclApi api;
    static bool ok = false;
    std::call_once(once, [] {
        void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) return;
        bool all = true;
        auto sym = [&](auto& fn, const char* name) {
            void* p = dlsym(lib, name);
            all &= p != nullptr;
            std::memcpy(&fn, &p, sizeof(p));
        };
        sym(api.get_unique_id, "ncclGetUniqueId");
        sym(api.comm_init_rank, "ncclCommInitRank");
        sym(api.comm_destroy, "ncclCommDestroy");
        sym(api.all_reduce, "ncclAllReduce");
        sym(api.reduce, "ncclReduce");
        sym(api.group_start, "ncclGroupStart");
        sym(api.group_end, "ncclGroupEnd");
        sym(api.error_string, "ncclGetErrorString");
        ok = all;
    });
    return ok ? &api : nullptr;
}

llmc_status need_nccl(const NcclApi** out) {
    *out = nccl_api();
    if (!*out) return fail(LLMC_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
    return LLMC_OK;
}

llmc_status nccl_check(const NcclApi* api, ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return LLMC_OK;
    return fail(LLMC_ERR_NCCL, "%s: %s", what, api->error_string ? api->error_string(r) : "NCCL error");
}

// Sum H (fp32 [d,d]) and the sample count over the communicator: onto every rank (root < 0)
// or onto `root`.  The count travels as one int64 through a workspace word.
llmc_status hessian_collective(llmc_hessian* h, void* comm, int root) {
    if (!h) return fail(LLMC_ERR_INVALID_ARG, "hessian must not be null");
    if (!comm) return fail(LLMC_ERR_INVALID_ARG, "comm must not be null");
    llmc_ctx* ctx = h->ctx;
    if (!ctx) return fail(LLMC_ERR_INVALID_ARG, "context must not be null");
    const NcclApi* api;
    LLMC_TRY(need_nccl(&api));
    LLMC_CUDA_TRY(cudaSetDevice(ctx->device));
    void* ws;
    LLMC_TRY(workspace(ctx, 64, &ws));
    int64_t* dcount = static_cast<int64_t*>(ws);
    int64_t count = h->samples;
    LLMC_CUDA_TRY(cudaMemcpyAsync(dcount, &count, sizeof(count), cudaMemcpyHostToDevice, ctx->stream));
    ncclComm_t c = static_cast<ncclComm_t>(comm);
    const size_t n = (size_t)h->d * (size_t)h->d;
    LLMC_TRY(nccl_check(api, api->group_start(), "ncclGroupStart"));
    ncclResult_t r1, r2;
    if (root < 0) {
        r1 = api->all_reduce(h->h, h->h, n, ncclFloat32, ncclSum, c, ctx->stream);
        r2 = api->all_reduce(dcount, dcount, 1, ncclInt64, ncclSum, c, ctx->stream);
    } else {
        r1 = api->reduce(h->h, h->h, n, ncclFloat32, ncclSum, root, c, ctx->stream);
        r2 = api->reduce(dcount, dcount, 1, ncclInt64, ncclSum, root, c, ctx->stream);
    }
    const ncclResult_t r3 = api->group_end();
    LLMC_TRY(nccl_check(api, r1, root < 0 ? "ncclAllReduce(H)" : "ncclReduce(H)"));
    LLMC_TRY(nccl_check(api, r2, root < 0 ? "ncclAllReduce(count)" : "ncclReduce(count)"));
    LLMC_TRY(nccl_check(api, r3, "ncclGroupEnd"));
    LLMC_CUDA_TRY(cudaMemcpyAsync(&count, dcount, sizeof(count), cudaMemcpyDeviceToHost, ctx->stream));
    LLMC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    h->samples = count;
    return LLMC_OK;
}

}  // namespace
}  // namespace llmc

using namespace llmc;

extern "C" {

llmc_status llmc_nccl_unique_id(uint8_t* out, int64_t size) {
    LLMC_ENTRY();
    if (!out) return fail(LLMC_ERR_INVALID_ARG, "out must not be null");
    if (size < (int64_t)sizeof(ncclUniqueId))
        return fail(LLMC_ERR_SHAPE, "unique id buffer of %lld bytes, need %zu", (long long)size, sizeof(ncclUniqueId));
    const NcclApi* api;
    LLMC_TRY(need_nccl(&api));
    ncclUniqueId id;
    LLMC_TRY(nccl_check(api, api->get_unique_id(&id), "ncclGetUniqueId"));
    std::memcpy(out, &id, sizeof(id));
    return LLMC_OK;
}

llmc_status llmc_nccl_comm_init(llmc_ctx* ctx, int32_t world, int32_t rank, const uint8_t* unique_id, int64_t size,
                                void** comm_out) {
    LLMC_ENTRY();
    if (!ctx || !unique_id || !comm_out) return fail(LLMC_ERR_INVALID_ARG, "ctx, unique_id and comm_out must not be null");
    *comm_out = nullptr;
    if (world < 1 || rank < 0 || rank >= world)
        return fail(LLMC_ERR_OUT_OF_RANGE, "rank %d outside a world of %d", rank, world);
    if (size < (int64_t)sizeof(ncclUniqueId))
        return fail(LLMC_ERR_SHAPE, "unique id of %lld bytes, need %zu", (long long)size, sizeof(ncclUniqueId));
    const NcclApi* api;
    LLMC_TRY(need_nccl(&api));
    LLMC_CUDA_TRY(cudaSetDevice(ctx->device));
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof(id));
    ncclComm_t c = nullptr;
    LLMC_TRY(nccl_check(api, api->comm_init_rank(&c, world, id, rank), "ncclCommInitRank"));
    *comm_out = c;
    return LLMC_OK;
}

llmc_status llmc_nccl_comm_destroy(void* comm) {
    LLMC_ENTRY();
    if (!comm) return LLMC_OK;
    const NcclApi* api;
    LLMC_TRY(need_nccl(&api));
    return nccl_check(api, api->comm_destroy(static_cast<ncclComm_t>(comm)), "ncclCommDestroy");
}

llmc_status llmc_hessian_allreduce(llmc_hessian* h, void* comm) {
    LLMC_ENTRY();
    return hessian_collective(h, comm, -1);
}

llmc_status llmc_hessian_reduce(llmc_hessian* h, void* comm, int32_t root) {
    LLMC_ENTRY();
    if (root < 0) return fail(LLMC_ERR_OUT_OF_RANGE, "root must be a rank (got %d)", root);
    return hessian_collective(h, comm, root);
}

}  // extern "C"
