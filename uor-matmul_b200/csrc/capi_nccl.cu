// capi_nccl.cu -- split-K across devices over NCCL, from the C ABI.
//
// One process (or thread) per GPU, each with its own context, all in one NCCL
// communicator. An entry point computes this rank's exact partial over its range of the
// reduction (the limbs or max-plus keys of capi_int.cu / capi_trop.cu), all-reduces it
// in place on the context's stream (sum of int64 limbs, max of int64 keys), and encodes
// the total once, so every rank's C holds the single-device bytes. The three steps are
// queued on one stream with no host round trip between them.
//
// NCCL is loaded on first use (dlopen of libnccl.so.2: the one a host process already
// loaded, e.g. PyTorch's, else the system's), so the library itself never depends on
// it; without it these entry points return UOR_B200_NCCL_ERROR.
#include <dlfcn.h>
#include <nccl.h>
#include <cstring>
#include <mutex>
#include "internal.h"
#include "splitk.cuh"

using namespace uor;

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_count)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*comm_cu_device)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    bool ok = false;
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        auto sym = [h](const char* name) { return dlsym(h, name); };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.comm_count = reinterpret_cast<decltype(api.comm_count)>(sym("ncclCommCount"));
        api.comm_cu_device = reinterpret_cast<decltype(api.comm_cu_device)>(sym("ncclCommCuDevice"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.comm_count &&
                 api.comm_cu_device && api.all_reduce;
    });
    return api;
}

// The exchange buffer of a context (a slot of its own: the partial and finish steps use
// the others).
int64_t* exchange_buffer(uor_b200_ctx* ctx, size_t count, int* st) {
    std::lock_guard<std::mutex> lock(ctx->mu);
    return static_cast<int64_t*>(ctx_buffer(ctx, SLOT_XCHG, count * sizeof(int64_t), st));
}

// The all-reduce on the context's stream, in the device-wide order of this library's calls.
int all_reduce(uor_b200_ctx* ctx, void* comm, int64_t* buf, size_t count, ncclRedOp_t op) {
    const NcclApi& api = nccl();
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceTurn turn(ctx);
    if (api.all_reduce(buf, buf, count, ncclInt64, op, static_cast<ncclComm_t>(comm), ctx->stream) !=
        ncclSuccess)
        return UOR_B200_NCCL_ERROR;
    return cuda_status(cudaGetLastError());
}

// The exchange with a failure flag: buf holds `count` values and one more int64, 0 from a
// rank whose partial succeeded and nonzero (bytes of 1) from one whose partial failed, so
// that a rank that fails after the checks still joins the collective (its peers never wait
// on it) and every rank learns of it. Sum and max both keep a nonzero flag nonzero.
int exchange(uor_b200_ctx* ctx, void* comm, int64_t* buf, size_t count, ncclRedOp_t op, int partial_status) {
    {
        std::lock_guard<std::mutex> lock(ctx->mu);
        const bool failed = partial_status != UOR_B200_OK;
        if (cudaMemsetAsync(failed ? buf : buf + count, failed ? 1 : 0,
                            (failed ? count + 1 : 1) * sizeof(int64_t), ctx->stream) != cudaSuccess)
            return UOR_B200_DEVICE_ERROR;
    }
    return all_reduce(ctx, comm, buf, count + 1, op);
}

// After a synchronous call: whether any rank's partial failed.
bool peer_failed(const int64_t* buf, size_t count) {
    int64_t flag = 0;
    if (cudaMemcpy(&flag, buf + count, sizeof(flag), cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return true;
    }
    return flag != 0;
}

// The checks every entry point shares: NCCL present, a communicator of this context's
// device, device pointers.
int check_call(void* comm, const uor_b200_call* call, uor_b200_ctx** ctx_out) {
    if (!comm || !call || !(call->flags & UOR_B200_DEVICE_POINTERS)) return UOR_B200_INVALID_ARGUMENT;
    const NcclApi& api = nccl();
    if (!api.ok) return UOR_B200_NCCL_ERROR;
    int st = UOR_B200_OK;
    uor_b200_ctx* ctx = resolve_ctx(call, &st);
    if (!ctx) return st;
    int dev = -1;
    if (api.comm_cu_device(static_cast<ncclComm_t>(comm), &dev) != ncclSuccess) return UOR_B200_NCCL_ERROR;
    if (dev != ctx->device) return UOR_B200_INVALID_ARGUMENT;
    *ctx_out = ctx;
    return UOR_B200_OK;
}

}  // namespace

extern "C" {

int uor_b200_nccl_unique_id(uint8_t* id, size_t id_len) {
    if (!id || id_len < sizeof(ncclUniqueId)) return UOR_B200_INVALID_ARGUMENT;
    const NcclApi& api = nccl();
    if (!api.ok) return UOR_B200_NCCL_ERROR;
    ncclUniqueId uid;
    if (api.get_unique_id(&uid) != ncclSuccess) return UOR_B200_NCCL_ERROR;
    std::memcpy(id, &uid, sizeof(uid));
    return UOR_B200_OK;
}

int uor_b200_nccl_comm_init(uor_b200_ctx* ctx, int nranks, const uint8_t* id, size_t id_len, int rank,
                            void** comm) {
    if (!comm || !id || id_len < sizeof(ncclUniqueId) || nranks < 1 || rank < 0 || rank >= nranks)
        return UOR_B200_INVALID_ARGUMENT;
    *comm = nullptr;
    const NcclApi& api = nccl();
    if (!api.ok) return UOR_B200_NCCL_ERROR;
    int st = UOR_B200_OK;
    if (!ctx && !(ctx = default_ctx(&st))) return st;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclComm_t c = nullptr;
    if (api.comm_init_rank(&c, nranks, uid, rank) != ncclSuccess) return UOR_B200_NCCL_ERROR;
    *comm = c;
    return UOR_B200_OK;
}

int uor_b200_nccl_comm_destroy(void* comm) {
    if (!comm) return UOR_B200_OK;
    const NcclApi& api = nccl();
    if (!api.ok) return UOR_B200_NCCL_ERROR;
    return api.comm_destroy(static_cast<ncclComm_t>(comm)) == ncclSuccess ? UOR_B200_OK : UOR_B200_NCCL_ERROR;
}

int uor_b200_gemm_splitk_nccl(void* comm, uor_b200_dtype elem, uor_b200_dtype out, const uor_b200_view* a,
                              const uor_b200_view* b, const uor_b200_view_mut* c, int64_t alpha,
                              int64_t beta, const uor_b200_call* call) {
    if (!a || !b || !c) return UOR_B200_INVALID_ARGUMENT;
    uor_b200_ctx* ctx = nullptr;
    int st = check_call(comm, call, &ctx);
    if (st != UOR_B200_OK) return st;
    if (a->rows != c->rows || b->cols != c->cols) return UOR_B200_NONCONFORMANT;
    const size_t count = SPLITK_LIMBS * a->rows * b->cols;
    if (count == 0) return UOR_B200_OK;
    int64_t* limbs = exchange_buffer(ctx, count + 1, &st);
    if (!limbs) return st;
    uor_b200_call step = *call;
    step.ctx = ctx;
    step.flags |= UOR_B200_ASYNC;  // the steps stay on the stream; the last one syncs as asked
    const int partial = uor_b200_gemm_partial_limbs(elem, a, b, limbs, count, &step);
    if ((st = exchange(ctx, comm, limbs, count, ncclSum, partial)) != UOR_B200_OK) return st;
    if (partial != UOR_B200_OK) return partial;
    step.flags = call->flags;
    step.route = nullptr;  // the route reported is the partial's
    if ((st = uor_b200_limbs_finish(elem, out, limbs, count, c, alpha, beta, &step)) != UOR_B200_OK)
        return st;
    return !(call->flags & UOR_B200_ASYNC) && peer_failed(limbs, count) ? UOR_B200_NCCL_ERROR
                                                                             : UOR_B200_OK;
}

int uor_b200_gemm_tropical_splitk_nccl(void* comm, uor_b200_dtype elem, uor_b200_dtype out,
                                       const uor_b200_view* a, const uor_b200_view* b,
                                       const uor_b200_view_mut* c, uor_b200_trop alpha, uor_b200_trop beta,
                                       const uor_b200_call* call) {
    if (!a || !b || !c) return UOR_B200_INVALID_ARGUMENT;
    uor_b200_ctx* ctx = nullptr;
    int st = check_call(comm, call, &ctx);
    if (st != UOR_B200_OK) return st;
    if (a->rows != c->rows || b->cols != c->cols) return UOR_B200_NONCONFORMANT;
    const size_t count = a->rows * b->cols;
    if (count == 0) return UOR_B200_OK;
    int64_t* keys = exchange_buffer(ctx, count + 1, &st);
    if (!keys) return st;
    uor_b200_call step = *call;
    step.ctx = ctx;
    step.flags |= UOR_B200_ASYNC;
    const int partial = uor_b200_trop_partial_keys(elem, a, b, keys, count, &step);
    if ((st = exchange(ctx, comm, keys, count, ncclMax, partial)) != UOR_B200_OK) return st;
    if (partial != UOR_B200_OK) return partial;
    step.flags = call->flags;
    step.route = nullptr;
    if ((st = uor_b200_trop_keys_finish(out, keys, count, c, alpha, beta, &step)) != UOR_B200_OK)
        return st;
    return !(call->flags & UOR_B200_ASYNC) && peer_failed(keys, count) ? UOR_B200_NCCL_ERROR
                                                                            : UOR_B200_OK;
}

}  // extern "C"
