// context.cu -- contexts, device buffers, view placement, tensor maps, status.
#include <cudaTypedefs.h>
#include <climits>
#include <cstring>
#include <new>
#include "internal.h"
#include "aux.cuh"
#include "ptx.cuh"

using namespace uor;

namespace uor {

int cuda_status(cudaError_t e) { return e == cudaSuccess ? UOR_B200_OK : UOR_B200_DEVICE_ERROR; }

size_t dtype_size(uor_b200_dtype t) {
    switch (t) {
    case UOR_B200_I8: return 1;
    case UOR_B200_I16: return 2;
    case UOR_B200_I32: return 4;
    case UOR_B200_I64: return 8;
    case UOR_B200_I128: return 16;
    case UOR_B200_F32: return 4;
    case UOR_B200_F64: return 8;
    case UOR_B200_TROP_I8: return 2;
    case UOR_B200_TROP_I16: return 4;
    case UOR_B200_TROP_I32: return 8;
    case UOR_B200_TROP_I64: return 16;
    default: return 0;
    }
}

void* ctx_buffer(uor_b200_ctx* ctx, int slot, size_t bytes, int* status) {
    if (bytes == 0) bytes = 256;
    if (ctx->cap[slot] >= bytes) return ctx->buf[slot];
    if (ctx->buf[slot]) {
        // The stream may still be using the old buffer.
        cudaStreamSynchronize(ctx->stream);
        cudaFree(ctx->buf[slot]);
        ctx->buf[slot] = nullptr;
        ctx->cap[slot] = 0;
    }
    size_t want = bytes + bytes / 8;  // headroom so nearby sizes reuse the buffer
    void* p = nullptr;
    if (cudaMalloc(&p, want) != cudaSuccess) {
        cudaGetLastError();
        if (cudaMalloc(&p, bytes) != cudaSuccess) {
            cudaGetLastError();
            *status = UOR_B200_DEVICE_ERROR;
            return nullptr;
        }
        want = bytes;
    }
    ctx->buf[slot] = p;
    ctx->cap[slot] = want;
    return p;
}

static uor_b200_ctx* g_default[64] = {};
static std::mutex g_default_mu;

uor_b200_ctx* default_ctx(int* status) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        *status = UOR_B200_DEVICE_ERROR;
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_default_mu);
    if (!g_default[dev]) {
        g_default[dev] = uor_b200_ctx_create(dev);
        if (!g_default[dev]) *status = UOR_B200_DEVICE_ERROR;
    }
    return g_default[dev];
}

uor_b200_ctx* resolve_ctx(const uor_b200_call* call, int* status) {
    uor_b200_ctx* ctx = call && call->ctx ? call->ctx : default_ctx(status);
    if (!ctx) return nullptr;
    if (cudaSetDevice(ctx->device) != cudaSuccess) {
        cudaGetLastError();
        *status = UOR_B200_DEVICE_ERROR;
        return nullptr;
    }
    return ctx;
}

namespace {
struct DeviceOrder {
    std::mutex mu;
    cudaEvent_t tail = nullptr;  // recorded after the last call's work on this device
};
DeviceOrder& device_order(int device) {
    static DeviceOrder order[64];
    return order[device & 63];
}
}  // namespace

DeviceTurn::DeviceTurn(uor_b200_ctx* ctx) : ctx_(ctx) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(ctx->stream, &cap) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    if (cap != cudaStreamCaptureStatusNone) return;
    DeviceOrder& o = device_order(ctx->device);
    o.mu.lock();
    held_ = true;
    if (!o.tail) {
        if (cudaEventCreateWithFlags(&o.tail, cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            o.tail = nullptr;
        }
    } else if (cudaStreamWaitEvent(ctx->stream, o.tail, 0) != cudaSuccess) {
        cudaGetLastError();
    }
}

DeviceTurn::~DeviceTurn() {
    if (!held_) return;
    DeviceOrder& o = device_order(ctx_->device);
    if (o.tail && cudaEventRecord(o.tail, ctx_->stream) != cudaSuccess) cudaGetLastError();
    o.mu.unlock();
}

int finish_call(uor_b200_ctx* ctx, const uor_b200_call* call) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    const bool async = call && (call->flags & UOR_B200_ASYNC) && (call->flags & UOR_B200_DEVICE_POINTERS);
    if (async) return UOR_B200_OK;
    return uor_b200_ctx_sync(ctx);
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        cudaGetLastError();
    });
    return fn;
}

bool make_tmap_u8(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1,
                  uint64_t stride1, uint32_t box0, uint32_t box1, bool swizzle128) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {dim0, dim1};
    cuuint64_t strides[1] = {stride1};
    cuuint32_t box[2] = {box0, box1};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_tmap_s32(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1,
                   uint64_t stride1_bytes, uint32_t box0, uint32_t box1) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {dim0, dim1};
    cuuint64_t strides[1] = {stride1_bytes};
    cuuint32_t box[2] = {box0, box1};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, const_cast<void*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_tmap_s32_3d(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1,
                      uint64_t dim2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                      uint32_t box1) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {dim0, dim1, dim2};
    cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
    cuuint32_t box[3] = {box0, box1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_INT32, 3, const_cast<void*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool view_extent(size_t rows, size_t cols, ptrdiff_t rs, ptrdiff_t cs, ptrdiff_t* lo,
                 ptrdiff_t* hi) {
    if (rows == 0 || cols == 0) {
        *lo = *hi = 0;
        return true;
    }
    if (rows - 1 > (size_t)PTRDIFF_MAX || cols - 1 > (size_t)PTRDIFF_MAX) return false;
    ptrdiff_t r, c;
    if (__builtin_mul_overflow((ptrdiff_t)(rows - 1), rs, &r)) return false;
    if (__builtin_mul_overflow((ptrdiff_t)(cols - 1), cs, &c)) return false;
    const ptrdiff_t rlo = rs < 0 ? r : 0, rhi = rs < 0 ? 0 : r;
    const ptrdiff_t clo = cs < 0 ? c : 0, chi = cs < 0 ? 0 : c;
    if (__builtin_add_overflow(rlo, clo, lo)) return false;
    if (__builtin_add_overflow(rhi, chi, hi)) return false;
    return true;
}

bool view_place(size_t len, size_t rows, size_t cols, ptrdiff_t rs, ptrdiff_t cs,
                size_t* origin) {
    if (rows == 0 || cols == 0) {
        *origin = 0;
        return true;
    }
    ptrdiff_t lo, hi;
    if (!view_extent(rows, cols, rs, cs, &lo, &hi)) return false;
    if (lo > 0) return false;
    const size_t o = (size_t)(-(lo + 1)) + 1;  // |lo| without overflow at PTRDIFF_MIN
    const size_t h = hi < 0 ? (size_t)(-(hi + 1)) + 1 : (size_t)hi;
    size_t top;
    if (__builtin_add_overflow(o, h, &top)) return false;
    if (top >= len) return false;
    *origin = lo == 0 ? 0 : o;
    return true;
}

static size_t gcd_sz(size_t a, size_t b) {
    while (b) {
        size_t t = a % b;
        a = b;
        b = t;
    }
    return a;
}

bool self_aliases(size_t rows, size_t cols, ptrdiff_t rs, ptrdiff_t cs) {
    if (rows == 0 || cols == 0) return false;
    if (rows <= 1 && cols <= 1) return false;
    if (rows > 1 && rs == 0) return true;
    if (cols > 1 && cs == 0) return true;
    if (rows <= 1 || cols <= 1) return false;
    const size_t a = rs < 0 ? (size_t)0 - (size_t)rs : (size_t)rs;
    const size_t b = cs < 0 ? (size_t)0 - (size_t)cs : (size_t)cs;
    const size_t g = gcd_sz(a, b);
    return (b / g) < rows && (a / g) < cols;
}

cudaStream_t ctx_fork(uor_b200_ctx* ctx) {
    if (!ctx->side && (cudaStreamCreateWithFlags(&ctx->side, cudaStreamNonBlocking) != cudaSuccess ||
                       cudaEventCreateWithFlags(&ctx->fork_ev, cudaEventDisableTiming) != cudaSuccess ||
                       cudaEventCreateWithFlags(&ctx->join_ev, cudaEventDisableTiming) != cudaSuccess)) {
        cudaGetLastError();
        return nullptr;
    }
    if (cudaEventRecord(ctx->fork_ev, ctx->stream) != cudaSuccess ||
        cudaStreamWaitEvent(ctx->side, ctx->fork_ev, 0) != cudaSuccess)
        return nullptr;
    return ctx->side;
}

bool ctx_join(uor_b200_ctx* ctx) {
    return cudaEventRecord(ctx->join_ev, ctx->side) == cudaSuccess &&
           cudaStreamWaitEvent(ctx->stream, ctx->join_ev, 0) == cudaSuccess;
}

}  // namespace uor

// ------------------------------------------------------------------ C ABI

extern "C" {

uor_b200_ctx* uor_b200_ctx_create(int device) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
        cudaGetLastError();
        return nullptr;
    }
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    auto* ctx = new (std::nothrow) uor_b200_ctx();
    if (!ctx) return nullptr;
    ctx->device = device;
    // A blocking stream: a call on the context's own stream is ordered after work the
    // caller queued on the legacy default stream (a fill of the output, a copy of an
    // operand) and before work queued there after it returns.
    bool ok = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamDefault) == cudaSuccess &&
              cudaMalloc(&ctx->d_status, sizeof(int)) == cudaSuccess &&
              cudaMemset(ctx->d_status, 0, sizeof(int)) == cudaSuccess &&
              cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device) ==
                  cudaSuccess;
    ctx->stream = ctx->own_stream;
    cudaSetDevice(prev);
    if (!ok) {
        cudaGetLastError();
        uor_b200_ctx_destroy(ctx);
        return nullptr;
    }
    return ctx;
}

void uor_b200_ctx_destroy(uor_b200_ctx* ctx) {
    if (!ctx) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    for (int i = 0; i < uor_b200_ctx::kSlots; ++i)
        if (ctx->buf[i]) cudaFree(ctx->buf[i]);
    if (ctx->d_status) cudaFree(ctx->d_status);
    for (int i = 0; i < ctx->nevents; ++i) cudaEventDestroy(ctx->events[i]);
    if (ctx->side) cudaStreamDestroy(ctx->side);
    if (ctx->fork_ev) cudaEventDestroy(ctx->fork_ev);
    if (ctx->join_ev) cudaEventDestroy(ctx->join_ev);
    if (ctx->copy_in) cudaStreamDestroy(ctx->copy_in);
    if (ctx->copy_out) cudaStreamDestroy(ctx->copy_out);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    cudaGetLastError();
    cudaSetDevice(prev);
    delete ctx;
}

int uor_b200_ctx_set_stream(uor_b200_ctx* ctx, void* stream) {
    if (!ctx) return UOR_B200_INVALID_ARGUMENT;
    ctx->stream = static_cast<cudaStream_t>(stream);  // NULL is the legacy default stream
    return UOR_B200_OK;
}

int uor_b200_ctx_set_wait_budget_ns(uor_b200_ctx* ctx, uint64_t ns) {
    if (!ctx || ns == 0) return UOR_B200_INVALID_ARGUMENT;
    ctx->budget_ns = ns;
    return UOR_B200_OK;
}

int uor_b200_ctx_sync(uor_b200_ctx* ctx) {
    if (!ctx) return UOR_B200_INVALID_ARGUMENT;
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    int st = 0;
    if (cudaMemcpy(&st, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
        return UOR_B200_DEVICE_ERROR;
    if (st != 0) {
        cudaMemset(ctx->d_status, 0, sizeof(int));
        return UOR_B200_TIMEOUT;
    }
    return UOR_B200_OK;
}

const char* uor_b200_status_string(int s) {
    switch (s) {
    case UOR_B200_OK: return "ok";
    case UOR_B200_NONCONFORMANT: return "not a product: nonconformant shapes";
    case UOR_B200_OUTPUT_ALIASES: return "not a product: the output aliases itself";
    case UOR_B200_DEVICE_ERROR: return "CUDA runtime error";
    case UOR_B200_TIMEOUT: return "a bounded device wait ran out";
    case UOR_B200_NCCL_ERROR: return "NCCL error";
    case UOR_B200_DOES_NOT_FIT: return "a buffer does not hold the view described";
    case UOR_B200_INVALID_ARGUMENT: return "invalid argument";
    case UOR_B200_UNSUPPORTED: return "element/output pair not supported";
    case UOR_B200_SCRATCH_LIMIT: return "the product needs more than the fixed no-allocation scratch";
    default: return "unknown status";
    }
}

int uor_b200_version(void) { return 100; }

int uor_b200_selftest_wait_timeout(uor_b200_ctx* ctx, uint64_t budget_ns) {
    int st = UOR_B200_OK;
    if (!ctx) ctx = default_ctx(&st);
    if (!ctx) return st;
    cudaSetDevice(ctx->device);
    if (selftest_wait(ctx->d_status, budget_ns, ctx->stream) != cudaSuccess)
        return UOR_B200_DEVICE_ERROR;
    return uor_b200_ctx_sync(ctx);
}

}  // extern "C"
