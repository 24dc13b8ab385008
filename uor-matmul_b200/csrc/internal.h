// internal.h -- host-side plumbing shared by the C ABI translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include <mutex>
#include "../../include/uor_b200.h"

struct uor_b200_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;  // the stream work is issued on
    cudaStream_t own_stream = nullptr;
    int* d_status = nullptr;        // device status word for bounded waits
    uint64_t budget_ns = 2000000000ull;
    int sm_count = 148;
    std::mutex mu;
    // Growable device buffers: workspace (gathers, chunk partials), the three
    // staging slots host-pointer calls copy operands through, an auxiliary buffer
    // for operands a path rebuilds (decoded codes), and a dense decoded operand
    // handed to a driver that uses the auxiliary buffer itself.
    // A seventh slot holds the exchange buffer of the collective entry points.
    static constexpr int kSlots = 7;
    void* buf[kSlots] = {};
    size_t cap[kSlots] = {};
    // Host-pointer pipelining: copy-in and copy-out streams and a pool of events,
    // created on first use.
    cudaStream_t copy_in = nullptr, copy_out = nullptr;
    // A side stream for work of one call that runs beside the call's stream, and the two
    // events that fork it from and join it back into the call's stream.
    cudaStream_t side = nullptr;
    cudaEvent_t fork_ev = nullptr, join_ev = nullptr;
    cudaEvent_t events[256] = {};
    int nevents = 0;
};

namespace uor {

enum Slot { SLOT_WS = 0, SLOT_A = 1, SLOT_B = 2, SLOT_C = 3, SLOT_AUX = 4, SLOT_DECODED = 5, SLOT_XCHG = 6 };

// A device buffer of at least `bytes` in the given slot (grown with cudaMalloc;
// the previous contents are not kept).
void* ctx_buffer(uor_b200_ctx* ctx, int slot, size_t bytes, int* status);

// The default context of the current device (created on first use).
uor_b200_ctx* default_ctx(int* status);

// Resolve the call's context and make its device current.
uor_b200_ctx* resolve_ctx(const uor_b200_call* call, int* status);

// Device-wide order of this library's device work. Held for the span of one call
// (after the context's lock): the call's stream first waits for everything the
// previous call on the same device queued, whichever context or stream issued it,
// and the call's own work becomes what the next call waits for. So no two calls'
// kernels ever run side by side on one GPU -- in particular no tensor-core kernel
// shares its SMs with another kernel of this library. Calls queued while their
// stream is being captured into a CUDA graph take no part (the graph's replays are
// ordered by whoever replays them).
class DeviceTurn {
  public:
    explicit DeviceTurn(uor_b200_ctx* ctx);
    ~DeviceTurn();
    DeviceTurn(const DeviceTurn&) = delete;
    DeviceTurn& operator=(const DeviceTurn&) = delete;

  private:
    uor_b200_ctx* ctx_;
    bool held_ = false;
};

// The side stream, made to wait for everything the context's stream has queued so far
// (created on first use); nullptr when it cannot be had, and the caller then queues
// everything on the context's stream. ctx_join makes the context's stream wait for the
// side stream's work. Both record and wait on events only, so they also work while the
// context's stream is being captured into a CUDA graph.
cudaStream_t ctx_fork(uor_b200_ctx* ctx);
bool ctx_join(uor_b200_ctx* ctx);

// After device work: synchronise (unless async) and fold the status word in.
int finish_call(uor_b200_ctx* ctx, const uor_b200_call* call);

int cuda_status(cudaError_t e);

// cuTensorMapEncodeTiled for a 2-D uint8 tensor with 128-byte swizzle.
// dim0 is the contiguous dimension; stride1 is the byte stride of dim1.
bool make_tmap_u8(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1,
                  uint64_t stride1, uint32_t box0, uint32_t box1, bool swizzle128 = true);

// A 2-D s32 tensor map (dims {dim0, dim1}, byte stride of dim1), for TMA stores of
// an s32 output; 128-byte swizzle.
bool make_tmap_s32(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1,
                   uint64_t stride1_bytes, uint32_t box0, uint32_t box1);
// s32 3-D map (planes of dim0 x dim1), 128-byte swizzle, box {box0, box1, 1}.
bool make_tmap_s32_3d(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1,
                      uint64_t dim2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                      uint32_t box1);

// A view after placement: origin pointer and the reach of the view in elements.
struct Placed {
    const uint8_t* origin;  // element (0,0)
    ptrdiff_t lo, hi;        // lowest/highest offsets the view reaches (elements)
    size_t rows, cols;
    ptrdiff_t rs, cs;
};

// Strides::extent (layout.rs:71-102); false when the reach overflows.
bool view_extent(size_t rows, size_t cols, ptrdiff_t rs, ptrdiff_t cs, ptrdiff_t* lo,
                 ptrdiff_t* hi);
// place (layout.rs:178-199): the origin index of a view inside `len` elements.
bool view_place(size_t len, size_t rows, size_t cols, ptrdiff_t rs, ptrdiff_t cs, size_t* origin);
// Strides::self_aliases (layout.rs:116-140).
bool self_aliases(size_t rows, size_t cols, ptrdiff_t rs, ptrdiff_t cs);

size_t dtype_size(uor_b200_dtype t);

}  // namespace uor
