// staging.h -- placing views and staging host operands through device buffers.
#pragma once
#include <cstddef>
#include <cstdint>
#include "internal.h"

namespace uor {

// A placed operand: where element (0,0) is, and the element offsets of the
// lowest and highest cells the view reaches, relative to it.
struct Operand {
    const uint8_t* origin = nullptr;
    ptrdiff_t lo = 0, hi = 0;
    size_t rows = 0, cols = 0;
    ptrdiff_t rs = 0, cs = 0;
    size_t es = 0;
};

// MatView::new (layout.rs:212): place a (data, len) buffer view. Returns
// DOES_NOT_FIT when no such view exists, INVALID_ARGUMENT for a null buffer
// that would have to hold cells.
int place_view(const void* data, size_t len, size_t rows, size_t cols, ptrdiff_t rs,
               ptrdiff_t cs, size_t es, Operand* out);

// raw.rs:98-188: an origin pointer with strides; false when the view's reach
// is not representable (the raw face then returns without writing).
bool raw_operand(const void* origin, size_t rows, size_t cols, ptrdiff_t rs, ptrdiff_t cs,
                 size_t es, Operand* out);

// Copy the span an input reaches to the device (slot), returning the device
// origin. With device pointers this is the identity.
int stage_in(uor_b200_ctx* ctx, int slot, const Operand& op, bool device, const uint8_t** dev);

// Output staging: copy the span in when it must be preserved or read, and
// copy it back after the device work.
struct OutStage {
    uint8_t* dev_origin = nullptr;
    uint8_t* dev_lo = nullptr;
    uint8_t* host_lo = nullptr;
    size_t bytes = 0;
    bool device = false;
};
int stage_out_begin(uor_b200_ctx* ctx, const Operand& op, bool device, bool reads_c,
                    OutStage* st, int slot = SLOT_C);
int stage_out_end(uor_b200_ctx* ctx, const OutStage& st);

}  // namespace uor
