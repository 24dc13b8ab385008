// staging.cu -- view placement and host<->device staging for host-pointer calls.
#include "staging.h"

namespace uor {

int place_view(const void* data, size_t len, size_t rows, size_t cols, ptrdiff_t rs,
               ptrdiff_t cs, size_t es, Operand* out) {
    size_t origin = 0;
    if (!view_place(len, rows, cols, rs, cs, &origin)) return UOR_B200_DOES_NOT_FIT;
    ptrdiff_t lo = 0, hi = 0;
    view_extent(rows, cols, rs, cs, &lo, &hi);
    if (rows && cols && !data) return UOR_B200_INVALID_ARGUMENT;
    out->origin = static_cast<const uint8_t*>(data) + origin * es;
    out->lo = lo;
    out->hi = hi;
    out->rows = rows;
    out->cols = cols;
    out->rs = rs;
    out->cs = cs;
    out->es = es;
    return UOR_B200_OK;
}

bool raw_operand(const void* origin, size_t rows, size_t cols, ptrdiff_t rs, ptrdiff_t cs,
                 size_t es, Operand* out) {
    ptrdiff_t lo = 0, hi = 0;
    if (!view_extent(rows, cols, rs, cs, &lo, &hi)) return false;
    out->origin = static_cast<const uint8_t*>(origin);
    out->lo = lo;
    out->hi = hi;
    out->rows = rows;
    out->cols = cols;
    out->rs = rs;
    out->cs = cs;
    out->es = es;
    return true;
}

int stage_in(uor_b200_ctx* ctx, int slot, const Operand& op, bool device, const uint8_t** dev) {
    if (device || op.rows == 0 || op.cols == 0) {
        *dev = op.origin;
        return UOR_B200_OK;
    }
    const size_t bytes = (size_t)(op.hi - op.lo + 1) * op.es;
    int st = UOR_B200_OK;
    auto* d = static_cast<uint8_t*>(ctx_buffer(ctx, slot, bytes, &st));
    if (!d) return st;
    if (cudaMemcpyAsync(d, op.origin + op.lo * (ptrdiff_t)op.es, bytes, cudaMemcpyHostToDevice,
                        ctx->stream) != cudaSuccess)
        return UOR_B200_DEVICE_ERROR;
    *dev = d - op.lo * (ptrdiff_t)op.es;
    return UOR_B200_OK;
}

int stage_out_begin(uor_b200_ctx* ctx, const Operand& op, bool device, bool reads_c,
                    OutStage* st, int slot) {
    st->device = device;
    if (device || op.rows == 0 || op.cols == 0) {
        st->dev_origin = const_cast<uint8_t*>(op.origin);
        return UOR_B200_OK;
    }
    const size_t span = (size_t)(op.hi - op.lo + 1);
    st->bytes = span * op.es;
    int s = UOR_B200_OK;
    auto* d = static_cast<uint8_t*>(ctx_buffer(ctx, slot, st->bytes, &s));
    if (!d) return s;
    st->dev_lo = d;
    st->host_lo = const_cast<uint8_t*>(op.origin) + op.lo * (ptrdiff_t)op.es;
    st->dev_origin = d - op.lo * (ptrdiff_t)op.es;
    // A view that does not cover its whole span leaves cells between its rows
    // that the copy back must not disturb; bring them along.
    const bool gaps = span != op.rows * op.cols;
    if (reads_c || gaps) {
        if (cudaMemcpyAsync(d, st->host_lo, st->bytes, cudaMemcpyHostToDevice, ctx->stream) !=
            cudaSuccess)
            return UOR_B200_DEVICE_ERROR;
    }
    return UOR_B200_OK;
}

int stage_out_end(uor_b200_ctx* ctx, const OutStage& st) {
    if (st.device || st.bytes == 0) return UOR_B200_OK;
    if (cudaMemcpyAsync(st.host_lo, st.dev_lo, st.bytes, cudaMemcpyDeviceToHost, ctx->stream) !=
        cudaSuccess)
        return UOR_B200_DEVICE_ERROR;
    return UOR_B200_OK;
}

}  // namespace uor
