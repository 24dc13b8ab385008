// capi_trop.cu -- the tropical family's C ABI (driver::gemm over Trop<E> with MaxPlus).
#include <climits>
#include "internal.h"
#include "staging.h"
#include "tropical.cuh"

using namespace uor;

namespace {

int trop_bytes(uor_b200_dtype t) {
    switch (t) {
    case UOR_B200_TROP_I8: return 1;
    case UOR_B200_TROP_I16: return 2;
    case UOR_B200_TROP_I32: return 4;
    case UOR_B200_TROP_I64: return 8;
    default: return 0;
    }
}

}  // namespace

namespace {

// driver::gemm / gemm_selected over Trop<E> with MaxPlus; `w` (a u64 view, or null) takes
// the selection witness.
int trop_common(uor_b200_dtype elem, uor_b200_dtype out, const uor_b200_view* a,
                const uor_b200_view* b, const uor_b200_view_mut* c, const uor_b200_view_mut* w,
                uor_b200_trop alpha, uor_b200_trop beta, const uor_b200_call* call) {
    if (!a || !b || !c) return UOR_B200_INVALID_ARGUMENT;
    const int eb = trop_bytes(elem), ob = trop_bytes(out);
    if (!eb || !ob) return UOR_B200_UNSUPPORTED;
    const int mode = call ? (int)call->encode : MODE_NEAREST;
    if (mode < 0 || mode > 3) return UOR_B200_INVALID_ARGUMENT;
    Operand A, B, C, W;
    int st;
    if ((st = place_view(a->data, a->len, a->rows, a->cols, a->rs, a->cs, dtype_size(elem), &A)))
        return st;
    if ((st = place_view(b->data, b->len, b->rows, b->cols, b->rs, b->cs, dtype_size(elem), &B)))
        return st;
    if ((st = place_view(c->data, c->len, c->rows, c->cols, c->rs, c->cs, dtype_size(out), &C)))
        return st;
    if (w && (st = place_view(w->data, w->len, w->rows, w->cols, w->rs, w->cs, 8, &W))) return st;
    if (a->cols != b->rows || c->rows != a->rows || c->cols != b->cols) return UOR_B200_NONCONFORMANT;
    if (self_aliases(c->rows, c->cols, c->rs, c->cs)) return UOR_B200_OUTPUT_ALIASES;
    // SelectedTriple::new (selection.rs:76-98): the witness is m x n and injective.
    if (w && (w->rows != a->rows || w->cols != b->cols)) return UOR_B200_NONCONFORMANT;
    if (w && self_aliases(w->rows, w->cols, w->rs, w->cs)) return UOR_B200_OUTPUT_ALIASES;
    uor_b200_route local{};
    uor_b200_route* route = call && call->route ? call->route : &local;
    *route = uor_b200_route{};
    const size_t m = a->rows, k = a->cols, n = b->cols;
    if (m == 0 || n == 0) return UOR_B200_OK;
    if (m > (size_t)INT_MAX / 2 || n > (size_t)INT_MAX / 2 || k > (size_t)INT_MAX / 2)
        return UOR_B200_UNSUPPORTED;

    uor_b200_ctx* ctx = resolve_ctx(call, &st);
    if (!ctx) return st;
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceTurn turn(ctx);
    const bool dev = call && (call->flags & UOR_B200_DEVICE_POINTERS);
    const uint8_t *da = nullptr, *db = nullptr;
    OutStage cs, ws_out;
    if ((st = stage_in(ctx, SLOT_A, A, dev, &da))) return st;
    if ((st = stage_in(ctx, SLOT_B, B, dev, &db))) return st;
    if ((st = stage_out_begin(ctx, C, dev, beta.finite != 0, &cs))) return st;
    if (w && (st = stage_out_begin(ctx, W, dev, false, &ws_out, SLOT_AUX))) return st;

    TropEpi e{};
    e.alpha = alpha.value;
    e.beta = beta.value;
    e.alpha_finite = alpha.finite != 0;
    e.beta_finite = beta.finite != 0;
    e.mode = mode;
    e.obytes = ob;
    e.c = cs.dev_origin;
    e.rsc = C.rs;
    e.csc = C.cs;
    e.m = (int)m;
    e.n = (int)n;
    route->kernel = UOR_B200_KERNEL_TROPICAL;
    cudaError_t err;
    uint64_t* wd = w ? reinterpret_cast<uint64_t*>(ws_out.dev_origin) : nullptr;
    if (eb == 1 && (!w || k <= (size_t)TROP_WITNESS_MAX_K)) {
        const size_t wsb = w ? trop_witness_workspace((int)m, (int)k, (int)n)
                             : trop_i8_workspace((int)m, (int)k, (int)n);
        void* ws = ctx_buffer(ctx, SLOT_WS, wsb, &st);
        if (!ws) return st;
        route->tile_m = 128;
        route->tile_n = 128;
        route->tile_k = w ? 16 : 32;
        err = w ? trop_i8_witness_launch(da, A.rs, A.cs, db, B.rs, B.cs, (int)m, (int)k, (int)n, ws,
                                         e, wd, W.rs, W.cs, ctx->stream)
                : trop_i8_launch(da, A.rs, A.cs, db, B.rs, B.cs, (int)m, (int)k, (int)n, ws, e,
                                 ctx->stream);
    } else {
        route->tile_m = 16;
        route->tile_n = 16;
        err = w ? trop_generic_witness_launch(da, A.rs, A.cs, db, B.rs, B.cs, eb, (int)m, (int)k,
                                              (int)n, e, wd, W.rs, W.cs, ctx->stream)
                : trop_generic_launch(da, A.rs, A.cs, db, B.rs, B.cs, eb, (int)m, (int)k, (int)n,
                                      e, ctx->stream);
    }
    if (err != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    if ((st = stage_out_end(ctx, cs))) return st;
    if (w && (st = stage_out_end(ctx, ws_out))) return st;
    if (!dev) return uor_b200_ctx_sync(ctx);
    return finish_call(ctx, call);
}

}  // namespace

extern "C" int uor_b200_gemm_tropical(uor_b200_dtype elem, uor_b200_dtype out,
                                      const uor_b200_view* a, const uor_b200_view* b,
                                      const uor_b200_view_mut* c, uor_b200_trop alpha,
                                      uor_b200_trop beta, const uor_b200_call* call) {
    return trop_common(elem, out, a, b, c, nullptr, alpha, beta, call);
}

extern "C" int uor_b200_gemm_tropical_selected(uor_b200_dtype elem, uor_b200_dtype out,
                                               const uor_b200_view* a, const uor_b200_view* b,
                                               const uor_b200_view_mut* c,
                                               const uor_b200_view_mut* witness,
                                               uor_b200_trop alpha, uor_b200_trop beta,
                                               const uor_b200_call* call) {
    if (!witness) return UOR_B200_INVALID_ARGUMENT;
    return trop_common(elem, out, a, b, c, witness, alpha, beta, call);
}

// ---------------------------------------------------------------- split-K exchange
// driver::gemm's reduction over Trop<E> cut into ranges on different devices: each range's
// (max, +) reduction as int64 keys, the keys' element-wise maximum across ranges, then
// MaxPlus::finish and the encode once. Device buffers only.

extern "C" int uor_b200_trop_partial_keys(uor_b200_dtype elem, const uor_b200_view* a,
                                          const uor_b200_view* b, int64_t* keys, size_t keys_len,
                                          const uor_b200_call* call) {
    if (!a || !b) return UOR_B200_INVALID_ARGUMENT;
    if (!call || !(call->flags & UOR_B200_DEVICE_POINTERS)) return UOR_B200_INVALID_ARGUMENT;
    const int eb = trop_bytes(elem);
    if (eb != 1 && eb != 2 && eb != 4) return UOR_B200_UNSUPPORTED;  // sums must fit in int64
    Operand A, B;
    int st;
    if ((st = place_view(a->data, a->len, a->rows, a->cols, a->rs, a->cs, dtype_size(elem), &A)))
        return st;
    if ((st = place_view(b->data, b->len, b->rows, b->cols, b->rs, b->cs, dtype_size(elem), &B)))
        return st;
    if (a->cols != b->rows) return UOR_B200_NONCONFORMANT;
    const size_t m = a->rows, k = a->cols, n = b->cols;
    if (m == 0 || n == 0) return UOR_B200_OK;
    if (m > (size_t)INT_MAX / 2 || n > (size_t)INT_MAX / 2 || k > (size_t)INT_MAX / 2)
        return UOR_B200_UNSUPPORTED;
    if (!keys || keys_len < m * n) return UOR_B200_DOES_NOT_FIT;
    uor_b200_ctx* ctx = resolve_ctx(call, &st);
    if (!ctx) return st;
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceTurn turn(ctx);
    uor_b200_route local{};
    uor_b200_route* route = call->route ? call->route : &local;
    *route = uor_b200_route{};
    route->kernel = UOR_B200_KERNEL_TROPICAL;
    TropEpi e{};
    e.alpha = 0;
    e.alpha_finite = 1;
    e.beta_finite = 0;
    e.mode = MODE_NEAREST;
    e.obytes = 0;  // keys
    e.c = keys;
    e.rsc = (int64_t)n;
    e.csc = 1;
    e.m = (int)m;
    e.n = (int)n;
    cudaError_t err;
    if (eb == 1) {
        void* ws = ctx_buffer(ctx, SLOT_WS, trop_i8_workspace((int)m, (int)k, (int)n), &st);
        if (!ws) return st;
        route->tile_m = route->tile_n = 128;
        route->tile_k = 32;
        err = trop_i8_launch(A.origin, A.rs, A.cs, B.origin, B.rs, B.cs, (int)m, (int)k, (int)n, ws,
                             e, ctx->stream);
    } else {
        route->tile_m = route->tile_n = 16;
        err = trop_generic_launch(A.origin, A.rs, A.cs, B.origin, B.rs, B.cs, eb, (int)m, (int)k,
                                  (int)n, e, ctx->stream);
    }
    if (err != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    return finish_call(ctx, call);
}

extern "C" int uor_b200_trop_keys_finish(uor_b200_dtype out, const int64_t* keys, size_t keys_len,
                                         const uor_b200_view_mut* c, uor_b200_trop alpha,
                                         uor_b200_trop beta, const uor_b200_call* call) {
    if (!c) return UOR_B200_INVALID_ARGUMENT;
    if (!call || !(call->flags & UOR_B200_DEVICE_POINTERS)) return UOR_B200_INVALID_ARGUMENT;
    const int ob = trop_bytes(out);
    if (!ob) return UOR_B200_UNSUPPORTED;
    const int mode = (int)call->encode;
    if (mode < 0 || mode > 3) return UOR_B200_INVALID_ARGUMENT;
    Operand C;
    int st;
    if ((st = place_view(c->data, c->len, c->rows, c->cols, c->rs, c->cs, dtype_size(out), &C)))
        return st;
    if (self_aliases(c->rows, c->cols, c->rs, c->cs)) return UOR_B200_OUTPUT_ALIASES;
    const size_t m = c->rows, n = c->cols;
    if (m == 0 || n == 0) return UOR_B200_OK;
    if (m > (size_t)INT_MAX / 2 || n > (size_t)INT_MAX / 2) return UOR_B200_UNSUPPORTED;
    if (!keys || keys_len < m * n) return UOR_B200_DOES_NOT_FIT;
    uor_b200_ctx* ctx = resolve_ctx(call, &st);
    if (!ctx) return st;
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceTurn turn(ctx);
    TropEpi e{};
    e.alpha = alpha.value;
    e.beta = beta.value;
    e.alpha_finite = alpha.finite != 0;
    e.beta_finite = beta.finite != 0;
    e.mode = mode;
    e.obytes = ob;
    e.c = const_cast<uint8_t*>(C.origin);
    e.rsc = C.rs;
    e.csc = C.cs;
    e.m = (int)m;
    e.n = (int)n;
    if (trop_keys_finish_launch(keys, e, ctx->stream) != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    return finish_call(ctx, call);
}
