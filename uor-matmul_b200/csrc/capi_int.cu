// capi_int.cu -- the integer family's C ABI: view API, slice face, typed
// W8A8 entries. Validation happens here, once, before any device work
// (Triple::new, layout.rs:534-561); everything after it is total.
#include "internal.h"
#include "int_gemm.h"
#include "splitk.cuh"
#include "staging.h"

using namespace uor;

namespace {

bool int_elem(uor_b200_dtype t) {
    return t == UOR_B200_I8 || t == UOR_B200_I16 || t == UOR_B200_I32 || t == UOR_B200_I64;
}

bool int_out(uor_b200_dtype t, int* kind) {
    switch (t) {
    case UOR_B200_I8: *kind = OUT_I8; return true;
    case UOR_B200_I16: *kind = OUT_I16; return true;
    case UOR_B200_I32: *kind = OUT_I32; return true;
    case UOR_B200_I64: *kind = OUT_I64; return true;
    case UOR_B200_I128: *kind = OUT_I128; return true;
    default: return false;
    }
}

int call_mode(const uor_b200_call* call, int* mode) {
    *mode = call ? (int)call->encode : MODE_NEAREST;
    return *mode >= 0 && *mode <= 3 ? UOR_B200_OK : UOR_B200_INVALID_ARGUMENT;
}

bool device_ptrs(const uor_b200_call* call) {
    return call && (call->flags & UOR_B200_DEVICE_POINTERS);
}

// Everything after validation, with the context locked: stage, compute, stage back.
int int_gemm_locked(uor_b200_ctx* ctx, uor_b200_dtype elem, int kind, const Operand& A,
                    const Operand& B, const Operand& C, int64_t alpha, int64_t beta, int mode,
                    const uor_b200_call* call, uor_b200_route* route, bool cplx = false) {
    const size_t m = A.rows, k = A.cols, n = B.cols;
    int st = UOR_B200_OK;
    const bool dev = device_ptrs(call);
    const LinearEpi epi{alpha, beta, mode, kind};
    if (!dev && !cplx && elem == UOR_B200_I8 && i8_pipeline_applies(A, B, C)) {
        st = run_i8_gemm_pipelined(ctx, A, B, C, epi, route);
        if (st != UOR_B200_UNSUPPORTED) return st;
    }
    const uint8_t *da = nullptr, *db = nullptr;
    OutStage cs;
    if ((st = stage_in(ctx, SLOT_A, A, dev, &da)) != UOR_B200_OK) return st;
    if ((st = stage_in(ctx, SLOT_B, B, dev, &db)) != UOR_B200_OK) return st;
    if ((st = stage_out_begin(ctx, C, dev, beta != 0, &cs)) != UOR_B200_OK) return st;

    if (elem == UOR_B200_I8 && !cplx)
        st = run_i8_gemm(ctx, reinterpret_cast<const int8_t*>(da), A.rs, A.cs,
                         reinterpret_cast<const int8_t*>(db), B.rs, B.cs, cs.dev_origin, C.rs,
                         C.cs, m, k, n, epi, route);
    else
        st = run_wide_gemm(ctx, (int)dtype_size(elem), da, A.rs, A.cs, db, B.rs, B.cs,
                           cs.dev_origin, C.rs, C.cs, m, k, n, epi, route, cplx,
                           call ? call->flags & (UOR_B200_DIGIT_SLICES | UOR_B200_MODULAR) : 0u);
    if (st != UOR_B200_OK) return st;
    if ((st = stage_out_end(ctx, cs)) != UOR_B200_OK) return st;
    if (!dev) return uor_b200_ctx_sync(ctx);
    return finish_call(ctx, call);
}

int int_gemm_placed(uor_b200_dtype elem, int kind, const Operand& A, const Operand& B,
                    const Operand& C, int64_t alpha, int64_t beta, int mode,
                    const uor_b200_call* call, bool cplx = false) {
    uor_b200_route local_route{};
    uor_b200_route* route = call && call->route ? call->route : &local_route;
    *route = uor_b200_route{};
    if (A.rows == 0 || B.cols == 0) return UOR_B200_OK;
    int st = UOR_B200_OK;
    uor_b200_ctx* ctx = resolve_ctx(call, &st);
    if (!ctx) return st;
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceTurn turn(ctx);
    return int_gemm_locked(ctx, elem, kind, A, B, C, alpha, beta, mode, call, route, cplx);
}

int gemm_views(uor_b200_dtype elem, uor_b200_dtype out, const void* a, size_t a_len, size_t am,
               size_t ak, ptrdiff_t rsa, ptrdiff_t csa, const void* b, size_t b_len, size_t bk,
               size_t bn, ptrdiff_t rsb, ptrdiff_t csb, void* c, size_t c_len, size_t cm,
               size_t cn, ptrdiff_t rsc, ptrdiff_t csc, int64_t alpha, int64_t beta,
               const uor_b200_call* call) {
    int kind = 0, mode = 0;
    if (!int_elem(elem) || !int_out(out, &kind)) return UOR_B200_UNSUPPORTED;
    if (call_mode(call, &mode) != UOR_B200_OK) return UOR_B200_INVALID_ARGUMENT;
    const size_t es = dtype_size(elem), os = dtype_size(out);
    Operand A, B, C;
    int st;
    if ((st = place_view(a, a_len, am, ak, rsa, csa, es, &A)) != UOR_B200_OK) return st;
    if ((st = place_view(b, b_len, bk, bn, rsb, csb, es, &B)) != UOR_B200_OK) return st;
    if ((st = place_view(c, c_len, cm, cn, rsc, csc, os, &C)) != UOR_B200_OK) return st;
    // Triple::new (layout.rs:534-561)
    if (ak != bk || cm != am || cn != bn) return UOR_B200_NONCONFORMANT;
    if (self_aliases(cm, cn, rsc, csc)) return UOR_B200_OUTPUT_ALIASES;
    return int_gemm_placed(elem, kind, A, B, C, alpha, beta, mode, call);
}

// Complex<i32 | i64> (alphabet.rs:656-776): views count complex elements, each
// {re, im} of the part type.
int gemm_complex_views(uor_b200_dtype elem, uor_b200_dtype out, const uor_b200_view* a,
                       const uor_b200_view* b, const uor_b200_view_mut* c, int64_t alpha,
                       int64_t beta, const uor_b200_call* call) {
    int kind = 0, mode = 0;
    if (!a || !b || !c) return UOR_B200_INVALID_ARGUMENT;
    if ((elem != UOR_B200_I32 && elem != UOR_B200_I64) || !int_out(out, &kind))
        return UOR_B200_UNSUPPORTED;
    if (call_mode(call, &mode) != UOR_B200_OK) return UOR_B200_INVALID_ARGUMENT;
    const size_t es = 2 * dtype_size(elem), os = 2 * dtype_size(out);
    Operand A, B, C;
    int st;
    if ((st = place_view(a->data, a->len, a->rows, a->cols, a->rs, a->cs, es, &A)) != UOR_B200_OK)
        return st;
    if ((st = place_view(b->data, b->len, b->rows, b->cols, b->rs, b->cs, es, &B)) != UOR_B200_OK)
        return st;
    if ((st = place_view(c->data, c->len, c->rows, c->cols, c->rs, c->cs, os, &C)) != UOR_B200_OK)
        return st;
    if (a->cols != b->rows || c->rows != a->rows || c->cols != b->cols)
        return UOR_B200_NONCONFORMANT;
    if (self_aliases(c->rows, c->cols, c->rs, c->cs)) return UOR_B200_OUTPUT_ALIASES;
    return int_gemm_placed(elem, kind, A, B, C, alpha, beta, mode, call, true);
}

}  // namespace

extern "C" {

int uor_b200_gemm_complex(uor_b200_dtype elem, uor_b200_dtype out, const uor_b200_view* a,
                          const uor_b200_view* b, const uor_b200_view_mut* c, int64_t alpha,
                          int64_t beta, const uor_b200_call* call) {
    return gemm_complex_views(elem, out, a, b, c, alpha, beta, call);
}

int uor_b200_gemm(uor_b200_dtype elem, uor_b200_dtype out, const uor_b200_view* a,
                  const uor_b200_view* b, const uor_b200_view_mut* c, int64_t alpha,
                  int64_t beta, const uor_b200_call* call) {
    if (!a || !b || !c) return UOR_B200_INVALID_ARGUMENT;
    return gemm_views(elem, out, a->data, a->len, a->rows, a->cols, a->rs, a->cs, b->data, b->len,
                      b->rows, b->cols, b->rs, b->cs, c->data, c->len, c->rows, c->cols, c->rs,
                      c->cs, alpha, beta, call);
}

int uor_b200_slice_gemm_ex(uor_b200_dtype elem, uor_b200_dtype out, size_t m, size_t k, size_t n,
                           int64_t alpha, const void* a, size_t a_len, size_t lda, const void* b,
                           size_t b_len, size_t ldb, int64_t beta, void* c, size_t c_len,
                           size_t ldc, void* scratch, size_t scratch_len,
                           const uor_b200_call* call) {
    (void)scratch;
    (void)scratch_len;  // the offer never changes bytes (slice.rs:23-41)
    return gemm_views(elem, out, a, a_len, m, k, (ptrdiff_t)lda, 1, b, b_len, k, n, (ptrdiff_t)ldb,
                      1, c, c_len, m, n, (ptrdiff_t)ldc, 1, alpha, beta, call);
}

int uor_b200_slice_gemm(uor_b200_dtype elem, uor_b200_dtype out, size_t m, size_t k, size_t n,
                        const void* a, size_t a_len, const void* b, size_t b_len, void* c,
                        size_t c_len, void* scratch, size_t scratch_len,
                        const uor_b200_call* call) {
    return uor_b200_slice_gemm_ex(elem, out, m, k, n, 1, a, a_len, k, b, b_len, n, 0, c, c_len, n,
                                  scratch, scratch_len, call);
}

int uor_b200_slice_gemm_ex_full(uor_b200_dtype elem, uor_b200_dtype out, size_t m, size_t k,
                                size_t n, int64_t alpha, const void* a, size_t a_len, size_t lda,
                                const void* b, size_t b_len, size_t ldb, int64_t beta, void* c,
                                size_t c_len, size_t ldc, void* panels, size_t panels_len,
                                void* accumulators, size_t accumulators_len,
                                const uor_b200_call* call) {
    (void)accumulators;
    (void)accumulators_len;
    return uor_b200_slice_gemm_ex(elem, out, m, k, n, alpha, a, a_len, lda, b, b_len, ldb, beta,
                                  c, c_len, ldc, panels, panels_len, call);
}

int uor_b200_gemm_i8_i32(size_t m, size_t k, size_t n, const int8_t* a, const int8_t* b,
                         int32_t* c, const uor_b200_call* call) {
    return uor_b200_slice_gemm(UOR_B200_I8, UOR_B200_I32, m, k, n, a, m * k, b, k * n, c, m * n,
                               nullptr, 0, call);
}

int uor_b200_gemm_ex_i8_i32(size_t m, size_t k, size_t n, int64_t alpha, const int8_t* a,
                            size_t lda, const int8_t* b, size_t ldb, int64_t beta, int32_t* c,
                            size_t ldc, const uor_b200_call* call) {
    // The slices are exactly as long as the leading dimensions require.
    const size_t a_len = m && k ? (m - 1) * lda + k : 0;
    const size_t b_len = k && n ? (k - 1) * ldb + n : 0;
    const size_t c_len = m && n ? (m - 1) * ldc + n : 0;
    return uor_b200_slice_gemm_ex(UOR_B200_I8, UOR_B200_I32, m, k, n, alpha, a, a_len, lda, b,
                                  b_len, ldb, beta, c, c_len, ldc, nullptr, 0, call);
}

int uor_b200_gemm_partial_limbs(uor_b200_dtype elem, const uor_b200_view* a,
                                const uor_b200_view* b, int64_t* limbs, size_t limbs_len,
                                const uor_b200_call* call) {
    if (!a || !b) return UOR_B200_INVALID_ARGUMENT;
    if (elem != UOR_B200_I8 && elem != UOR_B200_I16 && elem != UOR_B200_I32)
        return UOR_B200_UNSUPPORTED;
    if (!device_ptrs(call)) return UOR_B200_INVALID_ARGUMENT;
    const size_t es = dtype_size(elem);
    Operand A, B;
    int st;
    if ((st = place_view(a->data, a->len, a->rows, a->cols, a->rs, a->cs, es, &A)) != UOR_B200_OK)
        return st;
    if ((st = place_view(b->data, b->len, b->rows, b->cols, b->rs, b->cs, es, &B)) != UOR_B200_OK)
        return st;
    if (a->cols != b->rows) return UOR_B200_NONCONFORMANT;
    const size_t m = a->rows, n = b->cols;
    if (m == 0 || n == 0) return UOR_B200_OK;
    if (!limbs) return UOR_B200_INVALID_ARGUMENT;
    if (limbs_len < SPLITK_LIMBS * m * n) return UOR_B200_DOES_NOT_FIT;
    uor_b200_ctx* ctx = resolve_ctx(call, &st);
    if (!ctx) return st;
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceTurn turn(ctx);
    uor_b200_route local_route{};
    uor_b200_route* route = call->route ? call->route : &local_route;
    *route = uor_b200_route{};
    // The exact partial sum, as an i128 matrix in a context buffer.
    void* x = ctx_buffer(ctx, SLOT_AUX, 16 * m * n, &st);
    if (!x) return st;
    if (a->cols == 0 && cudaMemsetAsync(x, 0, 16 * m * n, ctx->stream) != cudaSuccess)
        return UOR_B200_DEVICE_ERROR;
    Operand X;
    X.origin = static_cast<const uint8_t*>(x);
    X.lo = 0;
    X.hi = static_cast<ptrdiff_t>(m * n) - 1;
    X.rows = m;
    X.cols = n;
    X.rs = static_cast<ptrdiff_t>(n);
    X.cs = 1;
    X.es = 16;
    uor_b200_call inner = *call;
    inner.flags |= UOR_B200_ASYNC;  // the conversion below still runs on the same stream
    if ((st = int_gemm_locked(ctx, elem, OUT_I128, A, B, X, 1, 0, MODE_WRAPPING, &inner, route)) !=
        UOR_B200_OK)
        return st;
    if (i128_to_limbs(x, limbs, m * n, ctx->stream) != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    return finish_call(ctx, call);
}

int uor_b200_limbs_finish(uor_b200_dtype elem, uor_b200_dtype out, const int64_t* limbs,
                          size_t limbs_len, const uor_b200_view_mut* c, int64_t alpha,
                          int64_t beta, const uor_b200_call* call) {
    if (!c) return UOR_B200_INVALID_ARGUMENT;
    if (elem != UOR_B200_I8 && elem != UOR_B200_I16 && elem != UOR_B200_I32)
        return UOR_B200_UNSUPPORTED;
    int kind = 0, mode = 0;
    if (!int_out(out, &kind)) return UOR_B200_UNSUPPORTED;
    if (call_mode(call, &mode) != UOR_B200_OK) return UOR_B200_INVALID_ARGUMENT;
    if (!device_ptrs(call)) return UOR_B200_INVALID_ARGUMENT;
    Operand C;
    int st;
    if ((st = place_view(c->data, c->len, c->rows, c->cols, c->rs, c->cs, dtype_size(out), &C)) !=
        UOR_B200_OK)
        return st;
    if (self_aliases(c->rows, c->cols, c->rs, c->cs)) return UOR_B200_OUTPUT_ALIASES;
    const size_t m = c->rows, n = c->cols;
    if (m == 0 || n == 0) return UOR_B200_OK;
    if (!limbs) return UOR_B200_INVALID_ARGUMENT;
    if (limbs_len < SPLITK_LIMBS * m * n) return UOR_B200_DOES_NOT_FIT;
    uor_b200_ctx* ctx = resolve_ctx(call, &st);
    if (!ctx) return st;
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceTurn turn(ctx);
    if (call->route) *call->route = uor_b200_route{};
    const LinearEpi epi{alpha, beta, mode, kind};
    if (limbs_finish(limbs, m, n, const_cast<uint8_t*>(C.origin), C.rs, C.cs, epi, ctx->stream) !=
        cudaSuccess)
        return UOR_B200_DEVICE_ERROR;
    return finish_call(ctx, call);
}

}  // extern "C"
