// capi_float.cu -- the exact float family's C ABI: the view API over f32/f64, the
// slice face (gemm_float_ex) and the raw face (sgemm / dgemm).
#include <climits>
#include "float_exact.h"
#include "internal.h"
#include "staging.h"

using namespace uor;

namespace {

bool float_type(uor_b200_dtype t) { return t == UOR_B200_F32 || t == UOR_B200_F64; }

int float_placed(uor_b200_dtype elem, uor_b200_dtype out, const Operand& A, const Operand& B,
                 const Operand& C, int64_t alpha, int64_t beta, int mode,
                 const uor_b200_call* call) {
    uor_b200_route local{};
    uor_b200_route* route = call && call->route ? call->route : &local;
    *route = uor_b200_route{};
    const size_t m = A.rows, k = A.cols, n = B.cols;
    if (m == 0 || n == 0) return UOR_B200_OK;
    int st = UOR_B200_OK;
    uor_b200_ctx* ctx = resolve_ctx(call, &st);
    if (!ctx) return st;
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceTurn turn(ctx);
    const bool dev = call && (call->flags & UOR_B200_DEVICE_POINTERS);
    const uint8_t *da = nullptr, *db = nullptr;
    OutStage cs;
    if ((st = stage_in(ctx, SLOT_A, A, dev, &da))) return st;
    if ((st = stage_in(ctx, SLOT_B, B, dev, &db))) return st;
    if ((st = stage_out_begin(ctx, C, dev, beta != 0, &cs))) return st;
    st = run_float_gemm(ctx, elem == UOR_B200_F64, out == UOR_B200_F64, da, A.rs, A.cs, db, B.rs,
                        B.cs, cs.dev_origin, C.rs, C.cs, m, k, n, alpha, beta, mode, route,
                        call ? call->flags & (UOR_B200_DIGIT_SLICES | UOR_B200_MODULAR) : 0u);
    if (st) return st;
    if ((st = stage_out_end(ctx, cs))) return st;
    if (!dev) return uor_b200_ctx_sync(ctx);
    return finish_call(ctx, call);
}

int float_views(uor_b200_dtype elem, uor_b200_dtype out, const void* a, size_t a_len, size_t am,
                size_t ak, ptrdiff_t rsa, ptrdiff_t csa, const void* b, size_t b_len, size_t bk,
                size_t bn, ptrdiff_t rsb, ptrdiff_t csb, void* c, size_t c_len, size_t cm,
                size_t cn, ptrdiff_t rsc, ptrdiff_t csc, int64_t alpha, int64_t beta,
                const uor_b200_call* call) {
    if (!float_type(elem) || !float_type(out)) return UOR_B200_UNSUPPORTED;
    const int mode = call ? (int)call->encode : MODE_NEAREST;
    if (mode < 0 || mode > 3) return UOR_B200_INVALID_ARGUMENT;
    Operand A, B, C;
    int st;
    if ((st = place_view(a, a_len, am, ak, rsa, csa, dtype_size(elem), &A))) return st;
    if ((st = place_view(b, b_len, bk, bn, rsb, csb, dtype_size(elem), &B))) return st;
    if ((st = place_view(c, c_len, cm, cn, rsc, csc, dtype_size(out), &C))) return st;
    if (ak != bk || cm != am || cn != bn) return UOR_B200_NONCONFORMANT;
    if (self_aliases(cm, cn, rsc, csc)) return UOR_B200_OUTPUT_ALIASES;
    return float_placed(elem, out, A, B, C, alpha, beta, mode, call);
}

// raw.rs:98-160: pointers name element (0,0); an unconstructible view or an
// aliasing output returns without writing.
int raw_gemm(uor_b200_dtype t, size_t m, size_t k, size_t n, int64_t alpha, const void* a,
             ptrdiff_t rsa, ptrdiff_t csa, const void* b, ptrdiff_t rsb, ptrdiff_t csb,
             int64_t beta, void* c, ptrdiff_t rsc, ptrdiff_t csc, const uor_b200_call* call) {
    if (m == 0 || n == 0) return UOR_B200_OK;
    const int mode = call ? (int)call->encode : MODE_NEAREST;
    if (mode < 0 || mode > 3) return UOR_B200_INVALID_ARGUMENT;
    const size_t es = dtype_size(t);
    Operand A, B, C;
    if (!raw_operand(a, m, k, rsa, csa, es, &A) || !raw_operand(b, k, n, rsb, csb, es, &B) ||
        !raw_operand(c, m, n, rsc, csc, es, &C))
        return UOR_B200_OK;
    if (self_aliases(m, n, rsc, csc)) return UOR_B200_OK;
    if ((k && (!a || !b)) || !c) return UOR_B200_INVALID_ARGUMENT;
    return float_placed(t, t, A, B, C, alpha, beta, mode, call);
}

}  // namespace

extern "C" {

int uor_b200_gemm_float(uor_b200_dtype elem, uor_b200_dtype out, const uor_b200_view* a,
                        const uor_b200_view* b, const uor_b200_view_mut* c, int64_t alpha,
                        int64_t beta, const uor_b200_call* call) {
    if (!a || !b || !c) return UOR_B200_INVALID_ARGUMENT;
    return float_views(elem, out, a->data, a->len, a->rows, a->cols, a->rs, a->cs, b->data,
                       b->len, b->rows, b->cols, b->rs, b->cs, c->data, c->len, c->rows, c->cols,
                       c->rs, c->cs, alpha, beta, call);
}

int uor_b200_slice_gemm_float_ex(uor_b200_dtype elem, uor_b200_dtype out, size_t m, size_t k,
                                 size_t n, int64_t alpha, const void* a, size_t a_len, size_t lda,
                                 const void* b, size_t b_len, size_t ldb, int64_t beta, void* c,
                                 size_t c_len, size_t ldc, void* pa, size_t pa_len, void* pb,
                                 size_t pb_len, const uor_b200_call* call) {
    (void)pa;
    (void)pa_len;
    (void)pb;
    (void)pb_len;  // PackedCode caches never change bytes (slice.rs:283-303)
    return float_views(elem, out, a, a_len, m, k, (ptrdiff_t)lda, 1, b, b_len, k, n,
                       (ptrdiff_t)ldb, 1, c, c_len, m, n, (ptrdiff_t)ldc, 1, alpha, beta, call);
}

int uor_b200_sgemm(size_t m, size_t k, size_t n, int64_t alpha, const float* a, ptrdiff_t rsa,
                   ptrdiff_t csa, const float* b, ptrdiff_t rsb, ptrdiff_t csb, int64_t beta,
                   float* c, ptrdiff_t rsc, ptrdiff_t csc, const uor_b200_call* call) {
    return raw_gemm(UOR_B200_F32, m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc, call);
}

int uor_b200_dgemm(size_t m, size_t k, size_t n, int64_t alpha, const double* a, ptrdiff_t rsa,
                   ptrdiff_t csa, const double* b, ptrdiff_t rsb, ptrdiff_t csb, int64_t beta,
                   double* c, ptrdiff_t rsc, ptrdiff_t csc, const uor_b200_call* call) {
    return raw_gemm(UOR_B200_F64, m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc, call);
}

}  // extern "C"
