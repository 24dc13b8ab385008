// capi_typed.cu -- one symbol per (element, output) pair: the slice face's
// monomorphisations (slice::gemm::<E, O>, crates/uor-matmul/src/slice.rs:184) with full
// strides and the raw face's conventions (raw::sgemm, crates/uor-matmul/src/raw.rs:45-64):
// a pointer names element (0,0), strides are element strides of either sign, m == 0 or
// n == 0 returns at once, and a view that cannot exist (its reach overflows, or the output
// maps two cells onto one) returns without writing (raw.rs:137-148). Each forwards to the
// generic entry of its family with the view that starts at the lowest element the
// pointer's strides reach, so the bytes are the generic entry's.
#include "internal.h"

namespace {

// The raw operand as a generic view: the buffer from the lowest element reached, its
// length the reach. False when the reach overflows.
bool raw_view(const void* p, size_t rows, size_t cols, ptrdiff_t rs, ptrdiff_t cs, size_t es,
              uor_b200_view* v) {
    ptrdiff_t lo = 0, hi = 0;
    if (!uor::view_extent(rows, cols, rs, cs, &lo, &hi)) return false;
    const bool empty = rows == 0 || cols == 0;
    v->data = empty ? p : static_cast<const uint8_t*>(p) + lo * static_cast<ptrdiff_t>(es);
    v->len = empty ? 0 : static_cast<size_t>(hi - lo) + 1;
    v->rows = rows;
    v->cols = cols;
    v->rs = rs;
    v->cs = cs;
    return true;
}

uor_b200_view_mut as_mut(const uor_b200_view& v) {
    return uor_b200_view_mut{const_cast<void*>(v.data), v.len, v.rows, v.cols, v.rs, v.cs};
}

// The three raw operands; false (nothing to do) for an empty product or a view that
// cannot exist.
bool raw_triple(size_t m, size_t k, size_t n, const void* a, ptrdiff_t rsa, ptrdiff_t csa, size_t ea,
                const void* b, ptrdiff_t rsb, ptrdiff_t csb, size_t eb, void* c, ptrdiff_t rsc,
                ptrdiff_t csc, size_t ec, uor_b200_view* A, uor_b200_view* B, uor_b200_view_mut* C) {
    if (m == 0 || n == 0) return false;
    uor_b200_view cv;
    if (!raw_view(a, m, k, rsa, csa, ea, A) || !raw_view(b, k, n, rsb, csb, eb, B) ||
        !raw_view(c, m, n, rsc, csc, ec, &cv))
        return false;
    if (uor::self_aliases(m, n, rsc, csc)) return false;
    *C = as_mut(cv);
    return true;
}

int raw_int(uor_b200_dtype elem, uor_b200_dtype out, size_t m, size_t k, size_t n, int64_t alpha,
            const void* a, ptrdiff_t rsa, ptrdiff_t csa, const void* b, ptrdiff_t rsb, ptrdiff_t csb,
            int64_t beta, void* c, ptrdiff_t rsc, ptrdiff_t csc, const uor_b200_call* call) {
    uor_b200_view A, B;
    uor_b200_view_mut C;
    if (!raw_triple(m, k, n, a, rsa, csa, uor::dtype_size(elem), b, rsb, csb, uor::dtype_size(elem), c,
                    rsc, csc, uor::dtype_size(out), &A, &B, &C))
        return UOR_B200_OK;
    return uor_b200_gemm(elem, out, &A, &B, &C, alpha, beta, call);
}

}  // namespace

extern "C" {

#define UOR_RAW_INT(NAME, ET, OT, EDT, ODT)                                                        \
    int NAME(size_t m, size_t k, size_t n, int64_t alpha, const ET* a, ptrdiff_t rsa, ptrdiff_t csa, \
             const ET* b, ptrdiff_t rsb, ptrdiff_t csb, int64_t beta, OT* c, ptrdiff_t rsc,        \
             ptrdiff_t csc, const uor_b200_call* call) {                                           \
        return raw_int(EDT, ODT, m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc, call); \
    }

UOR_RAW_INT(uor_b200_raw_gemm_i8_i32, int8_t, int32_t, UOR_B200_I8, UOR_B200_I32)
UOR_RAW_INT(uor_b200_raw_gemm_i8_i64, int8_t, int64_t, UOR_B200_I8, UOR_B200_I64)
UOR_RAW_INT(uor_b200_raw_gemm_i16_i64, int16_t, int64_t, UOR_B200_I16, UOR_B200_I64)
UOR_RAW_INT(uor_b200_raw_gemm_i32_i64, int32_t, int64_t, UOR_B200_I32, UOR_B200_I64)
UOR_RAW_INT(uor_b200_raw_gemm_i32_i128, int32_t, void, UOR_B200_I32, UOR_B200_I128)
UOR_RAW_INT(uor_b200_raw_gemm_i64_i128, int64_t, void, UOR_B200_I64, UOR_B200_I128)

#undef UOR_RAW_INT

int uor_b200_raw_gemm_trop_i8_i32(size_t m, size_t k, size_t n, uor_b200_trop alpha, const void* a,
                                  ptrdiff_t rsa, ptrdiff_t csa, const void* b, ptrdiff_t rsb,
                                  ptrdiff_t csb, uor_b200_trop beta, void* c, ptrdiff_t rsc,
                                  ptrdiff_t csc, const uor_b200_call* call) {
    uor_b200_view A, B;
    uor_b200_view_mut C;
    if (!raw_triple(m, k, n, a, rsa, csa, 2, b, rsb, csb, 2, c, rsc, csc, 8, &A, &B, &C))
        return UOR_B200_OK;
    return uor_b200_gemm_tropical(UOR_B200_TROP_I8, UOR_B200_TROP_I32, &A, &B, &C, alpha, beta, call);
}

int uor_b200_raw_coded_grid16_i8_i32(size_t m, size_t k, size_t n, int64_t alpha, const int8_t* a,
                                     ptrdiff_t rsa, ptrdiff_t csa, const uint8_t* codes,
                                     const int8_t* table, int64_t beta, int32_t* c, ptrdiff_t rsc,
                                     ptrdiff_t csc, const uor_b200_call* call) {
    uor_b200_view A, cv;
    if (m == 0 || n == 0) return UOR_B200_OK;
    if (!raw_view(a, m, k, rsa, csa, 1, &A) || !raw_view(c, m, n, rsc, csc, 4, &cv) ||
        uor::self_aliases(m, n, rsc, csc))
        return UOR_B200_OK;
    const uor_b200_view_mut C = as_mut(cv);
    return uor_b200_coded_gemm(UOR_B200_I32, &A, codes, k * (n / 2), k, n, 2, table, 16, &C,
                               alpha, beta, call);
}

int uor_b200_raw_tabulated_grid16_i8_i32(size_t m, size_t k, size_t n, int64_t alpha,
                                         const int8_t* a, ptrdiff_t rsa, ptrdiff_t csa,
                                         const uint8_t* codes, const int8_t* table, int64_t beta,
                                         int32_t* c, ptrdiff_t rsc, ptrdiff_t csc,
                                         const uor_b200_call* call) {
    uor_b200_view A, cv;
    if (m == 0 || n == 0) return UOR_B200_OK;
    if (!raw_view(a, m, k, rsa, csa, 1, &A) || !raw_view(c, m, n, rsc, csc, 4, &cv) ||
        uor::self_aliases(m, n, rsc, csc))
        return UOR_B200_OK;
    const uor_b200_view_mut C = as_mut(cv);
    return uor_b200_tabulated_gemm(UOR_B200_I32, &A, codes, n * (k / 2), k, n, 2, table, 16, &C,
                                   alpha, beta, call);
}

}  // extern "C"
