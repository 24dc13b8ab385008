/*
 * uor_b200.h -- C ABI of the B200 exact-GEMM library (libuor_b200.so).
 *
 * A drop-in for the exact-accumulation GEMM path of uor-matmul (the Rust crate
 * UOR-Foundation/uor-matmul). Each entry point below names the reference
 * interface it replaces (path:line in that crate). The semantics are the
 * reference's: every product is accumulated exactly, the result is encoded
 * exactly once (saturate, wrap, or round-to-nearest-even for floats), and the
 * bytes written are the bytes the reference writes for the same inputs.
 *
 * Conventions
 *   - Plain pointers and sizes; no C++ or framework types cross this boundary.
 *   - Sizes and lengths are in ELEMENTS of the named dtype; strides are signed
 *     element strides (Strides { rs, cs }, crates/uor-matmul-core/src/layout.rs:29).
 *   - i128 values are 16-byte little-endian two's complement.
 *   - Trop<E> is the reference's repr(C) { E value; bool finite } struct
 *     (crates/uor-matmul-core/src/tropical.rs:61-70): 2, 4, 8, 16 bytes for
 *     E = i8, i16, i32, i64. The semiring zero stores value 0 and finite 0.
 *   - Pointers are host pointers unless the call sets UOR_B200_DEVICE_POINTERS.
 *     Host-pointer calls stage operands through the context's device buffers.
 *   - Every call is synchronous (returns after the result is in C) unless the
 *     call sets UOR_B200_ASYNC, which is honoured only with device pointers;
 *     an asynchronous call's device status is reported by uor_b200_ctx_sync.
 *   - The library never reads C when beta is zero (epilogue.rs:73-77) and never
 *     when a tropical beta is the semiring zero (epilogue.rs:166-170).
 */
#ifndef UOR_B200_H
#define UOR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */

/* 1 and 2 are NotAProduct's two variants (crates/uor-matmul-core/src/error.rs:104-131),
 * reported where Triple::new reports them (layout.rs:534-561). The others have no
 * reference counterpart except UOR_B200_DOES_NOT_FIT, which is the slice face's
 * `does_not_fit` panic (crates/uor-matmul/src/slice.rs:104-116) returned as a code. */
typedef enum uor_b200_status {
    UOR_B200_OK = 0,
    UOR_B200_NONCONFORMANT = 1,    /* NotAProduct::Nonconformant */
    UOR_B200_OUTPUT_ALIASES = 2,   /* NotAProduct::OutputAliasesItself */
    UOR_B200_DEVICE_ERROR = 3,     /* a CUDA runtime error */
    UOR_B200_TIMEOUT = 4,          /* a bounded device wait ran out */
    UOR_B200_NCCL_ERROR = 5,       /* reserved for collective-backed calls */
    UOR_B200_DOES_NOT_FIT = 6,     /* a buffer does not hold the view its caller described */
    UOR_B200_INVALID_ARGUMENT = 7, /* unknown enum value, or a null pointer with extent */
    UOR_B200_UNSUPPORTED = 8,      /* an element/output pair outside the reference's surface */
    UOR_B200_SCRATCH_LIMIT = 9     /* the no-allocation entry needs more than its fixed scratch */
} uor_b200_status;

/* EncodeMode, crates/uor-matmul-core/src/policy.rs:20-48. */
typedef enum uor_b200_encode {
    UOR_B200_NEAREST = 0,     /* default: round half to even; saturate integers */
    UOR_B200_TOWARD_ZERO = 1,
    UOR_B200_SATURATING = 2,
    UOR_B200_WRAPPING = 3
} uor_b200_encode;

/* Element and output types. */
typedef enum uor_b200_dtype {
    UOR_B200_I8 = 1,
    UOR_B200_I16 = 2,
    UOR_B200_I32 = 3,
    UOR_B200_I64 = 4,
    UOR_B200_I128 = 5,
    UOR_B200_F32 = 6,
    UOR_B200_F64 = 7,
    UOR_B200_TROP_I8 = 8,
    UOR_B200_TROP_I16 = 9,
    UOR_B200_TROP_I32 = 10,
    UOR_B200_TROP_I64 = 11
} uor_b200_dtype;

/* ----------------------------------------------------------------- context */

/* A device, a stream, device workspaces, and a status word for bounded waits.
 * Distinct contexts may be used from distinct threads concurrently. The library orders
 * its device work device-wide: each call's stream first waits for the work of the
 * previous call on the same device (whichever context, stream or thread queued it), so
 * calls on different streams run one after another on the GPU, never side by side.
 * Calls queued into a CUDA graph capture and the no-allocation entry take no part in
 * that order; their callers order them. */
typedef struct uor_b200_ctx uor_b200_ctx;

uor_b200_ctx *uor_b200_ctx_create(int device);
void uor_b200_ctx_destroy(uor_b200_ctx *ctx);
/* Run this context's work on `stream` (a cudaStream_t); NULL is CUDA's legacy
 * default stream. A new context runs on a private blocking stream: its calls are
 * ordered with the work the caller queues on the legacy default stream. */
int uor_b200_ctx_set_stream(uor_b200_ctx *ctx, void *stream);
/* Upper bound on any single device-side wait, in nanoseconds (default 2 s). */
int uor_b200_ctx_set_wait_budget_ns(uor_b200_ctx *ctx, uint64_t ns);
/* Wait for the context's stream; report a device timeout or error. */
int uor_b200_ctx_sync(uor_b200_ctx *ctx);

/* Which factorization ran: the analogue of Route / RouteCensus
 * (crates/uor-matmul-gemm/src/kernel.rs:419-484). */
typedef enum uor_b200_kernel {
    UOR_B200_KERNEL_NONE = 0,          /* nothing to compute (m == 0 or n == 0) */
    UOR_B200_KERNEL_I8_TCGEN05 = 1,    /* K1: s8 x s8 -> s32 TMEM, exact epilogue */
    UOR_B200_KERNEL_LIMB_TCGEN05 = 2,  /* K2: byte-sliced limb GEMMs, exact recombination */
    UOR_B200_KERNEL_TROPICAL = 3,      /* K4: packed max-plus on CUDA cores */
    UOR_B200_KERNEL_CODED_TCGEN05 = 4, /* K1C: codebook decode feeding K1's MMA */
    UOR_B200_KERNEL_FLOAT_EXACT = 5,   /* K6+K7: exact float, one rounding */
    UOR_B200_KERNEL_EPILOGUE_ONLY = 6, /* k == 0: C := encode(beta * C) */
    UOR_B200_KERNEL_SKINNY = 7         /* <= 16 rows or columns: dp4a reduce / column kernels */
} uor_b200_kernel;

typedef struct uor_b200_route {
    uint32_t kernel;      /* uor_b200_kernel */
    uint32_t tile_m, tile_n, tile_k;
    uint32_t k_chunks;    /* exact reduction chunks (lane depth, kernel.rs:1431) */
    uint32_t a_layout;    /* 0 K-major, 1 MN-major, 2 gathered to K-major */
    uint32_t b_layout;
    uint32_t ctas;        /* CTAs launched per chunk */
    uint32_t pairs;       /* int8 slice-pair GEMMs run on the tensor cores (1 for K1) */
    uint32_t fixups;      /* exact float: cells recomputed exactly after the lazy digits */
    uint32_t moduli;      /* exact float / wide integers: moduli of the modular route (0: slices) */
    uint32_t crt;         /* modular route: 1 when the CRT's columns ran on the tensor cores */
} uor_b200_route;

#define UOR_B200_DEVICE_POINTERS 1u
#define UOR_B200_ASYNC 2u
/* Exact float and wide integers (i16 .. i64, Complex): take the digit / byte-slice route
 * even where the modular route (residues modulo coprime moduli and the CRT) would run
 * fewer GEMMs. Both are exact; the bytes are the same. */
#define UOR_B200_DIGIT_SLICES 4u
/* Exact float and wide integers: take the modular route wherever its moduli cover the
 * product's bound, whatever the estimated cost. Exact; the same bytes. */
#define UOR_B200_MODULAR 8u
/* Codec tier (Packed<Grid<N>, 2>): decode the codes on chip only, never into a dense copy
 * of the coded operand in device memory. The codes are decoded on chip (K1's CTA-pair GEMM
 * with the codes decoded straight into its shared-memory B stages, in exact k chunks past
 * one s32 lane) except for reductions past one s32 lane with 512 rows or more and fewer
 * 512 x 256 output tiles than resident CTA pairs, which the default decodes once into a
 * k x n workspace; the flag keeps those on chip too. The same bytes either way. */
#define UOR_B200_CODEC_ON_CHIP 16u

/* Per-call options: GemmOptions' encode (crates/uor-matmul-gemm/src/driver.rs:13-20)
 * plus where the pointers live. A NULL call means: Nearest, host pointers,
 * the default context of the current device. */
typedef struct uor_b200_call {
    uint32_t encode;        /* uor_b200_encode */
    uint32_t flags;         /* DEVICE_POINTERS | ASYNC | DIGIT_SLICES | MODULAR | CODEC_ON_CHIP */
    uor_b200_ctx *ctx;      /* NULL: the current device's default context */
    uor_b200_route *route;  /* optional out */
} uor_b200_call;

/* ------------------------------------------------------------------- views */

/* MatView / MatViewMut (layout.rs:158-219): a buffer of `len` elements borrowed
 * as rows x cols with arbitrary strides. The origin is placed so that the
 * lowest offset the view reaches is element 0 of the buffer (layout.rs:178-199). */
typedef struct uor_b200_view {
    const void *data;
    size_t len;
    size_t rows, cols;
    ptrdiff_t rs, cs;
} uor_b200_view;

typedef struct uor_b200_view_mut {
    void *data;
    size_t len;
    size_t rows, cols;
    ptrdiff_t rs, cs;
} uor_b200_view_mut;

/* --------------------------------------------------------- integer family */

/* The view API's default entry: gemm_auto(&mut Triple, &Linear{alpha, beta},
 * GemmOptions, &mut Scratch) (crates/uor-matmul-gemm/src/kernel.rs:523-558,
 * re-exported as uor_matmul::gemm, crates/uor-matmul/src/lib.rs:135).
 * elem in {I8, I16, I32, I64}; out in {I8, I16, I32, I64, I128}.
 * Errors as Triple::new (layout.rs:534-561); DOES_NOT_FIT as MatView::new's None. */
int uor_b200_gemm(uor_b200_dtype elem, uor_b200_dtype out, const uor_b200_view *a,
                  const uor_b200_view *b, const uor_b200_view_mut *c, int64_t alpha,
                  int64_t beta, const uor_b200_call *call);

/* slice::gemm_ex (crates/uor-matmul/src/slice.rs:144-178): row-major with
 * leading dimensions; `scratch` is the caller's panel offer, accepted and
 * ignored (the offer never changes bytes, slice.rs:23-41). */
int uor_b200_slice_gemm_ex(uor_b200_dtype elem, uor_b200_dtype out, size_t m, size_t k, size_t n,
                           int64_t alpha, const void *a, size_t a_len, size_t lda, const void *b,
                           size_t b_len, size_t ldb, int64_t beta, void *c, size_t c_len,
                           size_t ldc, void *scratch, size_t scratch_len,
                           const uor_b200_call *call);

/* slice::gemm (slice.rs:184-199): contiguous, alpha 1, beta 0. */
int uor_b200_slice_gemm(uor_b200_dtype elem, uor_b200_dtype out, size_t m, size_t k, size_t n,
                        const void *a, size_t a_len, const void *b, size_t b_len, void *c,
                        size_t c_len, void *scratch, size_t scratch_len,
                        const uor_b200_call *call);

/* slice::gemm_ex_full / gemm_full (slice.rs:221-283): the accumulator offer is
 * accepted and ignored as well. */
int uor_b200_slice_gemm_ex_full(uor_b200_dtype elem, uor_b200_dtype out, size_t m, size_t k,
                                size_t n, int64_t alpha, const void *a, size_t a_len, size_t lda,
                                const void *b, size_t b_len, size_t ldb, int64_t beta, void *c,
                                size_t c_len, size_t ldc, void *panels, size_t panels_len,
                                void *accumulators, size_t accumulators_len,
                                const uor_b200_call *call);

/* The canonical W8A8 instantiation, monomorphised: slice::gemm::<i8, i32> and
 * slice::gemm_ex::<i8, i32>. */
int uor_b200_gemm_i8_i32(size_t m, size_t k, size_t n, const int8_t *a, const int8_t *b,
                         int32_t *c, const uor_b200_call *call);
int uor_b200_gemm_ex_i8_i32(size_t m, size_t k, size_t n, int64_t alpha, const int8_t *a,
                            size_t lda, const int8_t *b, size_t ldb, int64_t beta, int32_t *c,
                            size_t ldc, const uor_b200_call *call);

/* One symbol per (element, output) monomorphisation of gemm_auto (kernel.rs:523; the slice
 * face's slice::gemm::<E, O>, slice.rs:184) with the raw face's conventions
 * (raw::sgemm, crates/uor-matmul/src/raw.rs:45-64): a pointer names element (0,0), strides
 * are element strides of either sign, m == 0 or n == 0 returns at once, and a view that
 * cannot exist (an overflowing reach, or an output that maps two cells onto one) returns
 * without writing (raw.rs:137-148). C := encode(alpha A B + beta C) as uor_b200_gemm.
 * i128 outputs are 16-byte little-endian two's complement; i64 elements accumulate in
 * Limbs<3> (acc.rs:215-402) and encode into i128. */
int uor_b200_raw_gemm_i8_i32(size_t m, size_t k, size_t n, int64_t alpha, const int8_t *a,
                             ptrdiff_t rsa, ptrdiff_t csa, const int8_t *b, ptrdiff_t rsb,
                             ptrdiff_t csb, int64_t beta, int32_t *c, ptrdiff_t rsc, ptrdiff_t csc,
                             const uor_b200_call *call);
int uor_b200_raw_gemm_i8_i64(size_t m, size_t k, size_t n, int64_t alpha, const int8_t *a,
                             ptrdiff_t rsa, ptrdiff_t csa, const int8_t *b, ptrdiff_t rsb,
                             ptrdiff_t csb, int64_t beta, int64_t *c, ptrdiff_t rsc, ptrdiff_t csc,
                             const uor_b200_call *call);
int uor_b200_raw_gemm_i16_i64(size_t m, size_t k, size_t n, int64_t alpha, const int16_t *a,
                              ptrdiff_t rsa, ptrdiff_t csa, const int16_t *b, ptrdiff_t rsb,
                              ptrdiff_t csb, int64_t beta, int64_t *c, ptrdiff_t rsc,
                              ptrdiff_t csc, const uor_b200_call *call);
int uor_b200_raw_gemm_i32_i64(size_t m, size_t k, size_t n, int64_t alpha, const int32_t *a,
                              ptrdiff_t rsa, ptrdiff_t csa, const int32_t *b, ptrdiff_t rsb,
                              ptrdiff_t csb, int64_t beta, int64_t *c, ptrdiff_t rsc,
                              ptrdiff_t csc, const uor_b200_call *call);
int uor_b200_raw_gemm_i32_i128(size_t m, size_t k, size_t n, int64_t alpha, const int32_t *a,
                               ptrdiff_t rsa, ptrdiff_t csa, const int32_t *b, ptrdiff_t rsb,
                               ptrdiff_t csb, int64_t beta, void *c, ptrdiff_t rsc, ptrdiff_t csc,
                               const uor_b200_call *call);
int uor_b200_raw_gemm_i64_i128(size_t m, size_t k, size_t n, int64_t alpha, const int64_t *a,
                               ptrdiff_t rsa, ptrdiff_t csa, const int64_t *b, ptrdiff_t rsb,
                               ptrdiff_t csb, int64_t beta, void *c, ptrdiff_t rsc, ptrdiff_t csc,
                               const uor_b200_call *call);

/* driver::gemm (crates/uor-matmul-gemm/src/driver.rs:67-79) over Complex<elem>
 * (crates/uor-matmul-core/src/alphabet.rs:656-776), encoding into Complex<out>
 * componentwise (EncodeFrom<ComplexAcc>, alphabet.rs:765-776). elem in {I32, I64}
 * (accumulators i128 and Limbs<3> per part); out in {I8, I16, I32, I64, I128}.
 * Buffers hold repr(C) {re, im} pairs; len, rows, cols and strides count complex
 * elements. The mac is re += a.re*w.re + a.im*(-w.im), im += a.re*w.im + a.im*w.re
 * with -w.im negated modulo 2^bits (the release build's negation: -MIN is MIN).
 * alpha and beta scale each part as Linear scales a scalar accumulator; alpha = 1,
 * beta = 0 is the plain encode. */
int uor_b200_gemm_complex(uor_b200_dtype elem, uor_b200_dtype out, const uor_b200_view *a,
                          const uor_b200_view *b, const uor_b200_view_mut *c, int64_t alpha,
                          int64_t beta, const uor_b200_call *call);

/* ----------------------------------------------------------- float family */

/* gemm_float_packed over a Triple (crates/uor-matmul-gemm/src/float.rs:1824)
 * with Linear: C := RNE-once(alpha * exact(A B) + beta * C).
 * elem in {F32, F64}; out in {F32, F64}. Also the entry for gemm_float
 * (float.rs:1761) and gemm_float_bridged (float.rs:1897): their pa/pb, scaled
 * and scratch offers are caches that never change bytes, so none is passed here,
 * and the size queries suggested_float_panels / suggested_bridge_scaled
 * (float.rs:1862-1882) have no device counterpart -- any offer, empty included,
 * gives these bytes. */
int uor_b200_gemm_float(uor_b200_dtype elem, uor_b200_dtype out, const uor_b200_view *a,
                        const uor_b200_view *b, const uor_b200_view_mut *c, int64_t alpha,
                        int64_t beta, const uor_b200_call *call);

/* slice::gemm_float_ex / gemm_float (slice.rs:304-429); pa/pb are the caller's
 * PackedCode caches (16 bytes each), accepted and ignored. */
int uor_b200_slice_gemm_float_ex(uor_b200_dtype elem, uor_b200_dtype out, size_t m, size_t k,
                                 size_t n, int64_t alpha, const void *a, size_t a_len, size_t lda,
                                 const void *b, size_t b_len, size_t ldb, int64_t beta, void *c,
                                 size_t c_len, size_t ldc, void *pa, size_t pa_len, void *pb,
                                 size_t pb_len, const uor_b200_call *call);

/* raw::sgemm / raw::dgemm (crates/uor-matmul/src/raw.rs:45-90): matrixmultiply's
 * signature with exact integer alpha/beta and arbitrary (even negative) strides;
 * a pointer names element (0,0). m == 0 or n == 0 returns at once, and a view
 * that cannot exist returns without writing (raw.rs:137-148). */
int uor_b200_sgemm(size_t m, size_t k, size_t n, int64_t alpha, const float *a, ptrdiff_t rsa,
                   ptrdiff_t csa, const float *b, ptrdiff_t rsb, ptrdiff_t csb, int64_t beta,
                   float *c, ptrdiff_t rsc, ptrdiff_t csc, const uor_b200_call *call);
int uor_b200_dgemm(size_t m, size_t k, size_t n, int64_t alpha, const double *a, ptrdiff_t rsa,
                   ptrdiff_t csa, const double *b, ptrdiff_t rsb, ptrdiff_t csb, int64_t beta,
                   double *c, ptrdiff_t rsc, ptrdiff_t csc, const uor_b200_call *call);

/* -------------------------------------------------------- tropical family */

/* A Trop<i64> scalar for MaxPlus (crates/uor-matmul-gemm/src/epilogue.rs:137-186). */
typedef struct uor_b200_trop {
    int64_t value;
    uint32_t finite; /* 0: the semiring zero (-inf) */
} uor_b200_trop;

/* driver::gemm over Alphabet<Trop<E>, _> with MaxPlus{alpha, beta}
 * (crates/uor-matmul-gemm/src/driver.rs:67-182): C := (alpha (x) A(x)B) (+) (beta (x) C)
 * in (max, +). elem in {TROP_I8, TROP_I16}; out in {TROP_I8 .. TROP_I64}. */
int uor_b200_gemm_tropical(uor_b200_dtype elem, uor_b200_dtype out, const uor_b200_view *a,
                           const uor_b200_view *b, const uor_b200_view_mut *c,
                           uor_b200_trop alpha, uor_b200_trop beta, const uor_b200_call *call);

/* driver::gemm_selected (crates/uor-matmul-gemm/src/selection.rs:212-330): the same
 * product, and beside it a witness matrix (u64 elements, m x n, its own strides): for
 * each cell the least index p attaining the maximum of the reduction (D-6's tie-break),
 * or 0 when every term is the semiring zero or k is 0. The witness is of the reduction,
 * before MaxPlus. A witness of another shape is NONCONFORMANT; one whose strides map two
 * cells onto one is OUTPUT_ALIASES (SelectedTriple::new). */
int uor_b200_gemm_tropical_selected(uor_b200_dtype elem, uor_b200_dtype out,
                                    const uor_b200_view *a, const uor_b200_view *b,
                                    const uor_b200_view_mut *c, const uor_b200_view_mut *witness,
                                    uor_b200_trop alpha, uor_b200_trop beta,
                                    const uor_b200_call *call);

/* uor_b200_gemm_tropical for Trop<i8> -> Trop<i32> with the raw face's
 * conventions (see uor_b200_raw_gemm_i8_i32): a and b are Trop<i8> (2 bytes each), c is
 * Trop<i32> (8 bytes), strides count those elements. */
int uor_b200_raw_gemm_trop_i8_i32(size_t m, size_t k, size_t n, uor_b200_trop alpha,
                                  const void *a, ptrdiff_t rsa, ptrdiff_t csa, const void *b,
                                  ptrdiff_t rsb, ptrdiff_t csb, uor_b200_trop beta, void *c,
                                  ptrdiff_t rsc, ptrdiff_t csc, const uor_b200_call *call);

/* ----------------------------------------------------------- codec family */

/* coded_gemm (crates/uor-matmul-gemm/src/coded.rs:98-142) with B a CodedMatrix
 * (crates/uor-matmul-codec/src/matrix.rs:15-219) of Packed<Grid<N>, P> codes
 * (codecs.rs:80-196): B is k x n, each byte holds P sub-codes of 8/P bits, low
 * sub-code first; element (r, c) decodes table[sub % N] with
 * sub = (codes[r * (n / P) + c / P] >> ((8 / P) * (c % P))) & mask.
 * A is a dense i8 view; out in {I8 .. I128}. P in {1, 2, 4, 8}; 1 <= N <= 256. P = 2 with
 * N <= 16, and P = 4 or 8 with code rows of whole 16-byte strides, decode on chip (K1C,
 * see UOR_B200_CODEC_ON_CHIP); the rest decode to a dense workspace first. */
int uor_b200_coded_gemm(uor_b200_dtype out, const uor_b200_view *a, const uint8_t *codes,
                        size_t codes_len, size_t k, size_t n, uint32_t per_byte,
                        const int8_t *table, size_t table_len, const uor_b200_view_mut *c,
                        int64_t alpha, int64_t beta, const uor_b200_call *call);

/* gemm_tabulated's product (crates/uor-matmul-gemm/src/tabulated.rs:600-660, 2555):
 * the same codec with W coded n x k (one coded row per output column), C = A W^T. */
int uor_b200_tabulated_gemm(uor_b200_dtype out, const uor_b200_view *a, const uint8_t *codes,
                            size_t codes_len, size_t k, size_t n, uint32_t per_byte,
                            const int8_t *table, size_t table_len, const uor_b200_view_mut *c,
                            int64_t alpha, int64_t beta, const uor_b200_call *call);

/* coded_gemm / gemm_tabulated for Packed<Grid<16>, 2> into i32 with the raw
 * face's conventions for A and C (see uor_b200_raw_gemm_i8_i32): codes are the whole
 * CodedMatrix, k x n (coded: k * n / 2 bytes, row-major) or n x k (tabulated: n * k / 2
 * bytes), table its 16 entries; n (coded) or k (tabulated) even. */
int uor_b200_raw_coded_grid16_i8_i32(size_t m, size_t k, size_t n, int64_t alpha,
                                     const int8_t *a, ptrdiff_t rsa, ptrdiff_t csa,
                                     const uint8_t *codes, const int8_t *table, int64_t beta,
                                     int32_t *c, ptrdiff_t rsc, ptrdiff_t csc,
                                     const uor_b200_call *call);
int uor_b200_raw_tabulated_grid16_i8_i32(size_t m, size_t k, size_t n, int64_t alpha,
                                         const int8_t *a, ptrdiff_t rsa, ptrdiff_t csa,
                                         const uint8_t *codes, const int8_t *table, int64_t beta,
                                         int32_t *c, ptrdiff_t rsc, ptrdiff_t csc,
                                         const uor_b200_call *call);

/* The other fixed-width tiers (crates/uor-matmul-codec/src/codecs.rs) through one
 * descriptor, and Offset<C, zero> over any of them (decoded value minus zero, the image
 * staying within i8, codecs.rs Offset::new). */
typedef enum uor_b200_codec_tier {
    UOR_B200_TIER_GRID = 0,    /* Packed<Grid<N>, P>: as uor_b200_coded_gemm (codecs.rs:80-196) */
    UOR_B200_TIER_SIGN = 1,    /* Sign<BLK, K>: bit t of the code is element t, set +1, clear -1,
                                  bits past the code's width -1 (codecs.rs:341-437) */
    UOR_B200_TIER_TERNARY = 2, /* Ternary<BLK, K>: digit t (bits 2t, 2t+1): 0 -> -1, 2 -> +1,
                                  1 and 3 -> 0; a digit past the code's width reads 0, so -1
                                  (codecs.rs:438-520) */
    UOR_B200_TIER_BOOK = 3     /* Book<N, BLK, K>: element t of block code q is table[q % N][t]
                                  (codecs.rs:268-308) */
} uor_b200_codec_tier;

typedef struct uor_b200_codec {
    uint32_t tier;        /* uor_b200_codec_tier */
    uint32_t per_byte;    /* GRID: sub-codes per byte P */
    uint32_t block;       /* SIGN / TERNARY / BOOK: elements per code (BLK) */
    uint32_t code_bytes;  /* SIGN / TERNARY / BOOK: 1 (u8 codes) or 2 (u16, little-endian) */
    const int8_t *table;  /* GRID: N entries; BOOK: N x BLK entries, row per code; else unused */
    size_t table_len;     /* N */
    int32_t zero;         /* Offset: subtracted from every decoded value (0: no offset) */
} uor_b200_codec;

/* coded_gemm (orientation 0: codes describe B, k x n) or gemm_tabulated's A W^T
 * (orientation 1: codes describe W, n x k) for any tier above. The codes hold exactly
 * rows * (cols / BLK) codes (CodedMatrix::new, matrix.rs:36-60), else DOES_NOT_FIT; a
 * table whose offset image leaves i8 is INVALID_ARGUMENT. Code bytes of whole elements
 * (SIGN with BLK = 8 K, TERNARY with BLK = 4 K, BOOK with K = 1 and BLK 4 or 8) are
 * decoded inside the tensor-core pipeline when cols is a multiple of 16 x the elements
 * per code byte (route b_layout 1 or 0; past one s32 lane in exact k chunks, route
 * k_chunks); other shapes decode once into a dense workspace (b_layout 3). The bytes of C
 * are the same either way. */
int uor_b200_codec_gemm(uor_b200_dtype out, const uor_b200_view *a, const uor_b200_codec *codec,
                        const uint8_t *codes, size_t codes_len, size_t k, size_t n,
                        uint32_t orientation, const uor_b200_view_mut *c, int64_t alpha,
                        int64_t beta, const uor_b200_call *call);

/* e8_table (crates/uor-matmul-codec/src/e8.rs:295-307): the E8 lattice codebook, 256
 * codewords of 8 i8 (2048 bytes, row per code, code 0 the origin) for TIER_BOOK with
 * block 8 -- e8_codec (u16 codes) or e8_codec_u8 (u8 codes). `bound` is the alphabet's
 * magnitude bound (0: Full<i8>); a bound below 32 admits no table: UNSUPPORTED, the
 * reference's None. DOES_NOT_FIT when len < 2048. Host only; no device work. */
int uor_b200_e8_table(uint32_t bound, int8_t *out, size_t len);

/* coded_gemm / gemm_tabulated over Arena<E, N, K> (crates/uor-matmul-codec/src/
 * codecs.rs:894-985): each code (u8, code_bytes 1, or u16 little-endian, 2) indexes a
 * table of N float symbols of elem's type modulo N, one element per code; the product
 * with a float A is gemm_float's (exact accumulation, one rounding). elem in {F32, F64}
 * names A's and the table's type, out in {F32, F64}. codes_len is in bytes and must be
 * exactly k * n * code_bytes (CodedMatrix::new), else DOES_NOT_FIT; orientation 0: codes
 * k x n, 1: codes n x k. */
int uor_b200_arena_gemm(uor_b200_dtype elem, uor_b200_dtype out, const uor_b200_view *a,
                        const void *table, size_t table_len, const uint8_t *codes,
                        size_t codes_len, uint32_t code_bytes, size_t k, size_t n,
                        uint32_t orientation, const uor_b200_view_mut *c, int64_t alpha,
                        int64_t beta, const uor_b200_call *call);

/* canonicalize (codecs.rs:990-1003): sort `len` float symbols of elem's type in place by
 * their bit patterns as unsigned integers and move the distinct patterns to the front;
 * *distinct receives their count, values[0 .. *distinct) is the Arena table. -0.0 and
 * +0.0, and NaNs with different payloads, are distinct symbols. Host only. */
int uor_b200_arena_canonicalize(uor_b200_dtype elem, void *values, size_t len, size_t *distinct);

/* ------------------------------------------------- split-K across devices */

/* The exact partial sum of one device's share of a split reduction, for an exchange
 * between devices (NCCL all-reduce, sum of int64). No reference counterpart: the
 * reference runs on one host; this extends its exact chunk fold (run_chunked_depth,
 * crates/uor-matmul-gemm/src/kernel.rs:1431) across devices, with the independent
 * tiles of Partition (partition.rs:34) handling the other axis.
 *
 * limbs[(i * n + j) * 3 + t] receives X_ij = sum_p a_ip b_pj (over the views given:
 * pass A's columns and B's rows of this device's reduction range) as
 *   X = l0 + l1 2^40 + l2 2^80,  l0, l1 in [0, 2^40),  l2 = X >> 80 (arithmetic),
 * so elementwise int64 sums over devices stay exact. elem in {I8, I16, I32} (their
 * accumulator is i128); device pointers required (UOR_B200_DEVICE_POINTERS);
 * limbs_len counts int64 entries (>= 3 m n). */
int uor_b200_gemm_partial_limbs(uor_b200_dtype elem, const uor_b200_view *a,
                                const uor_b200_view *b, int64_t *limbs, size_t limbs_len,
                                const uor_b200_call *call);

/* C := encode(alpha * X + beta * C) from summed limbs (as above), with the Linear
 * epilogue of elem's i128 accumulator (epilogue.rs:79-93, 280-288): the total is
 * encoded once, so a split-K product has the single-device bytes. Device pointers. */
int uor_b200_limbs_finish(uor_b200_dtype elem, uor_b200_dtype out, const int64_t *limbs,
                          size_t limbs_len, const uor_b200_view_mut *c, int64_t alpha,
                          int64_t beta, const uor_b200_call *call);

/* ------------------------------------------- tropical split-K exchange */

/* driver::gemm over Trop<E> (crates/uor-matmul-gemm/src/driver.rs:102-182) with the
 * reduction cut into ranges, e.g. one per device: the (max, +) reduction of A and B's
 * views (one range of the reduction) as int64 keys, keys[i n + j], row-major, with
 * INT64_MIN where no pair of finite terms exists (the semiring zero). The element-wise
 * maximum of several ranges' keys (an all-reduce with MAX) is the reduction over their
 * union, because max is associative and commutative -- the tropical Partition's
 * split-K form (partition.rs:34-111). elem in {TROP_I8, TROP_I16, TROP_I32} (every sum
 * fits in int64). Device pointers only (call->flags DEVICE_POINTERS). */
int uor_b200_trop_partial_keys(uor_b200_dtype elem, const uor_b200_view *a,
                               const uor_b200_view *b, int64_t *keys, size_t keys_len,
                               const uor_b200_call *call);
/* MaxPlus::finish (epilogue.rs:137-186) and the tropical encode (tropical.rs:336-351)
 * from summed keys: C := (alpha (x) X) (+) (beta (x) C) with X the keys (INT64_MIN =
 * -inf); out in {TROP_I8 .. TROP_I64}. Device pointers only. */
int uor_b200_trop_keys_finish(uor_b200_dtype out, const int64_t *keys, size_t keys_len,
                              const uor_b200_view_mut *c, uor_b200_trop alpha, uor_b200_trop beta,
                              const uor_b200_call *call);

/* ------------------------------------------------ split-K over NCCL */

/* The exchanges above driven from here: one process (or thread) per GPU, each with its
 * own context, all in one NCCL communicator (an ncclComm_t, passed as void*). Each rank
 * passes A's columns and B's rows of its own range of the reduction and the whole C;
 * the entry computes its partial, all-reduces it in place on the context's stream (sum
 * of int64 limbs; max of int64 keys for Trop<E>) and encodes the total once, so every
 * rank's C receives the single-device bytes. The three steps are queued on the context's
 * stream without a host round trip; the call returns when C is written unless it sets
 * UOR_B200_ASYNC. Every rank must make the same calls in the same order (NCCL's rule).
 * Device pointers only (call->flags DEVICE_POINTERS); the communicator's device must be
 * the context's. NCCL is loaded on first use (libnccl.so.2, the one the process already
 * has if any); without it these return UOR_B200_NCCL_ERROR, as they do for an NCCL
 * failure. route, when given, reports the partial's kernel. A rank whose own partial
 * fails (an argument its peers did not share) still joins the all-reduce, so no peer
 * waits on it, and returns that status; in a synchronous call every other rank then
 * returns UOR_B200_NCCL_ERROR (its C is not the product). The checks before the exchange
 * (communicator, device, m and n, the exchange buffer) fail on every rank alike when the
 * ranks' calls agree in m, n and elem, as NCCL requires. */
int uor_b200_gemm_splitk_nccl(void *comm, uor_b200_dtype elem, uor_b200_dtype out,
                              const uor_b200_view *a, const uor_b200_view *b,
                              const uor_b200_view_mut *c, int64_t alpha, int64_t beta,
                              const uor_b200_call *call);
int uor_b200_gemm_tropical_splitk_nccl(void *comm, uor_b200_dtype elem, uor_b200_dtype out,
                                       const uor_b200_view *a, const uor_b200_view *b,
                                       const uor_b200_view_mut *c, uor_b200_trop alpha,
                                       uor_b200_trop beta, const uor_b200_call *call);
/* A communicator without linking NCCL: rank 0 makes the 128-byte id, the caller hands it
 * to every rank (any channel), each rank joins on its context's device (NULL: the
 * current device's default context). */
int uor_b200_nccl_unique_id(uint8_t *id, size_t id_len);
int uor_b200_nccl_comm_init(uor_b200_ctx *ctx, int nranks, const uint8_t *id, size_t id_len,
                            int rank, void **comm);
int uor_b200_nccl_comm_destroy(void *comm);

/* ------------------------------------------------- no-allocation variant */

/* Size of the fixed device scratch the no-allocation entry point uses. */
#define UOR_B200_NOALLOC_SCRATCH_BYTES (16u << 20)

/* Exact i8 x i8 GEMM (gemm_ex semantics, row-major, device pointers) that never
 * allocates memory. This entry point has no counterpart in the reference; it exists
 * for callers that cannot let a library call cudaMalloc: callers that budget every
 * byte of device memory once at start-up (an inference server's fixed pool, another
 * allocator owning the device), callers built on the reference's own zero-allocation
 * contract, and code that must not make allocating CUDA calls at all.
 *
 * Reductions deeper than one s32 lane (k > 131071) are cut into exact chunks whose
 * partial sums live in one static device array of UOR_B200_NOALLOC_SCRATCH_BYTES,
 * which every GPU that loads this library holds until the process exits. A product
 * needing more (chunks * m * n * 4 bytes + 256) is refused with UOR_B200_SCRATCH_LIMIT.
 * The first call on a device looks up the array's device address (set-up done once
 * per device); make that first call before any stream capture. The address is kept for
 * the life of the process, so a cudaDeviceReset after the first call on a device is not
 * supported (the rebuilt context would not hold the cached address). Every call shares the
 * array, so calls that overlap on the GPU (other streams, other threads) race on it:
 * serialise them. Operands must be TMA-readable as given (16-byte-aligned pointers,
 * lda and ldb multiples of 16) or the call returns UOR_B200_UNSUPPORTED. Runs on
 * `stream` (NULL = legacy default stream) and returns after the result is in C.
 * out in {I8, I16, I32, I64, I128}; encode as uor_b200_encode. */
int uor_b200_gemm_ex_i8_noalloc(uor_b200_dtype out, size_t m, size_t k, size_t n,
                                int64_t alpha, const int8_t *a, size_t lda, const int8_t *b,
                                size_t ldb, int64_t beta, void *c, size_t ldc, uint32_t encode,
                                void *stream);

/* ----------------------------------------------------------------- misc */

const char *uor_b200_status_string(int status);
/* ABI version: major * 10000 + minor * 100 + patch. */
int uor_b200_version(void);
/* Self-test of the bounded-wait path: launches a kernel that waits on a barrier
 * nothing will complete, with the given budget; returns UOR_B200_TIMEOUT when
 * the wait gave up as designed, and leaves the context usable. */
int uor_b200_selftest_wait_timeout(uor_b200_ctx *ctx, uint64_t budget_ns);

#ifdef __cplusplus
}
#endif

#endif /* UOR_B200_H */
