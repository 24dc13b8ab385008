/*
 * uor_oracle.c -- CPU restatement of uor-matmul's exact-GEMM semantics.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker the CUDA path is compared
 * against (tests/, __graft_entry__.smoke(), and bench.py's cpu_baseline /
 * --impl reference legs). The product library never links, loads or calls it.
 *
 * Every routine restates one piece of the reference (UOR-Foundation/uor-matmul,
 * a Rust crate that cannot be built here: no cargo/rustc) and cites the file and
 * line it follows. The restatement computes the same function by the simplest
 * exact means available in C: __int128 and fixed-width limb arrays.
 *
 * Pinning: the integer path (i64 elements, Wrapping encode) and the tropical
 * path are checked byte-for-byte against the reference's committed NumPy golden
 * vectors (oracles/numpy, CX-10; oracles/tropical, CX-11) and against the KATs
 * in the reference's unit tests (tests/test_oracle_golden.py). The float path is
 * checked against an independent Python big-integer twin (oracle/oracle.py) and
 * against the reference's float encode KATs.
 *
 * Views are "origin" views: a pointer to element (0,0) and signed element
 * strides, as raw.rs:98-160 builds them. Buffer placement (layout.rs:178) and
 * the alias check (layout.rs:116) are host logic, restated in oracle/oracle.py.
 */
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef __int128 i128;
typedef unsigned __int128 u128;

#define I128_MAX ((i128)(((u128)1 << 127) - 1))
#define I128_MIN (-I128_MAX - 1)

/* EncodeMode, policy.rs:20-48. */
enum { MODE_NEAREST = 0, MODE_TOWARD_ZERO = 1, MODE_SATURATING = 2, MODE_WRAPPING = 3 };

static void set_threads(int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
}

/* ------------------------------------------------------------------------- */
/* Integer family                                                            */
/* ------------------------------------------------------------------------- */

static inline i128 load_int(const void *p, int bits, ptrdiff_t off) {
    switch (bits) {
    case 8: return ((const int8_t *)p)[off];
    case 16: return ((const int16_t *)p)[off];
    case 32: return ((const int32_t *)p)[off];
    case 64: return ((const int64_t *)p)[off];
    default: return ((const i128 *)p)[off];
    }
}

static inline void store_int(void *p, int bits, ptrdiff_t off, i128 v) {
    switch (bits) {
    case 8: ((int8_t *)p)[off] = (int8_t)v; break;
    case 16: ((int16_t *)p)[off] = (int16_t)v; break;
    case 32: ((int32_t *)p)[off] = (int32_t)v; break;
    case 64: ((int64_t *)p)[off] = (int64_t)v; break;
    default: ((i128 *)p)[off] = v; break;
    }
}

static inline i128 out_min(int bits) { return bits >= 128 ? I128_MIN : -((i128)1 << (bits - 1)); }
static inline i128 out_max(int bits) { return bits >= 128 ? I128_MAX : ((i128)1 << (bits - 1)) - 1; }

/* encode_i128_into, acc.rs:128-151: Wrapping reduces modulo the range span,
 * every other mode clamps. */
static i128 encode_i128_into(i128 acc, i128 mn, i128 mx, int mode) {
    if (mode == MODE_WRAPPING) {
        if (mn == I128_MIN && mx == I128_MAX) return acc;
        u128 span = (u128)mx - (u128)mn + 1;
        u128 off = (u128)acc - (u128)mn;
        return (i128)((off % span) + (u128)mn);
    }
    if (acc < mn) return mn;
    if (acc > mx) return mx;
    return acc;
}

/* i128::saturating_mul, the ScaleExact impl for i128 (epilogue.rs:280-288). */
static i128 sat_mul_i128(i128 a, int64_t f) {
    if (a == 0 || f == 0) return 0;
    u128 ua = a < 0 ? (u128)0 - (u128)a : (u128)a;
    u128 uf = f < 0 ? (u128)0 - (u128)(i128)f : (u128)(i128)f;
    int neg = (a < 0) != (f < 0);
    /* overflow iff ua * uf > limit */
    u128 limit = neg ? ((u128)1 << 127) : (((u128)1 << 127) - 1);
    if (ua > limit / uf) return neg ? I128_MIN : I128_MAX;
    u128 p = ua * uf;
    if (p > limit) return neg ? I128_MIN : I128_MAX;
    return neg ? (i128)((u128)0 - p) : (i128)p;
}

/* Limbs<3>: 192-bit two's complement, the accumulator of i64 (alphabet.rs:618-637,
 * acc.rs:215-402). */
typedef struct { uint64_t w[3]; } limbs3;

static inline void l3_add_i128(limbs3 *x, i128 v) {
    /* add_i128, acc.rs:354-378: sign-extended addend, carry through all limbs. */
    uint64_t ext = v < 0 ? ~(uint64_t)0 : 0;
    u128 uv = (u128)v;
    uint64_t add[3] = {(uint64_t)uv, (uint64_t)(uv >> 64), ext};
    unsigned carry = 0;
    for (int i = 0; i < 3; i++) {
        u128 s = (u128)x->w[i] + add[i] + carry;
        x->w[i] = (uint64_t)s;
        carry = (unsigned)(s >> 64);
    }
}

static inline limbs3 l3_combine(limbs3 a, limbs3 b) {
    limbs3 r;
    unsigned carry = 0;
    for (int i = 0; i < 3; i++) {
        u128 s = (u128)a.w[i] + b.w[i] + carry;
        r.w[i] = (uint64_t)s;
        carry = (unsigned)(s >> 64);
    }
    return r;
}

static inline limbs3 l3_neg(limbs3 a) {
    limbs3 r;
    unsigned carry = 1;
    for (int i = 0; i < 3; i++) {
        u128 s = (u128)(~a.w[i]) + carry;
        r.w[i] = (uint64_t)s;
        carry = (unsigned)(s >> 64);
    }
    return r;
}

/* ScaleExact for Limbs (epilogue.rs:307-329): double-and-add, modulo 2^192. */
static limbs3 l3_scale(limbs3 x, int64_t f) {
    int negf = f < 0;
    uint64_t mag = negf ? (uint64_t)0 - (uint64_t)f : (uint64_t)f;
    limbs3 acc = {{0, 0, 0}};
    limbs3 addend = negf ? l3_neg(x) : x;
    while (mag) {
        if (mag & 1) acc = l3_combine(acc, addend);
        addend = l3_combine(addend, addend);
        mag >>= 1;
    }
    return acc;
}

/* EncodeFrom<Limbs<L>> for a machine integer (acc.rs:405-444). */
static i128 l3_encode(limbs3 x, int obits, int mode) {
    i128 low = (i128)(((u128)x.w[1] << 64) | x.w[0]);
    if (mode == MODE_WRAPPING) return low; /* truncation by the store */
    int negative = (int)(x.w[2] >> 63);
    limbs3 m = negative ? l3_neg(x) : x;
    int exceeded = m.w[2] != 0;
    i128 mn = out_min(obits), mx = out_max(obits);
    if (exceeded) return negative ? mn : mx;
    u128 mag = ((u128)m.w[1] << 64) | m.w[0];
    u128 limit = negative ? ((u128)0 - (u128)mn) : (u128)mx;
    if (mag > limit) return negative ? mn : mx;
    return negative ? (i128)((u128)0 - mag) : (i128)mag;
}

/*
 * Integer GEMM: C := encode(alpha * sum_p a_ip b_pj + beta * C).
 *   driver.rs:102-182 (traversal), alphabet.rs:559-637 (mac),
 *   epilogue.rs:51-94 (Linear; C is read only when beta != 0),
 *   epilogue.rs:280-329 (scaling), acc.rs:128-151 / 405-444 (encode).
 * i128 combine is a plain add; the reference's release profile builds with
 * overflow-checks = false (Cargo.toml:52-56), so it wraps.
 */
int uor_oracle_gemm_int(int ebits, int obits, size_t m, size_t k, size_t n, int64_t alpha,
                        const void *a, ptrdiff_t rsa, ptrdiff_t csa, const void *b, ptrdiff_t rsb,
                        ptrdiff_t csb, int64_t beta, void *c, ptrdiff_t rsc, ptrdiff_t csc, int mode,
                        int threads) {
    if (m == 0 || n == 0) return 0;
    set_threads(threads);
    long long mm = (long long)m;
#pragma omp parallel for schedule(dynamic, 1)
    for (long long ii = 0; ii < mm; ii++) {
        size_t i = (size_t)ii;
        for (size_t j = 0; j < n; j++) {
            ptrdiff_t co = (ptrdiff_t)i * rsc + (ptrdiff_t)j * csc;
            i128 outv;
            if (ebits == 64) {
                limbs3 acc = {{0, 0, 0}};
                for (size_t p = 0; p < k; p++) {
                    i128 x = load_int(a, 64, (ptrdiff_t)i * rsa + (ptrdiff_t)p * csa);
                    i128 y = load_int(b, 64, (ptrdiff_t)p * rsb + (ptrdiff_t)j * csb);
                    l3_add_i128(&acc, x * y);
                }
                limbs3 tot = l3_scale(acc, alpha);
                if (beta != 0) {
                    limbs3 pr = {{0, 0, 0}};
                    l3_add_i128(&pr, load_int(c, obits, co));
                    tot = l3_combine(tot, l3_scale(pr, beta));
                }
                outv = l3_encode(tot, obits, mode);
            } else {
                i128 acc = 0;
                if (ebits == 8) {
                    /* i8 products fit an int64 run for any k < 2^49. */
                    int64_t s = 0;
                    for (size_t p = 0; p < k; p++)
                        s += (int64_t)((const int8_t *)a)[(ptrdiff_t)i * rsa + (ptrdiff_t)p * csa] *
                             (int64_t)((const int8_t *)b)[(ptrdiff_t)p * rsb + (ptrdiff_t)j * csb];
                    acc = s;
                } else {
                    for (size_t p = 0; p < k; p++) {
                        i128 x = load_int(a, ebits, (ptrdiff_t)i * rsa + (ptrdiff_t)p * csa);
                        i128 y = load_int(b, ebits, (ptrdiff_t)p * rsb + (ptrdiff_t)j * csb);
                        acc += x * y;
                    }
                }
                i128 tot = sat_mul_i128(acc, alpha);
                if (beta != 0) {
                    i128 pr = load_int(c, obits, co);
                    tot = (i128)((u128)tot + (u128)sat_mul_i128(pr, beta));
                }
                outv = encode_i128_into(tot, out_min(obits), out_max(obits), mode);
            }
            store_int(c, obits, co, outv);
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------- */
/* Complex<i32 | i64> elements                                                */
/* ------------------------------------------------------------------------- */

/* Complex<T> is repr(C) {T re; T im} (alphabet.rs:656-663); strides count whole
 * complex elements, part h of element e sits at scalar offset 2e + h. The mac is the
 * scalar mac applied to (re, re), (im, -w.im), (re, w.im), (im, re) (alphabet.rs:
 * 712-717); -w.im is the release build's wrapping negation, so -MIN is MIN. Each part
 * has its own exact accumulator (ComplexAcc: i128 for i32, Limbs<3> for i64) and is
 * encoded on its own (EncodeFrom<ComplexAcc>, alphabet.rs:765-776). alpha and beta
 * apply to each part as Linear applies to a scalar accumulator (epilogue.rs:79-93);
 * alpha = 1, beta = 0 is the plain encode. */
static inline i128 wrapneg(i128 y, int ebits) {
    if (ebits == 64) return (i128)(int64_t)(0 - (uint64_t)(int64_t)y);
    return (i128)(int32_t)(0u - (uint32_t)(int32_t)y);
}

int uor_oracle_gemm_complex(int ebits, int obits, size_t m, size_t k, size_t n, int64_t alpha,
                            const void *a, ptrdiff_t rsa, ptrdiff_t csa, const void *b,
                            ptrdiff_t rsb, ptrdiff_t csb, int64_t beta, void *c, ptrdiff_t rsc,
                            ptrdiff_t csc, int mode, int threads) {
    if (m == 0 || n == 0) return 0;
    set_threads(threads);
    long long mm = (long long)m;
#pragma omp parallel for schedule(dynamic, 1)
    for (long long ii = 0; ii < mm; ii++) {
        size_t i = (size_t)ii;
        for (size_t j = 0; j < n; j++) {
            limbs3 acc3[2] = {{{0, 0, 0}}, {{0, 0, 0}}};
            i128 acc[2] = {0, 0};
            for (size_t p = 0; p < k; p++) {
                ptrdiff_t ao = 2 * ((ptrdiff_t)i * rsa + (ptrdiff_t)p * csa);
                ptrdiff_t bo = 2 * ((ptrdiff_t)p * rsb + (ptrdiff_t)j * csb);
                i128 are = load_int(a, ebits, ao), aim = load_int(a, ebits, ao + 1);
                i128 bre = load_int(b, ebits, bo), bim = load_int(b, ebits, bo + 1);
                i128 t[4] = {are * bre, aim * wrapneg(bim, ebits), are * bim, aim * bre};
                if (ebits == 64) {
                    for (int q = 0; q < 4; q++) l3_add_i128(&acc3[q >> 1], t[q]);
                } else {
                    acc[0] += t[0] + t[1];
                    acc[1] += t[2] + t[3];
                }
            }
            for (int h = 0; h < 2; h++) {
                ptrdiff_t co = 2 * ((ptrdiff_t)i * rsc + (ptrdiff_t)j * csc) + h;
                i128 outv;
                if (ebits == 64) {
                    limbs3 tot = l3_scale(acc3[h], alpha);
                    if (beta != 0) {
                        limbs3 pr = {{0, 0, 0}};
                        l3_add_i128(&pr, load_int(c, obits, co));
                        tot = l3_combine(tot, l3_scale(pr, beta));
                    }
                    outv = l3_encode(tot, obits, mode);
                } else {
                    i128 tot = sat_mul_i128(acc[h], alpha);
                    if (beta != 0)
                        tot = (i128)((u128)tot + (u128)sat_mul_i128(load_int(c, obits, co), beta));
                    outv = encode_i128_into(tot, out_min(obits), out_max(obits), mode);
                }
                store_int(c, obits, co, outv);
            }
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------- */
/* Codec tier: Packed<Grid<N>, P> over i8                                     */
/* ------------------------------------------------------------------------- */

/* Packed::decode_element (codecs.rs:181-195): low sub-code first; Grid's decode
 * is table[code % N] (codecs.rs:102-104). CodedMatrix::at (matrix.rs:202-207):
 * codes[r * (cols / P) + c / P], sub-code c % P. */
static inline int decode_packed(const uint8_t *codes, size_t row, size_t col, size_t cols, int P,
                                const int8_t *table, size_t N) {
    int bits = 8 / P;
    unsigned mask = bits >= 8 ? 0xFFu : ((1u << bits) - 1u);
    uint8_t code = codes[row * (cols / (size_t)P) + col / (size_t)P];
    unsigned sub = (code >> (bits * (int)(col % (size_t)P))) & mask;
    return table[sub % N];
}

/*
 * coded_gemm (coded.rs:98-142), orientation 0: B is k x n coded, C = A decode(B).
 * gemm_tabulated (tabulated.rs:600-660, 2555), orientation 1: W is n x k coded,
 * C = A W^T. Both are the Linear epilogue over the i128 accumulator.
 */
int uor_oracle_coded_gemm(int obits, size_t m, size_t k, size_t n, int64_t alpha, const int8_t *a,
                          ptrdiff_t rsa, ptrdiff_t csa, const uint8_t *codes, int P,
                          const int8_t *table, size_t N, int orientation, int64_t beta, void *c,
                          ptrdiff_t rsc, ptrdiff_t csc, int mode, int threads) {
    if (m == 0 || n == 0) return 0;
    set_threads(threads);
    long long mm = (long long)m;
#pragma omp parallel for schedule(dynamic, 1)
    for (long long ii = 0; ii < mm; ii++) {
        size_t i = (size_t)ii;
        for (size_t j = 0; j < n; j++) {
            int64_t s = 0;
            for (size_t p = 0; p < k; p++) {
                int w = orientation == 0 ? decode_packed(codes, p, j, n, P, table, N)
                                         : decode_packed(codes, j, p, k, P, table, N);
                s += (int64_t)a[(ptrdiff_t)i * rsa + (ptrdiff_t)p * csa] * w;
            }
            ptrdiff_t co = (ptrdiff_t)i * rsc + (ptrdiff_t)j * csc;
            i128 tot = sat_mul_i128((i128)s, alpha);
            if (beta != 0) tot = (i128)((u128)tot + (u128)sat_mul_i128(load_int(c, obits, co), beta));
            store_int(c, obits, co, encode_i128_into(tot, out_min(obits), out_max(obits), mode));
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------- */
/* Tropical (max, +)                                                         */
/* ------------------------------------------------------------------------- */

/* Trop<E> is repr(C) { E value; bool finite } (tropical.rs:61-70): the flag sits
 * right after the value, and the struct is padded to E's alignment. */
static inline size_t trop_size(int bits) { return bits == 8 ? 2 : bits == 16 ? 4 : bits == 32 ? 8 : 16; }

static inline int trop_load(const void *p, int bits, ptrdiff_t idx, i128 *v) {
    const uint8_t *e = (const uint8_t *)p + idx * (ptrdiff_t)trop_size(bits);
    int fin = e[bits / 8] != 0;
    int64_t x;
    switch (bits) {
    case 8: x = *(const int8_t *)e; break;
    case 16: { int16_t t; memcpy(&t, e, 2); x = t; } break;
    case 32: { int32_t t; memcpy(&t, e, 4); x = t; } break;
    default: memcpy(&x, e, 8); break;
    }
    *v = x;
    return fin;
}

static inline void trop_store(void *p, int bits, ptrdiff_t idx, int fin, i128 v) {
    uint8_t *e = (uint8_t *)p + idx * (ptrdiff_t)trop_size(bits);
    memset(e, 0, trop_size(bits));
    int64_t x = fin ? (int64_t)v : 0; /* NEG_INF stores E::ZERO, tropical.rs:74-77 */
    memcpy(e, &x, (size_t)bits / 8);
    e[bits / 8] = (uint8_t)(fin ? 1 : 0);
}

/*
 * driver::gemm over Trop<E> (driver.rs:102-182) with MaxPlus (epilogue.rs:137-186):
 *   mac: if both finite, acc := max(acc, a + b)       (tropical.rs:311-324)
 *   alpha, beta are Trop<i64>; -inf absorbs            (epilogue.rs:199-215)
 *   C is read only when beta is finite                 (epilogue.rs:166-170)
 *   encode: -inf -> -inf; finite -> [MIN+1, MAX-1]     (tropical.rs:336-351)
 */
int uor_oracle_gemm_trop(int ebits, int obits, size_t m, size_t k, size_t n, int64_t alpha_v,
                         int alpha_finite, const void *a, ptrdiff_t rsa, ptrdiff_t csa,
                         const void *b, ptrdiff_t rsb, ptrdiff_t csb, int64_t beta_v,
                         int beta_finite, void *c, ptrdiff_t rsc, ptrdiff_t csc, int mode,
                         int threads) {
    if (m == 0 || n == 0) return 0;
    set_threads(threads);
    long long mm = (long long)m;
#pragma omp parallel for schedule(dynamic, 1)
    for (long long ii = 0; ii < mm; ii++) {
        size_t i = (size_t)ii;
        for (size_t j = 0; j < n; j++) {
            int have = 0;
            i128 best = 0;
            for (size_t p = 0; p < k; p++) {
                i128 x, y;
                int fx = trop_load(a, ebits, (ptrdiff_t)i * rsa + (ptrdiff_t)p * csa, &x);
                int fy = trop_load(b, ebits, (ptrdiff_t)p * rsb + (ptrdiff_t)j * csb, &y);
                if (fx && fy) {
                    i128 s = x + y;
                    if (!have || s > best) { best = s; have = 1; }
                }
            }
            /* shift_exact(alpha) */
            int fin = have && alpha_finite;
            i128 tot = fin ? best + (i128)alpha_v : 0;
            ptrdiff_t co = (ptrdiff_t)i * rsc + (ptrdiff_t)j * csc;
            if (beta_finite) {
                i128 pv;
                int pf = trop_load(c, obits, co, &pv);
                if (pf) {
                    i128 sh = pv + (i128)beta_v;
                    if (!fin || sh > tot) { tot = sh; fin = 1; }
                }
            }
            if (fin) tot = encode_i128_into(tot, out_min(obits) + 1, out_max(obits) - 1, mode);
            trop_store(c, obits, co, fin, tot);
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------- */
/* Float family: exact sum, flags, one encode                                 */
/* ------------------------------------------------------------------------- */

/*
 * The complete accumulator (acc.rs:469-1244) is a fixed-point register whose
 * bit 0 weighs 2^MIN_EXP (f32: -298, f64: -2148, generated.rs:116-126), plus the
 * non-finite flags {nan, +inf, -inf}. This restatement keeps the same value in a
 * wider two's complement limb array (CL limbs), which is exact for every input
 * the reference's own register holds.
 */
#define CL_MAX 72

typedef struct {
    int nl;       /* limbs in use */
    int min_exp;  /* exponent of bit 0 */
    uint64_t w[CL_MAX];
    int nan, pinf, ninf;
} cacc;

/* The register is L low limbs plus one signed extension word (acc.rs:469-476;
 * L = 10 for f32, 67 for f64, generated.rs:116-126), held here as L + 1 limbs of
 * one two's complement integer. */
static void cacc_init(cacc *x, int is64) {
    memset(x, 0, sizeof(*x));
    x->nl = is64 ? 68 : 11;
    x->min_exp = is64 ? -2148 : -298;
}

/* Add (or subtract) mag * 2^exp, exactly: Complete::add_scaled, acc.rs:939-998. */
static void cacc_add_scaled(cacc *x, u128 mag, int exp, int negative) {
    if (mag == 0) return;
    long shift = (long)exp - x->min_exp;
    if (shift < 0) return;
    int at = (int)(shift / 64), bit = (int)(shift % 64);
    /* A coordinate past the last low limb names no stored bit: dropped whole
     * (acc.rs:977-982). Parts reaching the extension word land there; parts past
     * it are dropped (add_at, acc.rs:157-187). */
    if (at >= x->nl - 1) return;
    /* mag * 2^bit spread over three words (radix_spread_u128, acc.rs:528-547) */
    uint64_t parts[3];
    if (bit == 0) {
        parts[0] = (uint64_t)mag;
        parts[1] = (uint64_t)(mag >> 64);
        parts[2] = 0;
    } else {
        parts[0] = (uint64_t)(mag << bit);
        parts[1] = (uint64_t)(mag >> (64 - bit));
        parts[2] = (uint64_t)(mag >> (128 - bit));
    }
    if (!negative) {
        unsigned carry = 0;
        for (int i = at, q = 0; i < x->nl && (q < 3 || carry); i++, q++) {
            u128 s = (u128)x->w[i] + (q < 3 ? parts[q] : 0) + carry;
            x->w[i] = (uint64_t)s;
            carry = (unsigned)(s >> 64);
        }
    } else {
        unsigned borrow = 0;
        for (int i = at, q = 0; i < x->nl && (q < 3 || borrow); i++, q++) {
            uint64_t p = q < 3 ? parts[q] : 0;
            u128 d = (u128)x->w[i] - p - borrow;
            x->w[i] = (uint64_t)d;
            borrow = (unsigned)((d >> 64) & 1);
        }
    }
}

static int cacc_is_neg(const cacc *x) { return (int)(x->w[x->nl - 1] >> 63); }

static void cacc_negate(cacc *x) {
    unsigned carry = 1;
    for (int i = 0; i < x->nl; i++) {
        u128 s = (u128)(~x->w[i]) + carry;
        x->w[i] = (uint64_t)s;
        carry = (unsigned)(s >> 64);
    }
}

static void cacc_add(cacc *x, const cacc *y) {
    unsigned carry = 0;
    for (int i = 0; i < x->nl; i++) {
        u128 s = (u128)x->w[i] + y->w[i] + carry;
        x->w[i] = (uint64_t)s;
        carry = (unsigned)(s >> 64);
    }
}

/* Multiply the finite value by an exact integer (two's complement, exact). */
static void cacc_mul_i64(cacc *x, int64_t f) {
    int neg = cacc_is_neg(x);
    if (neg) cacc_negate(x);
    uint64_t uf = f < 0 ? (uint64_t)0 - (uint64_t)f : (uint64_t)f;
    uint64_t carry = 0;
    for (int i = 0; i < x->nl; i++) {
        u128 p = (u128)x->w[i] * uf + carry;
        x->w[i] = (uint64_t)p;
        carry = (uint64_t)(p >> 64);
    }
    if (neg != (f < 0)) cacc_negate(x);
}

static int cacc_is_nan(const cacc *x) { return x->nan || (x->pinf && x->ninf); }
static int cacc_finite(const cacc *x) { return !x->nan && !x->pinf && !x->ninf; }

/* Complete::scale (acc.rs:1028-1069) as observed through the encode. */
static void cacc_scale(cacc *x, int64_t f) {
    if (cacc_is_nan(x)) return;
    if (f == 1) return;
    if (f == 0) {
        int inf = x->pinf || x->ninf;
        memset(x->w, 0, sizeof(x->w));
        if (inf) { x->nan = 1; x->pinf = x->ninf = 0; }
        return;
    }
    if (!cacc_finite(x)) {
        if (f < 0) { int t = x->pinf; x->pinf = x->ninf; x->ninf = t; }
        return;
    }
    cacc_mul_i64(x, f);
}

/* FloatElement::decode, alphabet.rs:905-946. kind: 0 finite, 1 inf, 2 nan. */
typedef struct { int kind, sign; uint64_t mant; int exp; } decoded;

static decoded decode_f32(uint32_t bits) {
    decoded d;
    uint32_t frac = bits & 0x7FFFFFu, biased = (bits >> 23) & 0xFFu;
    d.sign = (int)(bits >> 31);
    if (biased == 0xFF) { d.kind = frac ? 2 : 1; d.mant = 0; d.exp = 0; return d; }
    d.kind = 0;
    if (biased == 0) { d.mant = frac; d.exp = 1 - 127 - 23; }
    else { d.mant = frac | 0x800000u; d.exp = (int)biased - 127 - 23; }
    return d;
}

static decoded decode_f64(uint64_t bits) {
    decoded d;
    uint64_t frac = bits & 0xFFFFFFFFFFFFFull, biased = (bits >> 52) & 0x7FFu;
    d.sign = (int)(bits >> 63);
    if (biased == 0x7FF) { d.kind = frac ? 2 : 1; d.mant = 0; d.exp = 0; return d; }
    d.kind = 0;
    if (biased == 0) { d.mant = frac; d.exp = 1 - 1023 - 52; }
    else { d.mant = frac | 0x10000000000000ull; d.exp = (int)biased - 1023 - 52; }
    return d;
}

static inline decoded load_float(const void *p, int is64, ptrdiff_t off) {
    if (is64) { uint64_t u; memcpy(&u, (const double *)p + off, 8); return decode_f64(u); }
    uint32_t u; memcpy(&u, (const float *)p + off, 4); return decode_f32(u);
}

/* Element::mac for a float pair (alphabet.rs:856-886). */
static void cacc_mac(cacc *x, decoded a, decoded b) {
    if (a.kind == 2 || b.kind == 2) { x->nan = 1; return; }
    if (a.kind == 1 || b.kind == 1) {
        decoded inf = a.kind == 1 ? a : b, other = a.kind == 1 ? b : a;
        if (other.kind == 0 && other.mant == 0) { x->nan = 1; return; }
        if (inf.sign != other.sign) x->ninf = 1; else x->pinf = 1;
        return;
    }
    u128 p = (u128)a.mant * b.mant;
    cacc_add_scaled(x, p, a.exp + b.exp, a.sign != b.sign);
}

/* Complete::of (acc.rs:1007-1020): the exact value a float in C names. */
static void cacc_of(cacc *x, decoded d) {
    if (d.kind == 2) { x->nan = 1; return; }
    if (d.kind == 1) { if (d.sign) x->ninf = 1; else x->pinf = 1; return; }
    cacc_add_scaled(x, d.mant, d.exp, d.sign);
}

/* bit i of the magnitude */
static inline int mag_bit(const cacc *m, long i) {
    if (i < 0 || i >= 64L * m->nl) return 0;
    return (int)((m->w[i / 64] >> (i % 64)) & 1);
}

static inline int mag_any_below(const cacc *m, long i) {
    if (i <= 0) return 0;
    long full = i / 64;
    for (long j = 0; j < full && j < m->nl; j++) if (m->w[j]) return 1;
    if (full < m->nl) {
        int rem = (int)(i % 64);
        if (rem && (m->w[full] & ((1ull << rem) - 1))) return 1;
    }
    return 0;
}

static inline uint64_t mag_window(const cacc *m, long at, int n) {
    uint64_t out = 0;
    for (int q = 0; q < n; q++) out |= (uint64_t)mag_bit(m, at + q) << q;
    return out;
}

/* The correctly-rounded encode, acc.rs:1734-1868. Returns the raw bits. */
static uint64_t cacc_encode(const cacc *acc, int out64, int mode) {
    const int MANT = out64 ? 52 : 23, EXPO = out64 ? 11 : 8;
    const int P = MANT + 1;
    const int BIAS = (1 << (EXPO - 1)) - 1;
    const int SUB_LSB_EXP = 1 - BIAS - MANT;
    const uint64_t sign_bit = out64 ? (1ull << 63) : (1ull << 31);
    const uint64_t exp_all = (uint64_t)((1u << EXPO) - 1);
    if (cacc_is_nan(acc)) return out64 ? 0x7FF8000000000000ull : 0x7FC00000ull;
    if (acc->pinf || acc->ninf) return (acc->ninf ? sign_bit : 0) | (exp_all << MANT);
    cacc m = *acc;
    int negative = cacc_is_neg(&m);
    if (negative) cacc_negate(&m);
    long high = -1;
    for (int i = m.nl - 1; i >= 0; i--)
        if (m.w[i]) { high = 64L * i + (63 - __builtin_clzll(m.w[i])); break; }
    if (high < 0) return 0; /* exact zero encodes +0 */
    long exp = (long)m.min_exp + high;
    long lsb_exp = exp - (P - 1) < SUB_LSB_EXP ? SUB_LSB_EXP : exp - (P - 1);
    long lsb = lsb_exp - m.min_exp;
    if (lsb < 0) return 0; /* acc.rs: an undersized register encodes +0 */
    uint64_t sig = mag_window(&m, lsb, P);
    int round_bit = 0, sticky = 0;
    if (lsb > 0) { round_bit = mag_bit(&m, lsb - 1); sticky = mag_any_below(&m, lsb - 1); }
    int inc = mode == MODE_NEAREST ? (round_bit && (sticky || (sig & 1))) : 0;
    sig += (uint64_t)inc;
    if (sig >> P) { sig >>= 1; lsb_exp += 1; }
    if (sig == 0) return negative ? sign_bit : 0;
    int top = 63 - __builtin_clzll(sig);
    long value_exp = lsb_exp + top;
    if ((sig >> (P - 1)) == 1) {
        long biased = value_exp + BIAS;
        if (biased >= (long)exp_all) {
            if (mode == MODE_NEAREST) return (negative ? sign_bit : 0) | (exp_all << MANT);
            /* MAX finite */
            return (negative ? sign_bit : 0) | ((exp_all - 1) << MANT) | ((1ull << MANT) - 1);
        }
        return (negative ? sign_bit : 0) | ((uint64_t)biased << MANT) | (sig & ((1ull << MANT) - 1));
    }
    return (negative ? sign_bit : 0) | sig;
}

/*
 * gemm_float / gemm_float_ex / raw::sgemm / raw::dgemm (slice.rs:304-465,
 * raw.rs:45-160, float.rs:1761-1917): C := encode(alpha * exact(A B) + beta * C).
 * The Linear epilogue over Complete (epilogue.rs:79-93): scale(alpha), and if
 * beta != 0, combine with Complete::of(C).scale(beta); flags union on combine.
 */
int uor_oracle_gemm_float(int e64, int o64, size_t m, size_t k, size_t n, int64_t alpha,
                          const void *a, ptrdiff_t rsa, ptrdiff_t csa, const void *b, ptrdiff_t rsb,
                          ptrdiff_t csb, int64_t beta, void *c, ptrdiff_t rsc, ptrdiff_t csc,
                          int mode, int threads) {
    if (m == 0 || n == 0) return 0;
    set_threads(threads);
    long long mm = (long long)m;
#pragma omp parallel for schedule(dynamic, 1)
    for (long long ii = 0; ii < mm; ii++) {
        size_t i = (size_t)ii;
        cacc acc, pr;
        for (size_t j = 0; j < n; j++) {
            cacc_init(&acc, e64);
            for (size_t p = 0; p < k; p++) {
                decoded x = load_float(a, e64, (ptrdiff_t)i * rsa + (ptrdiff_t)p * csa);
                decoded y = load_float(b, e64, (ptrdiff_t)p * rsb + (ptrdiff_t)j * csb);
                cacc_mac(&acc, x, y);
            }
            cacc_scale(&acc, alpha);
            ptrdiff_t co = (ptrdiff_t)i * rsc + (ptrdiff_t)j * csc;
            if (beta != 0) {
                cacc_init(&pr, e64);
                cacc_of(&pr, load_float(c, o64, co));
                cacc_scale(&pr, beta);
                if (cacc_finite(&acc) && cacc_finite(&pr)) cacc_add(&acc, &pr);
                else {
                    acc.nan |= pr.nan; acc.pinf |= pr.pinf; acc.ninf |= pr.ninf;
                }
            }
            uint64_t bits = cacc_encode(&acc, o64, mode);
            if (o64) memcpy((double *)c + co, &bits, 8);
            else { uint32_t u = (uint32_t)bits; memcpy((float *)c + co, &u, 4); }
        }
    }
    return 0;
}

/*
 * A blocked restatement of the reference's kernel traversal for s8 x s8
 * (kernel.rs:1016-1377 with the I8_I32 tile family): B is packed K-major once
 * (pack_columns, kernel.rs:1703), each dot product runs in s32 lanes over chunks
 * of at most lane_depth = 131071 products (spec.rs:232-243) and folds into an
 * int64, then the Linear epilogue and encode run once per cell. Same bytes as
 * uor_oracle_gemm_int; it exists to time the CPU baseline fairly.
 * Row-major contiguous A (m x k) and B (k x n); C row-major with ldc.
 */
__attribute__((target("avx2"))) static int64_t dot_i8_avx2(const int8_t *x, const int8_t *y,
                                                           size_t k) {
    int64_t total = 0;
    for (size_t p0 = 0; p0 < k; p0 += 131071) {
        size_t end = p0 + 131071 < k ? p0 + 131071 : k;
        int32_t s = 0;
        for (size_t p = p0; p < end; p++) s += (int32_t)x[p] * (int32_t)y[p];
        total += s;
    }
    return total;
}

static int64_t dot_i8_generic(const int8_t *x, const int8_t *y, size_t k) {
    int64_t total = 0;
    for (size_t p0 = 0; p0 < k; p0 += 131071) {
        size_t end = p0 + 131071 < k ? p0 + 131071 : k;
        int32_t s = 0;
        for (size_t p = p0; p < end; p++) s += (int32_t)x[p] * (int32_t)y[p];
        total += s;
    }
    return total;
}

int uor_oracle_gemm_i8_blocked(size_t m, size_t k, size_t n, int64_t alpha, const int8_t *a,
                               const int8_t *b, int64_t beta, int32_t *c, size_t ldc, int mode,
                               int threads) {
    if (m == 0 || n == 0) return 0;
    set_threads(threads);
    int8_t *bt = (int8_t *)malloc(n * k + 64);
    if (!bt) return -1;
    long long nn = (long long)n;
#pragma omp parallel for schedule(static)
    for (long long jj = 0; jj < nn; jj++)
        for (size_t p = 0; p < k; p++) bt[(size_t)jj * k + p] = b[p * n + (size_t)jj];
    int avx2 = __builtin_cpu_supports("avx2");
    long long mm = (long long)m;
    const size_t JB = 64;
#pragma omp parallel for schedule(dynamic, 1)
    for (long long ii = 0; ii < mm; ii++) {
        size_t i = (size_t)ii;
        for (size_t j0 = 0; j0 < n; j0 += JB) {
            size_t j1 = j0 + JB < n ? j0 + JB : n;
            for (size_t j = j0; j < j1; j++) {
                int64_t acc = avx2 ? dot_i8_avx2(a + i * k, bt + j * k, k)
                                   : dot_i8_generic(a + i * k, bt + j * k, k);
                i128 tot = sat_mul_i128((i128)acc, alpha);
                if (beta != 0)
                    tot = (i128)((u128)tot + (u128)sat_mul_i128((i128)c[i * ldc + j], beta));
                c[i * ldc + j] = (int32_t)encode_i128_into(tot, out_min(32), out_max(32), mode);
            }
        }
    }
    free(bt);
    return 0;
}

/* The number of OpenMP threads a parallel region gets, for the baseline record. */
int uor_oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* The validate harness fill (validate/tests/common/mod.rs:9-19): xorshift64 from
 * 0x243F6A8885A308D3 ^ salt, each value `s >> 33` cast to i8 (massive.rs:130). Lets the
 * CPU baseline draw the benchmark's operands without the product library. */
int uor_oracle_corpus_i8(uint64_t salt, size_t count, int8_t *out) {
    uint64_t s = 0x243F6A8885A308D3ull ^ salt;
    for (size_t i = 0; i < count; i++) {
        s ^= s << 13;
        s ^= s >> 7;
        s ^= s << 17;
        out[i] = (int8_t)(s >> 33);
    }
    return 0;
}
