// float_exact.cu -- K6 + K7: exact float GEMM, rounded once.
//
// Replaces gemm_float / gemm_float_packed / raw::sgemm / raw::dgemm
// (crates/uor-matmul/src/slice.rs:304-465, raw.rs:45-160, crates/uor-matmul-gemm/src/
// float.rs:1761-1917): C := encode(alpha * exact(A B) + beta * C), with the product
// semantics of Element::mac for floats (alphabet.rs:856-886: NaN absorbs, inf * 0 is
// NaN, +inf and -inf make NaN), the Linear epilogue over the complete accumulator
// (Complete::scale / combine, acc.rs:1028-1244) and the one correctly rounded encode
// (acc.rs:1734-1868).
//
// Tensor-core route (K6): every row i of A and column j of B is scaled to an exact
// integer, x = +-mant * 2^(exp - lo), with lo the lowest set-bit exponent of that
// row (column); the integers are cut into L signed base-256 digits in [-128, 127],
// so A B = sum_{s,t} 2^(8 (s+t)) A_s B_t * 2^(lo_i + lo_j). The digit-pair products
// run on the slice-pair kernel (gemm_slices.cu), one s32 accumulator per diagonal
// s + t and reduction chunk, exactly. K7 (`fx_reduce_kernel`) rebuilds each cell's
// exact integer in 768-bit two's complement, applies alpha, adds beta * C exactly
// (out-of-window bits of the smaller term are jammed into a sticky bit, which cannot
// change the rounding because that term is then far below the result's last bit),
// and encodes once. Non-finite inputs are resolved by a separate flags kernel that
// visits only rows and columns holding them.
//
// Direct route: when a row or column spans more than 16 digits, each cell is
// accumulated in the reference's own fixed-point register (L low limbs plus an
// extension word) on CUDA cores. Exact, and slow; it exists so that no input has
// to be refused.
#include <climits>
#include <type_traits>
#include <vector>
#include "aux.cuh"
#include "float_exact.h"
#include "gemm_slices.cuh"
#include "modular.cuh"
#include "ptx.cuh"
#include "walk.cuh"

namespace uor {

// ------------------------------------------------------------ decoding

struct FDec {
    int kind;  // 0 finite, 1 infinite, 2 NaN
    int sign;
    uint64_t mant;
    int exp;
};

// FloatElement::decode (alphabet.rs:905-946) of a bit pattern (f32 in the low 32 bits).
__device__ __forceinline__ FDec fdecode_bits(uint64_t raw, bool f64) {
    FDec d;
    if (f64) {
        const uint64_t bits = raw;
        const uint64_t frac = bits & 0xFFFFFFFFFFFFFull, biased = (bits >> 52) & 0x7FF;
        d.sign = static_cast<int>(bits >> 63);
        if (biased == 0x7FF) {
            d.kind = frac ? 2 : 1, d.mant = 0, d.exp = 0;
            return d;
        }
        d.kind = 0;
        if (biased == 0) d.mant = frac, d.exp = 1 - 1023 - 52;
        else d.mant = frac | (1ull << 52), d.exp = static_cast<int>(biased) - 1023 - 52;
    } else {
        const uint32_t bits = static_cast<uint32_t>(raw);
        const uint32_t frac = bits & 0x7FFFFF, biased = (bits >> 23) & 0xFF;
        d.sign = static_cast<int>(bits >> 31);
        if (biased == 0xFF) {
            d.kind = frac ? 2 : 1, d.mant = 0, d.exp = 0;
            return d;
        }
        d.kind = 0;
        if (biased == 0) d.mant = frac, d.exp = 1 - 127 - 23;
        else d.mant = frac | 0x800000u, d.exp = static_cast<int>(biased) - 127 - 23;
    }
    return d;
}

// FloatElement::decode of element idx of an f32 / f64 array.
__device__ __forceinline__ FDec fdecode(const uint8_t* base, int64_t idx, bool f64) {
    return fdecode_bits(f64 ? reinterpret_cast<const uint64_t*>(base)[idx]
                            : reinterpret_cast<const uint32_t*>(base)[idx],
                        f64);
}

// Product flags of one term (alphabet.rs:862-873): bit 0 NaN, bit 1 +inf, bit 2 -inf.
__device__ __forceinline__ int term_flags(const FDec& a, const FDec& b) {
    if (a.kind == 2 || b.kind == 2) return 1;
    if (a.kind == 1 || b.kind == 1) {
        const FDec& inf = a.kind == 1 ? a : b;
        const FDec& other = a.kind == 1 ? b : a;
        if (other.kind == 0 && other.mant == 0) return 1;
        return (inf.sign != other.sign) ? 4 : 2;
    }
    return 0;
}

// ------------------------------------------------------------ big integers

constexpr int BW = 12;  // 768-bit two's complement window
struct Big {
    uint64_t w[BW];
};

__device__ __forceinline__ void big_zero(Big& x) {
#pragma unroll
    for (int i = 0; i < BW; ++i) x.w[i] = 0;
}
__device__ __forceinline__ bool big_neg(const Big& x) { return (x.w[BW - 1] >> 63) != 0; }
__device__ __forceinline__ bool big_is_zero(const Big& x) {
    uint64_t o = 0;
#pragma unroll
    for (int i = 0; i < BW; ++i) o |= x.w[i];
    return o == 0;
}
__device__ __forceinline__ void big_negate(Big& x) {
    uint64_t c = 1;
#pragma unroll
    for (int i = 0; i < BW; ++i) {
        const uint64_t s = ~x.w[i] + c;
        c = (c && s == 0) ? 1 : 0;
        x.w[i] = s;
    }
}
__device__ __forceinline__ void big_add(Big& x, const Big& y) {
    uint64_t c = 0;
#pragma unroll
    for (int i = 0; i < BW; ++i) {
        const uint64_t s = x.w[i] + y.w[i];
        const uint64_t c1 = s < x.w[i];
        const uint64_t s2 = s + c;
        const uint64_t c2 = s2 < s;
        x.w[i] = s2;
        c = c1 | c2;
    }
}
// x += v * 2^sh (v signed 64-bit, 0 <= sh < 64 * (BW - 2)).
__device__ __forceinline__ void big_add_i64_shl(Big& x, int64_t v, int sh) {
    const int wi = sh >> 6, b = sh & 63;
    const uint64_t ext = v < 0 ? ~0ull : 0ull;
    const uint64_t lo = static_cast<uint64_t>(v) << b;
    const uint64_t hi = b ? (static_cast<uint64_t>(v) >> (64 - b)) | (ext << b) : ext;
    uint64_t c = 0;
    for (int i = wi; i < BW; ++i) {
        const uint64_t add = i == wi ? lo : (i == wi + 1 ? hi : ext);
        const uint64_t s = x.w[i] + add;
        const uint64_t c1 = s < x.w[i];
        const uint64_t s2 = s + c;
        const uint64_t c2 = s2 < s;
        x.w[i] = s2;
        c = c1 | c2;
    }
}
// x := x * f, exact while the product fits the window (it always does here).
__device__ __forceinline__ void big_mul_i64(Big& x, int64_t f) {
    const bool nx = big_neg(x);
    if (nx) big_negate(x);
    const uint64_t uf = f < 0 ? 0ull - static_cast<uint64_t>(f) : static_cast<uint64_t>(f);
    uint64_t carry = 0;
#pragma unroll
    for (int i = 0; i < BW; ++i) {
        const u128 p = static_cast<u128>(x.w[i]) * uf + carry;
        x.w[i] = static_cast<uint64_t>(p);
        carry = static_cast<uint64_t>(p >> 64);
    }
    if (nx != (f < 0)) big_negate(x);
}
__device__ __forceinline__ int big_bitlen(const Big& mag) {
    for (int i = BW - 1; i >= 0; --i)
        if (mag.w[i]) return 64 * i + 64 - __clzll(static_cast<long long>(mag.w[i]));
    return 0;
}
// any bit at positions [0, pos)
__device__ __forceinline__ bool big_any_below(const Big& mag, int pos) {
    if (pos <= 0) return false;
    const int full = pos >> 6;
    for (int i = 0; i < full && i < BW; ++i)
        if (mag.w[i]) return true;
    if (full < BW && (pos & 63)) return (mag.w[full] & ((1ull << (pos & 63)) - 1)) != 0;
    return false;
}
// Magnitude shifted: mag * 2^sh for sh >= 0 (into the window), truncation with a
// sticky flag for sh < 0.
__device__ __forceinline__ void big_shift_mag(Big& m, int sh, bool* sticky) {
    *sticky = false;
    if (sh == 0) return;
    Big r;
    big_zero(r);
    if (sh > 0) {
        const int ws = sh >> 6, bs = sh & 63;
        for (int i = BW - 1; i >= ws; --i) {
            const uint64_t lo = m.w[i - ws] << bs;
            const uint64_t carry = (bs && i - ws - 1 >= 0) ? (m.w[i - ws - 1] >> (64 - bs)) : 0;
            r.w[i] = lo | carry;
        }
    } else {
        const int d = -sh;
        *sticky = big_any_below(m, d);
        const int ws = d >> 6, bs = d & 63;
        for (int i = 0; i + ws < BW; ++i) {
            const uint64_t lo = m.w[i + ws] >> bs;
            const uint64_t hi = (bs && i + ws + 1 < BW) ? (m.w[i + ws + 1] << (64 - bs)) : 0;
            r.w[i] = lo | hi;
        }
    }
    m = r;
}

// Word-array helpers for the encode (magnitudes, little-endian words).
template <int NW>
__device__ __forceinline__ int words_bitlen(const uint64_t (&m)[NW]) {
    for (int i = NW - 1; i >= 0; --i)
        if (m[i]) return 64 * i + 64 - __clzll(static_cast<long long>(m[i]));
    return 0;
}
template <int NW>
__device__ __forceinline__ int words_bit(const uint64_t (&m)[NW], int pos) {
    if (pos < 0 || pos >= 64 * NW) return 0;
    return static_cast<int>((m[pos >> 6] >> (pos & 63)) & 1);
}
template <int NW>
__device__ __forceinline__ bool words_any_below(const uint64_t (&m)[NW], int pos) {
    if (pos <= 0) return false;
    const int full = pos >> 6;
    for (int i = 0; i < full && i < NW; ++i)
        if (m[i]) return true;
    if (full < NW && (pos & 63)) return (m[full] & ((1ull << (pos & 63)) - 1)) != 0;
    return false;
}
template <int NW>
__device__ __forceinline__ void words_negate(uint64_t (&x)[NW]) {
    uint64_t c = 1;
    for (int i = 0; i < NW; ++i) {
        const uint64_t s = ~x[i] + c;
        c = (c && s == 0) ? 1 : 0;
        x[i] = s;
    }
}

// The correctly rounded encode (acc.rs:1734-1868) of the exact value W * 2^unit_exp
// (W two's complement over NW words). min_exp_e is the element register's bit-0
// exponent: a result whose last bit would fall below it encodes +0, as the
// reference's register index does.
template <int NW>
__device__ uint64_t encode_words(const uint64_t (&Win)[NW], int unit_exp, bool out64, int mode,
                                 int min_exp_e) {
    const int MANT = out64 ? 52 : 23, EXPO = out64 ? 11 : 8;
    const int P = MANT + 1;
    const int BIAS = (1 << (EXPO - 1)) - 1;
    const int SUB = 1 - BIAS - MANT;
    const uint64_t sign_bit = out64 ? (1ull << 63) : (1ull << 31);
    const uint64_t exp_all = (1ull << EXPO) - 1;
    uint64_t mag[NW];
    for (int i = 0; i < NW; ++i) mag[i] = Win[i];
    const bool neg = (mag[NW - 1] >> 63) != 0;
    if (neg) words_negate(mag);
    const int bl = words_bitlen(mag);
    if (bl == 0) return 0;  // exact zero encodes +0
    const int exp = unit_exp + bl - 1;
    int lsb_exp = exp - (P - 1) < SUB ? SUB : exp - (P - 1);
    if (lsb_exp - min_exp_e < 0) return 0;
    const int lsb = lsb_exp - unit_exp;
    uint64_t sig = 0;
    for (int q = 0; q < P; ++q) sig |= static_cast<uint64_t>(words_bit(mag, lsb + q)) << q;
    bool round_bit = false, sticky = false;
    if (lsb_exp - min_exp_e != 0) {
        round_bit = words_bit(mag, lsb - 1) != 0;
        sticky = words_any_below(mag, lsb - 1);
    }
    const bool inc = mode == MODE_NEAREST && round_bit && (sticky || (sig & 1));
    sig += inc ? 1 : 0;
    if (sig >> P) {
        sig >>= 1;
        lsb_exp += 1;
    }
    const uint64_t s = neg ? sign_bit : 0;
    if (sig == 0) return s;
    const int top = 63 - __clzll(static_cast<long long>(sig));
    const int value_exp = lsb_exp + top;
    if ((sig >> (P - 1)) == 1) {
        const int biased = value_exp + BIAS;
        if (biased >= static_cast<int>(exp_all)) {
            if (mode == MODE_NEAREST) return s | (exp_all << MANT);
            return s | ((exp_all - 1) << MANT) | ((1ull << MANT) - 1);
        }
        return s | (static_cast<uint64_t>(biased) << MANT) | (sig & ((1ull << MANT) - 1));
    }
    return s | sig;
}

// Register-resident helpers for a short magnitude (NW words, every index resolved by
// unrolled selects, so nothing spills to local memory).
template <int NW>
__device__ __forceinline__ uint64_t reg_word(const uint64_t (&m)[NW], int i) {
    uint64_t r = 0;
#pragma unroll
    for (int q = 0; q < NW; ++q) r = q == i ? m[q] : r;
    return r;
}
template <int NW>
__device__ __forceinline__ int reg_bitlen(const uint64_t (&m)[NW]) {
    int bl = 0;
#pragma unroll
    for (int q = 0; q < NW; ++q)
        if (m[q]) bl = 64 * q + 64 - __clzll(static_cast<long long>(m[q]));
    return bl;
}
// bits [pos, pos + 64) of the magnitude; positions below 0 read as zero (pos > -64).
template <int NW>
__device__ __forceinline__ uint64_t reg_window(const uint64_t (&m)[NW], int pos) {
    if (pos < 0) return m[0] << (-pos);
    const int wi = pos >> 6, b = pos & 63;
    const uint64_t lo = reg_word(m, wi);
    return b ? (lo >> b) | (reg_word(m, wi + 1) << (64 - b)) : lo;
}
template <int NW>
__device__ __forceinline__ bool reg_any_below(const uint64_t (&m)[NW], int pos) {
    uint64_t acc = 0;
#pragma unroll
    for (int q = 0; q < NW; ++q) {
        if (64 * q + 64 <= pos) acc |= m[q];
        else if (64 * q < pos) acc |= m[q] & ((1ull << (pos - 64 * q)) - 1);
    }
    return acc != 0;
}

// encode_words for a magnitude held in registers with its sign: the same rounding
// steps (acc.rs:1734-1868), the significand and round bit read as one 64-bit window.
template <int NW>
__device__ __forceinline__ uint64_t encode_mag_fast(const uint64_t (&mag)[NW], bool neg, int unit_exp, bool out64,
                                    int mode, int min_exp_e) {
    const int MANT = out64 ? 52 : 23, EXPO = out64 ? 11 : 8;
    const int P = MANT + 1;
    const int BIAS = (1 << (EXPO - 1)) - 1;
    const int SUB = 1 - BIAS - MANT;
    const uint64_t sign_bit = out64 ? (1ull << 63) : (1ull << 31);
    const uint64_t exp_all = (1ull << EXPO) - 1;
    const int bl = reg_bitlen(mag);
    if (bl == 0) return 0;  // exact zero encodes +0
    const int exp = unit_exp + bl - 1;
    int lsb_exp = exp - (P - 1) < SUB ? SUB : exp - (P - 1);
    if (lsb_exp - min_exp_e < 0) return 0;
    const int lsb = lsb_exp - unit_exp;  // >= bl - P > -64
    const uint64_t win = reg_window(mag, lsb - 1);
    uint64_t sig = (win >> 1) & ((1ull << P) - 1);
    bool round_bit = false, sticky = false;
    if (lsb_exp - min_exp_e != 0) {
        round_bit = (win & 1) != 0;
        sticky = reg_any_below(mag, lsb - 1);
    }
    const bool inc = mode == MODE_NEAREST && round_bit && (sticky || (sig & 1));
    sig += inc ? 1 : 0;
    if (sig >> P) {
        sig >>= 1;
        lsb_exp += 1;
    }
    const uint64_t s = neg ? sign_bit : 0;
    if (sig == 0) return s;
    const int top = 63 - __clzll(static_cast<long long>(sig));
    const int value_exp = lsb_exp + top;
    if ((sig >> (P - 1)) == 1) {
        const int biased = value_exp + BIAS;
        if (biased >= static_cast<int>(exp_all)) {
            if (mode == MODE_NEAREST) return s | (exp_all << MANT);
            return s | ((exp_all - 1) << MANT) | ((1ull << MANT) - 1);
        }
        return s | (static_cast<uint64_t>(biased) << MANT) | (sig & ((1ull << MANT) - 1));
    }
    return s | sig;
}

__device__ __forceinline__ uint64_t nan_bits(bool out64) {
    return out64 ? 0x7FF8000000000000ull : 0x7FC00000ull;
}
__device__ __forceinline__ uint64_t inf_bits(bool out64, bool neg) {
    return out64 ? ((neg ? 1ull << 63 : 0) | 0x7FF0000000000000ull)
                 : ((neg ? 1ull << 31 : 0) | 0x7F800000ull);
}

// Complete::scale's flag rules (acc.rs:1028-1069) on (flags, finite part).
// Returns true when the finite part must be multiplied by f.
__device__ __forceinline__ bool scale_flags(int& fl, bool& zero_out, int64_t f) {
    const bool nan = (fl & 1) || ((fl & 6) == 6);
    zero_out = false;
    if (nan || f == 1) return false;
    if (f == 0) {
        zero_out = true;
        if (fl & 6) fl = 1;
        return false;
    }
    if (fl & 6) {
        if (f < 0) fl = (fl & 1) | ((fl & 2) << 1) | ((fl & 4) >> 1);
        return false;
    }
    return true;
}

// Store raw bits into an f32/f64 output cell.
__device__ __forceinline__ void store_float(void* c, bool out64, int64_t off, uint64_t bits) {
    if (out64) reinterpret_cast<uint64_t*>(c)[off] = bits;
    else reinterpret_cast<uint32_t*>(c)[off] = static_cast<uint32_t>(bits);
}

// Place a magnitude at window shift sh. Bit 0 of the window is reserved: a term
// placed whole (sh >= 1) leaves it clear; a term cut at the window's bottom keeps
// its bits from position 1 up and sets bit 0 when anything was cut (a jammed sticky
// bit that only decides rounding, as that term is then far below the result).
__device__ __forceinline__ void place_jammed(Big& mag, int sh) {
    bool cut = false, unused = false;
    if (sh >= 1) {
        big_shift_mag(mag, sh, &unused);
        return;
    }
    big_shift_mag(mag, sh - 1, &cut);  // keep the bits from position 1 - sh up
    big_shift_mag(mag, 1, &unused);    // make room for the jam bit
    if (cut) mag.w[0] |= 1;
}

// beta * C, then the combine and the encode, for one cell whose product part is the
// exact X * 2^ex with flags fl (alpha already applied).
__device__ void finish_float(const FxEpi& e, int64_t off, Big& X, int ex, int fl) {
    int pf = 0;
    i128 Y = 0;
    int ey = 0;
    if (e.beta != 0) {
        const FDec d = fdecode(static_cast<const uint8_t*>(e.c), off, e.out64);
        if (d.kind == 2) pf = 1;
        else if (d.kind == 1) pf = d.sign ? 4 : 2;
        else {
            // Complete::of (acc.rs:1007-1020) through add_scaled's placement rules.
            const int sh = d.exp - e.min_exp_e;
            if (d.mant != 0 && sh >= 0 && (sh >> 6) < e.limbs_e) {
                Y = d.sign ? -static_cast<i128>(d.mant) : static_cast<i128>(d.mant);
                ey = d.exp;
            }
        }
        bool zy;
        if (scale_flags(pf, zy, e.beta)) Y = Y * static_cast<i128>(e.beta);
        if (zy) Y = 0;
    }
    const int flags = fl | pf;
    if (flags) {
        const bool nan = (flags & 1) || ((flags & 6) == 6);
        store_float(e.c, e.out64, off, nan ? nan_bits(e.out64) : inf_bits(e.out64, (flags & 4) != 0));
        return;
    }
    // Exact sum X * 2^ex + Y * 2^ey in a window whose unit is 2^(top - 760 - 1).
    Big mx = X;
    const bool nx = big_neg(mx);
    if (nx) big_negate(mx);
    const int blx = big_bitlen(mx);
    const bool ny = Y < 0;
    const u128 uy = ny ? static_cast<u128>(-Y) : static_cast<u128>(Y);
    const int bly = uy == 0 ? 0 : (uy >> 64 ? 128 - __clzll(static_cast<long long>(uy >> 64))
                                           : 64 - __clzll(static_cast<long long>(uy)));
    if (blx == 0 && bly == 0) {
        store_float(e.c, e.out64, off, 0);
        return;
    }
    int top = INT_MIN;
    if (blx) top = ex + blx;
    if (bly && ey + bly > top) top = ey + bly;
    const int unit = top - 760 - 1;
    Big W;
    big_zero(W);
    if (blx) {
        place_jammed(mx, ex - unit);
        if (nx) big_negate(mx);
        big_add(W, mx);
    }
    if (bly) {
        Big my;
        big_zero(my);
        my.w[0] = static_cast<uint64_t>(uy);
        my.w[1] = static_cast<uint64_t>(uy >> 64);
        place_jammed(my, ey - unit);
        if (ny) big_negate(my);
        big_add(W, my);
    }
    store_float(e.c, e.out64, off, encode_words<BW>(W.w, unit, e.out64, e.mode, e.min_exp_e));
}

// ------------------------------------------------------------ K6 pre-passes

// One warp per row of A: lowest set-bit and top-bit exponents over finite nonzero
// elements, and whether the row holds a non-finite element.
// Spans are recorded per row (0 for a row with no finite nonzero element); gmax[3]
// collects SPAN_CAP - (smallest nonzero span), gmax[0] the largest span.
constexpr int SPAN_CAP = 1 << 20;

// One f32 element's part of a row's or column's statistics from its bit pattern: the same
// exponents fdecode gives (bit 0 of the odd part, leading one), in 32-bit arithmetic.
__device__ __forceinline__ void fx_stat32(uint32_t bits, int& l, int& h, int& f) {
    const uint32_t biased = (bits >> 23) & 0xFFu, frac = bits & 0x7FFFFFu;
    if (biased == 0xFFu) {
        f = 1;
        return;
    }
    const uint32_t mant = biased ? (frac | 0x800000u) : frac;
    if (!mant) return;
    const int e = (biased ? static_cast<int>(biased) : 1) - 150;
    l = min(l, e + __ffs(static_cast<int>(mant)) - 1);
    h = max(h, e + 31 - __clz(static_cast<int>(mant)));
}

__global__ void fx_rows_kernel(const uint8_t* __restrict__ a, int64_t rsa, int64_t csa, int m,
                               int k, bool f64, int* __restrict__ lo, int* __restrict__ span,
                               uint8_t* __restrict__ nf, int* __restrict__ gmax) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= m) return;
    int l = INT_MAX, h = INT_MIN, f = 0;
    // f32 rows of unit stride on 16-byte boundaries: four elements per load, four loads
    // in flight per lane
    const bool vec = !f64 && csa == 1 && (k & 3) == 0 &&
                     ((reinterpret_cast<uintptr_t>(a) | static_cast<uintptr_t>(rsa * 4)) & 15) == 0;
    if (vec) {
        const uint4* row = reinterpret_cast<const uint4*>(a + static_cast<int64_t>(warp) * rsa * 4);
#pragma unroll 4
        for (int q = lane; q < (k >> 2); q += 32) {
            const uint4 v = __ldg(row + q);
            fx_stat32(v.x, l, h, f);
            fx_stat32(v.y, l, h, f);
            fx_stat32(v.z, l, h, f);
            fx_stat32(v.w, l, h, f);
        }
    }
    for (int p = vec ? k : lane; p < k; p += 32) {
        const FDec d = fdecode(a, static_cast<int64_t>(warp) * rsa + static_cast<int64_t>(p) * csa, f64);
        if (d.kind != 0) f = 1;
        else if (d.mant) {
            const int tz = __ffsll(static_cast<long long>(d.mant)) - 1;
            const int bl = 64 - __clzll(static_cast<long long>(d.mant));
            l = min(l, d.exp + tz);
            h = max(h, d.exp + bl - 1);
        }
    }
    for (int o = 16; o; o >>= 1) {
        l = min(l, __shfl_xor_sync(0xffffffffu, l, o));
        h = max(h, __shfl_xor_sync(0xffffffffu, h, o));
        f |= __shfl_xor_sync(0xffffffffu, f, o);
    }
    if (lane == 0) {
        lo[warp] = l == INT_MAX ? 0 : l;
        span[warp] = l == INT_MAX ? 0 : h - l + 1;
        nf[warp] = static_cast<uint8_t>(f);
        if (l != INT_MAX) {
            atomicMax(&gmax[0], h - l + 1);
            atomicMax(&gmax[3], SPAN_CAP - (h - l + 1));
        }
        if (f) atomicOr(&gmax[2], 1);
    }
}

// 32 columns of B per block of 32 x 32 threads: lane x owns column j0 + x, warp y
// walks rows y, y + 32, ...; the warps' results meet in shared memory.
__global__ void fx_cols_kernel(const uint8_t* __restrict__ b, int64_t rsb, int64_t csb, int k,
                               int n, bool f64, int* __restrict__ lo, int* __restrict__ span,
                               uint8_t* __restrict__ nf, int* __restrict__ gmax) {
    __shared__ int sl[32][33], sh[32][33], sf[32][33];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const int j = blockIdx.x * 32 + tx;
    int l = INT_MAX, h = INT_MIN, f = 0;
    if (j < n) {
        for (int p = ty; p < k; p += 32) {
            const FDec d = fdecode(b, static_cast<int64_t>(p) * rsb + static_cast<int64_t>(j) * csb, f64);
            if (d.kind != 0) f = 1;
            else if (d.mant) {
                const int tz = __ffsll(static_cast<long long>(d.mant)) - 1;
                const int bl = 64 - __clzll(static_cast<long long>(d.mant));
                l = min(l, d.exp + tz);
                h = max(h, d.exp + bl - 1);
            }
        }
    }
    sl[ty][tx] = l;
    sh[ty][tx] = h;
    sf[ty][tx] = f;
    __syncthreads();
    if (ty == 0 && j < n) {
        for (int r = 1; r < 32; ++r) {
            l = min(l, sl[r][tx]);
            h = max(h, sh[r][tx]);
            f |= sf[r][tx];
        }
        lo[j] = l == INT_MAX ? 0 : l;
        span[j] = l == INT_MAX ? 0 : h - l + 1;
        nf[j] = static_cast<uint8_t>(f);
        if (l != INT_MAX) {
            atomicMax(&gmax[1], h - l + 1);
            atomicMax(&gmax[4], SPAN_CAP - (h - l + 1));
        }
        if (f) atomicOr(&gmax[2], 1);
    }
}

// f32 columns of a row-major B with rows on 16-byte boundaries: 128 columns by a range of
// rows per block of 32 x 8 threads, lane x reading columns j0 + 4x .. j0 + 4x + 3 as one
// 16-byte load, warp y rows y, y + 8, ...; the block's partial minimum / maximum / flag per
// column meet in shared memory and then in the per-column words cl, ch, cf by atomics
// (cl starts at FX_CL0 = 0x7F7F7F7F, ch at 0x80808080, both beyond any exponent), which
// fx_cols_finish turns into lo, span, nf.
constexpr int FX_CL0 = 0x7F7F7F7F;

__global__ void fx_cols4_kernel(const uint8_t* __restrict__ b, int64_t rsb, int k, int n,
                                int rows_per_block, int* __restrict__ cl, int* __restrict__ ch,
                                int* __restrict__ cf) {
    __shared__ int sl[8][128], sh[8][128], sf[8][128];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const int j = blockIdx.x * 128 + 4 * tx;
    const int p0 = blockIdx.y * rows_per_block;
    const int p1 = min(k, p0 + rows_per_block);
    int l[4] = {INT_MAX, INT_MAX, INT_MAX, INT_MAX}, h[4] = {INT_MIN, INT_MIN, INT_MIN, INT_MIN};
    int f[4] = {0, 0, 0, 0};
    if (j < n) {
#pragma unroll 4
        for (int p = p0 + ty; p < p1; p += 8) {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(b + (static_cast<int64_t>(p) * rsb + j) * 4));
            fx_stat32(v.x, l[0], h[0], f[0]);
            fx_stat32(v.y, l[1], h[1], f[1]);
            fx_stat32(v.z, l[2], h[2], f[2]);
            fx_stat32(v.w, l[3], h[3], f[3]);
        }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        sl[ty][4 * tx + c] = l[c];
        sh[ty][4 * tx + c] = h[c];
        sf[ty][4 * tx + c] = f[c];
    }
    __syncthreads();
    const int t = ty * 32 + tx;
    if (t < 128) {
        int L = INT_MAX, H = INT_MIN, F = 0;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            L = min(L, sl[r][t]);
            H = max(H, sh[r][t]);
            F |= sf[r][t];
        }
        const int jj = blockIdx.x * 128 + t;
        if (jj < n) {
            if (L != INT_MAX) {
                atomicMin(cl + jj, L);
                atomicMax(ch + jj, H);
            }
            if (F) atomicOr(cf + jj, 1);
        }
    }
}

__global__ void fx_cols_finish(int n, const int* __restrict__ cl, const int* __restrict__ ch,
                               const int* __restrict__ cf, int* __restrict__ lo,
                               int* __restrict__ span, uint8_t* __restrict__ nf,
                               int* __restrict__ gmax) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    const bool in = j < n;
    const int l = in ? cl[j] : FX_CL0;
    const bool any = l != FX_CL0;
    const int sp = any ? ch[j] - l + 1 : 0;
    const int fl = in ? cf[j] : 0;
    if (in) {
        lo[j] = any ? l : 0;
        span[j] = sp;
        nf[j] = static_cast<uint8_t>(fl != 0);
    }
    // one atomic per warp for each global word
    const int mspan = __reduce_max_sync(0xffffffffu, any ? sp : 0);
    const int mcap = __reduce_max_sync(0xffffffffu, any ? SPAN_CAP - sp : 0);
    const int mf = __reduce_or_sync(0xffffffffu, fl != 0 ? 1 : 0);
    if ((threadIdx.x & 31) == 0) {
        if (mspan) atomicMax(&gmax[1], mspan);
        if (mcap) atomicMax(&gmax[4], mcap);
        if (mf) atomicOr(&gmax[2], 1);
    }
}

// Balanced base-256 digits of the exact scaled integer of one element.
__device__ __forceinline__ i128 fx_scaled(const FDec& d, int lo) {
    if (d.kind != 0 || d.mant == 0) return 0;
    const int tz = __ffsll(static_cast<long long>(d.mant)) - 1;
    const int sh = d.exp + tz - lo;  // >= 0 by the choice of lo
    const i128 v = static_cast<i128>(d.mant >> tz) << sh;
    return d.sign ? -v : v;
}

// Balanced digits from plain bytes: with C_L = sum_{s<L} 128 256^s, x + C_L lies in
// [0, 256^L) whenever x has an L-digit balanced form, and its byte s is d_s + 128; so digit
// s is byte s of the unsigned 128-bit x + C_L with its top bit flipped.
__device__ __forceinline__ void fx_biased(const FDec& d, int lo, u128 cl, uint64_t& ylo,
                                          uint64_t& yhi) {
    const u128 y = static_cast<u128>(fx_scaled(d, lo)) + cl;
    ylo = static_cast<uint64_t>(y);
    yhi = static_cast<uint64_t>(y >> 64);
}

// Byte s of four biased values, packed little-endian, as four digits.
__device__ __forceinline__ uint32_t fx_pack_digits(const uint64_t (&lo)[4], const uint64_t (&hi)[4],
                                                   int s) {
    uint32_t w = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint64_t v = s < 8 ? lo[c] >> (8 * s) : hi[c] >> (8 * (s - 8));
        w |= static_cast<uint32_t>(v & 255u) << (8 * c);
    }
    return w ^ 0x80808080u;
}

// A (m x k) -> As[L][mp][kp]: four consecutive reduction positions per thread, one 4-byte
// store per digit plane.
__global__ void fx_slice_a_kernel(int8_t* __restrict__ as, int L, int mp, int kp,
                                  const uint8_t* __restrict__ a, int64_t rsa, int64_t csa,
                                  bool f64, int m, int k, const int* __restrict__ lo, u128 cl) {
    const int qpr = kp >> 2;
    const int64_t total = static_cast<int64_t>(mp) * qpr;
    const int64_t plane = static_cast<int64_t>(mp) * kp;
    for (GridWalk wk(static_cast<size_t>(qpr)); wk.idx < static_cast<size_t>(total); wk.next()) {
        const int i = static_cast<int>(wk.i);
        const int p0 = static_cast<int>(wk.j) * 4;
        uint64_t ylo[4], yhi[4];
        const int li = i < m ? lo[i] : 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int p = p0 + c;
            FDec d{};
            d.kind = 0;
            d.mant = 0;
            if (i < m && p < k)
                d = fdecode(a, static_cast<int64_t>(i) * rsa + static_cast<int64_t>(p) * csa, f64);
            fx_biased(d, li, cl, ylo[c], yhi[c]);
        }
        int8_t* dst = as + static_cast<int64_t>(i) * kp + p0;
#pragma unroll
        for (int s = 0; s < 16; ++s)
            if (s < L) *reinterpret_cast<uint32_t*>(dst + s * plane) = fx_pack_digits(ylo, yhi, s);
    }
}

// B (k x n) -> Bs[L][np][kp] (transposed) through a shared tile of 64 reduction positions x
// 32 columns of biased values.
__global__ void fx_slice_b_kernel(int8_t* __restrict__ bs, int L, int np, int kp,
                                  const uint8_t* __restrict__ b, int64_t rsb, int64_t csb,
                                  bool f64, int k, int n, const int* __restrict__ lo, u128 cl) {
    __shared__ uint64_t tlo[32][65], thi[32][65];
    const int j0 = blockIdx.x * 32;
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    const int64_t plane = static_cast<int64_t>(np) * kp;
    const int lj = j0 + tx < n ? lo[j0 + tx] : 0;
    for (int p0 = blockIdx.y * 64; p0 < kp; p0 += gridDim.y * 64) {
        for (int r = ty; r < 64; r += 8) {
            const int p = p0 + r, j = j0 + tx;
            FDec d{};
            d.kind = 0;
            d.mant = 0;
            if (p < k && j < n)
                d = fdecode(b, static_cast<int64_t>(p) * rsb + static_cast<int64_t>(j) * csb, f64);
            fx_biased(d, lj, cl, tlo[tx][r], thi[tx][r]);
        }
        __syncthreads();
        // 32 columns x 16 quads of reduction positions: two (column, quad) items per thread.
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int item = (ty * 2 + h) * 32 + tx;  // 0 .. 511
            const int jj = item >> 4, q = item & 15;
            const int j = j0 + jj, p = p0 + 4 * q;
            if (j < np && p < kp) {
                const uint64_t vlo[4] = {tlo[jj][4 * q], tlo[jj][4 * q + 1], tlo[jj][4 * q + 2],
                                         tlo[jj][4 * q + 3]};
                const uint64_t vhi[4] = {thi[jj][4 * q], thi[jj][4 * q + 1], thi[jj][4 * q + 2],
                                         thi[jj][4 * q + 3]};
                int8_t* dst = bs + static_cast<int64_t>(j) * kp + p;
#pragma unroll
                for (int s = 0; s < 16; ++s)
                    if (s < L) *reinterpret_cast<uint32_t*>(dst + s * plane) = fx_pack_digits(vlo, vhi, s);
            }
        }
        __syncthreads();
    }
}

// Per-cell product flags, visiting only the reductions that touch a non-finite.
__global__ void fx_flags_kernel(const uint8_t* __restrict__ a, int64_t rsa, int64_t csa,
                                const uint8_t* __restrict__ b, int64_t rsb, int64_t csb, bool f64,
                                int m, int k, int n, const uint8_t* __restrict__ rnf,
                                const uint8_t* __restrict__ cnf, uint8_t* __restrict__ flags) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    for (int i = blockIdx.y; i < m; i += gridDim.y) {
    int f = 0;
    if (rnf[i] || cnf[j]) {
        for (int p = 0; p < k; ++p) {
            const FDec x = fdecode(a, static_cast<int64_t>(i) * rsa + static_cast<int64_t>(p) * csa, f64);
            const FDec y = fdecode(b, static_cast<int64_t>(p) * rsb + static_cast<int64_t>(j) * csb, f64);
            f |= term_flags(x, y);
        }
    }
    flags[static_cast<size_t>(i) * n + j] = static_cast<uint8_t>(f);
    }
}

// ------------------------------------------------------------ K7 reduce

// The common cell (beta 0, finite terms): the partials are summed as
// sum_g s_g 2^(8 g) in 128-bit column sums per 64-bit word (chunk by chunk, every
// load of a chunk issued before any is used), carried into NG / 8 + 2 words, scaled
// by alpha and encoded, all in registers. The product needs no window: it is encoded
// at its own scale, exactly as the windowed path would encode it.
template <int NG>
__device__ __forceinline__ void fx_reduce_fast(const int32_t* __restrict__ part, int chunks,
                                               int groups, size_t total, size_t idx, int ex,
                                               int64_t off, const FxEpi& e) {
    constexpr int NQ = (NG + 7) / 8;
    i128 col[NQ];
#pragma unroll
    for (int q = 0; q < NQ; ++q) col[q] = 0;
    for (int q = 0; q < chunks; ++q) {
        const int32_t* pq = part + static_cast<size_t>(q) * groups * total + idx;
        int32_t v[NG];
#pragma unroll
        for (int g = 0; g < NG; ++g) v[g] = g < groups ? __ldg(pq + g * total) : 0;
#pragma unroll
        for (int g = 0; g < NG; ++g) col[g >> 3] += static_cast<i128>(v[g]) << (8 * (g & 7));
    }
    uint64_t w[NQ + 2];
    i128 carry = 0;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
        const i128 t = col[q] + carry;
        w[q] = static_cast<uint64_t>(static_cast<u128>(t));
        carry = t >> 64;
    }
    w[NQ] = static_cast<uint64_t>(static_cast<u128>(carry));
    w[NQ + 1] = carry < 0 ? ~0ull : 0ull;
    bool neg = (w[NQ + 1] >> 63) != 0;
    if (neg) {
        uint64_t c = 1;
#pragma unroll
        for (int q = 0; q < NQ + 2; ++q) {
            const uint64_t sv = ~w[q] + c;
            c = (c && sv == 0) ? 1 : 0;
            w[q] = sv;
        }
    }
    if (e.alpha != 1) {
        // alpha 0 encodes +0 (Complete::scale by 0 of a finite value).
        const uint64_t uf = e.alpha < 0 ? 0ull - static_cast<uint64_t>(e.alpha)
                                        : static_cast<uint64_t>(e.alpha);
        uint64_t c = 0;
#pragma unroll
        for (int q = 0; q < NQ + 2; ++q) {
            const u128 pr = static_cast<u128>(w[q]) * uf + c;
            w[q] = static_cast<uint64_t>(pr);
            c = static_cast<uint64_t>(pr >> 64);
        }
        neg = neg != (e.alpha < 0);
    }
    store_float(e.c, e.out64, off, encode_mag_fast<NQ + 2>(w, neg, ex, e.out64, e.mode, e.min_exp_e));
}

template <int NG>
__global__ void fx_reduce_kernel(const int32_t* __restrict__ part, int chunks, int groups, int m,
                                 int n, const int* __restrict__ rlo, const int* __restrict__ clo,
                                 const uint8_t* __restrict__ flags, FxEpi e) {
    const size_t total = static_cast<size_t>(m) * n;
    for (GridWalk wk(static_cast<size_t>(n)); wk.idx < total; wk.next()) {
        const size_t idx = wk.idx;
        const int i = static_cast<int>(wk.i), j = static_cast<int>(wk.j);
        if (e.beta == 0 && !(flags && flags[idx])) {
            const int64_t off = static_cast<int64_t>(i) * e.rsc + static_cast<int64_t>(j) * e.csc;
            fx_reduce_fast<NG>(part, chunks, groups, total, idx, rlo[i] + clo[j], off, e);
            continue;
        }
        Big X;
        big_zero(X);
        for (int g = 0; g < groups; ++g) {
            int64_t s = 0;
            for (int q = 0; q < chunks; ++q) s += part[(static_cast<size_t>(q) * groups + g) * total + idx];
            if (s) big_add_i64_shl(X, s, 8 * g);
        }
        int fl = flags ? flags[idx] : 0;
        bool zero_out;
        if (scale_flags(fl, zero_out, e.alpha)) big_mul_i64(X, e.alpha);
        if (zero_out) big_zero(X);
        const int64_t off = static_cast<int64_t>(i) * e.rsc + static_cast<int64_t>(j) * e.csc;
        finish_float(e, off, X, rlo[i] + clo[j], fl);
    }
}

// ------------------------------------------------------------ lazy digits
//
// With beta 0 and finite inputs only the diagonals d >= D run on the tensor cores.
// The rest, R = sum_{d<D} S_d 256^d, is bounded without computing it:
// |S_d| <= k n_d 2^14 (n_d digit pairs on the diagonal, every digit in [-128, 127]), so
// |R| / 256^D <= Ebound. The encode of a float is monotone in the exact value, so when
// alpha (X_hi - Ebound) and alpha (X_hi + Ebound) (at scale 2^(ex + 8 D)) encode to the
// same bits, so does the exact alpha X; every other cell is listed and recomputed
// exactly, all diagonals, from the digit slices (fx_fix_kernel).

// encode_mag_fast for a magnitude below 2^128: the same steps in native 128-bit shifts.
__device__ __forceinline__ uint64_t encode_u128(u128 mag, bool neg, int unit_exp, bool out64,
                                                int mode, int min_exp_e) {
    const int MANT = out64 ? 52 : 23, EXPO = out64 ? 11 : 8;
    const int P = MANT + 1;
    const int BIAS = (1 << (EXPO - 1)) - 1;
    const int SUB = 1 - BIAS - MANT;
    const uint64_t sign_bit = out64 ? (1ull << 63) : (1ull << 31);
    const uint64_t exp_all = (1ull << EXPO) - 1;
    const uint64_t hi = static_cast<uint64_t>(mag >> 64), lo64 = static_cast<uint64_t>(mag);
    const int bl = hi ? 128 - __clzll(static_cast<long long>(hi))
                      : (lo64 ? 64 - __clzll(static_cast<long long>(lo64)) : 0);
    if (bl == 0) return 0;
    const int exp = unit_exp + bl - 1;
    int lsb_exp = exp - (P - 1) < SUB ? SUB : exp - (P - 1);
    if (lsb_exp - min_exp_e < 0) return 0;
    const int lsb = lsb_exp - unit_exp;
    uint64_t sig;
    bool round_bit = false, sticky = false;
    if (lsb <= 0) {
        sig = static_cast<uint64_t>(mag << (-lsb));  // exact: fewer than P bits
    } else if (lsb >= 128) {
        sig = 0;
        if (lsb_exp - min_exp_e != 0) {
            round_bit = lsb == 128 && (mag >> 127) != 0;
            sticky = lsb == 128 ? (mag & ((static_cast<u128>(1) << 127) - 1)) != 0 : mag != 0;
        }
    } else {
        sig = static_cast<uint64_t>(mag >> lsb) & ((1ull << P) - 1);
        if (lsb_exp - min_exp_e != 0) {
            round_bit = ((mag >> (lsb - 1)) & 1) != 0;
            sticky = lsb >= 2 && (mag & ((static_cast<u128>(1) << (lsb - 1)) - 1)) != 0;
        }
    }
    const bool inc = mode == MODE_NEAREST && round_bit && (sticky || (sig & 1));
    sig += inc ? 1 : 0;
    if (sig >> P) {
        sig >>= 1;
        lsb_exp += 1;
    }
    const uint64_t s = neg ? sign_bit : 0;
    if (sig == 0) return s;
    const int top = 63 - __clzll(static_cast<long long>(sig));
    const int value_exp = lsb_exp + top;
    if ((sig >> (P - 1)) == 1) {
        const int biased = value_exp + BIAS;
        if (biased >= static_cast<int>(exp_all)) {
            if (mode == MODE_NEAREST) return s | (exp_all << MANT);
            return s | ((exp_all - 1) << MANT) | ((1ull << MANT) - 1);
        }
        return s | (static_cast<uint64_t>(biased) << MANT) | (sig & ((1ull << MANT) - 1));
    }
    return s | sig;
}

template <int NW>
__device__ __forceinline__ uint64_t encode_signed_scaled(uint64_t (&w)[NW], int64_t alpha, int ex,
                                                         const FxEpi& e) {
    bool neg = (w[NW - 1] >> 63) != 0;
    if (neg) {
        uint64_t c = 1;
#pragma unroll
        for (int q = 0; q < NW; ++q) {
            const uint64_t sv = ~w[q] + c;
            c = (c && sv == 0) ? 1 : 0;
            w[q] = sv;
        }
    }
    if (alpha != 1) {
        const uint64_t uf = alpha < 0 ? 0ull - static_cast<uint64_t>(alpha)
                                      : static_cast<uint64_t>(alpha);
        uint64_t c = 0;
#pragma unroll
        for (int q = 0; q < NW; ++q) {
            const u128 pr = static_cast<u128>(w[q]) * uf + c;
            w[q] = static_cast<uint64_t>(pr);
            c = static_cast<uint64_t>(pr >> 64);
        }
        neg = neg != (alpha < 0);
    }
    return encode_mag_fast<NW>(w, neg, ex, e.out64, e.mode, e.min_exp_e);
}

template <int NG>
__global__ void fx_reduce_lazy_kernel(const int32_t* __restrict__ part, int chunks, int groups,
                                      int m, int n, const int* __restrict__ rlo,
                                      const int* __restrict__ clo, const int* __restrict__ rspan,
                                      const int* __restrict__ cspan, int D, uint64_t ebound,
                                      FxEpi e, uint32_t* __restrict__ list,
                                      uint32_t* __restrict__ count, uint32_t limit) {
    constexpr int NQ = (NG + 7) / 8;
    constexpr int NW = NQ + 2;
    const size_t total = static_cast<size_t>(m) * n;
    for (GridWalk wk(static_cast<size_t>(n)); wk.idx < total; wk.next()) {
        const size_t idx = wk.idx;
        const int i = static_cast<int>(wk.i), j = static_cast<int>(wk.j);
        const int64_t off = static_cast<int64_t>(i) * e.rsc + static_cast<int64_t>(j) * e.csc;
        if (rspan[i] == 0 || cspan[j] == 0) {  // a row or column of zeros: the sum is 0
            store_float(e.c, e.out64, off, 0);
            continue;
        }
        i128 col[NQ];
#pragma unroll
        for (int q = 0; q < NQ; ++q) col[q] = 0;
        for (int q = 0; q < chunks; ++q) {
            const int32_t* pq = part + static_cast<size_t>(q) * groups * total + idx;
            int32_t v[NG];
#pragma unroll
            for (int g = 0; g < NG; ++g) v[g] = g < groups ? __ldg(pq + g * total) : 0;
#pragma unroll
            for (int g = 0; g < NG; ++g) col[g >> 3] += static_cast<i128>(v[g]) << (8 * (g & 7));
        }
        uint64_t lo[NW], hi[NW];
        i128 carry_lo = -static_cast<i128>(ebound), carry_hi = static_cast<i128>(ebound);
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
            const i128 tl = col[q] + carry_lo, th = col[q] + carry_hi;
            lo[q] = static_cast<uint64_t>(static_cast<u128>(tl));
            hi[q] = static_cast<uint64_t>(static_cast<u128>(th));
            carry_lo = tl >> 64;
            carry_hi = th >> 64;
        }
        lo[NQ] = static_cast<uint64_t>(static_cast<u128>(carry_lo));
        hi[NQ] = static_cast<uint64_t>(static_cast<u128>(carry_hi));
        lo[NQ + 1] = carry_lo < 0 ? ~0ull : 0ull;
        hi[NQ + 1] = carry_hi < 0 ? ~0ull : 0ull;
        const int ex = rlo[i] + clo[j] + 8 * D;
        uint64_t blo, bhi;
        bool small = e.alpha == 1;
#pragma unroll
        for (int q = 2; q < NW; ++q) {
            small = small && lo[q] == static_cast<uint64_t>(static_cast<int64_t>(lo[1]) >> 63) &&
                    hi[q] == static_cast<uint64_t>(static_cast<int64_t>(hi[1]) >> 63);
        }
        if (small) {
            // Both ends fit 128 bits (the common case): native arithmetic.
            const i128 vl = static_cast<i128>((static_cast<u128>(lo[1]) << 64) | lo[0]);
            const i128 vh = static_cast<i128>((static_cast<u128>(hi[1]) << 64) | hi[0]);
            const u128 ml = vl < 0 ? static_cast<u128>(0) - static_cast<u128>(vl) : static_cast<u128>(vl);
            const u128 mh = vh < 0 ? static_cast<u128>(0) - static_cast<u128>(vh) : static_cast<u128>(vh);
            blo = encode_u128(ml, vl < 0, ex, e.out64, e.mode, e.min_exp_e);
            bhi = encode_u128(mh, vh < 0, ex, e.out64, e.mode, e.min_exp_e);
        } else {
            blo = encode_signed_scaled<NW>(lo, e.alpha, ex, e);
            bhi = encode_signed_scaled<NW>(hi, e.alpha, ex, e);
        }
        if (blo == bhi) {
            store_float(e.c, e.out64, off, blo);
        } else {
            const uint32_t slot = atomicAdd(count, 1u);
            if (slot < limit) list[slot] = static_cast<uint32_t>(idx);
        }
    }
}

// One warp per listed cell: S_d for every diagonal from the digit slices (4 digit
// products per dp4a, exact in 32-bit lanes summed in 64 bits), the cell's exact integer
// in the 768-bit window, alpha, and the encode.
__global__ void fx_fix_kernel(const uint32_t* __restrict__ list, const uint32_t* __restrict__ count,
                              uint32_t limit, const int8_t* __restrict__ as, int La, int mp,
                              const int8_t* __restrict__ bs, int Lb, int np, int kp, int n,
                              const int* __restrict__ rlo, const int* __restrict__ clo, FxEpi e) {
    const uint32_t cells = min(*count, limit);
    const int lane = threadIdx.x & 31;
    const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
    for (uint32_t w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < cells; w += warps) {
        const uint32_t idx = list[w];
        const int i = static_cast<int>(idx / n), j = static_cast<int>(idx % n);
        Big X;
        big_zero(X);
        for (int d = 0; d <= La + Lb - 2; ++d) {
            long long acc = 0;
            const int s0 = d - (Lb - 1) > 0 ? d - (Lb - 1) : 0;
            const int s1 = d < La - 1 ? d : La - 1;
            for (int sa = s0; sa <= s1; ++sa) {
                const int8_t* ar = as + (static_cast<int64_t>(sa) * mp + i) * kp;
                const int8_t* bc = bs + (static_cast<int64_t>(d - sa) * np + j) * kp;
                int part = 0;
                for (int p = lane * 4; p < kp; p += 128) {
                    part = __dp4a(*reinterpret_cast<const int*>(ar + p),
                                  *reinterpret_cast<const int*>(bc + p), part);
                    if (((p >> 7) & 1023) == 1023) {  // stay far inside 32 bits
                        acc += part;
                        part = 0;
                    }
                }
                acc += part;
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (lane == 0 && acc) big_add_i64_shl(X, static_cast<int64_t>(acc), 8 * d);
        }
        if (lane == 0) {
            if (e.alpha != 1) big_mul_i64(X, e.alpha);
            const int64_t off = static_cast<int64_t>(i) * e.rsc + static_cast<int64_t>(j) * e.csc;
            store_float(e.c, e.out64, off,
                        encode_words<BW>(X.w, rlo[i] + clo[j], e.out64, e.mode, e.min_exp_e));
        }
    }
}

// ------------------------------------------------------------ modular route
//
// The modular route (modular.cuh): the scaled integers of the digit route (A_ip 2^-lo_i,
// B_pj 2^-lo_j) reduced modulo nm coprime moduli into balanced int8 residues, one int8 GEMM
// per modulus, and the CRT rebuilding each cell's exact integer S, |S| <= k (2^span_A - 1)
// (2^span_B - 1). Then the epilogue and encode of the digit route.

// Bytes of the 2^s table in shared memory (beside the B slicer's 25 KB static tile).
constexpr int FM_TABLE_MAX = 160 * 1024;

// The table of words [2^sh, 2^(sh+8), 2^(sh+16), 0] mod p_g (f32 significands, W = 1), or
// two words covering 2^(sh + 8i) for i < 8 (f64, W = 2), in 16-byte columns of four moduli
// (column w NMP/4 + g/4 holds word w of moduli 4(g/4) .. 4(g/4) + 3), each column the rows
// 2 sh (positive) and 2 sh + 1 (negative) one after another: lanes reading different rows
// of one column spread over all the banks.
__device__ __forceinline__ void fm_fill_pow2(uint32_t* pw, const uint32_t* __restrict__ table,
                                             int words) {
    for (int idx = threadIdx.y * blockDim.x + threadIdx.x; idx < words;
         idx += blockDim.x * blockDim.y)
        pw[idx] = table[idx];
}

// One element's scaled integer as (odd-part mantissa, shift, sign); zero for a zero or
// non-finite element (non-finite terms are resolved by the flags pass).
__device__ __forceinline__ void fm_parts(const FDec& d, int lo, uint64_t& mant, int& sh, bool& neg) {
    if (d.kind != 0 || d.mant == 0) {
        mant = 0, sh = 0, neg = false;
        return;
    }
    const int tz = __ffsll(static_cast<long long>(d.mant)) - 1;
    mant = d.mant >> tz;
    sh = d.exp + tz - lo;
    neg = d.sign != 0;
}

// The residues of four elements for all NM moduli, packed four per 32-bit word and stored
// to dst + g * plane (one word per modulus). W: table words per (shift, modulus).
template <int NM, int W>
__device__ __forceinline__ void fm_store_residues(int8_t* dst, int64_t plane, const uint64_t (&mant)[4],
                                                  const int (&sh)[4], const bool (&neg)[4],
                                                  const uint32_t* pw, int rows, const FmParams& f) {
    constexpr int NMP = (NM + 3) / 4 * 4;
    // Modulus-outer: each modulus's constants and each element's coefficient words are read
    // once for the four elements, and each output word is stored as soon as it is complete.
    // A zero element reads row 0 and its residue comes out 0 (u = half).
    uint32_t lo32[4], hi32[4];
    int row[4];
    const uint4* tab = reinterpret_cast<const uint4*>(pw);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        lo32[c] = static_cast<uint32_t>(mant[c]);
        hi32[c] = static_cast<uint32_t>(mant[c] >> 32);
        // rows 2 sh (positive) and 2 sh + 1 (the coefficients of -2^(sh + 8i))
        row[c] = 2 * sh[c] + (neg[c] ? 1 : 0);
    }
#pragma unroll
    for (int g4 = 0; g4 < NMP / 4; ++g4) {
        uint4 cw[4], ch[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            cw[c] = tab[g4 * rows + row[c]];
            ch[c] = W == 2 ? tab[(NMP / 4 + g4) * rows + row[c]] : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int gi = 0; gi < 4; ++gi) {
            const int g = 4 * g4 + gi;
            if (g >= NM) break;
            const uint32_t half = f.half[g], pneg = f.pneg[g], mg = f.magic32[g], hneg = f.hneg[g];
            uint32_t word = 0;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t lo = gi == 0 ? cw[c].x : gi == 1 ? cw[c].y : gi == 2 ? cw[c].z : cw[c].w;
                uint32_t v = __dp4a(lo32[c], lo, half);  // v + half
                if (W == 2) {
                    const uint32_t hi = gi == 0 ? ch[c].x : gi == 1 ? ch[c].y : gi == 2 ? ch[c].z : ch[c].w;
                    v = __dp4a(hi32[c], hi, v);
                }
                word = fm_put_byte(word, fm_balanced_vh(v, pneg, mg, hneg), c);
            }
            *reinterpret_cast<uint32_t*>(dst + g * plane) = word;
        }
    }
}

// A (m x k) -> residue planes As[NM][mp][kp]: four consecutive reduction positions per
// thread, one 4-byte store per modulus.
template <int NM, bool F64>
__global__ void __launch_bounds__(256, 4) fm_slice_a_kernel(int8_t* __restrict__ as, int mp, int kp, const uint8_t* __restrict__ a,
                                  int64_t rsa, int64_t csa, int m, int k,
                                  const int* __restrict__ lo, const uint32_t* __restrict__ pow2,
                                  int shmax, FmParams f) {
    constexpr int NMP = (NM + 3) / 4 * 4;
    extern __shared__ __align__(16) uint32_t pw[];
    constexpr bool f64 = F64;
    constexpr int W = F64 ? 2 : 1;
    // f32 rows with unit column stride on 16-byte boundaries take one vector load per thread
    const bool vec = !f64 && csa == 1 && (reinterpret_cast<uintptr_t>(a) & 15) == 0 &&
                     ((rsa * 4) & 15) == 0;
    fm_fill_pow2(pw, pow2, 2 * shmax * W * NMP);
    __syncthreads();
    const int qpr = kp >> 2;
    const int64_t total = static_cast<int64_t>(mp) * qpr;
    const int64_t plane = static_cast<int64_t>(mp) * kp;
    // Each step's 16 bytes and row exponent are loaded one step ahead, so the loads are in
    // flight while the previous quad's residues are computed.
    auto fetch = [&](const GridWalk& w, uint4& q, int& l) {
        const int i = static_cast<int>(w.i), p0 = static_cast<int>(w.j) * 4;
        l = i < m ? __ldg(lo + i) : 0;
        q = (vec && i < m && p0 + 3 < k)
                ? __ldg(reinterpret_cast<const uint4*>(a + (static_cast<int64_t>(i) * rsa + p0) * 4))
                : make_uint4(0, 0, 0, 0);
    };
    GridWalk wk(static_cast<size_t>(qpr));
    uint4 qc = make_uint4(0, 0, 0, 0);
    int lc = 0;
    if (wk.idx < static_cast<size_t>(total)) fetch(wk, qc, lc);
    while (wk.idx < static_cast<size_t>(total)) {
        GridWalk nx = wk;
        nx.next();
        uint4 qn = make_uint4(0, 0, 0, 0);
        int ln = 0;
        if (nx.idx < static_cast<size_t>(total)) fetch(nx, qn, ln);
        const int i = static_cast<int>(wk.i);
        const int p0 = static_cast<int>(wk.j) * 4;
        uint64_t mant[4];
        int sh[4];
        bool neg[4];
        const int li = lc;
        if (vec && i < m && p0 + 3 < k) {
            // four consecutive f32 elements, one 16-byte load
            const uint32_t bits[4] = {qc.x, qc.y, qc.z, qc.w};
#pragma unroll
            for (int c = 0; c < 4; ++c) fm_parts(fdecode_bits(bits[c], false), li, mant[c], sh[c], neg[c]);
        } else {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int p = p0 + c;
                FDec d{};
                if (i < m && p < k)
                    d = fdecode(a, static_cast<int64_t>(i) * rsa + static_cast<int64_t>(p) * csa, f64);
                fm_parts(d, li, mant[c], sh[c], neg[c]);
            }
        }
        fm_store_residues<NM, W>(as + static_cast<int64_t>(i) * kp + p0, plane, mant, sh, neg, pw, 2 * shmax, f);
        wk = nx;
        qc = qn;
        lc = ln;
    }
}

// B (k x n) -> residue planes Bs[NM][np][kp] (transposed) through a shared tile of 64
// reduction positions x 32 columns of decoded elements.
template <int NM, bool F64>
__global__ void fm_slice_b_kernel(int8_t* __restrict__ bs, int np, int kp, const uint8_t* __restrict__ b,
                                  int64_t rsb, int64_t csb, int k, int n,
                                  const int* __restrict__ lo, const uint32_t* __restrict__ pow2,
                                  int shmax, FmParams f) {
    constexpr int NMP = (NM + 3) / 4 * 4;
    extern __shared__ __align__(16) uint32_t pw[];
    using MT = typename std::conditional<F64, uint64_t, uint32_t>::type;  // significand < 2^24 for f32
    __shared__ MT tm[32][65];
    __shared__ int ts[32][65];
    constexpr bool f64 = F64;
    constexpr int W = F64 ? 2 : 1;
    fm_fill_pow2(pw, pow2, 2 * shmax * W * NMP);
    const int j0 = blockIdx.x * 32;
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    const int64_t plane = static_cast<int64_t>(np) * kp;
    const int lj = j0 + tx < n ? lo[j0 + tx] : 0;
    __syncthreads();
    for (int p0 = blockIdx.y * 64; p0 < kp; p0 += gridDim.y * 64) {
        // eight rows per thread, their loads issued before any decode
        uint64_t raw[8];
        bool ok[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int p = p0 + ty + 8 * i, j = j0 + tx;
            ok[i] = p < k && j < n;
            const int64_t at = static_cast<int64_t>(p) * rsb + static_cast<int64_t>(j) * csb;
            raw[i] = !ok[i] ? 0ull
                     : f64  ? __ldg(reinterpret_cast<const unsigned long long*>(b) + at)
                            : __ldg(reinterpret_cast<const uint32_t*>(b) + at);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int r = ty + 8 * i;
            FDec d{};
            if (ok[i]) d = fdecode_bits(raw[i], f64);
            uint64_t mant;
            int sh;
            bool neg;
            fm_parts(d, lj, mant, sh, neg);
            tm[tx][r] = static_cast<MT>(mant);
            ts[tx][r] = sh | (neg ? 1 << 30 : 0);
        }
        __syncthreads();
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
            const int item = (ty * 2 + h) * 32 + tx;  // 32 columns x 16 quads
            const int jj = item >> 4, q = item & 15;
            const int j = j0 + jj, p = p0 + 4 * q;
            if (j < np && p < kp) {
                uint64_t mant[4];
                int sh[4];
                bool neg[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    mant[c] = tm[jj][4 * q + c];
                    sh[c] = ts[jj][4 * q + c] & ((1 << 30) - 1);
                    neg[c] = (ts[jj][4 * q + c] >> 30) != 0;
                }
                fm_store_residues<NM, W>(bs + static_cast<int64_t>(j) * kp + p, plane, mant, sh, neg, pw, 2 * shmax, f);
            }
        }
        __syncthreads();
    }
}

// The encode of S 2^ex from its 32-bit limbs (two's complement, sign extension ext) for
// alpha 1, rounding to nearest and a normal result: the top nonzero limb and the two below
// it, shifted so the leading one is bit 95, give the significand, the round bit and the
// window's sticky bits; the limbs further down only feed the sticky bit. False (nothing
// stored) when the result would be subnormal, overflow or sit at the element register's
// lowest bit; encode_mag_fast covers those.
template <int NL>
__device__ __forceinline__ bool fm_encode_fast(const uint32_t (&limb)[NL], uint32_t ext, int ex,
                                               const FxEpi& e, uint64_t& bits) {
    const bool neg = ext != 0;
    const uint32_t flip = neg ? ~0u : 0u;
    uint32_t mag[NL];
    uint32_t c = neg ? 1u : 0u;
#pragma unroll
    for (int l = 0; l < NL; ++l) {
        const uint64_t sum = static_cast<uint64_t>(limb[l] ^ flip) + c;
        mag[l] = static_cast<uint32_t>(sum);
        c = static_cast<uint32_t>(sum >> 32);
    }
    int h = -1;
    uint32_t top = 0, t1 = 0, t2 = 0, below = 0, acc = 0;  // acc: OR of mag[0 .. l - 3]
#pragma unroll
    for (int l = 0; l < NL; ++l) {
        if (mag[l]) {
            h = l;
            top = mag[l];
            t1 = l >= 1 ? mag[l >= 1 ? l - 1 : 0] : 0u;
            t2 = l >= 2 ? mag[l >= 2 ? l - 2 : 0] : 0u;
            below = acc;
        }
        if (l >= 2) acc |= mag[l >= 2 ? l - 2 : 0];
    }
    if (h < 0) {
        bits = 0;  // exact zero encodes +0
        return true;
    }
    const int lz = __clz(top);
    const uint32_t w_hi = __funnelshift_l(t1, top, lz);
    const uint32_t w_mid = __funnelshift_l(t2, t1, lz);
    const uint32_t w_lo = t2 << lz;
    const int exp = ex + 32 * h + 31 - lz;  // exponent of the leading one
    const int MANT = e.out64 ? 52 : 23;
    const int BIAS = e.out64 ? 1023 : 127;
    if (exp < 1 - BIAS || exp > BIAS - 1 || exp - MANT <= e.min_exp_e) return false;
    uint64_t sig;
    bool rnd, sticky;
    if (!e.out64) {
        sig = w_hi >> 8;
        rnd = ((w_hi >> 7) & 1u) != 0;
        sticky = ((w_hi & 0x7Fu) | w_mid | w_lo | below) != 0;
    } else {
        const uint64_t w64 = (static_cast<uint64_t>(w_hi) << 32) | w_mid;
        sig = w64 >> 11;
        rnd = ((w64 >> 10) & 1u) != 0;
        sticky = ((w_mid & 0x3FFu) | w_lo | below) != 0;
    }
    sig += (rnd && (sticky || (sig & 1))) ? 1 : 0;
    int be = exp + BIAS;
    if (sig >> (MANT + 1)) {
        sig >>= 1;
        ++be;
    }
    const uint64_t sgn = neg ? (e.out64 ? 1ull << 63 : 1ull << 31) : 0ull;
    bits = sgn | (static_cast<uint64_t>(be) << MANT) | (sig & ((1ull << MANT) - 1));
    return true;
}

// The fast case for f32 results from a 64-bit window of S's limbs: the limb h at the top
// that is not the sign's extension over the limb below it, or limb h alone under the
// extension word when its top bit disagrees with the sign; either way at least 31
// significant bits. The limbs under the window only decide whether S lies strictly
// between two steps of the window, so their OR is jammed into bit 0, seven or more bits
// below the round bit (a value strictly inside a step and the jammed window round alike;
// bit 0 is never a halfway point there), and the int64 -> f32 conversion, round to
// nearest even, rounds the window as it rounds S. The window's unit 2^(32 w + ex) then
// goes into the exponent field. False under the same conditions as fm_encode_fast.
template <int NL>
__device__ __forceinline__ bool fm_encode_f32_window(const uint32_t (&limb)[NL], uint32_t ext, int ex,
                                                     const FxEpi& e, uint64_t& bits) {
    uint32_t hi = ext, lo = limb[0];
    int w = 0;  // the window's low limb
    bool found = false;
#pragma unroll
    for (int l = NL - 1; l >= 1; --l) {
        const bool take = !found && limb[l] != ext;
        hi = take ? limb[l] : hi;
        lo = take ? limb[l - 1] : lo;
        w = take ? l - 1 : w;
        found = found || take;
    }
    if (found && ((hi ^ ext) >> 31) != 0) {
        lo = hi;
        hi = ext;
        ++w;
    }
    uint32_t below = 0;
#pragma unroll
    for (int l = 0; l < NL - 1; ++l) below |= l < w ? limb[l] : 0u;
    const int64_t W = static_cast<int64_t>((static_cast<uint64_t>(hi) << 32) | lo) | (below != 0 ? 1 : 0);
    const uint64_t mag = ext != 0 ? 0ull - static_cast<uint64_t>(W) : static_cast<uint64_t>(W);
    if (mag == 0) {
        bits = 0;  // exact zero encodes +0
        return true;
    }
    const int exp = ex + 32 * w + 63 - __clzll(static_cast<long long>(mag));  // of S's leading one
    if (exp < 1 - 127 || exp > 127 || exp - 23 <= e.min_exp_e) return false;
    bits = __float_as_uint(__ll2float_rn(W)) + static_cast<uint32_t>(ex + 32 * w) * (1u << 23);
    return true;
}

// beta != 0 or non-finite terms: the register form and finish_float.
template <int NW>
__device__ __forceinline__ void fm_finish_slow(const uint64_t (&w)[NW], uint64_t ext, int64_t off, int ex,
                                            int fl0, const FxEpi& e) {
    Big X;
#pragma unroll
    for (int q = 0; q < BW; ++q) X.w[q] = q < NW ? w[q] : ext;
    int fl = fl0;
    bool zero_out;
    if (scale_flags(fl, zero_out, e.alpha)) big_mul_i64(X, e.alpha);
    if (zero_out) big_zero(X);
    finish_float(e, off, X, ex, fl);
}

// A cell's limbs of S (sign extension ext) to its output: the fast encode (beta 0, finite
// terms) or finish_float.
template <int NM>
__device__ __forceinline__ void fm_finish_cell(const uint32_t (&limb)[FmLimbs<NM>::value], uint32_t ext32,
                                               int64_t off, int ex, int fl0, const FxEpi& e) {
    constexpr int NL = FmLimbs<NM>::value;
    constexpr int NW = (NL + 1) / 2 + 2;  // 64-bit words: the value, alpha's 64 bits, sign
    if (e.beta == 0 && !fl0 && e.alpha == 1 && e.mode == MODE_NEAREST) {
        uint64_t bits;
        if (e.out64 ? fm_encode_fast<NL>(limb, ext32, ex, e, bits)
                    : fm_encode_f32_window<NL>(limb, ext32, ex, e, bits)) {
            store_float(e.c, e.out64, off, bits);
            return;
        }
    }
    const uint64_t ext = ext32 ? ~0ull : 0ull;
    uint64_t w[NW];
#pragma unroll
    for (int q = 0; q < NW; ++q) {
        const uint64_t lo = 2 * q < NL ? limb[2 * q] : ext32;
        const uint64_t hi = 2 * q + 1 < NL ? limb[2 * q + 1] : ext32;
        w[q] = lo | hi << 32;
    }
    if (e.beta == 0 && !fl0) {
        store_float(e.c, e.out64, off, encode_signed_scaled<NW>(w, e.alpha, ex, e));
        return;
    }
    fm_finish_slow<NW>(w, ext, off, ex, fl0, e);
}

// One thread per cell: y_g (stored by the GEMM epilogue when there is one reduction
// chunk; else rebuilt from the chunks' residues), t, the base-256 columns of X - t M
// carried into signed 32-bit limbs, then the encode.
template <int NM>
__global__ void __launch_bounds__(256, 4) fm_crt_kernel(const uint8_t* __restrict__ res, int chunks, int m, int n,
                              const int* __restrict__ rlo, const int* __restrict__ clo,
                              const int* __restrict__ rspan, const int* __restrict__ cspan,
                              const uint8_t* __restrict__ flags, FxEpi e, FmParams f) {
    constexpr int NL = FmLimbs<NM>::value;
    const size_t total = static_cast<size_t>(m) * n;
    for (GridWalk wk(static_cast<size_t>(n)); wk.idx < total; wk.next()) {
        const size_t idx = wk.idx;
        const int i = static_cast<int>(wk.i), j = static_cast<int>(wk.j);
        const int64_t off = static_cast<int64_t>(i) * e.rsc + static_cast<int64_t>(j) * e.csc;
        const int fl0 = flags ? flags[idx] : 0;
        if (e.beta == 0 && !fl0 && (rspan[i] == 0 || cspan[j] == 0)) {
            store_float(e.c, e.out64, off, 0);  // a row or column of zeros: S = 0
            continue;
        }
        uint32_t y[NM];
        fm_load_y<NM>(res, chunks, total, idx, f, y);
        uint32_t limb[NL];
        const uint32_t ext = fm_crt<NM>(y, f, limb);
        fm_finish_cell<NM>(limb, ext, off, rlo[i] + clo[j], fl0, e);
    }
}

// The same for one reduction chunk and rows of a multiple of four cells, four cells per
// thread: one 32-bit load per residue plane covers the four cells' y_g, and two byte_perm
// per four moduli gather one cell's packed words (the residue planes are modulus-major, the
// columns want four moduli of one cell per word).
template <int NM>
__global__ void __launch_bounds__(256, 3) fm_crt4_kernel(const uint8_t* __restrict__ res, int m, int n,
                              const int* __restrict__ rlo, const int* __restrict__ clo,
                              const int* __restrict__ rspan, const int* __restrict__ cspan,
                              const uint8_t* __restrict__ flags, FxEpi e, FmParams f) {
    constexpr int NA = (NM + 3) / 4;
    constexpr int NL = FmLimbs<NM>::value;
    const size_t total = static_cast<size_t>(m) * n;
    const size_t quads = total >> 2;
    for (GridWalk wk(static_cast<size_t>(n >> 2)); wk.idx < quads; wk.next()) {
        const int i = static_cast<int>(wk.i), j0 = static_cast<int>(wk.j) * 4;
        const size_t idx0 = wk.idx * 4;
        uint32_t wq[4 * NA];  // wq[g]: y_g of the four cells, one per byte
#pragma unroll
        for (int g = 0; g < 4 * NA; ++g)
            wq[g] = g < NM ? __ldg(reinterpret_cast<const uint32_t*>(res + static_cast<size_t>(g) * total + idx0)) : 0u;
        const int li = rlo[i];
        const bool row_zero = rspan[i] == 0;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
            const int j = j0 + c;
            const size_t idx = idx0 + c;
            const int64_t off = static_cast<int64_t>(i) * e.rsc + static_cast<int64_t>(j) * e.csc;
            const int fl0 = flags ? flags[idx] : 0;
            if (e.beta == 0 && !fl0 && (row_zero || cspan[j] == 0)) {
                store_float(e.c, e.out64, off, 0);  // a row or column of zeros: S = 0
                continue;
            }
            // byte c of four words: [w0.c, w1.c] then [w2.c, w3.c], joined
            const uint32_t sel = static_cast<uint32_t>(c) | (static_cast<uint32_t>(c + 4) << 4);
            uint32_t ya[NA];
#pragma unroll
            for (int a = 0; a < NA; ++a)
                ya[a] = __byte_perm(__byte_perm(wq[4 * a], wq[4 * a + 1], sel),
                                    __byte_perm(wq[4 * a + 2], wq[4 * a + 3], sel), 0x5410);
            uint32_t limb[NL];
            const uint32_t ext = fm_crt_packed<NM>(ya, f, limb);
            fm_finish_cell<NM>(limb, ext, off, li + clo[j], fl0, e);
        }
    }
}

// ---- the CRT's columns on the tensor cores
//
// With one reduction chunk the residue planes hold y_g of every cell, and the CRT's
// columns are one small integer product per block of 128 cells: Y (cells x moduli, u8)
// times W (moduli x columns, u8), W's columns the four bytes of ceil(2^32 / p_g) (the
// fixed-point sum that gives t) and the NM - 1 bytes of M / p_g (X's base-256 columns).
// Each plane is a row of the MN-major A operand, so TMA copies the planes' 128-byte runs
// straight into it (moduli past NM read as zero) and tcgen05.mma.kind::i8 (M128, K32, N 32
// or 64) sums the columns exactly in s32 TMEM lanes (each below NM 255^2 < 2^22). One
// thread per cell then reads its lane, forms t and the limbs of X - t M and encodes, as
// fm_crt4_kernel does from its dp4a columns. The per-cell encode is the cost, so one CTA
// per SM keeps four epilogue warpgroups busy, each with its own blocks, and the whole TMEM
// as slots of N columns, so the MMAs run up to 512 / N blocks ahead of the epilogues.
//   warp 0      one elected thread: TMA of each block's planes into a ring of stages;
//   warp 1      TMEM (512 columns), one elected thread issues the MMAs;
//   warps 2-17  four warpgroups; block b of this CTA goes to warpgroup b % 4 and TMEM slot
//               b % (512 / N); one cell per thread: the limbs, the encode and the store.
template <int NM>
struct FmTc {
    static constexpr int NCOL = 4 + FmColumns<NM>::value;  // F_0 .. F_3, then X_b
    static constexpr int N = NCOL <= 32 ? 32 : 64;
    static constexpr int KCH = (NM + 31) / 32;              // K32 MMAs per block
    static constexpr int STAGE = KCH * 4096;                // 32 planes x 128 cells each
    static constexpr int STAGES = 16;
    static constexpr int SLOTS = 512 / N;
};
constexpr int FMT_GROUPS = 4;
constexpr int FMT_THREADS = 64 + 128 * FMT_GROUPS;
// Waits suspend in hardware for up to this long per poll (the roles that wait most, the
// producer and the MMA issuer, then take no issue slots from the epilogues).
constexpr uint32_t FMT_HINT_NS = 100000;
// More than half of an SM's shared memory: one CTA per SM, which owns the whole TMEM.
constexpr int FMT_SMEM = 140 * 1024;

template <int NM>
__global__ void __launch_bounds__(FMT_THREADS, 1)
    fm_crt_tc_kernel(const __grid_constant__ CUtensorMap tmY, size_t total, int n,
                     const int* __restrict__ rlo, const int* __restrict__ clo,
                     const int* __restrict__ rspan, const int* __restrict__ cspan, FxEpi e,
                     FmParams f, int* status, uint64_t budget_ns) {
    using T = FmTc<NM>;
    constexpr int NB = FmColumns<NM>::value;
    constexpr int NL = FmLimbs<NM>::value;
    constexpr int S = T::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* wmat = smem + S * T::STAGE;  // B: N rows (columns) x 128 bytes (moduli)
    uint64_t* bars = reinterpret_cast<uint64_t*>(wmat + T::N * 128);
    // bars: full[S], empty[S], tfull[SLOTS], tempty[SLOTS], drain
    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + S);
    const uint32_t tfull0 = smem_u32(bars + 2 * S);
    const uint32_t tempty0 = smem_u32(bars + 2 * S + T::SLOTS);
    const uint32_t drain = smem_u32(bars + 2 * S + 2 * T::SLOTS);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 2 * T::SLOTS + 1);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const size_t nblk = (total + 127) / 128;
    // blocks of this CTA: blockIdx.x + b gridDim.x for b < nlocal
    const int nlocal = blockIdx.x < nblk ? static_cast<int>((nblk - 1 - blockIdx.x) / gridDim.x + 1) : 0;

    // W, K-major with the 128-byte swizzle: column c's moduli in row c, byte g of a row
    // at 16-byte chunk (g / 16) ^ (c % 8).
    for (int x = threadIdx.x; x < T::N * 128; x += FMT_THREADS) {
        const int c = x >> 7, g = x & 127;
        uint32_t v = 0;
        if (g < NM) {
            if (c < 4) v = f.mg[g >> 2][c] >> (8 * (g & 3));
            else if (c - 4 < NB) v = f.md[g >> 2][c - 4] >> (8 * (g & 3));
        }
        wmat[c * 128 + ((((g >> 4) ^ c) & 7) << 4) + (g & 15)] = static_cast<uint8_t>(v);
    }
    fence_proxy_async();  // the generic writes above, before the tensor core reads them
    if (threadIdx.x == 0) {
        for (int q = 0; q < S; ++q) {
            mbar_init(full0 + 8 * q, 1);
            mbar_init(empty0 + 8 * q, 1);
        }
        for (int q = 0; q < T::SLOTS; ++q) {
            mbar_init(tfull0 + 8 * q, 1);
            mbar_init(tempty0 + 8 * q, 4);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmY);
    }
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (elect_one()) {
            const uint64_t pol = l2_policy_evict_first();
            int issued = 0;  // blocks whose copies were started
            bool ok = true;
            for (int b = 0; b < nlocal; ++b) {
                const int stage = b % S;
                if (!mbar_wait_hint(empty0 + 8 * stage, ((b / S) & 1) ^ 1, budget_ns, status, KERR_TIMEOUT_PRODUCER,
                                    FMT_HINT_NS)) {
                    ok = false;
                    break;
                }
                const uint32_t fb = full0 + 8 * stage;
                mbar_expect_tx(fb, T::STAGE);
                issued = b + 1;
                const uint32_t sa = smem_u32(smem + stage * T::STAGE);
                const int x = static_cast<int>((blockIdx.x + static_cast<size_t>(b) * gridDim.x) * 128);
#pragma unroll
                for (int kc = 0; kc < T::KCH; ++kc) tma_load_2d(sa + kc * 4096, &tmY, fb, x, kc * 32, pol);
            }
            if (!ok) {
                // Let every copy in flight land before the CTA exits: those of the last S
                // blocks issued, each on its stage's full barrier with its block's parity.
                for (int b = issued > S ? issued - S : 0; b < issued; ++b)
                    mbar_wait(full0 + 8 * (b % S), (b / S) & 1, budget_ns, status, KERR_TIMEOUT_DRAIN);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        constexpr uint32_t idesc = idesc_i8(128, T::N, false, false, true, false);
        const uint32_t sw = smem_u32(wmat);
        bool ok = true, issued = false;
        for (int b = 0; b < nlocal; ++b) {
            const int stage = b % S, slot = b % T::SLOTS;
            if (!mbar_wait_warp_hint(tempty0 + 8 * slot, ((b / T::SLOTS) & 1) ^ 1, budget_ns, status,
                                     KERR_TIMEOUT_MMA_ACC, FMT_HINT_NS) ||
                !mbar_wait_warp_hint(full0 + 8 * stage, (b / S) & 1, budget_ns, status, KERR_TIMEOUT_MMA_FULL,
                                     FMT_HINT_NS)) {
                ok = false;
                break;
            }
            tc_fence_after();
            if (elect_one()) {
                const uint32_t sa = smem_u32(smem + stage * T::STAGE);
#pragma unroll
                for (int kc = 0; kc < T::KCH; ++kc)
                    mma_i8(tmem_base + slot * T::N, smem_desc_sw128(sa + kc * 4096, 4096, 1024),
                           smem_desc_sw128(sw + kc * 32, 16, 1024), idesc, kc != 0);
                mma_commit(empty0 + 8 * stage);
                mma_commit(tfull0 + 8 * slot);
                issued = true;
            }
            __syncwarp();
        }
        if (!ok) {
            if (elect_one() && issued) {
                mma_commit(drain);
                mbar_wait(drain, 0, budget_ns, status, KERR_TIMEOUT_DRAIN);
            }
            __syncwarp();
        }
    } else {
        const int group = (warp - 2) >> 2;
        const int quarter = warp & 3;  // the TMEM lane quarter this warp may read
        const int row = quarter * 32 + lane;
        // The cells of this thread, first and stride below 2^31 (total is), walked in 32 bits.
        const uint32_t un = static_cast<uint32_t>(n);
        const uint32_t stride = static_cast<uint32_t>(FMT_GROUPS) * gridDim.x * 128;
        uint32_t cell = (blockIdx.x + static_cast<uint32_t>(group) * gridDim.x) * 128 + row;
        uint32_t ci = cell / un, cj = cell - ci * un;
        const uint32_t si = stride / un, sj = stride - si * un;
        // alpha 1, beta 0, nearest, f32 out: the window encode, the rest through fm_finish_cell
        const bool fast32 = e.beta == 0 && e.alpha == 1 && e.mode == MODE_NEAREST && !e.out64;
        for (int b = group; b < nlocal; b += FMT_GROUPS) {
            const int slot = b % T::SLOTS;
            if (!mbar_wait_warp_hint(tfull0 + 8 * slot, (b / T::SLOTS) & 1, budget_ns, status,
                                     KERR_TIMEOUT_EPILOGUE, FMT_HINT_NS))
                break;
            tc_fence_after();
            uint32_t r[T::N];
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + slot * T::N;
            __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp, converged
            tmem_ld32(taddr, *reinterpret_cast<uint32_t(*)[32]>(r));
            if constexpr (T::N == 64) tmem_ld32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty0 + 8 * slot);
            if (cell < total) {
                const int64_t off = static_cast<int64_t>(ci) * e.rsc + static_cast<int64_t>(cj) * e.csc;
                if (e.beta == 0 && (rspan[ci] == 0 || cspan[cj] == 0)) {
                    store_float(e.c, e.out64, off, 0);  // a row or column of zeros: S = 0
                } else {
                    const uint32_t F[4] = {r[0], r[1], r[2], r[3]};
                    uint32_t limb[NL];
                    const uint32_t ext =
                        fm_crt_limbs_signed<NM>(fm_crt_t(F), f, [&](int c) { return r[4 + c]; }, limb);
                    const int ex = rlo[ci] + clo[cj];
                    uint64_t bits;
                    if (fast32 && fm_encode_f32_window<NL>(limb, ext, ex, e, bits))
                        reinterpret_cast<uint32_t*>(e.c)[off] = static_cast<uint32_t>(bits);
                    else
                        fm_finish_cell<NM>(limb, ext, off, ex, 0, e);
                }
            }
            cell += stride;
            ci += si;
            cj += sj;
            if (cj >= un) {
                cj -= un;
                ++ci;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 512);
    }
}

// Launches for a moduli count (even, 2 .. 40): the limbs of X < NM M with M < 2^(8 NM).
template <int NM>
static void fm_launch_slices(int8_t* as, int mp, int8_t* bs, int np, int kp, const uint8_t* a,
                             int64_t rsa, int64_t csa, const uint8_t* b, int64_t rsb, int64_t csb,
                             bool f64, int m, int k, int n, const int* rlo, const int* clo,
                             const uint32_t* pw, int shmax, const FmParams& f, cudaStream_t s,
                             cudaStream_t side) {
    constexpr int NMP = (NM + 3) / 4 * 4;
    const size_t smem = static_cast<size_t>(shmax) * 2 * NMP * 4 * (f64 ? 2 : 1);
    // The B kernel adds a 25 KB static tile: allow the table's largest size beside it.
    auto ka = f64 ? fm_slice_a_kernel<NM, true> : fm_slice_a_kernel<NM, false>;
    auto kb = f64 ? fm_slice_b_kernel<NM, true> : fm_slice_b_kernel<NM, false>;
    cudaFuncSetAttribute(ka, cudaFuncAttributeMaxDynamicSharedMemorySize, FM_TABLE_MAX);
    cudaFuncSetAttribute(kb, cudaFuncAttributeMaxDynamicSharedMemorySize, FM_TABLE_MAX);
    const int64_t aquads = static_cast<int64_t>(mp) * (kp / 4);
    const int sgrid = static_cast<int>(aquads / 256 + 1 < 148 * 16 ? aquads / 256 + 1 : 148 * 16);
    ka<<<sgrid, 256, smem, s>>>(as, mp, kp, a, rsa, csa, m, k, rlo, pw, shmax, f);
    // Each block copies the coefficient table into shared memory once, so the blocks walk
    // the reduction in strides: about eight blocks per SM in all.
    const int gx = np / 32;
    int gy = (kp + 63) / 64;
    const int gy_cap = 148 * 8 / gx > 1 ? 148 * 8 / gx : 1;
    if (gy > gy_cap) gy = gy_cap;
    // B's slicer beside A's on the side stream (both CUDA-core kernels, each short of warps
    // to hide its latency alone), when there is one.
    kb<<<dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy)), dim3(32, 8), smem, side ? side : s>>>(
        bs, np, kp, b, rsb, csb, k, n, clo, pw, shmax, f);
}

// True when the tensor-core columns ran.
template <int NM>
static bool fm_launch_crt(const uint8_t* res, int chunks, int m, int n, const int* rlo,
                          const int* clo, const int* rspan, const int* cspan, const uint8_t* flags,
                          const FxEpi& e, const FmParams& f, int grid, int sm_count, int* status,
                          uint64_t budget_ns, cudaStream_t s) {
    const size_t total = static_cast<size_t>(m) * n;
    CUtensorMap tmY;
    // The tensor-core columns: one chunk, no non-finite terms, planes TMA can address.
    if (chunks == 1 && !flags && total % 16 == 0 && total < (size_t{1} << 31) &&
        make_tmap_u8(&tmY, res, total, NM, total, 128, 32)) {
        auto kern = fm_crt_tc_kernel<NM>;
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FMT_SMEM);
        const size_t nblk = (total + 127) / 128;
        const size_t cap = static_cast<size_t>(sm_count);
        kern<<<static_cast<int>(nblk < cap ? nblk : cap), FMT_THREADS, FMT_SMEM, s>>>(
            tmY, total, n, rlo, clo, rspan, cspan, e, f, status, budget_ns);
        return true;
    }
    if (chunks == 1 && (n & 3) == 0) {
        const size_t quads = static_cast<size_t>(m) * n / 4;
        const int g4 = static_cast<int>((quads + 255) / 256 < 148 * 16 ? (quads + 255) / 256 : 148 * 16);
        fm_crt4_kernel<NM><<<g4, 256, 0, s>>>(res, m, n, rlo, clo, rspan, cspan, flags, e, f);
    } else {
        fm_crt_kernel<NM><<<grid, 256, 0, s>>>(res, chunks, m, n, rlo, clo, rspan, cspan, flags, e, f);
    }
    return false;
}

// ------------------------------------------------------------ direct route

// The reference's register, Complete<L, MIN_EXP>: L low limbs and an extension word,
// here as L + 1 words of one two's complement integer (f64: 68 words, in local memory).
template <int NW>
__device__ void reg_add_scaled(uint64_t* r, int min_exp, u128 mag, int exp, bool negative) {
    if (mag == 0) return;
    const int sh = exp - min_exp;
    if (sh < 0) return;
    const int at = sh >> 6, bit = sh & 63;
    if (at >= NW - 1) return;
    uint64_t parts[3];
    if (bit == 0) {
        parts[0] = static_cast<uint64_t>(mag);
        parts[1] = static_cast<uint64_t>(mag >> 64);
        parts[2] = 0;
    } else {
        parts[0] = static_cast<uint64_t>(mag << bit);
        parts[1] = static_cast<uint64_t>(mag >> (64 - bit));
        parts[2] = static_cast<uint64_t>(mag >> (128 - bit));
    }
    if (!negative) {
        uint64_t c = 0;
        for (int i = at, q = 0; i < NW && (q < 3 || c); ++i, ++q) {
            const uint64_t add = q < 3 ? parts[q] : 0;
            const uint64_t s = r[i] + add;
            const uint64_t c1 = s < r[i];
            const uint64_t s2 = s + c;
            const uint64_t c2 = s2 < s;
            r[i] = s2;
            c = c1 | c2;
        }
    } else {
        uint64_t bw = 0;
        for (int i = at, q = 0; i < NW && (q < 3 || bw); ++i, ++q) {
            const uint64_t sub = q < 3 ? parts[q] : 0;
            const uint64_t d = r[i] - sub;
            const uint64_t b1 = r[i] < sub;
            const uint64_t d2 = d - bw;
            const uint64_t b2 = d < bw;
            r[i] = d2;
            bw = b1 | b2;
        }
    }
}

template <int NW>
__global__ void fx_direct_kernel(const uint8_t* __restrict__ a, int64_t rsa, int64_t csa,
                                 const uint8_t* __restrict__ b, int64_t rsb, int64_t csb, int m,
                                 int k, int n, FxEpi e) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    for (int i = blockIdx.y; i < m; i += gridDim.y) {
    uint64_t r[NW];
    for (int w = 0; w < NW; ++w) r[w] = 0;
    int fl = 0;
    for (int p = 0; p < k; ++p) {
        const FDec x = fdecode(a, static_cast<int64_t>(i) * rsa + static_cast<int64_t>(p) * csa, e.e64);
        const FDec y = fdecode(b, static_cast<int64_t>(p) * rsb + static_cast<int64_t>(j) * csb, e.e64);
        const int tf = term_flags(x, y);
        if (tf) fl |= tf;
        else reg_add_scaled<NW>(r, e.min_exp_e, static_cast<u128>(x.mant) * y.mant, x.exp + y.exp,
                                x.sign != y.sign);
    }
    // Linear::finish in the register itself: scale by alpha (exact: the register
    // spans the whole terminal expression), then add beta * Complete::of(C).
    bool zero_out;
    if (scale_flags(fl, zero_out, e.alpha)) {
        const bool nr = (r[NW - 1] >> 63) != 0;
        if (nr) words_negate(r);
        const uint64_t uf = e.alpha < 0 ? 0ull - static_cast<uint64_t>(e.alpha)
                                        : static_cast<uint64_t>(e.alpha);
        uint64_t carry = 0;
        for (int w = 0; w < NW; ++w) {
            const u128 pr = static_cast<u128>(r[w]) * uf + carry;
            r[w] = static_cast<uint64_t>(pr);
            carry = static_cast<uint64_t>(pr >> 64);
        }
        if (nr != (e.alpha < 0)) words_negate(r);
    }
    if (zero_out)
        for (int w = 0; w < NW; ++w) r[w] = 0;
    const int64_t off = static_cast<int64_t>(i) * e.rsc + static_cast<int64_t>(j) * e.csc;
    if (e.beta != 0) {
        const FDec d = fdecode(static_cast<const uint8_t*>(e.c), off, e.out64);
        int pf = 0;
        uint64_t q[NW];
        for (int w = 0; w < NW; ++w) q[w] = 0;
        if (d.kind == 2) pf = 1;
        else if (d.kind == 1) pf = d.sign ? 4 : 2;
        else reg_add_scaled<NW>(q, e.min_exp_e, d.mant, d.exp, d.sign != 0);
        bool zq;
        if (scale_flags(pf, zq, e.beta)) {
            const bool nq = (q[NW - 1] >> 63) != 0;
            if (nq) words_negate(q);
            const uint64_t uf = e.beta < 0 ? 0ull - static_cast<uint64_t>(e.beta)
                                           : static_cast<uint64_t>(e.beta);
            uint64_t carry = 0;
            for (int w = 0; w < NW; ++w) {
                const u128 pr = static_cast<u128>(q[w]) * uf + carry;
                q[w] = static_cast<uint64_t>(pr);
                carry = static_cast<uint64_t>(pr >> 64);
            }
            if (nq != (e.beta < 0)) words_negate(q);
        }
        if (fl || pf) {
            fl |= pf;
        } else {
            uint64_t c = 0;
            for (int w = 0; w < NW; ++w) {
                const uint64_t s1 = r[w] + q[w];
                const uint64_t c1 = s1 < r[w];
                const uint64_t s2 = s1 + c;
                const uint64_t c2 = s2 < s1;
                r[w] = s2;
                c = c1 | c2;
            }
        }
    }
    if (fl) {
        const bool nan = (fl & 1) || ((fl & 6) == 6);
        store_float(e.c, e.out64, off, nan ? nan_bits(e.out64) : inf_bits(e.out64, (fl & 4) != 0));
        continue;
    }
    store_float(e.c, e.out64, off, encode_words<NW>(r, e.min_exp_e, e.out64, e.mode, e.min_exp_e));
    }
}

// ------------------------------------------------------------ driver

static inline size_t rup(size_t x, size_t a) { return (x + a - 1) / a * a; }
constexpr int FX_MAX_DIGITS = 16;

int run_float_gemm(uor_b200_ctx* ctx, bool e64, bool o64, const uint8_t* a, ptrdiff_t rsa,
                   ptrdiff_t csa, const uint8_t* b, ptrdiff_t rsb, ptrdiff_t csb, void* c,
                   ptrdiff_t rsc, ptrdiff_t csc, size_t m, size_t k, size_t n, int64_t alpha,
                   int64_t beta, int mode, uor_b200_route* route, uint32_t route_flags) {
    const bool digits_only = (route_flags & UOR_B200_DIGIT_SLICES) != 0;
    const bool force_modular = !digits_only && (route_flags & UOR_B200_MODULAR) != 0;
    cudaStream_t s = ctx->stream;
    if (route) *route = uor_b200_route{};
    if (m == 0 || n == 0) return UOR_B200_OK;
    if (m > (size_t)INT_MAX / 4 || n > (size_t)INT_MAX / 4 || k > (size_t)INT_MAX / 4)
        return UOR_B200_UNSUPPORTED;
    FxEpi e{};
    e.alpha = alpha;
    e.beta = beta;
    e.mode = mode;
    e.e64 = e64;
    e.out64 = o64;
    e.min_exp_e = e64 ? -2148 : -298;
    e.limbs_e = e64 ? 67 : 10;
    e.c = c;
    e.rsc = rsc;
    e.csc = csc;
    if (route) {
        route->kernel = UOR_B200_KERNEL_FLOAT_EXACT;
        route->tile_m = KS_BM;
        route->tile_n = KS_BN;
        route->tile_k = KS_BK;
    }

    // ---- analysis: per-row / per-column exponent spans and non-finite markers
    int st = UOR_B200_OK;
    const size_t an_bytes = 2 * rup(m * 4, 256) + 5 * rup(n * 4, 256) + rup(m, 256) + rup(n, 256) + 256;
    uint8_t* an = static_cast<uint8_t*>(ctx_buffer(ctx, SLOT_AUX, an_bytes, &st));
    if (!an) return st;
    int* rlo = reinterpret_cast<int*>(an);
    int* rspan = reinterpret_cast<int*>(an + rup(m * 4, 256));
    int* clo = reinterpret_cast<int*>(an + 2 * rup(m * 4, 256));
    int* cspan = reinterpret_cast<int*>(an + 2 * rup(m * 4, 256) + rup(n * 4, 256));
    uint8_t* rnf = an + 2 * rup(m * 4, 256) + 2 * rup(n * 4, 256);
    uint8_t* cnf = rnf + rup(m, 256);
    int* gmax = reinterpret_cast<int*>(cnf + rup(n, 256));
    if (cudaMemsetAsync(gmax, 0, 32, s) != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    if (k > 0) {
        fx_rows_kernel<<<(int)((m * 32 + 255) / 256), 256, 0, s>>>(a, rsa, csa, (int)m, (int)k, e64,
                                                                   rlo, rspan, rnf, gmax);
        const bool cvec = !e64 && csb == 1 && (n & 3) == 0 &&
                          ((reinterpret_cast<uintptr_t>(b) | static_cast<uintptr_t>(rsb * 4)) & 15) == 0;
        if (cvec) {
            int* cl = reinterpret_cast<int*>(gmax + 64);
            int* ch = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(cl) + rup(n * 4, 256));
            int* cf = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(ch) + rup(n * 4, 256));
            if (cudaMemsetAsync(cl, 0x7F, n * 4, s) != cudaSuccess ||
                cudaMemsetAsync(ch, 0x80, n * 4, s) != cudaSuccess ||
                cudaMemsetAsync(cf, 0, n * 4, s) != cudaSuccess)
                return UOR_B200_DEVICE_ERROR;
            const int gx = (int)((n + 127) / 128);
            int gy = 148 * 8 / gx;
            const int gy_max = (int)((k + 63) / 64);
            gy = gy < 1 ? 1 : gy > gy_max ? gy_max : gy;
            const int rows = (int)(((k + gy - 1) / gy + 7) / 8 * 8);
            gy = (int)((k + rows - 1) / rows);
            fx_cols4_kernel<<<dim3((unsigned)gx, (unsigned)gy), dim3(32, 8), 0, s>>>(b, rsb, (int)k, (int)n,
                                                                                     rows, cl, ch, cf);
            fx_cols_finish<<<(int)((n + 255) / 256), 256, 0, s>>>((int)n, cl, ch, cf, clo, cspan, cnf, gmax);
        } else {
            fx_cols_kernel<<<(int)((n + 31) / 32), dim3(32, 32), 0, s>>>(b, rsb, csb, (int)k, (int)n,
                                                                          e64, clo, cspan, cnf, gmax);
        }
    } else {
        cudaMemsetAsync(rlo, 0, m * 4, s);
        cudaMemsetAsync(clo, 0, n * 4, s);
        cudaMemsetAsync(rspan, 0, m * 4, s);
        cudaMemsetAsync(cspan, 0, n * 4, s);
        cudaMemsetAsync(rnf, 0, m, s);
        cudaMemsetAsync(cnf, 0, n, s);
    }
    int g[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (cudaMemcpyAsync(g, gmax, 32, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return UOR_B200_DEVICE_ERROR;
    const int La = g[0] ? (g[0] + 2 + 7) / 8 : 0;
    const int Lb = g[1] ? (g[1] + 2 + 7) / 8 : 0;
    const bool any_nf = g[2] != 0;

    // ---- modular route: nm int8 GEMMs and the CRT
    FmParams fm;
    const bool mod_ok = !digits_only && k > 0 && g[0] > 0 && g[1] > 0 && fm_plan_spans(g[0], g[1], k, fm) &&
                        (size_t)((g[0] > g[1] ? g[0] : g[1]) + 1) * 2 * ((fm.nm + 3) / 4 * 4) * 4 *
                                (e64 ? 2 : 1) <= FM_TABLE_MAX;
    auto run_modular = [&]() -> int {
        const int nm = fm.nm;
        KSParams q{};
        q.num_groups = nm;
        for (int gg = 0; gg < nm; ++gg) {
            q.pair_begin[gg] = gg;
            q.pair_a[gg] = q.pair_b[gg] = static_cast<uint8_t>(gg);
            q.pair_sign[gg] = 3;  // balanced residues are signed on both sides
            q.res_mod[gg] = fm.p[gg];
            q.res_magic[gg] = fm.magic32[gg];
            q.res_off[gg] = static_cast<uint32_t>(fm.p[gg] * ((0x80000000ull + fm.p[gg] - 1) / fm.p[gg]));
        }
        q.pair_begin[nm] = nm;
        const int num_kb = (int)((k + KS_BK - 1) / KS_BK);
        // |residue product| <= 2^14: 1023 blocks keep |acc| < 2^31 - 2^21 (the epilogue's
        // 32-bit reduction relies on it)
        const int64_t lane = (int64_t)INT_MAX / 16384 / KS_BK;
        q.kb_per_chunk = (int)(lane < num_kb ? lane : num_kb);
        q.num_chunks = (num_kb + q.kb_per_chunk - 1) / q.kb_per_chunk;
        q.num_kb = num_kb;
        q.m = (int)m;
        q.n = (int)n;
        q.mp = (int)ks_rows_pad(m);
        q.np = (int)rup(n, KS_BN);
        ks_balance_chunks(q, ctx->sm_count);
        q.status = ctx->d_status;
        q.budget_ns = ctx->budget_ns;
        const size_t kp = rup(k, 16);
        const int shmax = (g[0] > g[1] ? g[0] : g[1]) + 1;
        const int nmp = (nm + 3) / 4 * 4;
        const int W = e64 ? 2 : 1;  // table words per (shift, modulus): significand bytes / 4
        if (q.num_chunks == 1)  // the epilogue stores y_g = r_g (M / p_g)^-1 mod p_g
            for (int gg = 0; gg < nm; ++gg) q.res_inv[gg] = fm.inv[gg];
        const size_t a_bytes = rup((size_t)nm * q.mp * kp, 256);
        const size_t b_bytes = rup((size_t)nm * q.np * kp, 256);
        const size_t res_bytes = rup((size_t)q.num_chunks * nm * m * n, 256);
        const size_t flag_bytes = any_nf ? rup(m * n, 256) : 0;
        const size_t pw_bytes = rup((size_t)nmp * shmax * 2 * W * 4, 256);
        int st2 = UOR_B200_OK;
        uint8_t* ws = static_cast<uint8_t*>(ctx_buffer(
            ctx, SLOT_WS, a_bytes + b_bytes + res_bytes + flag_bytes + pw_bytes + 256, &st2));
        if (!ws) return st2;
        int8_t* as = reinterpret_cast<int8_t*>(ws);
        int8_t* bs = reinterpret_cast<int8_t*>(ws + a_bytes);
        uint8_t* res = ws + a_bytes + b_bytes;
        uint8_t* flags = any_nf ? res + res_bytes : nullptr;
        uint32_t* pw = reinterpret_cast<uint32_t*>(res + res_bytes + flag_bytes);
        {
            // column (w, g / 4), row 2 sh + s, word g % 4: bytes i of (-1)^s 2^(sh + 8 (4 w + i)) mod p_g
            std::vector<uint32_t> tab((size_t)shmax * 2 * W * nmp, 0);
            for (int gg = 0; gg < nm; ++gg) {
                const uint32_t pg = fm.p[gg];
                uint32_t v = 1 % pg;  // 2^sh mod p
                for (int sh = 0; sh < shmax; ++sh) {
                    uint32_t c = v;
                    for (int bi = 0; bi < 4 * W; ++bi) {
                        const uint32_t cn = (pg - c) % pg;
                        const size_t col = (size_t)(bi / 4) * (nmp / 4) + gg / 4;  // 16-byte column
                        tab[((col * 2 * shmax + 2 * sh) * 4) + gg % 4] |= c << (8 * (bi % 4));
                        tab[((col * 2 * shmax + 2 * sh + 1) * 4) + gg % 4] |= cn << (8 * (bi % 4));
                        c = c * 256 % pg;
                    }
                    v = v * 2 % pg;
                }
            }
            if (cudaMemcpyAsync(pw, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice, s) != cudaSuccess)
                return UOR_B200_DEVICE_ERROR;
        }
        if (any_nf) {
            dim3 grid((unsigned)((n + 127) / 128), (unsigned)(m < 65535 ? m : 65535));
            fx_flags_kernel<<<grid, 128, 0, s>>>(a, rsa, csa, b, rsb, csb, e64, (int)m, (int)k, (int)n,
                                                  rnf, cnf, flags);
        }
        cudaStream_t side = ctx_fork(ctx);
        switch (nm) {
#define FM_SLICES(N)                                                                            \
    case N:                                                                                     \
        fm_launch_slices<N>(as, q.mp, bs, q.np, (int)kp, a, rsa, csa, b, rsb, csb, e64, (int)m, \
                            (int)k, (int)n, rlo, clo, pw, shmax, fm, s, side);                  \
        break;
            FM_EVEN_COUNTS(FM_SLICES)
#undef FM_SLICES
        default: return UOR_B200_UNSUPPORTED;
        }
        if (side && !ctx_join(ctx)) return UOR_B200_DEVICE_ERROR;
        if (cudaGetLastError() != cudaSuccess) return UOR_B200_DEVICE_ERROR;
        q.residue = res;
        q.partial = nullptr;
        if ((st2 = ks_run(as, nm, bs, nm, k, kp, q, ctx->sm_count, s, route ? &route->ctas : nullptr)) !=
            UOR_B200_OK)
            return st2;
        const size_t total = m * n;
        const int rgrid = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
        bool crt_tc = false;
        switch (nm) {
#define FM_CRT(N)                                                                               \
    case N:                                                                                     \
        crt_tc = fm_launch_crt<N>(res, q.num_chunks, (int)m, (int)n, rlo, clo, rspan, cspan, flags, e, fm, \
                         rgrid, ctx->sm_count, ctx->d_status, ctx->budget_ns, s);               \
        break;
            FM_EVEN_COUNTS(FM_CRT)
#undef FM_CRT
        default: return UOR_B200_UNSUPPORTED;
        }
        if (route) {
            route->moduli = (uint32_t)nm;
            route->pairs = (uint32_t)nm;
            route->a_layout = route->b_layout = (uint32_t)nm;
            route->k_chunks = (uint32_t)q.num_chunks;
            route->tile_m = (uint32_t)(m > 128 ? 256 : KS_BM);
            route->crt = crt_tc ? 1u : 0u;
        }
        return cuda_status(cudaGetLastError());
    };

    if (La > FX_MAX_DIGITS || Lb > FX_MAX_DIGITS) {
        if (mod_ok) return run_modular();
        // Direct route: the reference's register per cell on CUDA cores.
        if (route) route->tile_m = route->tile_n = route->tile_k = 0;
        dim3 grid((unsigned)((n + 127) / 128), (unsigned)(m < 65535 ? m : 65535));
        if (e64) fx_direct_kernel<68><<<grid, 128, 0, s>>>(a, rsa, csa, b, rsb, csb, (int)m, (int)k, (int)n, e);
        else fx_direct_kernel<11><<<grid, 128, 0, s>>>(a, rsa, csa, b, rsb, csb, (int)m, (int)k, (int)n, e);
        return cuda_status(cudaGetLastError());
    }

    // ---- lazy digits: how many low diagonals a typical cell cannot feel
    const int G = La && Lb ? La + Lb - 1 : 0;
    auto pairs_on = [&](int d) {
        int c = 0;
        for (int sa = 0; sa < La; ++sa)
            if (d - sa >= 0 && d - sa < Lb) ++c;
        return c;
    };
    int D = 0;
    uint64_t ebound = 0;
    if (!e64 && !o64 && beta == 0 && alpha != 0 && !any_nf && G >= 8 && k > 0 &&
        m * n < (size_t{1} << 32)) {
        // A cell's integer is near 2^(span_i + span_j) unless its terms cancel; take the
        // smallest spans, minus a margin, and skip the diagonals whose whole sum stays 16
        // bits below that cell's last significand bit.
        const int est = (SPAN_CAP - g[3]) + (SPAN_CAP - g[4]) - 8;
        const int lk = 64 - __builtin_clzll(static_cast<unsigned long long>(k));
        const int nmax = La < Lb ? La : Lb;
        const int ln = 32 - __builtin_clz(static_cast<unsigned>(nmax));
        const int t = est - 24 - 16 - 14 - lk - ln;
        D = t >= 0 ? t / 8 + 1 : 0;
        if (D > G - 1) D = G - 1;
        if (D < 3) D = 0;
        if (D) {
            // |R| / 256^D <= k 2^14 (n_{D-1} / 256 + n_{D-2} / 256^2 + nmax / (256^2 255)),
            // each term rounded up.
            const uint64_t kk = k;
            ebound = kk * 64 * pairs_on(D - 1) + (kk * pairs_on(D - 2) + 3) / 4 +
                     (kk * nmax + 1019) / 1020 + 1;
        }
    }
    if (mod_ok) {
        // The modular route when it runs fewer GEMMs than the digit pairs would.
        int digit_pairs = 0;
        for (int d = D; d < G; ++d) digit_pairs += pairs_on(d);
        if (force_modular || fm.nm < digit_pairs) return run_modular();
    }

    // ---- digit slices and the slice-pair product of diagonals d >= d_lo
    KSParams p{};
    int ngroups = 0, npairs = 0;
    auto build_groups = [&](int d_lo) {
        npairs = 0;
        ngroups = 0;
        int worst = 1;
        for (int d = d_lo; d < G; ++d) {
            p.pair_begin[ngroups] = npairs;
            int cnt = 0;
            for (int sa = 0; sa < La; ++sa) {
                const int sb = d - sa;
                if (sb < 0 || sb >= Lb) continue;
                p.pair_a[npairs] = (uint8_t)sa;
                p.pair_b[npairs] = (uint8_t)sb;
                p.pair_sign[npairs] = 3;  // balanced digits are signed on both sides
                ++npairs;
                ++cnt;
            }
            ++ngroups;
            if (cnt > worst) worst = cnt;
        }
        p.pair_begin[ngroups] = npairs;
        p.num_groups = ngroups;
        const int num_kb = (int)((k + KS_BK - 1) / KS_BK);
        // |digit product| <= 2^14; a diagonal of `worst` pairs must stay inside s32.
        const int64_t lane = (int64_t)INT_MAX / ((int64_t)worst * 16384) / KS_BK;
        p.kb_per_chunk = (int)(lane < num_kb ? lane : num_kb);
        if (p.kb_per_chunk < 1) p.kb_per_chunk = 1;
        p.num_chunks = num_kb ? (num_kb + p.kb_per_chunk - 1) / p.kb_per_chunk : 0;
        p.num_kb = num_kb;
    };
    build_groups(0);  // sizes the partial planes for every diagonal
    const int all_chunks = p.num_chunks, all_groups = ngroups;
    p.m = (int)m;
    p.n = (int)n;
    p.mp = (int)ks_rows_pad(m);
    p.np = (int)rup(n, KS_BN);
    p.status = ctx->d_status;
    p.budget_ns = ctx->budget_ns;
    const bool run_mma = npairs > 0 && p.num_kb > 0;

    const size_t total = m * n;
    const uint32_t limit = (uint32_t)(total < 4096 ? total : (total / 256 > 4096 ? total / 256 : 4096));
    const size_t kp = rup(k ? k : 1, 16);
    const size_t a_bytes = run_mma ? rup((size_t)La * p.mp * kp, 256) : 0;
    const size_t b_bytes = run_mma ? rup((size_t)Lb * p.np * kp, 256) : 0;
    const size_t part_bytes = run_mma ? rup((size_t)all_chunks * all_groups * m * n * 4, 256) : 0;
    const size_t flag_bytes = any_nf ? rup(m * n, 256) : 0;
    const size_t list_bytes = D ? rup((size_t)limit * 4, 256) + 256 : 0;
    uint8_t* ws = static_cast<uint8_t*>(ctx_buffer(
        ctx, SLOT_WS, a_bytes + b_bytes + part_bytes + flag_bytes + list_bytes + 256, &st));
    if (!ws) return st;
    int8_t* as = reinterpret_cast<int8_t*>(ws);
    int8_t* bs = reinterpret_cast<int8_t*>(ws + a_bytes);
    int32_t* part = reinterpret_cast<int32_t*>(ws + a_bytes + b_bytes);
    uint8_t* flags = any_nf ? ws + a_bytes + b_bytes + part_bytes : nullptr;
    uint32_t* count = reinterpret_cast<uint32_t*>(ws + a_bytes + b_bytes + part_bytes + flag_bytes);
    uint32_t* list = count + 64;
    p.partial = part;

    if (any_nf) {
        dim3 grid((unsigned)((n + 127) / 128), (unsigned)(m < 65535 ? m : 65535));
        fx_flags_kernel<<<grid, 128, 0, s>>>(a, rsa, csa, b, rsb, csb, e64, (int)m, (int)k, (int)n,
                                              rnf, cnf, flags);
    }
    const int rgrid = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
    auto full_reduce = [&]() {
        const int rchunks = run_mma ? p.num_chunks : 0, rgroups = run_mma ? ngroups : 0;
        // Groups are at most 2 * FX_MAX_DIGITS - 1 = 31.
        if (rgroups <= 8)
            fx_reduce_kernel<8><<<rgrid, 256, 0, s>>>(part, rchunks, rgroups, (int)m, (int)n, rlo, clo, flags, e);
        else if (rgroups <= 16)
            fx_reduce_kernel<16><<<rgrid, 256, 0, s>>>(part, rchunks, rgroups, (int)m, (int)n, rlo, clo, flags, e);
        else if (rgroups <= 24)
            fx_reduce_kernel<24><<<rgrid, 256, 0, s>>>(part, rchunks, rgroups, (int)m, (int)n, rlo, clo, flags, e);
        else
            fx_reduce_kernel<32><<<rgrid, 256, 0, s>>>(part, rchunks, rgroups, (int)m, (int)n, rlo, clo, flags, e);
        return cuda_status(cudaGetLastError());
    };
    if (!run_mma) return full_reduce();

    auto bias = [](int L) {  // sum_{s<L} 128 256^s
        u128 c = 0;
        for (int q = 0; q < L; ++q) c |= static_cast<u128>(0x80) << (8 * q);
        return c;
    };
    const int64_t aquads = (int64_t)p.mp * (kp / 4);
    const int sgrid = (int)(aquads / 256 + 1 < 148 * 16 ? aquads / 256 + 1 : 148 * 16);
    fx_slice_a_kernel<<<sgrid, 256, 0, s>>>(as, La, p.mp, (int)kp, a, rsa, csa, e64, (int)m, (int)k,
                                            rlo, bias(La));
    dim3 g2((unsigned)(p.np / 32), (unsigned)((kp + 63) / 64 < 65535 ? (kp + 63) / 64 : 65535));
    fx_slice_b_kernel<<<g2, dim3(32, 8), 0, s>>>(bs, Lb, p.np, (int)kp, b, rsb, csb, e64, (int)k,
                                                 (int)n, clo, bias(Lb));
    if (route) {
        route->a_layout = (uint32_t)La;  // digits per A element
        route->b_layout = (uint32_t)Lb;
        route->tile_m = (uint32_t)(m > 128 ? 256 : KS_BM);
    }
    auto run_pairs = [&](int d_lo) {
        build_groups(d_lo);
        if (route) {
            route->k_chunks = (uint32_t)p.num_chunks;
            route->pairs = (uint32_t)npairs;
        }
        return ks_run(as, La, bs, Lb, k, kp, p, ctx->sm_count, s, route ? &route->ctas : nullptr);
    };
    if (D == 0) {
        if ((st = run_pairs(0)) != UOR_B200_OK) return st;
        return full_reduce();
    }

    // Lazy: the top diagonals, the interval test per cell, exact recomputation of the rest.
    if ((st = run_pairs(D)) != UOR_B200_OK) return st;
    if (cudaMemsetAsync(count, 0, 4, s) != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    if (ngroups <= 8)
        fx_reduce_lazy_kernel<8><<<rgrid, 256, 0, s>>>(part, p.num_chunks, ngroups, (int)m, (int)n, rlo, clo, rspan, cspan, D, ebound, e, list, count, limit);
    else if (ngroups <= 16)
        fx_reduce_lazy_kernel<16><<<rgrid, 256, 0, s>>>(part, p.num_chunks, ngroups, (int)m, (int)n, rlo, clo, rspan, cspan, D, ebound, e, list, count, limit);
    else
        fx_reduce_lazy_kernel<24><<<rgrid, 256, 0, s>>>(part, p.num_chunks, ngroups, (int)m, (int)n, rlo, clo, rspan, cspan, D, ebound, e, list, count, limit);
    uint32_t unsure = 0;
    if (cudaMemcpyAsync(&unsure, count, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return UOR_B200_DEVICE_ERROR;
    if (route) route->fixups = unsure;
    if (unsure == 0) return UOR_B200_OK;
    if (unsure <= limit) {
        const uint32_t warps = unsure < 148u * 64u ? unsure : 148u * 64u;
        fx_fix_kernel<<<(warps + 7) / 8, 256, 0, s>>>(list, count, limit, as, La, p.mp, bs, Lb, p.np,
                                                      (int)kp, (int)n, rlo, clo, e);
        return cuda_status(cudaGetLastError());
    }
    // Too many cells cancel: every diagonal on the tensor cores after all.
    if ((st = run_pairs(0)) != UOR_B200_OK) return st;
    return full_reduce();
}

}  // namespace uor
