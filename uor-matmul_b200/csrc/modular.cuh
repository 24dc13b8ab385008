// modular.cuh -- exact integer products through residues modulo small coprime moduli,
// the integer core of Ozaki scheme II (Ozaki, Uchino and Imamura, "Ozaki Scheme II: A
// GEMM-oriented emulation of floating-point matrix multiplication using an integer
// modular technique", 2025), shared by the exact float and the wide-integer paths.
//
// Integer operands are reduced modulo nm pairwise coprime moduli p_g <= 256 into balanced
// residues, which are int8; one int8 GEMM per modulus on the tensor cores gives S mod p_g
// exactly (the slice-pair kernel reduces its s32 accumulator in the epilogue, and with one
// reduction chunk stores y_g = r_g (M / p_g)^-1 mod p_g directly); the Chinese remainder
// theorem then rebuilds each cell's exact integer S. M = prod p_g is chosen above
// 2 (1 + 2^-10) times a bound on |S|, so S is the representative of X = sum_g y_g M / p_g
// nearest to zero: S = X - t M with t the integer nearest X / M = sum_g y_g / p_g. X / M
// lies within 1/2 - 2^-11 of t, and the 32-bit fixed-point sum sum_g y_g ceil(2^32 / p_g)
// overshoots X / M 2^32 by less than 40 * 255 (2^-18.6 after scaling), so rounding it
// finds t. X is summed in base-256 columns, X_b = sum_g y_g byte_b(M / p_g), four moduli
// per dp4a, and carried into signed 32-bit limbs.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace uor {

constexpr int FM_MAX = 40;  // moduli (the 40 moduli's product is 291 bits)

struct FmParams {
    int nm;                           // moduli (even)
    uint32_t p[FM_MAX];               // 32-bit words: kernels read them as instruction operands
    uint32_t inv[FM_MAX];             // (M / p_g)^-1 mod p_g
    uint32_t magic32[FM_MAX];         // ceil(2^32 / p_g)
    uint32_t mg[FM_MAX / 4][4];       // [a][b]: byte b of ceil(2^32 / p_g) for g = 4a .. 4a + 3
    uint32_t half[FM_MAX];            // (p_g - 1) / 2, and 127 for 256
    uint32_t pneg[FM_MAX];            // 2^32 - p_g
    uint32_t hneg[FM_MAX];            // 2^32 - half_g
    uint32_t md[FM_MAX / 4][FM_MAX];  // [a][b]: byte b of M / p_g for g = 4a .. 4a + 3
    uint32_t mm[FM_MAX / 4 + 1];      // 32-bit limbs of M (M < 2^(8 nm))
    int32_t nmb[FM_MAX];              // -byte b of M
};

// The smallest even prefix of the moduli (256, 255, 253, 251, 247 and primes) whose
// product M exceeds 2 (1 + 2^-10) bound, and the CRT constants; bound is a little-endian
// array of 32-bit limbs. False when 40 moduli are not enough.
bool fm_plan_bound(const uint32_t* bound, int limbs, FmParams& f);
// bound = k (2^sa - 1)(2^sb - 1): products of integers below 2^sa and 2^sb in magnitude.
bool fm_plan_spans(int span_a, int span_b, size_t k, FmParams& f);
// bound = k 2^(2 bits - 2): products of two's-complement integers of `bits` bits.
bool fm_plan_ints(int bits, size_t k, FmParams& f);

// x mod p for x < 2^24: floor(x ceil(2^32 / p) / 2^32) is exact there (the error term
// x (ceil(2^32/p) - 2^32/p) / 2^32 < 2^-8 never reaches the next multiple).
__device__ __forceinline__ uint32_t fm_mod24(uint32_t x, uint32_t p, uint32_t magic32) {
    return x - __umulhi(x, magic32) * p;
}

// The balanced residue of v < 2^24 - half (v - q p, q = floor((v + half) / p), half =
// (p - 1) / 2 and 127 for 256) in its low byte: it lies in [-(p-1)/2, (p-1)/2] for odd p
// and in [-127, 128] for 256, whose byte 128 is the int8 -128, the same residue modulo 256.
// It takes vh = v + half (the slicers' dp4a adds half through its accumulator), so
// q = floor(vh / p) is one high multiply (fm_mod24's bound), and vh - q p - half is one
// multiply-add and one add with the negated constants: single-word operations only.
__device__ __forceinline__ uint32_t fm_balanced_vh(uint32_t vh, uint32_t pneg, uint32_t magic32,
                                                   uint32_t hneg) {
    return vh + __umulhi(vh, magic32) * pneg + hneg;
}

// word with its byte c replaced by the low byte of b (c = 0 .. 3, a compile-time constant).
__device__ __forceinline__ uint32_t fm_put_byte(uint32_t word, uint32_t b, int c) {
    // __byte_perm selectors: 0-3 pick word's bytes, 4 picks b's low byte
    const uint32_t sel = c == 0 ? 0x3214u : c == 1 ? 0x3240u : c == 2 ? 0x3410u : 0x4210u;
    return __byte_perm(word, b, sel);
}

// y_g of one cell from the residue planes res[chunk][g][total] (idx the cell): the
// epilogue's y_g with one chunk, else rebuilt from the chunks' residues.
template <int NM>
__device__ __forceinline__ void fm_load_y(const uint8_t* __restrict__ res, int chunks, size_t total,
                                          size_t idx, const FmParams& f, uint32_t (&y)[NM]) {
    if (chunks == 1) {
#pragma unroll
        for (int g = 0; g < NM; ++g) y[g] = __ldg(res + g * total + idx);
        return;
    }
#pragma unroll
    for (int g = 0; g < NM; ++g) y[g] = 0;
    for (int q = 0; q < chunks; ++q) {
#pragma unroll
        for (int g = 0; g < NM; ++g) y[g] += __ldg(res + (static_cast<size_t>(q) * NM + g) * total + idx);
    }
#pragma unroll
    for (int g = 0; g < NM; ++g)
        y[g] = fm_mod24(fm_mod24(y[g], f.p[g], f.magic32[g]) * f.inv[g], f.p[g], f.magic32[g]);
}

// 32-bit limbs of |S| < M / 2 < 2^(8 NM - 1), one spare for the sign.
template <int NM>
struct FmLimbs {
    static constexpr int value = (NM + 1 + 3) / 4;
};

// Base-256 columns X_b of X: from three moduli on, M / p_g is a product of NM - 1 moduli of
// which at most one is 256, so it stays below 256^(NM - 1) and its byte NM - 1 is zero.
template <int NM>
struct FmColumns {
    static constexpr int value = NM >= 3 ? NM - 1 : NM;
};

// t, the integer nearest X / M, from the four byte columns F_b of the fixed-point sum
// sum_g y_g ceil(2^32 / p_g) (each F_b below NM 255^2 < 2^22, so F_0 + 2^8 F_1 and
// F_2 + 2^8 F_3 stay in 32 bits).
__device__ __forceinline__ uint32_t fm_crt_t(const uint32_t (&F)[4]) {
    const uint64_t fx = (static_cast<uint64_t>(F[2] + (F[3] << 8)) << 16) + (F[0] + (F[1] << 8)) +
                        0x80000000ull;  // + 1/2
    return static_cast<uint32_t>(fx >> 32);
}

// S = X - t M as two's complement 32-bit limbs, least significant first, from the columns
// col(b) = X_b (each below NM 255^2 < 2^22), four to a limb, minus t M limb by limb; returns
// the sign extension (0 or ~0) of the limbs above.
template <int NM, typename Col>
__device__ __forceinline__ uint32_t fm_crt_limbs(uint32_t t, const FmParams& f, Col col,
                                                 uint32_t (&limb)[FmLimbs<NM>::value]) {
    constexpr int NL = FmLimbs<NM>::value;
    constexpr int NB = FmColumns<NM>::value;
    int64_t carry = 0;
#pragma unroll
    for (int l = 0; l < NL; ++l) {
        uint32_t c[4];
#pragma unroll
        for (int bi = 0; bi < 4; ++bi) c[bi] = 4 * l + bi < NB ? col(4 * l + bi) : 0u;
        const uint64_t v = (static_cast<uint64_t>(c[2] + (c[3] << 8)) << 16) + (c[0] + (c[1] << 8));
        const uint32_t ml = l < FM_MAX / 4 + 1 ? f.mm[l] : 0u;
        const int64_t sv = static_cast<int64_t>(v) + carry - static_cast<int64_t>(static_cast<uint64_t>(t) * ml);
        limb[l] = static_cast<uint32_t>(sv);
        carry = sv >> 32;
    }
    return carry < 0 ? ~0u : 0u;
}

// The same limbs from the signed byte columns d_b = X_b - t M_b, mostly multiply-adds: t is
// below NM (X < NM M), so |d_b| < 2^22; e = d_4l + 2^8 d_4l+1 + carry and
// e' = d_4l+2 + 2^8 d_4l+3 stay inside 31 bits, and L = 2^16 e' + e (|L| < 2^47) is one
// widening multiply-add whose low word is the limb and whose high word is the next carry.
template <int NM, typename Col>
__device__ __forceinline__ uint32_t fm_crt_limbs_signed(uint32_t t, const FmParams& f, Col col,
                                                        uint32_t (&limb)[FmLimbs<NM>::value]) {
    constexpr int NL = FmLimbs<NM>::value;
    constexpr int NB = FmColumns<NM>::value;
    int32_t carry = 0;
#pragma unroll
    for (int l = 0; l < NL; ++l) {
        int32_t d[4];
#pragma unroll
        for (int bi = 0; bi < 4; ++bi) {
            const int b = 4 * l + bi;
            const int32_t x = b < NB ? static_cast<int32_t>(col(b)) : 0;
            d[bi] = b < FM_MAX ? x + static_cast<int32_t>(t) * f.nmb[b < FM_MAX ? b : 0] : x;
        }
        const int32_t e0 = d[0] + d[1] * 256 + carry;
        const int32_t e1 = d[2] + d[3] * 256;
        const int64_t L = static_cast<int64_t>(e1) * 65536 + e0;
        limb[l] = static_cast<uint32_t>(L);
        carry = static_cast<int32_t>(L >> 32);
    }
    return carry < 0 ? ~0u : 0u;
}

// S from the packed y words ya[a] (byte gi = y_{4a+gi}): the columns F_b and X_b by dp4a,
// four moduli per instruction.
template <int NM>
__device__ __forceinline__ uint32_t fm_crt_packed(const uint32_t (&ya)[(NM + 3) / 4], const FmParams& f,
                                                  uint32_t (&limb)[FmLimbs<NM>::value]) {
    constexpr int NA = (NM + 3) / 4;
    uint32_t F[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        F[b] = 0;
#pragma unroll
        for (int a = 0; a < NA; ++a) F[b] = __dp4a(ya[a], f.mg[a][b], F[b]);
    }
    return fm_crt_limbs<NM>(fm_crt_t(F), f, [&](int b) {
        uint32_t c = 0;
#pragma unroll
        for (int a = 0; a < NA; ++a) c = __dp4a(ya[a], f.md[a][b], c);
        return c;
    }, limb);
}

// The same from the unpacked y_g.
template <int NM>
__device__ __forceinline__ uint32_t fm_crt(const uint32_t (&y)[NM], const FmParams& f,
                                           uint32_t (&limb)[FmLimbs<NM>::value]) {
    constexpr int NA = (NM + 3) / 4;
    uint32_t ya[NA];
#pragma unroll
    for (int a = 0; a < NA; ++a) {
        ya[a] = 0;
#pragma unroll
        for (int gi = 0; gi < 4; ++gi)
            if (4 * a + gi < NM) ya[a] |= y[4 * a + gi] << (8 * gi);
    }
    return fm_crt_packed<NM>(ya, f, limb);
}

#define FM_EVEN_COUNTS(X) X(2) X(4) X(6) X(8) X(10) X(12) X(14) X(16) X(18) X(20) X(22) X(24) \
    X(26) X(28) X(30) X(32) X(34) X(36) X(38) X(40)

}  // namespace uor
