// int_epilogue.cuh -- the integer Linear epilogue and single encode, on device.
//
// Restates, per output cell:
//   Linear::finish (epilogue.rs:79-93): total = acc.saturating_mul(alpha)
//     [+ prior.saturating_mul(beta) when beta != 0, the i128 add wrapping as the
//     reference's release build does];
//   encode_i128_into (acc.rs:128-151): clamp to the output range, or reduce
//     modulo it under Wrapping.
#pragma once
#include <cstdint>

namespace uor {

typedef __int128 i128;
typedef unsigned __int128 u128;

enum OutKind : int { OUT_I8 = 0, OUT_I16 = 1, OUT_I32 = 2, OUT_I64 = 3, OUT_I128 = 4 };
enum Mode : int { MODE_NEAREST = 0, MODE_TOWARD_ZERO = 1, MODE_SATURATING = 2, MODE_WRAPPING = 3 };

__host__ __device__ __forceinline__ int out_bits(int kind) { return 8 << kind; }
__host__ __device__ __forceinline__ int out_bytes(int kind) { return 1 << kind; }

__device__ __forceinline__ i128 i128_max() { return (i128)(((u128)1 << 127) - 1); }
__device__ __forceinline__ i128 i128_min() { return -i128_max() - 1; }

// i128::saturating_mul by an i64 scalar.
__device__ __forceinline__ i128 sat_mul(i128 a, int64_t f) {
    if (a == 0 || f == 0) return 0;
    const bool neg = (a < 0) != (f < 0);
    const u128 ua = a < 0 ? (u128)0 - (u128)a : (u128)a;
    const u128 uf = f < 0 ? (u128)0 - (u128)(i128)f : (u128)(i128)f;
    const u128 limit = neg ? ((u128)1 << 127) : (((u128)1 << 127) - 1);
    if (ua > limit / uf) return neg ? i128_min() : i128_max();
    const u128 p = ua * uf;
    if (p > limit) return neg ? i128_min() : i128_max();
    return neg ? (i128)((u128)0 - p) : (i128)p;
}

// Both factors fit an i64: the product fits an i128 and cannot saturate.
__device__ __forceinline__ i128 mul_small(int64_t a, int64_t f) { return (i128)a * (i128)f; }

__device__ __forceinline__ i128 load_out(const void* base, int kind, int64_t off) {
    switch (kind) {
    case OUT_I8: return ((const int8_t*)base)[off];
    case OUT_I16: return ((const int16_t*)base)[off];
    case OUT_I32: return ((const int32_t*)base)[off];
    case OUT_I64: return ((const int64_t*)base)[off];
    default: {
        const uint64_t* p = (const uint64_t*)base + 2 * off;
        return (i128)(((u128)p[1] << 64) | p[0]);
    }
    }
}

__device__ __forceinline__ void store_out(void* base, int kind, int64_t off, i128 v) {
    switch (kind) {
    case OUT_I8: ((int8_t*)base)[off] = (int8_t)v; break;
    case OUT_I16: ((int16_t*)base)[off] = (int16_t)v; break;
    case OUT_I32: ((int32_t*)base)[off] = (int32_t)v; break;
    case OUT_I64: ((int64_t*)base)[off] = (int64_t)v; break;
    default: {
        uint64_t* p = (uint64_t*)base + 2 * off;
        p[0] = (uint64_t)(u128)v;
        p[1] = (uint64_t)((u128)v >> 64);
    }
    }
}

// encode_i128_into for a machine-integer output of `bits` bits.
__device__ __forceinline__ i128 encode_int(i128 v, int bits, int mode) {
    if (bits >= 128) return v;
    if (mode == MODE_WRAPPING) {
        // Two's complement truncation: the store keeps the low `bits` bits.
        return v;
    }
    const i128 mx = ((i128)1 << (bits - 1)) - 1;
    const i128 mn = -mx - 1;
    return v < mn ? mn : (v > mx ? mx : v);
}

struct LinearEpi {
    int64_t alpha, beta;
    int mode;
    int kind;  // OutKind
};

// One output cell: exact accumulator `acc` (an i64 sum of exact i32 chunks).
__device__ __forceinline__ void finish_cell(const LinearEpi& e, void* c, int64_t off, int64_t acc) {
    i128 tot = e.alpha == 1 ? (i128)acc : mul_small(acc, e.alpha);
    if (e.beta != 0) {
        const i128 prior = load_out(c, e.kind, off);
        const i128 s = e.kind == OUT_I128 ? sat_mul(prior, e.beta) : mul_small((int64_t)prior, e.beta);
        tot = (i128)((u128)tot + (u128)s);
    }
    store_out(c, e.kind, off, encode_int(tot, out_bits(e.kind), e.mode));
}

}  // namespace uor
