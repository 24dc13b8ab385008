// gemm_slices.cuh -- the slice-pair tensor-core GEMM shared by the wide-integer
// (K2) and exact-float (K6) paths.
//
// Both operands arrive as stacks of int8 "slices" (byte planes of a wider integer,
// or signed digits of a scaled float significand), K-major, padded so that no tile
// crosses a slice: A slices are [La][mp][kp] (mp a multiple of 128), B slices are
// [Lb][np][kp] (B transposed, np a multiple of 256). The product is organised in
// groups of slice pairs (s, t) that share a weight -- a diagonal s + t = d -- and
// every work unit (group, reduction chunk, 128x256 tile) accumulates all pairs of
// its group over its chunk in one s32 TMEM accumulator, then writes the s32 partial
// sums to partial[chunk][group][m][n]. The host sizes the chunk so that no partial
// can overflow; a family-specific kernel then combines the partials exactly.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace uor {

constexpr int KS_BM = 128;
constexpr int KS_BN = 256;
constexpr int KS_BK = 128;
constexpr int KS_STAGES = 4;
constexpr int KS_THREADS = 192;
constexpr int KS_A_BYTES = KS_BM * KS_BK;
constexpr int KS_B_BYTES = KS_BN * KS_BK;
constexpr int KS_STAGE_BYTES = KS_A_BYTES + KS_B_BYTES;
constexpr int KS_SMEM_BYTES = KS_STAGES * KS_STAGE_BYTES + 1024 + 256;
constexpr int KS_MAX_GROUPS = 40;
constexpr int KS_MAX_PAIRS = 256;

struct KSParams {
    int m, n;                 // output extent
    int mp, np;               // padded rows per slice in the A and B stacks
    int tiles_m, tiles_n, num_tiles, group_m;
    int num_chunks, kb_per_chunk, num_kb;  // reduction blocks per chunk, in total
    int num_groups;
    int32_t* partial;         // [num_chunks][num_groups][m][n]
    int* status;
    uint64_t budget_ns;
    int tma_store;            // pair kernel: partials written by TMA through a 3-D map
    // Residue mode (residue != nullptr): instead of s32 partials, each unit writes its
    // accumulator reduced modulo res_mod[group] as one byte in [0, res_mod) to
    // residue[chunk][group][m][n]; res_magic[group] = ceil(2^64 / res_mod[group]).
    // With res_inv[group] != 0 the stored byte is (r res_inv) mod res_mod instead.
    // res_magic = ceil(2^32 / res_mod); res_off = res_mod ceil(2^31 / res_mod) mod 2^32.
    uint8_t* residue;
    uint16_t res_mod[KS_MAX_GROUPS];
    uint16_t res_inv[KS_MAX_GROUPS];
    uint32_t res_magic[KS_MAX_GROUPS];
    uint32_t res_off[KS_MAX_GROUPS];
    int pair_begin[KS_MAX_GROUPS + 1];
    uint8_t pair_a[KS_MAX_PAIRS];
    uint8_t pair_b[KS_MAX_PAIRS];
    uint8_t pair_sign[KS_MAX_PAIRS];  // bit 0: A slice signed, bit 1: B slice signed
    uint32_t pair_idesc[KS_MAX_PAIRS];
};

// x mod p for 0 <= x < 2^40 and 2 <= p <= 256, with magic = ceil(2^64 / p): the quotient
// floor(x magic / 2^64) is exact because x (magic - 2^64 / p) / 2^64 < 2^-24 stays below the
// gap 1/p between x/p's fractional part and 1.
__device__ __forceinline__ uint32_t ks_mod(uint64_t x, uint32_t p, uint64_t magic) {
    const uint64_t q = __umul64hi(x, magic);
    return static_cast<uint32_t>(x - q * p);
}

// One epilogue fragment in residue mode: 32 consecutive s32 accumulators of one row
// (lim of them inside the output) reduced into [0, p), multiplied by inv modulo p when
// inv is not 0, and stored as bytes. A chunk holds at most 1023 blocks of 128 products of
// at most 2^14, so |acc| < 2^31 - 2^21 and x = acc + off (off = p ceil(2^31 / p) <=
// 2^31 + 255) lies in [0, 2^32); the quotient estimate umulhi(x, ceil(2^32 / p)) is
// floor(x / p) or one more, so one correction gives x mod p. (r inv < 2^16: the same
// estimate is exact there.)
__device__ __forceinline__ void ks_store_residues(uint8_t* dst, const uint32_t (&r)[32], int lim,
                                                  uint32_t p, uint32_t magic, uint32_t off,
                                                  uint32_t inv) {
    uint32_t w[8];
#pragma unroll
    for (int v = 0; v < 8; ++v) {
        w[v] = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const uint32_t x = r[4 * v + b] + off;
            int32_t y = static_cast<int32_t>(x - __umulhi(x, magic) * p);
            y += (y >> 31) & static_cast<int32_t>(p);
            uint32_t u = static_cast<uint32_t>(y);
            if (inv) {
                u *= inv;
                u -= __umulhi(u, magic) * p;
            }
            w[v] |= u << (8 * b);
        }
    }
    if (lim == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
        reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (j < lim) dst[j] = static_cast<uint8_t>(w[j >> 2] >> (8 * (j & 3)));
    }
}

// Rows per slice in the A stack: whole tiles of the kernel ks_run will choose.
inline size_t ks_rows_pad(size_t m) {
    const size_t t = m > 128 ? 256 : 128;
    return (m + t - 1) / t * t;
}

// tmA: dims {k, La * mp}, box {128, 128}; tmB: dims {k, Lb * np}, box {128, 256};
// both uint8 with 128-byte swizzle.
cudaError_t ks_launch(const CUtensorMap& tmA, const CUtensorMap& tmB, const KSParams& p,
                      int grid, cudaStream_t stream);

// The same product on CTA pairs (tcgen05 cta_group::2): 256 x 256 tiles, mp a multiple
// of 256, tmB box {128, 128}; with p.tma_store the partials go out through tmC, an s32
// 3-D map {n, m, chunks * groups} with box {32, 32, 1}.
cudaError_t ks_pair_launch(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmC,
                           const KSParams& p, cudaStream_t stream);
int ks_pair_max_clusters();

// More reduction chunks than the lane bound asks for when the work units (groups x
// chunks x tiles) would leave the last wave over the resident CTAs (pairs) mostly empty:
// a deep product of few tiles (configs[3]: 10 moduli x 16 tiles = 160 units on 74 pairs,
// its third wave 16 % full) splits k further, each chunk's partial summed afterwards as
// any chunk's is. Unless the waves are nine tenths full already: between p.num_chunks and
// 8 x that, at least 16 k-blocks a chunk, the count with the fullest waves (the smallest
// on ties). Needs p.num_kb, p.kb_per_chunk,
// p.num_groups, p.m, p.mp, p.np; updates p.kb_per_chunk and p.num_chunks.
void ks_balance_chunks(KSParams& p, int sm_count);

// Runs the slice-pair product: `as` is the A stack [La][mp][kp] (mp = ks_rows_pad(m)),
// `bs` the B stack [Lb][np][kp] (np a multiple of 256). p holds m, n, mp, np, the
// groups (pair_begin, pair_a, pair_b, pair_sign), the chunking and the partial buffer;
// ks_run fills the tiles and instruction descriptors, picks CTA pairs when m > 128,
// builds the tensor maps and launches on `stream`. Returns a uor_b200_status.
int ks_run(const void* as, int La, const void* bs, int Lb, size_t k, size_t kp, KSParams& p,
           int sm_count, cudaStream_t stream, uint32_t* ctas);

}  // namespace uor
