// gemm_coded.cuh -- K5: exact GEMM against a nibble-coded operand, decoded in the
// MMA pipeline (no dense copy of the coded operand ever reaches HBM).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include "gemm_i8.cuh"
#include "int_epilogue.cuh"

namespace uor {

constexpr int K5_BM = 128;  // decoded weight columns j per tile (TMEM lanes)
constexpr int K5_BN = 256;  // activation rows i per tile (TMEM columns)
constexpr int K5_BK = 128;  // reduction per stage
constexpr int K5_STAGES = 4;
constexpr int K5_DEC_WARPS = 8;
constexpr int K5_THREADS = 32 * (6 + K5_DEC_WARPS);  // TMA, MMA, 4 epilogue, decoders
constexpr int K5_W_BYTES = K5_BM * K5_BK;            // decoded weights, 16 KiB
constexpr int K5_X_BYTES = K5_BN * K5_BK;            // activations, 32 KiB
constexpr int K5_C_BYTES = K5_BM * K5_BK / 2;        // codes, 8 KiB
constexpr int K5_STAGE_BYTES = K5_W_BYTES + K5_X_BYTES + K5_C_BYTES;
constexpr int K5_SMEM_BYTES = K5_STAGES * K5_STAGE_BYTES + 1024 + 256;

struct K5Params {
    int m, n, k;            // C is m x n; activations m x k; weights k x n (decoded)
    int tiles_j, tiles_i, num_tiles, group_j;
    int num_kb;
    int orientation;        // 0: codes k x n (coded_gemm); 1: codes n x k (tabulated)
    uint32_t table[4];      // 16 decoded int8 values, table[v % N] for v in 0..15
    void* c;
    int64_t rsc, csc;
    LinearEpi epi;
    int fast;               // s32 output, alpha 1, beta 0
    uint32_t idesc;
    int* status;
    uint64_t budget_ns;
};

// Eight nibbles (first element lowest) -> eight table bytes (.x: elements 0-3, .y: 4-7).
// __byte_perm reads three bits of each selector nibble (and only the low 16 bits of the
// selector), so the code nibbles themselves pick among table[0..7] (t0:t1) and
// table[8..15] (t2:t3); a third permute takes, byte by byte, the half that the
// nibble's bit 3 names.
__device__ __forceinline__ uint2 dec8(uint32_t w, uint32_t t0, uint32_t t1, uint32_t t2,
                                     uint32_t t3) {
    const uint32_t pick = ((w >> 1) & 0x44444444u) | 0x32103210u;
    const uint32_t wh = w >> 16, ph = pick >> 16;
    uint2 r;
    r.x = __byte_perm(__byte_perm(t0, t1, w), __byte_perm(t2, t3, w), pick);
    r.y = __byte_perm(__byte_perm(t0, t1, wh), __byte_perm(t2, t3, wh), ph);
    return r;
}

// tmX: activations K-major, dims {k, m}, box {128, 256}, 128-byte swizzle.
// tmC: codes, no swizzle, box {64 bytes, 128 rows}:
//   orientation 0: dims {n/2, k}; orientation 1: dims {k/2, n}.
cudaError_t k5_launch(const CUtensorMap& tmX, const CUtensorMap& tmC, const K5Params& p, int grid,
                      cudaStream_t stream);

// K1C: K1's CTA-pair GEMM (256 x 256 tiles, p.idesc M256 N256) with B decoded on chip.
// Code bytes of p.epb elements each:
//   2: Packed<Grid<N>, 2> nibbles through the 16-entry table (4 words, table[v % N] for v
//      in 0..15, or read from dtable);
//   4, 8: one code byte holds epb consecutive elements of a coded row, decoded through a
//      256-entry table the kernel builds in shared memory from byte_tier: K1C_BOOK
//      (book[(b % book_n) * epb + t], Book with one-byte codes and blocks of epb), K1C_SIGN
//      (bit t: +1 set, -1 clear; Sign with blocks of 8 per code byte) or K1C_TERNARY
//      (digit t = bits 2t..2t+1: 0 -> -1, 2 -> +1, 1 and 3 -> 0; Ternary with blocks of 4
//      per code byte), K1C_GRID (Packed<Grid<N>, epb>: book[sub-code t % book_n], the
//      sub-codes 8 / epb bits wide, low first), every value minus zero.
constexpr int K1C_BOOK = 0, K1C_SIGN = 1, K1C_TERNARY = 2, K1C_GRID = 3;
struct K1CParams : K1Params {
    uint32_t table[4];
    const int8_t* dtable;  // when set: the table in device memory, read by the kernel
    int table_len;         // its entries N (1..16)
    int epb;               // elements per code byte: 2, 4 or 8
    int byte_tier;         // epb 4 or 8: K1C_BOOK, K1C_SIGN, K1C_TERNARY or K1C_GRID
    const int8_t* book;    // K1C_BOOK: the book in device memory, book_n x epb bytes;
                           // K1C_GRID: the book_n-entry table in device memory
    int book_n;
    int zero;              // subtracted from every decoded value (Offset)
};
// tmA: activations K-major, dims {k, m}, box {128, 128}, 128-byte swizzle.
// tmQ: codes, no swizzle, box {128 / epb bytes, 128 rows}: orientation 0 dims {n/epb, k},
//      orientation 1 dims {k/epb, n}. With p.tma_store, tmC is the s32 output map
//      (dims {n, m}, box {32, 32}, 128-byte swizzle). k must not exceed K1_LANE_DEPTH.
// tall: 512 x 256 tiles (p.tiles_m counts 512-row tiles), each decoded B stage feeding two
// M256 halves; else 256 x 256.
cudaError_t k1c_launch(const CUtensorMap& tmA, const CUtensorMap& tmQ, const CUtensorMap& tmC,
                       int orientation, bool tall, const K1CParams& p, cudaStream_t stream);
int k1c_max_clusters();

}  // namespace uor
