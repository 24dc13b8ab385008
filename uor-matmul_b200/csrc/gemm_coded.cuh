// gemm_coded.cuh -- the codec tier's decode helpers and K1C, K1's CTA-pair GEMM with the
// coded operand decoded on chip (no dense copy of it ever reaches HBM).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include "gemm_i8.cuh"
#include "int_epilogue.cuh"

namespace uor {

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
