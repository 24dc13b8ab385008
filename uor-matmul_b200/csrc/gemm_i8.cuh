// gemm_i8.cuh -- K1: the exact int8 GEMM on the 5th-generation tensor cores.
//
// Replaces the reference's blocked kernel traversal for i8 (gemm_auto ->
// gemm_packed_impl -> run, kernel.rs:523-1377, with the I8_I32 tile families of
// isa/portable.rs:85 and isa/x86.rs:80-713): C := encode(alpha * A B + beta * C)
// with the products accumulated exactly in s32 TMEM lanes.
//
// Exactness: an s8 x s8 product is at most 2^14 in magnitude, so a 32-bit lane
// holds any run of at most lane_depth = floor((2^31 - 1) / 2^14) = 131071
// products (spec.rs:232-243). The host cuts deeper reductions into chunks of at
// most that depth and sums the chunks in 64 bits; the kernel never sees k deeper
// than one lane can hold.
#pragma once
#include <cstdint>
#include <cuda.h>
#include "int_epilogue.cuh"

namespace uor {

// CTA tile: 128 rows x 256 columns, 128 bytes of the reduction per stage.
constexpr int K1_BM = 128;
constexpr int K1_BN = 256;
constexpr int K1_BK = 128;
constexpr int K1_STAGES = 4;
constexpr int K1_THREADS = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int K1_A_BYTES = K1_BM * K1_BK;
constexpr int K1_B_BYTES = K1_BN * K1_BK;
constexpr int K1_STAGE_BYTES = K1_A_BYTES + K1_B_BYTES;
constexpr int K1_ACC_COLS = K1_BN;       // s32 accumulator columns per tile
constexpr int K1_TMEM_COLS = 2 * K1_BN;  // two accumulators: epilogue overlaps the next tile
constexpr int K1_SMEM_BYTES = K1_STAGES * K1_STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;

// The largest reduction one s32 lane holds exactly for full-range s8 x s8,
// rounded down to a whole number of stages.
constexpr int64_t K1_LANE_DEPTH = 131071;
constexpr int64_t K1_CHUNK_K = (K1_LANE_DEPTH / K1_BK) * K1_BK;  // 130944

struct K1Params {
    int m, n;            // output extent of this launch
    int k_begin;         // first reduction coordinate of this launch
    int num_kb;          // reduction blocks of K1_BK
    int tiles_m, tiles_n, num_tiles, group_m;
    void* c;             // element (0,0) of the output view
    int64_t rsc, csc;    // output element strides
    LinearEpi epi;
    int fast;            // s32 output, alpha 1, beta 0, unit column stride, 16-byte rows
    int tma_store;       // pair kernel: fast output written by TMA stores through tmC
    uint32_t idesc;
    int* status;
    uint64_t budget_ns;
};

// Launch on `stream`. tmA/tmB are 2-D uint8 tensor maps with 128-byte swizzle:
//   A K-major: dims {k, m}, box {128, 128};   A MN-major: dims {m, k}, box {128, 128}
//   B K-major: dims {k, n}, box {128, 256};   B MN-major: dims {n, k}, box {128, 128}
cudaError_t k1_launch(const CUtensorMap& tmA, const CUtensorMap& tmB, bool a_mn, bool b_mn,
                      const K1Params& p, int grid, cudaStream_t stream);

// The same GEMM on CTA pairs (tcgen05 cta_group::2): 256 x 256 tiles, p.tiles_m counts
// 256-row tiles and p.idesc must describe M256 N256. Grid and cluster size are chosen
// here (clusters of 2, as many as can be resident). With p.tma_store, tmC is an s32
// tensor map of the output (dims {n, m}, box {32, 32}, 128-byte swizzle).
cudaError_t k1_pair_launch(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmC,
                           bool a_mn, bool b_mn, const K1Params& p, cudaStream_t stream);
int k1_pair_max_clusters();

}  // namespace uor
