// gemm_i8.cu -- K1 kernel body. See gemm_i8.cuh for what it computes.
//
// Persistent, warp-specialised, one CTA per SM:
//   warp 0      one elected thread issues TMA loads into a 4-stage ring;
//   warp 1      allocates 512 TMEM columns; one elected thread issues
//               tcgen05.mma.kind::i8 (M128 N256 K32) and commits stages back;
//   warps 2-5   epilogue: tcgen05.ld the s32 accumulator (each warp owns the
//               32 TMEM lanes its warp index permits), apply Linear + encode,
//               store. Two accumulators let the epilogue of tile i overlap the
//               mainloop of tile i+1.
// No TMA multicast anywhere: the same binary runs under multi-GPU launches.
#include <cuda_runtime.h>
#include "gemm_i8.cuh"
#include "ptx.cuh"

namespace uor {

__device__ __forceinline__ void k1_tile_coords(int t, const K1Params& p, int& tm, int& tn) {
    // Rasterise in groups of group_m row-tiles so that concurrently resident
    // CTAs share A row-panels and B column-panels in L2.
    const int group = p.group_m * p.tiles_n;
    const int g = t / group;
    const int first_m = g * p.group_m;
    const int rows = min(p.tiles_m - first_m, p.group_m);
    const int r = t - g * group;
    tm = first_m + r % rows;
    tn = r / rows;
}

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(K1_THREADS, 1)
    k1_gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB, const K1Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + K1_STAGES * K1_STAGE_BYTES);
    // bars: full[S], empty[S], tfull[2], tempty[2], drain
    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + K1_STAGES);
    const uint32_t tfull0 = smem_u32(bars + 2 * K1_STAGES);
    const uint32_t tempty0 = smem_u32(bars + 2 * K1_STAGES + 2);
    const uint32_t drain = smem_u32(bars + 2 * K1_STAGES + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * K1_STAGES + 5);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < K1_STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull0 + 8 * b, 1);
            mbar_init(tempty0 + 8 * b, 4);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), K1_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (elect_one()) {
            const uint64_t pol_a = l2_policy_evict_last();
            const uint64_t pol_b = l2_policy_evict_last();
            int stage = 0;
            uint32_t phase = 0;
            uint32_t armed_parity[K1_STAGES];
            bool armed[K1_STAGES];
            for (int s = 0; s < K1_STAGES; ++s) armed[s] = false, armed_parity[s] = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
                int tm, tn;
                k1_tile_coords(t, p, tm, tn);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.budget_ns, p.status,
                                   KERR_TIMEOUT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = full0 + 8 * stage;
                    mbar_expect_tx(fb, K1_STAGE_BYTES);
                    armed[stage] = true;
                    armed_parity[stage] = phase;
                    const uint32_t sa = smem_u32(smem + stage * K1_STAGE_BYTES);
                    const uint32_t sb = sa + K1_A_BYTES;
                    const int kc = p.k_begin + kb * K1_BK;
                    if (A_MN) tma_load_2d(sa, &tmA, fb, tm * K1_BM, kc, pol_a);
                    else tma_load_2d(sa, &tmA, fb, kc, tm * K1_BM, pol_a);
                    if (B_MN) {
                        tma_load_2d(sb, &tmB, fb, tn * K1_BN, kc, pol_b);
                        tma_load_2d(sb + K1_BK * 128, &tmB, fb, tn * K1_BN + 128, kc, pol_b);
                    } else {
                        tma_load_2d(sb, &tmB, fb, kc, tn * K1_BN, pol_b);
                    }
                    if (++stage == K1_STAGES) stage = 0, phase ^= 1;
                }
            }
            if (!ok) {
                // Let every copy this thread started land before the CTA exits.
                for (int s = 0; s < K1_STAGES; ++s)
                    if (armed[s])
                        mbar_wait(full0 + 8 * s, armed_parity[s], p.budget_ns, p.status,
                                  KERR_TIMEOUT_DRAIN);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        int stage = 0;
        uint32_t phase = 0;
        int local = 0;
        bool ok = true;
        bool issued = false;
        for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++local) {
            const int buf = local & 1;
            const uint32_t aphase = (local >> 1) & 1;
            if (!mbar_wait_warp(tempty0 + 8 * buf, aphase ^ 1, p.budget_ns, p.status,
                                KERR_TIMEOUT_MMA_ACC)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t d = tmem_base + buf * K1_ACC_COLS;
            for (int kb = 0; kb < p.num_kb; ++kb) {
                if (!mbar_wait_warp(full0 + 8 * stage, phase, p.budget_ns, p.status,
                                    KERR_TIMEOUT_MMA_FULL)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (elect_one()) {
                    const uint32_t sa = smem_u32(smem + stage * K1_STAGE_BYTES);
                    const uint32_t sb = sa + K1_A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < K1_BK / 32; ++kk) {
                        // K-major: step 32 bytes along the swizzled row.
                        // MN-major: step 32 reduction rows = 4 atoms of 1 KiB.
                        const uint64_t ad = A_MN ? smem_desc_sw128(sa + kk * 4096, K1_BK * 128, 1024)
                                                 : smem_desc_sw128(sa + kk * 32, 16, 1024);
                        const uint64_t bd = B_MN ? smem_desc_sw128(sb + kk * 4096, K1_BK * 128, 1024)
                                                 : smem_desc_sw128(sb + kk * 32, 16, 1024);
                        mma_i8(d, ad, bd, p.idesc, (kb | kk) != 0);
                    }
                    mma_commit(empty0 + 8 * stage);
                    issued = true;
                }
                __syncwarp();
                if (++stage == K1_STAGES) stage = 0, phase ^= 1;
            }
            if (!ok) break;
            if (elect_one()) mma_commit(tfull0 + 8 * buf);
            __syncwarp();
        }
        if (!ok) {
            // Wait for the MMAs already issued before the accumulator is freed.
            if (elect_one()) {
                if (issued) {
                    mma_commit(drain);
                    mbar_wait(drain, 0, p.budget_ns, p.status, KERR_TIMEOUT_DRAIN);
                }
            }
            __syncwarp();
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int quarter = warp & 3;  // the TMEM lane quarter this warp may read
        const int row_in_tile = quarter * 32 + lane;
        int local = 0;
        for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++local) {
            const int buf = local & 1;
            const uint32_t aphase = (local >> 1) & 1;
            if (!mbar_wait_warp(tfull0 + 8 * buf, aphase, p.budget_ns, p.status,
                                KERR_TIMEOUT_EPILOGUE))
                break;
            tc_fence_after();
            int tm, tn;
            k1_tile_coords(t, p, tm, tn);
            const int row = tm * K1_BM + row_in_tile;
            const bool row_ok = row < p.m;
#pragma unroll 1
            for (int cc = 0; cc < K1_BN / 32; ++cc) {
                uint32_t r[32];
                const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                       buf * K1_ACC_COLS + cc * 32;
                __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp, converged
                tmem_ld32(taddr, r);
                tmem_ld_wait();
                const int col0 = tn * K1_BN + cc * 32;
                if (row_ok && col0 < p.n) {
                    if (p.fast && col0 + 32 <= p.n) {
                        int4* dst = reinterpret_cast<int4*>(static_cast<int32_t*>(p.c) +
                                                            static_cast<int64_t>(row) * p.rsc + col0);
#pragma unroll
                        for (int v = 0; v < 8; ++v)
                            dst[v] = make_int4(static_cast<int>(r[4 * v]),
                                               static_cast<int>(r[4 * v + 1]),
                                               static_cast<int>(r[4 * v + 2]),
                                               static_cast<int>(r[4 * v + 3]));
                    } else {
                        const int lim = min(32, p.n - col0);
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if (j < lim) {
                                const int64_t off = static_cast<int64_t>(row) * p.rsc +
                                                    static_cast<int64_t>(col0 + j) * p.csc;
                                finish_cell(p.epi, p.c, off, static_cast<int32_t>(r[j]));
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty0 + 8 * buf);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, K1_TMEM_COLS);
    }
}

template <bool A_MN, bool B_MN>
static cudaError_t k1_launch_t(const CUtensorMap& tmA, const CUtensorMap& tmB, const K1Params& p,
                               int grid, cudaStream_t stream) {
    auto kern = k1_gemm_i8_kernel<A_MN, B_MN>;
    // The dynamic shared-memory opt-in is per device; remember it per device.
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_done[dev]) {
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, K1_SMEM_BYTES);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_done[dev] = true;
    }
    kern<<<grid, K1_THREADS, K1_SMEM_BYTES, stream>>>(tmA, tmB, p);
    return cudaGetLastError();
}

cudaError_t k1_launch(const CUtensorMap& tmA, const CUtensorMap& tmB, bool a_mn, bool b_mn,
                      const K1Params& p, int grid, cudaStream_t stream) {
    if (a_mn) {
        return b_mn ? k1_launch_t<true, true>(tmA, tmB, p, grid, stream)
                    : k1_launch_t<true, false>(tmA, tmB, p, grid, stream);
    }
    return b_mn ? k1_launch_t<false, true>(tmA, tmB, p, grid, stream)
                : k1_launch_t<false, false>(tmA, tmB, p, grid, stream);
}

}  // namespace uor
