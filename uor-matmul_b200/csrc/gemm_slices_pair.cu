// gemm_slices_pair.cu -- the slice-pair product (gemm_slices.cuh) on CTA pairs.
//
// The walk of gemm_slices.cu -- work units (diagonal group, reduction chunk, tile), each
// accumulating every slice pair of its group over its chunk in one s32 TMEM
// accumulator -- with the pipeline of gemm_i8_pair.cu: a cluster of two CTAs shares a
// 256 x 256 tile, each CTA loads its own 128 rows of the A slice and its own 128 columns
// of the B slice per (pair, k-block), pairs outermost, and the leader issues M256 N256 K32
// tcgen05.mma.cta_group::2 instructions with that pair's descriptor (u8 or s8 per
// operand). The epilogue stages 32 x 32 blocks in swizzled shared memory and writes the
// partial planes with 3-D TMA stores (plane = chunk * groups + group). Every TMA load is
// issued by the CTA that consumes it; no load is shared between the CTAs.
#include <cuda_runtime.h>
#include "gemm_slices.cuh"
#include "ptx.cuh"

namespace uor {

constexpr int KQ_BM = 256;
constexpr int KQ_BN = 256;
constexpr int KQ_BK = 128;
constexpr int KQ_STAGES = 6;
constexpr int KQ_THREADS = 192;
constexpr int KQ_A_BYTES = 128 * KQ_BK;
constexpr int KQ_B_BYTES = 128 * KQ_BK;
constexpr int KQ_STAGE_BYTES = KQ_A_BYTES + KQ_B_BYTES;
constexpr int KQ_EPI_BYTES = 4 * 2 * 4096;
constexpr int KQ_SMEM_BYTES = KQ_STAGES * KQ_STAGE_BYTES + KQ_EPI_BYTES + 1024 + 256;

struct KQUnit {
    int g, q, tm, tn;
};

__device__ __forceinline__ KQUnit kq_unit(int u, const KSParams& p) {
    KQUnit r;
    const int per_group = p.num_chunks * p.num_tiles;
    r.g = u / per_group;
    const int rem = u - r.g * per_group;
    r.q = rem / p.num_tiles;
    const int t = rem - r.q * p.num_tiles;
    const int group = p.group_m * p.tiles_n;
    const int gi = t / group;
    const int first_m = gi * p.group_m;
    const int rows = min(p.tiles_m - first_m, p.group_m);
    const int rr = t - gi * group;
    r.tm = first_m + rr % rows;
    r.tn = rr / rows;
    return r;
}

__device__ __forceinline__ int kq_unit_blocks(const KSParams& p, int q) {
    const int left = p.num_kb - q * p.kb_per_chunk;
    return left < p.kb_per_chunk ? left : p.kb_per_chunk;
}

__global__ void __launch_bounds__(KQ_THREADS, 1)
    ks_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ KSParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* epi_smem = smem + KQ_STAGES * KQ_STAGE_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(epi_smem + KQ_EPI_BYTES);
    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + KQ_STAGES);
    const uint32_t tfull0 = smem_u32(bars + 2 * KQ_STAGES);
    const uint32_t tempty0 = smem_u32(bars + 2 * KQ_STAGES + 2);
    const uint32_t drain = smem_u32(bars + 2 * KQ_STAGES + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * KQ_STAGES + 5);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cid = static_cast<int>(cluster_id_x());
    const int ncl = static_cast<int>(nclusters_x());
    const int units = p.num_groups * p.num_chunks * p.num_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < KQ_STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull0 + 8 * b, 1);
            mbar_init(tempty0 + 8 * b, 8);  // 4 epilogue warps in each CTA of the pair
        }
        mbar_init(drain, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (p.tma_store) tma_prefetch_desc(&tmC);
    }
    if (warp == 1) tmem_alloc_pair(smem_u32(tmem_slot), 2 * KQ_BN);
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (elect_one()) {
            const uint64_t pol = l2_policy_evict_last();
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            bool armed[KQ_STAGES];
            uint32_t armed_parity[KQ_STAGES];
            for (int s = 0; s < KQ_STAGES; ++s) armed[s] = false, armed_parity[s] = 0;
            for (int u = cid; u < units && ok; u += ncl) {
                const KQUnit w = kq_unit(u, p);
                const int nb = kq_unit_blocks(p, w.q);
                const int kb0 = w.q * p.kb_per_chunk;
                const int row0 = w.tm * KQ_BM + static_cast<int>(rank) * 128;
                const int col0 = w.tn * KQ_BN + static_cast<int>(rank) * 128;
                for (int pr = p.pair_begin[w.g]; pr < p.pair_begin[w.g + 1] && ok; ++pr) {
                    for (int kb = 0; kb < nb; ++kb) {
                        if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.budget_ns, p.status,
                                       KERR_TIMEOUT_PRODUCER)) {
                            ok = false;
                            break;
                        }
                        const uint32_t fb_local = full0 + 8 * stage;
                        if (leader) {
                            mbar_expect_tx(fb_local, 2 * KQ_STAGE_BYTES);
                            armed[stage] = true;
                            armed_parity[stage] = phase;
                        }
                        const uint32_t fb = mapa_shared(fb_local, 0);
                        const uint32_t sa = smem_u32(smem + stage * KQ_STAGE_BYTES);
                        const int kc = (kb0 + kb) * KQ_BK;
                        tma_load_2d_pair(sa, &tmA, fb, kc, p.pair_a[pr] * p.mp + row0, pol);
                        tma_load_2d_pair(sa + KQ_A_BYTES, &tmB, fb, kc, p.pair_b[pr] * p.np + col0,
                                         pol);
                        if (++stage == KQ_STAGES) stage = 0, phase ^= 1;
                    }
                }
            }
            if (!ok && leader)
                for (int s = 0; s < KQ_STAGES; ++s)
                    if (armed[s])
                        mbar_wait(full0 + 8 * s, armed_parity[s], p.budget_ns, p.status,
                                  KERR_TIMEOUT_DRAIN);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA (leader only)
        if (leader) {
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            bool ok = true, issued = false;
            for (int u = cid; u < units && ok; u += ncl, ++local) {
                const KQUnit w = kq_unit(u, p);
                const int nb = kq_unit_blocks(p, w.q);
                const int buf = local & 1;
                const uint32_t aphase = (local >> 1) & 1;
                if (!mbar_wait_warp(tempty0 + 8 * buf, aphase ^ 1, p.budget_ns, p.status,
                                    KERR_TIMEOUT_MMA_ACC)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + buf * KQ_BN;
                int step = 0;
                for (int pr = p.pair_begin[w.g]; pr < p.pair_begin[w.g + 1] && ok; ++pr) {
                    for (int kb = 0; kb < nb; ++kb, ++step) {
                        if (!mbar_wait_warp(full0 + 8 * stage, phase, p.budget_ns, p.status,
                                            KERR_TIMEOUT_MMA_FULL)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        if (elect_one()) {
                            const uint32_t sa = smem_u32(smem + stage * KQ_STAGE_BYTES);
                            const uint32_t sb = sa + KQ_A_BYTES;
                            const uint32_t idesc = p.pair_idesc[pr];
#pragma unroll
                            for (int kk = 0; kk < KQ_BK / 32; ++kk)
                                mma_i8_pair(d, smem_desc_sw128(sa + kk * 32, 16, 1024),
                                            smem_desc_sw128(sb + kk * 32, 16, 1024), idesc,
                                            (step | kk) != 0);
                            mma_commit_pair(empty0 + 8 * stage, 0x3);
                            issued = true;
                        }
                        __syncwarp();
                        if (++stage == KQ_STAGES) stage = 0, phase ^= 1;
                    }
                }
                if (!ok) break;
                if (elect_one()) mma_commit_pair(tfull0 + 8 * buf, 0x3);
                __syncwarp();
            }
            if (!ok) {
                if (elect_one() && issued) {
                    mma_commit_pair(drain, 0x1);
                    mbar_wait(drain, 0, p.budget_ns, p.status, KERR_TIMEOUT_DRAIN);
                }
                __syncwarp();
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue (both CTAs)
        const int quarter = warp & 3;
        const int row_in_tile = static_cast<int>(rank) * 128 + quarter * 32 + lane;
        uint8_t* stage_w = epi_smem + quarter * 2 * 4096;
        const uint64_t out_policy = l2_policy_evict_first();
        int local = 0, nstore = 0;
        for (int u = cid; u < units; u += ncl, ++local) {
            const KQUnit w = kq_unit(u, p);
            const int buf = local & 1;
            const uint32_t aphase = (local >> 1) & 1;
            if (!mbar_wait_warp(tfull0 + 8 * buf, aphase, p.budget_ns, p.status,
                                KERR_TIMEOUT_EPILOGUE))
                break;
            tc_fence_after();
            const int plane = w.q * p.num_groups + w.g;
            const int row = w.tm * KQ_BM + row_in_tile;
            const int wrow0 = w.tm * KQ_BM + static_cast<int>(rank) * 128 + quarter * 32;
            int32_t* pl = p.partial + static_cast<size_t>(plane) * static_cast<size_t>(p.m) * p.n;
#pragma unroll 1
            for (int cc = 0; cc < KQ_BN / 32; ++cc) {
                uint32_t r[32];
                const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                       buf * KQ_BN + cc * 32;
                __syncwarp();
                tmem_ld32(taddr, r);
                tmem_ld_wait();
                if (cc == KQ_BN / 32 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(mapa_shared(tempty0 + 8 * buf, 0));
                }
                const int col0 = w.tn * KQ_BN + cc * 32;
                if (p.residue) {
                    if (row < p.m && col0 < p.n)
                        ks_store_residues(p.residue + static_cast<size_t>(plane) * p.m * p.n +
                                              static_cast<size_t>(row) * p.n + col0,
                                          r, min(32, p.n - col0), p.res_mod[w.g], p.res_magic[w.g],
                                          p.res_off[w.g], p.res_inv[w.g]);
                } else if (p.tma_store) {
                    if (wrow0 < p.m && col0 < p.n) {
                        uint8_t* sb = stage_w + (nstore & 1) * 4096;
                        if (lane == 0) bulk_wait_read<1>();
                        __syncwarp();
#pragma unroll
                        for (int v = 0; v < 8; ++v)
                            *reinterpret_cast<int4*>(sb + lane * 128 + ((v ^ (lane & 7)) << 4)) =
                                make_int4(static_cast<int>(r[4 * v]), static_cast<int>(r[4 * v + 1]),
                                          static_cast<int>(r[4 * v + 2]),
                                          static_cast<int>(r[4 * v + 3]));
                        fence_proxy_async();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_3d_hint(&tmC, smem_u32(sb), col0, wrow0, plane, out_policy);
                            bulk_commit();
                        }
                        ++nstore;
                    }
                } else if (row < p.m && col0 < p.n) {
                    int32_t* dst = pl + static_cast<size_t>(row) * p.n + col0;
                    const int lim = min(32, p.n - col0);
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (j < lim) dst[j] = static_cast<int32_t>(r[j]);
                }
            }
        }
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, 2 * KQ_BN);
    }
}

static cudaLaunchConfig_t kq_config(int clusters, cudaStream_t stream, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    cfg.blockDim = dim3(KQ_THREADS, 1, 1);
    cfg.dynamicSmemBytes = KQ_SMEM_BYTES;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

static bool kq_attr(int dev) {
    static bool done[64] = {};
    if (dev >= 0 && dev < 64 && done[dev]) return true;
    if (cudaFuncSetAttribute(ks_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             KQ_SMEM_BYTES) != cudaSuccess)
        return false;
    if (dev >= 0 && dev < 64) done[dev] = true;
    return true;
}

int ks_pair_max_clusters() {
    static int cached[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
    kq_attr(dev);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = kq_config(512, nullptr, attr);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, ks_pair_kernel, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        n = sms / 2;
    }
    if (dev >= 0 && dev < 64) cached[dev] = n;
    return n;
}

cudaError_t ks_pair_launch(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmC,
                           const KSParams& p, cudaStream_t stream) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (!kq_attr(dev)) return cudaGetLastError();
    const int units = p.num_groups * p.num_chunks * p.num_tiles;
    const int mc = ks_pair_max_clusters();
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = kq_config(units < mc ? units : mc, stream, attr);
    return cudaLaunchKernelEx(&cfg, ks_pair_kernel, tmA, tmB, tmC, p);
}

}  // namespace uor
