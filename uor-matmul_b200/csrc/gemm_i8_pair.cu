// gemm_i8_pair.cu -- K1 on CTA pairs: the exact i8 GEMM with tcgen05.mma.cta_group::2.
//
// Same computation and epilogue as gemm_i8.cu (see gemm_i8.cuh), on a 256 x 256 output
// tile shared by a cluster of two CTAs on neighbouring SMs. Each CTA loads its own 128
// rows of A and its own 128 columns of B (no TMA multicast); the leader CTA issues
// M256 N256 K32 MMAs that read A by rows and B by columns from both CTAs' shared
// memory, and each CTA's TMEM holds the accumulator for its own 128 rows. Per SM this
// halves the B bytes a tile needs and leaves room for 6 pipeline stages of 32 KiB.
//
// Barriers: both CTAs' TMA loads complete on the leader's full[s] (armed by the leader
// for both CTAs' bytes); the leader's commits arrive on empty[s] and tfull[b] in both
// CTAs at once; both CTAs' epilogue warps arrive on the leader's tempty[b].
#include <cuda_runtime.h>
#include "gemm_i8.cuh"
#include "ptx.cuh"

namespace uor {

constexpr int KP_BM = 256;  // rows per CTA pair (128 per CTA)
constexpr int KP_BN = 256;
constexpr int KP_BK = 128;
constexpr int KP_STAGES = 6;
constexpr int KP_THREADS = 192;
constexpr int KP_A_BYTES = 128 * KP_BK;
constexpr int KP_B_BYTES = 128 * KP_BK;
constexpr int KP_STAGE_BYTES = KP_A_BYTES + KP_B_BYTES;
// Epilogue staging for TMA stores: per epilogue warp two 32 x 32 s32 blocks (4 KiB each).
constexpr int KP_EPI_BYTES = 4 * 2 * 4096;
constexpr int KP_SMEM_BYTES = KP_STAGES * KP_STAGE_BYTES + KP_EPI_BYTES + 1024 + 256;

__device__ __forceinline__ void kp_tile(int t, const K1Params& p, int& tm, int& tn) {
    const int group = p.group_m * p.tiles_n;
    const int g = t / group;
    const int first = g * p.group_m;
    const int rows = min(p.tiles_m - first, p.group_m);
    const int r = t - g * group;
    tm = first + r % rows;
    tn = r / rows;
}

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(KP_THREADS, 1)
    k1_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const K1Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* epi_smem = smem + KP_STAGES * KP_STAGE_BYTES;  // 1 KiB aligned
    uint64_t* bars = reinterpret_cast<uint64_t*>(epi_smem + KP_EPI_BYTES);
    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + KP_STAGES);
    const uint32_t tfull0 = smem_u32(bars + 2 * KP_STAGES);
    const uint32_t tempty0 = smem_u32(bars + 2 * KP_STAGES + 2);
    const uint32_t drain = smem_u32(bars + 2 * KP_STAGES + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * KP_STAGES + 5);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cid = static_cast<int>(cluster_id_x());
    const int ncl = static_cast<int>(nclusters_x());

    if (threadIdx.x == 0) {
        for (int s = 0; s < KP_STAGES; ++s) {
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
    if (warp == 1) tmem_alloc_pair(smem_u32(tmem_slot), 2 * KP_BN);
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers exist before either signals the other
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (elect_one()) {
            const uint64_t pol = l2_policy_evict_last();
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            bool armed[KP_STAGES];
            uint32_t armed_parity[KP_STAGES];
            for (int s = 0; s < KP_STAGES; ++s) armed[s] = false, armed_parity[s] = 0;
            for (int t = cid; t < p.num_tiles && ok; t += ncl) {
                int tm, tn;
                kp_tile(t, p, tm, tn);
                const int row0 = tm * KP_BM + static_cast<int>(rank) * 128;
                const int col0 = tn * KP_BN + static_cast<int>(rank) * 128;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.budget_ns, p.status,
                                   KERR_TIMEOUT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb_local = full0 + 8 * stage;
                    if (leader) {
                        mbar_expect_tx(fb_local, 2 * KP_STAGE_BYTES);
                        armed[stage] = true;
                        armed_parity[stage] = phase;
                    }
                    const uint32_t fb = mapa_shared(fb_local, 0);
                    const uint32_t sa = smem_u32(smem + stage * KP_STAGE_BYTES);
                    const uint32_t sb = sa + KP_A_BYTES;
                    const int kc = p.k_begin + kb * KP_BK;
                    if (A_MN) tma_load_2d_pair(sa, &tmA, fb, row0, kc, pol);
                    else tma_load_2d_pair(sa, &tmA, fb, kc, row0, pol);
                    if (B_MN) tma_load_2d_pair(sb, &tmB, fb, col0, kc, pol);
                    else tma_load_2d_pair(sb, &tmB, fb, kc, col0, pol);
                    if (++stage == KP_STAGES) stage = 0, phase ^= 1;
                }
            }
            if (!ok && leader)
                for (int s = 0; s < KP_STAGES; ++s)
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
            const uint32_t idesc = p.idesc;
            for (int t = cid; t < p.num_tiles && ok; t += ncl, ++local) {
                const int buf = local & 1;
                const uint32_t aphase = (local >> 1) & 1;
                if (!mbar_wait_warp(tempty0 + 8 * buf, aphase ^ 1, p.budget_ns, p.status,
                                    KERR_TIMEOUT_MMA_ACC)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + buf * KP_BN;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait_warp(full0 + 8 * stage, phase, p.budget_ns, p.status,
                                        KERR_TIMEOUT_MMA_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (elect_one()) {
                        const uint32_t sa = smem_u32(smem + stage * KP_STAGE_BYTES);
                        const uint32_t sb = sa + KP_A_BYTES;
#pragma unroll
                        for (int kk = 0; kk < KP_BK / 32; ++kk) {
                            const uint64_t ad = A_MN ? smem_desc_sw128(sa + kk * 4096, KP_BK * 128, 1024)
                                                     : smem_desc_sw128(sa + kk * 32, 16, 1024);
                            const uint64_t bd = B_MN ? smem_desc_sw128(sb + kk * 4096, KP_BK * 128, 1024)
                                                     : smem_desc_sw128(sb + kk * 32, 16, 1024);
                            mma_i8_pair(d, ad, bd, idesc, (kb | kk) != 0);
                        }
                        mma_commit_pair(empty0 + 8 * stage, 0x3);
                        issued = true;
                    }
                    __syncwarp();
                    if (++stage == KP_STAGES) stage = 0, phase ^= 1;
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
        // Two 4 KiB staging blocks per warp, 128-byte swizzled as the C tensor map expects.
        uint8_t* stage_w = epi_smem + quarter * 2 * 4096;
        const uint64_t out_policy = l2_policy_evict_first();  // C is written once, never re-read
        int local = 0, nstore = 0;
        for (int t = cid; t < p.num_tiles; t += ncl, ++local) {
            const int buf = local & 1;
            const uint32_t aphase = (local >> 1) & 1;
            if (!mbar_wait_warp(tfull0 + 8 * buf, aphase, p.budget_ns, p.status,
                                KERR_TIMEOUT_EPILOGUE))
                break;
            tc_fence_after();
            int tm, tn;
            kp_tile(t, p, tm, tn);
            const int row = tm * KP_BM + row_in_tile;
            const bool row_ok = row < p.m;
            const int wrow0 = tm * KP_BM + static_cast<int>(rank) * 128 + quarter * 32;
#pragma unroll 1
            for (int cc = 0; cc < KP_BN / 32; ++cc) {
                uint32_t r[32];
                const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                       buf * KP_BN + cc * 32;
                __syncwarp();
                tmem_ld32(taddr, r);
                tmem_ld_wait();
                if (cc == KP_BN / 32 - 1) {
                    // The accumulator is in registers: hand TMEM back before storing.
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(mapa_shared(tempty0 + 8 * buf, 0));
                }
                const int col0 = tn * KP_BN + cc * 32;
                if (p.tma_store) {
                    if (wrow0 < p.m && col0 < p.n) {
                        uint8_t* sb = stage_w + (nstore & 1) * 4096;
                        if (lane == 0) bulk_wait_read<1>();  // this block's previous store has read it
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
                            tma_store_2d_hint(&tmC, smem_u32(sb), col0, wrow0, out_policy);
                            bulk_commit();
                        }
                        ++nstore;
                    }
                } else if (row_ok && col0 < p.n) {
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
        }
        if (lane == 0) bulk_wait_all();  // every store has left shared memory
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // neither CTA leaves while the other may still signal it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, 2 * KP_BN);
    }
}

template <bool A_MN, bool B_MN>
static cudaError_t kp_launch_t(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmC,
                               const K1Params& p, int max_clusters, cudaStream_t stream) {
    auto kern = k1_pair_kernel<A_MN, B_MN>;
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_done[dev]) {
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, KP_SMEM_BYTES);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_done[dev] = true;
    }
    const int clusters = p.num_tiles < max_clusters ? p.num_tiles : max_clusters;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    cfg.blockDim = dim3(KP_THREADS, 1, 1);
    cfg.dynamicSmemBytes = KP_SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, tmA, tmB, tmC, p);
}

// How many CTA pairs of this kernel can be resident at once (queried once per device).
int k1_pair_max_clusters() {
    static int cached[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
    auto kern = k1_pair_kernel<false, true>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, KP_SMEM_BYTES);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 512, 1, 1);
    cfg.blockDim = dim3(KP_THREADS, 1, 1);
    cfg.dynamicSmemBytes = KP_SMEM_BYTES;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        n = sms / 2;
    }
    if (dev >= 0 && dev < 64) cached[dev] = n;
    return n;
}

cudaError_t k1_pair_launch(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmC,
                           bool a_mn, bool b_mn, const K1Params& p, cudaStream_t stream) {
    const int mc = k1_pair_max_clusters();
    if (a_mn) {
        return b_mn ? kp_launch_t<true, true>(tmA, tmB, tmC, p, mc, stream)
                    : kp_launch_t<true, false>(tmA, tmB, tmC, p, mc, stream);
    }
    return b_mn ? kp_launch_t<false, true>(tmA, tmB, tmC, p, mc, stream)
                : kp_launch_t<false, false>(tmA, tmB, tmC, p, mc, stream);
}

}  // namespace uor
