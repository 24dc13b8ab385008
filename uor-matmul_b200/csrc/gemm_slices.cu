// gemm_slices.cu -- the slice-pair tensor-core GEMM (see gemm_slices.cuh).
//
// Same pipeline as K1 (gemm_i8.cu): warp 0 TMA producer, warp 1 TMEM allocator and
// single-thread tcgen05.mma issuer, warps 2-5 epilogue, two TMEM accumulators. The
// difference is the walk: a unit's mainloop visits (slice pair, reduction block) in
// that order -- units running side by side then stream the same slice at the same
// time, so a band of one slice rather than of every slice of the diagonal lives in
// L2 -- and each pair carries its own instruction descriptor so that unsigned and
// signed slices mix exactly (kind::i8 takes u8 or s8 per operand).
#include "gemm_slices.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace uor {

struct KSUnit {
    int g, q, tm, tn;
};

__device__ __forceinline__ KSUnit ks_unit(int u, const KSParams& p) {
    KSUnit r;
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

__device__ __forceinline__ int ks_unit_blocks(const KSParams& p, int q) {
    const int first = q * p.kb_per_chunk;
    const int left = p.num_kb - first;
    return left < p.kb_per_chunk ? left : p.kb_per_chunk;
}

__global__ void __launch_bounds__(KS_THREADS, 1)
    ks_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __grid_constant__ KSParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + KS_STAGES * KS_STAGE_BYTES);
    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + KS_STAGES);
    const uint32_t tfull0 = smem_u32(bars + 2 * KS_STAGES);
    const uint32_t tempty0 = smem_u32(bars + 2 * KS_STAGES + 2);
    const uint32_t drain = smem_u32(bars + 2 * KS_STAGES + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * KS_STAGES + 5);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int units = p.num_groups * p.num_chunks * p.num_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < KS_STAGES; ++s) {
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
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 2 * KS_BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (elect_one()) {
            const uint64_t pol = l2_policy_evict_last();
            int stage = 0;
            uint32_t phase = 0;
            bool armed[KS_STAGES];
            uint32_t armed_parity[KS_STAGES];
            for (int s = 0; s < KS_STAGES; ++s) armed[s] = false, armed_parity[s] = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                const KSUnit w = ks_unit(u, p);
                const int nb = ks_unit_blocks(p, w.q);
                const int kb0 = w.q * p.kb_per_chunk;
                for (int pr = p.pair_begin[w.g]; pr < p.pair_begin[w.g + 1] && ok; ++pr) {
                    for (int kb = 0; kb < nb; ++kb) {
                        if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.budget_ns, p.status,
                                       KERR_TIMEOUT_PRODUCER)) {
                            ok = false;
                            break;
                        }
                        const uint32_t fb = full0 + 8 * stage;
                        mbar_expect_tx(fb, KS_STAGE_BYTES);
                        armed[stage] = true;
                        armed_parity[stage] = phase;
                        const uint32_t sa = smem_u32(smem + stage * KS_STAGE_BYTES);
                        const int kc = (kb0 + kb) * KS_BK;
                        tma_load_2d(sa, &tmA, fb, kc, p.pair_a[pr] * p.mp + w.tm * KS_BM, pol);
                        tma_load_2d(sa + KS_A_BYTES, &tmB, fb, kc,
                                    p.pair_b[pr] * p.np + w.tn * KS_BN, pol);
                        if (++stage == KS_STAGES) stage = 0, phase ^= 1;
                    }
                }
            }
            if (!ok) {
                for (int s = 0; s < KS_STAGES; ++s)
                    if (armed[s])
                        mbar_wait(full0 + 8 * s, armed_parity[s], p.budget_ns, p.status,
                                  KERR_TIMEOUT_DRAIN);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        int stage = 0;
        uint32_t phase = 0;
        int local = 0;
        bool ok = true, issued = false;
        for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++local) {
            const KSUnit w = ks_unit(u, p);
            const int nb = ks_unit_blocks(p, w.q);
            const int buf = local & 1;
            const uint32_t aphase = (local >> 1) & 1;
            if (!mbar_wait_warp(tempty0 + 8 * buf, aphase ^ 1, p.budget_ns, p.status,
                                KERR_TIMEOUT_MMA_ACC)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t d = tmem_base + buf * KS_BN;
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
                        const uint32_t sa = smem_u32(smem + stage * KS_STAGE_BYTES);
                        const uint32_t sb = sa + KS_A_BYTES;
                        const uint32_t idesc = p.pair_idesc[pr];
#pragma unroll
                        for (int kk = 0; kk < KS_BK / 32; ++kk)
                            mma_i8(d, smem_desc_sw128(sa + kk * 32, 16, 1024),
                                   smem_desc_sw128(sb + kk * 32, 16, 1024), idesc,
                                   (step | kk) != 0);
                        mma_commit(empty0 + 8 * stage);
                        issued = true;
                    }
                    __syncwarp();
                    if (++stage == KS_STAGES) stage = 0, phase ^= 1;
                }
            }
            if (!ok) break;
            if (elect_one()) mma_commit(tfull0 + 8 * buf);
            __syncwarp();
        }
        if (!ok) {
            if (elect_one() && issued) {
                mma_commit(drain);
                mbar_wait(drain, 0, p.budget_ns, p.status, KERR_TIMEOUT_DRAIN);
            }
            __syncwarp();
        }
    } else {
        const int quarter = warp & 3;
        const int row_in_tile = quarter * 32 + lane;
        int local = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++local) {
            const KSUnit w = ks_unit(u, p);
            const int buf = local & 1;
            const uint32_t aphase = (local >> 1) & 1;
            if (!mbar_wait_warp(tfull0 + 8 * buf, aphase, p.budget_ns, p.status,
                                KERR_TIMEOUT_EPILOGUE))
                break;
            tc_fence_after();
            const int row = w.tm * KS_BM + row_in_tile;
            const bool row_ok = row < p.m;
            int32_t* plane = p.partial + (static_cast<size_t>(w.q) * p.num_groups + w.g) *
                                             static_cast<size_t>(p.m) * p.n;
#pragma unroll 1
            for (int cc = 0; cc < KS_BN / 32; ++cc) {
                uint32_t r[32];
                const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                       buf * KS_BN + cc * 32;
                __syncwarp();
                tmem_ld32(taddr, r);
                tmem_ld_wait();
                const int col0 = w.tn * KS_BN + cc * 32;
                if (p.residue) {
                    if (row_ok && col0 < p.n)
                        ks_store_residues(p.residue + (static_cast<size_t>(w.q) * p.num_groups + w.g) *
                                                          static_cast<size_t>(p.m) * p.n +
                                              static_cast<size_t>(row) * p.n + col0,
                                          r, min(32, p.n - col0), p.res_mod[w.g], p.res_magic[w.g],
                                          p.res_off[w.g], p.res_inv[w.g]);
                } else if (row_ok && col0 < p.n) {
                    int32_t* dst = plane + static_cast<size_t>(row) * p.n + col0;
                    if (col0 + 32 <= p.n && (p.n & 3) == 0) {
#pragma unroll
                        for (int v = 0; v < 8; ++v)
                            reinterpret_cast<int4*>(dst)[v] =
                                make_int4(static_cast<int>(r[4 * v]), static_cast<int>(r[4 * v + 1]),
                                          static_cast<int>(r[4 * v + 2]),
                                          static_cast<int>(r[4 * v + 3]));
                    } else {
                        const int lim = min(32, p.n - col0);
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < lim) dst[j] = static_cast<int32_t>(r[j]);
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
        tmem_dealloc(tmem_base, 2 * KS_BN);
    }
}

cudaError_t ks_launch(const CUtensorMap& tmA, const CUtensorMap& tmB, const KSParams& p, int grid,
                      cudaStream_t stream) {
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(ks_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             KS_SMEM_BYTES);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_done[dev] = true;
    }
    ks_kernel<<<grid, KS_THREADS, KS_SMEM_BYTES, stream>>>(tmA, tmB, p);
    return cudaGetLastError();
}

void ks_balance_chunks(KSParams& p, int sm_count) {
    const bool pair = p.m > 128;
    const int tiles = (p.mp / (pair ? 256 : KS_BM)) * (p.np / KS_BN);
    const int resident = pair ? ks_pair_max_clusters() : sm_count;
    const int per_chunk = p.num_groups * tiles;
    const int c0 = p.num_chunks;
    int c_max = 8 * c0;
    if (c_max > p.num_kb / 16) c_max = p.num_kb / 16;
    if (per_chunk <= 0 || resident <= 0 || c_max <= c0) return;
    auto fill = [&](int c) {
        const long long units = static_cast<long long>(per_chunk) * c;
        const long long waves = (units + resident - 1) / resident;
        return static_cast<double>(units) / (static_cast<double>(waves) * resident);
    };
    if (fill(c0) >= 0.9) return;  // already nine tenths full: more partials only cost
    int best = c0;
    double best_fill = fill(c0);
    for (int c = c0 + 1; c <= c_max; ++c)
        if (fill(c) > best_fill + 1e-9) best_fill = fill(c), best = c;
    p.kb_per_chunk = (p.num_kb + best - 1) / best;
    p.num_chunks = (p.num_kb + p.kb_per_chunk - 1) / p.kb_per_chunk;
}

int ks_run(const void* as, int La, const void* bs, int Lb, size_t k, size_t kp, KSParams& p,
           int sm_count, cudaStream_t s, uint32_t* ctas) {
    const bool pair = p.m > 128;
    const int bm = pair ? 256 : KS_BM;
    p.tiles_m = p.mp / bm;
    p.tiles_n = p.np / KS_BN;
    p.num_tiles = p.tiles_m * p.tiles_n;
    p.group_m = p.tiles_m < 16 ? p.tiles_m : 16;
    for (int pr = 0; pr < p.pair_begin[p.num_groups]; ++pr)
        p.pair_idesc[pr] = idesc_i8(bm, KS_BN, (p.pair_sign[pr] & 1) != 0,
                                    (p.pair_sign[pr] & 2) != 0, false, false);
    CUtensorMap tmA, tmB;
    if (!make_tmap_u8(&tmA, as, k, static_cast<uint64_t>(La) * p.mp, kp, 128, 128) ||
        !make_tmap_u8(&tmB, bs, k, static_cast<uint64_t>(Lb) * p.np, kp, 128, pair ? 128 : 256))
        return UOR_B200_DEVICE_ERROR;
    const int units = p.num_groups * p.num_chunks * p.num_tiles;
    cudaError_t e;
    if (!pair) {
        const int grid = units < sm_count ? units : sm_count;
        p.tma_store = 0;
        if (ctas) *ctas = static_cast<uint32_t>(grid);
        e = ks_launch(tmA, tmB, p, grid, s);
    } else {
        CUtensorMap tmC;
        const uint64_t planes = static_cast<uint64_t>(p.num_chunks) * p.num_groups;
        p.tma_store = !p.residue && (p.n % 4) == 0 &&
                      make_tmap_s32_3d(&tmC, p.partial, p.n, p.m, planes, static_cast<uint64_t>(p.n) * 4,
                                       static_cast<uint64_t>(p.m) * p.n * 4, 32, 32);
        if (!p.tma_store) memset(&tmC, 0, sizeof(tmC));
        const int mc = ks_pair_max_clusters();
        if (ctas) *ctas = static_cast<uint32_t>(2 * (units < mc ? units : mc));
        e = ks_pair_launch(tmA, tmB, tmC, p, s);
    }
    return e == cudaSuccess ? UOR_B200_OK : UOR_B200_DEVICE_ERROR;
}

}  // namespace uor
