// gemm_coded.cu -- K5: C = A decode(B) with the codebook decode fused into the
// tensor-core pipeline.
//
// Replaces coded_gemm (crates/uor-matmul-gemm/src/coded.rs:98-142; one scalar decode
// per multiply) and the product gemm_tabulated computes (tabulated.rs:2555) for the
// fixed-width tier Packed<Grid<N>, 2> (codecs.rs:80-196): element (r, c) of the coded
// matrix is table[nibble % N], nibble c % 2 of byte c / 2 of row r, low nibble first.
//
// The decoded weights are the MMA's M operand (128 weight columns per tile) and the
// activations its N operand (256 rows), so each decoded element feeds 256 products.
// Per stage: TMA brings 8 KiB of raw codes (no swizzle) and 32 KiB of activations
// (128-byte swizzle); eight decoder warps turn each 8-byte group of codes (16
// nibbles) into 16 int8 values with byte permutes against the 16-entry table held
// in registers (three permutes per four values), and store them straight into the swizzled operand layout
// (MN-major for codes laid k x n, K-major for codes laid n x k -- the same index
// arithmetic either way). fence.proxy.async makes those stores visible to the
// tensor core. The accumulator is the transposed tile C^T; lanes map to consecutive
// output columns, so the epilogue's stores stay coalesced.
#include "gemm_coded.cuh"
#include "ptx.cuh"

namespace uor {

__device__ __forceinline__ void k5_tile(int t, const K5Params& p, int& tj, int& ti) {
    const int group = p.group_j * p.tiles_i;
    const int g = t / group;
    const int first = g * p.group_j;
    const int rows = min(p.tiles_j - first, p.group_j);
    const int r = t - g * group;
    tj = first + r % rows;
    ti = r / rows;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__global__ void __launch_bounds__(K5_THREADS, 1)
    k5_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmC,
              const __grid_constant__ K5Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    // stage s: [decoded weights 16 KiB | activations 32 KiB | codes 8 KiB]
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + K5_STAGES * K5_STAGE_BYTES);
    const uint32_t full0 = smem_u32(bars);
    const uint32_t dec0 = smem_u32(bars + K5_STAGES);
    const uint32_t empty0 = smem_u32(bars + 2 * K5_STAGES);
    const uint32_t tfull0 = smem_u32(bars + 3 * K5_STAGES);
    const uint32_t tempty0 = smem_u32(bars + 3 * K5_STAGES + 2);
    const uint32_t drain = smem_u32(bars + 3 * K5_STAGES + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * K5_STAGES + 5);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < K5_STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(dec0 + 8 * s, K5_DEC_WARPS / 2);  // one decoder group per stage
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull0 + 8 * b, 1);
            mbar_init(tempty0 + 8 * b, 4);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmC);
    }
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 2 * K5_BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (elect_one()) {
            const uint64_t pol = l2_policy_evict_last();
            int stage = 0;
            uint32_t phase = 0;
            bool armed[K5_STAGES];
            uint32_t armed_parity[K5_STAGES];
            for (int s = 0; s < K5_STAGES; ++s) armed[s] = false, armed_parity[s] = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
                int tj, ti;
                k5_tile(t, p, tj, ti);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.budget_ns, p.status,
                                   KERR_TIMEOUT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = full0 + 8 * stage;
                    mbar_expect_tx(fb, K5_X_BYTES + K5_C_BYTES);
                    armed[stage] = true;
                    armed_parity[stage] = phase;
                    const uint32_t base = smem_u32(smem + stage * K5_STAGE_BYTES);
                    const int kc = kb * K5_BK;
                    tma_load_2d(base + K5_W_BYTES, &tmX, fb, kc, ti * K5_BN, pol);
                    if (p.orientation == 0)
                        tma_load_2d(base + K5_W_BYTES + K5_X_BYTES, &tmC, fb, tj * (K5_BM / 2), kc,
                                    pol);
                    else
                        tma_load_2d(base + K5_W_BYTES + K5_X_BYTES, &tmC, fb, kc / 2, tj * K5_BM,
                                    pol);
                    if (++stage == K5_STAGES) stage = 0, phase ^= 1;
                }
            }
            if (!ok)
                for (int s = 0; s < K5_STAGES; ++s)
                    if (armed[s])
                        mbar_wait(full0 + 8 * s, armed_parity[s], p.budget_ns, p.status,
                                  KERR_TIMEOUT_DRAIN);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        int stage = 0;
        uint32_t phase = 0;
        int local = 0;
        bool ok = true, issued = false;
        for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++local) {
            const int buf = local & 1;
            const uint32_t aphase = (local >> 1) & 1;
            if (!mbar_wait_warp(tempty0 + 8 * buf, aphase ^ 1, p.budget_ns, p.status,
                                KERR_TIMEOUT_MMA_ACC)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t d = tmem_base + buf * K5_BN;
            for (int kb = 0; kb < p.num_kb; ++kb) {
                if (!mbar_wait_warp(full0 + 8 * stage, phase, p.budget_ns, p.status,
                                    KERR_TIMEOUT_MMA_FULL) ||
                    !mbar_wait_warp(dec0 + 8 * stage, phase, p.budget_ns, p.status,
                                    KERR_TIMEOUT_MMA_FULL)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (elect_one()) {
                    const uint32_t sw = smem_u32(smem + stage * K5_STAGE_BYTES);
                    const uint32_t sx = sw + K5_W_BYTES;
#pragma unroll
                    for (int kk = 0; kk < K5_BK / 32; ++kk) {
                        const uint64_t ad = p.orientation == 0
                                                ? smem_desc_sw128(sw + kk * 4096, K5_BK * 128, 1024)
                                                : smem_desc_sw128(sw + kk * 32, 16, 1024);
                        const uint64_t bd = smem_desc_sw128(sx + kk * 32, 16, 1024);
                        mma_i8(d, ad, bd, p.idesc, (kb | kk) != 0);
                    }
                    mma_commit(empty0 + 8 * stage);
                    issued = true;
                }
                __syncwarp();
                if (++stage == K5_STAGES) stage = 0, phase ^= 1;
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
    } else if (warp < 6) {
        // ------------------------------------------------------------ epilogue
        const int quarter = warp & 3;
        int local = 0;
        for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++local) {
            const int buf = local & 1;
            const uint32_t aphase = (local >> 1) & 1;
            if (!mbar_wait_warp(tfull0 + 8 * buf, aphase, p.budget_ns, p.status,
                                KERR_TIMEOUT_EPILOGUE))
                break;
            tc_fence_after();
            int tj, ti;
            k5_tile(t, p, tj, ti);
            const int j = tj * K5_BM + quarter * 32 + lane;
            const bool j_ok = j < p.n;
#pragma unroll 1
            for (int cc = 0; cc < K5_BN / 32; ++cc) {
                uint32_t r[32];
                const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                       buf * K5_BN + cc * 32;
                __syncwarp();
                tmem_ld32(taddr, r);
                tmem_ld_wait();
                const int i0 = ti * K5_BN + cc * 32;
                if (j_ok && i0 < p.m) {
                    const int lim = min(32, p.m - i0);
#pragma unroll
                    for (int x = 0; x < 32; ++x) {
                        if (x < lim) {
                            const int64_t off = static_cast<int64_t>(i0 + x) * p.rsc +
                                                static_cast<int64_t>(j) * p.csc;
                            if (p.fast) static_cast<int32_t*>(p.c)[off] = static_cast<int32_t>(r[x]);
                            else finish_cell(p.epi, p.c, off, static_cast<int32_t>(r[x]));
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty0 + 8 * buf);
        }
    } else {
        // ------------------------------------------------------------ decoders
        // Two groups of K5_DEC_WARPS / 2 warps take alternate stages, so two stages are
        // decoded at once while the MMA consumes a third.
        constexpr int GW = K5_DEC_WARPS / 2;
        const int grp = (warp - 6) / GW;
        const int dt = threadIdx.x - (6 + grp * GW) * 32;  // 0 .. 32 * GW - 1
        const uint32_t t0 = p.table[0], t1 = p.table[1], t2 = p.table[2], t3 = p.table[3];
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        int it = 0;
        for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
            for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
                if ((it & 1) == grp) {
                    if (!mbar_wait_warp(full0 + 8 * stage, phase, p.budget_ns, p.status,
                                        KERR_TIMEOUT_MMA_FULL)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sw = smem + stage * K5_STAGE_BYTES;
                    const uint8_t* sc = sw + K5_W_BYTES + K5_X_BYTES;
                    // 128 code rows x 8 groups of 8 bytes; each group decodes to one
                    // swizzled 16-byte unit: row r, unit q lands at r*128 + ((q ^ (r&7)) * 16).
#pragma unroll
                    for (int rep = 0; rep < (128 * 8) / (32 * GW); ++rep) {
                        const int u = dt + rep * 32 * GW;
                        const int r = u >> 3, q = u & 7;
                        const uint2 cw = *reinterpret_cast<const uint2*>(sc + r * 64 + q * 8);
                        const uint2 d0 = dec8(cw.x, t0, t1, t2, t3);
                        const uint2 d1 = dec8(cw.y, t0, t1, t2, t3);
                        const uint4 o = make_uint4(d0.x, d0.y, d1.x, d1.y);
                        *reinterpret_cast<uint4*>(sw + r * 128 + ((q ^ (r & 7)) << 4)) = o;
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(dec0 + 8 * stage);
                }
                if (++stage == K5_STAGES) stage = 0, phase ^= 1;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 2 * K5_BN);
    }
}

cudaError_t k5_launch(const CUtensorMap& tmX, const CUtensorMap& tmC, const K5Params& p, int grid,
                      cudaStream_t stream) {
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(k5_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             K5_SMEM_BYTES);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_done[dev] = true;
    }
    k5_kernel<<<grid, K5_THREADS, K5_SMEM_BYTES, stream>>>(tmX, tmC, p);
    return cudaGetLastError();
}

}  // namespace uor
