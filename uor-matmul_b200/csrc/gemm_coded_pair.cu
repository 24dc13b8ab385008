// gemm_coded_pair.cu -- K1C: the codec tier's product on CTA pairs with the codebook decode
// inside the tensor-core pipeline.
//
// Replaces coded_gemm (crates/uor-matmul-gemm/src/coded.rs:98-142) and gemm_tabulated's
// product (tabulated.rs:2555) for Packed<Grid<N>, 2> (codecs.rs:80-196) when there are
// activation rows to fill 256-row tiles: C = A decode(codes), exact s32 accumulation.
//
// It is K1's pair kernel (gemm_i8_pair.cu: 256 x 256 output tile per cluster of two
// CTAs, M256 N256 K32 tcgen05 MMAs issued by the leader, double-buffered TMEM
// accumulators, TMA-store epilogue) with the B stage produced on chip instead of loaded:
// the producer brings A (128 rows per CTA) and this CTA's 8 KiB of raw codes for 128
// weight columns; eight decoder warps per CTA expand the nibbles through the 16-entry
// codebook held in registers (dec8: byte permutes) straight into the 128-byte-swizzled
// operand layout a TMA load of a dense B would have produced, fence the writes to the
// async proxy, and arrive on the leader's dec barrier. No dense B exists anywhere: each
// code byte is read from HBM/L2 once per 256-row activation tile and decoded once per
// CTA pair tile.
//
// Orientation 0 (codes k x n, coded_gemm): B is MN-major, row r of the tile is k index r
// and its 128 bytes are 128 consecutive weight columns. Orientation 1 (codes n x k,
// gemm_tabulated's A W^T): B is K-major, row r is weight column r and its bytes are
// consecutive k. The decode and the swizzled store are the same in both: code byte b of a
// row holds elements 2b (low nibble) and 2b + 1 (high nibble); 16-byte unit q of row r is
// stored at r * 128 + ((q ^ (r & 7)) << 4).
//
// The fixed-width tiers whose code byte holds EPB = 4 or 8 whole elements (Sign, Ternary,
// Book with one-byte codes: codecs.rs:362-660, matrix.rs:202-207) take the same pipeline
// with 128 / EPB code bytes per row and stage: byte b of a row holds elements EPB b ..
// EPB b + EPB - 1, expanded through a 256-entry table of EPB bytes per code byte that the
// decoder warps build once in shared memory.
//
// Two rings. The A/B ring (KC_STAGES): TMA brings A; the decoders fill B. full[s]
// (leader) counts both CTAs' A bytes and, as the sign that both CTAs' decoded halves are in
// place, one 16-byte bulk copy from each CTA into the leader's shared memory, issued after
// the CTA's decoder warps have fenced their stores to the async proxy and met at a named
// barrier; empty[s] (each CTA) is the leader's MMA commit, multicast to the pair. The codes
// ring (KC_QSTAGES, its own producer warp) runs ahead of it: cfull[q] counts a slot's code
// bytes, cempty[q] takes one arrival per decoder warp once the slot is decoded. So every
// wait on the MMA's path completes on an async-proxy event (TMA bytes, bulk-copy bytes,
// tcgen05 commits), as in K1, and the codes' load latency is off that path.
#include <cuda_runtime.h>
#include "gemm_coded.cuh"
#include "gemm_i8.cuh"
#include "ptx.cuh"

namespace uor {

constexpr int KC_BM = 256, KC_BN = 256, KC_BK = 128;
constexpr int KC_STAGES = 5;   // A/B ring
constexpr int KC_QSTAGES = 6;  // codes ring
constexpr int KC_DEC_WARPS = 8;
// warp 0 A producer, 1 MMA, 2-5 epilogue, 6 codes producer, 7-14 decoders
constexpr int KC_DEC_WARP0 = 7;
constexpr int KC_THREADS = 32 * (KC_DEC_WARP0 + KC_DEC_WARPS);
constexpr int KC_A_BYTES = 128 * KC_BK;      // this CTA's activation rows
constexpr int KC_B_BYTES = 128 * KC_BK;      // this CTA's decoded weight columns
constexpr int KC_C_BYTES = 128 * KC_BK / 2;  // their codes
constexpr int KC_STAGE_BYTES = KC_A_BYTES + KC_B_BYTES;
constexpr int KC_EPI_BYTES = 4 * 4096;  // one 32 x 32 s32 staging block per epilogue warp
constexpr int KC_RELAY = 16;            // bytes of one decode-done signal copy
constexpr int KC_SMEM_BYTES = KC_STAGES * KC_STAGE_BYTES + KC_QSTAGES * KC_C_BYTES +
                              KC_EPI_BYTES + 1024 + 256 + 256;
static_assert(KC_SMEM_BYTES <= 232448, "K1C exceeds the opt-in shared memory per block");
static_assert(2 * (2 * KC_STAGES + 2 * KC_QSTAGES + 5) * 4 + 8 <= 256, "barrier area");

__device__ __forceinline__ void kc_tile(int t, const K1CParams& p, int& tm, int& tn) {
    const int group = p.group_m * p.tiles_n;
    const int g = t / group;
    const int first = g * p.group_m;
    const int rows = min(p.tiles_m - first, p.group_m);
    const int r = t - g * group;
    tm = first + r % rows;
    tn = r / rows;
}

// Byte tiers (EPB 4 or 8 elements per code byte): the decoded elements of every code byte
// b, the first in the lowest byte, minus zero, as table[b * EPB + t]. Built once by the
// decoder warps (dt = 0 .. 32 * KC_DEC_WARPS - 1), which then meet at named barrier 3.
template <int EPB>
__device__ void kc_build_byte_table(uint8_t* tab, const K1CParams& p, int dt) {
    for (int e = dt; e < 256 * EPB; e += 32 * KC_DEC_WARPS) {
        const int b = e / EPB, t = e % EPB;
        int v;
        if (p.byte_tier == K1C_BOOK) {
            v = p.book[static_cast<int64_t>(b % p.book_n) * EPB + t];  // Book: table[code % N]
        } else if (p.byte_tier == K1C_GRID) {
            // Packed<Grid<N>, EPB>: sub-code t is bits (8 / EPB) t .. of the byte, low first
            constexpr int BITS = 8 / EPB;
            v = p.book[((b >> (BITS * t)) & ((1 << BITS) - 1)) % p.book_n];
        } else if (p.byte_tier == K1C_SIGN) {
            v = (b >> t) & 1 ? 1 : -1;
        } else {
            const int d = (b >> (2 * t)) & 3;
            v = d == 0 ? -1 : (d == 2 ? 1 : 0);
        }
        tab[e] = static_cast<uint8_t>(v - p.zero);
    }
    asm volatile("bar.sync 3, %0;" ::"r"(32 * KC_DEC_WARPS) : "memory");
}

// The code bytes of 16-byte unit u (operand row u / 8, column group u % 8) of a codes slot
// holding 128 / EPB bytes per row.
template <int EPB>
__device__ __forceinline__ uint32_t kc_byte_codes(const uint8_t* sq, int u) {
    constexpr int QROW = 128 / EPB;
    if constexpr (EPB == 8)
        return *reinterpret_cast<const uint16_t*>(sq + (u >> 3) * QROW + (u & 7) * 2);
    else
        return *reinterpret_cast<const uint32_t*>(sq + (u >> 3) * QROW + (u & 7) * 4);
}

// Those code bytes decoded: sixteen operand bytes.
template <int EPB>
__device__ __forceinline__ uint4 kc_byte_unit(uint32_t c, const uint8_t* tab) {
    if constexpr (EPB == 8) {
        const uint2* t8 = reinterpret_cast<const uint2*>(tab);
        const uint2 e0 = t8[c & 255u], e1 = t8[(c >> 8) & 255u];
        return make_uint4(e0.x, e0.y, e1.x, e1.y);
    } else {
        const uint32_t* t4 = reinterpret_cast<const uint32_t*>(tab);
        return make_uint4(t4[c & 255u], t4[(c >> 8) & 255u], t4[(c >> 16) & 255u], t4[c >> 24]);
    }
}

template <bool B_MN, int EPB>
__global__ void __launch_bounds__(KC_THREADS, 1)
    k1c_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmQ,
                    const __grid_constant__ CUtensorMap tmC, const K1CParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* codes = smem + KC_STAGES * KC_STAGE_BYTES;             // 1 KiB aligned
    uint8_t* epi_smem = codes + KC_QSTAGES * KC_C_BYTES;             // 1 KiB aligned
    uint64_t* bars = reinterpret_cast<uint64_t*>(epi_smem + KC_EPI_BYTES);
    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + KC_STAGES);
    const uint32_t cfull0 = smem_u32(bars + 2 * KC_STAGES);
    const uint32_t cempty0 = smem_u32(bars + 2 * KC_STAGES + KC_QSTAGES);
    const uint32_t tfull0 = smem_u32(bars + 2 * KC_STAGES + 2 * KC_QSTAGES);
    const uint32_t tempty0 = tfull0 + 16;
    const uint32_t drain = tfull0 + 32;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * KC_STAGES + 2 * KC_QSTAGES + 5);
    // decode-done signals: a 16-byte source, and per stage and rank a 16-byte landing slot
    // in the leader
    const uint32_t relay_src = smem_u32(reinterpret_cast<uint8_t*>(bars) + 256);
    const uint32_t relay_dst0 = relay_src + KC_RELAY;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cid = static_cast<int>(cluster_id_x());
    const int ncl = static_cast<int>(nclusters_x());

    if (threadIdx.x == 0) {
        for (int s = 0; s < KC_STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int q = 0; q < KC_QSTAGES; ++q) {
            mbar_init(cfull0 + 8 * q, 1);
            mbar_init(cempty0 + 8 * q, KC_DEC_WARPS / 2);  // the decoder group of that step
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull0 + 8 * b, 1);
            mbar_init(tempty0 + 8 * b, 8);  // 4 epilogue warps in each CTA of the pair
        }
        mbar_init(drain, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmQ);
        if (p.tma_store) tma_prefetch_desc(&tmC);
    }
    if (warp == 1) tmem_alloc_pair(smem_u32(tmem_slot), 2 * KC_BN);
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers exist before either signals the other
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ A producer (both CTAs)
        if (elect_one()) {
            const uint64_t pol = l2_policy_evict_last();
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            bool armed[KC_STAGES];
            uint32_t armed_parity[KC_STAGES];
            for (int s = 0; s < KC_STAGES; ++s) armed[s] = false, armed_parity[s] = 0;
            for (int t = cid; t < p.num_tiles && ok; t += ncl) {
                int tm, tn;
                kc_tile(t, p, tm, tn);
                const int row0 = tm * KC_BM + static_cast<int>(rank) * 128;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.budget_ns, p.status,
                                   KERR_TIMEOUT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb_local = full0 + 8 * stage;
                    if (leader) {
                        mbar_expect_tx(fb_local, 2 * KC_A_BYTES + 2 * KC_RELAY);
                        armed[stage] = true;
                        armed_parity[stage] = phase;
                    }
                    tma_load_2d_pair(smem_u32(smem + stage * KC_STAGE_BYTES), &tmA,
                                     mapa_shared(fb_local, 0), kb * KC_BK, row0, pol);
                    if (++stage == KC_STAGES) stage = 0, phase ^= 1;
                }
            }
            if (!ok && leader)
                for (int s = 0; s < KC_STAGES; ++s)
                    if (armed[s])
                        mbar_wait(full0 + 8 * s, armed_parity[s], p.budget_ns, p.status,
                                  KERR_TIMEOUT_DRAIN);
        }
        __syncwarp();
    } else if (warp == 6) {
        // ------------------------------------------------------------ codes producer (both CTAs)
        if (elect_one()) {
            const uint64_t pol = l2_policy_evict_last();
            int q = 0;
            uint32_t qph = 0;
            bool ok = true;
            bool armed[KC_QSTAGES];
            uint32_t armed_parity[KC_QSTAGES];
            for (int i = 0; i < KC_QSTAGES; ++i) armed[i] = false, armed_parity[i] = 0;
            for (int t = cid; t < p.num_tiles && ok; t += ncl) {
                int tm, tn;
                kc_tile(t, p, tm, tn);
                const int col0 = tn * KC_BN + static_cast<int>(rank) * 128;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(cempty0 + 8 * q, qph ^ 1, p.budget_ns, p.status,
                                   KERR_TIMEOUT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    const uint32_t cb = cfull0 + 8 * q;
                    mbar_expect_tx(cb, 128 * (KC_BK / EPB));  // 128 rows of 128 / EPB code bytes
                    armed[q] = true;
                    armed_parity[q] = qph;
                    const uint32_t sq = smem_u32(codes + q * KC_C_BYTES);
                    const int kc = kb * KC_BK;
                    if (B_MN) tma_load_2d(sq, &tmQ, cb, col0 / EPB, kc, pol);
                    else tma_load_2d(sq, &tmQ, cb, kc / EPB, col0, pol);
                    if (++q == KC_QSTAGES) q = 0, qph ^= 1;
                }
            }
            if (!ok)
                for (int i = 0; i < KC_QSTAGES; ++i)
                    if (armed[i])
                        mbar_wait(cfull0 + 8 * i, armed_parity[i], p.budget_ns, p.status,
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
                const uint32_t d = tmem_base + buf * KC_BN;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait_warp(full0 + 8 * stage, phase, p.budget_ns, p.status,
                                        KERR_TIMEOUT_MMA_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (elect_one()) {
                        const uint32_t sa = smem_u32(smem + stage * KC_STAGE_BYTES);
                        const uint32_t sb = sa + KC_A_BYTES;
#pragma unroll
                        for (int kk = 0; kk < KC_BK / 32; ++kk) {
                            const uint64_t ad = smem_desc_sw128(sa + kk * 32, 16, 1024);
                            const uint64_t bd = B_MN ? smem_desc_sw128(sb + kk * 4096, KC_BK * 128, 1024)
                                                     : smem_desc_sw128(sb + kk * 32, 16, 1024);
                            mma_i8_pair(d, ad, bd, idesc, (kb | kk) != 0);
                        }
                        mma_commit_pair(empty0 + 8 * stage, 0x3);
                        issued = true;
                    }
                    __syncwarp();
                    if (++stage == KC_STAGES) stage = 0, phase ^= 1;
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
    } else if (warp < 6) {
        // ------------------------------------------------------------ epilogue (both CTAs)
        const int quarter = warp & 3;
        const int row_in_tile = static_cast<int>(rank) * 128 + quarter * 32 + lane;
        uint8_t* stage_w = epi_smem + quarter * 4096;
        const uint64_t out_policy = l2_policy_evict_first();  // C is written once, never re-read
        int local = 0;
        for (int t = cid; t < p.num_tiles; t += ncl, ++local) {
            const int buf = local & 1;
            const uint32_t aphase = (local >> 1) & 1;
            if (!mbar_wait_warp(tfull0 + 8 * buf, aphase, p.budget_ns, p.status,
                                KERR_TIMEOUT_EPILOGUE))
                break;
            tc_fence_after();
            int tm, tn;
            kc_tile(t, p, tm, tn);
            const int row = tm * KC_BM + row_in_tile;
            const bool row_ok = row < p.m;
            const int wrow0 = tm * KC_BM + static_cast<int>(rank) * 128 + quarter * 32;
#pragma unroll 1
            for (int cc = 0; cc < KC_BN / 32; ++cc) {
                uint32_t r[32];
                const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                       buf * KC_BN + cc * 32;
                __syncwarp();
                tmem_ld32(taddr, r);
                tmem_ld_wait();
                if (cc == KC_BN / 32 - 1) {
                    // the accumulator is in registers: hand TMEM back before storing
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(mapa_shared(tempty0 + 8 * buf, 0));
                }
                const int col0 = tn * KC_BN + cc * 32;
                if (p.tma_store) {
                    if (wrow0 < p.m && col0 < p.n) {
                        if (lane == 0) bulk_wait_read<0>();  // the previous store has read it
                        __syncwarp();
#pragma unroll
                        for (int v = 0; v < 8; ++v)
                            *reinterpret_cast<int4*>(stage_w + lane * 128 + ((v ^ (lane & 7)) << 4)) =
                                make_int4(static_cast<int>(r[4 * v]), static_cast<int>(r[4 * v + 1]),
                                          static_cast<int>(r[4 * v + 2]),
                                          static_cast<int>(r[4 * v + 3]));
                        fence_proxy_async();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_2d_hint(&tmC, smem_u32(stage_w), col0, wrow0, out_policy);
                            bulk_commit();
                        }
                    }
                } else if (row_ok && col0 < p.n) {
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
        if (lane == 0) bulk_wait_all();  // every store has left shared memory
        __syncwarp();
    } else {
        // ------------------------------------------------------------ decoders (both CTAs)
        const int dt = threadIdx.x - KC_DEC_WARP0 * 32;  // 0 .. 32 * KC_DEC_WARPS - 1
        uint32_t tw[4] = {p.table[0], p.table[1], p.table[2], p.table[3]};
        // byte tiers: the 256-entry table in the tail of codes slot 0 (TMA fills only the
        // first 128 x 128 / EPB bytes of each slot)
        uint8_t* const btab = codes + 128 * (KC_BK / EPB);
        if constexpr (EPB != 2) kc_build_byte_table<EPB>(btab, p, dt);
        if (EPB == 2 && p.dtable) {
            // the 16-entry table table[v % N], built from the device copy of the book
            for (int w = 0; w < 4; ++w) {
                uint32_t word = 0;
                for (int b = 0; b < 4; ++b)
                    word |= static_cast<uint32_t>(static_cast<uint8_t>(
                                p.dtable[(4 * w + b) % p.table_len])) << (8 * b);
                tw[w] = word;
            }
        }
        const uint32_t t0 = tw[0], t1 = tw[1], t2 = tw[2], t3 = tw[3];
        const uint32_t full_leader = mapa_shared(full0, 0);
        const uint32_t slot_leader = mapa_shared(relay_dst0, 0) + rank * KC_RELAY;
        int stage = 0, q = 0;
        uint32_t phase = 0, qph = 0;
        bool ok = true;
        // Two groups of four warps take alternate steps, so that one group's waits, fence,
        // barrier and relay overlap the other's decode; two and not more, for the reason the
        // tall kernel's decoders give (with five A/B stages and six codes stages a group's
        // previous step still implies the use of its stage before the awaited one).
        constexpr int GW = KC_DEC_WARPS / 2;
        const int group = dt / (32 * GW);
        const int gt = dt - group * 32 * GW;
        int it = 0;
        for (int t = cid; t < p.num_tiles && ok; t += ncl) {
            for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
                if ((it & 1) == group) {
                    // this step's codes have landed and the MMA is done with the B slot
                    const bool got =
                        mbar_wait_warp(cfull0 + 8 * q, qph, p.budget_ns, p.status, KERR_TIMEOUT_MMA_FULL) &&
                        mbar_wait_warp(empty0 + 8 * stage, phase ^ 1, p.budget_ns, p.status,
                                       KERR_TIMEOUT_MMA_FULL);
                    if (got) {
                        uint8_t* sb = smem + stage * KC_STAGE_BYTES + KC_A_BYTES;
                        const uint8_t* sq = codes + q * KC_C_BYTES;
                        // all of this thread's code bytes first (loads in flight together),
                        // then the decodes and the swizzled stores: 128 code rows x 8 units,
                        // each unit 16 bytes of an operand row
                        constexpr int REPS = (128 * 8) / (32 * GW);
                        if constexpr (EPB != 2) {
                            // byte tiers: each unit's code bytes, then the table lookups
                            uint32_t cb8[REPS];
#pragma unroll
                            for (int rep = 0; rep < REPS; ++rep)
                                cb8[rep] = kc_byte_codes<EPB>(sq, gt + rep * 32 * GW);
#pragma unroll
                            for (int rep = 0; rep < REPS; ++rep) {
                                const int u = gt + rep * 32 * GW;
                                const int r = u >> 3, qq = u & 7;
                                *reinterpret_cast<uint4*>(sb + r * 128 + ((qq ^ (r & 7)) << 4)) =
                                    kc_byte_unit<EPB>(cb8[rep], btab);
                            }
                        } else {
                            uint2 cw[REPS];
#pragma unroll
                            for (int rep = 0; rep < REPS; ++rep) {
                                const int u = gt + rep * 32 * GW;
                                cw[rep] = *reinterpret_cast<const uint2*>(sq + (u >> 3) * 64 + (u & 7) * 8);
                            }
#pragma unroll
                            for (int rep = 0; rep < REPS; ++rep) {
                                const int u = gt + rep * 32 * GW;
                                const int r = u >> 3, qq = u & 7;
                                const uint2 d0 = dec8(cw[rep].x, t0, t1, t2, t3);
                                const uint2 d1 = dec8(cw[rep].y, t0, t1, t2, t3);
                                *reinterpret_cast<uint4*>(sb + r * 128 + ((qq ^ (r & 7)) << 4)) =
                                    make_uint4(d0.x, d0.y, d1.x, d1.y);
                            }
                        }
                        // the codes slot is decoded: hand it back to the codes producer
                        __syncwarp();
                        if (lane == 0) mbar_arrive(cempty0 + 8 * q);
                    }
                    fence_proxy_async();  // the tensor core (async proxy) reads these bytes
                    // every warp of the group is done with the step (or gave up: all of them
                    // reach this barrier every step of the group and leave together, so none
                    // waits on a warp that left); one thread signals the leader's full barrier
                    // with a bulk copy (an async-proxy completion)
                    if (!bar_and_all(1 + group, 32 * GW, got)) {
                        ok = false;
                        break;
                    }
                    if (gt == 0)
                        bulk_copy_s2c(slot_leader + 2 * KC_RELAY * stage, relay_src, KC_RELAY,
                                      full_leader + 8 * stage);
                }
                if (++stage == KC_STAGES) stage = 0, phase ^= 1;
                if (++q == KC_QSTAGES) q = 0, qph ^= 1;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // neither CTA leaves while the other may still signal it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, 2 * KC_BN);
    }
}

// ---------------------------------------------------------------- K1C tall: 512 x 256 tiles
// The same pipeline with each decoded B stage feeding 512 activation rows: two M256 halves
// (rows 256 h .. of the tile, CTA rank r holding rows 256 h + 128 r + [0, 128) of each)
// share the stage, so every decoded weight serves twice the products and the decode costs
// half the issue slots per MAC. Both accumulators fill TMEM (half h in columns 256 h ..),
// so there is no second buffer: the epilogue hands the halves back one at a time and the
// MMA issuer starts the next tile's first-half MMAs as soon as half 0 is free, holding the
// second-half MMAs of the stages it consumes until half 1 is free. The decoder warps work
// in two groups of four on alternate stages: each stage's chain of waits, decode, proxy
// fence, named barrier and relay is latency, not issue, and two chains in flight overlap.
constexpr int KT_BM = 512;
constexpr int KT_STAGES = 3;   // A/B ring: 2 x 16 KiB of A and 16 KiB of decoded B per CTA
constexpr int KT_QSTAGES = 4;  // codes ring
constexpr int KT_STAGE_BYTES = 2 * KC_A_BYTES + KC_B_BYTES;
constexpr int KT_EPI_BYTES = 4 * 2 * 4096;
constexpr int KT_SMEM_BYTES = KT_STAGES * KT_STAGE_BYTES + KT_QSTAGES * KC_C_BYTES +
                              KT_EPI_BYTES + 1024 + 256 + 256;
static_assert(KT_SMEM_BYTES <= 232448, "K1C tall exceeds the opt-in shared memory per block");

template <bool B_MN>
__device__ __forceinline__ void kt_issue_half(uint32_t d, uint32_t sa, uint32_t sb, uint32_t idesc, int kb) {
#pragma unroll
    for (int kk = 0; kk < KC_BK / 32; ++kk) {
        const uint64_t ad = smem_desc_sw128(sa + kk * 32, 16, 1024);
        const uint64_t bd = B_MN ? smem_desc_sw128(sb + kk * 4096, KC_BK * 128, 1024)
                                 : smem_desc_sw128(sb + kk * 32, 16, 1024);
        mma_i8_pair(d, ad, bd, idesc, (kb | kk) != 0);
    }
}

template <bool B_MN, int EPB>
__global__ void __launch_bounds__(KC_THREADS, 1)
    k1c_tall_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmQ,
                    const __grid_constant__ CUtensorMap tmC, const K1CParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* codes = smem + KT_STAGES * KT_STAGE_BYTES;
    uint8_t* epi_smem = codes + KT_QSTAGES * KC_C_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(epi_smem + KT_EPI_BYTES);
    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + KT_STAGES);
    const uint32_t cfull0 = smem_u32(bars + 2 * KT_STAGES);
    const uint32_t cempty0 = smem_u32(bars + 2 * KT_STAGES + KT_QSTAGES);
    const uint32_t tfull = smem_u32(bars + 2 * KT_STAGES + 2 * KT_QSTAGES);
    const uint32_t tempty0 = tfull + 8;  // + 8 h: half h drained
    const uint32_t drain = tfull + 24;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * KT_STAGES + 2 * KT_QSTAGES + 4);
    const uint32_t relay_src = smem_u32(reinterpret_cast<uint8_t*>(bars) + 256);
    const uint32_t relay_dst0 = relay_src + KC_RELAY;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cid = static_cast<int>(cluster_id_x());
    const int ncl = static_cast<int>(nclusters_x());

    if (threadIdx.x == 0) {
        for (int s = 0; s < KT_STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int q = 0; q < KT_QSTAGES; ++q) {
            mbar_init(cfull0 + 8 * q, 1);
            mbar_init(cempty0 + 8 * q, KC_DEC_WARPS / 2);  // the decoder group of that stage
        }
        mbar_init(tfull, 1);
        mbar_init(tempty0, 8);  // 4 epilogue warps in each CTA of the pair
        mbar_init(tempty0 + 8, 8);
        mbar_init(drain, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmQ);
        if (p.tma_store) tma_prefetch_desc(&tmC);
    }
    if (warp == 1) tmem_alloc_pair(smem_u32(tmem_slot), 2 * KC_BN);
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ A producer (both CTAs)
        if (elect_one()) {
            const uint64_t pol = l2_policy_evict_last();
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            bool armed[KT_STAGES];
            uint32_t armed_parity[KT_STAGES];
            for (int s = 0; s < KT_STAGES; ++s) armed[s] = false, armed_parity[s] = 0;
            for (int t = cid; t < p.num_tiles && ok; t += ncl) {
                int tm, tn;
                kc_tile(t, p, tm, tn);
                const int row0 = tm * KT_BM + static_cast<int>(rank) * 128;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.budget_ns, p.status,
                                   KERR_TIMEOUT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb_local = full0 + 8 * stage;
                    if (leader) {
                        mbar_expect_tx(fb_local, 4 * KC_A_BYTES + 2 * KC_RELAY);
                        armed[stage] = true;
                        armed_parity[stage] = phase;
                    }
                    const uint32_t fb = mapa_shared(fb_local, 0);
                    const uint32_t sa = smem_u32(smem + stage * KT_STAGE_BYTES);
                    tma_load_2d_pair(sa, &tmA, fb, kb * KC_BK, row0, pol);
                    tma_load_2d_pair(sa + KC_A_BYTES, &tmA, fb, kb * KC_BK, row0 + 256, pol);
                    if (++stage == KT_STAGES) stage = 0, phase ^= 1;
                }
            }
            if (!ok && leader)
                for (int s = 0; s < KT_STAGES; ++s)
                    if (armed[s])
                        mbar_wait(full0 + 8 * s, armed_parity[s], p.budget_ns, p.status,
                                  KERR_TIMEOUT_DRAIN);
        }
        __syncwarp();
    } else if (warp == 6) {
        // ------------------------------------------------------------ codes producer (both CTAs)
        if (elect_one()) {
            const uint64_t pol = l2_policy_evict_last();
            int q = 0;
            uint32_t qph = 0;
            bool ok = true;
            bool armed[KT_QSTAGES];
            uint32_t armed_parity[KT_QSTAGES];
            for (int i = 0; i < KT_QSTAGES; ++i) armed[i] = false, armed_parity[i] = 0;
            for (int t = cid; t < p.num_tiles && ok; t += ncl) {
                int tm, tn;
                kc_tile(t, p, tm, tn);
                const int col0 = tn * KC_BN + static_cast<int>(rank) * 128;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(cempty0 + 8 * q, qph ^ 1, p.budget_ns, p.status,
                                   KERR_TIMEOUT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    const uint32_t cb = cfull0 + 8 * q;
                    mbar_expect_tx(cb, 128 * (KC_BK / EPB));  // 128 rows of 128 / EPB code bytes
                    armed[q] = true;
                    armed_parity[q] = qph;
                    const uint32_t sq = smem_u32(codes + q * KC_C_BYTES);
                    const int kc = kb * KC_BK;
                    if (B_MN) tma_load_2d(sq, &tmQ, cb, col0 / EPB, kc, pol);
                    else tma_load_2d(sq, &tmQ, cb, kc / EPB, col0, pol);
                    if (++q == KT_QSTAGES) q = 0, qph ^= 1;
                }
            }
            if (!ok)
                for (int i = 0; i < KT_QSTAGES; ++i)
                    if (armed[i])
                        mbar_wait(cfull0 + 8 * i, armed_parity[i], p.budget_ns, p.status,
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
            const uint32_t d0 = tmem_base, d1 = tmem_base + 256;
            for (int t = cid; t < p.num_tiles && ok; t += ncl, ++local) {
                const uint32_t aparity = (static_cast<uint32_t>(local) & 1u) ^ 1u;
                if (!mbar_wait_warp(tempty0, aparity, p.budget_ns, p.status, KERR_TIMEOUT_MMA_ACC)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                bool h1 = false;
                int defer_n = 0, defer_stage = 0, defer_kb = 0;
                auto flush = [&]() {
                    if (elect_one()) {
                        for (int j = 0; j < defer_n; ++j) {
                            int s = defer_stage + j;
                            if (s >= KT_STAGES) s -= KT_STAGES;
                            const uint32_t sa = smem_u32(smem + s * KT_STAGE_BYTES);
                            kt_issue_half<B_MN>(d1, sa + KC_A_BYTES, sa + 2 * KC_A_BYTES, idesc,
                                                defer_kb + j);
                            mma_commit_pair(empty0 + 8 * s, 0x3);
                        }
                    }
                    __syncwarp();
                    defer_n = 0;
                };
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!h1 && defer_n == KT_STAGES) {
                        if (!mbar_wait_warp(tempty0 + 8, aparity, p.budget_ns, p.status,
                                            KERR_TIMEOUT_MMA_ACC)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        h1 = true;
                        flush();
                    }
                    if (!mbar_wait_warp(full0 + 8 * stage, phase, p.budget_ns, p.status,
                                        KERR_TIMEOUT_MMA_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (!h1) {
                        h1 = __all_sync(0xffffffffu, mbar_try_wait(tempty0 + 8, aparity) != 0);
                        if (h1) {
                            tc_fence_after();
                            flush();
                        }
                    }
                    const uint32_t sa = smem_u32(smem + stage * KT_STAGE_BYTES);
                    if (elect_one()) {
                        kt_issue_half<B_MN>(d0, sa, sa + 2 * KC_A_BYTES, idesc, kb);
                        if (h1) {
                            kt_issue_half<B_MN>(d1, sa + KC_A_BYTES, sa + 2 * KC_A_BYTES, idesc, kb);
                            mma_commit_pair(empty0 + 8 * stage, 0x3);
                        }
                        issued = true;
                    }
                    __syncwarp();
                    if (!h1) {
                        if (defer_n == 0) defer_stage = stage, defer_kb = kb;
                        ++defer_n;
                    }
                    if (++stage == KT_STAGES) stage = 0, phase ^= 1;
                }
                if (!ok) break;
                if (!h1) {
                    if (!mbar_wait_warp(tempty0 + 8, aparity, p.budget_ns, p.status,
                                        KERR_TIMEOUT_MMA_ACC)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    flush();
                }
                if (elect_one()) mma_commit_pair(tfull, 0x3);
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
    } else if (warp < 6) {
        // ------------------------------------------------------------ epilogue (both CTAs)
        const int quarter = warp & 3;
        uint8_t* stage_w = epi_smem + quarter * 2 * 4096;
        const uint64_t out_policy = l2_policy_evict_first();
        int local = 0, nstore = 0;
        for (int t = cid; t < p.num_tiles; t += ncl, ++local) {
            if (!mbar_wait_warp(tfull, static_cast<uint32_t>(local) & 1u, p.budget_ns, p.status,
                                KERR_TIMEOUT_EPILOGUE))
                break;
            tc_fence_after();
            int tm, tn;
            kc_tile(t, p, tm, tn);
#pragma unroll 1
            for (int h = 0; h < 2; ++h) {
                const int wrow0 = tm * KT_BM + h * 256 + static_cast<int>(rank) * 128 + quarter * 32;
                const int row = wrow0 + lane;
                const bool row_ok = row < p.m;
#pragma unroll 1
                for (int cc = 0; cc < KC_BN / 32; ++cc) {
                    uint32_t r[32];
                    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                           256 * h + cc * 32;
                    __syncwarp();
                    tmem_ld32(taddr, r);
                    tmem_ld_wait();
                    if (cc == KC_BN / 32 - 1) {
                        // this half is in registers: hand it back before storing
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive_cluster(mapa_shared(tempty0 + 8 * h, 0));
                    }
                    const int col0 = tn * KC_BN + cc * 32;
                    if (p.tma_store) {
                        if (wrow0 < p.m && col0 < p.n) {
                            uint8_t* sbuf = stage_w + (nstore & 1) * 4096;
                            if (lane == 0) bulk_wait_read<1>();
                            __syncwarp();
#pragma unroll
                            for (int v = 0; v < 8; ++v)
                                *reinterpret_cast<int4*>(sbuf + lane * 128 + ((v ^ (lane & 7)) << 4)) =
                                    make_int4(static_cast<int>(r[4 * v]), static_cast<int>(r[4 * v + 1]),
                                              static_cast<int>(r[4 * v + 2]),
                                              static_cast<int>(r[4 * v + 3]));
                            fence_proxy_async();
                            __syncwarp();
                            if (lane == 0) {
                                tma_store_2d_hint(&tmC, smem_u32(sbuf), col0, wrow0, out_policy);
                                bulk_commit();
                            }
                            ++nstore;
                        }
                    } else if (row_ok && col0 < p.n) {
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
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    } else {
        // ------------------------------------------------------------ decoders (both CTAs)
        const int dt = threadIdx.x - KC_DEC_WARP0 * 32;
        uint32_t tw[4] = {p.table[0], p.table[1], p.table[2], p.table[3]};
        // byte tiers: the 256-entry table in the tail of codes slot 0 (TMA fills only the
        // first 128 x 128 / EPB bytes of each slot)
        uint8_t* const btab = codes + 128 * (KC_BK / EPB);
        if constexpr (EPB != 2) kc_build_byte_table<EPB>(btab, p, dt);
        if (EPB == 2 && p.dtable) {
            for (int w = 0; w < 4; ++w) {
                uint32_t word = 0;
                for (int b = 0; b < 4; ++b)
                    word |= static_cast<uint32_t>(static_cast<uint8_t>(
                                p.dtable[(4 * w + b) % p.table_len])) << (8 * b);
                tw[w] = word;
            }
        }
        const uint32_t t0 = tw[0], t1 = tw[1], t2 = tw[2], t3 = tw[3];
        const uint32_t full_leader = mapa_shared(full0, 0);
        const uint32_t slot_leader = mapa_shared(relay_dst0, 0) + rank * KC_RELAY;
        int stage = 0, q = 0;
        uint32_t phase = 0, qph = 0;
        bool ok = true;
        // Two groups of four warps take alternate stages, so that one group's wait, fence,
        // barrier and relay overlap the other's decode. Not more than two: the waits below
        // are parity waits, which cannot tell a barrier one phase behind from one that has
        // caught up. A group reaching iteration i has finished iteration i - 2, whose wait
        // needed MMA i - 5; the MMAs commit in order, so MMA i - 6 (the use of this
        // iteration's stage before the one it waits for) is done as well, and the parity can
        // only mean the right phase. With four groups iteration i - 4 would imply only MMA
        // i - 7. The codes ring is safe the same way: an even number of codes stages makes
        // each stage's previous use the same group's.
        constexpr int GW = KC_DEC_WARPS / 2;
        const int group = dt / (32 * GW);
        const int gt = dt - group * 32 * GW;
        int it = 0;
        for (int t = cid; t < p.num_tiles && ok; t += ncl) {
            for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
                if ((it & 1) == group) {
                    const bool got =
                        mbar_wait_warp(cfull0 + 8 * q, qph, p.budget_ns, p.status, KERR_TIMEOUT_MMA_FULL) &&
                        mbar_wait_warp(empty0 + 8 * stage, phase ^ 1, p.budget_ns, p.status,
                                       KERR_TIMEOUT_MMA_FULL);
                    if (got) {
                        uint8_t* sb = smem + stage * KT_STAGE_BYTES + 2 * KC_A_BYTES;
                        const uint8_t* sq = codes + q * KC_C_BYTES;
                        constexpr int REPS = (128 * 8) / (32 * GW);
                        if constexpr (EPB != 2) {
                            // byte tiers: each unit's code bytes, then the table lookups
                            uint32_t cb8[REPS];
#pragma unroll
                            for (int rep = 0; rep < REPS; ++rep)
                                cb8[rep] = kc_byte_codes<EPB>(sq, gt + rep * 32 * GW);
#pragma unroll
                            for (int rep = 0; rep < REPS; ++rep) {
                                const int u = gt + rep * 32 * GW;
                                const int r = u >> 3, qq = u & 7;
                                *reinterpret_cast<uint4*>(sb + r * 128 + ((qq ^ (r & 7)) << 4)) =
                                    kc_byte_unit<EPB>(cb8[rep], btab);
                            }
                        } else {
                            uint2 cw[REPS];
#pragma unroll
                            for (int rep = 0; rep < REPS; ++rep) {
                                const int u = gt + rep * 32 * GW;
                                cw[rep] = *reinterpret_cast<const uint2*>(sq + (u >> 3) * 64 + (u & 7) * 8);
                            }
#pragma unroll
                            for (int rep = 0; rep < REPS; ++rep) {
                                const int u = gt + rep * 32 * GW;
                                const int r = u >> 3, qq = u & 7;
                                const uint2 e0 = dec8(cw[rep].x, t0, t1, t2, t3);
                                const uint2 e1 = dec8(cw[rep].y, t0, t1, t2, t3);
                                *reinterpret_cast<uint4*>(sb + r * 128 + ((qq ^ (r & 7)) << 4)) =
                                    make_uint4(e0.x, e0.y, e1.x, e1.y);
                            }
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(cempty0 + 8 * q);
                    }
                    fence_proxy_async();
                    if (!bar_and_all(1 + group, 32 * GW, got)) {
                        ok = false;
                        break;
                    }
                    if (gt == 0)
                        bulk_copy_s2c(slot_leader + 2 * KC_RELAY * stage, relay_src, KC_RELAY,
                                      full_leader + 8 * stage);
                }
                if (++stage == KT_STAGES) stage = 0, phase ^= 1;
                if (++q == KT_QSTAGES) q = 0, qph ^= 1;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, 2 * KC_BN);
    }
}

template <bool B_MN, bool TALL, int EPB>
static cudaError_t kc_launch_t(const CUtensorMap& tmA, const CUtensorMap& tmQ, const CUtensorMap& tmC,
                               const K1CParams& p, int max_clusters, cudaStream_t stream) {
    auto kern = TALL ? k1c_tall_kernel<B_MN, EPB> : k1c_pair_kernel<B_MN, EPB>;
    const int smem = TALL ? KT_SMEM_BYTES : KC_SMEM_BYTES;
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_done[dev] = true;
    }
    const int clusters = p.num_tiles < max_clusters ? p.num_tiles : max_clusters;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    cfg.blockDim = dim3(KC_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, tmA, tmQ, tmC, p);
}

int k1c_max_clusters() {
    static int cached[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
    auto kern = k1c_pair_kernel<true, 2>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, KC_SMEM_BYTES);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 512, 1, 1);
    cfg.blockDim = dim3(KC_THREADS, 1, 1);
    cfg.dynamicSmemBytes = KC_SMEM_BYTES;
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

template <int EPB>
static cudaError_t kc_launch_e(const CUtensorMap& tmA, const CUtensorMap& tmQ, const CUtensorMap& tmC,
                               int orientation, bool tall, const K1CParams& p, int mc, cudaStream_t stream) {
    if (tall)
        return orientation == 0 ? kc_launch_t<true, true, EPB>(tmA, tmQ, tmC, p, mc, stream)
                                : kc_launch_t<false, true, EPB>(tmA, tmQ, tmC, p, mc, stream);
    return orientation == 0 ? kc_launch_t<true, false, EPB>(tmA, tmQ, tmC, p, mc, stream)
                            : kc_launch_t<false, false, EPB>(tmA, tmQ, tmC, p, mc, stream);
}

cudaError_t k1c_launch(const CUtensorMap& tmA, const CUtensorMap& tmQ, const CUtensorMap& tmC,
                       int orientation, bool tall, const K1CParams& p, cudaStream_t stream) {
    const int mc = k1c_max_clusters();
    if (p.epb == 8) return kc_launch_e<8>(tmA, tmQ, tmC, orientation, tall, p, mc, stream);
    if (p.epb == 4) return kc_launch_e<4>(tmA, tmQ, tmC, orientation, tall, p, mc, stream);
    if (p.epb == 2) return kc_launch_e<2>(tmA, tmQ, tmC, orientation, tall, p, mc, stream);
    return cudaErrorInvalidValue;
}

}  // namespace uor
