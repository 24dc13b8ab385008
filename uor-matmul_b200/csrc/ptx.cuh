// ptx.cuh -- thin inline-PTX wrappers for sm_100a: mbarriers, TMA, tcgen05.
//
// Everything the warp-specialised kernels need and nothing else. Every wait on
// an mbarrier is bounded by a %globaltimer budget: on expiry the waiting thread
// records an error code in the launch's status word and the caller unwinds,
// so a broken pipeline ends the kernel instead of hanging the GPU.
#pragma once
#include <cstdint>
#include <cuda.h>

namespace uor {

// Error codes a kernel writes into its status word (first writer wins).
enum : int {
    KERR_NONE = 0,
    KERR_TIMEOUT_PRODUCER = 0x101,   // TMA producer waited too long on a free stage
    KERR_TIMEOUT_MMA_FULL = 0x102,   // MMA issuer waited too long on a loaded stage
    KERR_TIMEOUT_MMA_ACC = 0x103,    // MMA issuer waited too long on a drained accumulator
    KERR_TIMEOUT_EPILOGUE = 0x104,   // epilogue waited too long on a finished accumulator
    KERR_TIMEOUT_DRAIN = 0x105,      // teardown waited too long for copies in flight
    KERR_TIMEOUT_SELFTEST = 0x1FF,   // the self-test's deliberately unsatisfied wait
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n .reg .b32 r;\n .reg .pred p;\n elect.sync r|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(pred));
    return pred;
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ uint32_t mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok;
}

// Wait for the phase with the given parity to complete, at most budget_ns.
// Returns false (after recording `code`) when the budget runs out, or when
// another role has already recorded an error.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint64_t budget_ns,
                                          int* status, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    uint32_t spins = 0;
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((++spins & 63u) == 0) {
            if (*(volatile int*)status != 0) return false;
            if (globaltimer() - t0 > budget_ns) {
                atomicCAS(status, 0, code);
                return false;
            }
        }
    }
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the phase
// completes or about hint_ns have passed, so a role that waits long takes no issue slots
// from the warps doing the work.
__device__ __forceinline__ uint32_t mbar_try_wait_hint(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok;
}

// mbar_wait with hinted polls.
__device__ __forceinline__ bool mbar_wait_hint(uint32_t bar, uint32_t parity, uint64_t budget_ns,
                                               int* status, int code, uint32_t hint_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (true) {
        if (mbar_try_wait_hint(bar, parity, hint_ns)) return true;
        if (*(volatile int*)status != 0) return false;
        if (globaltimer() - t0 > budget_ns) {
            atomicCAS(status, 0, code);
            return false;
        }
    }
}

__device__ __forceinline__ bool mbar_wait_warp_hint(uint32_t bar, uint32_t parity, uint64_t budget_ns,
                                                    int* status, int code, uint32_t hint_ns) {
    const bool ok = mbar_wait_hint(bar, parity, budget_ns, status, code, hint_ns);
    return __all_sync(0xffffffffu, ok);
}

// The same wait, made warp-uniform: every lane polls (each gets the acquire),
// and the warp proceeds only if all lanes saw the phase complete, so a timeout
// can never split the warp ahead of a .sync.aligned instruction.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, uint64_t budget_ns,
                                               int* status, int code) {
    const bool ok = mbar_wait(bar, parity, budget_ns, status, code);
    return __all_sync(0xffffffffu, ok);
}

// Named barrier `id` over `count` threads that also ANDs a predicate across them: every
// participant gets true only if all passed true.
__device__ __forceinline__ bool bar_and_all(int id, int count, bool pred) {
    uint32_t out;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n"
        " selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(out)
        : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(count)
        : "memory");
    return out != 0;
}

// ---------------------------------------------------------------- TMA

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load into shared memory, completion counted on `bar` in bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t x, int32_t y, uint64_t cache_hint) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "l"(cache_hint)
        : "memory");
}

// L2 eviction-priority policies for the operand loads.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ---------------------------------------------------------------- tcgen05

// Allocate `ncols` TMEM columns (power of two >= 32); the base address lands in
// shared memory at `dst`. Executed by one whole warp.
__device__ __forceinline__ void tmem_alloc(uint32_t dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) x B(smem desc), integer kind, one CTA.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on `bar` when every tcgen05 op this thread issued has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
        : "memory");
}

// 32 lanes x 32 bits, 32 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a 128-byte-swizzled operand tile
// (tcgen05 "matrix descriptor"): start address, leading and stride byte offsets
// (all >> 4), descriptor version 1, layout SWIZZLE_128B (2) in bits 61-63.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;  // version (Blackwell)
    d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
    return d;
}

// Instruction descriptor for kind::i8 with a 32-bit signed accumulator.
//   bits 4-5: D format (2 = s32); 7-9: A format (1 = s8, 0 = u8); 10-12: B format;
//   15: A major (1 = MN); 16: B major; 17-22: N >> 3; 24-28: M >> 4.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n, bool a_signed, bool b_signed,
                                                bool a_mn, bool b_mn) {
    return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | ((b_signed ? 1u : 0u) << 10) |
           ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
           ((static_cast<uint32_t>(n) >> 3) << 17) | ((static_cast<uint32_t>(m) >> 4) << 24);
}

}  // namespace uor

// ---------------------------------------------------------------- CTA pairs
// Helpers for the 2-CTA (cta_group::2) kernels: a cluster of two CTAs whose tensor
// cores cooperate on one M256 tile. No TMA multicast is used anywhere.
namespace uor {

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t nclusters_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}

// The shared::cluster address of `local` (a shared::cta address) in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}

// Arrive on an mbarrier of a CTA in the cluster (address from mapa_shared).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}

// TMA load into this CTA's shared memory whose completion is counted on an mbarrier
// that may live in the peer CTA of the pair (cluster address).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int32_t x, int32_t y,
                                                 uint64_t cache_hint) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "l"(cache_hint)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// D(tmem, both CTAs) (+)= A (M/2 rows per CTA) x B (N/2 columns per CTA).
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on the barrier at the same offset in every CTA of `mask` when the pair's
// tcgen05 ops issued by this thread complete.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar, uint16_t mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(bar),
        "h"(mask)
        : "memory");
}

}  // namespace uor

// ---------------------------------------------------------------- TMA stores
namespace uor {

// Shared -> global tiled store of a box at coordinates (x, y); completion tracked by
// the issuing thread's bulk groups.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int32_t x,
                                             int32_t y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(src), "r"(x), "r"(y)
                 : "memory");
}
// The same store with an L2 eviction-priority hint (the output is written once).
__device__ __forceinline__ void tma_store_2d_hint(const CUtensorMap* map, uint32_t src, int32_t x,
                                                  int32_t y, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(src), "r"(x), "r"(y), "l"(policy)
        : "memory");
}
// 3-D tiled store (x innermost, then y, then z) with an L2 cache hint.
__device__ __forceinline__ void tma_store_3d_hint(const CUtensorMap* map, uint32_t src, int32_t x,
                                                  int32_t y, int32_t z, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3, %4}], [%1], %5;" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(src), "r"(x), "r"(y), "r"(z), "l"(policy)
        : "memory");
}
// Shared-memory copy from this CTA to a CTA of the cluster (dst and bar are shared::cluster
// addresses of the same CTA), counted in bytes on that CTA's mbarrier: an async-proxy
// completion, i.e. the same kind of event a TMA load delivers.
__device__ __forceinline__ void bulk_copy_s2c(uint32_t dst_cluster, uint32_t src, uint32_t bytes,
                                              uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            dst_cluster),
        "r"(src), "r"(bytes), "r"(bar_cluster)
        : "memory");
}
__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most N committed groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

}  // namespace uor
