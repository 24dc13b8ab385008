// int_gemm.cu -- the integer family's device driver: operand layout selection,
// gathers, lane-depth chunking, and the K1 launches.
//
// Mirrors gemm_packed_impl's plan (crates/uor-matmul-gemm/src/kernel.rs:566-673):
// pick the exact lane for the element type, cut the reduction where the lane
// could overflow (run_chunked_depth, kernel.rs:1431), fold the chunks into the
// wide accumulator, and run the Linear epilogue once per cell.
#include <climits>
#include "int_gemm.h"
#include "aux.cuh"
#include "gemm_i8.cuh"
#include "ptx.cuh"

namespace uor {

static inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Can a [rows x cols] byte matrix with unit stride along `cols` be described to
// TMA as dims {cols, rows} with row stride `rstride`? Returns the stride to use.
static bool tma_rows(const void* base, size_t rows, size_t cols, ptrdiff_t unit, ptrdiff_t rstride,
                     uint64_t* stride_out) {
    if (!aligned16(base)) return false;
    if (cols > 1 && unit != 1) return false;
    if (rows <= 1) {
        *stride_out = round_up(cols, 16);
        return true;
    }
    if (rstride <= 0 || (size_t)rstride < cols || (rstride & 15) != 0) return false;
    if ((uint64_t)rstride >= (1ull << 40)) return false;
    *stride_out = (uint64_t)rstride;
    return true;
}

int run_i8_gemm(uor_b200_ctx* ctx, const int8_t* a, ptrdiff_t rsa, ptrdiff_t csa,
                const int8_t* b, ptrdiff_t rsb, ptrdiff_t csb, void* c, ptrdiff_t rsc,
                ptrdiff_t csc, size_t m, size_t k, size_t n, const LinearEpi& epi,
                uor_b200_route* route) {
    cudaStream_t s = ctx->stream;
    if (route) {
        *route = uor_b200_route{};
        route->tile_m = K1_BM;
        route->tile_n = K1_BN;
        route->tile_k = K1_BK;
    }
    if (m == 0 || n == 0) return UOR_B200_OK;
    if (m > (size_t)INT_MAX / 2 || n > (size_t)INT_MAX / 2 || k > (size_t)INT_MAX / 2)
        return UOR_B200_UNSUPPORTED;
    if (k == 0) {
        if (route) route->kernel = UOR_B200_KERNEL_EPILOGUE_ONLY;
        return cuda_status(epilogue_only(c, rsc, csc, m, n, epi, s));
    }
    if (i8_skinny_applies(m, k, n)) {
        const int st = run_i8_skinny(ctx, a, rsa, csa, b, rsb, csb, c, rsc, csc, m, k, n, epi, route);
        if (st != UOR_B200_UNSUPPORTED) return st;
    }

    // ---- operand layouts
    uint64_t a_stride = 0, b_stride = 0;
    int a_layout, b_layout;
    if (tma_rows(a, m, k, csa, rsa, &a_stride)) a_layout = 0;        // K-major {k, m}
    else if (tma_rows(a, k, m, rsa, csa, &a_stride)) a_layout = 1;   // MN-major {m, k}
    else a_layout = 2;
    if (tma_rows(b, k, n, csb, rsb, &b_stride)) b_layout = 1;        // MN-major {n, k}
    else if (tma_rows(b, n, k, rsb, csb, &b_stride)) b_layout = 0;   // K-major {k, n}
    else b_layout = 2;

    const bool chunked = (int64_t)k > K1_LANE_DEPTH;
    const int chunks = chunked ? (int)((k + K1_CHUNK_K - 1) / K1_CHUNK_K) : 1;

    // ---- workspace: [gathered A | gathered B | chunk partials]
    const size_t ldk = round_up(k, 16);
    const size_t a_bytes = a_layout == 2 ? round_up(m * ldk, 256) : 0;
    const size_t b_bytes = b_layout == 2 ? round_up(n * ldk, 256) : 0;
    const size_t p_bytes = chunked ? (size_t)chunks * m * n * sizeof(int32_t) : 0;
    int st = UOR_B200_OK;
    uint8_t* ws = nullptr;
    if (a_bytes + b_bytes + p_bytes) {
        ws = static_cast<uint8_t*>(ctx_buffer(ctx, SLOT_WS, a_bytes + b_bytes + p_bytes, &st));
        if (!ws) return st;
    }
    if (a_layout == 2) {
        if (gather_2d(ws, ldk, a, m, k, rsa, csa, 1, s) != cudaSuccess) return UOR_B200_DEVICE_ERROR;
        a = reinterpret_cast<const int8_t*>(ws);
        a_stride = m <= 1 ? ldk : ldk;
        a_layout = 0;
        if (route) route->a_layout = 2;
    } else if (route) {
        route->a_layout = a_layout;
    }
    if (b_layout == 2) {
        // B^T gathered: row j of the buffer is column j of B.
        if (gather_2d(ws + a_bytes, ldk, b, n, k, csb, rsb, 1, s) != cudaSuccess)
            return UOR_B200_DEVICE_ERROR;
        b = reinterpret_cast<const int8_t*>(ws + a_bytes);
        b_stride = ldk;
        b_layout = 0;
        if (route) route->b_layout = 2;
    } else if (route) {
        route->b_layout = b_layout;
    }

    // Tiles of 256 rows on CTA pairs when there are rows to fill them; 128-row tiles
    // on single CTAs otherwise. A pair's CTAs each load 128 columns of B.
    const bool pair = m > 128;
    CUtensorMap tmA, tmB;
    bool ok = a_layout == 0 ? make_tmap_u8(&tmA, a, k, m, a_stride, 128, 128)
                            : make_tmap_u8(&tmA, a, m, k, a_stride, 128, 128);
    ok = ok && (b_layout == 0 ? make_tmap_u8(&tmB, b, k, n, b_stride, 128, pair ? 128 : 256)
                              : make_tmap_u8(&tmB, b, n, k, b_stride, 128, 128));
    if (!ok) return UOR_B200_DEVICE_ERROR;

    const int bm = pair ? 256 : K1_BM;
    K1Params p{};
    p.m = (int)m;
    p.n = (int)n;
    p.tiles_m = (int)((m + bm - 1) / bm);
    p.tiles_n = (int)((n + K1_BN - 1) / K1_BN);
    p.num_tiles = p.tiles_m * p.tiles_n;
    p.group_m = p.tiles_m < 16 ? p.tiles_m : 16;
    p.idesc = idesc_i8(bm, K1_BN, true, true, a_layout == 1, b_layout == 1);
    p.status = ctx->d_status;
    p.budget_ns = ctx->budget_ns;
    int grid = p.num_tiles < ctx->sm_count ? p.num_tiles : ctx->sm_count;
    if (pair) {
        const int mc = k1_pair_max_clusters();
        grid = 2 * (p.num_tiles < mc ? p.num_tiles : mc);
    }
    // The pair kernel writes an s32 output it can describe to TMA with bulk stores.
    CUtensorMap tmC;
    auto launch = [&](K1Params q) {
        if (!pair) return k1_launch(tmA, tmB, a_layout == 1, b_layout == 1, q, grid, s);
        const int64_t ld = q.rsc;
        q.tma_store = q.fast && aligned16(q.c) && (m == 1 || (ld > 0 && (ld & 3) == 0 &&
                                                             ld >= (int64_t)n)) &&
                      make_tmap_s32(&tmC, q.c, n, m, (uint64_t)(m == 1 ? ((n + 3) / 4 * 4) : ld) * 4,
                                    32, 32);
        return k1_pair_launch(tmA, tmB, tmC, a_layout == 1, b_layout == 1, q, s);
    };
    if (route) {
        route->kernel = UOR_B200_KERNEL_I8_TCGEN05;
        route->tile_m = (uint32_t)bm;
        route->k_chunks = (uint32_t)chunks;
        route->ctas = (uint32_t)grid;
        route->pairs = 1;
    }

    if (!chunked) {
        p.k_begin = 0;
        p.num_kb = (int)((k + K1_BK - 1) / K1_BK);
        p.c = c;
        p.rsc = rsc;
        p.csc = csc;
        p.epi = epi;
        p.fast = epi.kind == OUT_I32 && epi.alpha == 1 && epi.beta == 0 && csc == 1 &&
                 (m == 1 || (rsc > 0 && (rsc & 3) == 0)) && aligned16(c);
        return cuda_status(launch(p));
    }

    // Deep reduction: exact s32 partials per chunk, then one exact fold.
    int32_t* part = reinterpret_cast<int32_t*>(ws + a_bytes + b_bytes);
    for (int q = 0; q < chunks; ++q) {
        const size_t k0 = (size_t)q * K1_CHUNK_K;
        const size_t kl = (k - k0) < (size_t)K1_CHUNK_K ? (k - k0) : (size_t)K1_CHUNK_K;
        p.k_begin = (int)k0;
        p.num_kb = (int)((kl + K1_BK - 1) / K1_BK);
        p.c = part + (size_t)q * m * n;
        p.rsc = (ptrdiff_t)n;
        p.csc = 1;
        p.epi = LinearEpi{1, 0, MODE_NEAREST, OUT_I32};
        p.fast = (n % 4) == 0;
        cudaError_t e = launch(p);
        if (e != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    }
    return cuda_status(reduce_chunks(part, chunks, m, n, c, rsc, csc, epi, s));
}

}  // namespace uor
