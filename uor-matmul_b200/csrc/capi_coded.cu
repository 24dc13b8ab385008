// capi_coded.cu -- the codec tier's C ABI: coded_gemm (codes k x n) and the product
// of gemm_tabulated (codes n x k), over Packed<Grid<N>, P> codes, and codec_gemm over the
// fixed-width tiers (Sign, Ternary, Book, Offset).
#include <algorithm>
#include <climits>
#include <cstdlib>
#include <cstring>
#include <vector>
#include "aux.cuh"
#include "gemm_coded.cuh"
#include "gemm_i8.cuh"
#include "int_gemm.h"
#include "internal.h"
#include "staging.h"
#include "ptx.cuh"
#include "walk.cuh"

using namespace uor;

namespace {

// Decode a Packed<Grid<N>, P> coded matrix to a dense row-major int8 k x n matrix
// (used only off the on-chip paths: P = 1, N > 16 with P = 2, or code rows the TMA
// cannot read).
__global__ void decode_dense_kernel(int8_t* __restrict__ out, const uint8_t* __restrict__ codes,
                                    const int8_t* __restrict__ table, int N, int P,
                                    int orientation, int k, int n) {
    const int64_t total = static_cast<int64_t>(k) * n;
    const int bits = 8 / P;
    const unsigned mask = bits >= 8 ? 0xFFu : ((1u << bits) - 1u);
    for (GridWalk wk(static_cast<size_t>(n)); wk.idx < static_cast<size_t>(total); wk.next()) {
        const int64_t idx = static_cast<int64_t>(wk.idx);
        const int p = static_cast<int>(wk.i), j = static_cast<int>(wk.j);
        // CodedMatrix::at (matrix.rs:202-207) on the codec's own rows and columns
        const int row = orientation == 0 ? p : j, col = orientation == 0 ? j : p;
        const int cols = orientation == 0 ? n : k;
        const uint8_t code = codes[static_cast<int64_t>(row) * (cols / P) + col / P];
        const unsigned sub = (code >> (bits * (col % P))) & mask;
        out[idx] = table[sub % N];
    }
}

// Packed<Grid<N>, 2> codes decoded to dense int8 in the coded matrix's own layout: byte b
// holds elements 2b (low nibble) and 2b + 1, so the map is flat over the code bytes. Sixteen
// code bytes per thread through the 16-entry register table (dec8), 32 bytes stored.
__global__ void decode_nibbles_kernel(int8_t* __restrict__ out, const uint8_t* __restrict__ codes,
                                      size_t bytes, uint32_t t0, uint32_t t1, uint32_t t2,
                                      uint32_t t3, const int8_t* __restrict__ dtab, int N) {
    if (dtab) {  // the table in device memory: the register words table[v % N], v < 16
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            w[q] = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b)
                w[q] |= static_cast<uint32_t>(static_cast<uint8_t>(__ldg(dtab + (4 * q + b) % N))) << (8 * b);
        }
        t0 = w[0], t1 = w[1], t2 = w[2], t3 = w[3];
    }
    const size_t groups = bytes / 16;
    const size_t nt = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t tid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    // four groups in flight per thread, each load coalesced across the warp
    for (size_t g0 = tid; g0 < groups; g0 += 4 * nt) {
        uint4 w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const size_t gi = g0 + u * nt;
            w[u] = gi < groups ? __ldg(reinterpret_cast<const uint4*>(codes) + gi) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const size_t gi = g0 + u * nt;
            if (gi >= groups) break;
            const uint2 a = dec8(w[u].x, t0, t1, t2, t3), b = dec8(w[u].y, t0, t1, t2, t3);
            const uint2 c = dec8(w[u].z, t0, t1, t2, t3), d = dec8(w[u].w, t0, t1, t2, t3);
            uint4* o = reinterpret_cast<uint4*>(out + 32 * gi);
            o[0] = make_uint4(a.x, a.y, b.x, b.y);
            o[1] = make_uint4(c.x, c.y, d.x, d.y);
        }
    }
    // the last bytes % 16 code bytes, one byte per thread
    const size_t tail = bytes - 16 * groups;
    const size_t t = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    if (t < tail) {
        const uint32_t code = codes[16 * groups + t];
        const uint2 v = dec8(code, t0, t1, t2, t3);
        out[32 * groups + 2 * t] = static_cast<int8_t>(v.x & 0xFF);
        out[32 * groups + 2 * t + 1] = static_cast<int8_t>((v.x >> 8) & 0xFF);
    }
}

// K1C (gemm_coded_pair.cu) over device codes of p.epb elements per code byte, p's decode
// fields set by the caller: the activations as K1's A (K-major rows, gathered if TMA cannot
// read them as given), the codes map, 512 x 256 tiles from 512 activation rows up (each
// decoded stage serving both halves) and 256 x 256 below; fills the route. A reduction
// deeper than one s32 lane runs as exact chunks of K1_CHUNK_K (whole stages), each launch
// with its activation and code maps re-based at the chunk's first k and writing an s32
// plane, folded in 64 bits by reduce_chunks with the Linear epilogue (the analogue of
// run_chunked_depth, kernel.rs:1431).
int launch_k1c(uor_b200_ctx* ctx, K1CParams p, const Operand& A, const uint8_t* da,
               const uint8_t* dcodes, size_t m, size_t k, size_t n, int orientation, int kind,
               int64_t alpha, int64_t beta, const LinearEpi& epi, const Operand& C,
               const OutStage& cs, uor_b200_route* route) {
    cudaStream_t s = ctx->stream;
    int st = UOR_B200_OK;
    const size_t ldk = (k + 15) / 16 * 16;
    const bool a_ok = (reinterpret_cast<uintptr_t>(da) & 15u) == 0 && (k == 1 || A.cs == 1) &&
                      (m == 1 || (A.rs > 0 && (size_t)A.rs >= k && (A.rs & 15) == 0));
    const bool chunked = (int64_t)k > K1_LANE_DEPTH;
    const int chunks = chunked ? (int)((k + K1_CHUNK_K - 1) / K1_CHUNK_K) : 1;
    const size_t g_bytes = a_ok ? 0 : (m * ldk + 255) / 256 * 256;
    size_t p_bytes = 0;
    if (chunked && (__builtin_mul_overflow(m, n, &p_bytes) ||
                    __builtin_mul_overflow(p_bytes, (size_t)chunks * sizeof(int32_t), &p_bytes)))
        return UOR_B200_UNSUPPORTED;
    uint8_t* ws = nullptr;
    if (g_bytes + p_bytes) {
        ws = static_cast<uint8_t*>(ctx_buffer(ctx, SLOT_WS, g_bytes + p_bytes, &st));
        if (!ws) return st;
    }
    const uint8_t* xa = da;
    uint64_t xstride = 0;
    if (a_ok) {
        xstride = m == 1 ? ldk : (uint64_t)A.rs;
    } else {
        if (gather_2d(ws, ldk, da, m, k, A.rs, A.cs, 1, s) != cudaSuccess) return UOR_B200_DEVICE_ERROR;
        xa = ws;
        xstride = ldk;
    }
    const size_t epb = (size_t)p.epb;
    p.m = (int)m;
    p.n = (int)n;
    p.k_begin = 0;
    const bool tall = m >= 512;
    p.tiles_m = (int)((m + (tall ? 511 : 255)) / (tall ? 512 : 256));
    p.tiles_n = (int)((n + 255) / 256);
    p.num_tiles = p.tiles_m * p.tiles_n;
    p.group_m = p.tiles_m < 16 ? p.tiles_m : 16;
    p.idesc = idesc_i8(256, 256, true, true, false, orientation == 0);
    p.status = ctx->d_status;
    p.budget_ns = ctx->budget_ns;
    const int mc = k1c_max_clusters();
    route->kernel = UOR_B200_KERNEL_CODED_TCGEN05;
    route->tile_m = tall ? 512 : 256;
    route->tile_n = 256;
    route->tile_k = K1_BK;
    route->k_chunks = (uint32_t)chunks;
    route->ctas = (uint32_t)(2 * (p.num_tiles < mc ? p.num_tiles : mc));
    route->pairs = 1;
    route->a_layout = a_ok ? 0 : 2;
    route->b_layout = orientation == 0 ? 1 : 0;  // decoded on chip, never materialised
    int32_t* part = chunked ? reinterpret_cast<int32_t*>(ws + g_bytes) : nullptr;
    for (int q = 0; q < chunks; ++q) {
        const size_t k0 = (size_t)q * K1_CHUNK_K;  // a multiple of 128: every base stays aligned
        const size_t kl = chunked ? std::min((size_t)K1_CHUNK_K, k - k0) : k;
        CUtensorMap tmA, tmQ, tmO;
        bool ok = make_tmap_u8(&tmA, xa + k0, kl, m, xstride, 128, 128);
        if (orientation == 0)
            ok = ok && make_tmap_u8(&tmQ, dcodes + k0 * (n / epb), n / epb, kl, n / epb, 128 / epb, 128,
                                    false);
        else
            ok = ok && make_tmap_u8(&tmQ, dcodes + k0 / epb, kl / epb, n, k / epb, 128 / epb, 128, false);
        if (!ok) return UOR_B200_DEVICE_ERROR;
        p.num_kb = (int)((kl + K1_BK - 1) / K1_BK);
        if (chunked) {
            // this chunk's exact s32 plane, m x n row-major
            int32_t* plane = part + (size_t)q * m * n;
            p.c = plane;
            p.rsc = (int64_t)n;
            p.csc = 1;
            p.epi = LinearEpi{1, 0, MODE_NEAREST, OUT_I32};
            p.fast = 1;
            p.tma_store = n % 4 == 0 && (reinterpret_cast<uintptr_t>(plane) & 15u) == 0 &&
                          make_tmap_s32(&tmO, plane, n, m, (uint64_t)n * 4, 32, 32);
        } else {
            p.c = cs.dev_origin;
            p.rsc = C.rs;
            p.csc = C.cs;
            p.epi = epi;
            p.fast = kind == OUT_I32 && alpha == 1 && beta == 0 && C.cs == 1 &&
                     (m == 1 || (C.rs > 0 && (C.rs & 3) == 0 && (size_t)C.rs >= n)) &&
                     (reinterpret_cast<uintptr_t>(cs.dev_origin) & 15u) == 0;
            p.tma_store = p.fast && make_tmap_s32(&tmO, cs.dev_origin, n, m,
                                                  (uint64_t)(m == 1 ? (n + 3) / 4 * 4 : (size_t)C.rs) * 4,
                                                  32, 32);
        }
        if (k1c_launch(tmA, tmQ, tmO, orientation, tall, p, s) != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    }
    if (chunked && reduce_chunks(part, chunks, m, n, cs.dev_origin, C.rs, C.cs, epi, s) != cudaSuccess)
        return UOR_B200_DEVICE_ERROR;
    return UOR_B200_OK;
}

int coded_common(uor_b200_dtype out, const uor_b200_view* a, const uint8_t* codes,
                 size_t codes_len, size_t k, size_t n, uint32_t per_byte, const int8_t* table,
                 size_t table_len, const uor_b200_view_mut* c, int64_t alpha, int64_t beta,
                 const uor_b200_call* call, int orientation, bool table_on_host = false) {
    int kind;
    switch (out) {
    case UOR_B200_I8: kind = OUT_I8; break;
    case UOR_B200_I16: kind = OUT_I16; break;
    case UOR_B200_I32: kind = OUT_I32; break;
    case UOR_B200_I64: kind = OUT_I64; break;
    case UOR_B200_I128: kind = OUT_I128; break;
    default: return UOR_B200_UNSUPPORTED;
    }
    if (!a || !c) return UOR_B200_INVALID_ARGUMENT;
    const int mode = call ? (int)call->encode : MODE_NEAREST;
    if (mode < 0 || mode > 3) return UOR_B200_INVALID_ARGUMENT;
    // Packed::new (codecs.rs:166-172): P divides 8; a Grid with no entries decodes nothing.
    if (per_byte == 0 || 8 % per_byte != 0 || table_len == 0 || table_len > 256 || !table)
        return UOR_B200_INVALID_ARGUMENT;
    // CodedMatrix::new (matrix.rs:36-60): the codes describe exactly the declared shape.
    const size_t rows = orientation == 0 ? k : n, cols = orientation == 0 ? n : k;
    if (cols % per_byte != 0 || rows * (cols / per_byte) != codes_len) return UOR_B200_DOES_NOT_FIT;
    Operand A, C;
    int st;
    if ((st = place_view(a->data, a->len, a->rows, a->cols, a->rs, a->cs, 1, &A))) return st;
    if ((st = place_view(c->data, c->len, c->rows, c->cols, c->rs, c->cs, dtype_size(out), &C)))
        return st;
    // CodedTriple::new / TabulatedTriple::new: conformance, then aliasing.
    if (a->cols != k || c->rows != a->rows || c->cols != n) return UOR_B200_NONCONFORMANT;
    if (self_aliases(c->rows, c->cols, c->rs, c->cs)) return UOR_B200_OUTPUT_ALIASES;
    uor_b200_route local{};
    uor_b200_route* route = call && call->route ? call->route : &local;
    *route = uor_b200_route{};
    const size_t m = a->rows;
    if (m == 0 || n == 0) return UOR_B200_OK;
    if (m > (size_t)INT_MAX / 2 || n > (size_t)INT_MAX / 2 || k > (size_t)INT_MAX / 2)
        return UOR_B200_UNSUPPORTED;
    if (codes_len && !codes) return UOR_B200_INVALID_ARGUMENT;

    uor_b200_ctx* ctx = resolve_ctx(call, &st);
    if (!ctx) return st;
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceTurn turn(ctx);
    const bool dev = call && (call->flags & UOR_B200_DEVICE_POINTERS);
    cudaStream_t s = ctx->stream;

    const uint8_t* da = nullptr;
    OutStage cs;
    if ((st = stage_in(ctx, SLOT_A, A, dev, &da))) return st;
    const uint8_t* dcodes = codes;
    if (!dev && codes_len) {
        uint8_t* d = static_cast<uint8_t*>(ctx_buffer(ctx, SLOT_B, codes_len, &st));
        if (!d) return st;
        if (cudaMemcpyAsync(d, codes, codes_len, cudaMemcpyHostToDevice, s) != cudaSuccess)
            return UOR_B200_DEVICE_ERROR;
        dcodes = d;
    }
    if ((st = stage_out_begin(ctx, C, dev, beta != 0, &cs))) return st;
    const LinearEpi epi{alpha, beta, mode, kind};

    const bool fused = per_byte == 2 && table_len <= 16 && k > 0 &&
                       (orientation == 0 ? (n % 32 == 0) : (k % 32 == 0)) &&
                       (reinterpret_cast<uintptr_t>(dcodes) & 15u) == 0;
    // K1C, K1's CTA-pair pipeline with the codes decoded into its B stages -- no dense B
    // anywhere -- with 512 x 256 tiles (each decoded stage feeding two M256 halves) from 512
    // activation rows up and 256 x 256 tiles below (configs[1] 0.099-0.104 ms against 0.117
    // for decode-once; at 32 x 8192 x 8192 0.043 ms and at 384 rows 0.046, against 0.064
    // and 0.085 for the former fused kernel that put the decoded weights on the M side).
    // Past one s32 lane it runs in exact chunks, one launch per chunk, except where those
    // launches would leave most CTA pairs idle: from 512 rows with fewer 512 x 256 tiles
    // than resident pairs the default decodes once into a k x n workspace and runs K1's
    // chunks (1024 x 262016 x 2048: 0.80 ms against 1.20; 2048 x 262016 x 8192, 128 tiles:
    // 3.72 ms against 2.88 for K1C), unless UOR_B200_CODEC_ON_CHIP forbids the workspace.
    const bool on_chip = call && (call->flags & UOR_B200_CODEC_ON_CHIP);
    const bool shallow = (int64_t)k <= K1_LANE_DEPTH;
    const bool decode_once = fused && !shallow && !on_chip && m >= 512 &&
                             ((m + 511) / 512) * ((n + 255) / 256) < (size_t)k1c_max_clusters();
    const bool pair_fused = fused && !decode_once;
    // Four or eight sub-codes per byte (Packed<Grid<N>, 4 | 8>): K1C with the byte table
    // built on chip from the N-entry table, in exact chunks past one s32 lane (code rows
    // whole 16-byte TMA strides).
    const size_t code_cols = orientation == 0 ? n : k;
    const bool byte_fused = (per_byte == 4 || per_byte == 8) && k > 0 &&
                            (code_cols / per_byte) % 16 == 0 &&
                            (reinterpret_cast<uintptr_t>(dcodes) & 15u) == 0;
    // The 16-entry effective table the fused decode uses: table[v % N]; a device table on
    // the decode-once route is read by the decode kernel itself (no host round trip).
    const bool table_in_kernel = (decode_once || pair_fused || byte_fused) && dev && !table_on_host;
    int8_t tab[256];
    const size_t tl = table_len < 256 ? table_len : 256;
    if (dev && !table_on_host) {
        if (!table_in_kernel && cudaMemcpy(tab, table, tl, cudaMemcpyDeviceToHost) != cudaSuccess)
            return UOR_B200_DEVICE_ERROR;
    } else {
        std::memcpy(tab, table, tl);
    }
    if (decode_once) {
        uint8_t* dense = static_cast<uint8_t*>(ctx_buffer(ctx, SLOT_AUX, k * n + 256, &st));
        if (!dense) return st;
        uint32_t tw[4] = {0, 0, 0, 0};
        if (!table_in_kernel)
            for (int w = 0; w < 4; ++w)
                for (int bpos = 0; bpos < 4; ++bpos)
                    tw[w] |= (uint32_t)(uint8_t)tab[(4 * w + bpos) % table_len] << (8 * bpos);
        const size_t groups = codes_len / 16;
        const int grid = (int)((groups + 255) / 256 < 148 * 8 ? (groups + 255) / 256 + 1 : 148 * 8);
        decode_nibbles_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<int8_t*>(dense), dcodes, codes_len,
                                                   tw[0], tw[1], tw[2], tw[3],
                                                   table_in_kernel ? table : nullptr, (int)table_len);
        if (cudaGetLastError() != cudaSuccess) return UOR_B200_DEVICE_ERROR;
        // orientation 0: dense k x n row-major; 1: n x k row-major, i.e. B K-major
        const ptrdiff_t rsb = orientation == 0 ? (ptrdiff_t)n : 1;
        const ptrdiff_t csb = orientation == 0 ? 1 : (ptrdiff_t)k;
        st = run_i8_gemm(ctx, reinterpret_cast<const int8_t*>(da), A.rs, A.cs,
                         reinterpret_cast<const int8_t*>(dense), rsb, csb, cs.dev_origin, C.rs, C.cs,
                         m, k, n, epi, route);
        if (st) return st;
        route->kernel = UOR_B200_KERNEL_CODED_TCGEN05;
        route->b_layout = 3;  // decoded to a dense workspace first
    } else if (pair_fused) {
        K1CParams p{};
        p.epb = 2;
        if (table_in_kernel) {
            p.dtable = table;  // the decoders read the device table themselves
            p.table_len = (int)table_len;
        } else {
            for (int w = 0; w < 4; ++w) {
                uint32_t word = 0;
                for (int bpos = 0; bpos < 4; ++bpos)
                    word |= (uint32_t)(uint8_t)tab[(4 * w + bpos) % table_len] << (8 * bpos);
                p.table[w] = word;
            }
        }
        if ((st = launch_k1c(ctx, p, A, da, dcodes, m, k, n, orientation, kind, alpha, beta, epi, C,
                             cs, route)))
            return st;
    } else if (byte_fused) {
        K1CParams p{};
        p.epb = (int)per_byte;
        p.byte_tier = K1C_GRID;
        p.book_n = (int)table_len;
        if (table_in_kernel) {
            p.book = table;
        } else {
            // the first min(N, 256) entries: every sub-code is below 256
            int8_t* dt = static_cast<int8_t*>(ctx_buffer(ctx, SLOT_AUX, 256, &st));
            if (!dt) return st;
            if (cudaMemcpyAsync(dt, tab, tl, cudaMemcpyHostToDevice, s) != cudaSuccess)
                return UOR_B200_DEVICE_ERROR;
            p.book = dt;
        }
        if ((st = launch_k1c(ctx, p, A, da, dcodes, m, k, n, orientation, kind, alpha, beta, epi, C,
                             cs, route)))
            return st;
    } else {
        // Off the on-chip paths (see decode_dense_kernel): decode to a dense row-major
        // k x n int8 matrix in the auxiliary slot, then K1.
        uint8_t* buf = static_cast<uint8_t*>(ctx_buffer(ctx, SLOT_AUX, 256 + k * n, &st));
        if (!buf) return st;
        int8_t* dtable = reinterpret_cast<int8_t*>(buf);
        int8_t* dense = reinterpret_cast<int8_t*>(buf + 256);
        if (cudaMemcpyAsync(dtable, tab, tl, cudaMemcpyHostToDevice, s) != cudaSuccess)
            return UOR_B200_DEVICE_ERROR;
        if (cudaStreamSynchronize(s) != cudaSuccess) return UOR_B200_DEVICE_ERROR;
        if (k) {
            const int64_t total = (int64_t)k * n;
            const int grid = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
            decode_dense_kernel<<<grid, 256, 0, s>>>(dense, dcodes, dtable, (int)table_len,
                                                     (int)per_byte, orientation, (int)k, (int)n);
        }
        st = run_i8_gemm(ctx, reinterpret_cast<const int8_t*>(da), A.rs, A.cs, dense,
                         (ptrdiff_t)n, 1, cs.dev_origin, C.rs, C.cs, m, k, n, epi, route);
        if (st) return st;
        route->kernel = UOR_B200_KERNEL_CODED_TCGEN05;
        route->b_layout = 3;  // decoded to a dense workspace first
    }
    if ((st = stage_out_end(ctx, cs))) return st;
    if (!dev) return uor_b200_ctx_sync(ctx);
    return finish_call(ctx, call);
}

// Sign / Ternary / Book codes of `cb` bytes per block of `blk` elements (little-endian
// codes), decoded exactly as CodedMatrix::at does for a fixed-width tier (matrix.rs:202-207):
// code = codes[row * (cols / blk) + col / blk], element col % blk of it; every value minus
// `zero` (Offset, codecs.rs: decode - zero). One thread per code writes the code's blk
// elements, in the coded matrix's own rows x cols layout, four bytes to a store.
__device__ __forceinline__ int decode_elem(int tier, uint32_t code, int t, int cb,
                                           const int8_t* __restrict__ row) {
    if (tier == UOR_B200_TIER_SIGN)  // bit t set: +1; clear, or past the code's width: -1
        return (t < 8 * cb && ((code >> t) & 1u)) ? 1 : -1;
    if (tier == UOR_B200_TIER_TERNARY) {
        // digit t: 0 -> -1, 2 -> +1, 1 and 3 -> 0; a digit past the code's width reads 0, so -1
        const uint32_t d = 2 * t < 8 * cb ? (code >> (2 * t)) & 3u : 0u;
        return d == 0 ? -1 : (d == 2 ? 1 : 0);
    }
    return row[t];  // Book: table[code % N][t] (codecs.rs:306-308)
}

__global__ void decode_block_kernel(int8_t* __restrict__ out, const uint8_t* __restrict__ codes,
                                    const int8_t* __restrict__ table, int tier, int N, int blk,
                                    int cb, int zero, int64_t rows, int64_t cols) {
    const int64_t cpr = cols / blk;
    const int64_t total = rows * cpr;
    const bool words = (blk & 3) == 0;
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const uint8_t* cp = codes + t * cb;
        const uint32_t code = cb == 1 ? cp[0] : (static_cast<uint32_t>(cp[0]) | (static_cast<uint32_t>(cp[1]) << 8));
        const int8_t* brow = tier == UOR_B200_TIER_BOOK
                                 ? table + static_cast<int64_t>(code % static_cast<uint32_t>(N)) * blk
                                 : nullptr;
        int8_t* dst = out + t * blk;  // row r = t / cpr, column block t % cpr
        if (words) {
            for (int e = 0; e < blk; e += 4) {
                uint32_t w = 0;
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    w |= static_cast<uint32_t>(static_cast<uint8_t>(decode_elem(tier, code, e + q, cb, brow) - zero))
                         << (8 * q);
                *reinterpret_cast<uint32_t*>(dst + e) = w;
            }
        } else {
            for (int e = 0; e < blk; ++e)
                dst[e] = static_cast<int8_t>(decode_elem(tier, code, e, cb, brow) - zero);
        }
    }
}

// Book codes whose block is a whole number of 8-byte words, against a book already minus
// `zero`: each code's row copied word by word (the E8 codebook: one 8-byte load, one store).
__global__ void decode_book8_kernel(int8_t* __restrict__ out, const uint8_t* __restrict__ codes,
                                    const int8_t* __restrict__ table, uint32_t N, int blk, int cb,
                                    int64_t ncodes) {
    const int words = blk / 8;
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < ncodes;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const uint32_t code = cb == 1 ? codes[t]
                                      : (static_cast<uint32_t>(codes[2 * t]) | (static_cast<uint32_t>(codes[2 * t + 1]) << 8));
        const uint32_t r = code < N ? code : code % N;  // Book::decode: table[code % N]
        const uint2* src = reinterpret_cast<const uint2*>(table + static_cast<int64_t>(r) * blk);
        uint2* dst = reinterpret_cast<uint2*>(out + t * blk);
        for (int e = 0; e < words; ++e) dst[e] = __ldg(src + e);
    }
}

// The E8 shape (8-byte codewords, u8 codes, N = 256 so code % N is the code): eight codes
// per thread from one 8-byte load, their codewords from the book in shared memory, 64 bytes
// stored. ncodes % 8 == 0.
__global__ void decode_book8_u8_kernel(int8_t* __restrict__ out, const uint8_t* __restrict__ codes,
                                       const int8_t* __restrict__ table, int64_t ncodes) {
    __shared__ uint2 book[256];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) book[i] = __ldg(reinterpret_cast<const uint2*>(table) + i);
    __syncthreads();
    const int64_t groups = ncodes / 8;
    for (int64_t gi = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; gi < groups;
         gi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const uint2 c = __ldg(reinterpret_cast<const uint2*>(codes) + gi);
        uint4* o = reinterpret_cast<uint4*>(out + 64 * gi);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t word = q < 2 ? c.x : c.y;
            const int sh = 16 * (q & 1);
            const uint2 e0 = book[(word >> sh) & 255u], e1 = book[(word >> (sh + 8)) & 255u];
            o[q] = make_uint4(e0.x, e0.y, e1.x, e1.y);
        }
    }
}

int codec_common(uor_b200_dtype out, const uor_b200_view* a, const uor_b200_codec* codec,
                 const uint8_t* codes, size_t codes_len, size_t k, size_t n, uint32_t orientation,
                 const uor_b200_view_mut* c, int64_t alpha, int64_t beta,
                 const uor_b200_call* call) {
    if (!codec || !a || !c || orientation > 1) return UOR_B200_INVALID_ARGUMENT;
    const bool dev = call && (call->flags & UOR_B200_DEVICE_POINTERS);
    const int zero = codec->zero;
    // The decoded range of each tier, for Offset::new's bound (the image must stay i8).
    auto fits = [&](int lo, int hi) { return lo - zero >= -128 && hi - zero <= 127; };
    if (codec->tier == UOR_B200_TIER_GRID) {
        const size_t N = codec->table_len;
        if (!codec->table || N == 0 || N > 256) return UOR_B200_INVALID_ARGUMENT;
        int8_t tab[256];
        if (dev) {
            if (cudaMemcpy(tab, codec->table, N, cudaMemcpyDeviceToHost) != cudaSuccess)
                return UOR_B200_DEVICE_ERROR;
        } else {
            std::memcpy(tab, codec->table, N);
        }
        for (size_t q = 0; q < N; ++q) {
            if (!fits(tab[q], tab[q])) return UOR_B200_INVALID_ARGUMENT;
            tab[q] = static_cast<int8_t>(tab[q] - zero);
        }
        return coded_common(out, a, codes, codes_len, k, n, codec->per_byte, tab, N, c, alpha,
                            beta, call, (int)orientation, true);
    }
    const int tier = (int)codec->tier;
    const size_t blk = codec->block, cb = codec->code_bytes;
    if (tier != UOR_B200_TIER_SIGN && tier != UOR_B200_TIER_TERNARY && tier != UOR_B200_TIER_BOOK)
        return UOR_B200_UNSUPPORTED;
    if (blk == 0 || (cb != 1 && cb != 2)) return UOR_B200_INVALID_ARGUMENT;
    size_t N = 0, tbytes = 0;
    if (tier == UOR_B200_TIER_BOOK) {
        N = codec->table_len;
        if (!codec->table || N == 0 || blk > 4096 || N > (size_t{1} << 20) / blk)
            return UOR_B200_INVALID_ARGUMENT;
        tbytes = N * blk;
    } else if (!fits(-1, 1)) {
        return UOR_B200_INVALID_ARGUMENT;
    }
    int kind;
    switch (out) {
    case UOR_B200_I8: kind = OUT_I8; break;
    case UOR_B200_I16: kind = OUT_I16; break;
    case UOR_B200_I32: kind = OUT_I32; break;
    case UOR_B200_I64: kind = OUT_I64; break;
    case UOR_B200_I128: kind = OUT_I128; break;
    default: return UOR_B200_UNSUPPORTED;
    }
    const int mode = call ? (int)call->encode : MODE_NEAREST;
    if (mode < 0 || mode > 3) return UOR_B200_INVALID_ARGUMENT;
    // CodedMatrix::new (matrix.rs:36-60): whole blocks, and exactly the declared shape.
    const size_t rows = orientation == 0 ? k : n, cols = orientation == 0 ? n : k;
    if (cols % blk != 0 || rows * (cols / blk) * cb != codes_len) return UOR_B200_DOES_NOT_FIT;
    Operand A, C;
    int st;
    if ((st = place_view(a->data, a->len, a->rows, a->cols, a->rs, a->cs, 1, &A))) return st;
    if ((st = place_view(c->data, c->len, c->rows, c->cols, c->rs, c->cs, dtype_size(out), &C)))
        return st;
    if (a->cols != k || c->rows != a->rows || c->cols != n) return UOR_B200_NONCONFORMANT;
    if (self_aliases(c->rows, c->cols, c->rs, c->cs)) return UOR_B200_OUTPUT_ALIASES;
    uor_b200_route local{};
    uor_b200_route* route = call && call->route ? call->route : &local;
    *route = uor_b200_route{};
    const size_t m = a->rows;
    if (m == 0 || n == 0) return UOR_B200_OK;
    if (m > (size_t)INT_MAX / 2 || n > (size_t)INT_MAX / 2 || k > (size_t)INT_MAX / 2)
        return UOR_B200_UNSUPPORTED;
    if (codes_len && !codes) return UOR_B200_INVALID_ARGUMENT;
    std::vector<int8_t> book;
    if (tier == UOR_B200_TIER_BOOK && zero != 0) {
        // Offset's bound over the whole book (with zero 0 every i8 entry fits)
        int8_t lo = 127, hi = -128;
        book.resize(tbytes);
        if (dev) {
            if (cudaMemcpy(book.data(), codec->table, tbytes, cudaMemcpyDeviceToHost) != cudaSuccess)
                return UOR_B200_DEVICE_ERROR;
        } else {
            std::memcpy(book.data(), codec->table, tbytes);
        }
        for (int8_t v : book) lo = v < lo ? v : lo, hi = v > hi ? v : hi;
        if (!fits(lo, hi)) return UOR_B200_INVALID_ARGUMENT;
    }

    uor_b200_ctx* ctx = resolve_ctx(call, &st);
    if (!ctx) return st;
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceTurn turn(ctx);
    cudaStream_t s = ctx->stream;
    const uint8_t* da = nullptr;
    OutStage cs;
    if ((st = stage_in(ctx, SLOT_A, A, dev, &da))) return st;
    const uint8_t* dcodes = codes;
    if (!dev && codes_len) {
        uint8_t* d = static_cast<uint8_t*>(ctx_buffer(ctx, SLOT_B, codes_len, &st));
        if (!d) return st;
        if (cudaMemcpyAsync(d, codes, codes_len, cudaMemcpyHostToDevice, s) != cudaSuccess)
            return UOR_B200_DEVICE_ERROR;
        dcodes = d;
    }
    if ((st = stage_out_begin(ctx, C, dev, beta != 0, &cs))) return st;
    const LinearEpi epi{alpha, beta, mode, kind};
    // Code bytes of 4 or 8 whole elements each (Book with one-byte codes and blocks of 4 or
    // 8, Sign with 8 elements per code byte, Ternary with 4): K1C decodes them through a
    // 256-entry byte table it builds in shared memory, in exact chunks past one s32 lane,
    // so no dense B exists anywhere. The code rows must be whole 16-byte TMA strides.
    int epb = 0, btier = K1C_BOOK;
    if (tier == UOR_B200_TIER_BOOK && cb == 1 && (blk == 4 || blk == 8)) epb = (int)blk;
    else if (tier == UOR_B200_TIER_SIGN && blk == 8 * cb) epb = 8, btier = K1C_SIGN;
    else if (tier == UOR_B200_TIER_TERNARY && blk == 4 * cb) epb = 4, btier = K1C_TERNARY;
    const bool chip = epb != 0 && k > 0 && (cols / epb) % 16 == 0 &&
                      (reinterpret_cast<uintptr_t>(dcodes) & 15u) == 0;
    if (chip) {
        K1CParams p{};
        p.epb = epb;
        p.byte_tier = btier;
        p.zero = zero;
        if (tier == UOR_B200_TIER_BOOK) {
            p.book = reinterpret_cast<const int8_t*>(codec->table);  // read by the kernel
            p.book_n = (int)N;
            if (!dev) {
                uint8_t* db = static_cast<uint8_t*>(ctx_buffer(ctx, SLOT_AUX, (tbytes + 255) / 256 * 256, &st));
                if (!db) return st;
                if (cudaMemcpyAsync(db, codec->table, tbytes, cudaMemcpyHostToDevice, s) != cudaSuccess)
                    return UOR_B200_DEVICE_ERROR;
                p.book = reinterpret_cast<const int8_t*>(db);
            }
        }
        if ((st = launch_k1c(ctx, p, A, da, dcodes, m, k, n, (int)orientation, kind, alpha, beta, epi,
                             C, cs, route)))
            return st;
        if (!dev && tbytes && (st = uor_b200_ctx_sync(ctx))) return st;  // the host book was read
        if ((st = stage_out_end(ctx, cs))) return st;
        if (!dev) return uor_b200_ctx_sync(ctx);
        return finish_call(ctx, call);
    }
    const size_t tb = (tbytes + 255) / 256 * 256;
    uint8_t* buf = static_cast<uint8_t*>(ctx_buffer(ctx, SLOT_AUX, tb + k * n + 256, &st));
    if (!buf) return st;
    const int8_t* dtable = nullptr;
    // Books of whole 8-byte words take the word-copy decode from the book minus zero.
    const bool book8 = tier == UOR_B200_TIER_BOOK && blk % 8 == 0;
    if (book8 && zero != 0) {
        for (auto& v : book) v = static_cast<int8_t>(v - zero);
        if (cudaMemcpyAsync(buf, book.data(), tbytes, cudaMemcpyHostToDevice, s) != cudaSuccess)
            return UOR_B200_DEVICE_ERROR;
        dtable = reinterpret_cast<const int8_t*>(buf);
    } else if (tbytes) {
        if (cudaMemcpyAsync(buf, codec->table, tbytes,
                            dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s) != cudaSuccess)
            return UOR_B200_DEVICE_ERROR;
        dtable = reinterpret_cast<const int8_t*>(buf);
    }
    int8_t* dense = reinterpret_cast<int8_t*>(buf + tb);
    if (k && book8) {
        const int64_t ncodes = (int64_t)rows * (int64_t)(cols / blk);
        const int grid = (int)((ncodes + 255) / 256 < 148 * 16 ? (ncodes + 255) / 256 : 148 * 16);
        if (blk == 8 && cb == 1 && N == 256 && ncodes % 8 == 0 && (reinterpret_cast<uintptr_t>(dcodes) & 7) == 0) {
            const int64_t groups = ncodes / 8;
            const int g8 = (int)((groups + 255) / 256 < 148 * 8 ? (groups + 255) / 256 : 148 * 8);
            decode_book8_u8_kernel<<<g8, 256, 0, s>>>(dense, dcodes, dtable, ncodes);
        } else {
            decode_book8_kernel<<<grid, 256, 0, s>>>(dense, dcodes, dtable, (uint32_t)N, (int)blk, (int)cb,
                                                     ncodes);
        }
        if (cudaGetLastError() != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    } else if (k) {
        const int64_t total = (int64_t)k * n;
        const int grid = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
        // dense holds the coded matrix itself: k x n (orientation 0) or n x k (1)
        decode_block_kernel<<<grid, 256, 0, s>>>(dense, dcodes, dtable, tier, (int)N, (int)blk,
                                                 (int)cb, zero, (int64_t)rows, (int64_t)cols);
        if (cudaGetLastError() != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    }
    // B = dense (k x n row-major) or its transpose read K-major (dense n x k)
    const ptrdiff_t rsb = orientation == 0 ? (ptrdiff_t)n : 1;
    const ptrdiff_t csb = orientation == 0 ? 1 : (ptrdiff_t)k;
    st = run_i8_gemm(ctx, reinterpret_cast<const int8_t*>(da), A.rs, A.cs, dense, rsb, csb,
                     cs.dev_origin, C.rs, C.cs, m, k, n, epi, route);
    if (st) return st;
    route->kernel = UOR_B200_KERNEL_CODED_TCGEN05;
    route->b_layout = 3;  // decoded to a dense workspace first
    if (!dev && tbytes && (st = uor_b200_ctx_sync(ctx))) return st;  // the host book was read
    if ((st = stage_out_end(ctx, cs))) return st;
    if (!dev) return uor_b200_ctx_sync(ctx);
    return finish_call(ctx, call);
}

}  // namespace

extern "C" {

int uor_b200_coded_gemm(uor_b200_dtype out, const uor_b200_view* a, const uint8_t* codes,
                        size_t codes_len, size_t k, size_t n, uint32_t per_byte,
                        const int8_t* table, size_t table_len, const uor_b200_view_mut* c,
                        int64_t alpha, int64_t beta, const uor_b200_call* call) {
    return coded_common(out, a, codes, codes_len, k, n, per_byte, table, table_len, c, alpha, beta,
                        call, 0);
}

int uor_b200_tabulated_gemm(uor_b200_dtype out, const uor_b200_view* a, const uint8_t* codes,
                            size_t codes_len, size_t k, size_t n, uint32_t per_byte,
                            const int8_t* table, size_t table_len, const uor_b200_view_mut* c,
                            int64_t alpha, int64_t beta, const uor_b200_call* call) {
    return coded_common(out, a, codes, codes_len, k, n, per_byte, table, table_len, c, alpha, beta,
                        call, 1);
}

int uor_b200_codec_gemm(uor_b200_dtype out, const uor_b200_view* a, const uor_b200_codec* codec,
                        const uint8_t* codes, size_t codes_len, size_t k, size_t n,
                        uint32_t orientation, const uor_b200_view_mut* c, int64_t alpha,
                        int64_t beta, const uor_b200_call* call) {
    return codec_common(out, a, codec, codes, codes_len, k, n, orientation, c, alpha, beta, call);
}

// The E8 lattice codebook (crates/uor-matmul-codec/src/e8.rs): the lattice points
// whose coordinates lie in {0, +-1/2, +-1} -- the integer vectors of D8 (even coordinate
// sum) and the half-integer coset with an even count of negative coordinates -- scaled
// by 32 into i8, ordered by norm and then lexicographically on the scaled coordinates,
// first 256. Code 0 is the origin; codes 1..240 are the 240 minimal vectors.
int uor_b200_e8_table(uint32_t bound, int8_t* out, size_t len) {
    constexpr int kEntries = 256, kBlock = 8;
    if (bound != 0 && bound < 32) return UOR_B200_UNSUPPORTED;  // e8_table's None
    if (!out) return UOR_B200_INVALID_ARGUMENT;
    if (len < (size_t)kEntries * kBlock) return UOR_B200_DOES_NOT_FIT;
    struct Point {
        int8_t v[kBlock];
        int norm;
    };
    std::vector<Point> pts;
    pts.reserve(6561 + 256);
    for (int code = 0; code < 6561; ++code) {  // {-32, 0, 32}^8
        Point p{};
        int sum = 0, c = code;
        for (int t = kBlock - 1; t >= 0; --t, c /= 3) {
            p.v[t] = static_cast<int8_t>((c % 3 - 1) * 32);
            sum += c % 3 - 1;
            p.norm += p.v[t] * p.v[t];
        }
        if ((sum & 1) == 0) pts.push_back(p);
    }
    for (int bits = 0; bits < 256; ++bits) {  // {-16, 16}^8, an even count of -16
        if (__builtin_popcount(bits) & 1) continue;
        Point p{};
        for (int t = 0; t < kBlock; ++t) {
            p.v[t] = (bits >> (kBlock - 1 - t) & 1) ? -16 : 16;
            p.norm += 256;
        }
        pts.push_back(p);
    }
    std::stable_sort(pts.begin(), pts.end(), [](const Point& x, const Point& y) {
        if (x.norm != y.norm) return x.norm < y.norm;
        return std::lexicographical_compare(x.v, x.v + kBlock, y.v, y.v + kBlock);
    });
    for (int e = 0; e < kEntries; ++e) std::memcpy(out + e * kBlock, pts[e].v, kBlock);
    return UOR_B200_OK;
}

}  // extern "C"
