// gemm_skinny.cu -- exact i8 products with a narrow side, on CUDA cores.
//
// The tensor-core kernel (K1) produces 256 columns (or 128 rows) per tile whether they
// exist or not, and a product with 16 or fewer rows or columns leaves most SMs idle. The
// reference meets the same shapes with its reduce factorization -- vector lanes on k rather
// than on the columns of C (R_I8_I32 / REDUCE_I8, crates/uor-matmul-kernels/src/spec.rs:
// 485-526) -- and with narrow panels (I8_NARROW, spec.rs:474-484). Here:
//
// * sk_reduce: out[r][v] = sum_p X[r][p] V[v][p] with X and the (at most 16) vectors V both
//   K-major; one warp per row and reduction chunk, lanes striding the chunk 16 bytes at a
//   time, four dp4a per 16 bytes and vector. Used for n <= 16 (X = A, V = B^T) and for
//   m <= 16 when B is K-major (X = B^T, V = A, the output transposed on the way out).
// * sk_cols: m <= 16 against a row-major B: each thread owns four columns, loads four rows
//   of them as words, transposes the 4 x 4 bytes with byte permutes and feeds dp4a against
//   A's four bytes (staged in shared memory).
//
// Both are HBM-bound for small m (n): the long operand is read exactly once. Exactness: a
// chunk is at most 130048 (cols) / 131056 (reduce) deep, so every s32 partial sum of s8 x s8
// products is exact (lane_depth, spec.rs:232-243); reduce_chunks folds the chunk planes in
// 64 bits and runs the Linear epilogue -- the same fold K1 uses for deep k.
#include <climits>
#include "aux.cuh"
#include "int_gemm.h"

namespace uor {

constexpr int SK_MAXV = 16;
constexpr int64_t SK_REDUCE_CHUNK_MAX = 131056;  // multiple of 16 inside one s32 lane
constexpr int SK_COLS_KT = 128;                  // A bytes per row staged per step
constexpr int64_t SK_COLS_CHUNK_MAX = 130816;    // multiple of SK_COLS_KT inside one lane
constexpr int SK_COLS_THREADS = 128;             // 4 columns each: 512 columns per block

// Where the partial sums go: chunk planes for reduce_chunks, or -- with one chunk -- the
// output itself through the Linear epilogue.
struct SkOut {
    int32_t* part;
    int out_rows, out_cols;
    bool direct;
    void* c;
    int64_t rsc, csc;
    LinearEpi epi;
};

__device__ __forceinline__ void sk_emit(const SkOut& o, int q, int i, int j, int32_t v) {
    if (o.direct)
        finish_cell(o.epi, o.c, static_cast<int64_t>(i) * o.rsc + static_cast<int64_t>(j) * o.csc, v);
    else
        o.part[(static_cast<size_t>(q) * o.out_rows + i) * o.out_cols + j] = v;
}

template <int NV>
__global__ void __launch_bounds__(128)
    sk_reduce_kernel(const int8_t* __restrict__ X, int64_t ldx, int rows,
                     const int8_t* __restrict__ V, int64_t ldv, int nv, int64_t k, int64_t kchunk,
                     SkOut o, bool swap) {
    const int q = blockIdx.y;
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const int64_t k0 = static_cast<int64_t>(q) * kchunk;
    const int64_t k1 = k0 + kchunk < k ? k0 + kchunk : k;
    const int8_t* xr = X + static_cast<int64_t>(r) * ldx;
    int acc[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) acc[v] = 0;
    const int64_t full = k0 + ((k1 - k0) & ~static_cast<int64_t>(15));
#pragma unroll 4
    for (int64_t p = k0 + lane * 16; p < full; p += 512) {
        const int4 xa = *reinterpret_cast<const int4*>(xr + p);
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            if (v < nv) {
                const int4 vb = *reinterpret_cast<const int4*>(V + v * ldv + p);
                acc[v] = __dp4a(xa.x, vb.x, acc[v]);
                acc[v] = __dp4a(xa.y, vb.y, acc[v]);
                acc[v] = __dp4a(xa.z, vb.z, acc[v]);
                acc[v] = __dp4a(xa.w, vb.w, acc[v]);
            }
        }
    }
    for (int64_t p = full + lane; p < k1; p += 32) {
        const int xv = xr[p];
#pragma unroll
        for (int v = 0; v < NV; ++v)
            if (v < nv) acc[v] += xv * static_cast<int>(V[v * ldv + p]);
    }
#pragma unroll
    for (int v = 0; v < NV; ++v) {
#pragma unroll
        for (int o = 16; o; o >>= 1) acc[v] += __shfl_xor_sync(0xffffffffu, acc[v], o);
    }
    if (lane == 0) {
#pragma unroll
        for (int v = 0; v < NV; ++v)
            if (v < nv) sk_emit(o, q, swap ? v : r, swap ? r : v, acc[v]);
    }
}

// Four rows (w0..w3) of four columns -> four columns of four rows (byte c of each word).
__device__ __forceinline__ void sk_transpose4(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3,
                                              uint32_t (&c)[4]) {
    const uint32_t a = __byte_perm(w0, w1, 0x5140), b = __byte_perm(w0, w1, 0x7362);
    const uint32_t d = __byte_perm(w2, w3, 0x5140), e = __byte_perm(w2, w3, 0x7362);
    c[0] = __byte_perm(a, d, 0x5410);
    c[1] = __byte_perm(a, d, 0x7632);
    c[2] = __byte_perm(b, e, 0x5410);
    c[3] = __byte_perm(b, e, 0x7632);
}

template <int MM>
__global__ void __launch_bounds__(SK_COLS_THREADS)
    sk_cols_kernel(const int8_t* __restrict__ A, int64_t rsa, int64_t csa, int m,
                   const int8_t* __restrict__ B, int64_t ldb, int n, int64_t k, int64_t kchunk,
                   SkOut o) {
    __shared__ __align__(16) int8_t As[MM][SK_COLS_KT + 16];
    const int q = blockIdx.y;
    const int j0 = (blockIdx.x * SK_COLS_THREADS + threadIdx.x) * 4;
    const int64_t k0 = static_cast<int64_t>(q) * kchunk;
    const int64_t k1 = k0 + kchunk < k ? k0 + kchunk : k;
    int acc[MM][4];
#pragma unroll
    for (int i = 0; i < MM; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[i][c] = 0;
    const bool full_cols = j0 + 3 < n;
    for (int64_t t0 = k0; t0 < k1; t0 += SK_COLS_KT) {
        const int kt = static_cast<int>(k1 - t0 < SK_COLS_KT ? k1 - t0 : SK_COLS_KT);
        __syncthreads();
        for (int x = threadIdx.x; x < MM * SK_COLS_KT; x += SK_COLS_THREADS) {
            const int i = x / SK_COLS_KT, pp = x - i * SK_COLS_KT;
            As[i][pp] = (i < m && pp < kt) ? A[i * rsa + (t0 + pp) * csa] : int8_t{0};
        }
        __syncthreads();
        if (j0 < n) {
            // 16 rows per step, all sixteen loads issued before any is used, and the next
            // step's sixteen issued before this step's products (two steps in flight)
            auto load16 = [&](int pp, uint32_t (&w)[16]) {
#pragma unroll
                for (int rr = 0; rr < 16; ++rr) {
                    const int8_t* row = B + (t0 + pp + rr) * ldb + j0;
                    if (pp + rr >= kt) {
                        w[rr] = 0;
                    } else if (full_cols) {
                        w[rr] = __ldg(reinterpret_cast<const unsigned int*>(row));
                    } else {
                        uint32_t v = 0;
                        for (int cc = 0; cc < 4; ++cc)
                            if (j0 + cc < n)
                                v |= static_cast<uint32_t>(static_cast<uint8_t>(row[cc])) << (8 * cc);
                        w[rr] = v;
                    }
                }
            };
            uint32_t wn[16];
            load16(0, wn);
            for (int pp = 0; pp < kt; pp += 16) {
                uint32_t w[16];
#pragma unroll
                for (int rr = 0; rr < 16; ++rr) w[rr] = wn[rr];
                if (pp + 16 < kt) load16(pp + 16, wn);
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    uint32_t col[4];
                    sk_transpose4(w[4 * g], w[4 * g + 1], w[4 * g + 2], w[4 * g + 3], col);
#pragma unroll
                    for (int i = 0; i < MM; ++i) {
                        if (i < m) {
                            const int aw = *reinterpret_cast<const int*>(&As[i][pp + 4 * g]);
#pragma unroll
                            for (int c = 0; c < 4; ++c)
                                acc[i][c] = __dp4a(aw, static_cast<int>(col[c]), acc[i][c]);
                        }
                    }
                }
            }
        }
    }
    if (j0 < n) {
#pragma unroll
        for (int i = 0; i < MM; ++i)
            if (i < m)
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    if (j0 + c < n) sk_emit(o, q, i, j0 + c, acc[i][c]);
    }
}

static int round_pow2_16(int x) { return x <= 1 ? 1 : x <= 2 ? 2 : x <= 4 ? 4 : x <= 8 ? 8 : 16; }

static bool k_major_rows(const int8_t* base, ptrdiff_t rs, ptrdiff_t cs, size_t rows, size_t k) {
    // rows of k bytes, unit stride along k, 16-byte-aligned starts
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
    if (k > 1 && cs != 1) return false;
    if (rows > 1 && (rs <= 0 || (size_t)rs < k || (rs & 15) != 0)) return false;
    return true;
}

bool i8_skinny_applies(size_t m, size_t k, size_t n) {
    return k > 0 && (n <= SK_MAXV || m <= SK_MAXV);
}

int run_i8_skinny(uor_b200_ctx* ctx, const int8_t* a, ptrdiff_t rsa, ptrdiff_t csa, const int8_t* b,
                  ptrdiff_t rsb, ptrdiff_t csb, void* c, ptrdiff_t rsc, ptrdiff_t csc, size_t m,
                  size_t k, size_t n, const LinearEpi& epi, uor_b200_route* route) {
    cudaStream_t s = ctx->stream;
    if (m > (size_t)INT_MAX / 2 || n > (size_t)INT_MAX / 2 || k > (size_t)INT_MAX / 2)
        return UOR_B200_UNSUPPORTED;
    const size_t ldk = (k + 15) / 16 * 16;
    // Which factorization, and which operands need a K-major copy.
    enum { REDUCE_A, REDUCE_BT, COLS } plan;
    if (n <= SK_MAXV) plan = REDUCE_A;
    else if (k_major_rows(b, csb, rsb, n, k)) plan = REDUCE_BT;  // B^T rows are B's columns
    else if (csb == 1 && rsb > 0 && (rsb & 3) == 0 && (reinterpret_cast<uintptr_t>(b) & 3u) == 0)
        plan = COLS;
    else plan = REDUCE_BT;  // any other B: its columns gathered into K-major rows first

    // the row operand X and the vectors V, K-major, 16-byte-aligned rows
    const int8_t *X = nullptr, *V = nullptr;
    int64_t ldx = 0, ldv = 0;
    size_t xrows = 0, nv = 0;
    size_t gx_bytes = 0, gv_bytes = 0;
    bool gather_x = false, gather_v = false;
    if (plan == REDUCE_A) {
        xrows = m, nv = n;
        gather_x = !k_major_rows(a, rsa, csa, m, k);
        gather_v = !k_major_rows(b, csb, rsb, n, k);
    } else if (plan == REDUCE_BT) {
        xrows = n, nv = m;
        gather_x = !k_major_rows(b, csb, rsb, n, k);
        gather_v = !k_major_rows(a, rsa, csa, m, k);
    }
    if (gather_x) gx_bytes = (xrows * ldk + 255) / 256 * 256;
    if (gather_v) gv_bytes = (nv * ldk + 255) / 256 * 256;

    // reduction chunks: enough blocks to cover the SMs, each chunk within one s32 lane
    int chunks;
    int64_t kchunk;
    int grid_x;
    if (plan == COLS) {
        grid_x = (int)((n + 4 * SK_COLS_THREADS - 1) / (4 * SK_COLS_THREADS));
        const int64_t max_chunks = (int64_t)((k + SK_COLS_KT - 1) / SK_COLS_KT);
        int64_t want = (8 * ctx->sm_count + grid_x - 1) / grid_x;
        const int64_t need = (int64_t)((k + SK_COLS_CHUNK_MAX - 1) / SK_COLS_CHUNK_MAX);
        want = want < max_chunks ? want : max_chunks;
        want = want > need ? want : need;
        kchunk = (((int64_t)k + want - 1) / want + SK_COLS_KT - 1) / SK_COLS_KT * SK_COLS_KT;
        chunks = (int)(((int64_t)k + kchunk - 1) / kchunk);
    } else {
        grid_x = (int)((xrows + 3) / 4);
        const int64_t max_chunks = (int64_t)((k + 511) / 512);
        int64_t want = (8 * ctx->sm_count + grid_x - 1) / grid_x;
        const int64_t need = (int64_t)((k + SK_REDUCE_CHUNK_MAX - 1) / SK_REDUCE_CHUNK_MAX);
        want = want < max_chunks ? want : max_chunks;
        want = want > need ? want : need;
        kchunk = (((int64_t)k + want - 1) / want + 15) / 16 * 16;
        chunks = (int)(((int64_t)k + kchunk - 1) / kchunk);
    }
    if (chunks > 65535) return UOR_B200_UNSUPPORTED;
    const size_t p_bytes = (size_t)chunks * m * n * sizeof(int32_t);
    int st = UOR_B200_OK;
    uint8_t* ws = static_cast<uint8_t*>(ctx_buffer(ctx, SLOT_WS, gx_bytes + gv_bytes + p_bytes + 256, &st));
    if (!ws) return st;
    int32_t* part = reinterpret_cast<int32_t*>(ws + gx_bytes + gv_bytes);

    if (plan == REDUCE_A) {
        X = a, ldx = m > 1 ? rsa : (int64_t)ldk;
        V = b, ldv = n > 1 ? csb : (int64_t)ldk;
        if (gather_x) {
            if (gather_2d(ws, ldk, a, m, k, rsa, csa, 1, s) != cudaSuccess) return UOR_B200_DEVICE_ERROR;
            X = reinterpret_cast<const int8_t*>(ws), ldx = (int64_t)ldk;
        }
        if (gather_v) {
            // B^T: row j of the copy is column j of B
            if (gather_2d(ws + gx_bytes, ldk, b, n, k, csb, rsb, 1, s) != cudaSuccess)
                return UOR_B200_DEVICE_ERROR;
            V = reinterpret_cast<const int8_t*>(ws + gx_bytes), ldv = (int64_t)ldk;
        }
    } else if (plan == REDUCE_BT) {
        X = b, ldx = n > 1 ? csb : (int64_t)ldk;
        V = a, ldv = m > 1 ? rsa : (int64_t)ldk;
        if (gather_x) {
            if (gather_2d(ws, ldk, b, n, k, csb, rsb, 1, s) != cudaSuccess) return UOR_B200_DEVICE_ERROR;
            X = reinterpret_cast<const int8_t*>(ws), ldx = (int64_t)ldk;
        }
        if (gather_v) {
            if (gather_2d(ws + gx_bytes, ldk, a, m, k, rsa, csa, 1, s) != cudaSuccess)
                return UOR_B200_DEVICE_ERROR;
            V = reinterpret_cast<const int8_t*>(ws + gx_bytes), ldv = (int64_t)ldk;
        }
    }

    SkOut o{};
    o.part = part;
    o.out_rows = (int)m;
    o.out_cols = (int)n;
    o.direct = chunks == 1;  // one chunk: the kernel runs the epilogue itself
    o.c = c;
    o.rsc = rsc;
    o.csc = csc;
    o.epi = epi;
    if (plan == COLS) {
        const dim3 grid((unsigned)grid_x, (unsigned)chunks);
        switch (round_pow2_16((int)m)) {
        case 1: sk_cols_kernel<1><<<grid, SK_COLS_THREADS, 0, s>>>(a, rsa, csa, (int)m, b, rsb, (int)n, (int64_t)k, kchunk, o); break;
        case 2: sk_cols_kernel<2><<<grid, SK_COLS_THREADS, 0, s>>>(a, rsa, csa, (int)m, b, rsb, (int)n, (int64_t)k, kchunk, o); break;
        case 4: sk_cols_kernel<4><<<grid, SK_COLS_THREADS, 0, s>>>(a, rsa, csa, (int)m, b, rsb, (int)n, (int64_t)k, kchunk, o); break;
        case 8: sk_cols_kernel<8><<<grid, SK_COLS_THREADS, 0, s>>>(a, rsa, csa, (int)m, b, rsb, (int)n, (int64_t)k, kchunk, o); break;
        default: sk_cols_kernel<16><<<grid, SK_COLS_THREADS, 0, s>>>(a, rsa, csa, (int)m, b, rsb, (int)n, (int64_t)k, kchunk, o); break;
        }
    } else {
        const dim3 grid((unsigned)grid_x, (unsigned)chunks);
        const bool swap = plan == REDUCE_BT;
        switch (round_pow2_16((int)nv)) {
        case 1: sk_reduce_kernel<1><<<grid, 128, 0, s>>>(X, ldx, (int)xrows, V, ldv, (int)nv, (int64_t)k, kchunk, o, swap); break;
        case 2: sk_reduce_kernel<2><<<grid, 128, 0, s>>>(X, ldx, (int)xrows, V, ldv, (int)nv, (int64_t)k, kchunk, o, swap); break;
        case 4: sk_reduce_kernel<4><<<grid, 128, 0, s>>>(X, ldx, (int)xrows, V, ldv, (int)nv, (int64_t)k, kchunk, o, swap); break;
        case 8: sk_reduce_kernel<8><<<grid, 128, 0, s>>>(X, ldx, (int)xrows, V, ldv, (int)nv, (int64_t)k, kchunk, o, swap); break;
        default: sk_reduce_kernel<16><<<grid, 128, 0, s>>>(X, ldx, (int)xrows, V, ldv, (int)nv, (int64_t)k, kchunk, o, swap); break;
        }
    }
    if (cudaGetLastError() != cudaSuccess) return UOR_B200_DEVICE_ERROR;
    if (route) {
        *route = uor_b200_route{};
        route->kernel = UOR_B200_KERNEL_SKINNY;
        route->tile_m = plan == COLS ? (uint32_t)m : (plan == REDUCE_A ? 1u : (uint32_t)m);
        route->tile_n = plan == COLS ? 4u * SK_COLS_THREADS : (uint32_t)(plan == REDUCE_A ? n : 1);
        route->tile_k = (uint32_t)(kchunk < UINT32_MAX ? kchunk : UINT32_MAX);
        route->k_chunks = (uint32_t)chunks;
        route->a_layout = plan == COLS ? 0u : (uint32_t)(plan == REDUCE_A ? (gather_x ? 2 : 0) : (gather_v ? 2 : 0));
        route->b_layout = plan == COLS ? 1u : (uint32_t)(plan == REDUCE_A ? (gather_v ? 2 : 0) : (gather_x ? 2 : 0));
        route->ctas = (uint32_t)(grid_x * chunks);
        route->pairs = 0;
    }
    if (o.direct) return UOR_B200_OK;
    return cuda_status(reduce_chunks(part, chunks, m, n, c, rsc, csc, epi, s));
}

}  // namespace uor
