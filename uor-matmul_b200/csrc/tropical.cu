// tropical.cu -- K4: the (max, +) product on CUDA cores.
//
// Replaces driver::gemm over Alphabet<Trop<E>, _> (crates/uor-matmul-gemm/src/driver.rs:67-182)
// whose mac is `if both finite: acc := max(acc, a + b)` (tropical.rs:311-324), followed by
// MaxPlus::finish (epilogue.rs:171-185) and the encode clamp to [MIN+1, MAX-1]
// (tropical.rs:336-351).
//
// Fast path, Trop<i8>: the operands are packed once into 16-bit lanes with the semiring
// zero as -16384 (the same idea as the reference's packed lane, kernels/src/tropical.rs:91-179,
// with a sentinel chosen so that a plain wrapping add never overflows: every finite sum is
// in [-256, 254], every sum touching -inf is at most -16384 + 127, and -inf + -inf is
// -32768). Then one fused add-max per 16x2 pair (__viaddmax_s16x2: max(a + b, acc),
// wrapping add) evaluates two terms per instruction, register-blocked 8x8 per thread
// over 128x128 tiles staged through shared memory with cp.async.
// Any result below -8192 decodes to -inf.
#include <cuda_runtime.h>
#include <climits>
#include "tropical.cuh"
#include "walk.cuh"

namespace uor {

constexpr int TR_BM = 128, TR_BN = 128, TR_BK = 32, TR_THREADS = 256;
constexpr int TR_ZERO16 = -16384;

__device__ __forceinline__ uint32_t dup16(int v) {
    const uint32_t u = static_cast<uint16_t>(static_cast<int16_t>(v));
    return u | (u << 16);
}

// Trop<E> load: repr(C) {E value; bool finite} at element index `idx`.
__device__ __forceinline__ bool trop_load(const uint8_t* base, int ebytes, int64_t idx, i128* v) {
    const uint8_t* e = base + idx * (ebytes == 1 ? 2 : ebytes == 2 ? 4 : ebytes == 4 ? 8 : 16);
    int64_t x;
    switch (ebytes) {
    case 1: x = static_cast<int8_t>(e[0]); break;
    case 2: x = *reinterpret_cast<const int16_t*>(e); break;
    case 4: x = *reinterpret_cast<const int32_t*>(e); break;
    default: x = *reinterpret_cast<const int64_t*>(e); break;
    }
    *v = x;
    return e[ebytes] != 0;
}

__device__ __forceinline__ void trop_store(uint8_t* base, int obytes, int64_t idx, bool fin, i128 v) {
    const int64_t x = fin ? static_cast<int64_t>(v) : 0;  // the semiring zero stores E::ZERO
    switch (obytes) {
    case 1:
        reinterpret_cast<uint16_t*>(base)[idx] =
            static_cast<uint16_t>(static_cast<uint8_t>(x) | (fin ? 0x100u : 0u));
        break;
    case 2:
        reinterpret_cast<uint32_t*>(base)[idx] =
            static_cast<uint32_t>(static_cast<uint16_t>(x)) | (fin ? 0x10000u : 0u);
        break;
    case 4:
        reinterpret_cast<uint64_t*>(base)[idx] =
            static_cast<uint64_t>(static_cast<uint32_t>(x)) | (fin ? (1ull << 32) : 0ull);
        break;
    default: {
        uint64_t* p = reinterpret_cast<uint64_t*>(base) + 2 * idx;
        p[0] = static_cast<uint64_t>(x);
        p[1] = fin ? 1ull : 0ull;
    }
    }
}

// MaxPlus::finish + the tropical encode, for one cell whose reduction is (fin, v).
__device__ __forceinline__ void trop_finish(const TropEpi& e, int64_t off, bool fin, i128 v) {
    if (e.obytes == 0) {
        // split-K key: the raw reduction of this range, the semiring zero as INT64_MIN
        static_cast<int64_t*>(e.c)[off] = fin ? static_cast<int64_t>(v) : INT64_MIN;
        return;
    }
    // alpha (x) acc: -inf absorbs (ShiftExact, epilogue.rs:199-215)
    bool f = fin && e.alpha_finite;
    i128 t = f ? v + static_cast<i128>(e.alpha) : 0;
    if (e.beta_finite) {
        i128 pv;
        if (trop_load(static_cast<const uint8_t*>(e.c), e.obytes, off, &pv)) {
            const i128 s = pv + static_cast<i128>(e.beta);
            if (!f || s > t) t = s, f = true;
        }
    }
    if (f) {
        // encode_i128_into(v, MIN+1, MAX-1, mode)
        const int bits = 8 * e.obytes;
        const i128 mx = (static_cast<i128>(1) << (bits - 1)) - 2;  // MAX - 1
        const i128 mn = -mx - 1;                                     // MIN + 1
        if (e.mode == MODE_WRAPPING) {
            // The reference's arithmetic exactly (acc.rs:128-151): u128 wrapping
            // subtraction, remainder by the span (2^w - 2, not a power of two, so a
            // negative accumulator does not reduce as a true modulus), wrapping add.
            const u128 span = static_cast<u128>(mx) - static_cast<u128>(mn) + 1;
            const u128 off = static_cast<u128>(t) - static_cast<u128>(mn);
            t = static_cast<i128>(off % span + static_cast<u128>(mn));
        } else {
            t = t < mn ? mn : (t > mx ? mx : t);
        }
    }
    trop_store(static_cast<uint8_t*>(e.c), e.obytes, off, f, t);
}

// ------------------------------------------------------------ packing

__global__ void trop_pack_a_kernel(uint32_t* __restrict__ at, int mp, int kp,
                                   const uint8_t* __restrict__ a, int64_t rsa, int64_t csa, int m,
                                   int k) {
    const int64_t total = static_cast<int64_t>(mp) * kp;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int p = static_cast<int>(idx / mp), i = static_cast<int>(idx % mp);
        int v = TR_ZERO16;
        if (i < m && p < k) {
            const uint8_t* e = a + (static_cast<int64_t>(i) * rsa + static_cast<int64_t>(p) * csa) * 2;
            if (e[1]) v = static_cast<int8_t>(e[0]);
        }
        at[idx] = dup16(v);
    }
}

__global__ void trop_pack_b_kernel(int16_t* __restrict__ bt, int np, int kp,
                                   const uint8_t* __restrict__ b, int64_t rsb, int64_t csb, int k,
                                   int n) {
    const int64_t total = static_cast<int64_t>(np) * kp;
    for (GridWalk wk(static_cast<size_t>(np)); wk.idx < static_cast<size_t>(total); wk.next()) {
        const int64_t idx = static_cast<int64_t>(wk.idx);
        const int p = static_cast<int>(wk.i), j = static_cast<int>(wk.j);
        int v = TR_ZERO16;
        if (j < n && p < k) {
            const uint8_t* e = b + (static_cast<int64_t>(p) * rsb + static_cast<int64_t>(j) * csb) * 2;
            if (e[1]) v = static_cast<int8_t>(e[0]);
        }
        bt[idx] = static_cast<int16_t>(v);
    }
}

// ------------------------------------------------------------ main kernel

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(TR_THREADS)
    trop_i8_kernel(const uint32_t* __restrict__ at, const int16_t* __restrict__ bt, int mp, int np,
                   int kp, TropEpi e) {
    __shared__ __align__(16) uint32_t As[2][TR_BK][TR_BM];  // 32 KiB
    __shared__ __align__(16) int16_t Bs[2][TR_BK][TR_BN];   // 16 KiB
    const int t = threadIdx.x;
    const int m0 = blockIdx.y * TR_BM, n0 = blockIdx.x * TR_BN;
    const int ty = t >> 4, tx = t & 15;

    auto load_tile = [&](int buf, int k0) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {  // A: 32 rows x 512 B = 1024 chunks of 16 B
            const int c = t * 4 + q, r = c >> 5, col = (c & 31) * 4;
            cp_async16(&As[buf][r][col], at + static_cast<int64_t>(k0 + r) * mp + m0 + col);
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {  // B: 32 rows x 256 B = 512 chunks of 16 B
            const int c = t * 2 + q, r = c >> 4, col = (c & 15) * 8;
            cp_async16(&Bs[buf][r][col], bt + static_cast<int64_t>(k0 + r) * np + n0 + col);
        }
        cp_async_commit();
    };

    uint32_t acc[8][4];
#pragma unroll
    for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[r][q] = dup16(-32768);

    const int tiles = kp / TR_BK;
    if (tiles > 0) load_tile(0, 0);
    for (int kt = 0; kt < tiles; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < tiles) {
            load_tile(buf ^ 1, (kt + 1) * TR_BK);
            cp_async_wait_1();
        } else {
            cp_async_wait_0();
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < TR_BK; ++kk) {
            const uint4 a0 = *reinterpret_cast<const uint4*>(&As[buf][kk][ty * 8]);
            const uint4 a1 = *reinterpret_cast<const uint4*>(&As[buf][kk][ty * 8 + 4]);
            const uint4 b = *reinterpret_cast<const uint4*>(&Bs[buf][kk][tx * 8]);
            const uint32_t av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const uint32_t bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int r = 0; r < 8; ++r)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[r][q] = __viaddmax_s16x2(av[r], bv[q], acc[r][q]);
        }
        __syncthreads();
    }

#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const int i = m0 + ty * 8 + r;
        if (i >= e.m) continue;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int j = n0 + tx * 8 + 2 * q + h;
                if (j >= e.n) continue;
                const int v = static_cast<int16_t>(h ? (acc[r][q] >> 16) : (acc[r][q] & 0xFFFF));
                const bool fin = v > -8192;
                trop_finish(e, static_cast<int64_t>(i) * e.rsc + static_cast<int64_t>(j) * e.csc, fin,
                            static_cast<i128>(v));
            }
        }
    }
}

// Any element width, exact in 128-bit arithmetic; one thread per output cell.
__global__ void trop_generic_kernel(const uint8_t* __restrict__ a, int64_t rsa, int64_t csa,
                                    const uint8_t* __restrict__ b, int64_t rsb, int64_t csb,
                                    int ebytes, int k, TropEpi e) {
    const int i = blockIdx.y * blockDim.y + threadIdx.y;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= e.m || j >= e.n) return;
    bool have = false;
    i128 best = 0;
    for (int p = 0; p < k; ++p) {
        i128 x, y;
        const bool fx = trop_load(a, ebytes, static_cast<int64_t>(i) * rsa + static_cast<int64_t>(p) * csa, &x);
        const bool fy = trop_load(b, ebytes, static_cast<int64_t>(p) * rsb + static_cast<int64_t>(j) * csb, &y);
        if (fx && fy) {
            const i128 s = x + y;
            if (!have || s > best) best = s, have = true;
        }
    }
    trop_finish(e, static_cast<int64_t>(i) * e.rsc + static_cast<int64_t>(j) * e.csc, have, best);
}

// ------------------------------------------------------------ selection witness
//
// One key per term carries both halves of D-6's order: key = (a + b) 2^16 + (65535 - p)
// for finite a, b -- a greater sum wins, and on equal sums the smaller index, exactly
// Lex::combine (selection.rs) -- so one fused add-max per term reduces value and witness
// together. A semiring zero contributes -2^30 to its side, which keeps every key it
// touches below -2^29 while every finite key lies in [-2^24, 2^24]; a cell whose best key
// is that low has no finite term, and its witness is 0 (the least index, selection.rs).
constexpr int TW_BM = 128, TW_BN = 128, TW_BK = 16, TW_THREADS = 256;
constexpr int32_t TW_ZERO = -(1 << 30);

__global__ void trop_witness_pack_a_kernel(int32_t* __restrict__ at, int mp, int kp,
                                           const uint8_t* __restrict__ a, int64_t rsa,
                                           int64_t csa, int m, int k) {
    const int64_t total = static_cast<int64_t>(mp) * kp;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int p = static_cast<int>(idx / mp), i = static_cast<int>(idx % mp);
        int32_t v = TW_ZERO;
        if (i < m && p < k) {
            const uint8_t* el = a + (static_cast<int64_t>(i) * rsa + static_cast<int64_t>(p) * csa) * 2;
            if (el[1]) v = static_cast<int32_t>(static_cast<int8_t>(el[0])) * 65536;
        }
        at[idx] = v;
    }
}

__global__ void trop_witness_pack_b_kernel(int32_t* __restrict__ bt, int np, int kp,
                                           const uint8_t* __restrict__ b, int64_t rsb,
                                           int64_t csb, int k, int n) {
    const int64_t total = static_cast<int64_t>(np) * kp;
    for (GridWalk wk(static_cast<size_t>(np)); wk.idx < static_cast<size_t>(total); wk.next()) {
        const int64_t idx = static_cast<int64_t>(wk.idx);
        const int p = static_cast<int>(wk.i), j = static_cast<int>(wk.j);
        int32_t v = TW_ZERO;
        if (j < n && p < k) {
            const uint8_t* el = b + (static_cast<int64_t>(p) * rsb + static_cast<int64_t>(j) * csb) * 2;
            if (el[1]) v = static_cast<int32_t>(static_cast<int8_t>(el[0])) * 65536 + (65535 - p);
        }
        bt[idx] = v;
    }
}

__global__ void __launch_bounds__(TW_THREADS)
    trop_i8_witness_kernel(const int32_t* __restrict__ at, const int32_t* __restrict__ bt, int mp,
                           int np, int kp, TropEpi e, uint64_t* __restrict__ w, int64_t rsw,
                           int64_t csw) {
    __shared__ __align__(16) int32_t As[2][TW_BK][TW_BM];
    __shared__ __align__(16) int32_t Bs[2][TW_BK][TW_BN];
    const int t = threadIdx.x;
    const int m0 = blockIdx.y * TW_BM, n0 = blockIdx.x * TW_BN;
    const int ty = t >> 4, tx = t & 15;

    auto load_tile = [&](int buf, int k0) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {  // A: 16 rows x 512 B = 512 chunks of 16 B
            const int c = t * 2 + q, r = c >> 5, col = (c & 31) * 4;
            cp_async16(&As[buf][r][col], at + static_cast<int64_t>(k0 + r) * mp + m0 + col);
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int c = t * 2 + q, r = c >> 5, col = (c & 31) * 4;
            cp_async16(&Bs[buf][r][col], bt + static_cast<int64_t>(k0 + r) * np + n0 + col);
        }
        cp_async_commit();
    };

    int32_t acc[8][8];
#pragma unroll
    for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[r][q] = INT_MIN;

    const int tiles = kp / TW_BK;
    if (tiles > 0) load_tile(0, 0);
    for (int kt = 0; kt < tiles; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < tiles) {
            load_tile(buf ^ 1, (kt + 1) * TW_BK);
            cp_async_wait_1();
        } else {
            cp_async_wait_0();
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < TW_BK; ++kk) {
            const int4 a0 = *reinterpret_cast<const int4*>(&As[buf][kk][ty * 8]);
            const int4 a1 = *reinterpret_cast<const int4*>(&As[buf][kk][ty * 8 + 4]);
            const int4 b0 = *reinterpret_cast<const int4*>(&Bs[buf][kk][tx * 8]);
            const int4 b1 = *reinterpret_cast<const int4*>(&Bs[buf][kk][tx * 8 + 4]);
            const int av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const int bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int r = 0; r < 8; ++r)
#pragma unroll
                for (int q = 0; q < 8; ++q) acc[r][q] = __viaddmax_s32(av[r], bv[q], acc[r][q]);
        }
        __syncthreads();
    }

#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const int i = m0 + ty * 8 + r;
        if (i >= e.m) continue;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int j = n0 + tx * 8 + q;
            if (j >= e.n) continue;
            const int32_t key = acc[r][q];
            const bool fin = key > -(1 << 29);
            const int32_t v = fin ? (key >> 16) : 0;  // floor: the index field is non-negative
            const uint64_t at_p = fin ? static_cast<uint64_t>(65535 - (key & 0xFFFF)) : 0;
            trop_finish(e, static_cast<int64_t>(i) * e.rsc + static_cast<int64_t>(j) * e.csc, fin,
                        static_cast<i128>(v));
            w[static_cast<int64_t>(i) * rsw + static_cast<int64_t>(j) * csw] = at_p;
        }
    }
}

// Any Trop<E>: the reduction in 128-bit arithmetic with D-6's witness.
__global__ void trop_generic_witness_kernel(const uint8_t* __restrict__ a, int64_t rsa, int64_t csa,
                                            const uint8_t* __restrict__ b, int64_t rsb, int64_t csb,
                                            int ebytes, int k, TropEpi e, uint64_t* __restrict__ w,
                                            int64_t rsw, int64_t csw) {
    const int i = blockIdx.y * blockDim.y + threadIdx.y;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= e.m || j >= e.n) return;
    bool have = false;
    i128 best = 0;
    int64_t at_p = 0;
    for (int p = 0; p < k; ++p) {
        i128 x, y;
        const bool fx = trop_load(a, ebytes, static_cast<int64_t>(i) * rsa + static_cast<int64_t>(p) * csa, &x);
        const bool fy = trop_load(b, ebytes, static_cast<int64_t>(p) * rsb + static_cast<int64_t>(j) * csb, &y);
        if (fx && fy) {
            const i128 s = x + y;
            if (!have || s > best) best = s, have = true, at_p = p;  // strictly greater: least index
        }
    }
    trop_finish(e, static_cast<int64_t>(i) * e.rsc + static_cast<int64_t>(j) * e.csc, have, best);
    w[static_cast<int64_t>(i) * rsw + static_cast<int64_t>(j) * csw] = static_cast<uint64_t>(at_p);
}

// MaxPlus::finish and the encode over summed split-K keys (one thread per cell).
__global__ void trop_keys_finish_kernel(const int64_t* __restrict__ keys, int m, int n, TropEpi e) {
    const int64_t total = static_cast<int64_t>(m) * n;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t i = idx / n, j = idx - i * n;
        const int64_t key = keys[idx];
        trop_finish(e, i * e.rsc + j * e.csc, key != INT64_MIN, static_cast<i128>(key));
    }
}

static int grid_for(int64_t total) {
    const int64_t g = (total + 255) / 256;
    return static_cast<int>(g < 148 * 32 ? g : 148 * 32);
}

cudaError_t trop_i8_launch(const uint8_t* a, int64_t rsa, int64_t csa, const uint8_t* b,
                           int64_t rsb, int64_t csb, int m, int k, int n, void* ws,
                           const TropEpi& e, cudaStream_t s) {
    const int mp = (m + TR_BM - 1) / TR_BM * TR_BM;
    const int np = (n + TR_BN - 1) / TR_BN * TR_BN;
    const int kp = (k + TR_BK - 1) / TR_BK * TR_BK;
    uint32_t* at = static_cast<uint32_t*>(ws);
    int16_t* bt = reinterpret_cast<int16_t*>(at + static_cast<int64_t>(mp) * kp);
    if (kp > 0) {  // k == 0 reduces nothing: every cell is the semiring zero
        trop_pack_a_kernel<<<grid_for(static_cast<int64_t>(mp) * kp), 256, 0, s>>>(at, mp, kp, a,
                                                                                  rsa, csa, m, k);
        trop_pack_b_kernel<<<grid_for(static_cast<int64_t>(np) * kp), 256, 0, s>>>(bt, np, kp, b,
                                                                                  rsb, csb, k, n);
    }
    dim3 grid(np / TR_BN, mp / TR_BM);
    trop_i8_kernel<<<grid, TR_THREADS, 0, s>>>(at, bt, mp, np, kp, e);
    return cudaGetLastError();
}

size_t trop_i8_workspace(int m, int k, int n) {
    const size_t mp = (m + TR_BM - 1) / TR_BM * TR_BM;
    const size_t np = (n + TR_BN - 1) / TR_BN * TR_BN;
    const size_t kp = (k + TR_BK - 1) / TR_BK * TR_BK;
    return kp * mp * 4 + kp * np * 2;
}

cudaError_t trop_generic_launch(const uint8_t* a, int64_t rsa, int64_t csa, const uint8_t* b,
                                int64_t rsb, int64_t csb, int ebytes, int m, int k, int n,
                                const TropEpi& e, cudaStream_t s) {
    dim3 block(16, 16);
    dim3 grid((n + 15) / 16, (m + 15) / 16);
    trop_generic_kernel<<<grid, block, 0, s>>>(a, rsa, csa, b, rsb, csb, ebytes, k, e);
    return cudaGetLastError();
}

size_t trop_witness_workspace(int m, int k, int n) {
    const size_t mp = (m + TW_BM - 1) / TW_BM * TW_BM;
    const size_t np = (n + TW_BN - 1) / TW_BN * TW_BN;
    const size_t kp = (k + TW_BK - 1) / TW_BK * TW_BK;
    return kp * (mp + np) * 4;
}

cudaError_t trop_i8_witness_launch(const uint8_t* a, int64_t rsa, int64_t csa, const uint8_t* b,
                                   int64_t rsb, int64_t csb, int m, int k, int n, void* ws,
                                   const TropEpi& e, uint64_t* w, int64_t rsw, int64_t csw,
                                   cudaStream_t s) {
    const int mp = (m + TW_BM - 1) / TW_BM * TW_BM;
    const int np = (n + TW_BN - 1) / TW_BN * TW_BN;
    const int kp = (k + TW_BK - 1) / TW_BK * TW_BK;
    int32_t* at = static_cast<int32_t*>(ws);
    int32_t* bt = at + static_cast<int64_t>(mp) * kp;
    if (kp > 0) {
        trop_witness_pack_a_kernel<<<grid_for(static_cast<int64_t>(mp) * kp), 256, 0, s>>>(
            at, mp, kp, a, rsa, csa, m, k);
        trop_witness_pack_b_kernel<<<grid_for(static_cast<int64_t>(np) * kp), 256, 0, s>>>(
            bt, np, kp, b, rsb, csb, k, n);
    }
    dim3 grid(np / TW_BN, mp / TW_BM);
    trop_i8_witness_kernel<<<grid, TW_THREADS, 0, s>>>(at, bt, mp, np, kp, e, w, rsw, csw);
    return cudaGetLastError();
}

cudaError_t trop_generic_witness_launch(const uint8_t* a, int64_t rsa, int64_t csa,
                                        const uint8_t* b, int64_t rsb, int64_t csb, int ebytes,
                                        int m, int k, int n, const TropEpi& e, uint64_t* w,
                                        int64_t rsw, int64_t csw, cudaStream_t s) {
    dim3 block(16, 16);
    dim3 grid((n + 15) / 16, (m + 15) / 16);
    trop_generic_witness_kernel<<<grid, block, 0, s>>>(a, rsa, csa, b, rsb, csb, ebytes, k, e, w,
                                                       rsw, csw);
    return cudaGetLastError();
}

cudaError_t trop_keys_finish_launch(const int64_t* keys, const TropEpi& e, cudaStream_t s) {
    const int64_t total = static_cast<int64_t>(e.m) * e.n;
    if (total == 0) return cudaSuccess;
    trop_keys_finish_kernel<<<grid_for(total), 256, 0, s>>>(keys, e.m, e.n, e);
    return cudaGetLastError();
}

}  // namespace uor
