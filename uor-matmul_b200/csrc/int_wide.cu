// int_wide.cu -- K2/K3: exact i16 / i32 / i64 GEMM by byte slicing.
//
// Replaces the exact lanes of Kernelized for i16 / i32 / i64
// (crates/uor-matmul-gemm/src/kernel.rs:224-399; the I16_I64, I32_I64, I64_I128 tile
// families of isa/portable.rs:91-130), which fold every product (lane_depth = 1 for
// i32) into i128, or into Limbs<3> for i64 (alphabet.rs:618-637).
//
// An L-byte integer is the exact sum of its two's-complement bytes:
//   x = sum_{s < L-1} u_s 256^s + s_{L-1} 256^(L-1)   (u_s unsigned, s_{L-1} signed),
// so A B = sum_{s,t} 256^(s+t) A_s B_t with A_s, B_t int8 matrices. The slice-pair
// kernel (gemm_slices.cu) accumulates every pair on a diagonal d = s + t exactly in
// s32 over a reduction chunk short enough that no partial can overflow, and
// `wide_reduce` adds the partials back as sum_q sum_d partial * 2^(8 d) in 192-bit
// two's complement, then runs the Linear epilogue in the element's own accumulator
// (i128 for i16/i32, Limbs<3> for i64) and encodes once.
#include <climits>
#include <type_traits>
#include "int_gemm.h"
#include "aux.cuh"
#include "gemm_slices.cuh"
#include "modular.cuh"
#include "ptx.cuh"
#include "walk.cuh"

namespace uor {

// ------------------------------------------------------------ slicing kernels

// One eb-byte little-endian element; `aligned` when the buffer is aligned to eb.
template <int EB>
__device__ __forceinline__ uint64_t load_elem(const uint8_t* __restrict__ base, int64_t idx,
                                              bool aligned) {
    const uint8_t* e = base + idx * EB;
    if (aligned) {
        if (EB == 2) return *reinterpret_cast<const uint16_t*>(e);
        if (EB == 4) return *reinterpret_cast<const uint32_t*>(e);
        if (EB == 8) return *reinterpret_cast<const uint64_t*>(e);
    }
    uint64_t v = 0;
#pragma unroll
    for (int s = 0; s < EB; ++s) v |= static_cast<uint64_t>(e[s]) << (8 * s);
    return v;
}

// Byte s of four elements, packed little-endian into one word.
__device__ __forceinline__ uint32_t pack_byte(const uint64_t (&v)[4], int s) {
    return static_cast<uint32_t>((v[0] >> (8 * s)) & 255) |
           static_cast<uint32_t>((v[1] >> (8 * s)) & 255) << 8 |
           static_cast<uint32_t>((v[2] >> (8 * s)) & 255) << 16 |
           static_cast<uint32_t>((v[3] >> (8 * s)) & 255) << 24;
}

// A (m x k, EB-byte elements, strided view) -> As[EB][mp][kp], byte s of each element;
// four consecutive reduction positions per thread, one 4-byte store per slice.
//
// With `cplx` the operand is Complex<T> (repr(C) {re, im}, alphabet.rs:656-663), its
// strides count complex elements, and the sliced matrix is its real image: A's row i
// is (re, im, re, im, ...) over 2k reduction positions, and B's 2k x 2n image holds
// the 2 x 2 block [[w.re, w.im], [-w.im, w.re]] for each element w, so that one real
// product gives (re, im) of every output cell in adjacent columns -- the mac
// re += a.re w.re + a.im (-w.im), im += a.re w.im + a.im w.re (alphabet.rs:712-717).
// -w.im is negated modulo 2^(8 EB), the reference's release-build negation (-MIN = MIN).
__device__ __forceinline__ int64_t cplx_a_index(int i, int q, int64_t rsa, int64_t csa, bool cplx) {
    return cplx ? 2 * (static_cast<int64_t>(i) * rsa + static_cast<int64_t>(q >> 1) * csa) + (q & 1)
                : static_cast<int64_t>(i) * rsa + static_cast<int64_t>(q) * csa;
}

template <int EB>
__global__ void slice_a_kernel(uint8_t* __restrict__ as, int mp, int kp,
                               const uint8_t* __restrict__ a, int64_t rsa, int64_t csa,
                               bool aligned, int m, int k, bool cplx) {
    const int qpr = kp >> 2;
    const int64_t total = static_cast<int64_t>(mp) * qpr;
    const int64_t plane = static_cast<int64_t>(mp) * kp;
    for (GridWalk wk(static_cast<size_t>(qpr)); wk.idx < static_cast<size_t>(total); wk.next()) {
        const int i = static_cast<int>(wk.i);
        const int p0 = static_cast<int>(wk.j) * 4;
        uint64_t v[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int p = p0 + c;
            v[c] = (i < m && p < k) ? load_elem<EB>(a, cplx_a_index(i, p, rsa, csa, cplx), aligned)
                                    : 0;
        }
        uint8_t* dst = as + static_cast<int64_t>(i) * kp + p0;
#pragma unroll
        for (int s = 0; s < EB; ++s) *reinterpret_cast<uint32_t*>(dst + s * plane) = pack_byte(v, s);
    }
}

// B (k x n, strided view) -> Bs[EB][np][kp] (transposed) through a shared tile of 128
// reduction positions x 32 columns: loads run along B's rows, stores along the slices'.
template <int EB>
__global__ void slice_b_kernel(uint8_t* __restrict__ bs, int np, int kp,
                               const uint8_t* __restrict__ b, int64_t rsb, int64_t csb,
                               bool aligned, int k, int n, bool cplx) {
    constexpr uint64_t mask = EB == 8 ? ~0ull : (1ull << (8 * EB)) - 1;
    __shared__ uint64_t tile[32][129];
    const int j0 = blockIdx.x * 32;
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    const int64_t plane = static_cast<int64_t>(np) * kp;
    for (int p0 = blockIdx.y * 128; p0 < kp; p0 += gridDim.y * 128) {
        // sixteen rows per thread with a fixed trip count, so their loads issue together
#pragma unroll 8
        for (int ri = 0; ri < 16; ++ri) {
            const int r = ty + 8 * ri;
            const int p = p0 + r, j = j0 + tx;
            uint64_t v = 0;
            if (p < k && j < n) {
                if (cplx) {
                    const int64_t e = static_cast<int64_t>(p >> 1) * rsb + static_cast<int64_t>(j >> 1) * csb;
                    v = load_elem<EB>(b, 2 * e + ((p ^ j) & 1), aligned);
                    if ((p & 1) && !(j & 1)) v = (0ull - v) & mask;
                } else {
                    v = load_elem<EB>(b, static_cast<int64_t>(p) * rsb + static_cast<int64_t>(j) * csb,
                                      aligned);
                }
            }
            tile[tx][r] = v;
        }
        __syncthreads();
        const int p = p0 + 4 * tx;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int jj = ty * 4 + q, j = j0 + jj;
            if (j < np && p < kp) {
                const uint64_t v[4] = {tile[jj][4 * tx], tile[jj][4 * tx + 1], tile[jj][4 * tx + 2],
                                       tile[jj][4 * tx + 3]};
                uint8_t* dst = bs + static_cast<int64_t>(j) * kp + p;
#pragma unroll
                for (int s = 0; s < EB; ++s)
                    *reinterpret_cast<uint32_t*>(dst + s * plane) = pack_byte(v, s);
            }
        }
        __syncthreads();
    }
}

template <int EB>
static void launch_slicing(uint8_t* as, uint8_t* bs, int mp, int np, int kp, const uint8_t* a,
                           int64_t rsa, int64_t csa, const uint8_t* b, int64_t rsb, int64_t csb,
                           int m, int k, int n, bool cplx, cudaStream_t s) {
    const int64_t quads = static_cast<int64_t>(mp) * (kp / 4);
    const int grid = static_cast<int>(quads / 256 + 1 < 148 * 16 ? quads / 256 + 1 : 148 * 16);
    slice_a_kernel<EB><<<grid, 256, 0, s>>>(as, mp, kp, a, rsa, csa,
                                            reinterpret_cast<uintptr_t>(a) % EB == 0, m, k, cplx);
    const int gy = (kp + 127) / 128 < 65535 ? (kp + 127) / 128 : 65535;
    slice_b_kernel<EB><<<dim3(np / 32, gy), dim3(32, 8), 0, s>>>(
        bs, np, kp, b, rsb, csb, reinterpret_cast<uintptr_t>(b) % EB == 0, k, n, cplx);
}

// ------------------------------------------------------------ exact recombination

struct L3 {
    uint64_t w[3];
};

__device__ __forceinline__ void l3_add(L3& x, const L3& y) {
    uint64_t c = 0;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        const uint64_t s = x.w[i] + y.w[i];
        const uint64_t c1 = s < x.w[i];
        const uint64_t s2 = s + c;
        const uint64_t c2 = s2 < s;
        x.w[i] = s2;
        c = c1 | c2;
    }
}

__device__ __forceinline__ L3 l3_of(i128 v) {
    L3 r;
    r.w[0] = static_cast<uint64_t>(static_cast<u128>(v));
    r.w[1] = static_cast<uint64_t>(static_cast<u128>(v) >> 64);
    r.w[2] = v < 0 ? ~0ull : 0ull;
    return r;
}

__device__ __forceinline__ L3 l3_neg(L3 x) {
    L3 r;
    uint64_t c = 1;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        const uint64_t s = ~x.w[i] + c;
        c = (c && s == 0) ? 1 : 0;
        r.w[i] = s;
    }
    return r;
}

// ScaleExact for Limbs (epilogue.rs:307-329): double-and-add modulo 2^192.
__device__ __forceinline__ L3 l3_scale(L3 x, int64_t f) {
    const bool negf = f < 0;
    uint64_t mag = negf ? 0ull - static_cast<uint64_t>(f) : static_cast<uint64_t>(f);
    L3 acc = {{0, 0, 0}};
    L3 add = negf ? l3_neg(x) : x;
    while (mag) {
        if (mag & 1) l3_add(acc, add);
        L3 d = add;
        l3_add(add, d);
        mag >>= 1;
    }
    return acc;
}

// EncodeFrom<Limbs<3>> for a machine integer (acc.rs:405-444).
__device__ __forceinline__ i128 l3_encode(L3 x, int bits, int mode) {
    const i128 low = static_cast<i128>((static_cast<u128>(x.w[1]) << 64) | x.w[0]);
    if (mode == MODE_WRAPPING) return low;
    const bool neg = (x.w[2] >> 63) != 0;
    const L3 mag3 = neg ? l3_neg(x) : x;
    const i128 mx = bits >= 128 ? i128_max() : ((static_cast<i128>(1) << (bits - 1)) - 1);
    const i128 mn = bits >= 128 ? i128_min() : (-mx - 1);
    if (mag3.w[2] != 0) return neg ? mn : mx;
    const u128 mag = (static_cast<u128>(mag3.w[1]) << 64) | mag3.w[0];
    const u128 limit = neg ? static_cast<u128>(0) - static_cast<u128>(mn) : static_cast<u128>(mx);
    if (mag > limit) return neg ? mn : mx;
    return neg ? static_cast<i128>(static_cast<u128>(0) - mag) : static_cast<i128>(mag);
}

struct WideEpi {
    LinearEpi lin;
    int limbs3;  // 1: i64 elements (Limbs<3> accumulator); 0: i16/i32 (i128 accumulator)
    int cplx;    // 1: C is Complex<O>; real column j is part j & 1 of complex column j >> 1
};

// The exact accumulator of cell idx (row-major over m x n) through the Linear epilogue
// (epilogue.rs:79-93) in the element's own accumulator, encoded and stored.
__device__ __forceinline__ void wide_finish(const WideEpi& e, const L3& acc, size_t i, size_t j,
                                            void* c, int64_t rsc, int64_t csc) {
    const int64_t off =
        e.cplx ? 2 * (static_cast<int64_t>(i) * rsc + static_cast<int64_t>(j >> 1) * csc) +
                     static_cast<int64_t>(j & 1)
               : static_cast<int64_t>(i) * rsc + static_cast<int64_t>(j) * csc;
    const LinearEpi& L = e.lin;
    i128 outv;
    if (e.limbs3) {
        L3 tot = L.alpha == 1 ? acc : l3_scale(acc, L.alpha);
        if (L.beta != 0) {
            const L3 pr = l3_scale(l3_of(load_out(c, L.kind, off)), L.beta);
            l3_add(tot, pr);
        }
        outv = l3_encode(tot, out_bits(L.kind), L.mode);
    } else {
        const i128 a = static_cast<i128>((static_cast<u128>(acc.w[1]) << 64) | acc.w[0]);
        i128 tot = L.alpha == 1 ? a : sat_mul(a, L.alpha);
        if (L.beta != 0)
            tot = static_cast<i128>(static_cast<u128>(tot) +
                                    static_cast<u128>(sat_mul(load_out(c, L.kind, off), L.beta)));
        outv = encode_int(tot, out_bits(L.kind), L.mode);
    }
    store_out(c, L.kind, off, outv);
}

// Group g is the diagonal d = g, weighted 2^(8 g). The partials of a cell are summed
// in 128-bit column sums per 64-bit word (chunk by chunk, every load of a chunk issued
// before any is used) and carried into 192-bit two's complement.
template <int NG>
__global__ void wide_reduce_kernel(const int32_t* __restrict__ part, int chunks, int groups,
                                   size_t m, size_t n, void* c, int64_t rsc, int64_t csc,
                                   WideEpi e) {
    constexpr int NQ = (NG + 7) / 8;
    static_assert(NQ <= 2, "at most 16 diagonals");
    const size_t total = m * n;
    for (GridWalk wk(n); wk.idx < total; wk.next()) {
        const size_t idx = wk.idx;
        i128 col[NQ];
#pragma unroll
        for (int q = 0; q < NQ; ++q) col[q] = 0;
        for (int q = 0; q < chunks; ++q) {
            const int32_t* pq = part + static_cast<size_t>(q) * groups * total + idx;
            int32_t v[NG];
#pragma unroll
            for (int g = 0; g < NG; ++g) v[g] = g < groups ? __ldg(pq + g * total) : 0;
#pragma unroll
            for (int g = 0; g < NG; ++g) col[g >> 3] += static_cast<i128>(v[g]) << (8 * (g & 7));
        }
        L3 acc;
        {
            const i128 t0 = col[0];
            acc.w[0] = static_cast<uint64_t>(static_cast<u128>(t0));
            i128 carry = t0 >> 64;
            if (NQ == 2) {
                const i128 t1 = col[NQ - 1] + carry;
                acc.w[1] = static_cast<uint64_t>(static_cast<u128>(t1));
                carry = t1 >> 64;
                acc.w[2] = static_cast<uint64_t>(static_cast<u128>(carry));
            } else {
                acc.w[1] = static_cast<uint64_t>(static_cast<u128>(carry));
                acc.w[2] = carry < 0 ? ~0ull : 0ull;
            }
        }
        wide_finish(e, acc, wk.i, wk.j, c, rsc, csc);
    }
}

// ------------------------------------------------------------ modular route
//
// The modular route (modular.cuh) for i32 / i64 elements: every element is an integer of
// 8 EB bits, |S| <= k 2^(16 EB - 2), and nm coprime moduli cover twice that; one int8
// GEMM per modulus replaces the L^2 byte-slice pairs whenever nm is smaller (10 moduli
// against 16 pairs for i32 at k = 65536, 20 against 64 for i64).

// Weights of an EB-byte integer's bytes modulo p_g. The value x is read as the unsigned
// x + 2^(8 EB - 1) (its sign bit flipped), and bias folds the -2^(8 EB - 1) back in; the
// balanced residue's shift half_g rides in it too (fm_balanced_vh).
struct WmWeights {
    uint32_t w0[FM_MAX];    // bytes i of 256^i mod p_g, i < 4
    uint32_t w1[FM_MAX];    // bytes i - 4 of 256^i mod p_g, 4 <= i < 8
    uint32_t bias[FM_MAX];  // (p_g - 2^(8 EB - 1) mod p_g) + half_g
};

template <int EB, int NM>
__device__ __forceinline__ void wm_store(int8_t* dst, int64_t plane, const uint64_t (&v)[4],
                                         const FmParams& f, const WmWeights& w) {
    constexpr uint64_t sign = 1ull << (8 * EB - 1);
    uint32_t lo[4], hi[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        lo[c] = static_cast<uint32_t>(v[c] ^ sign);
        hi[c] = static_cast<uint32_t>((v[c] ^ sign) >> 32);
    }
#pragma unroll
    for (int g = 0; g < NM; ++g) {
        uint32_t word = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            uint32_t v = __dp4a(lo[c], w.w0[g], w.bias[g]);  // the bias includes half_g
            if (EB == 8) v = __dp4a(hi[c], w.w1[g], v);
            word = fm_put_byte(word, fm_balanced_vh(v, f.pneg[g], f.magic32[g], f.hneg[g]), c);
        }
        *reinterpret_cast<uint32_t*>(dst + g * plane) = word;
    }
}

// A (m x k, EB-byte elements) -> residue planes As[NM][mp][kp], four reduction positions
// per thread (the complex real image as slice_a_kernel reads it).
template <int EB, int NM>
__global__ void wm_slice_a_kernel(int8_t* __restrict__ as, int mp, int kp,
                                  const uint8_t* __restrict__ a, int64_t rsa, int64_t csa,
                                  bool aligned, int m, int k, bool cplx, FmParams f, WmWeights w) {
    // Rows of consecutive elements (unit column stride; a complex row's parts are then
    // consecutive too) starting on 16-byte boundaries take vector loads.
    const bool vec = csa == 1 && (EB == 4 || EB == 8) &&
                     (reinterpret_cast<uintptr_t>(a) & 15) == 0 && ((rsa * EB * (cplx ? 2 : 1)) & 15) == 0;
    const int qpr = kp >> 2;
    const int64_t total = static_cast<int64_t>(mp) * qpr;
    const int64_t plane = static_cast<int64_t>(mp) * kp;
    // The vector loads of the next step are issued before this step's residues (in flight
    // while they are computed).
    auto fetch = [&](const GridWalk& wv, uint4& q0, uint4& q1) {
        const int i = static_cast<int>(wv.i), p0 = static_cast<int>(wv.j) * 4;
        q0 = q1 = make_uint4(0, 0, 0, 0);
        if (vec && i < m && p0 + 3 < k) {
            const uint4* src = reinterpret_cast<const uint4*>(a + cplx_a_index(i, p0, rsa, csa, cplx) * EB);
            q0 = __ldg(src);
            if (EB == 8) q1 = __ldg(src + 1);
        }
    };
    GridWalk wk(static_cast<size_t>(qpr));
    uint4 c0 = make_uint4(0, 0, 0, 0), c1 = c0;
    if (wk.idx < static_cast<size_t>(total)) fetch(wk, c0, c1);
    while (wk.idx < static_cast<size_t>(total)) {
        GridWalk nx = wk;
        nx.next();
        uint4 n0 = make_uint4(0, 0, 0, 0), n1 = n0;
        if (nx.idx < static_cast<size_t>(total)) fetch(nx, n0, n1);
        const int i = static_cast<int>(wk.i);
        const int p0 = static_cast<int>(wk.j) * 4;
        uint64_t v[4];
        const int64_t e0 = cplx_a_index(i, p0, rsa, csa, cplx);
        if (vec && i < m && p0 + 3 < k) {
            // four consecutive elements in one or two 16-byte loads
            if (EB == 4) {
                v[0] = c0.x, v[1] = c0.y, v[2] = c0.z, v[3] = c0.w;
            } else if (EB == 8) {
                v[0] = c0.x | static_cast<uint64_t>(c0.y) << 32, v[1] = c0.z | static_cast<uint64_t>(c0.w) << 32;
                v[2] = c1.x | static_cast<uint64_t>(c1.y) << 32, v[3] = c1.z | static_cast<uint64_t>(c1.w) << 32;
            } else {
#pragma unroll
                for (int c = 0; c < 4; ++c) v[c] = load_elem<EB>(a, e0 + c, aligned);
            }
        } else {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int p = p0 + c;
                v[c] = (i < m && p < k) ? load_elem<EB>(a, cplx_a_index(i, p, rsa, csa, cplx), aligned) : 0;
            }
        }
        wm_store<EB, NM>(as + static_cast<int64_t>(i) * kp + p0, plane, v, f, w);
        wk = nx;
        c0 = n0;
        c1 = n1;
    }
}

// B (k x n) -> residue planes Bs[NM][np][kp] (transposed) through a shared tile of 128
// reduction positions x 32 columns, the complex real image as slice_b_kernel builds it.
template <int EB, int NM>
__global__ void wm_slice_b_kernel(int8_t* __restrict__ bs, int np, int kp,
                                  const uint8_t* __restrict__ b, int64_t rsb, int64_t csb,
                                  bool aligned, int k, int n, bool cplx, FmParams f, WmWeights w) {
    constexpr uint64_t mask = EB == 8 ? ~0ull : (1ull << (8 * EB)) - 1;
    // Elements of up to four bytes sit in 32-bit words with 16-byte rows, so a quad is one
    // 16-byte read; 8-byte elements keep an odd row stride.
    using TT = typename std::conditional<EB == 8, uint64_t, uint32_t>::type;
    constexpr int TS = EB == 8 ? 129 : 132;
    __shared__ __align__(16) TT tile[32][TS];
    const int j0 = blockIdx.x * 32;
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    const int64_t plane = static_cast<int64_t>(np) * kp;
    for (int p0 = blockIdx.y * 128; p0 < kp; p0 += gridDim.y * 128) {
        // sixteen rows per thread with a fixed trip count, so their loads issue together
#pragma unroll 8
        for (int ri = 0; ri < 16; ++ri) {
            const int r = ty + 8 * ri;
            const int p = p0 + r, j = j0 + tx;
            uint64_t v = 0;
            if (p < k && j < n) {
                if (cplx) {
                    const int64_t e = static_cast<int64_t>(p >> 1) * rsb + static_cast<int64_t>(j >> 1) * csb;
                    v = load_elem<EB>(b, 2 * e + ((p ^ j) & 1), aligned);
                    if ((p & 1) && !(j & 1)) v = (0ull - v) & mask;
                } else {
                    v = load_elem<EB>(b, static_cast<int64_t>(p) * rsb + static_cast<int64_t>(j) * csb,
                                      aligned);
                }
            }
            tile[tx][r] = static_cast<TT>(v);
        }
        __syncthreads();
        const int p = p0 + 4 * tx;
#pragma unroll 1
        for (int q = 0; q < 4; ++q) {
            const int jj = ty * 4 + q, j = j0 + jj;
            if (j < np && p < kp) {
                uint64_t v[4];
                if (EB == 8) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) v[c] = tile[jj][4 * tx + c];
                } else {
                    const uint4 t4 = *reinterpret_cast<const uint4*>(&tile[jj][4 * tx]);
                    v[0] = t4.x, v[1] = t4.y, v[2] = t4.z, v[3] = t4.w;
                }
                wm_store<EB, NM>(bs + static_cast<int64_t>(j) * kp + p, plane, v, f, w);
            }
        }
        __syncthreads();
    }
}

// One thread per cell: y, the CRT value, and the element's Linear epilogue and encode.
template <int NM>
__global__ void wm_crt_kernel(const uint8_t* __restrict__ res, int chunks, size_t m, size_t n,
                              void* c, int64_t rsc, int64_t csc, WideEpi e, FmParams f) {
    constexpr int NL = FmLimbs<NM>::value;
    const size_t total = m * n;
    for (GridWalk wk(n); wk.idx < total; wk.next()) {
        const size_t idx = wk.idx;
        uint32_t y[NM];
        fm_load_y<NM>(res, chunks, total, idx, f, y);
        uint32_t limb[NL];
        const uint32_t ext = fm_crt<NM>(y, f, limb);
        L3 acc;
#pragma unroll
        for (int q = 0; q < 3; ++q) {
            const uint64_t lo = 2 * q < NL ? limb[2 * q] : ext;
            const uint64_t hi = 2 * q + 1 < NL ? limb[2 * q + 1] : ext;
            acc.w[q] = lo | hi << 32;
        }
        wide_finish(e, acc, wk.i, wk.j, c, rsc, csc);
    }
}

// The same for rows of a multiple of four cells, four cells per thread: one 32-bit load per
// chunk and residue plane covers the four cells, and the chunks' residues are summed two
// cells to a register in 16-bit lanes (bytes 0 and 2, bytes 1 and 3; at most 256 chunks
// of residues below 256 keep each lane below 2^16).
template <int NM>
__global__ void __launch_bounds__(256) wm_crt4_kernel(const uint8_t* __restrict__ res, int chunks,
                                                      size_t m, size_t n, void* c, int64_t rsc,
                                                      int64_t csc, WideEpi e, FmParams f) {
    constexpr int NL = FmLimbs<NM>::value;
    const size_t total = m * n;
    const size_t quads = total >> 2;
    for (GridWalk wk(n >> 2); wk.idx < quads; wk.next()) {
        const size_t idx0 = wk.idx * 4;
        uint32_t ev[NM], od[NM];
#pragma unroll
        for (int g = 0; g < NM; ++g) ev[g] = od[g] = 0;
        for (int q = 0; q < chunks; ++q) {
#pragma unroll
            for (int g = 0; g < NM; ++g) {
                const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(
                    res + (static_cast<size_t>(q) * NM + g) * total + idx0));
                ev[g] += w & 0x00FF00FFu;
                od[g] += (w >> 8) & 0x00FF00FFu;
            }
        }
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
            uint32_t y[NM];
#pragma unroll
            for (int g = 0; g < NM; ++g) {
                const uint32_t sum = (cc & 1) ? od[g] : ev[g];
                const uint32_t v = (cc >> 1) ? sum >> 16 : sum & 0xFFFFu;
                // one chunk: the epilogue stored y_g itself; more: the summed residues
                y[g] = chunks == 1 ? v
                                   : fm_mod24(fm_mod24(v, f.p[g], f.magic32[g]) * f.inv[g], f.p[g],
                                              f.magic32[g]);
            }
            uint32_t limb[NL];
            const uint32_t ext = fm_crt<NM>(y, f, limb);
            L3 acc;
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                const uint64_t lo = 2 * q < NL ? limb[2 * q] : ext;
                const uint64_t hi = 2 * q + 1 < NL ? limb[2 * q + 1] : ext;
                acc.w[q] = lo | hi << 32;
            }
            wide_finish(e, acc, wk.i, wk.j * 4 + cc, c, rsc, csc);
        }
    }
}

template <int EB, int NM>
static void wm_launch(int8_t* as, int mp, int8_t* bs, int np, int kp, const uint8_t* a,
                      int64_t rsa, int64_t csa, const uint8_t* b, int64_t rsb, int64_t csb, int m,
                      int k, int n, bool cplx, const FmParams& f, const WmWeights& w,
                      cudaStream_t s, cudaStream_t side) {
    const int64_t quads = static_cast<int64_t>(mp) * (kp / 4);
    const int grid = static_cast<int>(quads / 256 + 1 < 148 * 16 ? quads / 256 + 1 : 148 * 16);
    wm_slice_a_kernel<EB, NM><<<grid, 256, 0, s>>>(as, mp, kp, a, rsa, csa,
                                                   reinterpret_cast<uintptr_t>(a) % EB == 0, m, k,
                                                   cplx, f, w);
    const int gy = (kp + 127) / 128 < 65535 ? (kp + 127) / 128 : 65535;
    // B's slicer beside A's on the side stream when there is one (both CUDA-core kernels).
    wm_slice_b_kernel<EB, NM><<<dim3(np / 32, gy), dim3(32, 8), 0, side ? side : s>>>(
        bs, np, kp, b, rsb, csb, reinterpret_cast<uintptr_t>(b) % EB == 0, k, n, cplx, f, w);
}

#define WM_COUNTS(X) X(8) X(10) X(12) X(14) X(16) X(18) X(20) X(22) X(24)

// ------------------------------------------------------------ driver

static inline size_t rup(size_t x, size_t a) { return (x + a - 1) / a * a; }

static void launch_wide_reduce(const int32_t* part, int chunks, int groups, size_t m, size_t n,
                               void* c, ptrdiff_t rsc, ptrdiff_t csc, const WideEpi& we,
                               cudaStream_t s) {
    const size_t total = m * n;
    const int rgrid = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
    if (groups <= 8)
        wide_reduce_kernel<8><<<rgrid, 256, 0, s>>>(part, chunks, groups, m, n, c, rsc, csc, we);
    else
        wide_reduce_kernel<16><<<rgrid, 256, 0, s>>>(part, chunks, groups, m, n, c, rsc, csc, we);
}

int run_wide_gemm(uor_b200_ctx* ctx, int eb, const uint8_t* a, ptrdiff_t rsa, ptrdiff_t csa,
                  const uint8_t* b, ptrdiff_t rsb, ptrdiff_t csb, void* c, ptrdiff_t rsc,
                  ptrdiff_t csc, size_t m, size_t k, size_t n, const LinearEpi& epi,
                  uor_b200_route* route, bool cplx, uint32_t route_flags) {
    const bool digits_only = (route_flags & UOR_B200_DIGIT_SLICES) != 0;
    const bool force_modular = !digits_only && (route_flags & UOR_B200_MODULAR) != 0;
    cudaStream_t s = ctx->stream;
    if (route) {
        *route = uor_b200_route{};
        route->tile_m = KS_BM;
        route->tile_n = KS_BN;
        route->tile_k = KS_BK;
    }
    if (m == 0 || n == 0) return UOR_B200_OK;
    // A complex product is the real product of the operands' real images (2k x 2n B).
    if (cplx) {
        k *= 2;
        n *= 2;
    }
    if (m > (size_t)INT_MAX / 4 || n > (size_t)INT_MAX / 4 || k > (size_t)INT_MAX / 4)
        return UOR_B200_UNSUPPORTED;
    const WideEpi we{epi, eb == 8 ? 1 : 0, cplx ? 1 : 0};
    if (k == 0) {
        // A zero accumulator through the same epilogue, in the element's own accumulator.
        if (route) route->kernel = UOR_B200_KERNEL_EPILOGUE_ONLY;
        launch_wide_reduce(nullptr, 0, 0, m, n, c, rsc, csc, we, s);
        return cuda_status(cudaGetLastError());
    }
    const int L = eb;
    // Slice pairs grouped by diagonal; under Wrapping into <= 64-bit outputs the
    // diagonals at or above the output width vanish modulo 2^bits.
    const int max_prod_uu = 255 * 255, max_prod_us = 255 * 128, max_prod_ss = 128 * 128;
    const int obits = out_bits(epi.kind);
    KSParams p{};
    int npairs = 0, ngroups = 0;
    int64_t worst = 1;
    for (int d = 0; d <= 2 * L - 2; ++d) {
        if (epi.mode == MODE_WRAPPING && obits <= 64 && 8 * d >= obits) break;
        p.pair_begin[ngroups] = npairs;
        int64_t sum = 0;
        for (int sa = 0; sa < L; ++sa) {
            const int sb = d - sa;
            if (sb < 0 || sb >= L) continue;
            const bool as = sa == L - 1, bs = sb == L - 1;
            p.pair_a[npairs] = static_cast<uint8_t>(sa);
            p.pair_b[npairs] = static_cast<uint8_t>(sb);
            p.pair_sign[npairs] = static_cast<uint8_t>((as ? 1 : 0) | (bs ? 2 : 0));
            sum += as && bs ? max_prod_ss : (as || bs ? max_prod_us : max_prod_uu);
            ++npairs;
        }
        ++ngroups;
        if (sum > worst) worst = sum;
    }
    p.pair_begin[ngroups] = npairs;
    p.num_groups = ngroups;

    // The modular route when its estimated time is below the byte-slice route's. Rates
    // measured on B200 at 1024 x 65536 x 1024: a GEMM 8.1e-16 s per multiply-add;
    // residue slicing 4.5e-13 s per element and modulus; byte slicing 5.1e-13 s per
    // element and plane; the slice route's recombination 1.1e-12 s per cell and partial
    // plane; the CRT 1.5e-11 s per cell.
    FmParams fm;
    bool modular = false;
    if (!digits_only && (eb == 4 || eb == 8) && fm_plan_ints(8 * eb, k, fm) && fm.nm >= 8 &&
        fm.nm <= 24) {
        const double mnk = static_cast<double>(m) * n * k, elems = static_cast<double>(k) * (m + n);
        const double lane_d = static_cast<double>(INT_MAX) / worst;
        const double chunks_d = static_cast<double>(k) / lane_d + 1.0;
        const double t_mod = fm.nm * (mnk * 8.1e-16 + elems * 4.5e-13) + 1.5e-11 * m * n;
        const double t_dig = npairs * mnk * 8.1e-16 + L * elems * 5.1e-13 +
                             1.1e-12 * m * n * chunks_d * ngroups;
        modular = force_modular || t_mod < t_dig;
    }
    if (modular) {
        const int nm = fm.nm;
        KSParams q{};
        q.num_groups = nm;
        for (int g = 0; g < nm; ++g) {
            q.pair_begin[g] = g;
            q.pair_a[g] = q.pair_b[g] = static_cast<uint8_t>(g);
            q.pair_sign[g] = 3;
            q.res_mod[g] = fm.p[g];
            q.res_magic[g] = fm.magic32[g];
            q.res_off[g] = static_cast<uint32_t>(fm.p[g] * ((0x80000000ull + fm.p[g] - 1) / fm.p[g]));
        }
        q.pair_begin[nm] = nm;
        const int num_kb = static_cast<int>((k + KS_BK - 1) / KS_BK);
        // |residue product| <= 2^14: 1023 blocks keep |acc| < 2^31 - 2^21
        const int64_t lane_m = (int64_t)INT_MAX / 16384 / KS_BK;
        q.kb_per_chunk = static_cast<int>(lane_m < num_kb ? lane_m : num_kb);
        q.num_chunks = (num_kb + q.kb_per_chunk - 1) / q.kb_per_chunk;
        q.num_kb = num_kb;
        q.m = static_cast<int>(m);
        q.mp = static_cast<int>(ks_rows_pad(m));
        q.np = static_cast<int>(rup(n, KS_BN));
        ks_balance_chunks(q, ctx->sm_count);
        if (q.num_chunks == 1)
            for (int g = 0; g < nm; ++g) q.res_inv[g] = fm.inv[g];
        q.m = static_cast<int>(m);
        q.n = static_cast<int>(n);
        q.mp = static_cast<int>(ks_rows_pad(m));
        q.np = static_cast<int>(rup(n, KS_BN));
        q.status = ctx->d_status;
        q.budget_ns = ctx->budget_ns;
        WmWeights w{};
        for (int g = 0; g < nm; ++g) {
            const uint32_t pg = fm.p[g];
            uint32_t c = 1 % pg;
            for (int i = 0; i < 8; ++i) {
                (i < 4 ? w.w0[g] : w.w1[g]) |= c << (8 * (i & 3));
                c = c * 256 % pg;
            }
            uint32_t top = 1 % pg;  // 2^(8 eb - 1) mod p
            for (int i = 0; i < 8 * eb - 1; ++i) top = top * 2 % pg;
            w.bias[g] = (pg - top) % pg + fm.half[g];  // and the balanced residue's shift
        }
        const size_t kp = rup(k, 16);
        const size_t a_bytes = rup((size_t)nm * q.mp * kp, 256);
        const size_t b_bytes = rup((size_t)nm * q.np * kp, 256);
        const size_t res_bytes = rup((size_t)q.num_chunks * nm * m * n, 256);
        int st = UOR_B200_OK;
        uint8_t* ws = static_cast<uint8_t*>(ctx_buffer(ctx, SLOT_WS, a_bytes + b_bytes + res_bytes, &st));
        if (!ws) return st;
        int8_t* as = reinterpret_cast<int8_t*>(ws);
        int8_t* bs = reinterpret_cast<int8_t*>(ws + a_bytes);
        uint8_t* res = ws + a_bytes + b_bytes;
        cudaStream_t side = ctx_fork(ctx);
        switch (eb * 100 + nm) {
#define WM_SLICE4(N) \
    case 400 + N: wm_launch<4, N>(as, q.mp, bs, q.np, (int)kp, a, rsa, csa, b, rsb, csb, (int)m, (int)k, (int)n, cplx, fm, w, s, side); break;
#define WM_SLICE8(N) \
    case 800 + N: wm_launch<8, N>(as, q.mp, bs, q.np, (int)kp, a, rsa, csa, b, rsb, csb, (int)m, (int)k, (int)n, cplx, fm, w, s, side); break;
            WM_COUNTS(WM_SLICE4)
            WM_COUNTS(WM_SLICE8)
#undef WM_SLICE4
#undef WM_SLICE8
        default: return UOR_B200_UNSUPPORTED;
        }
        if (side && !ctx_join(ctx)) return UOR_B200_DEVICE_ERROR;
        if (cudaGetLastError() != cudaSuccess) return UOR_B200_DEVICE_ERROR;
        q.residue = res;
        if (route) {
            route->kernel = UOR_B200_KERNEL_LIMB_TCGEN05;
            route->k_chunks = static_cast<uint32_t>(q.num_chunks);
            route->pairs = static_cast<uint32_t>(nm);
            route->moduli = static_cast<uint32_t>(nm);
        }
        if ((st = ks_run(as, nm, bs, nm, k, kp, q, ctx->sm_count, s, route ? &route->ctas : nullptr)) !=
            UOR_B200_OK)
            return st;
        if (route) route->tile_m = static_cast<uint32_t>(q.m > 128 ? 256 : KS_BM);
        const WideEpi we{epi, eb == 8 ? 1 : 0, cplx ? 1 : 0};
        const size_t total = m * n;
        const int rgrid = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
        const bool quad = n % 4 == 0 && q.num_chunks <= 256;
        const size_t qn = total / 4;
        const int qgrid = (int)((qn + 255) / 256 < 148 * 16 ? (qn + 255) / 256 : 148 * 16);
        switch (nm) {
#define WM_CRT(N)                                                                                   \
    case N:                                                                                         \
        if (quad) wm_crt4_kernel<N><<<qgrid, 256, 0, s>>>(res, q.num_chunks, m, n, c, rsc, csc, we, fm); \
        else wm_crt_kernel<N><<<rgrid, 256, 0, s>>>(res, q.num_chunks, m, n, c, rsc, csc, we, fm);      \
        break;
            WM_COUNTS(WM_CRT)
#undef WM_CRT
        default: return UOR_B200_UNSUPPORTED;
        }
        return cuda_status(cudaGetLastError());
    }

    // The longest reduction a diagonal's s32 lane holds exactly, in whole blocks.
    const int64_t lane = (static_cast<int64_t>(INT_MAX) / worst) / KS_BK;
    const int num_kb = static_cast<int>((k + KS_BK - 1) / KS_BK);
    p.kb_per_chunk = static_cast<int>(lane < num_kb ? lane : num_kb);
    p.num_chunks = (num_kb + p.kb_per_chunk - 1) / p.kb_per_chunk;
    p.num_kb = num_kb;
    p.m = static_cast<int>(m);
    p.n = static_cast<int>(n);
    p.mp = static_cast<int>(ks_rows_pad(m));
    p.np = static_cast<int>(rup(n, KS_BN));
    p.status = ctx->d_status;
    p.budget_ns = ctx->budget_ns;

    const size_t kp = rup(k, 16);
    const size_t a_bytes = rup((size_t)L * p.mp * kp, 256);
    const size_t b_bytes = rup((size_t)L * p.np * kp, 256);
    const size_t part_bytes = (size_t)p.num_chunks * ngroups * m * n * sizeof(int32_t);
    int st = UOR_B200_OK;
    uint8_t* ws = static_cast<uint8_t*>(
        ctx_buffer(ctx, SLOT_WS, a_bytes + b_bytes + rup(part_bytes, 256), &st));
    if (!ws) return st;
    uint8_t* as = ws;
    uint8_t* bs = ws + a_bytes;
    int32_t* part = reinterpret_cast<int32_t*>(ws + a_bytes + b_bytes);
    p.partial = part;

    if (eb == 2)
        launch_slicing<2>(as, bs, p.mp, p.np, (int)kp, a, rsa, csa, b, rsb, csb, (int)m, (int)k, (int)n, cplx, s);
    else if (eb == 4)
        launch_slicing<4>(as, bs, p.mp, p.np, (int)kp, a, rsa, csa, b, rsb, csb, (int)m, (int)k, (int)n, cplx, s);
    else
        launch_slicing<8>(as, bs, p.mp, p.np, (int)kp, a, rsa, csa, b, rsb, csb, (int)m, (int)k, (int)n, cplx, s);
    if (route) route->kernel = UOR_B200_KERNEL_LIMB_TCGEN05;
    if (route) route->k_chunks = (uint32_t)p.num_chunks;
    if (route) route->pairs = (uint32_t)npairs;
    if ((st = ks_run(as, L, bs, L, k, kp, p, ctx->sm_count, s, route ? &route->ctas : nullptr)) !=
        UOR_B200_OK)
        return st;
    if (route) route->tile_m = (uint32_t)(p.m > 128 ? 256 : KS_BM);
    launch_wide_reduce(part, p.num_chunks, ngroups, m, n, c, rsc, csc, we, s);
    return cuda_status(cudaGetLastError());
}

}  // namespace uor
