// splitk.cu -- the limb conversion and finish kernels of the split-K exchange
// (see splitk.cuh). Both are HBM-bound elementwise passes.
#include "splitk.cuh"
#include "walk.cuh"

namespace uor {

__global__ void i128_to_limbs_kernel(const uint64_t* __restrict__ x, int64_t* __restrict__ limbs,
                                     size_t cells) {
    const int64_t mask = (int64_t{1} << SPLITK_LIMB_BITS) - 1;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < cells;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const i128 v = static_cast<i128>((static_cast<u128>(x[2 * i + 1]) << 64) | x[2 * i]);
        limbs[3 * i] = static_cast<int64_t>(v) & mask;
        limbs[3 * i + 1] = static_cast<int64_t>(v >> SPLITK_LIMB_BITS) & mask;
        limbs[3 * i + 2] = static_cast<int64_t>(v >> (2 * SPLITK_LIMB_BITS));
    }
}

// The accumulator of i8/i16/i32 elements is i128: alpha scales it saturating
// (ScaleExact for i128, epilogue.rs:280-288), beta C is added wrapping, then the
// output's encode.
__global__ void limbs_finish_kernel(const int64_t* __restrict__ limbs, size_t m, size_t n, void* c,
                                    int64_t rsc, int64_t csc, LinearEpi e) {
    const size_t total = m * n;
    for (GridWalk wk(n); wk.idx < total; wk.next()) {
        const size_t idx = wk.idx;
        const i128 x = static_cast<i128>(limbs[3 * idx]) +
                       (static_cast<i128>(limbs[3 * idx + 1]) << SPLITK_LIMB_BITS) +
                       (static_cast<i128>(limbs[3 * idx + 2]) << (2 * SPLITK_LIMB_BITS));
        const size_t i = wk.i, j = wk.j;
        const int64_t off = static_cast<int64_t>(i) * rsc + static_cast<int64_t>(j) * csc;
        i128 tot = e.alpha == 1 ? x : sat_mul(x, e.alpha);
        if (e.beta != 0)
            tot = static_cast<i128>(static_cast<u128>(tot) +
                                    static_cast<u128>(sat_mul(load_out(c, e.kind, off), e.beta)));
        store_out(c, e.kind, off, encode_int(tot, out_bits(e.kind), e.mode));
    }
}

static int grid_for(size_t work) {
    const size_t g = (work + 255) / 256;
    return static_cast<int>(g < 148 * 16 ? (g ? g : 1) : 148 * 16);
}

cudaError_t i128_to_limbs(const void* x, int64_t* limbs, size_t cells, cudaStream_t s) {
    if (cells == 0) return cudaSuccess;
    i128_to_limbs_kernel<<<grid_for(cells), 256, 0, s>>>(static_cast<const uint64_t*>(x), limbs,
                                                          cells);
    return cudaGetLastError();
}

cudaError_t limbs_finish(const int64_t* limbs, size_t m, size_t n, void* c, int64_t rsc,
                         int64_t csc, const LinearEpi& e, cudaStream_t s) {
    if (m == 0 || n == 0) return cudaSuccess;
    limbs_finish_kernel<<<grid_for(m * n), 256, 0, s>>>(limbs, m, n, c, rsc, csc, e);
    return cudaGetLastError();
}

}  // namespace uor
