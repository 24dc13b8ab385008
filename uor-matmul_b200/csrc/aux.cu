// aux.cu -- helper kernels: strided gather, epilogue-only, chunk reduction,
// and the bounded-wait self-test.
#include "aux.cuh"
#include "walk.cuh"
#include "ptx.cuh"

namespace uor {

template <int ES>
struct Elem {
    uint8_t b[ES];
};

template <int ES>
__global__ void gather_2d_kernel(uint8_t* __restrict__ dst, size_t ld,
                                 const uint8_t* __restrict__ src, size_t rows, size_t cols,
                                 ptrdiff_t rs, ptrdiff_t cs) {
    const size_t total = rows * cols;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        const size_t r = idx / cols, c = idx - (idx / cols) * cols;
        const ptrdiff_t off = (ptrdiff_t)r * rs + (ptrdiff_t)c * cs;
        *reinterpret_cast<Elem<ES>*>(dst + (r * ld + c) * ES) =
            *reinterpret_cast<const Elem<ES>*>(src + off * ES);
    }
}

cudaError_t gather_2d(void* dst, size_t ld, const void* src, size_t rows, size_t cols,
                      ptrdiff_t rs, ptrdiff_t cs, int esize, cudaStream_t s) {
    if (rows == 0 || cols == 0) return cudaSuccess;
    const size_t total = rows * cols;
    const int block = 256;
    const int grid = (int)((total + block - 1) / block < 148 * 16 ? (total + block - 1) / block
                                                                   : 148 * 16);
    auto d = static_cast<uint8_t*>(dst);
    auto src8 = static_cast<const uint8_t*>(src);
    switch (esize) {
    case 1: gather_2d_kernel<1><<<grid, block, 0, s>>>(d, ld, src8, rows, cols, rs, cs); break;
    case 2: gather_2d_kernel<2><<<grid, block, 0, s>>>(d, ld, src8, rows, cols, rs, cs); break;
    case 4: gather_2d_kernel<4><<<grid, block, 0, s>>>(d, ld, src8, rows, cols, rs, cs); break;
    case 8: gather_2d_kernel<8><<<grid, block, 0, s>>>(d, ld, src8, rows, cols, rs, cs); break;
    case 16: gather_2d_kernel<16><<<grid, block, 0, s>>>(d, ld, src8, rows, cols, rs, cs); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

__global__ void epilogue_only_kernel(void* c, int64_t rsc, int64_t csc, size_t m, size_t n,
                                     LinearEpi e) {
    const size_t total = m * n;
    for (GridWalk wk(n); wk.idx < total; wk.next()) {
        const size_t i = wk.i, j = wk.j;
        finish_cell(e, c, (int64_t)i * rsc + (int64_t)j * csc, 0);
    }
}

cudaError_t epilogue_only(void* c, int64_t rsc, int64_t csc, size_t m, size_t n,
                          const LinearEpi& e, cudaStream_t s) {
    if (m == 0 || n == 0) return cudaSuccess;
    const size_t total = m * n;
    const int grid = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
    epilogue_only_kernel<<<grid, 256, 0, s>>>(c, rsc, csc, m, n, e);
    return cudaGetLastError();
}

__global__ void reduce_chunks_kernel(const int32_t* __restrict__ part, int chunks, size_t m,
                                     size_t n, void* c, int64_t rsc, int64_t csc, LinearEpi e) {
    const size_t total = m * n;
    for (GridWalk wk(n); wk.idx < total; wk.next()) {
        const size_t idx = wk.idx;
        // sixteen planes' loads in flight at a time (few cells over many chunk planes would
        // otherwise wait on one load per plane); |sum| < chunks 2^31 fits an int64 in any order
        int64_t acc = 0;
        int q = 0;
        for (; q + 16 <= chunks; q += 16) {
            int32_t v[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) v[u] = __ldg(part + (size_t)(q + u) * total + idx);
#pragma unroll
            for (int u = 0; u < 16; ++u) acc += v[u];
        }
        for (; q < chunks; ++q) acc += __ldg(part + (size_t)q * total + idx);
        const size_t i = wk.i, j = wk.j;
        finish_cell(e, c, (int64_t)i * rsc + (int64_t)j * csc, acc);
    }
}

cudaError_t reduce_chunks(const int32_t* part, int chunks, size_t m, size_t n, void* c,
                          int64_t rsc, int64_t csc, const LinearEpi& e, cudaStream_t s) {
    if (m == 0 || n == 0) return cudaSuccess;
    const size_t total = m * n;
    const int grid = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
    reduce_chunks_kernel<<<grid, 256, 0, s>>>(part, chunks, m, n, c, rsc, csc, e);
    return cudaGetLastError();
}

// One thread initialises a barrier expecting one arrival and then waits on it
// without anyone arriving: the wait must give up at the budget and record
// KERR_TIMEOUT_SELFTEST, after which the kernel returns normally.
__global__ void selftest_wait_kernel(int* status, uint64_t budget_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        fence_barrier_init();
        mbar_wait(smem_u32(&bar), 0, budget_ns, status, KERR_TIMEOUT_SELFTEST);
    }
}

cudaError_t selftest_wait(int* status, uint64_t budget_ns, cudaStream_t s) {
    selftest_wait_kernel<<<1, 32, 0, s>>>(status, budget_ns);
    return cudaGetLastError();
}

}  // namespace uor
