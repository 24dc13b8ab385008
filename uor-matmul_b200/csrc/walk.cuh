// walk.cuh -- grid-stride walks over a row-major range without a division per element.
#pragma once
#include <cstddef>
#include <cuda_runtime.h>

namespace uor {

// idx = i * n + j over a row-major range with rows of n, one thread per element, strided
// by the whole grid: the first (i, j) costs one division, every later step adds the
// stride's quotient and remainder with one compare (a 64-bit division per element would
// otherwise be a long software sequence in every iteration).
struct GridWalk {
    size_t idx, i, j, n, step, step_i, step_j;
    __device__ __forceinline__ explicit GridWalk(size_t cols) : n(cols) {
        idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
        step = static_cast<size_t>(gridDim.x) * blockDim.x;
        i = idx / n;
        j = idx - i * n;
        step_i = step / n;
        step_j = step - step_i * n;
    }
    // Cells first, first + stride, ... (a walk whose threads cover unequal spans).
    __device__ __forceinline__ GridWalk(size_t cols, size_t first, size_t stride) : n(cols) {
        idx = first;
        step = stride;
        i = idx / n;
        j = idx - i * n;
        step_i = step / n;
        step_j = step - step_i * n;
    }
    __device__ __forceinline__ void next() {
        idx += step;
        i += step_i;
        j += step_j;
        if (j >= n) {
            j -= n;
            ++i;
        }
    }
};

}  // namespace uor
