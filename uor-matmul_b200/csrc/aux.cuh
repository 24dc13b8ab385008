// aux.cuh -- small HBM-bound helper kernels around the tensor-core GEMMs.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include "int_epilogue.cuh"

namespace uor {

// Copy a strided view of `esize`-byte elements into a dense [rows][ld] buffer.
// Used when an operand's strides cannot be described to TMA (negative, zero,
// unaligned, or neither dimension unit-stride).
cudaError_t gather_2d(void* dst, size_t ld, const void* src_origin, size_t rows, size_t cols,
                      ptrdiff_t rs, ptrdiff_t cs, int esize, cudaStream_t s);

// The k == 0 product: every accumulator is zero, so C := encode(beta * C)
// (and C is not read when beta == 0).
cudaError_t epilogue_only(void* c, int64_t rsc, int64_t csc, size_t m, size_t n,
                          const LinearEpi& e, cudaStream_t s);

// C := encode(alpha * sum_c part[c] + beta * C) for s32 chunk planes
// part[chunks][m][n]: the exact combine of lane-depth chunks (kernel.rs:1431).
cudaError_t reduce_chunks(const int32_t* part, int chunks, size_t m, size_t n, void* c,
                          int64_t rsc, int64_t csc, const LinearEpi& e, cudaStream_t s);

// A kernel that waits on an mbarrier nothing completes, with a bounded wait.
cudaError_t selftest_wait(int* status, uint64_t budget_ns, cudaStream_t s);

}  // namespace uor
