// splitk.cuh -- exact partial sums exchanged between devices as radix-2^40 limbs.
//
// A split-K product hands each device a range of the reduction. Its exact partial sum
// X_r (an i128 for i8/i16/i32 elements) is written as three int64 limbs
//   X_r = l0 + l1 2^40 + l2 2^80,  l0, l1 in [0, 2^40),  l2 = X_r >> 80 (signed),
// so that an elementwise int64 sum over up to 2^23 devices cannot overflow and the
// summed limbs still name sum_r X_r exactly. The finish carries the limbs back into
// one i128 and runs the Linear epilogue once, as the single-device call would
// (Linear::finish, epilogue.rs:79-93, over the exact total: kernel.rs:1431's fold of
// lane-depth chunks, extended across devices).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>
#include "int_epilogue.cuh"

namespace uor {

constexpr int SPLITK_LIMBS = 3;
constexpr int SPLITK_LIMB_BITS = 40;

// x: cells little-endian i128 values (16 bytes each) -> limbs[cell][3].
cudaError_t i128_to_limbs(const void* x, int64_t* limbs, size_t cells, cudaStream_t s);

// limbs[i * n + j][3] (summed over devices) -> C(i, j) := encode(alpha X + beta C).
cudaError_t limbs_finish(const int64_t* limbs, size_t m, size_t n, void* c, int64_t rsc,
                         int64_t csc, const LinearEpi& e, cudaStream_t s);

}  // namespace uor
