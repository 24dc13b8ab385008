// tropical.cuh -- K4 launchers.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include "int_epilogue.cuh"

namespace uor {

// MaxPlus{alpha, beta} and the output view (Trop<O>, obytes = sizeof(O)). obytes == 0
// selects the split-K key output: int64 per cell, the raw reduction (alpha and beta are
// not applied) or INT64_MIN where no term is finite.
struct TropEpi {
    int64_t alpha, beta;
    int alpha_finite, beta_finite;
    int mode;
    int obytes;
    void* c;
    int64_t rsc, csc;
    int m, n;
};

// Trop<i8> x Trop<i8>: packed 16-bit lanes; `ws` holds trop_i8_workspace() bytes.
cudaError_t trop_i8_launch(const uint8_t* a, int64_t rsa, int64_t csa, const uint8_t* b,
                           int64_t rsb, int64_t csb, int m, int k, int n, void* ws,
                           const TropEpi& e, cudaStream_t s);
size_t trop_i8_workspace(int m, int k, int n);

// Any Trop<E> (ebytes = sizeof(E)), exact in 128-bit arithmetic.
cudaError_t trop_generic_launch(const uint8_t* a, int64_t rsa, int64_t csa, const uint8_t* b,
                                int64_t rsb, int64_t csb, int ebytes, int m, int k, int n,
                                const TropEpi& e, cudaStream_t s);

// driver::gemm_selected (crates/uor-matmul-gemm/src/selection.rs:212-330): the product
// and, per cell, the least index attaining the maximum of the reduction (D-6); 0 when
// every term is the semiring zero or k is 0. `w` is the witness (u64) view's origin.
// Trop<i8> with k <= 65536: one pass over (value, index) keys; `ws` holds
// trop_witness_workspace() bytes.
cudaError_t trop_i8_witness_launch(const uint8_t* a, int64_t rsa, int64_t csa, const uint8_t* b,
                                   int64_t rsb, int64_t csb, int m, int k, int n, void* ws,
                                   const TropEpi& e, uint64_t* w, int64_t rsw, int64_t csw,
                                   cudaStream_t s);
size_t trop_witness_workspace(int m, int k, int n);
constexpr int TROP_WITNESS_MAX_K = 65536;
// Any Trop<E>, any k: one thread per cell.
cudaError_t trop_generic_witness_launch(const uint8_t* a, int64_t rsa, int64_t csa,
                                        const uint8_t* b, int64_t rsb, int64_t csb, int ebytes,
                                        int m, int k, int n, const TropEpi& e, uint64_t* w,
                                        int64_t rsw, int64_t csw, cudaStream_t s);

// MaxPlus::finish and the encode into e's output view, from int64 keys (m x n, row-major;
// INT64_MIN = no finite term), e.g. the element-wise max of several ranges' keys.
cudaError_t trop_keys_finish_launch(const int64_t* keys, const TropEpi& e, cudaStream_t s);

}  // namespace uor
