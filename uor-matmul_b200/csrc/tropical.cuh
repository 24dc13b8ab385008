// tropical.cuh -- K4 launchers.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include "int_epilogue.cuh"

namespace uor {

// MaxPlus{alpha, beta} and the output view (Trop<O>, obytes = sizeof(O)).
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

}  // namespace uor
