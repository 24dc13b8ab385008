// float_exact.h -- the exact float family's device driver.
#pragma once
#include <cstddef>
#include <cstdint>
#include "int_epilogue.cuh"
#include "internal.h"

namespace uor {

// The Linear epilogue of the float family and the output view.
struct FxEpi {
    int64_t alpha, beta;
    int mode;
    bool e64, out64;   // element and output formats
    int min_exp_e;     // bit-0 exponent of the element's register (-298 f32, -2148 f64)
    int limbs_e;       // its low limb count (10 f32, 67 f64)
    void* c;
    int64_t rsc, csc;
};

// The exact float product: the modular route (Ozaki scheme II) where its moduli cover the
// operands' exponent spans and it runs fewer GEMMs, else the digit-slice route, else the
// direct route. route_flags: UOR_B200_DIGIT_SLICES skips the modular route,
// UOR_B200_MODULAR takes it wherever the moduli cover the spans.
int run_float_gemm(uor_b200_ctx* ctx, bool e64, bool o64, const uint8_t* a, ptrdiff_t rsa,
                   ptrdiff_t csa, const uint8_t* b, ptrdiff_t rsb, ptrdiff_t csb, void* c,
                   ptrdiff_t rsc, ptrdiff_t csc, size_t m, size_t k, size_t n, int64_t alpha,
                   int64_t beta, int mode, uor_b200_route* route, uint32_t route_flags = 0);

}  // namespace uor
