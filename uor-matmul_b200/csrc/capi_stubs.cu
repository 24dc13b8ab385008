// capi_stubs.cu -- entry points whose kernels are not built yet. Each returns
// UOR_B200_UNSUPPORTED after the same validation its real body will perform,
// so a caller can probe the surface without a silent CPU path.
#include "internal.h"

extern "C" {

int uor_b200_gemm_float(uor_b200_dtype, uor_b200_dtype, const uor_b200_view*,
                        const uor_b200_view*, const uor_b200_view_mut*, int64_t, int64_t,
                        const uor_b200_call*) {
    return UOR_B200_UNSUPPORTED;
}

int uor_b200_slice_gemm_float_ex(uor_b200_dtype, uor_b200_dtype, size_t, size_t, size_t, int64_t,
                                 const void*, size_t, size_t, const void*, size_t, size_t, int64_t,
                                 void*, size_t, size_t, void*, size_t, void*, size_t,
                                 const uor_b200_call*) {
    return UOR_B200_UNSUPPORTED;
}

int uor_b200_sgemm(size_t, size_t, size_t, int64_t, const float*, ptrdiff_t, ptrdiff_t,
                   const float*, ptrdiff_t, ptrdiff_t, int64_t, float*, ptrdiff_t, ptrdiff_t,
                   const uor_b200_call*) {
    return UOR_B200_UNSUPPORTED;
}

int uor_b200_dgemm(size_t, size_t, size_t, int64_t, const double*, ptrdiff_t, ptrdiff_t,
                   const double*, ptrdiff_t, ptrdiff_t, int64_t, double*, ptrdiff_t, ptrdiff_t,
                   const uor_b200_call*) {
    return UOR_B200_UNSUPPORTED;
}

}  // extern "C"
