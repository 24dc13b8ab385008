// int_gemm.h -- device-pointer drivers of the integer family.
#pragma once
#include <cstddef>
#include <cstdint>
#include "internal.h"
#include "int_epilogue.cuh"

namespace uor {

// s8 x s8 GEMM through K1. Pointers are device pointers to element (0,0);
// strides are element strides. The Linear epilogue `epi` writes C.
int run_i8_gemm(uor_b200_ctx* ctx, const int8_t* a, ptrdiff_t rsa, ptrdiff_t csa,
                const int8_t* b, ptrdiff_t rsb, ptrdiff_t csb, void* c, ptrdiff_t rsc,
                ptrdiff_t csc, size_t m, size_t k, size_t n, const LinearEpi& epi,
                uor_b200_route* route);

// i16 / i32 / i64 GEMM (eb = element bytes): the modular route (residue GEMMs and the
// CRT) where it runs fewer GEMMs, else byte slicing through the slice-pair kernel and an
// exact recombination in the element's accumulator. route_flags: UOR_B200_DIGIT_SLICES
// keeps the byte slices, UOR_B200_MODULAR takes the modular route wherever it applies. With `cplx` the
// operands and C are Complex<T> / Complex<O> (eb = bytes of one part; strides and
// m, k, n in complex elements).
int run_wide_gemm(uor_b200_ctx* ctx, int eb, const uint8_t* a, ptrdiff_t rsa, ptrdiff_t csa,
                  const uint8_t* b, ptrdiff_t rsb, ptrdiff_t csb, void* c, ptrdiff_t rsc,
                  ptrdiff_t csc, size_t m, size_t k, size_t n, const LinearEpi& epi,
                  uor_b200_route* route, bool cplx = false, uint32_t route_flags = 0);

// Products with at most 16 rows or columns (k > 0): dp4a kernels on CUDA cores that
// keep every SM busy where a tensor-core tile would be mostly padding. Returns
// UOR_B200_UNSUPPORTED when the operands' layout suits neither factorization.
bool i8_skinny_applies(size_t m, size_t k, size_t n);
int run_i8_skinny(uor_b200_ctx* ctx, const int8_t* a, ptrdiff_t rsa, ptrdiff_t csa, const int8_t* b,
                  ptrdiff_t rsb, ptrdiff_t csb, void* c, ptrdiff_t rsc, ptrdiff_t csc, size_t m,
                  size_t k, size_t n, const LinearEpi& epi, uor_b200_route* route);

struct Operand;

// Host-pointer i8 GEMM with the copies pipelined against the compute (row-major
// operands with unit column strides, at least 4 Mi output cells).
bool i8_pipeline_applies(const Operand& A, const Operand& B, const Operand& C);
int run_i8_gemm_pipelined(uor_b200_ctx* ctx, const Operand& A, const Operand& B, const Operand& C,
                          const LinearEpi& epi, uor_b200_route* route);

}  // namespace uor
