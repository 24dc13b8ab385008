/*
 * uor_b200_corpus.h -- deterministic operand generators for tests and benchmarks.
 *
 * Not part of the GEMM surface. They restate the reference's recorded fill
 * (crates/uor-matmul-validate/tests/common/mod.rs:9-19): s = 0x243F6A8885A308D3 ^ salt,
 * then per element s ^= s << 13; s ^= s >> 7; s ^= s << 17; v = s >> 33, so that
 * benchmark operands are the reference corpus's operands. Host-side C, no GPU.
 */
#ifndef UOR_B200_CORPUS_H
#define UOR_B200_CORPUS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum uor_b200_corpus_kind {
    UOR_B200_CORPUS_I8 = 0,       /* int8: v as i8 (massive.rs:130) */
    UOR_B200_CORPUS_I32_FULL = 1, /* int32: (s as u32) as i32, the full range */
    UOR_B200_CORPUS_RAW = 2,      /* uint64: v itself */
    UOR_B200_CORPUS_NIBBLES = 3,  /* uint8 codes: nibble i = v & 0xF, two per byte, low first */
    UOR_B200_CORPUS_TROP_I8 = 4,  /* Trop<i8>: (v mod 128) - 64, -inf when (v >> 20) mod 100 < 5 */
    UOR_B200_CORPUS_F32_WIDE = 5  /* float: sign s & 1, mantissa 2^23 + ((s >> 33) mod 2^23),
                                     exponent ((s >> 8) mod 61) - 30: value +-m * 2^(e - 23) */
} uor_b200_corpus_kind;

/* Write `count` elements of `kind` (count = nibbles for NIBBLES). Returns 0, or 7 on a bad kind. */
int uor_b200_corpus_fill(uint64_t salt, uint32_t kind, size_t count, void *out);

#ifdef __cplusplus
}
#endif

#endif
