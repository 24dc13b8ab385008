"""The no-allocation entry point (uor_b200_gemm_ex_i8_noalloc), through the C ABI.

It serves callers that cannot let a library allocate device memory: hosts that fix
their device memory budget at start-up, and callers relying on the reference's
zero-allocation contract. Its working memory is one fixed static device array, so the
tests make two calls in a row (the second reusing the array the first left behind)
and check each against the CPU oracle bit for bit, and against the ordinary
allocating entry point; a product larger than the array is refused. Collected last on
purpose: it must pass both alone in a fresh process and after every other test.
"""
import ctypes

import numpy as np
import pytest

import uor_b200 as U
from gpu_util import i128_values, needs_gpu, oracle_int, torch

pytestmark = [pytest.mark.gpu, needs_gpu]

SCRATCH_LIMIT = 9
TORCH_OUT = {U.I8: "int8", U.I16: "int16", U.I32: "int32", U.I64: "int64", U.I128: "int64"}
NP_OUT = {U.I8: np.int8, U.I16: np.int16, U.I32: np.int32, U.I64: np.int64, U.I128: np.int64}


def _noalloc(out, m, k, n, alpha, a, lda, b, ldb, beta, c, ldc, encode=U.NEAREST, stream=None):
    fn = U.lib().uor_b200_gemm_ex_i8_noalloc
    fn.argtypes = [ctypes.c_int, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                   ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                   ctypes.c_size_t, ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t,
                   ctypes.c_uint32, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn(out, m, k, n, alpha, a.data_ptr(), lda, b.data_ptr(), ldb, beta, c.data_ptr(), ldc,
              encode, stream)


def _prior(out, salt, cells):
    """A prior C with values spread over the whole output range."""
    raw = U.corpus(salt, U.CORPUS_RAW, cells * (2 if out == U.I128 else 1)).astype(np.uint64)
    wide = (raw << np.uint64(31)) ^ raw
    return wide.view(np.int64).astype(NP_OUT[out], casting="unsafe")


def _same(out, x, y):
    if out == U.I128:
        return i128_values(x) == i128_values(y)
    return np.array_equal(x, y)


def _check_two_calls(out, mode, m, k, n, lda, ldb, ldc, scalars, salt):
    for call, (alpha, beta) in enumerate(scalars):
        a = U.corpus(salt + call, U.CORPUS_I8, m * lda)
        b = U.corpus(salt + 10 + call, U.CORPUS_I8, k * ldb)
        prior = _prior(out, salt + 20 + call, m * ldc)
        want = prior.copy()
        oracle_int(a, (m, k, lda, 1, 0), b, (k, n, ldb, 1, 0), want, (m, n, ldc, 1, 0), alpha,
                   beta, mode, out)
        dt = getattr(torch, TORCH_OUT[out])
        got = torch.from_numpy(prior.copy()).to(dt).cuda()
        ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        assert _noalloc(out, m, k, n, alpha, ta, lda, tb, ldb, beta, got, ldc, mode) == U.OK
        assert _same(out, got.cpu().numpy(), want), f"call {call} vs the oracle"
        # and the same bytes as the allocating entry point
        ordinary = torch.from_numpy(prior.copy()).to(dt).cuda()
        U.slice_gemm_ex(U.I8, out, m, k, n, alpha, ta, lda, tb, ldb, beta, ordinary, ldc,
                        encode=mode)
        assert torch.equal(got, ordinary), f"call {call} vs uor_b200_slice_gemm_ex"


@pytest.mark.parametrize("out", [U.I8, U.I16, U.I32, U.I64, U.I128])
@pytest.mark.parametrize("mode", [U.NEAREST, U.SATURATING, U.WRAPPING])
def test_noalloc_deep_product_two_calls_against_the_oracle(out, mode):
    # past the s32 lane depth: two exact chunks live in the static scratch, and the
    # second call reuses what the first left there
    _check_two_calls(out, mode, 64, 140_000, 96, 140_000, 96, 96, [(1, 0), (3, -2)], 40)


def test_noalloc_padded_output_rows_and_one_row():
    # ldc > n leaves the gaps as they were; m == 1 takes the single-row stride path
    _check_two_calls(U.I64, U.NEAREST, 48, 140_000, 80, 140_000, 80, 83,
                     [(1, 1), (-5, 2)], 140)
    _check_two_calls(U.I32, U.SATURATING, 1, 262_200, 128, 262_200, 128, 128,
                     [(1, 0), (2**40, -1)], 160)


def test_noalloc_shallow_and_refusals():
    _check_two_calls(U.I32, U.NEAREST, 200, 4096, 320, 4096, 320, 320, [(1, 0), (7, 1)], 70)
    # chunks * m * n * 4 bytes beyond the fixed array is refused, not allocated
    m2, k2, n2 = 2048, 140_000, 1024
    a2 = torch.zeros(m2 * k2, dtype=torch.int8, device="cuda")
    b2 = torch.zeros(k2 * n2, dtype=torch.int8, device="cuda")
    c2 = torch.zeros(m2 * n2, dtype=torch.int64, device="cuda")
    assert _noalloc(U.I64, m2, k2, n2, 1, a2, k2, b2, n2, 0, c2, n2) == SCRATCH_LIMIT
