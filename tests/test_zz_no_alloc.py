"""The no-allocation entry point (uor_b200_gemm_ex_i8_noalloc), through the C ABI.

It serves callers that cannot let a library allocate device memory: hosts that fix
their device memory budget at start-up, and callers relying on the reference's
zero-allocation contract. Its working memory is one fixed static device array, so the
test checks that two calls in a row (the second reusing the array the first left
behind) give exactly what the ordinary entry point gives, and that a product larger
than the array is refused. Collected last on purpose: it must pass both alone in a
fresh process and after every other test.
"""
import ctypes

import numpy as np
import pytest

import uor_b200 as U
from gpu_util import needs_gpu, torch

pytestmark = [pytest.mark.gpu, needs_gpu]

SCRATCH_LIMIT = 9


def _noalloc(out, m, k, n, alpha, a, lda, b, ldb, beta, c, ldc, encode=U.NEAREST, stream=None):
    fn = U.lib().uor_b200_gemm_ex_i8_noalloc
    fn.argtypes = [ctypes.c_int, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                   ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                   ctypes.c_size_t, ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t,
                   ctypes.c_uint32, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn(out, m, k, n, alpha, a.data_ptr(), lda, b.data_ptr(), ldb, beta, c.data_ptr(), ldc,
              encode, stream)


def _reference_entry(out, m, k, n, alpha, a, b, beta, c):
    U.slice_gemm_ex(U.I8, out, m, k, n, alpha, a, k, b, n, beta, c, n)


@pytest.mark.parametrize("out,dtype", [(U.I64, torch.int64 if torch else None),
                                       (U.I32, torch.int32 if torch else None)])
def test_noalloc_matches_the_allocating_entry_on_two_calls(out, dtype):
    m, k, n = 64, 140_000, 96  # past lane depth: two exact chunks live in the static scratch
    for call, (alpha, beta) in enumerate([(1, 0), (3, -2)]):
        a = torch.from_numpy(U.corpus(40 + call, U.CORPUS_I8, m * k)).cuda()
        b = torch.from_numpy(U.corpus(50 + call, U.CORPUS_I8, k * n)).cuda()
        prior = torch.from_numpy(
            U.corpus(60 + call, U.CORPUS_RAW, m * n).astype(np.int64)).to(dtype).cuda()
        got = prior.clone()
        want = prior.clone()
        assert _noalloc(out, m, k, n, alpha, a, k, b, n, beta, got, n) == U.OK
        _reference_entry(out, m, k, n, alpha, a, b, beta, want)
        assert torch.equal(got, want), f"call {call}"


def test_noalloc_shallow_and_refusals():
    m, k, n = 200, 4096, 320
    a = torch.from_numpy(U.corpus(70, U.CORPUS_I8, m * k)).cuda()
    b = torch.from_numpy(U.corpus(71, U.CORPUS_I8, k * n)).cuda()
    got = torch.zeros(m * n, dtype=torch.int32, device="cuda")
    want = torch.zeros(m * n, dtype=torch.int32, device="cuda")
    assert _noalloc(U.I32, m, k, n, 1, a, k, b, n, 0, got, n) == U.OK
    _reference_entry(U.I32, m, k, n, 1, a, b, 0, want)
    assert torch.equal(got, want)
    # chunks * m * n * 4 bytes beyond the fixed array is refused, not allocated
    m2, k2, n2 = 2048, 140_000, 1024
    a2 = torch.zeros(m2 * k2, dtype=torch.int8, device="cuda")
    b2 = torch.zeros(k2 * n2, dtype=torch.int8, device="cuda")
    c2 = torch.zeros(m2 * n2, dtype=torch.int64, device="cuda")
    assert _noalloc(U.I64, m2, k2, n2, 1, a2, k2, b2, n2, 0, c2, n2) == SCRATCH_LIMIT
