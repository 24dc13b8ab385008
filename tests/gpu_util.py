"""Shared helpers for the GPU parity tests (the oracle is the checker)."""
import numpy as np
import pytest

import uor_b200 as U
from oracle import oracle as orc
from oracle.oracle import View

try:
    import torch
    HAVE_CUDA = torch.cuda.is_available()
except Exception:  # pragma: no cover
    torch = None
    HAVE_CUDA = False

needs_gpu = pytest.mark.skipif(not HAVE_CUDA, reason="needs a CUDA device")

NP_OUT = {U.I8: np.int8, U.I16: np.int16, U.I32: np.int32, U.I64: np.int64}


def out_array(out, count):
    if out == U.I128:
        return np.zeros(count * 2, dtype=np.int64)  # 16-byte little-endian pairs
    return np.zeros(count, dtype=NP_OUT[out])


def i128_values(arr):
    lo = arr[0::2].astype(np.uint64).astype(object)
    hi = arr[1::2].astype(object)
    return [int(h) * (1 << 64) + int(l) for l, h in zip(lo, hi)]


def oracle_int(a, av, b, bv, c, cv, alpha, beta, mode, out):
    """Run the C oracle over the same buffers/views (views are (rows, cols, rs, cs, origin))."""
    obits = {U.I8: 8, U.I16: 16, U.I32: 32, U.I64: 64, U.I128: 128}[out]
    A = View(a, av[0], av[1], av[2], av[3], av[4] if len(av) > 4 else 0)
    B = View(b, bv[0], bv[1], bv[2], bv[3], bv[4] if len(bv) > 4 else 0)
    C = View(c, cv[0], cv[1], cv[2], cv[3], cv[4] if len(cv) > 4 else 0)
    orc.gemm_int(A, B, C, alpha=alpha, beta=beta, mode=mode, out_bits=obits)


def i8(salt, count):
    return U.corpus(salt, U.CORPUS_I8, count)
