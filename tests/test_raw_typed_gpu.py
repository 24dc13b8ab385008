"""The typed raw-face spellings (uor_b200_raw_gemm_<E>_<O>, _trop_i8_i32, the packed-grid
coded and tabulated forms): each, called with a pointer at element (0,0) and strides of
both signs (B read as its transpose, C's rows written bottom-up), gives the generic entry's
bytes, and those equal the oracle's; empty products and self-aliasing outputs return
without writing, as the raw face does."""
import ctypes

import numpy as np
import pytest

import uor_b200 as U
from oracle import oracle as orc
from gpu_util import needs_gpu

pytestmark = [pytest.mark.gpu, needs_gpu]

NP = {U.I8: np.int8, U.I16: np.int16, U.I32: np.int32, U.I64: np.int64}
OUT = {U.I32: (np.int32, 1), U.I64: (np.int64, 1), U.I128: (np.int64, 2)}


def _ptr(arr, elem_offset=0, es=None):
    es = es or arr.itemsize
    return arr.ctypes.data + elem_offset * es


@pytest.mark.parametrize("elem,out", [(U.I8, U.I32), (U.I8, U.I64), (U.I16, U.I64), (U.I32, U.I64),
                                      (U.I32, U.I128), (U.I64, U.I128)])
def test_raw_int_spellings_equal_the_generic_call(elem, out):
    name = {U.I8: "i8", U.I16: "i16", U.I32: "i32", U.I64: "i64"}[elem] + "_" + \
        {U.I32: "i32", U.I64: "i64", U.I128: "i128"}[out]
    fn = getattr(U.lib(), "uor_b200_raw_gemm_" + name)
    m, k, n = 37, 300, 45
    kind = U.CORPUS_I8 if elem == U.I8 else U.CORPUS_I32_FULL
    a = U.corpus(11, kind, m * k).astype(NP[elem], casting="unsafe")
    bt = U.corpus(12, kind, k * n).astype(NP[elem], casting="unsafe")  # stored n x k
    dt, w = OUT[out]
    prior = U.corpus(13, U.CORPUS_I32_FULL, m * n * w).astype(dt, casting="unsafe")
    want = prior.copy()
    U.gemm(elem, out, a, (m, k, k, 1), bt, (k, n, 1, k), want, (m, n, n, 1), 3, -1, U.SATURATING)
    # C written bottom-up: element (0, 0) is the first cell of the buffer's last row
    got = prior.reshape(m, n * w)[::-1].copy().reshape(-1)
    call = U.make_call(U.SATURATING, False, None, None, False)
    st = fn(m, k, n, 3, _ptr(a), k, 1, _ptr(bt), 1, k, -1, _ptr(got, (m - 1) * n * w), -n, 1,
            ctypes.byref(call))
    assert st == U.OK
    assert np.array_equal(got.reshape(m, n * w)[::-1].reshape(-1), want), name
    # the oracle agrees with the generic entry
    if out != U.I128:
        ref = prior.copy()
        orc.gemm_int(orc.View(a, m, k, k, 1), orc.View(bt, k, n, 1, k), orc.View(ref, m, n, n, 1),
                     alpha=3, beta=-1, mode=U.SATURATING, out_bits=8 * np.dtype(dt).itemsize)
        assert np.array_equal(ref, want)
    # empty products and a self-aliasing output return without writing
    before = got.copy()
    assert fn(0, k, n, 3, _ptr(a), k, 1, _ptr(bt), 1, k, -1, _ptr(got), n, 1, ctypes.byref(call)) == U.OK
    assert fn(m, k, n, 3, _ptr(a), k, 1, _ptr(bt), 1, k, -1, _ptr(got), 0, 1, ctypes.byref(call)) == U.OK
    assert np.array_equal(got, before)


def test_raw_trop_and_codec_spellings_equal_the_generic_calls():
    lib = U.lib()
    TD = orc.TROP_DTYPES
    m, k, n = 33, 200, 40
    raw = U.corpus(21, U.CORPUS_RAW, m * k)
    a = np.zeros(m * k, TD[8])
    a["v"] = (raw % np.uint64(128)).astype(np.int64) - 64
    a["f"] = (raw >> np.uint64(20)) % np.uint64(100) >= np.uint64(5)
    raw = U.corpus(22, U.CORPUS_RAW, k * n)
    b = np.zeros(k * n, TD[8])
    b["v"] = (raw % np.uint64(128)).astype(np.int64) - 64
    b["f"] = (raw >> np.uint64(20)) % np.uint64(100) >= np.uint64(5)
    want = np.zeros(m * n, TD[32])
    U.gemm_tropical(U.TROP_I8, U.TROP_I32, a.view(np.uint8), (m, k, k, 1), b.view(np.uint8),
                    (k, n, n, 1), want.view(np.uint8), (m, n, n, 1), (5, True), (0, False))
    got = np.zeros(m * n, TD[32])
    call = U.make_call(U.NEAREST, False, None, None, False)
    st = lib.uor_b200_raw_gemm_trop_i8_i32(m, k, n, U.Trop(5, 1), a.ctypes.data, k, 1, b.ctypes.data,
                                           n, 1, U.Trop(0, 0), got.ctypes.data, n, 1,
                                           ctypes.byref(call))
    assert st == U.OK
    assert np.array_equal(got.view(np.uint8), want.view(np.uint8))

    m, k, n = 64, 256, 96
    x = U.corpus(1, U.CORPUS_I8, m * k)
    codes = U.corpus(2, U.CORPUS_NIBBLES, k * n)
    table = U.corpus(7, U.CORPUS_I8, 16)
    for tab in (False, True):
        want = np.zeros(m * n, np.int32)
        U.coded_gemm(U.I32, x, (m, k, k, 1), codes, k, n, 2, table, want, (m, n, n, 1), 2, 0,
                     tabulated=tab)
        got = np.zeros(m * n, np.int32)
        fn = lib.uor_b200_raw_tabulated_grid16_i8_i32 if tab else lib.uor_b200_raw_coded_grid16_i8_i32
        # A read through a negative row stride: element (0, 0) starts the buffer's last row
        xr = x.reshape(m, k)[::-1].copy().reshape(-1)
        st = fn(m, k, n, 2, _ptr(xr, (m - 1) * k), -k, 1, codes.ctypes.data, table.ctypes.data, 0,
                got.ctypes.data, n, 1, ctypes.byref(call))
        assert st == U.OK
        assert np.array_equal(got, want), tab
