"""gemm_selected on the GPU: values bit for bit against the oracle's max-plus GEMM and
witnesses against the restated D-6 reference (least index attaining the maximum), on a
tie-heavy draw, for the one-pass key kernel (Trop<i8>, k <= 65536) and the generic one."""
import numpy as np
import pytest

import uor_b200 as U
from oracle import oracle as orc
from gpu_util import needs_gpu

pytestmark = [pytest.mark.gpu, needs_gpu]

TD = orc.TROP_DTYPES
OUT = {8: U.TROP_I8, 16: U.TROP_I16, 32: U.TROP_I32, 64: U.TROP_I64}


def draw(rng, count, bits, masked, lo=-1, hi=1):
    t = np.zeros(count, dtype=TD[bits])
    t["v"] = rng.integers(lo, hi, size=count, endpoint=True)
    t["f"] = rng.random(count) >= masked
    t["v"][t["f"] == 0] = 0
    return t


def run(m, k, n, ebits=8, obits=32, masked=0.2, seed=0, alpha=(0, True), beta=(0, False),
        lo=-1, hi=1):
    rng = np.random.default_rng(seed)
    a = draw(rng, m * k, ebits, masked, lo, hi)
    b = draw(rng, k * n, ebits, masked, lo, hi)
    c0 = draw(rng, m * n, obits, 0.3, -5, 5)
    got, want = c0.copy(), c0.copy()
    w = np.full(m * n, 12345, np.uint64)
    route = U.Route()
    U.gemm_tropical_selected(OUT[ebits], OUT[obits], a.view(np.uint8), (m, k, k, 1),
                             b.view(np.uint8), (k, n, n, 1), got.view(np.uint8), (m, n, n, 1),
                             w, (m, n, n, 1), alpha, beta, route=route)
    orc.gemm_trop(orc.View(a, m, k, k, 1), orc.View(b, k, n, n, 1), orc.View(want, m, n, n, 1),
                  ebits=ebits, obits=obits, alpha=alpha, beta=beta)
    same = np.array_equal(got["f"], want["f"]) and np.array_equal(
        np.where(got["f"] != 0, got["v"], 0), np.where(want["f"] != 0, want["v"], 0))
    assert same, "values"
    wref = orc.trop_witness(a["v"].reshape(m, k), a["f"].reshape(m, k) != 0,
                            b["v"].reshape(k, n), b["f"].reshape(k, n) != 0)
    assert np.array_equal(w.reshape(m, n), wref), "witness"
    return route


@pytest.mark.parametrize("shape", [(1, 1, 1), (37, 300, 45), (130, 1000, 129), (5, 4097, 3)])
def test_key_kernel_ties(shape):
    route = run(*shape, seed=sum(shape))
    assert route.tile_k == 16


def test_wider_values_and_epilogue():
    run(64, 700, 80, masked=0.05, lo=-64, hi=63, seed=3, alpha=(7, True), beta=(-2, True))
    run(64, 700, 80, obits=64, masked=0.5, seed=4, alpha=(0, False))


def test_generic_elements_and_deep_k():
    run(20, 333, 17, ebits=16, obits=32, seed=5, lo=-300, hi=300)
    run(9, 200, 11, ebits=32, obits=64, seed=6, lo=-(1 << 30), hi=1 << 30)
    route = run(2, 70_000, 3, ebits=8, obits=32, seed=7)  # past the key's index field
    assert route.tile_m == 16


def test_degenerate_rows_and_depth_zero():
    # every term -inf in some rows; k = 0 everywhere
    run(16, 64, 16, masked=0.9, seed=8)
    m, n = 3, 4
    a = np.zeros(0, TD[8])
    w = np.full(m * n, 7, np.uint64)
    c = np.zeros(m * n, TD[32])
    U.gemm_tropical_selected(U.TROP_I8, U.TROP_I32, a.view(np.uint8), (m, 0, 0, 1),
                             a.view(np.uint8), (0, n, n, 1), c.view(np.uint8), (m, n, n, 1),
                             w, (m, n, n, 1))
    assert (w == 0).all() and (c["f"] == 0).all()


def test_witness_view_is_validated():
    a = np.zeros(4, TD[8])
    c = np.zeros(4, TD[32])
    w = np.zeros(4, np.uint64)
    with pytest.raises(U.NotAProduct):
        U.gemm_tropical_selected(U.TROP_I8, U.TROP_I32, a.view(np.uint8), (2, 2, 2, 1),
                                 a.view(np.uint8), (2, 2, 2, 1), c.view(np.uint8), (2, 2, 2, 1),
                                 w, (1, 4, 4, 1))
    with pytest.raises(U.NotAProduct):
        U.gemm_tropical_selected(U.TROP_I8, U.TROP_I32, a.view(np.uint8), (2, 2, 2, 1),
                                 a.view(np.uint8), (2, 2, 2, 1), c.view(np.uint8), (2, 2, 2, 1),
                                 w, (2, 2, 1, 1))
