"""K4 ((max, +) on CUDA cores) against the oracle and the reference's CX-11 vectors."""
import hashlib
import json
import os

import numpy as np
import pytest

import uor_b200 as U
from oracle import oracle as orc
from gpu_util import needs_gpu, torch

pytestmark = [pytest.mark.gpu, needs_gpu]

TD = orc.TROP_DTYPES
OUT = {8: U.TROP_I8, 16: U.TROP_I16, 32: U.TROP_I32, 64: U.TROP_I64}
MANIFEST = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "cx_manifest.json")))


def rand_trop(rng, count, bits=8, lo=-64, hi=63, masked=0.05):
    t = np.zeros(count, dtype=TD[bits])
    t["v"] = rng.integers(lo, hi, size=count, endpoint=True)
    fin = rng.random(count) >= masked
    t["f"] = fin
    t["v"][~fin] = 0
    return t


def both(ta, av, tb, bv, tc0, cv, ebits=8, obits=32, alpha=(0, True), beta=(0, False),
         mode=U.NEAREST):
    got = tc0.copy()
    want = tc0.copy()
    route = U.Route()
    U.gemm_tropical(OUT[ebits], OUT[obits], ta, av, tb, bv, got, cv, alpha, beta, mode,
                    route=route)
    o = lambda v: -orc.extent(v[0], v[1], v[2], v[3])[0]
    orc.gemm_trop(orc.View(ta, *av, o(av)), orc.View(tb, *bv, o(bv)), orc.View(want, *cv, o(cv)),
                  ebits=ebits, obits=obits, alpha=alpha, beta=beta, mode=mode)
    return got, want, route


def same(x, y):
    """Compare Trop arrays by fields (value only where finite)."""
    return np.array_equal(x["f"], y["f"]) and np.array_equal(np.where(x["f"] != 0, x["v"], 0),
                                                             np.where(y["f"] != 0, y["v"], 0))


NEG_INF = -(1 << 63)
GOLD = 0x9E3779B97F4A7C15


@pytest.mark.parametrize("idx", range(len(MANIFEST["cx11"]["cases"])))
def test_cx11_golden_on_gpu(idx):
    rec = MANIFEST["cx11"]
    case = rec["cases"][idx]
    m, k, n = (case["shape"][x] for x in "mkn")
    order = [(1, 0, 1), (3, 0, 4), (0, 0, 0), (0, 5, 7), (5, 7, 0), (1, 1, 1), (7, 1, 5),
             (35, 1, 35), (3, 7, 11), (13, 17, 19), (23, 29, 31), (2, 97, 3), (1, 1024, 1),
             (4, 4093, 4), (128, 3, 128), (16, 64, 16)]
    seed = rec["seed"] + order.index((m, k, n))

    def draw(length, salt, mask):
        states, _ = orc.xorshift_stream(seed ^ ((salt * GOLD) & orc.MASK64), length)
        vals = (states >> np.uint64(33)).astype(np.int64) % 3 - 1
        i = np.arange(length)
        return np.where(i % mask[0] == mask[1], NEG_INF, vals)

    a = draw(m * k, 1, (rec["mask_a"]["period"], rec["mask_a"]["phase"]))
    b = draw(k * n, 2, (rec["mask_b"]["period"], rec["mask_b"]["phase"]))
    ta = np.zeros(max(m * k, 1), TD[8])
    tb = np.zeros(max(k * n, 1), TD[8])
    ta["f"][: m * k] = a != NEG_INF
    ta["v"][: m * k] = np.where(a != NEG_INF, a, 0)
    tb["f"][: k * n] = b != NEG_INF
    tb["v"][: k * n] = np.where(b != NEG_INF, b, 0)
    tc = np.zeros(max(m * n, 1), TD[64])
    U.gemm_tropical(U.TROP_I8, U.TROP_I64, ta, (m, k, k, 1), tb, (k, n, n, 1), tc, (m, n, n, 1))
    got = np.where(tc["f"][: m * n] != 0, tc["v"][: m * n], NEG_INF).astype("<i8")
    assert "sha256:" + hashlib.sha256(got.tobytes()).hexdigest() == case["expected_sha256"]


def test_tropical_kats_gpu():
    f = lambda vals: np.array([(v, 1) for v in vals], dtype=TD[8])
    c = np.zeros(4, TD[32])
    U.gemm_tropical(U.TROP_I8, U.TROP_I32, f([1, 2, 3, 4]), (2, 2, 2, 1), f([5, 6, 7, 8]),
                    (2, 2, 2, 1), c, (2, 2, 2, 1))
    assert c["v"].tolist() == [9, 10, 11, 12] and c["f"].tolist() == [1, 1, 1, 1]


@pytest.mark.parametrize("shape", [(1, 1, 1), (3, 7, 11), (13, 17, 19), (129, 33, 130),
                                   (200, 300, 257), (256, 512, 384), (5, 0, 7)])
def test_random_i8_against_oracle(shape):
    m, k, n = shape
    rng = np.random.default_rng(m * 7 + n)
    ta = rand_trop(rng, max(m * k, 1))
    tb = rand_trop(rng, max(k * n, 1))
    tc = np.zeros(m * n, TD[32])
    got, want, route = both(ta, (m, k, k, 1), tb, (k, n, n, 1), tc, (m, n, n, 1))
    assert same(got, want)
    assert route.kernel == 3


@pytest.mark.parametrize("obits", [8, 16, 32, 64])
@pytest.mark.parametrize("mode", [U.NEAREST, U.WRAPPING])
def test_outputs_alpha_beta(obits, mode):
    m, k, n = 40, 70, 50
    rng = np.random.default_rng(obits + mode)
    ta = rand_trop(rng, m * k, lo=-128, hi=127, masked=0.2)
    tb = rand_trop(rng, k * n, lo=-128, hi=127, masked=0.2)
    tc0 = rand_trop(rng, m * n, bits=obits, lo=-100, hi=100, masked=0.3)
    for alpha, beta in [((0, True), (0, False)), ((37, True), (5, True)), ((-40, True), (0, True)),
                        ((0, False), (3, True)), ((2**40, True), (-2**40, True))]:
        got, want, _ = both(ta, (m, k, k, 1), tb, (k, n, n, 1), tc0, (m, n, n, 1), 8, obits,
                            alpha, beta, mode)
        assert same(got, want), (alpha, beta)


@pytest.mark.parametrize("ebits", [16, 32, 64])
def test_wide_elements_generic_path(ebits):
    m, k, n = 17, 23, 19
    rng = np.random.default_rng(ebits)
    lim = {16: 30000, 32: 2**31 - 1, 64: 2**62}[ebits]
    ta = rand_trop(rng, m * k, bits=ebits, lo=-lim, hi=lim, masked=0.1)
    tb = rand_trop(rng, k * n, bits=ebits, lo=-lim, hi=lim, masked=0.1)
    tc = np.zeros(m * n, TD[64])
    got, want, _ = both(ta, (m, k, k, 1), tb, (k, n, n, 1), tc, (m, n, n, 1), ebits, 64)
    assert same(got, want)


def test_strided_views():
    m, k, n = 64, 48, 80
    rng = np.random.default_rng(3)
    ta = rand_trop(rng, m * k)
    tb = rand_trop(rng, k * n)
    tc = np.zeros(m * n, TD[32])
    # A read as a transpose, B read backwards
    got, want, _ = both(ta, (m, k, 1, m), tb, (k, n, -n, 1), tc, (m, n, 1, m))
    assert same(got, want)
