"""K2/K3 (byte-sliced i16 / i32 / i64 GEMM with exact recombination) against the
oracle and the reference's CX-10 NumPy vectors."""
import hashlib
import json
import os

import numpy as np
import pytest

import uor_b200 as U
from oracle import oracle as orc
from gpu_util import i128_values, needs_gpu, oracle_int, out_array, torch

pytestmark = [pytest.mark.gpu, needs_gpu]

MANIFEST = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "cx_manifest.json")))
ELEM = {16: U.I16, 32: U.I32, 64: U.I64}
NP = {16: np.int16, 32: np.int32, 64: np.int64}


def cx10_cases():
    s = MANIFEST["cx10"]["seed"]
    for case in MANIFEST["cx10"]["cases"]:
        m, k, n = (case["shape"][x] for x in "mkn")
        states, s = orc.xorshift_stream(s, m * k + k * n)
        vals = (states >> np.uint64(33)).astype(np.int64) % 1000 - 500
        yield case, vals[: m * k], vals[m * k:]


@pytest.mark.parametrize("idx", range(len(MANIFEST["cx10"]["cases"])))
def test_cx10_i64_wrapping_on_gpu(idx):
    case, a, b = list(cx10_cases())[idx]
    m, k, n = (case["shape"][x] for x in "mkn")
    c = np.zeros(max(m * n, 1), np.int64)
    if m and n:
        U.slice_gemm_ex(U.I64, U.I64, m, k, n, 1, a, k, b, n, 0, c, n, encode=U.WRAPPING)
    got = c[: m * n].astype("<i8")
    assert "sha256:" + hashlib.sha256(got.tobytes()).hexdigest() == case["expected_sha256"]


def rand_full(rng, bits, count):
    info = np.iinfo(NP[bits])
    return rng.integers(info.min, info.max, size=count, endpoint=True).astype(NP[bits])


@pytest.mark.parametrize("path", ["auto", "digits", "modular"])
@pytest.mark.parametrize("bits", [16, 32, 64])
@pytest.mark.parametrize("out", [U.I32, U.I64, U.I128])
def test_random_full_range(bits, out, path):
    """The byte-slice pairs (forced, and for i16 always), the modular route (residue GEMMs
    and the CRT, forced for i32 / i64) and the library's own choice."""
    rng = np.random.default_rng(bits * 10 + out)
    for (m, k, n) in [(1, 1, 1), (13, 17, 19), (130, 300, 270), (300, 200, 261)]:
        a, b = rand_full(rng, bits, m * k), rand_full(rng, bits, k * n)
        c0 = out_array(out, m * n)
        c0[:] = rng.integers(-1000, 1000, size=c0.size)
        for alpha, beta, mode in [(1, 0, U.NEAREST), (3, -1, U.WRAPPING), (-(2**63), 5, U.NEAREST),
                                  (2**62, 2**62, U.SATURATING)]:
            got, want = c0.copy(), c0.copy()
            route = U.Route()
            U.gemm(ELEM[bits], out, a, (m, k, k, 1), b, (k, n, n, 1), got, (m, n, n, 1), alpha,
                   beta, mode, route=route, digits=path == "digits", modular=path == "modular")
            oracle_int(a, (m, k, k, 1, 0), b, (k, n, n, 1, 0), want, (m, n, n, 1, 0), alpha, beta,
                       mode, out)
            if out == U.I128:
                assert i128_values(got) == i128_values(want), (m, k, n, alpha, beta, mode)
            else:
                assert np.array_equal(got, want), (m, k, n, alpha, beta, mode)
            assert route.kernel == 2
            if path == "digits" or bits == 16:
                assert route.moduli == 0, route.as_dict()
            elif path == "modular":
                assert route.moduli > 0, route.as_dict()


@pytest.mark.parametrize("digits", [False, True])
def test_deep_i32_chunks_and_strides(digits):
    rng = np.random.default_rng(5)
    m, k, n = 40, 30000, 24
    a, b = rand_full(rng, 32, m * k), rand_full(rng, 32, k * n)
    got = np.zeros(m * n * 2, np.int64)
    want = got.copy()
    route = U.Route()
    # B read as its own transpose: stored n x k
    bt = np.ascontiguousarray(b.reshape(k, n).T).reshape(-1)
    U.gemm(U.I32, U.I128, a, (m, k, k, 1), bt, (k, n, 1, k), got, (m, n, n, 1), route=route,
           digits=digits, modular=not digits)
    oracle_int(a, (m, k, k, 1, 0), bt, (k, n, 1, k, 0), want, (m, n, n, 1, 0), 1, 0, U.NEAREST,
               U.I128)
    assert i128_values(got) == i128_values(want)
    # byte slices: an s32 diagonal lane holds ~8 Ki products; residues: 1023 blocks of 128
    # hold k, and the few tiles split it further so the waves fill (ks_balance_chunks)
    assert route.k_chunks >= 3 if digits else (route.k_chunks > 1 and route.moduli > 0)


def test_modular_two_chunks_and_i64_extremes():
    """k past 1023 blocks of 128 splits the residue GEMMs into two chunks summed in the
    CRT; i64 MIN / MAX everywhere drive |S| to its bound k 2^126."""
    rng = np.random.default_rng(9)
    m, k, n = 5, 140000, 7
    a, b = rand_full(rng, 32, m * k), rand_full(rng, 32, k * n)
    got, want = np.zeros(m * n * 2, np.int64), np.zeros(m * n * 2, np.int64)
    route = U.Route()
    U.gemm(U.I32, U.I128, a, (m, k, k, 1), b, (k, n, n, 1), got, (m, n, n, 1), route=route,
           modular=True)
    oracle_int(a, (m, k, k, 1, 0), b, (k, n, n, 1, 0), want, (m, n, n, 1, 0), 1, 0, U.NEAREST,
               U.I128)
    assert i128_values(got) == i128_values(want)
    assert route.k_chunks >= 2 and route.moduli > 0
    m, k, n = 9, 3000, 11
    lo, hi = np.iinfo(np.int64).min, np.iinfo(np.int64).max
    a = rng.choice([lo, hi, lo + 1, -1, 0], size=m * k).astype(np.int64)
    b = rng.choice([lo, hi, lo], size=k * n).astype(np.int64)
    for mode in (U.NEAREST, U.WRAPPING):
        got, want = np.zeros(m * n * 2, np.int64), np.zeros(m * n * 2, np.int64)
        route = U.Route()
        U.gemm(U.I64, U.I128, a, (m, k, k, 1), b, (k, n, n, 1), got, (m, n, n, 1), 3, 0, mode,
               route=route, modular=True)
        oracle_int(a, (m, k, k, 1, 0), b, (k, n, n, 1, 0), want, (m, n, n, 1, 0), 3, 0, mode,
                   U.I128)
        assert i128_values(got) == i128_values(want), mode
        assert route.moduli > 0
