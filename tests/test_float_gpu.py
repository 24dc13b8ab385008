"""K6 + K7 (exact float GEMM, one rounding) against the oracle, bit for bit."""
import struct

import numpy as np
import pytest

import uor_b200 as U
from oracle import oracle as orc
from oracle.oracle import View
from float_data import config3
from gpu_util import needs_gpu, torch

pytestmark = [pytest.mark.gpu, needs_gpu]

FT = {U.F32: np.float32, U.F64: np.float64}
UT = {U.F32: np.uint32, U.F64: np.uint64}


def run_both(elem, out, a, b, m, k, n, alpha=1, beta=0, c0=None, mode=U.NEAREST, av=None,
             bv=None, digits=False):
    av = av or (m, k, k, 1)
    bv = bv or (k, n, n, 1)
    c0 = np.zeros(m * n, FT[out]) if c0 is None else c0
    got, want = c0.copy(), c0.copy()
    route = U.Route()
    U.gemm_float(elem, out, a, av, b, bv, got, (m, n, n, 1), alpha, beta, mode, route=route,
                 digits=digits)
    oa = -orc.extent(*av)[0]
    ob = -orc.extent(*bv)[0]
    orc.gemm_float(View(a, *av, oa), View(b, *bv, ob), View(want, m, n, n, 1), alpha=alpha,
                   beta=beta, mode=mode)
    return got.view(UT[out]), want.view(UT[out]), route


def f32b(x):
    return struct.unpack("<I", struct.pack("<f", x))[0]


def gpu_f32(a, b, m, k, n, alpha=1, beta=0, c=None, mode=U.NEAREST):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    c = np.zeros(m * n, np.float32) if c is None else np.asarray(c, np.float32).copy()
    U.gemm_float(U.F32, U.F32, a, (m, k, k, 1), b, (k, n, n, 1), c, (m, n, n, 1), alpha, beta,
                 mode)
    return c.view(np.uint32).tolist()


def test_float_kats_on_gpu():
    # epilogue.rs:411-518 and the encode/decode KATs, through the device path
    for mode in (U.NEAREST, U.TOWARD_ZERO, U.SATURATING, U.WRAPPING):
        assert gpu_f32([0.5], [1.0], 1, 1, 1, -(2**63), 2**62, [1.0], mode) == [0]
    big = float(np.finfo(np.float32).max)
    assert gpu_f32([big], [big], 1, 1, 1, 2**63 - 1) == [f32b(float("inf"))]
    assert gpu_f32([big], [big], 1, 1, 1, -(2**63)) == [f32b(float("-inf"))]
    for mode in (U.TOWARD_ZERO, U.SATURATING, U.WRAPPING):
        assert gpu_f32([big], [big], 1, 1, 1, 2**63 - 1, mode=mode) == [f32b(big)]
    assert gpu_f32([float("inf")], [1.0], 1, 1, 1, -1) == [f32b(float("-inf"))]
    assert gpu_f32([float("inf")], [1.0], 1, 1, 1, 0) == [0x7FC00000]
    assert gpu_f32([float("inf")], [0.0], 1, 1, 1) == [0x7FC00000]
    assert gpu_f32([float("inf"), float("inf")], [1.0, -1.0], 1, 2, 1) == [0x7FC00000]
    assert gpu_f32([1.5, 1.5], [2.0, -2.0], 1, 2, 1) == [0]
    e = 2.0 ** -24
    assert gpu_f32([1.0, e, e], [1.0, 1.0, 1.0], 1, 3, 1) == [f32b(1.0 + 2.0 ** -23)]


def rand_bits(rng, count, f64, specials):
    if f64:
        x = rng.integers(0, 2**64, size=count, dtype=np.uint64).view(np.float64).copy()
    else:
        x = rng.integers(0, 2**32, size=count, dtype=np.uint64).astype(np.uint32).view(
            np.float32).copy()
    if not specials:
        x[~np.isfinite(x)] = 1.0
    return x


@pytest.mark.parametrize("elem,out", [(U.F32, U.F32), (U.F64, U.F64), (U.F32, U.F64),
                                      (U.F64, U.F32)])
def test_random_bit_patterns_and_specials(elem, out):
    """Uniform random bit patterns: every exponent (the direct route), NaN, +-inf,
    subnormals, zeros."""
    rng = np.random.default_rng(elem * 10 + out)
    for (m, k, n) in [(1, 1, 1), (5, 7, 3), (9, 33, 17)]:
        for specials in (True, False):
            a = rand_bits(rng, m * k, elem == U.F64, specials)
            b = rand_bits(rng, k * n, elem == U.F64, specials)
            c0 = rand_bits(rng, m * n, out == U.F64, False)
            for alpha, beta, mode in [(1, 0, U.NEAREST), (3, -2, U.TOWARD_ZERO),
                                      (-1, 1, U.NEAREST)]:
                got, want, _ = run_both(elem, out, a, b, m, k, n, alpha, beta, c0, mode)
                assert np.array_equal(got, want), (m, k, n, specials, alpha, beta, mode)


@pytest.mark.parametrize("digits", [False, True])
@pytest.mark.parametrize("elem,out", [(U.F32, U.F32), (U.F64, U.F64), (U.F32, U.F64)])
@pytest.mark.parametrize("shape", [(3, 10, 7), (130, 96, 270), (64, 700, 40), (257, 64, 130)])
def test_moderate_exponents_tensor_route(elem, out, shape, digits):
    """Exponent spans small enough for the tensor cores: the modular route (residues and
    the CRT) and, forced, the digit-slice route."""
    m, k, n = shape
    rng = np.random.default_rng(m + k + n)
    a = (rng.standard_normal(m * k) * np.exp2(rng.integers(-8, 8, m * k))).astype(FT[elem])
    b = (rng.standard_normal(k * n) * np.exp2(rng.integers(-8, 8, k * n))).astype(FT[elem])
    b[::5] = 0.0
    c0 = rng.standard_normal(m * n).astype(FT[out])
    for alpha, beta, mode in [(1, 0, U.NEAREST), (-3, 2, U.NEAREST), (2**40, -1, U.TOWARD_ZERO)]:
        got, want, route = run_both(elem, out, a, b, m, k, n, alpha, beta, c0, mode,
                                    digits=digits)
        assert np.array_equal(got, want), (alpha, beta, mode)
        assert (route.moduli == 0) == digits
        if elem == U.F32:
            # 256-row tiles on CTA pairs past 128 rows, 128-row tiles below
            assert route.kernel == 5 and route.tile_m == (256 if m > 128 else 128)


@pytest.mark.parametrize("digits", [False, True])
def test_nonfinite_on_the_tensor_route(digits):
    m, k, n = 70, 200, 90
    rng = np.random.default_rng(7)
    a = rng.standard_normal(m * k).astype(np.float32)
    b = rng.standard_normal(k * n).astype(np.float32)
    a[5 * k + 3] = np.inf
    a[9 * k + 10] = -np.inf
    b[3 * n + 4] = 0.0
    b[100 * n + 7] = np.nan
    b[50 * n + 11] = -np.inf
    for alpha, beta in ((1, 0), (-2, 3)):
        c0 = rng.standard_normal(m * n).astype(np.float32)
        got, want, route = run_both(U.F32, U.F32, a, b, m, k, n, alpha, beta, c0, digits=digits)
        assert np.array_equal(got, want), (alpha, beta)
        assert route.tile_m == 128 and (route.moduli == 0) == digits


@pytest.mark.parametrize("digits", [False, True])
def test_config3_cancellation_moderate(digits):
    m, k, n = 96, 256, 130
    a, b = config3(m, k, n)
    got, want, route = run_both(U.F32, U.F32, a.reshape(-1), b.reshape(-1), m, k, n,
                                digits=digits)
    assert np.array_equal(got, want)
    for j in range(0, n, 10):
        assert got[(j % m) * n + j] == 0, "an exactly cancelling row encodes +0"


def test_lazy_digits_interval_test_and_exact_fixups():
    """Wide exponent spans take the lazy route: only the top diagonals run on the tensor
    cores, each cell is accepted only when both ends of its error interval encode alike,
    and the rest (here the exactly cancelling cells) are recomputed exactly."""
    m, k, n = 300, 512, 260
    a, b = config3(m, k, n)
    a, b = a.reshape(-1), b.reshape(-1)
    for alpha, mode in [(1, U.NEAREST), (-3, U.NEAREST), (5, U.TOWARD_ZERO)]:
        got, want, route = run_both(U.F32, U.F32, a, b, m, k, n, alpha, 0, None, mode,
                                    digits=True)
        assert np.array_equal(got, want), (alpha, mode)
        assert route.pairs < route.a_layout * route.b_layout, "the low diagonals were skipped"
        assert route.fixups >= n // 10, "every cancelling cell is recomputed exactly"
    # a row and a column of zeros encode +0 without a fixup
    a2, b2 = a.copy(), b.copy()
    a2[7 * k:8 * k] = 0.0
    b2[np.arange(k) * n + 3] = 0.0
    for digits in (True, False):
        got, want, route = run_both(U.F32, U.F32, a2, b2, m, k, n, digits=digits)
        assert np.array_equal(got, want)
        assert (got.reshape(m, n)[7] == 0).all() and (got.reshape(m, n)[:, 3] == 0).all()


def test_lazy_digits_fall_back_when_many_cells_cancel():
    """Every column cancels one of four rows: more unsure cells than the fixup list
    holds, so every diagonal runs on the tensor cores after all -- same bytes."""
    m, k, n = 4, 256, 8192
    a, b = config3(m, k, n)
    kk = k - k % 2
    sign = np.where(np.arange(k) % 2 == 0, 1.0, -1.0).astype(np.float32)
    for j in range(n):
        b[:kk, j] = a[j % m, np.arange(kk) ^ 1] * sign[:kk] * np.float32(2.0 ** ((j % 9) - 4))
    got, want, route = run_both(U.F32, U.F32, a.reshape(-1), np.ascontiguousarray(b).reshape(-1),
                                m, k, n, digits=True)
    assert np.array_equal(got, want)
    assert route.fixups > 4096
    assert route.pairs == route.a_layout * route.b_layout


def test_register_drop_quirk_on_gpu():
    a = np.array([1.0], np.float32)
    b = np.array([2.0], np.float32)
    for prior in (2.0 ** 400, 1.5 * 2.0 ** -297, 3.0):
        c = np.array([prior], np.float64)
        w = c.copy()
        U.gemm_float(U.F32, U.F64, a, (1, 1, 1, 1), b, (1, 1, 1, 1), c, (1, 1, 1, 1), 1, 1)
        orc.gemm_float(View(a, 1, 1, 1, 1), View(b, 1, 1, 1, 1), View(w, 1, 1, 1, 1), beta=1)
        assert c.view(np.uint64)[0] == w.view(np.uint64)[0]


def test_raw_faces_negative_strides():
    m, k, n = 20, 30, 25
    rng = np.random.default_rng(3)
    for dt, fn in ((np.float32, U.sgemm), (np.float64, U.dgemm)):
        a = rng.standard_normal(m * k).astype(dt)
        b = rng.standard_normal(k * n).astype(dt)
        c = rng.standard_normal(m * n).astype(dt)
        want = c.copy()
        # B walked backwards: origin at the last row, rsb = -n
        fn(m, k, n, 3, a, k, 1, b, -n, 1, -1, c, n, 1, origin=(0, (k - 1) * n, 0))
        orc.gemm_float(View(a, m, k, k, 1), View(b, k, n, -n, 1, (k - 1) * n),
                       View(want, m, n, n, 1), alpha=3, beta=-1)
        assert np.array_equal(c.view(np.uint8), want.view(np.uint8))
    # an aliasing output returns without writing (raw.rs:146-148)
    c = np.arange(4, dtype=np.float32)
    U.sgemm(2, 1, 2, 1, np.ones(2, np.float32), 1, 1, np.ones(2, np.float32), 2, 1, 0, c, 0, 1)
    assert c.tolist() == [0.0, 1.0, 2.0, 3.0]


def test_modular_route_config3_all_epilogues():
    """configs[2]'s distribution on the modular route: 24 int8 GEMMs and the CRT give the
    oracle's bytes, cancelling cells (+0) included, under every epilogue."""
    m, k, n = 300, 512, 260
    a, b = config3(m, k, n)
    a, b = a.reshape(-1), b.reshape(-1)
    rng = np.random.default_rng(8)
    c0 = rng.standard_normal(m * n).astype(np.float32)
    for alpha, beta, mode in [(1, 0, U.NEAREST), (-3, 0, U.TOWARD_ZERO), (7, -2, U.NEAREST),
                              (2**62, 1, U.SATURATING)]:
        got, want, route = run_both(U.F32, U.F32, a, b, m, k, n, alpha, beta, c0, mode)
        assert np.array_equal(got, want), (alpha, beta, mode)
        assert route.moduli > 0 and route.fixups == 0


def test_modular_route_spans_past_sixteen_digits():
    """Exponents over [-50, 50]: 124-bit spans, more than 16 base-256 digits (the digit
    route would run on CUDA cores); 35 moduli cover them on the tensor cores."""
    m, k, n = 70, 100, 60
    rng = np.random.default_rng(21)

    def wide(count):
        mant = rng.integers(1 << 23, 1 << 24, size=count).astype(np.float64)
        e = rng.integers(-50, 51, size=count)
        s = rng.choice([-1.0, 1.0], size=count)
        return (s * np.ldexp(mant, e - 23)).astype(np.float32)
    a, b = wide(m * k), wide(k * n)
    for out in (U.F32, U.F64):
        got, want, route = run_both(U.F32, out, a, b, m, k, n, 3, 0)
        assert np.array_equal(got, want)
        assert route.moduli >= 30 and route.tile_k == 128


def test_modular_route_two_reduction_chunks():
    """k past 1023 blocks of 128: the residues of two reduction chunks are summed in the CRT."""
    m, k, n = 6, 140000, 9
    rng = np.random.default_rng(4)
    a = (rng.standard_normal(m * k) * np.exp2(rng.integers(-4, 4, m * k))).astype(np.float32)
    b = (rng.standard_normal(k * n) * np.exp2(rng.integers(-4, 4, k * n))).astype(np.float32)
    got, want, route = run_both(U.F32, U.F32, a, b, m, k, n, 1, 0)
    assert np.array_equal(got, want)
    assert route.moduli > 0 and route.k_chunks >= 2


@pytest.mark.parametrize("exp_range,moduli", [(8, (2, 28)), (40, (29, 32)), (50, (33, 40))])
@pytest.mark.parametrize("m,k,n", [(70, 100, 56), (200, 300, 200)])
def test_modular_route_crt_on_tensor_cores(exp_range, moduli, m, k, n):
    """The CRT's columns as a tensor-core product (one reduction chunk, finite operands,
    m n a multiple of 16): W with 32 columns (up to 28 moduli), 64 columns, and two K32
    steps past 32 moduli; 3920 cells leave a ragged last block of 128. Every epilogue,
    f32 and f64 outputs, bit for bit against the oracle."""
    rng = np.random.default_rng(exp_range * 1000 + m)

    def draw(count):
        mant = rng.integers(1 << 23, 1 << 24, size=count).astype(np.float64)
        e = rng.integers(-exp_range, exp_range + 1, size=count)
        return (rng.choice([-1.0, 1.0], size=count) * np.ldexp(mant, e - 23)).astype(np.float32)
    a, b = draw(m * k), draw(k * n)
    b[3 * n:4 * n] = 0.0  # a zero row of B
    a[5 * k:6 * k] = 0.0  # a zero row of A: its output row is exactly +0
    for out in (U.F32, U.F64):
        c0 = rng.standard_normal(m * n).astype(FT[out])
        for alpha, beta, mode in [(1, 0, U.NEAREST), (-3, 2, U.NEAREST), (2**40, -1, U.TOWARD_ZERO)]:
            got, want, route = run_both(U.F32, out, a, b, m, k, n, alpha, beta, c0, mode)
            assert np.array_equal(got, want), (out, alpha, beta, mode)
            assert route.crt == 1 and moduli[0] <= route.moduli <= moduli[1], route.moduli


@pytest.mark.parametrize("nonfinite", [True, False])
@pytest.mark.parametrize("elem,m,k,n", [(U.F32, 1000, 300, 4096), (U.F64, 1100, 64, 4096)])
def test_modular_route_tall_products(elem, m, k, n, nonfinite):
    """Tall, wide products on the modular route (several row tiles of CTA pairs, a ragged
    last tile): the whole result equals the digit-slice route's bit for bit, and rows
    spread over the tiles equal the oracle's, under beta != 0, with non-finite values in
    two rows (the CRT on CUDA cores) or without (its columns on the tensor cores, many
    blocks of 128 cells per CTA)."""
    rng = np.random.default_rng(30 + m)
    dt = FT[elem]
    if elem == U.F32:
        a, b = config3(m, k, n)
        a, b = a.reshape(-1).copy(), b.reshape(-1).copy()
    else:
        def draw(count):
            mant = rng.integers(1 << 52, 1 << 53, size=count, dtype=np.int64).astype(np.float64)
            return rng.choice([-1.0, 1.0], size=count) * np.ldexp(mant, rng.integers(-30, 31, count) - 52)
        a, b = draw(m * k), draw(k * n)
    if nonfinite:
        a[900 * k + 5] = np.inf
        a[950 * k + 7] = np.nan
    c0 = rng.standard_normal(m * n).astype(dt)
    outs = {}
    for digits in (False, True):
        c = c0.copy()
        route = U.Route()
        U.gemm_float(elem, elem, a, (m, k, k, 1), b, (k, n, n, 1), c, (m, n, n, 1), 3, -2,
                     route=route, digits=digits)
        outs[digits] = c.view(UT[elem])
        assert (route.moduli > 0) != digits
        assert route.crt == (not digits and not nonfinite)
    assert np.array_equal(outs[False], outs[True])
    for i in (0, 511, 512, 767, 768, 900, 950, m - 1):
        w = c0[i * n:(i + 1) * n].copy()
        orc.gemm_float(View(a, 1, k, k, 1, i * k), View(b, k, n, n, 1), View(w, 1, n, n, 1),
                       alpha=3, beta=-2)
        assert np.array_equal(outs[False][i * n:(i + 1) * n], w.view(UT[elem])), i
