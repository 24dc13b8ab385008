"""The narrow-side i8 kernels (dp4a reduce factorization and column kernel) against the
CPU oracle: bit-exact, every output type and encode, the operand layouts each route
takes, and reductions deeper than one s32 lane."""
import numpy as np
import pytest

import uor_b200 as U
from oracle import oracle as orc
from gpu_util import i8, i128_values, needs_gpu, out_array

pytestmark = [pytest.mark.gpu, needs_gpu]

SKINNY = 7


def run(m, k, n, av_of, bv_of, out=U.I32, alpha=1, beta=0, mode=U.NEAREST, seed=0):
    a, av = av_of(i8(40 + seed, m * k), m, k)
    b, bv = bv_of(i8(41 + seed, k * n), k, n)
    c0 = out_array(out, m * n)
    rng = np.random.default_rng(seed)
    if out != U.I128:
        info = np.iinfo(c0.dtype)
        c0[:] = rng.integers(info.min, info.max, size=c0.size, endpoint=True, dtype=c0.dtype)
    else:
        c0[:] = rng.integers(-(2**62), 2**62, size=c0.size)
    got, want = c0.copy(), c0.copy()
    route = U.Route()
    U.gemm(U.I8, out, a, av, b, bv, got, (m, n, n, 1), alpha, beta, mode, route=route)
    bits = {U.I8: 8, U.I16: 16, U.I32: 32, U.I64: 64, U.I128: 128}[out]
    orc.gemm_int(orc.View(a, *av), orc.View(b, *bv), orc.View(want, m, n, n, 1), alpha=alpha,
                 beta=beta, mode=mode, out_bits=bits)
    if out == U.I128:
        assert i128_values(got) == i128_values(want)
    else:
        assert np.array_equal(got, want)
    return route


def row_major(x, r, c):
    return x, (r, c, c, 1)


def transposed(x, r, c):  # stored c x r, read with Strides { rs: 1, cs: r }
    t = np.ascontiguousarray(x.reshape(r, c).T).reshape(-1)
    return t, (r, c, 1, r)


def padded(x, r, c):  # row-major with a leading dimension that breaks 16-byte alignment
    ld = c + 3
    p = np.zeros(r * ld, np.int8)
    p.reshape(r, ld)[:, :c] = x.reshape(r, c)
    return p, (r, c, ld, 1)


@pytest.mark.parametrize("shape", [(1, 8192, 8192), (8192, 8192, 1), (3, 1000, 5000),
                                   (5000, 777, 7), (16, 4096, 300), (300, 4096, 16),
                                   (1, 1, 1), (2, 33, 40), (40, 33, 2)])
def test_row_major_shapes(shape):
    m, k, n = shape
    route = run(m, k, n, row_major, row_major, seed=m + n)
    assert route.kernel == SKINNY


@pytest.mark.parametrize("av_of", [row_major, transposed, padded])
@pytest.mark.parametrize("bv_of", [row_major, transposed, padded])
def test_layouts_thin_m_and_thin_n(av_of, bv_of):
    for (m, k, n) in [(5, 700, 1000), (1000, 700, 5)]:
        route = run(m, k, n, av_of, bv_of, seed=7)
        assert route.kernel == SKINNY, (m, n, av_of.__name__, bv_of.__name__)


@pytest.mark.parametrize("out", [U.I8, U.I16, U.I32, U.I64, U.I128])
@pytest.mark.parametrize("mode", [U.NEAREST, U.WRAPPING, U.SATURATING])
def test_outputs_modes_alpha_beta(out, mode):
    for (m, k, n) in [(4, 300, 600), (600, 300, 4)]:
        for alpha, beta in [(1, 0), (3, -1), (-(2**63), 2**62), (2**63 - 1, -7)]:
            run(m, k, n, row_major, row_major, out, alpha, beta, mode, seed=out * 10 + mode)


def test_deeper_than_one_lane():
    # -128 x -128 = 2^14 over 300000 terms exceeds an s32 lane: chunked and folded exactly
    for (m, k, n) in [(1, 300_000, 3), (3, 300_000, 1), (2, 200_003, 40)]:
        route = run(m, k, n, row_major, row_major, U.I64, seed=3)
        assert route.k_chunks >= 2
    k = 300_000
    a = np.full(k, -128, np.int8)
    b = np.full(k * 2, -128, np.int8)
    c = np.zeros(2, np.int64)
    U.gemm(U.I8, U.I64, a, (1, k, k, 1), b, (k, 2, 2, 1), c, (1, 2, 2, 1))
    assert c.tolist() == [k * 16384, k * 16384]
