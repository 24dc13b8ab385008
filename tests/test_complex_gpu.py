"""Complex<i32 | i64> GEMM (alphabet.rs:656-776) through the byte-sliced path, against
the oracle's componentwise restatement."""
import numpy as np
import pytest

import uor_b200 as U
from oracle import oracle as orc
from gpu_util import i128_values, needs_gpu, out_array, torch

pytestmark = [pytest.mark.gpu, needs_gpu]

ELEM = {32: U.I32, 64: U.I64}
NP = {32: np.int32, 64: np.int64}
OBITS = {U.I8: 8, U.I16: 16, U.I32: 32, U.I64: 64, U.I128: 128}


def rand_parts(rng, bits, count, min_share=0.0):
    info = np.iinfo(NP[bits])
    x = rng.integers(info.min, info.max, size=2 * count, endpoint=True).astype(NP[bits])
    if min_share:
        x[rng.random(x.size) < min_share] = info.min
    return x


def oracle(a, av, b, bv, c, cv, alpha, beta, mode, out):
    orc.gemm_complex(orc.View(a, *av), orc.View(b, *bv), orc.View(c, *cv), alpha=alpha,
                     beta=beta, mode=mode, out_bits=OBITS[out])


def same(got, want, out):
    if out == U.I128:
        return i128_values(got) == i128_values(want)
    return np.array_equal(got, want)


@pytest.mark.parametrize("bits", [32, 64])
@pytest.mark.parametrize("out", [U.I32, U.I64, U.I128])
@pytest.mark.parametrize("digits", [False, True])
def test_random_full_range(bits, out, digits):
    rng = np.random.default_rng(bits + 7 * out)
    for (m, k, n) in [(1, 1, 1), (13, 17, 19), (130, 300, 135), (257, 64, 70)]:
        a = rand_parts(rng, bits, m * k)
        b = rand_parts(rng, bits, k * n, min_share=0.05)
        c0 = out_array(out, 2 * m * n)
        c0[:] = rng.integers(-1000, 1000, size=c0.size)
        for alpha, beta, mode in [(1, 0, U.NEAREST), (3, -1, U.WRAPPING),
                                  (-(2**63), 5, U.NEAREST), (2**62, 2**62, U.SATURATING)]:
            got, want = c0.copy(), c0.copy()
            route = U.Route()
            U.gemm_complex(ELEM[bits], out, a, (m, k, k, 1), b, (k, n, n, 1), got, (m, n, n, 1),
                           alpha, beta, mode, route=route, digits=digits, modular=not digits)
            oracle(a, (m, k, k, 1), b, (k, n, n, 1), want, (m, n, n, 1), alpha, beta, mode, out)
            assert same(got, want, out), (m, k, n, alpha, beta, mode)
            assert route.kernel == 2  # the limb (byte-sliced) path


def test_reference_kat():
    """(3 + 4i)(5 - 2i) = 23 + 14i (alphabet.rs:824-833)."""
    a, b = np.array([3, 4], np.int32), np.array([5, -2], np.int32)
    c = np.zeros(2, np.int32)
    U.gemm_complex(U.I32, U.I32, a, (1, 1, 1, 1), b, (1, 1, 1, 1), c, (1, 1, 1, 1))
    assert c.tolist() == [23, 14]


def test_min_imaginary_parts_negate_as_the_release_build():
    """Every w.im = MIN: -w.im wraps to MIN, the reference's release-build value."""
    for bits in (32, 64):
        rng = np.random.default_rng(bits)
        m, k, n = 9, 40, 11
        a = rand_parts(rng, bits, m * k)
        b = rand_parts(rng, bits, k * n)
        b[1::2] = np.iinfo(NP[bits]).min
        got, want = out_array(U.I128, 2 * m * n), out_array(U.I128, 2 * m * n)
        U.gemm_complex(ELEM[bits], U.I128, a, (m, k, k, 1), b, (k, n, n, 1), got, (m, n, n, 1))
        oracle(a, (m, k, k, 1), b, (k, n, n, 1), want, (m, n, n, 1), 1, 0, U.NEAREST, U.I128)
        assert same(got, want, U.I128)


def test_strided_views_and_transposed_b():
    rng = np.random.default_rng(3)
    m, k, n = 70, 150, 45
    a = rand_parts(rng, 32, m * k)
    bt = rand_parts(rng, 32, k * n)  # stored n x k: B(p, j) at j * k + p
    c0 = np.zeros(2 * m * 2 * n, np.int64)  # C in every other column of a wider buffer
    c0[:] = rng.integers(-50, 50, size=c0.size)
    got, want = c0.copy(), c0.copy()
    U.gemm_complex(U.I32, U.I64, a, (m, k, k, 1), bt, (k, n, 1, k), got, (m, n, 2 * n, 2), 2, 3)
    oracle(a, (m, k, k, 1), bt, (k, n, 1, k), want, (m, n, 2 * n, 2), 2, 3, U.NEAREST, U.I64)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("digits", [False, True])
def test_deep_reduction_several_chunks(digits):
    rng = np.random.default_rng(11)
    m, k, n = 20, 20000, 12
    a = rand_parts(rng, 32, m * k)
    b = rand_parts(rng, 32, k * n)
    got, want = out_array(U.I128, 2 * m * n), out_array(U.I128, 2 * m * n)
    route = U.Route()
    U.gemm_complex(U.I32, U.I128, a, (m, k, k, 1), b, (k, n, n, 1), got, (m, n, n, 1),
                   route=route, digits=digits, modular=not digits)
    oracle(a, (m, k, k, 1), b, (k, n, n, 1), want, (m, n, n, 1), 1, 0, U.NEAREST, U.I128)
    assert same(got, want, U.I128)
    assert route.k_chunks >= 2 if digits else route.moduli > 0


def test_k_zero_applies_beta_in_the_accumulator():
    """k = 0: C := encode(beta * C) per part; for Complex<i64> the prior is scaled in
    Limbs<3> (modulo 2^192), so Wrapping into i128 keeps the low 128 bits."""
    c0 = np.array([0, 1 << 62, 5, 0, -3, -1, 7, 0], np.int64)  # two Complex<i128>
    for bits in (32, 64):
        got, want = c0.copy(), c0.copy()
        a = np.zeros(2, NP[bits])
        U.gemm_complex(ELEM[bits], U.I128, a, (1, 0, 0, 1), a, (0, 2, 2, 1), got, (1, 2, 2, 1),
                       1, 4, U.WRAPPING)
        oracle(a, (1, 0, 0, 1), a, (0, 2, 2, 1), want, (1, 2, 2, 1), 1, 4, U.WRAPPING, U.I128)
        assert same(got, want, U.I128), bits


def test_device_pointers():
    rng = np.random.default_rng(5)
    m, k, n = 100, 128, 96
    a = rand_parts(rng, 64, m * k)
    b = rand_parts(rng, 64, k * n)
    want = np.zeros(2 * m * n, np.int64)
    oracle(a, (m, k, k, 1), b, (k, n, n, 1), want, (m, n, n, 1), 1, 0, U.NEAREST, U.I64)
    ad, bd = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    cd = torch.zeros(2 * m * n, dtype=torch.int64, device="cuda")
    U.gemm_complex(U.I64, U.I64, ad, (m, k, k, 1), bd, (k, n, n, 1), cd, (m, n, n, 1))
    assert np.array_equal(cd.cpu().numpy(), want)


def test_errors():
    a = np.zeros(2 * 6, np.int32)
    c = np.zeros(2 * 9, np.int32)
    with pytest.raises(U.NotAProduct):
        U.gemm_complex(U.I32, U.I32, a, (2, 3, 3, 1), a, (2, 3, 3, 1), c, (2, 3, 3, 1))
    with pytest.raises(U.NotAProduct):  # C aliases itself
        U.gemm_complex(U.I32, U.I32, a, (3, 2, 2, 1), a, (2, 3, 3, 1), c, (3, 3, 1, 1))
    with pytest.raises(U.UorError):  # Complex<i16> has no Element impl in the reference
        U.gemm_complex(U.I16, U.I32, a.view(np.int16), (2, 3, 3, 1), a.view(np.int16),
                       (3, 2, 2, 1), c, (2, 2, 2, 1))
