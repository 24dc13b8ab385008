"""Arena<E, N, K> (codecs.rs:894-985) through uor_b200_arena_gemm: the decoded float
symbols times a float A, against the oracle's exact float GEMM of the same decoded
matrix, bit for bit -- on the reference's CK-14 corpus and on tables with signed zeros,
subnormals and non-finite symbols."""
import numpy as np
import pytest

import uor_b200 as U
from oracle import oracle as orc
from gpu_util import needs_gpu, torch
from test_arena_cpu import ck14_codebook, ck14_codes

pytestmark = [pytest.mark.gpu, needs_gpu]


def rand_f32(rng, count, lo=-20, hi=20):
    m = rng.integers(1 << 23, 1 << 24, size=count).astype(np.float64)
    e = rng.integers(lo, hi, size=count)
    s = rng.choice([-1.0, 1.0], size=count)
    return (s * np.ldexp(m, e - 23)).astype(np.float32)


def check(m, k, n, table, codes, orientation, code_bytes=1, out=U.F32, alpha=1, beta=0,
          seed=0, a=None):
    rng = np.random.default_rng(seed)
    elem = U.F64 if table.dtype == np.float64 else U.F32
    if a is None:
        a = rand_f32(rng, m * k).astype(table.dtype)
    rows, cols = (k, n) if orientation == 0 else (n, k)
    dense = orc.decode_arena(table, codes, rows, cols, code_bytes)
    odt = np.float64 if out == U.F64 else np.float32
    c0 = rand_f32(rng, m * n).astype(odt)
    got, want = c0.copy(), c0.copy()
    route = U.Route()
    U.arena_gemm(elem, out, a, (m, k, k, 1), table, codes, k, n, got, (m, n, n, 1),
                 code_bytes=code_bytes, orientation=orientation, alpha=alpha, beta=beta,
                 route=route)
    bv = (k, n, n, 1) if orientation == 0 else (k, n, 1, k)
    orc.gemm_float(orc.View(a, m, k, k, 1), orc.View(np.ascontiguousarray(dense).reshape(-1), *bv),
                   orc.View(want, m, n, n, 1), alpha=alpha, beta=beta)
    assert np.array_equal(got.view(np.uint8), want.view(np.uint8))
    assert route.kernel == 5 and route.b_layout == 3
    return got


@pytest.mark.parametrize("idx", [0, 1])
def test_ck14_corpus_tabulated(idx):
    """The CK-14 artifact as gemm_tabulated holds it (W n x k, C = A W^T), u8 codes."""
    case, codes = ck14_codes(idx)
    n, k = case["shape"]["n"], case["shape"]["k"]
    m = 64 if idx == 0 else 256
    check(m, k, n, ck14_codebook(), codes, 1, seed=idx)


def test_ck14_codebook_coded_orientation_and_epilogue():
    _, codes = ck14_codes(0)  # 13 x 257 codes read as a k x n coded B
    check(40, 13, 257, ck14_codebook(), codes, 0, alpha=3, beta=-2, seed=5)
    check(40, 13, 257, ck14_codebook(), codes, 0, out=U.F64, alpha=-1, beta=1, seed=6)


def test_u16_codes_modulo_a_table_with_special_symbols():
    rng = np.random.default_rng(9)
    vals = rand_f32(rng, 997, -60, 60)
    vals[:4] = [0.0, -0.0, np.float32(2.0 ** -140), -np.float32(2.0 ** -149)]
    table = vals.copy()
    m, k, n = 70, 300, 90
    codes = rng.integers(0, 256, size=k * n * 2, dtype=np.uint8)
    for orientation in (0, 1):
        check(m, k, n, table, codes, orientation, code_bytes=2, seed=10 + orientation)


def test_non_finite_symbols_follow_the_float_rules():
    """An infinite symbol meets finite and zero A values: the float family's NaN and
    infinity rules apply to the decoded matrix unchanged."""
    table = np.array([1.0, np.inf, -2.0, 0.5], np.float32)
    m, k, n = 9, 16, 12
    rng = np.random.default_rng(4)
    codes = rng.integers(0, 4, size=k * n, dtype=np.uint8)
    a = rand_f32(rng, m * k)
    a[::5] = 0.0
    check(m, k, n, table, codes, 0, a=a, seed=4)


def test_f64_symbols():
    rng = np.random.default_rng(12)
    table = rng.standard_normal(300) * 2.0 ** rng.integers(-40, 40, size=300)
    m, k, n = 33, 64, 48
    codes = rng.integers(0, 256, size=k * n * 2, dtype=np.uint8)
    check(m, k, n, table, codes, 1, code_bytes=2, out=U.F64, seed=12)


def test_device_pointers():
    table = ck14_codebook()
    _, codes = ck14_codes(0)
    n, k, m = 13, 257, 50
    rng = np.random.default_rng(2)
    a = rand_f32(rng, m * k)
    want = np.zeros(m * n, np.float32)
    dense = orc.decode_arena(table, codes, n, k)
    orc.gemm_float(orc.View(a, m, k, k, 1), orc.View(dense.reshape(-1), k, n, 1, k),
                   orc.View(want, m, n, n, 1))
    cd = torch.zeros(m * n, dtype=torch.float32, device="cuda")
    U.arena_gemm(U.F32, U.F32, torch.from_numpy(a).cuda(), (m, k, k, 1),
                 torch.from_numpy(table).cuda(), torch.from_numpy(codes).cuda(), k, n, cd,
                 (m, n, n, 1), orientation=1)
    assert np.array_equal(cd.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_validation():
    a = np.zeros(4, np.float32)
    c = np.zeros(4, np.float32)
    t = np.ones(3, np.float32)
    with pytest.raises(U.DoesNotFit):  # one code short
        U.arena_gemm(U.F32, U.F32, a, (1, 4, 4, 1), t, np.zeros(15, np.uint8), 4, 4, c,
                     (1, 4, 4, 1))
    with pytest.raises(U.NotAProduct):
        U.arena_gemm(U.F32, U.F32, a, (1, 4, 4, 1), t, np.zeros(16, np.uint8), 4, 4, c,
                     (2, 2, 2, 1))
    with pytest.raises(U.UorError):  # integer elements are not an Arena
        U.arena_gemm(U.I32, U.F32, a, (1, 4, 4, 1), t, np.zeros(16, np.uint8), 4, 4, c,
                     (1, 4, 4, 1))
