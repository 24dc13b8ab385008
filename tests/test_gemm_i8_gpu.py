"""K1 (exact i8 GEMM on tcgen05) against the CPU oracle, through the C ABI.

Bit-exact comparison everywhere: the integer path has no tolerance."""
import ctypes

import numpy as np
import pytest

import uor_b200 as U
from oracle import oracle as orc
from gpu_util import HAVE_CUDA, i8, i128_values, needs_gpu, oracle_int, out_array, torch

pytestmark = [pytest.mark.gpu, needs_gpu]


def run_both(m, k, n, a, av, b, bv, c0, cv, out=U.I32, alpha=1, beta=0, mode=U.NEAREST,
             a_len=None):
    """GPU through uor_b200_gemm (host pointers) and the oracle; return both outputs."""
    got = c0.copy()
    want = c0.copy()
    route = U.Route()
    U.gemm(U.I8, out, a, av, b, bv, got, cv, alpha, beta, mode, route=route)
    oracle_int(a, av + (_origin(av),), b, bv + (_origin(bv),), want, cv + (_origin(cv),), alpha,
               beta, mode, out)
    return got, want, route


def _origin(v):
    rows, cols, rs, cs = v
    lo = orc.extent(rows, cols, rs, cs)[0]
    return -lo


def test_readme_kat_gpu():
    a = np.array([1, 2, 3, 4], np.int8)
    b = np.array([5, 6, 7, 8], np.int8)
    c = np.zeros(4, np.int32)
    U.gemm_i8_i32(2, 2, 2, a, b, c)
    assert c.tolist() == [19, 22, 43, 50]


def test_config1_512_cubed_all_spellings():
    m = k = n = 512
    a, b = i8(1, m * k), i8(2, k * n)
    prior = U.corpus(3, U.CORPUS_RAW, m * n).astype(np.int64).astype(np.int32)
    # slice::gemm
    got = np.zeros(m * n, np.int32)
    route = U.Route()
    U.slice_gemm(U.I8, U.I32, m, k, n, a, b, got, route=route)
    want = np.zeros(m * n, np.int32)
    orc.gemm_int(orc.View.row_major(a, m, k), orc.View.row_major(b, k, n),
                 orc.View.row_major(want, m, n))
    assert np.array_equal(got, want)
    assert route.kernel == 1 and route.k_chunks == 1
    # gemm_ex alpha=3, beta=-1 with a prior C
    got = prior.copy()
    U.slice_gemm_ex(U.I8, U.I32, m, k, n, 3, a, k, b, n, -1, got, n)
    want = prior.copy()
    orc.gemm_int(orc.View.row_major(a, m, k), orc.View.row_major(b, k, n),
                 orc.View.row_major(want, m, n), alpha=3, beta=-1)
    assert np.array_equal(got, want)
    # the transposed-B view: B stored n x k, read with Strides { rs: 1, cs: k }
    bt = np.ascontiguousarray(b.reshape(k, n).T).reshape(-1)
    got = np.zeros(m * n, np.int32)
    route = U.Route()
    U.gemm(U.I8, U.I32, a, (m, k, k, 1), bt, (k, n, 1, k), got, (m, n, n, 1), route=route)
    assert np.array_equal(got, want_plain(a, b, m, k, n))
    assert route.b_layout == 0  # K-major straight from the buffer


def want_plain(a, b, m, k, n):
    w = np.zeros(m * n, np.int32)
    orc.gemm_int(orc.View.row_major(a, m, k), orc.View.row_major(b, k, n),
                 orc.View.row_major(w, m, n))
    return w


SHAPES = [(1, 1, 1), (3, 7, 11), (13, 17, 19), (5, 97, 7), (127, 129, 255), (128, 256, 128),
          (129, 257, 130), (200, 1000, 300), (1, 4096, 1), (2, 4096, 2), (300, 64, 520)]


@pytest.mark.parametrize("shape", SHAPES)
def test_shapes_row_major(shape):
    m, k, n = shape
    a, b = i8(10 + m, m * k), i8(20 + n, k * n)
    c0 = np.zeros(m * n, np.int32)
    got, want, route = run_both(m, k, n, a, (m, k, k, 1), b, (k, n, n, 1), c0, (m, n, n, 1))
    assert np.array_equal(got, want), shape


@pytest.mark.parametrize("out", [U.I8, U.I16, U.I32, U.I64, U.I128])
@pytest.mark.parametrize("mode", [U.NEAREST, U.WRAPPING, U.SATURATING])
def test_outputs_and_modes(out, mode):
    m, k, n = 37, 300, 45
    a, b = i8(5, m * k), i8(6, k * n)
    rng = np.random.default_rng(out * 10 + mode)
    c0 = out_array(out, m * n)
    c0[:] = rng.integers(np.iinfo(c0.dtype).min, np.iinfo(c0.dtype).max, size=c0.size,
                         endpoint=True, dtype=c0.dtype)
    for alpha, beta in [(1, 0), (3, -1), (-(2**63), 2**62), (2**63 - 1, -7), (0, 1)]:
        got, want, _ = run_both(m, k, n, a, (m, k, k, 1), b, (k, n, n, 1), c0, (m, n, n, 1), out,
                                alpha, beta, mode)
        if out == U.I128:
            assert i128_values(got) == i128_values(want), (alpha, beta)
        else:
            assert np.array_equal(got, want), (out, mode, alpha, beta)


def test_layouts_transposed_gathered_and_negative():
    m, k, n = 160, 200, 170  # m * 1 byte is a multiple of 16: A^T is TMA-readable
    a, b = i8(7, m * k), i8(8, k * n)
    base = want_plain(a, b, m, k, n)
    at = np.ascontiguousarray(a.reshape(m, k).T).reshape(-1)   # A^T stored k x m
    cases = []
    # A MN-major (A stored k x m): Strides { rs: 1, cs: m }
    cases.append((at, (m, k, 1, m), b, (k, n, n, 1), 1, None))
    # B read backwards: reverse rows of B storage, negative row stride
    brev = b.reshape(k, n)[::-1].copy().reshape(-1)
    cases.append((a, (m, k, k, 1), brev, (k, n, -n, 1), None, 2))
    # an unaligned leading dimension forces the gather
    lda = k + 3
    apad = np.zeros(m * lda, np.int8)
    apad.reshape(m, lda)[:, :k] = a.reshape(m, k)
    cases.append((apad, (m, k, lda, 1), b, (k, n, n, 1), 2, None))
    for aa, av, bb, bv, a_layout, b_layout in cases:
        got = np.zeros(m * n, np.int32)
        route = U.Route()
        U.gemm(U.I8, U.I32, aa, av, bb, bv, got, (m, n, n, 1), route=route)
        assert np.array_equal(got, base)
        if a_layout is not None:
            assert route.a_layout == a_layout
        if b_layout is not None:
            assert route.b_layout == b_layout


def test_broadcast_zero_stride_input():
    m, k, n = 9, 33, 17
    row = i8(9, k)
    b = i8(10, k * n)
    got = np.zeros(m * n, np.int32)
    U.gemm(U.I8, U.I32, row, (m, k, 0, 1), b, (k, n, n, 1), got, (m, n, n, 1))
    want = np.zeros(m * n, np.int32)
    orc.gemm_int(orc.View(row, m, k, 0, 1), orc.View.row_major(b, k, n),
                 orc.View.row_major(want, m, n))
    assert np.array_equal(got, want)


def test_strided_output_with_gaps_is_preserved():
    m, k, n, ldc = 20, 50, 30, 41
    a, b = i8(11, m * k), i8(12, k * n)
    c = np.full(m * ldc, 12345, np.int32)
    U.slice_gemm_ex(U.I8, U.I32, m, k, n, 2, a, k, b, n, 1, c, ldc)
    want = np.full(m * ldc, 12345, np.int32)
    orc.gemm_int(orc.View.row_major(a, m, k), orc.View.row_major(b, k, n),
                 orc.View(want, m, n, ldc, 1), alpha=2, beta=1)
    assert np.array_equal(c, want)


def test_k_zero_is_the_epilogue_alone():
    m, n = 5, 7
    c = np.arange(m * n, dtype=np.int32)
    U.slice_gemm_ex(U.I8, U.I32, m, 0, n, 5, np.zeros(0, np.int8), 0, np.zeros(0, np.int8), n,
                    -3, c, n)
    assert np.array_equal(c, -3 * np.arange(m * n, dtype=np.int32))


def test_depth_past_the_lane_is_exact():
    # driver.rs:743-759: k = 150000 of i8::MIN^2 into i64, past lane_depth = 131071
    k = 150_000
    a = np.full(k, -128, np.int8)
    b = np.full(k, -128, np.int8)
    c = np.zeros(1, np.int64)
    route = U.Route()
    U.slice_gemm_ex(U.I8, U.I64, 1, k, 1, 1, a, k, b, 1, 0, c, 1, route=route)
    assert c[0] == k * 128 * 128
    assert route.k_chunks >= 2  # chunked within the s32 lane depth (skinny dp4a route here)
    # and a random deep product against the oracle, saturating into i32
    m, n, k = 6, 10, 140_000
    a, b = i8(13, m * k), i8(14, k * n)
    for out in (U.I32, U.I64):
        got, want, route = run_both(m, k, n, a, (m, k, k, 1), b, (k, n, n, 1),
                                    out_array(out, m * n), (m, n, n, 1), out, 3, 0)
        assert np.array_equal(got, want)


def test_device_pointers_zero_copy():
    m, k, n = 256, 512, 384
    a, b = i8(15, m * k), i8(16, k * n)
    ta = torch.from_numpy(a).cuda()
    tb = torch.from_numpy(b).cuda()
    tc = torch.zeros(m * n, dtype=torch.int32, device="cuda")
    U.gemm_i8_i32(m, k, n, ta, tb, tc)
    assert np.array_equal(tc.cpu().numpy(), want_plain(a, b, m, k, n))


def test_host_pointer_pipeline_blocks_are_exact():
    """Host-pointer calls of at least 4 Mi cells are cut into blocks whose copies
    overlap the compute; the bytes are those of the whole call, ragged blocks,
    padded leading dimensions, gaps in the output and a read C included."""
    m, k, n = 2304, 272, 2048
    a, b = i8(31, m * k), i8(32, k * n)
    c0 = np.zeros(m * n, np.int32)
    got, want, route = run_both(m, k, n, a, (m, k, k, 1), b, (k, n, n, 1), c0, (m, n, n, 1))
    assert np.array_equal(got, want)
    assert route.kernel == 1
    m, k, n, lda, ldb, ldc = 1100, 160, 4160, 176, 4176, 4170
    a, b = i8(33, m * lda), i8(34, k * ldb)
    rng = np.random.default_rng(5)
    c0 = rng.integers(-(2**62), 2**62, size=m * ldc, dtype=np.int64)
    for alpha, beta, mode in [(3, -2, U.NEAREST), (2**40, 2**30, U.WRAPPING)]:
        got, want, route = run_both(m, k, n, a, (m, k, lda, 1), b, (k, n, ldb, 1), c0,
                                    (m, n, ldc, 1), U.I64, alpha, beta, mode)
        assert np.array_equal(got, want), (alpha, beta)


@pytest.mark.parametrize("pinned", [False, True])
def test_host_pipeline_split_first_row_and_whole_blocks(pinned):
    """Several row and column blocks: the first row of blocks is cut into narrower
    pieces, the rows after it into whole blocks; a pinned C takes the interleaved
    copy-out. Every cell, with and without a read C."""
    m, k, n = 4400, 96, 4200
    a, b = i8(35, m * k), i8(36, k * n)
    rng = np.random.default_rng(7)
    prior = rng.integers(-(2**31), 2**31, size=m * n, dtype=np.int64).astype(np.int32)
    for alpha, beta in [(1, 0), (-3, 2)]:
        want = prior.copy()
        oracle_int(a, (m, k, k, 1, 0), b, (k, n, n, 1, 0), want, (m, n, n, 1, 0), alpha, beta,
                   U.NEAREST, U.I32)
        if pinned:
            host = torch.from_numpy(prior.copy()).pin_memory()
            got = host.numpy()
        else:
            got = prior.copy()
        route = U.Route()
        U.gemm(U.I8, U.I32, a, (m, k, k, 1), b, (k, n, n, 1), got, (m, n, n, 1), alpha, beta,
               route=route)
        assert np.array_equal(got, want), (alpha, beta)
        assert route.kernel == 1


def test_bounded_wait_gives_up_and_context_survives():
    ctx = U.Context(0)
    assert U.selftest_wait_timeout(ctx, 50_000_000) == U.TIMEOUT
    a = np.array([1, 2, 3, 4], np.int8)
    b = np.array([5, 6, 7, 8], np.int8)
    c = np.zeros(4, np.int32)
    U.gemm_i8_i32(2, 2, 2, a, b, c, ctx=ctx)
    assert c.tolist() == [19, 22, 43, 50]
    ctx.close()
