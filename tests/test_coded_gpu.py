"""The codec tier against the oracle's coded_gemm / gemm_tabulated restatement: K1C (K1's
CTA-pair pipeline with the codes decoded into its B stages, no dense copy anywhere), with
512-row tiles from 512 activation rows up and 256-row tiles below -- nibbles through the
register table, 2- and 1-bit sub-codes through a byte table built on chip -- in exact
chunks past one s32 lane; deep nibble products of 512 rows and more decode once into a
dense workspace and run K1's chunks unless CODEC_ON_CHIP forbids the workspace."""
import numpy as np
import pytest

import uor_b200 as U
from oracle import oracle as orc
from gpu_util import i128_values, needs_gpu, out_array, torch

pytestmark = [pytest.mark.gpu, needs_gpu]


def make_codes(rng, rows, cols, P):
    bits = 8 // P
    subs = rng.integers(0, 1 << bits, size=(rows, cols))
    codes = np.zeros((rows, cols // P), np.uint8)
    for e in range(P):
        codes |= (subs[:, e::P] << (bits * e)).astype(np.uint8)
    return codes.reshape(-1)


def run(m, k, n, P, N, orientation, out=U.I32, alpha=1, beta=0, mode=U.NEAREST, seed=0,
        av=None, on_chip=False):
    rng = np.random.default_rng(seed)
    a = rng.integers(-128, 128, size=m * k).astype(np.int8)
    rows, cols = (k, n) if orientation == 0 else (n, k)
    codes = make_codes(rng, rows, cols, P)
    table = rng.integers(-128, 128, size=N).astype(np.int8)
    c0 = out_array(out, m * n)
    c0[:] = rng.integers(-1000, 1000, size=c0.size)
    got, want = c0.copy(), c0.copy()
    route = U.Route()
    av = av or (m, k, k, 1)
    U.coded_gemm(out, a, av, codes, k, n, P, table, got, (m, n, n, 1), alpha, beta, mode,
                 route=route, tabulated=orientation == 1, on_chip=on_chip)
    obits = {U.I32: 32, U.I64: 64, U.I128: 128, U.I16: 16, U.I8: 8}[out]
    origin = -orc.extent(*av)[0]
    if out != U.I128:
        orc.coded_gemm(orc.View(a, *av, origin), codes, P, table, orc.View(want, m, n, n, 1), k,
                       n, orientation, alpha, beta, mode)
    else:  # 16-byte cells held as int64 pairs
        orc.lib().uor_oracle_coded_gemm(128, m, k, n, alpha, a.ctypes.data + origin, av[2], av[3],
                                        codes.ctypes.data, P, table.ctypes.data, N, orientation,
                                        beta, want.ctypes.data, n, 1, mode, 0)
    if out == U.I128:
        return i128_values(got), i128_values(want), route
    return got, want, route


def test_nibble_order_gpu():
    # codec/tests/codec.rs:91: low nibble first
    table = (np.arange(16) * 3 - 20).astype(np.int8)
    codes = np.zeros(16, np.uint8)
    codes[0], codes[1] = 0x21, 0x43  # row 0 of a 1 x 32 coded matrix: elements 1, 2, 3, 4, 0...
    a = np.array([1], np.int8)
    c = np.zeros(32, np.int32)
    U.coded_gemm(U.I32, a, (1, 1, 1, 1), codes, 1, 32, 2, table, c, (1, 32, 32, 1))
    assert c[:5].tolist() == [int(table[1]), int(table[2]), int(table[3]), int(table[4]),
                              int(table[0])]


@pytest.mark.parametrize("orientation", [0, 1])
@pytest.mark.parametrize("shape", [(1, 32, 32), (3, 64, 96), (129, 160, 288), (300, 512, 256),
                                   (200, 8192, 64)])
def test_fused_nibbles(orientation, shape):
    m, k, n = shape
    got, want, route = run(m, k, n, 2, 16, orientation, seed=m + n)
    assert np.array_equal(got, want)
    assert route.kernel == 4 and route.b_layout != 3


@pytest.mark.parametrize("orientation", [0, 1])
def test_default_many_rows_decode_on_chip(orientation):
    """By default, any row count: K1C, 512-row tiles from 512 rows and 256-row tiles below,
    never a dense B."""
    for m, k, n, out, alpha, beta, N in [(512, 256, 96, U.I32, 1, 0, 16),
                                         (1030, 96, 288, U.I8, -2, 5, 16),
                                         (40, 512, 160, U.I32, 1, 0, 16),
                                         (300, 320, 64, U.I64, 3, -1, 9)]:
        got, want, route = run(m, k, n, 2, N, orientation, out, alpha, beta, seed=m + N)
        assert np.array_equal(got, want), (m, k, n, out)
        assert route.kernel == 4 and route.b_layout != 3
        assert route.tile_m == (512 if m >= 512 else 256)


@pytest.mark.parametrize("orientation", [0, 1])
def test_pair_decode_many_rows(orientation):
    """CODEC_ON_CHIP, 256 activation rows and more: K1C decodes the nibbles into the
    swizzled B stages of K1's CTA-pair pipeline (never a dense B); ragged rows, columns
    and reductions (the TMA fills codes past the edge with zeros, which decode to
    table[0] but meet zero activations), every output width and the exact Linear
    epilogue."""
    for m, k, n, out, alpha, beta, N in [(512, 256, 96, U.I32, 1, 0, 16),
                                         (600, 320, 64, U.I64, 3, -1, 7),
                                         (1030, 96, 288, U.I8, -2, 5, 16),
                                         (256, 128, 512, U.I32, 1, 0, 16),
                                         (777, 992, 608, U.I32, 1, 0, 16),
                                         (520, 4096, 320, U.I128, 2**40, 1, 11)]:
        got, want, route = run(m, k, n, 2, N, orientation, out, alpha, beta, seed=m + N,
                               on_chip=True)
        assert np.array_equal(got, want), (m, k, n, out)
        assert route.kernel == 4 and route.b_layout != 3 and route.tile_m == (512 if m >= 512 else 256)


def test_pair_decode_gathered_activations():
    m, k, n = 320, 96, 64
    got, want, route = run(m, k, n, 2, 16, 0, av=(m, k, 1, m), seed=19, on_chip=True)
    assert np.array_equal(got, want)
    assert route.a_layout == 2 and route.tile_m == 256


@pytest.mark.parametrize("orientation", [0, 1])
def test_decode_once_past_the_lane(orientation):
    """k past the s32 lane depth with 512+ rows: decoded once to dense int8 (flat over the
    code bytes, low nibble first), then K1 in exact chunks; with CODEC_ON_CHIP, K1C's
    chunks instead (no workspace)."""
    m, k, n = 512, 131_200, 32
    got, want, route = run(m, k, n, 2, 16, orientation, U.I64, seed=5)
    assert np.array_equal(got, want)
    assert route.kernel == 4 and route.b_layout == 3 and route.k_chunks == 2
    got, want, route = run(m, k, n, 2, 16, orientation, U.I64, seed=5, on_chip=True)
    assert np.array_equal(got, want)
    assert route.kernel == 4 and route.b_layout != 3 and route.k_chunks == 2
    assert route.tile_m == 512


@pytest.mark.parametrize("orientation", [0, 1])
def test_deep_reductions_below_512_rows_on_chip(orientation):
    """Fewer than 512 activation rows and k past the s32 lane: K1C's exact chunks on
    256-row tiles (no workspace), a ragged row count, chunk planes folded in 64 bits."""
    m, k, n = 70, 131_200, 64
    got, want, route = run(m, k, n, 2, 16, orientation, U.I64, 3, -1, seed=6)
    assert np.array_equal(got, want)
    assert route.kernel == 4 and route.b_layout != 3 and route.k_chunks == 2 and route.tile_m == 256


@pytest.mark.parametrize("orientation", [0, 1])
@pytest.mark.parametrize("on_chip", [False, True])
def test_decoded_nibbles_device_table(orientation, on_chip):
    """Device pointers and a device table (a 7-entry book, so table[v % 7]) read by K1C's
    decoders themselves, with and without CODEC_ON_CHIP."""
    m, k, n, N = 640, 192, 160, 7
    rng = np.random.default_rng(70 + orientation)
    a = rng.integers(-128, 128, size=m * k).astype(np.int8)
    rows, cols = (k, n) if orientation == 0 else (n, k)
    codes = make_codes(rng, rows, cols, 2)
    table = rng.integers(-128, 128, size=N).astype(np.int8)
    want = np.zeros(m * n, np.int32)
    orc.coded_gemm(orc.View(a, m, k, k, 1), codes, 2, table, orc.View(want, m, n, n, 1), k, n,
                   orientation)
    tc = torch.zeros(m * n, dtype=torch.int32, device="cuda")
    route = U.Route()
    U.coded_gemm(U.I32, torch.from_numpy(a).cuda(), (m, k, k, 1), torch.from_numpy(codes).cuda(),
                 k, n, 2, torch.from_numpy(table).cuda(), tc, (m, n, n, 1), route=route,
                 tabulated=orientation == 1, on_chip=on_chip)
    assert np.array_equal(tc.cpu().numpy(), want)
    assert route.kernel == 4 and route.b_layout != 3


@pytest.mark.parametrize("orientation", [0, 1])
@pytest.mark.parametrize("m", [70, 260])  # one CTA per tile / CTA pairs
def test_short_table_alpha_beta_outputs(orientation, m):
    for out in (U.I8, U.I32, U.I64, U.I128):
        for alpha, beta, mode in [(3, -1, U.NEAREST), (-(2**63), 2**62, U.WRAPPING)]:
            got, want, _ = run(m, 96, 64, 2, 7, orientation, out, alpha, beta, mode, seed=out)
            assert (got == want) if out == U.I128 else np.array_equal(got, want), (out, alpha)


@pytest.mark.parametrize("orientation", [0, 1])
@pytest.mark.parametrize("P,N", [(4, 4), (4, 3), (8, 2), (8, 200)])
@pytest.mark.parametrize("m", [70, 520])
def test_quarter_and_bit_packings_on_chip(P, N, orientation, m):
    """Packed<Grid<N>, 4> and <N, 8> (2- and 1-bit sub-codes, table[sub % N]) decode inside
    K1C through the byte table its decoders build from the N-entry table: route.b_layout
    1 or 0, 256- or 512-row tiles, a reduction that is not a whole number of stages; the
    general epilogue (i64, alpha 3, beta -1) beside the s32 store."""
    k, n = (200, 256) if orientation == 0 else (256, 200)
    for out, alpha, beta in ((U.I32, 1, 0), (U.I64, 3, -1)):
        got, want, route = run(m, k, n, P, N, orientation, out, alpha, beta, seed=P * 7 + N + m)
        assert np.array_equal(got, want), (out, alpha)
        assert route.kernel == 4 and route.b_layout == (1 if orientation == 0 else 0)
        assert route.tile_m == (512 if m >= 512 else 256)


@pytest.mark.parametrize("orientation", [0, 1])
@pytest.mark.parametrize("P", [4, 8])
def test_quarter_and_bit_packings_deep_reduction(P, orientation):
    """Past one s32 lane (k = 131200: a 130944 chunk and 256 more) the byte-table route
    runs K1C per exact chunk and folds the s32 planes in 64 bits."""
    m, k, n = 300, 131200, 128
    got, want, route = run(m, k, n, P, 3, orientation, U.I64, 3, -1, seed=P + orientation)
    assert np.array_equal(got, want)
    assert route.kernel == 4 and route.k_chunks == 2
    assert route.b_layout == (1 if orientation == 0 else 0)


@pytest.mark.parametrize("P", [4, 8])
def test_quarter_and_bit_packings_device_table(P):
    """Device pointers and a device table read by K1C's decoders themselves."""
    m, k, n, N = 300, 128, 384, 3
    rng = np.random.default_rng(90 + P)
    a = rng.integers(-128, 128, size=m * k).astype(np.int8)
    codes = make_codes(rng, k, n, P)
    table = rng.integers(-128, 128, size=N).astype(np.int8)
    want = np.zeros(m * n, np.int32)
    orc.coded_gemm(orc.View(a, m, k, k, 1), codes, P, table, orc.View(want, m, n, n, 1), k, n, 0)
    tc = torch.zeros(m * n, dtype=torch.int32, device="cuda")
    route = U.Route()
    U.coded_gemm(U.I32, torch.from_numpy(a).cuda(), (m, k, k, 1), torch.from_numpy(codes).cuda(),
                 k, n, P, torch.from_numpy(table).cuda(), tc, (m, n, n, 1), route=route)
    assert np.array_equal(tc.cpu().numpy(), want)
    assert route.kernel == 4 and route.b_layout == 1


@pytest.mark.parametrize("P,N", [(1, 200), (4, 4), (8, 2), (2, 16)])
def test_other_packings_and_ragged(P, N):
    # n = 24 is not a multiple of 32 (rows the TMA cannot address): the decoded route
    m, k, n = 33, 40, 24
    for orientation in (0, 1):
        got, want, route = run(m, k, n, P, N, orientation, seed=P * 10 + N)
        assert np.array_equal(got, want), (P, N, orientation)


def test_strided_activations_gathered():
    m, k, n = 64, 96, 64
    got, want, route = run(m, k, n, 2, 16, 0, av=(m, k, 1, m), seed=9)
    assert np.array_equal(got, want)
    assert route.a_layout == 2


def test_codes_must_describe_the_shape():
    a = np.zeros(4, np.int8)
    codes = np.zeros(3, np.uint8)
    c = np.zeros(4, np.int32)
    with pytest.raises(U.DoesNotFit):
        U.coded_gemm(U.I32, a, (1, 4, 4, 1), codes, 4, 4, 2, np.zeros(16, np.int8), c,
                     (1, 4, 4, 1))
