"""The other fixed-width codec tiers -- Sign, Ternary, Book, and Offset over any tier --
through uor_b200_codec_gemm, against the oracle's decode restatement and integer GEMM,
bit for bit, on both routes (code bytes of 4 or 8 whole elements decoded on chip, the
other shapes through a dense workspace); and the reference's spelling equivalences
CK-11 / CK-12."""
import numpy as np
import pytest

import uor_b200 as U
from oracle import oracle as orc
from gpu_util import i8, needs_gpu, out_array

pytestmark = [pytest.mark.gpu, needs_gpu]


def check(m, k, n, tier, codes, orientation=0, out=U.I32, alpha=1, beta=0, seed=0, **kw):
    a = i8(60 + seed, m * k)
    rows, cols = (k, n) if orientation == 0 else (n, k)
    dense = orc.decode_codec(tier, codes, rows, cols, kw.get("table"), kw.get("per_byte", 0),
                             kw.get("block", 1), kw.get("code_bytes", 1), kw.get("zero", 0))
    c0 = out_array(out, m * n)
    c0[:] = np.random.default_rng(seed).integers(-1000, 1000, size=c0.size)
    got, want = c0.copy(), c0.copy()
    route = U.Route()
    U.codec_gemm(out, a, (m, k, k, 1), tier, codes, k, n, got, (m, n, n, 1), alpha=alpha,
                 beta=beta, route=route, orientation=orientation, **kw)
    bv = (k, n, n, 1) if orientation == 0 else (k, n, 1, k)
    orc.gemm_int(orc.View(a, m, k, k, 1), orc.View(dense.reshape(-1), *bv),
                 orc.View(want, m, n, n, 1), alpha=alpha, beta=beta,
                 out_bits={U.I32: 32, U.I64: 64, U.I128: 128}[out])
    assert np.array_equal(got, want)
    return got, route


def codes_for(rows, cols, block, code_bytes, seed):
    count = rows * (cols // block) * code_bytes
    return U.corpus(seed, U.CORPUS_RAW, count).astype(np.uint8)


@pytest.mark.parametrize("orientation", [0, 1])
@pytest.mark.parametrize("block,cb", [(8, 1), (16, 2), (12, 2), (20, 2)])
def test_sign(orientation, block, cb):
    m, k, n = 70, 240, 240  # both multiples of every block width tested
    rows, cols = (k, n) if orientation == 0 else (n, k)
    codes = codes_for(rows, cols, block, cb, 5 + block)
    for zero in (0, -3):
        check(m, k, n, U.TIER_SIGN, codes, orientation, block=block, code_bytes=cb, zero=zero,
              seed=block)


@pytest.mark.parametrize("orientation", [0, 1])
@pytest.mark.parametrize("block,cb", [(4, 1), (8, 2), (6, 1), (12, 2)])
def test_ternary(orientation, block, cb):
    m, k, n = 300, 96, 144
    rows, cols = (k, n) if orientation == 0 else (n, k)
    codes = codes_for(rows, cols, block, cb, 9 + block)
    for zero, out in ((0, U.I32), (2, U.I64)):
        check(m, k, n, U.TIER_TERNARY, codes, orientation, out, 3, -1, block=block,
              code_bytes=cb, zero=zero, seed=block)


@pytest.mark.parametrize("orientation", [0, 1])
def test_book(orientation):
    # the E8 shape Book<256, 8> with u8 codes, a wider book with u16 codes, and 16-byte
    # blocks of a 300-entry book behind an Offset (u16 codes reduced modulo 300)
    for (N, block, cb, zero) in [(256, 8, 1, 0), (1000, 4, 2, 0), (300, 16, 2, -3)]:
        m, k, n = 130, 256, 192
        table = U.corpus(7, U.CORPUS_I8, N * block)
        if zero:
            # decode minus zero must stay i8 (Offset::new)
            table = np.clip(table, max(-128, -128 + zero), min(127, 127 + zero)).astype(np.int8)
        rows, cols = (k, n) if orientation == 0 else (n, k)
        codes = codes_for(rows, cols, block, cb, 11 + N)
        check(m, k, n, U.TIER_BOOK, codes, orientation, table=table, block=block, code_bytes=cb,
              zero=zero, seed=N)


@pytest.mark.parametrize("orientation", [0, 1])
@pytest.mark.parametrize("cb", [1, 2])
def test_e8_codebook(orientation, cb):
    """e8_codec_u8 (u8 codes) and e8_codec (u16 codes, taken modulo 256 rows) over the
    library's own E8 table (e8.rs); a zeroed code stream decodes to zero."""
    m, k, n = 96, 512, 256
    table = U.e8_table()
    rows, cols = (k, n) if orientation == 0 else (n, k)
    codes = codes_for(rows, cols, 8, cb, 21 + cb)
    check(m, k, n, U.TIER_BOOK, codes, orientation, table=table, block=8, code_bytes=cb,
          seed=30 + cb)
    zeros = np.zeros_like(codes)
    got, _ = check(m, k, n, U.TIER_BOOK, zeros, orientation, table=table, block=8,
                   code_bytes=cb, seed=40)
    assert not got.any()


@pytest.mark.parametrize("orientation", [0, 1])
@pytest.mark.parametrize("m", [1, 130, 600])
@pytest.mark.parametrize("tier,block,cb,N,zero", [
    (U.TIER_SIGN, 8, 1, 0, 0), (U.TIER_SIGN, 16, 2, 0, -3),
    (U.TIER_TERNARY, 4, 1, 0, 2), (U.TIER_TERNARY, 8, 2, 0, 0),
    (U.TIER_BOOK, 8, 1, 256, 0), (U.TIER_BOOK, 8, 1, 100, 0), (U.TIER_BOOK, 4, 1, 256, -3)])
def test_byte_codes_on_chip(orientation, m, tier, block, cb, N, zero):
    """Code bytes of 8 (Sign, Book<N, 8> with u8 codes) or 4 (Ternary, Book<N, 4>) whole
    elements decode inside the tensor-core pipeline through the byte table it builds
    (route.b_layout 1 or 0, never the dense workspace 3): 256-row tiles below 512 rows,
    512-row tiles from there, a reduction that is not a whole number of stages in
    orientation 0 and output columns that are not a whole number of tiles in orientation 1;
    Offset and the general epilogue (i64, alpha 3, beta -1) beside the plain s32 store."""
    k, n = (200, 384) if orientation == 0 else (384, 200)
    rows, cols = (k, n) if orientation == 0 else (n, k)
    kw = dict(block=block, code_bytes=cb, zero=zero)
    if tier == U.TIER_BOOK:
        table = U.corpus(17 + N, U.CORPUS_I8, N * block)
        kw["table"] = np.clip(table, -128 + max(zero, 0), 127 + min(zero, 0)).astype(np.int8)
    codes = codes_for(rows, cols, block, cb, 31 + block + N)
    out, alpha, beta = (U.I64, 3, -1) if zero else (U.I32, 1, 0)
    _, route = check(m, k, n, tier, codes, orientation, out, alpha, beta, seed=m + block, **kw)
    assert route.b_layout == (1 if orientation == 0 else 0)
    assert route.tile_m == (512 if m >= 512 else 256)


@pytest.mark.parametrize("orientation", [0, 1])
@pytest.mark.parametrize("m", [70, 520])
@pytest.mark.parametrize("tier,block,cb", [(U.TIER_SIGN, 16, 2), (U.TIER_TERNARY, 4, 1),
                                           (U.TIER_BOOK, 8, 1)])
def test_byte_codes_on_chip_deep_reduction(orientation, m, tier, block, cb):
    """A reduction deeper than one s32 lane (k = 131456: a full 130944 chunk and a ragged
    512) still decodes on chip: K1C per exact chunk into s32 planes, folded in 64 bits by
    the Linear epilogue (i64 out, alpha 3, beta -1)."""
    k, n = 131456, 128
    rows, cols = (k, n) if orientation == 0 else (n, k)
    a = i8(80 + m, m * k)
    codes = codes_for(rows, cols, block, cb, 50 + block)
    table = U.corpus(23, U.CORPUS_I8, 256 * block) if tier == U.TIER_BOOK else None
    dense = orc.decode_codec_np(tier, codes, rows, cols, table, block, cb).reshape(-1)
    c0 = np.random.default_rng(m).integers(-1000, 1000, size=m * n).astype(np.int64)
    got, want = c0.copy(), c0.copy()
    route = U.Route()
    kw = {"table": table} if table is not None else {}
    U.codec_gemm(U.I64, a, (m, k, k, 1), tier, codes, k, n, got, (m, n, n, 1), alpha=3, beta=-1,
                 route=route, orientation=orientation, block=block, code_bytes=cb, **kw)
    bv = (k, n, n, 1) if orientation == 0 else (k, n, 1, k)
    orc.gemm_int(orc.View(a, m, k, k, 1), orc.View(dense, *bv), orc.View(want, m, n, n, 1),
                 alpha=3, beta=-1)
    assert np.array_equal(got, want)
    assert route.k_chunks == 2 and route.b_layout == (1 if orientation == 0 else 0)
    assert route.tile_m == (512 if m >= 512 else 256)


@pytest.mark.parametrize("P", [2, 4])
def test_grid_with_offset(P):
    m, k, n = 260, 128, 96
    table = np.arange(-8, 8, dtype=np.int8)[: (16 if P == 2 else 4)]
    codes = U.corpus(3, U.CORPUS_RAW, k * n // P).astype(np.uint8)
    got, route = check(m, k, n, U.TIER_GRID, codes, table=table, per_byte=P, zero=5, seed=P)
    assert route.kernel == 4


def test_spellings_agree_ck11_ck12():
    """Sign<8> is Packed<Grid<2>, 8> over {-1, +1}; Ternary<4> is Packed<Grid<4>, 4> over
    {-1, 0, +1, 0}: the same bytes, the same product."""
    m, k, n = 50, 64, 256
    a = i8(70, m * k)
    for tier, P, table in [(U.TIER_SIGN, 8, [-1, 1]), (U.TIER_TERNARY, 4, [-1, 0, 1, 0])]:
        codes = U.corpus(13, U.CORPUS_RAW, k * n // P).astype(np.uint8)
        x = np.zeros(m * n, np.int32)
        y = np.zeros(m * n, np.int32)
        U.codec_gemm(U.I32, a, (m, k, k, 1), tier, codes, k, n, x, (m, n, n, 1), block=P,
                     code_bytes=1)
        U.coded_gemm(U.I32, a, (m, k, k, 1), codes, k, n, P, np.array(table, np.int8), y,
                     (m, n, n, 1))
        assert np.array_equal(x, y), tier


def test_validation():
    a = np.zeros(4, np.int8)
    c = np.zeros(4, np.int32)
    with pytest.raises(U.DoesNotFit):  # codes for 3 of 4 rows
        U.codec_gemm(U.I32, a, (1, 4, 4, 1), U.TIER_SIGN, np.zeros(3, np.uint8), 4, 4, c,
                     (1, 4, 4, 1), block=4, code_bytes=1)
    with pytest.raises(U.UorError):  # Offset image leaves i8
        U.codec_gemm(U.I32, a, (1, 4, 4, 1), U.TIER_SIGN, np.zeros(4, np.uint8), 4, 4, c,
                     (1, 4, 4, 1), block=4, code_bytes=1, zero=128)
