"""Every BASELINE configuration at its full size, with whole blocks of output rows
compared against the CPU oracle bit for bit (no sampling of cells inside a row).

Each test runs the product once on the GPU through the C ABI, then recomputes 64 or
more complete rows with the oracle: a block that straddles a 256-row tile boundary of
the tensor-core kernels, plus the first and last rows. Sizes and operand
distributions are those of BASELINE.json's configs (the reference's xorshift corpus).
"""
import numpy as np
import pytest

import uor_b200 as U
from oracle import oracle as orc
from oracle.oracle import View
from float_data import config3
from gpu_util import needs_gpu, torch

pytestmark = [pytest.mark.gpu, needs_gpu, pytest.mark.slow]

THREADS = 0  # the oracle's OpenMP default: every host core


def row_blocks(m, block=64):
    """Row ranges checked: a block across the tile boundary nearest m / 2, the first
    and the last row."""
    mid = (m // 2) // 256 * 256
    lo = max(0, mid - block // 2)
    return [(lo, min(m, lo + block)), (0, 1), (m - 1, m)]


def test_i8_headline_8192_cubed_row_blocks():
    m = k = n = 8192
    a = U.corpus(1, U.CORPUS_I8, m * k)
    b = U.corpus(2, U.CORPUS_I8, k * n)
    tc = torch.empty(m * n, dtype=torch.int32, device="cuda")
    route = U.Route()
    U.gemm_i8_i32(m, k, n, torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), tc,
                  route=route)
    assert route.kernel == 1 and route.pairs == 1
    c = tc.cpu().numpy()
    for r0, r1 in row_blocks(m, 256):
        want = np.zeros((r1 - r0) * n, np.int32)
        orc.gemm_i8_blocked(a[r0 * k:r1 * k], b, want, r1 - r0, k, n)
        assert np.array_equal(c[r0 * n:r1 * n], want), (r0, r1)


@pytest.mark.parametrize("size", [4096, 8192])
def test_exact_f32_config3_row_blocks(size):
    """configs[2] at 4096^3, and the metric's second half at 8192^3 with the same
    distribution: rows 0, 10, 20, ... of the cancellation columns sum to exactly zero."""
    m = k = n = size
    a, b = config3(m, k, n)
    tc = torch.empty(m * n, dtype=torch.float32, device="cuda")
    route = U.Route()
    U.gemm_float(U.F32, U.F32, torch.from_numpy(a).reshape(-1).cuda(), (m, k, k, 1),
                 torch.from_numpy(b).reshape(-1).cuda(), (k, n, n, 1), tc, (m, n, n, 1),
                 route=route)
    assert route.kernel == 5
    c = tc.cpu().numpy().view(np.uint32)
    blocks = row_blocks(m) + [(0, 64)]
    for r0, r1 in blocks:
        want = np.zeros((r1 - r0) * n, np.float32)
        orc.gemm_float(View(a.reshape(-1), r1 - r0, k, k, 1, r0 * k),
                       View(b.reshape(-1), k, n, n, 1), View(want, r1 - r0, n, n, 1),
                       threads=THREADS)
        assert np.array_equal(c[r0 * n:r1 * n], want.view(np.uint32)), (size, r0, r1)
    for j in range(0, n, 10):
        assert c[(j % m) * n + j] == 0  # exact cancellation rounds to +0.0


def test_wide_i32_to_i128_config4_row_blocks():
    """i32 over the full range, k = 65536, every one of the 128 bits."""
    m, k, n = 1024, 65536, 1024
    a = U.corpus(4, U.CORPUS_I32_FULL, m * k)
    b = U.corpus(5, U.CORPUS_I32_FULL, k * n)
    tc = torch.zeros(m * n * 2, dtype=torch.int64, device="cuda")
    U.gemm(U.I32, U.I128, torch.from_numpy(a).cuda(), (m, k, k, 1), torch.from_numpy(b).cuda(),
           (k, n, n, 1), tc, (m, n, n, 1))
    c = tc.cpu().numpy()
    for r0, r1 in row_blocks(m):
        want = np.zeros((r1 - r0) * n * 2, np.int64)
        orc.gemm_int(View(a, r1 - r0, k, k, 1, r0 * k), View(b, k, n, n, 1),
                     View(want, r1 - r0, n, n, 1), out_bits=128, threads=THREADS)
        assert np.array_equal(c[2 * r0 * n:2 * r1 * n], want), (r0, r1)
    # the worst-case sums really leave the i64 range somewhere in the checked rows
    hi = c[1::2].astype(np.int64)
    lo = c[0::2]
    assert np.any((hi != 0) & (hi != -1)) or np.any((hi == 0) & (lo < 0))


@pytest.mark.parametrize("on_chip", [False, True])
def test_codec_config2_row_blocks(on_chip):
    """2048 x 8192 activations, 8192 x 8192 nibble codes, 16-entry book,
    decoded on chip (K1C, 512-row tiles), with and without CODEC_ON_CHIP."""
    m, k, n = 2048, 8192, 8192
    a = U.corpus(1, U.CORPUS_I8, m * k)
    q = U.corpus(2, U.CORPUS_NIBBLES, k * n)
    t = U.corpus(7, U.CORPUS_I8, 16)
    tc = torch.empty(m * n, dtype=torch.int32, device="cuda")
    route = U.Route()
    U.coded_gemm(U.I32, torch.from_numpy(a).cuda(), (m, k, k, 1), torch.from_numpy(q).cuda(), k,
                 n, 2, torch.from_numpy(t).cuda(), tc, (m, n, n, 1), route=route, on_chip=on_chip)
    assert route.b_layout != 3 and route.tile_m == 512
    c = tc.cpu().numpy()
    for r0, r1 in row_blocks(m):
        want = np.zeros((r1 - r0) * n, np.int32)
        orc.coded_gemm(View(a, r1 - r0, k, k, 1, r0 * k), q, 2, t, View(want, r1 - r0, n, n, 1),
                       k, n, threads=THREADS)
        assert np.array_equal(c[r0 * n:r1 * n], want), (r0, r1)


@pytest.mark.parametrize("tier,block,orientation", [(U.TIER_BOOK, 8, 0), (U.TIER_TERNARY, 4, 1)])
def test_byte_codec_tiers_full_size_row_blocks(tier, block, orientation):
    """configs[1]'s shape over codec tiers whose code byte holds whole elements, decoded on
    chip through K1C's byte table: the E8 book (Book<256, 8>, u8 codes, the bench's
    codec-e8 line) with codes k x n, and Ternary<4> with codes n x k (gemm_tabulated's
    layout)."""
    m, k, n = 2048, 8192, 8192
    a = U.corpus(1, U.CORPUS_I8, m * k)
    q = U.corpus(3, U.CORPUS_RAW, k * n // block).astype(np.uint8)
    table = U.e8_table() if tier == U.TIER_BOOK else None
    kw = {"table": torch.from_numpy(table).cuda()} if table is not None else {}
    tc = torch.empty(m * n, dtype=torch.int32, device="cuda")
    route = U.Route()
    U.codec_gemm(U.I32, torch.from_numpy(a).cuda(), (m, k, k, 1), tier, torch.from_numpy(q).cuda(),
                 k, n, tc, (m, n, n, 1), block=block, code_bytes=1, orientation=orientation,
                 route=route, **kw)
    assert route.b_layout == (1 if orientation == 0 else 0) and route.tile_m == 512
    rows, cols = (k, n) if orientation == 0 else (n, k)
    dense = orc.decode_codec_np(tier, q, rows, cols, table, block).reshape(-1)
    bv = View(dense, k, n, n, 1) if orientation == 0 else View(dense, k, n, 1, k)
    c = tc.cpu().numpy()
    for r0, r1 in row_blocks(m):
        want = np.zeros((r1 - r0) * n, np.int32)
        orc.gemm_int(View(a, r1 - r0, k, k, 1, r0 * k), bv, View(want, r1 - r0, n, n, 1),
                     threads=THREADS)
        assert np.array_equal(c[r0 * n:r1 * n], want), (r0, r1)


def test_tropical_config5_8192_cubed_row_blocks():
    """configs[4]'s max-plus half at its full size: Trop<i8> in [-64, 63] with 5 % -inf,
    Trop<i32> out; the value is compared where the cell is finite, the flag everywhere."""
    TD = orc.TROP_DTYPES
    m = k = n = 8192
    a = U.corpus(1, U.CORPUS_TROP_I8, m * k)
    b = U.corpus(2, U.CORPUS_TROP_I8, k * n)
    tc = torch.zeros(m * n * 8, dtype=torch.uint8, device="cuda")
    U.gemm_tropical(U.TROP_I8, U.TROP_I32, torch.from_numpy(a).cuda(), (m, k, k, 1),
                    torch.from_numpy(b).cuda(), (k, n, n, 1), tc, (m, n, n, 1))
    c = tc.cpu().numpy().view(TD[32])
    av, bv = a.view(TD[8]), b.view(TD[8])
    for r0, r1 in row_blocks(m):
        want = np.zeros((r1 - r0) * n, TD[32])
        orc.gemm_trop(View(av, r1 - r0, k, k, 1, r0 * k), View(bv, k, n, n, 1),
                      View(want, r1 - r0, n, n, 1), ebits=8, obits=32, threads=THREADS)
        got = c[r0 * n:r1 * n]
        assert np.array_equal(got["f"], want["f"]), (r0, r1)
        fin = want["f"] != 0
        assert np.array_equal(got["v"][fin], want["v"][fin]), (r0, r1)
