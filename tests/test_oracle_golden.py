"""The oracle pinned to the reference's golden vectors and known answers.

CX-10 / CX-11 are the reference's out-of-ecosystem NumPy oracles
(oracles/numpy, oracles/tropical). Their inputs come from a recorded generator
(oracles/numpy/generate.py, oracles/tropical/generate.py), restated here; the
regenerated inputs and the oracle's outputs must hash to the digests the
reference committed (tests/golden/cx_manifest.json).
"""
import hashlib
import json
import os
import struct

import numpy as np
import pytest

from oracle import oracle as orc
from oracle.oracle import View

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "cx_manifest.json")
MANIFEST = json.load(open(GOLDEN))


def sha(arr) -> str:
    return "sha256:" + hashlib.sha256(np.ascontiguousarray(arr).astype("<i8").tobytes()).hexdigest()


def cx10_inputs():
    """oracles/numpy/generate.py: one xorshift stream from SEED, values v % 1000 - 500."""
    seed = MANIFEST["cx10"]["seed"]
    s = seed
    for case in MANIFEST["cx10"]["cases"]:
        m, k, n = (case["shape"][x] for x in "mkn")
        states, s = orc.xorshift_stream(s, m * k + k * n)
        vals = (states >> np.uint64(33)).astype(np.int64) % 1000 - 500
        yield case, vals[: m * k].reshape(m, k), vals[m * k:].reshape(k, n)


@pytest.mark.parametrize("idx", range(len(MANIFEST["cx10"]["cases"])))
def test_cx10_int64_wrapping_matches_numpy_golden(idx):
    case, a, b = list(cx10_inputs())[idx]
    m, k, n = (case["shape"][x] for x in "mkn")
    assert sha(a) == case["a_sha256"], "the restated generator must reproduce the inputs"
    assert sha(b) == case["b_sha256"]
    c = np.zeros((m, n), dtype=np.int64)
    if m and n:
        orc.gemm_int(View.row_major(a, m, k), View.row_major(b, k, n), View.row_major(c, m, n),
                     mode=orc.WRAPPING)
    assert sha(c) == case["expected_sha256"]


def test_cx10_is_falsifiable():
    """A planted defect (one cell off by one) must change the digest."""
    case, a, b = list(cx10_inputs())[3]
    m, k, n = (case["shape"][x] for x in "mkn")
    c = np.zeros((m, n), dtype=np.int64)
    orc.gemm_int(View.row_major(a, m, k), View.row_major(b, k, n), View.row_major(c, m, n),
                 mode=orc.WRAPPING)
    c[0, 0] += 1
    assert sha(c) != case["expected_sha256"]


NEG_INF = -(1 << 63)
GOLD = 0x9E3779B97F4A7C15


def cx11_draw(seed, length, salt, mask, span=3):
    period, phase = mask
    states, _ = orc.xorshift_stream(seed ^ ((salt * GOLD) & orc.MASK64), length)
    vals = (states >> np.uint64(33)).astype(np.int64) % span - span // 2
    idx = np.arange(length)
    return np.where(idx % period == phase, NEG_INF, vals).astype(np.int64)


def to_trop8(vals):
    t = np.zeros(len(vals), dtype=orc.TROP_DTYPES[8])
    fin = vals != NEG_INF
    t["v"] = np.where(fin, vals, 0).astype(np.int8)
    t["f"] = fin.astype(np.uint8)
    return t


@pytest.mark.parametrize("idx", range(len(MANIFEST["cx11"]["cases"])))
def test_cx11_max_plus_matches_numpy_golden(idx):
    rec = MANIFEST["cx11"]
    case = rec["cases"][idx]
    m, k, n = (case["shape"][x] for x in "mkn")
    # Case i of the reference corpus draws from SEED + i (tropical/generate.py).
    order = [(1, 0, 1), (3, 0, 4), (0, 0, 0), (0, 5, 7), (5, 7, 0), (1, 1, 1), (7, 1, 5),
             (35, 1, 35), (3, 7, 11), (13, 17, 19), (23, 29, 31), (2, 97, 3), (1, 1024, 1),
             (4, 4093, 4), (128, 3, 128), (16, 64, 16)]
    seed = rec["seed"] + order.index((m, k, n))
    ma = (rec["mask_a"]["period"], rec["mask_a"]["phase"])
    mb = (rec["mask_b"]["period"], rec["mask_b"]["phase"])
    a = cx11_draw(seed, m * k, 1, ma)
    b = cx11_draw(seed, k * n, 2, mb)
    assert sha(a) == case["a_sha256"]
    assert sha(b) == case["b_sha256"]
    ta, tb = to_trop8(a), to_trop8(b)
    tc = np.zeros(m * n, dtype=orc.TROP_DTYPES[64])
    if m and n:
        orc.gemm_trop(View(ta, m, k, k, 1), View(tb, k, n, n, 1), View(tc, m, n, n, 1),
                      ebits=8, obits=64)
    got = np.where(tc["f"] != 0, tc["v"], NEG_INF).astype(np.int64)
    assert sha(got) == case["expected_sha256"]


# ---------------------------------------------------------------- KATs ------

def run_i8(a, b, m, k, n, alpha=1, beta=0, c=None, out=np.int32, mode=orc.NEAREST):
    a = np.asarray(a, dtype=np.int8)
    b = np.asarray(b, dtype=np.int8)
    c = np.zeros(m * n, dtype=out) if c is None else np.asarray(c, dtype=out).copy()
    orc.gemm_int(View.row_major(a, m, k), View.row_major(b, k, n), View.row_major(c, m, n),
                 alpha=alpha, beta=beta, mode=mode)
    return c.tolist()


def test_readme_kat():
    # README.md:38-42, driver.rs docs: [1,2;3,4] * [5,6;7,8] = [19,22;43,50]
    assert run_i8([1, 2, 3, 4], [5, 6, 7, 8], 2, 2, 2) == [19, 22, 43, 50]


def test_beta_zero_does_not_read_c():
    # driver.rs:356-372 (CS-04): C full of i32::MIN is overwritten.
    assert run_i8([1, 2, 3, 4], [5, 6, 7, 8], 2, 2, 2, c=[-2**31] * 4) == [19, 22, 43, 50]


def test_alpha_beta_exact():
    # driver.rs:377-392 (CS-05)
    got = run_i8([1, 2, 3, 4], [5, 6, 7, 8], 2, 2, 2, alpha=3, beta=-2, c=[100, 200, 300, 400])
    assert got == [3 * 19 - 200, 3 * 22 - 400, 3 * 43 - 600, 3 * 50 - 800]


def test_transposed_view():
    # driver.rs:408-439 (CS-06): A^T read through strides.
    a = np.array([1, 2, 3, 4, 5, 6], dtype=np.int8)
    b = np.array([1, 2, 3, 4, 5, 6], dtype=np.int8)
    d = np.zeros(9, dtype=np.int32)
    orc.gemm_int(View(a, 3, 2, 1, 3), View.row_major(b, 2, 3), View.row_major(d, 3, 3))
    assert d.tolist() == [17, 22, 27, 22, 29, 36, 27, 36, 45]


def test_depth_past_every_threshold():
    # driver.rs:743-759 (CT-01): k = 150000 of i8::MIN^2 into i64.
    k = 150_000
    a = np.full(k, -128, dtype=np.int8)
    b = np.full(k, -128, dtype=np.int8)
    c = np.zeros(1, dtype=np.int64)
    orc.gemm_int(View.row_major(a, 1, k), View.row_major(b, k, 1), View.row_major(c, 1, 1))
    assert c[0] == k * 128 * 128


def test_encode_kats():
    # acc.rs:1304-1328: 300 -> i8 saturates to 127 and wraps to 44; -300 -> -128 / -44.
    one = [1]
    assert run_i8([100], [3], 1, 1, 1, out=np.int8, mode=orc.SATURATING) == [127]
    assert run_i8([100], [3], 1, 1, 1, out=np.int8, mode=orc.WRAPPING) == [44]
    assert run_i8([-100], [3], 1, 1, 1, out=np.int8, mode=orc.SATURATING) == [-128]
    assert run_i8([-100], [3], 1, 1, 1, out=np.int8, mode=orc.WRAPPING) == [-44]
    assert run_i8([100], [3], 1, 1, 1, out=np.int32, mode=orc.SATURATING) == [300]
    del one


def test_i64_needs_192_bits():
    # acc.rs:1270-1283: 4 * i64::MIN^2 = 2^128 saturates an i128 output.
    a = np.full(4, -2**63, dtype=np.int64)
    b = np.full(4, -2**63, dtype=np.int64)
    c = np.zeros(1, dtype=np.int64)
    orc.gemm_int(View.row_major(a, 1, 4), View.row_major(b, 4, 1), View.row_major(c, 1, 1))
    assert c[0] == 2**63 - 1
    orc.gemm_int(View.row_major(a, 1, 4), View.row_major(b, 4, 1), View.row_major(c, 1, 1),
                 mode=orc.WRAPPING)
    assert c[0] == 0


def trop(vals, bits=8):
    t = np.zeros(len(vals), dtype=orc.TROP_DTYPES[bits])
    for i, v in enumerate(vals):
        if v is not None:
            t[i]["v"], t[i]["f"] = v, 1
    return t


def untrop(t):
    return [int(x["v"]) if x["f"] else None for x in t]


def run_trop(av, bv, m, k, n, alpha=(0, True), beta=(0, False), prior=None, obits=32):
    ta, tb = trop(av), trop(bv)
    tc = trop(prior if prior is not None else [None] * (m * n), obits)
    orc.gemm_trop(View.row_major(ta, m, k), View.row_major(tb, k, n), View.row_major(tc, m, n),
                  ebits=8, obits=obits, alpha=alpha, beta=beta)
    return untrop(tc)


def test_tropical_kats():
    # driver.rs:447-470 (CD-29): max-plus of [1,2;3,4],[5,6;7,8] = [9,10;11,12]
    assert run_trop([1, 2, 3, 4], [5, 6, 7, 8], 2, 2, 2) == [9, 10, 11, 12]
    # driver.rs:484-507 (CS-11): -inf beta overwrites a C holding i32::MAX
    assert run_trop([1, 2, 3, 4], [5, 6, 7, 8], 2, 2, 2, prior=[2**31 - 1] * 4) == [9, 10, 11, 12]
    # driver.rs:564-576 (CS-12): alpha shifts the product
    for alpha in (-40, -1, 0, 1, 37):
        assert run_trop([1, 2, 3, 4], [5, 6, 7, 8], 2, 2, 2, alpha=(alpha, True)) == \
            [9 + alpha, 10 + alpha, 11 + alpha, 12 + alpha]
    # driver.rs:578-593: beta shifts C, max takes the larger
    for beta, prior, want in [(0, -100, [9, 10, 11, 12]), (0, 100, [100] * 4),
                              (0, 10, [10, 10, 11, 12]), (5, 0, [9, 10, 11, 12]),
                              (-100, 100, [9, 10, 11, 12])]:
        assert run_trop([1, 2, 3, 4], [5, 6, 7, 8], 2, 2, 2, beta=(beta, True),
                        prior=[prior] * 4) == want
    # driver.rs:645-664: alpha at -inf absorbs everything
    assert run_trop([1, 2, 3, 4], [5, 6, 7, 8], 2, 2, 2, alpha=(0, False),
                    prior=[0] * 4) == [None] * 4
    # -inf in C under a finite beta contributes nothing
    assert run_trop([-5, -6, -7, -8], [-5, -6, -7, -8], 2, 2, 2, beta=(0, True),
                    prior=[None] * 4) == [-10, -11, -12, -13]
    # tropical.rs:336-351: finite values clamp to [MIN+1, MAX-1] of the output
    assert run_trop([127], [127], 1, 1, 1, obits=8) == [126]
    assert run_trop([-128], [-128], 1, 1, 1, obits=8) == [-127]


def test_nibble_order():
    # codecs.rs:181-195 / codec/tests/codec.rs:91: low sub-code first.
    table = np.arange(16, dtype=np.int8) * 3 - 20
    codes = np.array([0x21, 0x43], dtype=np.uint8)  # k=1 row, n=4 columns: 1,2,3,4
    a = np.array([1], dtype=np.int8)
    c = np.zeros(4, dtype=np.int32)
    orc.coded_gemm(View.row_major(a, 1, 1), codes, 2, table, View.row_major(c, 1, 4), 1, 4)
    assert c.tolist() == [int(table[1]), int(table[2]), int(table[3]), int(table[4])]


# ------------------------------------------------ C vs Python restatements ---

@pytest.mark.parametrize("seed", range(6))
def test_c_int_matches_python_twin(seed):
    rng = np.random.default_rng(seed)
    m, k, n = rng.integers(1, 9, size=3)
    for ebits, obits in ((8, 32), (16, 64), (32, 64), (8, 8), (32, 16)):
        et = orc.INT_DTYPES[ebits]
        info = np.iinfo(et)
        a = rng.integers(info.min, info.max, size=(m, k), endpoint=True).astype(et)
        b = rng.integers(info.min, info.max, size=(k, n), endpoint=True).astype(et)
        ot = orc.INT_DTYPES[obits]
        oinfo = np.iinfo(ot)
        c0 = rng.integers(oinfo.min, oinfo.max, size=(m, n), endpoint=True).astype(ot)
        for alpha, beta in ((1, 0), (3, -1), (-(2**63), 2**62), (2**63 - 1, -7)):
            for mode in (orc.NEAREST, orc.WRAPPING):
                c = c0.copy()
                orc.gemm_int(View.row_major(a, m, k), View.row_major(b, k, n),
                             View.row_major(c, m, n), alpha=alpha, beta=beta, mode=mode)
                want = orc.int_gemm_py(a.tolist(), b.tolist(), alpha, beta, c0.tolist(), obits,
                                       mode)
                assert c.tolist() == want, (ebits, obits, alpha, beta, mode)


def _rand_floats(rng, shape, is64, specials=True):
    """Random finite floats over a wide exponent range, plus zeros/subnormals/non-finites."""
    if is64:
        bits = rng.integers(0, 2**63, size=shape, dtype=np.uint64) | (
            rng.integers(0, 2, size=shape).astype(np.uint64) << np.uint64(63))
        x = bits.view(np.float64)
    else:
        bits = rng.integers(0, 2**32, size=shape, dtype=np.uint64).astype(np.uint32)
        x = bits.view(np.float32)
    x = x.copy()
    if not specials:
        x[~np.isfinite(x)] = 1.5
    return x


@pytest.mark.parametrize("seed", range(8))
def test_c_float_matches_big_int_twin(seed):
    rng = np.random.default_rng(100 + seed)
    for e64, o64 in ((False, False), (True, True), (False, True), (True, False)):
        m, k, n = rng.integers(1, 5, size=3)
        et = np.float64 if e64 else np.float32
        ot = np.float64 if o64 else np.float32
        a = _rand_floats(rng, (m, k), e64, specials=seed % 2 == 0)
        b = _rand_floats(rng, (k, n), e64, specials=seed % 2 == 0)
        # tame half of the exponents so cancellation and normal ranges are hit too
        if seed % 3 == 0:
            a = (rng.standard_normal((m, k)) * 8).astype(et)
            b = (rng.standard_normal((k, n)) * 8).astype(et)
            b[:, 0] = -a[0, ::-1] if k == m else b[:, 0]
        c0 = (rng.standard_normal((m, n))).astype(ot)
        for alpha, beta in ((1, 0), (3, -2), (0, 1), (-1, 5)):
            for mode in (orc.NEAREST, orc.TOWARD_ZERO):
                c = c0.copy()
                orc.gemm_float(View.row_major(a, m, k), View.row_major(b, k, n),
                               View.row_major(c, m, n), alpha=alpha, beta=beta, mode=mode)
                want = orc.float_gemm_py(a.tolist(), b.tolist(), alpha, beta, c0.tolist(),
                                         e64, o64, mode)
                got = c.view(np.uint64 if o64 else np.uint32).tolist()
                assert got == want, (e64, o64, alpha, beta, mode)


def f32bits(x):
    return struct.unpack("<I", struct.pack("<f", x))[0]


def run_f32(a, b, m, k, n, alpha=1, beta=0, c=None, mode=orc.NEAREST):
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    c = np.zeros(m * n, dtype=np.float32) if c is None else np.asarray(c, dtype=np.float32).copy()
    orc.gemm_float(View.row_major(a, m, k), View.row_major(b, k, n), View.row_major(c, m, n),
                   alpha=alpha, beta=beta, mode=mode)
    return c.view(np.uint32).tolist()


def test_float_epilogue_kats():
    # epilogue.rs:420-440: alpha = i64::MIN, beta = 2^62 cancels 0.5 against 1.0 exactly -> +0
    for mode in (orc.NEAREST, orc.TOWARD_ZERO, orc.SATURATING, orc.WRAPPING):
        assert run_f32([0.5], [1.0], 1, 1, 1, alpha=-(2**63), beta=2**62, c=[1.0],
                       mode=mode) == [0]
    big = np.finfo(np.float32).max
    # epilogue.rs:442-476: overflow is inf under Nearest, MAX under the directed modes
    assert run_f32([big], [big], 1, 1, 1, alpha=2**63 - 1) == [f32bits(float("inf"))]
    assert run_f32([big], [big], 1, 1, 1, alpha=-(2**63)) == [f32bits(float("-inf"))]
    for mode in (orc.TOWARD_ZERO, orc.SATURATING, orc.WRAPPING):
        assert run_f32([big], [big], 1, 1, 1, alpha=2**63 - 1, mode=mode) == [f32bits(big)]
        assert run_f32([big], [big], 1, 1, 1, alpha=-(2**63), mode=mode) == [f32bits(-big)]
    # epilogue.rs:478-497: -1 flips an infinity; 0 times infinity is NaN
    assert run_f32([float("inf")], [1.0], 1, 1, 1, alpha=-1) == [f32bits(float("-inf"))]
    assert run_f32([float("inf")], [1.0], 1, 1, 1, alpha=0) == [0x7FC00000]
    # alphabet.rs:866-870: inf * 0 is NaN; +inf and -inf make NaN
    assert run_f32([float("inf")], [0.0], 1, 1, 1) == [0x7FC00000]
    assert run_f32([float("inf"), float("inf")], [1.0, -1.0], 1, 2, 1) == [0x7FC00000]
    # acc.rs:1760-1766: exact cancellation is +0, never -0
    assert run_f32([1.5, 1.5], [2.0, -2.0], 1, 2, 1) == [0]
    # correctly rounded, not BLAS-rounded: 1 + 2^-24 + 2^-24 rounds to 1 + 2^-23
    e = 2.0 ** -24
    assert run_f32([1.0, e, e], [1.0, 1.0, 1.0], 1, 3, 1) == [f32bits(1.0 + 2.0 ** -23)]


def test_complete_register_drops_out_of_range_coordinates():
    """Complete::add_scaled (acc.rs:939-998) drops a coordinate whose lowest bit is
    below the register or whose first limb is past its last low limb. Reachable only
    through beta * C with f32 elements and an f64 output: C = 2^400 or 1.5 * 2^-297
    contributes nothing, while C = 3 contributes."""
    a = np.array([1.0], np.float32)
    b = np.array([2.0], np.float32)
    for prior, want in ((2.0 ** 400, 2.0), (1.5 * 2.0 ** -297, 2.0), (3.0, 5.0)):
        c = np.array([prior], np.float64)
        orc.gemm_float(View(a, 1, 1, 1, 1), View(b, 1, 1, 1, 1), View(c, 1, 1, 1, 1), beta=1)
        twin = orc.float_gemm_py([[1.0]], [[2.0]], 1, 1, [[prior]], False, True)[0][0]
        assert int(c.view(np.uint64)[0]) == twin
        assert c[0] == want


def test_codec_tier_decode_restatement():
    """The fixed-width tiers' decode (codecs.rs): Sign bit order (low first, set +1),
    Ternary digits (0 -> -1, 1 -> 0, 2 -> +1, 3 -> 0; past the code's width -> -1),
    Book rows, Offset, and Packed sub-code order (CK-03)."""
    dec = orc.decode_codec
    assert dec(1, np.array([0b10110001], np.uint8), 1, 8, block=8).tolist() == [
        [1, -1, -1, -1, 1, 1, -1, 1]]
    assert dec(1, np.array([0xFF, 0x01], np.uint8), 1, 20, block=20, code_bytes=2).tolist() == [
        [1] * 9 + [-1] * 11]
    assert dec(2, np.array([0b11100100], np.uint8), 1, 6, block=6).tolist() == [
        [-1, 0, 1, 0, -1, -1]]
    book = np.arange(-6, 6, dtype=np.int8)  # N = 3 rows of BLK = 4
    assert dec(3, np.array([1, 5], np.uint8), 1, 8, table=book, block=4).tolist() == [
        [-2, -1, 0, 1, 2, 3, 4, 5]]
    assert dec(0, np.array([0x21], np.uint8), 1, 2, table=np.arange(16, dtype=np.int8),
               per_byte=2, zero=3).tolist() == [[-2, -1]]


@pytest.mark.parametrize("seed", range(6))
def test_codec_decode_numpy_twin_matches_loops(seed):
    """decode_codec_np (whole-array numpy, for full-size cases) against the element loops,
    on random shapes of every fixed-width tier, u8 and u16 codes, widths past the code's
    bits, and Offset."""
    rng = np.random.default_rng(200 + seed)
    for tier in (1, 2, 3):
        for cb in (1, 2):
            block = int(rng.integers(1, 21))
            rows, cpr = int(rng.integers(1, 6)), int(rng.integers(1, 5))
            cols = cpr * block
            codes = rng.integers(0, 256, size=rows * cpr * cb).astype(np.uint8)
            table = (rng.integers(-100, 100, size=int(rng.integers(1, 40)) * block)
                     .astype(np.int8) if tier == 3 else None)
            zero = int(rng.integers(-3, 4))
            want = orc.decode_codec(tier, codes, rows, cols, table, 0, block, cb, zero)
            got = orc.decode_codec_np(tier, codes, rows, cols, table, block, cb, zero)
            assert np.array_equal(got, want), (tier, cb, block)


def test_complex_mac_kat():
    """complex_mac_is_componentwise_ck_01 (alphabet.rs:824-833): (3 + 4i)(5 - 2i) = 23 + 14i."""
    a, b = np.array([3, 4], np.int32), np.array([5, -2], np.int32)
    c = np.zeros(2, np.int32)
    orc.gemm_complex(View(a, 1, 1, 1, 1), View(b, 1, 1, 1, 1), View(c, 1, 1, 1, 1))
    assert c.tolist() == [23, 14]
    assert orc.complex_gemm_py([[(3, 4)]], [[(5, -2)]]) == [[(23, 14)]]


def test_complex_negation_wraps_like_the_release_build():
    """-w.im of MIN is MIN (Cargo.toml's release profile has overflow-checks off), so
    a.im * (-w.im) = a.im * MIN there."""
    for ebits, et in ((32, np.int32), (64, np.int64)):
        lo = int(np.iinfo(et).min)
        a, b = np.array([0, 1], et), np.array([0, lo], et)
        c = np.zeros(4, np.int64)  # Complex<i128>
        orc.gemm_complex(View(a, 1, 1, 1, 1), View(b, 1, 1, 1, 1), View(c, 1, 1, 1, 1),
                         out_bits=128)
        re = int(c[0].astype(np.uint64)) + (int(c[1]) << 64)
        assert re == lo  # not -lo
        assert orc.complex_gemm_py([[(0, 1)]], [[(0, lo)]], ebits, out_bits=128) == [[(lo, 0)]]


@pytest.mark.parametrize("seed", range(4))
def test_c_complex_matches_python_twin(seed):
    rng = np.random.default_rng(100 + seed)
    m, k, n = (int(x) for x in rng.integers(1, 7, size=3))
    for ebits, obits in ((32, 32), (32, 64), (64, 64), (64, 16)):
        et, ot = orc.INT_DTYPES[ebits], orc.INT_DTYPES[obits]
        info, oinfo = np.iinfo(et), np.iinfo(ot)
        a = rng.integers(info.min, info.max, size=2 * m * k, endpoint=True).astype(et)
        b = rng.integers(info.min, info.max, size=2 * k * n, endpoint=True).astype(et)
        b[1::7] = info.min  # imaginary parts at MIN exercise the wrapping negation
        c0 = rng.integers(oinfo.min, oinfo.max, size=2 * m * n, endpoint=True).astype(ot)
        pairs = lambda x, r, q: [[(int(x[2 * (i * q + j)]), int(x[2 * (i * q + j) + 1]))
                                  for j in range(q)] for i in range(r)]
        for alpha, beta in ((1, 0), (3, -1), (-(2**63), 2**62)):
            for mode in (orc.NEAREST, orc.WRAPPING):
                c = c0.copy()
                orc.gemm_complex(View(a, m, k, k, 1), View(b, k, n, n, 1), View(c, m, n, n, 1),
                                 alpha=alpha, beta=beta, mode=mode)
                want = orc.complex_gemm_py(pairs(a, m, k), pairs(b, k, n), ebits, alpha, beta,
                                           pairs(c0, m, n), obits, mode)
                assert pairs(c, m, n) == want, (ebits, obits, alpha, beta, mode)
