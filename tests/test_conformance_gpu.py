"""The reference's determinism gates (CONFORMANCE.md, the CD-* table) run against the
GPU path through the C ABI, every result also compared with the CPU oracle bit for bit.

CD-01  backend choice does not change bytes (byte slices, modular residues, default)
CD-04  operand traversal and layout do not change bytes
CD-05 / CD-28  for a fixed accumulation only the encode mode changes bytes
CD-02  tile count and completion order do not change bytes
CD-07  splitting the operand stream at any index sums the parts
CD-10  every scratch offer gives the same bytes (slice::gemm_ex_full)
CD-19 / CD-30  every public float spelling gives the exact reference bytes
CD-22  the default entry names a route in the census, and every route returns the
       reference's bytes
CD-24  the selection witness is invariant under partition and order
"""
import ctypes

import numpy as np
import pytest

import uor_b200 as U
import uor_b200_dist as D
from oracle import oracle as orc
from oracle.oracle import View
from gpu_util import i8, i128_values, needs_gpu, oracle_int, out_array, torch

pytestmark = [pytest.mark.gpu, needs_gpu]

FT = {U.F32: np.float32, U.F64: np.float64}
UT = {U.F32: np.uint32, U.F64: np.uint64}


def _oracle_i8(a, b, m, k, n, out=U.I32, alpha=1, beta=0, prior=None, mode=U.NEAREST):
    want = out_array(out, m * n) if prior is None else prior.copy()
    oracle_int(a, (m, k, k, 1, 0), b, (k, n, n, 1, 0), want, (m, n, n, 1, 0), alpha, beta, mode,
               out)
    return want


# ------------------------------------------------------------------ CD-01

@pytest.mark.parametrize("elem,out", [(U.I16, U.I64), (U.I32, U.I128), (U.I64, U.I128)])
def test_cd01_backend_choice_does_not_change_bytes(elem, out):
    """The byte-slice pairs, the modular residue route and the library's own choice."""
    m, k, n = 150, 700, 130
    dt = {U.I16: np.int16, U.I32: np.int32, U.I64: np.int64}[elem]
    raw_a = U.corpus(81, U.CORPUS_RAW, m * k)
    raw_b = U.corpus(82, U.CORPUS_RAW, k * n)
    a = (raw_a << np.uint64(31) ^ raw_a).view(np.int64).astype(dt, casting="unsafe")
    b = (raw_b << np.uint64(31) ^ raw_b).view(np.int64).astype(dt, casting="unsafe")
    want = out_array(out, m * n)
    oracle_int(a, (m, k, k, 1, 0), b, (k, n, n, 1, 0), want, (m, n, n, 1, 0), 1, 0,
               U.WRAPPING, out)
    results = []
    for flags in ({"digits": True}, {"modular": True}, {}):
        got = out_array(out, m * n)
        U.gemm(elem, out, a, (m, k, k, 1), b, (k, n, n, 1), got, (m, n, n, 1),
               encode=U.WRAPPING, **flags)
        results.append(got)
        assert i128_values(got) == i128_values(want) if out == U.I128 else \
            np.array_equal(got, want), flags
    assert all(np.array_equal(results[0], r) for r in results[1:])


# ------------------------------------------------------------------ CD-02

@pytest.mark.parametrize("tiles", [1, 2, 3, 5, 8, 64, "cells"])
def test_cd02_tile_count_and_order_do_not_change_bytes(tiles):
    """C computed tile by tile (partition.rs:34-111), the tiles in a shuffled order,
    equals the one-call result and the oracle."""
    m, k, n = 23, 300, 29
    a, b = i8(90, m * k), i8(91, k * n)
    prior = U.corpus(92, U.CORPUS_RAW, m * n).astype(np.int64)
    want = _oracle_i8(a, b, m, k, n, U.I64, 3, -2, prior)
    if tiles == "cells":
        part = D.Partition(m, n, 1, 1)
    else:
        per = -(-m * n // tiles)
        tc = max(1, min(n, per))
        tr = max(1, -(-per // tc))
        part = D.Partition(m, n, tr, tc)
    order = np.random.default_rng(7).permutation(len(part))
    got = prior.copy()
    for idx in order:
        t = part.tile(int(idx))
        off = t.row * n + t.col
        U.gemm(U.I8, U.I64, a[t.row * k:], (t.rows, k, k, 1), b[t.col:], (k, t.cols, n, 1),
               got[off:], (t.rows, t.cols, n, 1), 3, -2)
    assert np.array_equal(got, want)


# ------------------------------------------------------------------ CD-07

@pytest.mark.parametrize("split", [0, 1, 127, 128, 129, 1000, 2047, 2048])
def test_cd07_splitting_the_operand_stream_sums_the_parts(split):
    """C = A[:, :s] B[:s] then C += A[:, s:] B[s:] (beta = 1) equals the whole
    product at every split index, on the device path."""
    m, k, n = 40, 2048, 72
    a, b = i8(93, m * k), i8(94, k * n)
    want = _oracle_i8(a, b, m, k, n, U.I64)
    a2 = a.reshape(m, k)
    left = np.ascontiguousarray(a2[:, :split]).reshape(-1)
    right = np.ascontiguousarray(a2[:, split:]).reshape(-1)
    got = np.zeros(m * n, np.int64)
    U.slice_gemm_ex(U.I8, U.I64, m, split, n, 1, left, split, b, n, 0, got, n)
    U.slice_gemm_ex(U.I8, U.I64, m, k - split, n, 1, right, k - split, b[split * n:], n, 1, got, n)
    assert np.array_equal(got, want)


# ------------------------------------------------------------------ CD-10

def test_cd10_every_scratch_offer_gives_the_same_bytes():
    """slice::gemm_ex_full with no offer, one byte, one short of a panel, a panel and
    ten panels, for both the panel and the accumulator offers."""
    m, k, n = 130, 400, 150
    a, b = i8(95, m * k), i8(96, k * n)
    prior = U.corpus(97, U.CORPUS_RAW, m * n).astype(np.int64).astype(np.int32)
    want = _oracle_i8(a, b, m, k, n, U.I32, -5, 3, prior)
    panel = k * 128
    for offer in (0, 1, panel - 1, panel, 10 * panel):
        scratch = np.full(max(offer, 1), 0x5A, np.int8)
        acc = np.full(max(offer, 1), -1, np.int32)
        got = prior.copy()
        call = U.make_call()
        st = U.lib().uor_b200_slice_gemm_ex_full(
            U.I8, U.I32, m, k, n, -5, a.ctypes.data, a.size, k, b.ctypes.data, b.size, n, 3,
            got.ctypes.data, got.size, n, scratch.ctypes.data if offer else None, offer,
            acc.ctypes.data if offer else None, offer, ctypes.byref(call))
        assert st == U.OK
        assert np.array_equal(got, want), offer


# ------------------------------------------------------------------ CD-19 / CD-30

def _float_operands(elem, m, k, n):
    """Values spread over every IEEE code class: normals of wide exponent, subnormals,
    signed zeros, and (in one row and one column) infinities and a NaN."""
    rng = np.random.default_rng(11 + elem)
    dt, ut = FT[elem], UT[elem]
    bits = 32 if elem == U.F32 else 64

    def draw(count):
        x = (rng.standard_normal(count) * np.exp2(rng.integers(-40, 40, count))).astype(dt)
        pick = rng.integers(0, 40, count)
        x[pick == 0] = dt(0.0)
        x[pick == 1] = -dt(0.0)
        sub = rng.integers(1, 1 << 20, count).astype(ut)
        x[pick == 2] = sub[pick == 2].view(dt)
        return x
    a, b = draw(m * k), draw(k * n)
    a[3 * k + 1] = np.inf
    b[5 * n + 2] = -np.inf
    a[7 * k + 4] = np.nan
    assert bits in (32, 64)
    return a, b


@pytest.mark.parametrize("elem,out", [(U.F32, U.F32), (U.F32, U.F64), (U.F64, U.F64),
                                      (U.F64, U.F32)])
def test_cd19_cd30_every_float_spelling_gives_the_reference_bytes(elem, out):
    """gemm_float over views, slice::gemm_float_ex with and without PackedCode offers,
    and raw::sgemm / raw::dgemm all give the oracle's bytes."""
    m, k, n = 37, 90, 41
    a, b = _float_operands(elem, m, k, n)
    prior = np.random.default_rng(2).standard_normal(m * n).astype(FT[out])
    alpha, beta = 3, -1
    want = prior.copy()
    orc.gemm_float(View(a, m, k, k, 1), View(b, k, n, n, 1), View(want, m, n, n, 1),
                   alpha=alpha, beta=beta)
    want_bits = want.view(UT[out])
    # the view API
    got = prior.copy()
    U.gemm_float(elem, out, a, (m, k, k, 1), b, (k, n, n, 1), got, (m, n, n, 1), alpha, beta)
    assert np.array_equal(got.view(UT[out]), want_bits)
    # slice::gemm_float_ex: no offer, then 16-byte PackedCode caches of several sizes
    for offer in (0, 1, m * k, 10 * m * k):
        pa = np.zeros(max(1, 2 * offer), np.int64)
        pb = np.zeros(max(1, 2 * offer), np.int64)
        got = prior.copy()
        call = U.make_call()
        st = U.lib().uor_b200_slice_gemm_float_ex(
            elem, out, m, k, n, alpha, a.ctypes.data, a.size, k, b.ctypes.data, b.size, n, beta,
            got.ctypes.data, got.size, n, pa.ctypes.data if offer else None, offer,
            pb.ctypes.data if offer else None, offer, ctypes.byref(call))
        assert st == U.OK
        assert np.array_equal(got.view(UT[out]), want_bits), offer
    if elem == out:
        got = prior.copy()
        fn = U.sgemm if elem == U.F32 else U.dgemm
        fn(m, k, n, alpha, a, k, 1, b, n, 1, beta, got, n, 1)
        assert np.array_equal(got.view(UT[out]), want_bits)


def test_cd30_python_wrapper_of_the_slice_spelling():
    m, k, n = 20, 33, 18
    a, b = _float_operands(U.F32, m, k, n)
    got = np.zeros(m * n, np.float32)
    U.slice_gemm_float_ex(U.F32, U.F32, m, k, n, 1, a, k, b, n, 0, got, n)
    want = np.zeros(m * n, np.float32)
    orc.gemm_float(View(a, m, k, k, 1), View(b, k, n, n, 1), View(want, m, n, n, 1))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ------------------------------------------------------------------ CD-22

@pytest.mark.parametrize("elem,out,shape", [
    (U.I8, U.I32, (1, 4096, 1)), (U.I8, U.I32, (3, 50, 5000)), (U.I8, U.I32, (300, 256, 300)),
    (U.I8, U.I64, (1, 8192, 640)), (U.I8, U.I32, (640, 8192, 1)),
    (U.I16, U.I64, (70, 300, 90)), (U.I32, U.I128, (130, 600, 120))])
def test_cd22_default_entry_names_a_route_and_returns_the_reference_bytes(elem, out, shape):
    m, k, n = shape
    dt = {U.I8: np.int8, U.I16: np.int16, U.I32: np.int32}[elem]
    a = U.corpus(98, U.CORPUS_I32_FULL, m * k).astype(dt, casting="unsafe")
    b = U.corpus(99, U.CORPUS_I32_FULL, k * n).astype(dt, casting="unsafe")
    got = out_array(out, m * n)
    route = U.Route()
    U.gemm(elem, out, a, (m, k, k, 1), b, (k, n, n, 1), got, (m, n, n, 1), route=route)
    assert route.kernel != 0 and route.as_dict()["kernel_name"] not in ("none", "?")
    want = out_array(out, m * n)
    oracle_int(a, (m, k, k, 1, 0), b, (k, n, n, 1, 0), want, (m, n, n, 1, 0), 1, 0, U.NEAREST,
               out)
    if out == U.I128:
        assert i128_values(got) == i128_values(want)
    else:
        assert np.array_equal(got, want)


# ------------------------------------------------------------------ CD-24

def test_cd24_selection_witness_is_invariant_under_partition_and_order():
    """gemm_selected over the whole product and tile by tile (several tile shapes, the
    tiles in shuffled orders) writes the same values and the same witness indices."""
    TD = orc.TROP_DTYPES
    m, k, n = 33, 257, 47
    raw_a = U.corpus(100, U.CORPUS_RAW, m * k)
    raw_b = U.corpus(101, U.CORPUS_RAW, k * n)
    a = np.zeros(m * k, TD[8])
    b = np.zeros(k * n, TD[8])
    # values in {-1, 0, 1}: many ties, so the least-index rule decides most witnesses
    a["v"] = (raw_a % np.uint64(3)).astype(np.int8) - 1
    b["v"] = (raw_b % np.uint64(3)).astype(np.int8) - 1
    a["f"] = (raw_a >> np.uint64(20)) % np.uint64(10) != 0
    b["f"] = (raw_b >> np.uint64(20)) % np.uint64(10) != 0
    a["v"][a["f"] == 0] = 0  # the semiring zero stores value 0 (tropical.rs:61-70)
    b["v"][b["f"] == 0] = 0
    ab, bb = a.view(np.uint8), b.view(np.uint8)
    whole_c = np.zeros(m * n * 8, np.uint8)
    whole_w = np.zeros(m * n, np.uint64)
    U.gemm_tropical_selected(U.TROP_I8, U.TROP_I32, ab, (m, k, k, 1), bb, (k, n, n, 1), whole_c,
                             (m, n, n, 1), whole_w, (m, n, n, 1))
    for tr, tc, seed in [(1, 1, 0), (5, 7, 1), (33, 1, 2), (8, 47, 3)]:
        part = D.Partition(m, n, tr, tc)
        c = np.zeros(m * n * 8, np.uint8)
        w = np.zeros(m * n, np.uint64)
        for idx in np.random.default_rng(seed).permutation(len(part)):
            t = part.tile(int(idx))
            off = t.row * n + t.col
            U.gemm_tropical_selected(U.TROP_I8, U.TROP_I32, ab[2 * t.row * k:], (t.rows, k, k, 1),
                                     bb[2 * t.col:], (k, t.cols, n, 1), c[8 * off:],
                                     (t.rows, t.cols, n, 1), w[off:], (t.rows, t.cols, n, 1))
        assert np.array_equal(w, whole_w), (tr, tc)
        cv, wv = c.view(TD[32]), whole_c.view(TD[32])
        assert np.array_equal(cv["f"], wv["f"])
        fin = wv["f"] != 0
        assert np.array_equal(cv["v"][fin], wv["v"][fin])
    # and the values agree with the oracle's max-plus product
    want = np.zeros(m * n, TD[32])
    orc.gemm_trop(View(a, m, k, k, 1), View(b, k, n, n, 1), View(want, m, n, n, 1), ebits=8,
                  obits=32)
    wv = whole_c.view(TD[32])
    assert np.array_equal(wv["f"], want["f"])
    fin = want["f"] != 0
    assert np.array_equal(wv["v"][fin], want["v"][fin])
    # the witness attains the maximum at the least index
    wi = orc.trop_witness(a["v"].reshape(m, k), a["f"].reshape(m, k) != 0,
                          b["v"].reshape(k, n), b["f"].reshape(k, n) != 0)
    assert np.array_equal(np.asarray(wi, np.uint64).reshape(-1), whole_w)


# ------------------------------------------------------------------ CD-04, CD-05 / CD-28

def test_cd04_traversal_and_layout_do_not_change_bytes():
    """The same product through every operand layout the device path distinguishes (A
    K-major, A MN-major, A gathered; B MN-major, K-major, read backwards, gathered), and
    through the host-pointer pipeline and device pointers: one set of bytes."""
    m, k, n = 288, 400, 272
    a, b = i8(110, m * k), i8(111, k * n)
    want = _oracle_i8(a, b, m, k, n, U.I64, 5, 0)
    at = np.ascontiguousarray(a.reshape(m, k).T).reshape(-1)
    bt = np.ascontiguousarray(b.reshape(k, n).T).reshape(-1)
    brev = b.reshape(k, n)[::-1].copy().reshape(-1)
    apad = np.zeros(m * (k + 3), np.int8)
    apad.reshape(m, k + 3)[:, :k] = a.reshape(m, k)
    cases = [(a, (m, k, k, 1), b, (k, n, n, 1)), (at, (m, k, 1, m), b, (k, n, n, 1)),
             (a, (m, k, k, 1), bt, (k, n, 1, k)), (a, (m, k, k, 1), brev, (k, n, -n, 1)),
             (apad, (m, k, k + 3, 1), b, (k, n, n, 1)), (at, (m, k, 1, m), bt, (k, n, 1, k))]
    layouts = set()
    for aa, av, bb, bv in cases:
        got = np.zeros(m * n, np.int64)
        route = U.Route()
        U.gemm(U.I8, U.I64, aa, av, bb, bv, got, (m, n, n, 1), 5, 0, route=route)
        assert np.array_equal(got, want), (av, bv)
        layouts.add((route.a_layout, route.b_layout))
    assert len(layouts) >= 4  # the cases really took different operand layouts
    got = torch.zeros(m * n, dtype=torch.int64, device="cuda")
    U.gemm(U.I8, U.I64, torch.from_numpy(a).cuda(), (m, k, k, 1), torch.from_numpy(b).cuda(),
           (k, n, n, 1), got, (m, n, n, 1), 5, 0)
    assert np.array_equal(got.cpu().numpy(), want)


@pytest.mark.parametrize("out", [U.I8, U.I16, U.I32])
def test_cd05_cd28_only_the_encode_mode_changes_bytes(out):
    """For one fixed accumulation each encode gives the oracle's bytes (into an integer
    output Nearest, TowardZero and Saturating all clamp, acc.rs:128-151, and Wrapping
    truncates), and nothing else -- host or device buffers, a padded output -- changes the
    bytes of a given encode."""
    m, k, n = 40, 700, 56
    a, b = i8(112, m * k), i8(113, k * n)
    alpha = 2**20  # pushes most cells past the narrow output ranges
    outs = {}
    for mode in (U.NEAREST, U.TOWARD_ZERO, U.SATURATING, U.WRAPPING):
        want = _oracle_i8(a, b, m, k, n, out, alpha, 0, mode=mode)
        got = out_array(out, m * n)
        U.gemm(U.I8, out, a, (m, k, k, 1), b, (k, n, n, 1), got, (m, n, n, 1), alpha, 0, mode)
        assert np.array_equal(got, want), mode
        # the same encode through device buffers and a padded output gives the same bytes
        ldc = n + 5
        dev = torch.zeros(m * ldc, dtype={U.I8: torch.int8, U.I16: torch.int16,
                                          U.I32: torch.int32}[out], device="cuda")
        U.gemm(U.I8, out, torch.from_numpy(a).cuda(), (m, k, k, 1), torch.from_numpy(b).cuda(),
               (k, n, n, 1), dev, (m, n, ldc, 1), alpha, 0, mode)
        assert np.array_equal(dev.cpu().numpy().reshape(m, ldc)[:, :n].reshape(-1), want), mode
        outs[mode] = got.tobytes()
    assert outs[U.NEAREST] == outs[U.SATURATING]  # Nearest saturates integer outputs
    assert outs[U.WRAPPING] != outs[U.SATURATING]  # the wrap differs once cells overflow
