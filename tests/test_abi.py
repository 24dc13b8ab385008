"""CPU-side checks of the C ABI: the library loads, exports every declared
symbol, and performs the reference's host-side validation (MatView::new,
Triple::new) before touching a device. No compute call runs here."""
import ctypes
import os
import re

import numpy as np
import pytest

import uor_b200 as U
from oracle import oracle as orc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        if h.endswith(".h"):
            src = open(os.path.join(ROOT, "include", h)).read()
            names |= set(re.findall(r"\b(uor_b200_[a-z0-9_]+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol():
    exported = set(U.exported_symbols())
    declared = declared_symbols()
    assert declared, "the headers declare entry points"
    missing = declared - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_version_and_status_strings():
    assert U.lib().uor_b200_version() >= 100
    assert "nonconformant" in U.status_string(U.NONCONFORMANT)
    assert "aliases" in U.status_string(U.OUTPUT_ALIASES)


def test_corpus_matches_reference_generator():
    # validate/tests/common/mod.rs:9-19, restated independently in oracle.corpus_fill
    raw = U.corpus(1, U.CORPUS_RAW, 1000)
    assert np.array_equal(raw, orc.corpus_fill(1, 1000))
    i8 = U.corpus(2, U.CORPUS_I8, 1000)
    assert np.array_equal(i8, orc.corpus_fill(2, 1000).astype(np.uint8).view(np.int8))
    nib = U.corpus(3, U.CORPUS_NIBBLES, 1001)
    v = orc.corpus_fill(3, 1001) & np.uint64(0xF)
    assert nib[0] == (v[0] | (v[1] << np.uint64(4)))
    assert nib[-1] == v[-1]


def _gemm_status(m, k, n, a_len, b_len, c_len, rsa, csa, rsb, csb, rsc, csc, am=None, bk=None,
                 cn=None):
    a = np.zeros(max(a_len, 1), np.int8)
    b = np.zeros(max(b_len, 1), np.int8)
    c = np.zeros(max(c_len, 1), np.int32)
    A = U.View(a.ctypes.data, a_len, m if am is None else am, k, rsa, csa)
    B = U.View(b.ctypes.data, b_len, k if bk is None else bk, n, rsb, csb)
    C = U.View(c.ctypes.data, c_len, m, n if cn is None else cn, rsc, csc)
    call = U.make_call()
    import ctypes
    return U.lib().uor_b200_gemm(U.I8, U.I32, ctypes.byref(A), ctypes.byref(B), ctypes.byref(C),
                                 1, 0, ctypes.byref(call))


def test_nonconformant_is_reported_before_any_device_work():
    assert _gemm_status(2, 3, 4, 6, 12, 8, 3, 1, 4, 1, 4, 1, bk=2) == U.NONCONFORMANT
    assert _gemm_status(2, 3, 4, 6, 12, 8, 3, 1, 4, 1, 4, 1, cn=3) == U.NONCONFORMANT


def test_short_buffer_does_not_fit():
    assert _gemm_status(2, 3, 4, 5, 12, 8, 3, 1, 4, 1, 4, 1) == U.DOES_NOT_FIT
    assert _gemm_status(2, 3, 4, 6, 12, 7, 3, 1, 4, 1, 4, 1) == U.DOES_NOT_FIT


def test_empty_products_need_no_device():
    assert _gemm_status(0, 3, 4, 0, 12, 0, 3, 1, 4, 1, 4, 1) == U.OK
    assert _gemm_status(2, 3, 0, 6, 0, 0, 3, 1, 0, 1, 0, 1) == U.OK


def test_unsupported_pairs_are_refused():
    import ctypes
    a = np.zeros(4, np.int8)
    v = U.View(a.ctypes.data, 4, 2, 2, 2, 1)
    call = U.make_call()
    # f32 output from an integer element is outside the reference's surface
    assert U.lib().uor_b200_gemm(U.I8, U.F32, ctypes.byref(v), ctypes.byref(v), ctypes.byref(v),
                                 1, 0, ctypes.byref(call)) == U.UNSUPPORTED


@pytest.mark.parametrize("seed", range(20))
def test_alias_and_placement_agree_with_the_reference_rules(seed):
    """Strides::self_aliases and place (layout.rs:116, 178), restated in the oracle,
    against the library: an aliasing output is refused; a placeable, non-aliasing
    one gets past validation (and then needs a device, which CPU runs lack)."""
    rng = np.random.default_rng(seed)
    for _ in range(40):
        m, n = (int(x) for x in rng.integers(0, 6, size=2))
        rsc, csc = (int(x) for x in rng.integers(-7, 8, size=2))
        lo_hi = orc.extent(m, n, rsc, csc)
        span = 0 if lo_hi is None else lo_hi[1] - lo_hi[0] + 1
        c_len = span + int(rng.integers(0, 2))
        st = _gemm_status(m, 1, n, m, n, c_len, 1, 1, n, 1, rsc, csc)
        placed = orc.place(c_len, m, n, rsc, csc) is not None
        if not placed:
            assert st == U.DOES_NOT_FIT, (m, n, rsc, csc, c_len)
        elif orc.self_aliases(m, n, rsc, csc):
            assert st == U.OUTPUT_ALIASES, (m, n, rsc, csc)
        elif m == 0 or n == 0:
            assert st == U.OK
        else:
            assert st in (U.OK, U.DEVICE_ERROR), (m, n, rsc, csc, st)


def test_e8_table_is_the_reference_codebook():
    """uor_b200_e8_table derives the E8 codebook (e8.rs) on the host; its bytes match
    the digest of the reference's literal table, and it has the lattice property
    e8_is_the_lattice_it_claims checks (e8.rs:335-365)."""
    import hashlib
    import json
    rec = json.load(open(os.path.join(ROOT, "tests", "golden", "e8_digest.json")))
    t = U.e8_table()
    assert t.shape == (256, 8)
    assert hashlib.sha256(t.tobytes()).hexdigest() == rec["sha256"]
    assert not t[0].any()
    for w in t[1:].astype(int):
        all32 = all(v % 32 == 0 for v in w)
        all16 = all(v % 32 == 16 for v in w)
        assert all32 or all16
        if all32:
            assert (w // 32).sum() % 2 == 0
    assert len({bytes(r) for r in t.view(np.uint8)}) == 256


def test_e8_table_bound_and_length():
    """a_bound_too_narrow_has_no_table (e8.rs:369-374): Bnd<8> has no table."""
    assert U.e8_table(128).tobytes() == U.e8_table().tobytes()
    assert U.e8_table(32).tobytes() == U.e8_table().tobytes()
    with pytest.raises(U.UorError):
        U.e8_table(8)
    short = np.zeros(2047, np.int8)
    assert U.lib().uor_b200_e8_table(0, short.ctypes.data, short.size) == U.DOES_NOT_FIT


def test_noalloc_refuses_oversized_products_before_any_device_work():
    """The no-allocation entry compares chunks x m x n partials against its fixed array
    without forming the product (which can wrap size_t for sizes near its INT_MAX / 2
    cap); such calls return UOR_B200_SCRATCH_LIMIT before any CUDA call, so this runs
    without a GPU. The pointers are never read."""
    import ctypes
    fn = U.lib().uor_b200_gemm_ex_i8_noalloc
    fn.argtypes = [ctypes.c_int, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                   ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                   ctypes.c_size_t, ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t,
                   ctypes.c_uint32, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    fake = 1 << 20  # 16-byte aligned, non-null, never dereferenced
    cap = (2**31 - 1) // 2
    for m, k, n in [(cap, cap, cap), (2**29, 2**28, 2**29), (2**20, 140_000, 2**20),
                    (1, cap, 2**22), (2048, 140_000, 1024)]:
        st = fn(U.I64, m, k, n, 1, fake, k, fake, n, 0, fake, n, U.NEAREST, None)
        assert st == 9, (m, k, n, st)  # UOR_B200_SCRATCH_LIMIT
    # past the int-sized cap is unsupported, still before any device work
    assert fn(U.I64, cap + 1, 140_000, 4, 1, fake, 140_000, fake, 4, 0, fake, 4, U.NEAREST,
              None) == U.UNSUPPORTED


def test_reference_arm_runs_without_the_product_library():
    """bench.py --impl reference times the reference semantics through the oracle alone:
    the process must never load libuor_b200.so (the comparison would not be against the
    reference otherwise), and it prints the GPU arm's config."""
    import json
    import subprocess
    import sys
    code = ("import runpy, sys; sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', "
            "'--warmup', '0', '--size', '512']; runpy.run_path('bench.py', run_name='__main__'); "
            "maps = open('/proc/self/maps').read(); "
            "print('LOADED' if 'libuor_b200' in maps else 'CLEAN')")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = out.stdout.strip().splitlines()
    assert lines[-1] == "CLEAN"
    line = json.loads(lines[-2])
    assert line["impl"] == "reference" and line["config"]["m"] == 512
    assert line["cpu_baseline"]["kind"] == "port"


def test_nccl_entries_validate_before_loading_nccl():
    """The collective entries refuse a missing communicator, host pointers and a bad
    rank before they load NCCL or touch a device."""
    lib = U.lib()
    A = U.View(0, 0, 0, 0, 0, 1)
    C = U.View(0, 0, 0, 0, 0, 1)
    call = U.make_call(U.NEAREST, True, None, None, False)
    for fn in (lib.uor_b200_gemm_splitk_nccl,):
        assert fn(None, U.I8, U.I32, ctypes.byref(A), ctypes.byref(A), ctypes.byref(C), 1, 0,
                  ctypes.byref(call)) == U.INVALID_ARGUMENT
    host = U.make_call(U.NEAREST, False, None, None, False)
    assert lib.uor_b200_gemm_tropical_splitk_nccl(
        1, U.TROP_I8, U.TROP_I32, ctypes.byref(A), ctypes.byref(A), ctypes.byref(C),
        U.Trop(0, 1), U.Trop(0, 0), ctypes.byref(host)) == U.INVALID_ARGUMENT
    out = ctypes.c_void_p()
    uid = (ctypes.c_uint8 * 128)()
    assert lib.uor_b200_nccl_comm_init(None, 2, ctypes.addressof(uid), 128, 2,
                                       ctypes.byref(out)) == U.INVALID_ARGUMENT
    assert lib.uor_b200_nccl_comm_init(None, 2, ctypes.addressof(uid), 100, 0,
                                       ctypes.byref(out)) == U.INVALID_ARGUMENT
    assert lib.uor_b200_nccl_unique_id(ctypes.addressof(uid), 64) == U.INVALID_ARGUMENT
    assert lib.uor_b200_nccl_comm_destroy(None) == U.OK


def _status(fn, *args, **kw):
    try:
        fn(*args, **kw)
    except U.UorError as e:
        return e.status
    return U.OK


def test_codec_entries_validate_before_any_device_work():
    """coded_gemm / gemm_tabulated / codec_gemm report the reference's construction
    failures from the host, before any device work: Packed::new (codecs.rs:166-172: P
    divides 8, a table with entries), CodedMatrix::new (matrix.rs:36-60: the codes describe
    exactly the declared shape), CodedTriple::new (coded.rs:48-70: conformance, then
    aliasing), Offset::new (the offset image stays i8), an unknown tier; an empty product
    returns at once."""
    m, k, n = 2, 8, 16
    a = np.zeros(m * k, np.int8)
    c = np.zeros(m * n, np.int32)
    t16 = np.arange(16, dtype=np.int8)
    q2 = np.zeros(k * n // 2, np.uint8)
    av, cv = (m, k, k, 1), (m, n, n, 1)
    cg, xg = U.coded_gemm, U.codec_gemm
    assert _status(cg, U.I32, a, av, q2, k, n, 3, t16, c, cv) == U.INVALID_ARGUMENT  # P = 3
    assert _status(cg, U.I32, a, av, q2, k, n, 2, t16[:0], c, cv) == U.INVALID_ARGUMENT
    assert _status(cg, U.I32, a, av, q2[:-1], k, n, 2, t16, c, cv) == U.DOES_NOT_FIT
    assert _status(cg, U.I32, a, av, q2[:-1], k, n, 2, t16, c, cv, tabulated=True) == U.DOES_NOT_FIT
    assert _status(cg, U.I32, a, (m, k - 1, k, 1), q2, k, n, 2, t16, c, cv) == U.NONCONFORMANT
    assert _status(cg, U.I32, a, av, q2, k, n, 2, t16, c, (m, n, 0, 0)) == U.OUTPUT_ALIASES
    assert _status(cg, U.I32, a[:0], (0, k, k, 1), q2, k, n, 2, t16, c[:0], (0, n, n, 1)) == U.OK
    q8 = np.zeros(k * n // 8, np.uint8)
    assert _status(xg, U.I32, a, av, 7, q8, k, n, c, cv, block=8) == U.UNSUPPORTED  # no tier 7
    assert _status(xg, U.I32, a, av, U.TIER_SIGN, q8, k, n, c, cv, block=8,
                   code_bytes=3) == U.INVALID_ARGUMENT
    assert _status(xg, U.I32, a, av, U.TIER_SIGN, q8[:-1], k, n, c, cv, block=8) == U.DOES_NOT_FIT
    assert _status(xg, U.I32, a, av, U.TIER_SIGN, q8, k, n, c, cv, block=8,
                   zero=128) == U.INVALID_ARGUMENT  # -1 - 128 leaves i8
    book = np.full(256 * 8, 100, np.int8)
    assert _status(xg, U.I32, a, av, U.TIER_BOOK, q8, k, n, c, cv, table=book, block=8,
                   zero=-28) == U.INVALID_ARGUMENT  # 100 + 28 leaves i8
    assert _status(xg, U.I32, a, av, U.TIER_BOOK, q8, k, n, c, cv, table=book[:0],
                   block=8) == U.INVALID_ARGUMENT  # a book with no rows
    assert _status(xg, U.I32, a, av, U.TIER_TERNARY, np.zeros(k * n // 4, np.uint8), k, n, c,
                   (m, n, 0, 0), block=4) == U.OUTPUT_ALIASES


def test_float_tropical_complex_entries_validate_before_any_device_work():
    """gemm_float, driver::gemm over Trop<E> and over Complex<T> report Triple::new's two
    failures (layout.rs:534-561), a short buffer and an unsupported pair from the host; an
    empty product returns at once (raw.rs:137-148 for sgemm)."""
    m, k, n = 2, 3, 4
    af, bf = np.zeros(m * k, np.float32), np.zeros((k + 1) * n, np.float32)
    cf = np.zeros(m * n, np.float32)
    good, wide = (k, n, n, 1), (k + 1, n, n, 1)
    g = U.gemm_float
    assert _status(g, U.F32, U.F32, af, (m, k, k, 1), bf, wide, cf, (m, n, n, 1)) == U.NONCONFORMANT
    assert _status(g, U.F32, U.F32, af, (m, k, k, 1), bf, good, cf, (m, n, 0, 0)) == U.OUTPUT_ALIASES
    assert _status(g, U.F32, U.F32, af[:-1], (m, k, k, 1), bf, good, cf, (m, n, n, 1)) == U.DOES_NOT_FIT
    assert _status(g, U.F32, U.I32, af, (m, k, k, 1), bf, good, cf, (m, n, n, 1)) == U.UNSUPPORTED
    assert _status(g, U.F32, U.F32, af[:0], (0, k, k, 1), bf, good, cf[:0], (0, n, n, 1)) == U.OK
    assert _status(U.sgemm, 0, k, n, 1, af, k, 1, bf, n, 1, 0, cf, n, 1) == U.OK
    at = np.zeros(m * k * 2, np.uint8)   # Trop<i8>: 2 bytes
    bt = np.zeros((k + 1) * n * 2, np.uint8)
    ct = np.zeros(m * n * 8, np.uint8)   # Trop<i32>: 8 bytes
    t = U.gemm_tropical
    assert _status(t, U.TROP_I8, U.TROP_I32, at, (m, k, k, 1), bt, wide, ct,
                   (m, n, n, 1)) == U.NONCONFORMANT
    assert _status(t, U.TROP_I8, U.TROP_I32, at, (m, k, k, 1), bt, good, ct,
                   (m, n, 0, 0)) == U.OUTPUT_ALIASES
    assert _status(t, U.TROP_I8, U.TROP_I32, at[:0], (0, k, k, 1), bt, good, ct[:0],
                   (0, n, n, 1)) == U.OK
    ac, bc = np.zeros(2 * m * k, np.int32), np.zeros(2 * (k + 1) * n, np.int32)
    cc = np.zeros(2 * m * n, np.int32)
    x = U.gemm_complex
    assert _status(x, U.I32, U.I32, ac, (m, k, k, 1), bc, wide, cc, (m, n, n, 1)) == U.NONCONFORMANT
    assert _status(x, U.I32, U.I32, ac, (m, k, k, 1), bc, good, cc, (m, n, 0, 0)) == U.OUTPUT_ALIASES
