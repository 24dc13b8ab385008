"""CPU oracle for uor-matmul's exact-GEMM semantics -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs may
import this module, and only as the checker. The product (the CUDA library under
``uor-matmul_b200/``) never imports, links or calls anything here.

Two independent restatements of the reference (UOR-Foundation/uor-matmul):

* ``liboracle.so`` (``uor_oracle.c``): the C restatement, fast enough for the
  CPU baseline and for parity checks at test sizes.
* pure-Python twins below: big-integer float GEMM, tropical GEMM, integer GEMM,
  view placement (``layout.rs:54-199``) and the alias test (``layout.rs:116``),
  used to cross-check the C restatement on small cases.

Parity pins (tests/test_oracle_golden.py): the reference's committed NumPy golden
vectors CX-10 (``oracles/numpy``, int64 wrapping matmul) and CX-11
(``oracles/tropical``, max-plus), identified by the SHA-256 digests recorded in
``tests/golden/cx_manifest.json``, plus the reference's unit-test KATs.
"""
from __future__ import annotations

import ctypes
import os
import struct
import subprocess
from fractions import Fraction

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

NEAREST, TOWARD_ZERO, SATURATING, WRAPPING = 0, 1, 2, 3

# Trop<E> is repr(C) {E value; bool finite} (tropical.rs:61-70).
TROP_DTYPES = {
    8: np.dtype([("v", "i1"), ("f", "u1")]),
    16: np.dtype([("v", "<i2"), ("f", "u1"), ("pad", "u1")]),
    32: np.dtype([("v", "<i4"), ("f", "u1"), ("pad", "3u1")]),
    64: np.dtype([("v", "<i8"), ("f", "u1"), ("pad", "7u1")]),
}

INT_DTYPES = {8: np.int8, 16: np.int16, 32: np.int32, 64: np.int64}


def lib():
    """Load (building on first use) the C restatement."""
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            subprocess.check_call(["make", "-s", "-C", HERE])
        _LIB = ctypes.CDLL(path)
        P, Z, D, I, L = (ctypes.c_void_p, ctypes.c_size_t, ctypes.c_ssize_t, ctypes.c_int,
                         ctypes.c_int64)
        _LIB.uor_oracle_gemm_int.argtypes = [I, I, Z, Z, Z, L, P, D, D, P, D, D, L, P, D, D, I, I]
        _LIB.uor_oracle_gemm_float.argtypes = [I, I, Z, Z, Z, L, P, D, D, P, D, D, L, P, D, D, I, I]
        _LIB.uor_oracle_gemm_trop.argtypes = [I, I, Z, Z, Z, L, I, P, D, D, P, D, D, L, I, P, D, D,
                                              I, I]
        _LIB.uor_oracle_coded_gemm.argtypes = [I, Z, Z, Z, L, P, D, D, P, I, P, Z, I, L, P, D, D,
                                               I, I]
        _LIB.uor_oracle_gemm_complex.argtypes = [I, I, Z, Z, Z, L, P, D, D, P, D, D, L, P, D, D,
                                                 I, I]
        _LIB.uor_oracle_max_threads.restype = I
        _LIB.uor_oracle_gemm_i8_blocked.argtypes = [Z, Z, Z, L, P, P, L, P, Z, I, I]
        _LIB.uor_oracle_corpus_i8.argtypes = [ctypes.c_uint64, Z, P]
    return _LIB


def max_threads() -> int:
    return lib().uor_oracle_max_threads()


class View:
    """An origin view: ``arr`` holds the buffer, ``origin`` indexes element (0,0).

    ``rs``/``cs`` are signed element strides, as ``Strides`` (layout.rs:29).
    """

    def __init__(self, arr, rows, cols, rs, cs, origin=0):
        self.arr, self.rows, self.cols = arr, rows, cols
        self.rs, self.cs, self.origin = rs, cs, origin

    @classmethod
    def row_major(cls, arr, rows, cols, ld=None):
        return cls(arr, rows, cols, cols if ld is None else ld, 1, 0)

    def ptr(self):
        return self.arr.ctypes.data + self.origin * self.arr.itemsize

    def at(self, i, j):
        return self.arr.reshape(-1)[self.origin + i * self.rs + j * self.cs]


def _bits_of(dtype) -> int:
    return np.dtype(dtype).itemsize * 8


# --------------------------------------------------------------------------
# ctypes wrappers around the C restatement
# --------------------------------------------------------------------------

def gemm_int(a: View, b: View, c: View, alpha=1, beta=0, mode=NEAREST, threads=0,
             out_bits=None):
    """``C := encode(alpha A B + beta C)`` for i8/i16/i32/i64 elements."""
    ebits = _bits_of(a.arr.dtype)
    obits = out_bits or _bits_of(c.arr.dtype)
    lib().uor_oracle_gemm_int(ebits, obits, a.rows, a.cols, b.cols, alpha, a.ptr(), a.rs, a.cs,
                              b.ptr(), b.rs, b.cs, beta, c.ptr(), c.rs, c.cs, mode, threads)


def gemm_complex(a: View, b: View, c: View, alpha=1, beta=0, mode=NEAREST, threads=0,
                 out_bits=None):
    """Complex<i32|i64> GEMM (alphabet.rs:656-776) with the per-part epilogue.

    Each view's ``arr`` holds the interleaved parts (re, im); ``rows``, ``cols``,
    strides and ``origin`` count whole complex elements."""
    ebits = _bits_of(a.arr.dtype)
    obits = out_bits or _bits_of(c.arr.dtype)

    def ptr(v, bits):
        return v.arr.ctypes.data + 2 * v.origin * (bits // 8)

    lib().uor_oracle_gemm_complex(ebits, obits, a.rows, a.cols, b.cols, alpha, ptr(a, ebits),
                                  a.rs, a.cs, ptr(b, ebits), b.rs, b.cs, beta, ptr(c, obits), c.rs,
                                  c.cs, mode, threads)


def gemm_i8_blocked(a, b, c, m, k, n, alpha=1, beta=0, ldc=None, mode=NEAREST, threads=0):
    """The blocked s8 restatement (contiguous row-major operands), for CPU timing."""
    lib().uor_oracle_gemm_i8_blocked(m, k, n, alpha, a.ctypes.data, b.ctypes.data, beta,
                                     c.ctypes.data, n if ldc is None else ldc, mode, threads)


def gemm_float(a: View, b: View, c: View, alpha=1, beta=0, mode=NEAREST, threads=0):
    """``C := encode(alpha exact(A B) + beta C)`` for f32/f64 (gemm_float semantics)."""
    e64 = 1 if a.arr.dtype == np.float64 else 0
    o64 = 1 if c.arr.dtype == np.float64 else 0
    lib().uor_oracle_gemm_float(e64, o64, a.rows, a.cols, b.cols, alpha, a.ptr(), a.rs, a.cs,
                                b.ptr(), b.rs, b.cs, beta, c.ptr(), c.rs, c.cs, mode, threads)


def gemm_trop(a: View, b: View, c: View, ebits=8, obits=32, alpha=(0, True),
              beta=(0, False), mode=NEAREST, threads=0):
    """Max-plus GEMM over Trop<E> with the MaxPlus epilogue."""
    lib().uor_oracle_gemm_trop(ebits, obits, a.rows, a.cols, b.cols, alpha[0], int(alpha[1]),
                               a.ptr(), a.rs, a.cs, b.ptr(), b.rs, b.cs, beta[0], int(beta[1]),
                               c.ptr(), c.rs, c.cs, mode, threads)


def coded_gemm(a: View, codes: np.ndarray, P: int, table: np.ndarray, c: View, k: int, n: int,
               orientation=0, alpha=1, beta=0, mode=NEAREST, threads=0):
    """coded_gemm (orientation 0, codes k x n) / gemm_tabulated (1, codes n x k)."""
    obits = _bits_of(c.arr.dtype)
    lib().uor_oracle_coded_gemm(obits, a.rows, k, n, alpha, a.ptr(), a.rs, a.cs,
                                codes.ctypes.data, P, table.ctypes.data, len(table), orientation,
                                beta, c.ptr(), c.rs, c.cs, mode, threads)


def decode_codec(tier, codes, rows, cols, table=None, per_byte=0, block=1, code_bytes=1, zero=0):
    """The dense rows x cols int8 matrix a fixed-width coded matrix names.

    CodedMatrix::at (crates/uor-matmul-codec/src/matrix.rs:202-207): code q of row r
    holds elements q*BLK .. q*BLK+BLK-1. Tiers (codecs.rs): Packed<Grid<N>,P> (tier 0,
    :181-195: sub-code c % P of byte c / P, low first, table[sub % N]); Sign (1,
    :386-400: bit t set +1, else -1); Ternary (2, :480-496: digit t 0 -> -1, 2 -> +1,
    else 0, a digit past the code's width reads 0); Book (3, :306-308:
    table[code % N][t]). Offset (zero): every value minus zero."""
    codes = np.asarray(codes, np.uint8)
    out = np.zeros((rows, cols), np.int64)
    if tier == 0:
        bits = 8 // per_byte
        mask = 0xFF if bits >= 8 else (1 << bits) - 1
        tab = np.asarray(table, np.int64)
        cpr = cols // per_byte
        for r in range(rows):
            for c in range(cols):
                sub = (int(codes[r * cpr + c // per_byte]) >> (bits * (c % per_byte))) & mask
                out[r, c] = tab[sub % len(tab)]
    else:
        cpr = cols // block
        for r in range(rows):
            for c in range(cols):
                at = (r * cpr + c // block) * code_bytes
                code = int(codes[at]) | (int(codes[at + 1]) << 8 if code_bytes == 2 else 0)
                t = c % block
                if tier == 1:
                    out[r, c] = 1 if t < 8 * code_bytes and (code >> t) & 1 else -1
                elif tier == 2:
                    d = (code >> (2 * t)) & 3 if 2 * t < 8 * code_bytes else 0
                    out[r, c] = -1 if d == 0 else (1 if d == 2 else 0)
                else:
                    tab = np.asarray(table, np.int64).reshape(-1, block)
                    out[r, c] = tab[code % tab.shape[0], t]
    return (out - zero).astype(np.int8)


def decode_codec_np(tier, codes, rows, cols, table=None, block=1, code_bytes=1, zero=0):
    """decode_codec's fixed-width tiers (Sign, Ternary, Book, Offset) as whole-array numpy
    steps, for full-size cases: the same CodedMatrix::at indexing and per-tier rules
    (matrix.rs:202-207, codecs.rs:306-308, :386-400, :480-496), checked against the
    element loops above on the CPU."""
    codes = np.asarray(codes, np.uint8)
    cpr = cols // block
    raw = codes[: rows * cpr * code_bytes].reshape(rows, cpr, code_bytes).astype(np.int64)
    code = raw[..., 0] | (raw[..., 1] << 8) if code_bytes == 2 else raw[..., 0]
    t = np.arange(block, dtype=np.int64)
    width = 8 * code_bytes
    if tier == 1:
        bit = (code[..., None] >> np.minimum(t, 63)) & 1
        out = np.where((t < width) & (bit == 1), 1, -1)
    elif tier == 2:
        d = np.where(2 * t < width, (code[..., None] >> np.minimum(2 * t, 63)) & 3, 0)
        out = np.where(d == 0, -1, np.where(d == 2, 1, 0))
    elif tier == 3:
        tab = np.asarray(table, np.int64).reshape(-1, block)
        out = tab[code % tab.shape[0]]
    else:
        raise ValueError("decode_codec_np covers tiers 1-3")
    return (out.reshape(rows, cols) - zero).astype(np.int8)


def decode_arena(table, codes, rows, cols, code_bytes=1):
    """Arena::decode_element (codecs.rs:961-965) over a CodedMatrix of one-element blocks:
    element (r, c) is table[code % N] with code the (r * cols + c)-th u8 or little-endian
    u16 code; the symbols are copied as bit patterns."""
    codes = np.asarray(codes, np.uint8)
    if code_bytes == 2:
        idx = codes[0::2].astype(np.int64) | (codes[1::2].astype(np.int64) << 8)
    else:
        idx = codes.astype(np.int64)
    return np.asarray(table)[idx[: rows * cols] % len(table)].reshape(rows, cols)


def trop_witness(av, af, bv, bf):
    """D-6's witness (crates/uor-matmul-gemm/src/selection.rs; the differential reference of
    validate/tests/selection.rs): per cell the least index attaining the maximum of the
    finite terms a_ip + b_pj, and 0 when no term is finite (or k is 0). av/af are the
    m x k values and finite flags of A, bv/bf the k x n ones of B."""
    m, k = av.shape
    n = bv.shape[1]
    w = np.zeros((m, n), np.uint64)
    if k == 0:
        return w
    big = np.int64(-(1 << 62))
    for i in range(m):
        terms = np.where(af[i][:, None] & bf, av[i].astype(np.int64)[:, None] + bv.astype(np.int64),
                         big)  # k x n
        w[i] = np.argmax(terms, axis=0)  # the first maximum: the least index
    return w


# --------------------------------------------------------------------------
# Pure-Python restatements (small cases only)
# --------------------------------------------------------------------------

def extent(rows, cols, rs, cs, isize_bits=64):
    """Strides::extent (layout.rs:71-102): lowest and highest reach, or None."""
    if rows == 0 or cols == 0:
        return (0, 0)
    lim = 1 << (isize_bits - 1)
    r = (rows - 1) * rs
    c = (cols - 1) * cs
    if not (-lim <= r < lim and -lim <= c < lim):
        return None
    r_lo, r_hi = (r, 0) if rs < 0 else (0, r)
    c_lo, c_hi = (c, 0) if cs < 0 else (0, c)
    lo, hi = r_lo + c_lo, r_hi + c_hi
    if not (-lim <= lo < lim and -lim <= hi < lim):
        return None
    return (lo, hi)


def place(length, rows, cols, rs, cs):
    """``place`` (layout.rs:178-199): origin index of a view inside ``length``."""
    if rows == 0 or cols == 0:
        return 0
    e = extent(rows, cols, rs, cs)
    if e is None:
        return None
    lo, hi = e
    if lo > 0:
        return None
    origin = -lo
    top = origin + abs(hi)
    if top >= (1 << 64):
        return None
    return origin if top < length else None


def self_aliases(rows, cols, rs, cs):
    """Strides::self_aliases (layout.rs:116-140): exact collision test by gcd."""
    from math import gcd
    if rows == 0 or cols == 0:
        return False
    if rows <= 1 and cols <= 1:
        return False
    if rows > 1 and rs == 0:
        return True
    if cols > 1 and cs == 0:
        return True
    if rows <= 1 or cols <= 1:
        return False
    a, b = abs(rs), abs(cs)
    g = gcd(a, b)
    return (b // g) < rows and (a // g) < cols


def int_gemm_py(A, B, alpha=1, beta=0, C=None, out_bits=32, mode=NEAREST):
    """Pure-Python integer Linear GEMM on nested lists (i8..i32 elements)."""
    mn, mx = -(1 << (out_bits - 1)), (1 << (out_bits - 1)) - 1
    lo128, hi128 = -(1 << 127), (1 << 127) - 1

    def sat(v):
        return max(lo128, min(hi128, v))

    def wrap128(v):
        v &= (1 << 128) - 1
        return v - (1 << 128) if v >> 127 else v

    m, k, n = len(A), len(B), len(B[0]) if B else 0
    out = []
    for i in range(m):
        row = []
        for j in range(n):
            acc = sum(int(A[i][p]) * int(B[p][j]) for p in range(k))
            tot = sat(acc * alpha)
            if beta != 0:
                tot = wrap128(tot + sat(int(C[i][j]) * beta))
            if mode == WRAPPING:
                span = mx - mn + 1
                tot = (tot - mn) % span + mn
            else:
                tot = max(mn, min(mx, tot))
            row.append(tot)
        out.append(row)
    return out


def complex_gemm_py(A, B, ebits=32, alpha=1, beta=0, C=None, out_bits=32, mode=NEAREST):
    """Pure-Python twin of gemm_complex on nested lists of (re, im) pairs.

    mac: re += a.re w.re + a.im (-w.im), im += a.re w.im + a.im w.re
    (alphabet.rs:712-717), -w.im wrapping in ebits (the release build's negation)."""
    half = 1 << (ebits - 1)

    def wrapneg(v):
        v = (-v) & ((1 << ebits) - 1)
        return v - (1 << ebits) if v >= half else v

    m, k, n = len(A), len(B), len(B[0]) if B else 0
    re = [[sum(A[i][p][0] * B[p][j][0] + A[i][p][1] * wrapneg(B[p][j][1]) for p in range(k))
           for j in range(n)] for i in range(m)]
    im = [[sum(A[i][p][0] * B[p][j][1] + A[i][p][1] * B[p][j][0] for p in range(k))
           for j in range(n)] for i in range(m)]
    acc_bits = 192 if ebits == 64 else 128
    lo, hi = -(1 << (acc_bits - 1)), (1 << (acc_bits - 1)) - 1
    mn, mx = -(1 << (out_bits - 1)), (1 << (out_bits - 1)) - 1

    def wrap(v, bits):
        v &= (1 << bits) - 1
        return v - (1 << bits) if v >> (bits - 1) else v

    def part(acc, prior):
        # ScaleExact: saturating for i128 (epilogue.rs:280-288), modular for Limbs<3>.
        tot = wrap(acc * alpha, 192) if ebits == 64 else max(lo, min(hi, acc * alpha))
        if beta != 0:
            pr = wrap(prior * beta, 192) if ebits == 64 else max(lo, min(hi, prior * beta))
            tot = wrap(tot + pr, acc_bits)
        if mode == WRAPPING:
            return wrap(tot, out_bits)
        return max(mn, min(mx, tot))

    return [[(part(re[i][j], C[i][j][0] if C else 0), part(im[i][j], C[i][j][1] if C else 0))
             for j in range(n)] for i in range(m)]


# ---- float twin: exact rationals, one RNE encode (acc.rs:1734-1868) ------

def _decode(x: float, is64: bool):
    """FloatElement::decode (alphabet.rs:905-946) -> ('nan'|'inf'|'fin', sign, mant, exp)."""
    if is64:
        bits = struct.unpack("<Q", struct.pack("<d", x))[0]
        mant_bits, exp_bits, bias = 52, 11, 1023
    else:
        bits = struct.unpack("<I", struct.pack("<f", x))[0]
        mant_bits, exp_bits, bias = 23, 8, 127
    frac = bits & ((1 << mant_bits) - 1)
    biased = (bits >> mant_bits) & ((1 << exp_bits) - 1)
    sign = bits >> (mant_bits + exp_bits)
    if biased == (1 << exp_bits) - 1:
        return ("nan" if frac else "inf", sign, 0, 0)
    if biased == 0:
        return ("fin", sign, frac, 1 - bias - mant_bits)
    return ("fin", sign, frac | (1 << mant_bits), biased - bias - mant_bits)


class _Complete:
    """Exact value (an int at scale 2^min_exp) plus the three flags."""

    def __init__(self, min_exp):
        self.min_exp, self.v = min_exp, 0
        self.limbs = 67 if min_exp == -2148 else 10  # low limbs of Complete<L, MIN_EXP>
        self.nan = self.pinf = self.ninf = False

    def is_nan(self):
        return self.nan or (self.pinf and self.ninf)

    def finite(self):
        return not (self.nan or self.pinf or self.ninf)

    def add(self, sign, mag, exp):
        """Complete::add_scaled (acc.rs:939-998): a coordinate below bit 0 or past the
        last low limb is dropped whole; the register is wide enough for the rest."""
        sh = exp - self.min_exp
        if sh < 0 or mag == 0 or sh // 64 >= self.limbs:
            return
        self.v += (-1 if sign else 1) * (mag << sh)

    def mac(self, da, db):
        if da[0] == "nan" or db[0] == "nan":
            self.nan = True
            return
        if da[0] == "inf" or db[0] == "inf":
            inf, other = (da, db) if da[0] == "inf" else (db, da)
            if other[0] == "fin" and other[2] == 0:
                self.nan = True
            elif inf[1] != other[1]:
                self.ninf = True
            else:
                self.pinf = True
            return
        self.add(da[1] ^ db[1], da[2] * db[2], da[3] + db[3])

    def scale(self, f):
        if self.is_nan() or f == 1:
            return
        if f == 0:
            inf = self.pinf or self.ninf
            self.v = 0
            if inf:
                self.nan, self.pinf, self.ninf = True, False, False
            return
        if not self.finite():
            if f < 0:
                self.pinf, self.ninf = self.ninf, self.pinf
            return
        self.v *= f


def _encode(acc: _Complete, out64: bool, mode: int) -> int:
    MANT, EXPO = (52, 11) if out64 else (23, 8)
    P = MANT + 1
    BIAS = (1 << (EXPO - 1)) - 1
    SUB = 1 - BIAS - MANT
    sign_bit = 1 << (MANT + EXPO)
    exp_all = (1 << EXPO) - 1
    if acc.is_nan():
        return 0x7FF8000000000000 if out64 else 0x7FC00000
    if acc.pinf or acc.ninf:
        return (sign_bit if acc.ninf else 0) | (exp_all << MANT)
    neg = acc.v < 0
    mag = -acc.v if neg else acc.v
    if mag == 0:
        return 0
    high = mag.bit_length() - 1
    e = acc.min_exp + high
    lsb_exp = max(e - (P - 1), SUB)
    lsb = lsb_exp - acc.min_exp
    if lsb < 0:
        return 0
    sig = (mag >> lsb) & ((1 << P) - 1)
    rb = (mag >> (lsb - 1)) & 1 if lsb > 0 else 0
    sticky = (mag & ((1 << (lsb - 1)) - 1)) != 0 if lsb > 1 else False
    inc = 1 if (mode == NEAREST and rb and (sticky or (sig & 1))) else 0
    sig += inc
    if sig >> P:
        sig >>= 1
        lsb_exp += 1
    if sig == 0:
        return sign_bit if neg else 0
    top = sig.bit_length() - 1
    vexp = lsb_exp + top
    s = sign_bit if neg else 0
    if sig >> (P - 1) == 1:
        biased = vexp + BIAS
        if biased >= exp_all:
            if mode == NEAREST:
                return s | (exp_all << MANT)
            return s | ((exp_all - 1) << MANT) | ((1 << MANT) - 1)
        return s | (biased << MANT) | (sig & ((1 << MANT) - 1))
    return s | sig


def float_gemm_py(A, B, alpha=1, beta=0, C=None, e64=False, o64=False, mode=NEAREST):
    """Big-integer twin of gemm_float: returns raw output bits per cell."""
    min_exp = -2148 if e64 else -298
    m, k = len(A), len(A[0]) if A else 0
    n = len(B[0]) if B else 0
    out = []
    for i in range(m):
        row = []
        for j in range(n):
            acc = _Complete(min_exp)
            for p in range(k):
                acc.mac(_decode(A[i][p], e64), _decode(B[p][j], e64))
            acc.scale(alpha)
            if beta != 0:
                pr = _Complete(min_exp)
                d = _decode(C[i][j], o64)
                if d[0] == "nan":
                    pr.nan = True
                elif d[0] == "inf":
                    pr.ninf, pr.pinf = bool(d[1]), not d[1]
                else:
                    pr.add(d[1], d[2], d[3])
                pr.scale(beta)
                if acc.finite() and pr.finite():
                    acc.v += pr.v
                else:
                    acc.nan |= pr.nan
                    acc.pinf |= pr.pinf
                    acc.ninf |= pr.ninf
            row.append(_encode(acc, o64, mode))
        out.append(row)
    return out


def exact_value(A, B, i, j, e64=False):
    """The exact rational value of cell (i, j) of A B (finite inputs)."""
    tot = Fraction(0)
    for p in range(len(B)):
        tot += Fraction(A[i][p]) * Fraction(B[p][j])
    return tot


# ---- reference generators --------------------------------------------------

MASK64 = (1 << 64) - 1


def xorshift_stream(state: int, count: int):
    """xorshift64 (s ^= s<<13; s ^= s>>7; s ^= s<<17), yielding the state."""
    out = np.empty(count, dtype=np.uint64)
    s = state & MASK64
    for idx in range(count):
        s ^= (s << 13) & MASK64
        s ^= s >> 7
        s ^= (s << 17) & MASK64
        out[idx] = s
    return out, s


def corpus_fill(salt: int, count: int) -> np.ndarray:
    """The validate harness fill (validate/tests/common/mod.rs:9-19): ``s >> 33``."""
    states, _ = xorshift_stream(0x243F6A8885A308D3 ^ salt, count)
    return states >> np.uint64(33)


def corpus_i8(salt: int, count: int) -> np.ndarray:
    """``corpus_fill(salt, count)`` cast to i8, from the C restatement (fast enough for
    the 8192^3 operands the CPU baseline draws)."""
    out = np.empty(count, dtype=np.int8)
    lib().uor_oracle_corpus_i8(salt, count, out.ctypes.data)
    return out
