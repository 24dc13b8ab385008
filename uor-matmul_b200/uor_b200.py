"""Python binding of libuor_b200.so (ctypes), mirroring uor-matmul's public surface.

The names follow the reference crate's facade (crates/uor-matmul/src/{slice,raw}.rs)
and view API (uor_matmul::gemm over a Triple). Operands are NumPy arrays (host
memory; the library stages them through device buffers) or torch CUDA tensors
(device memory, zero-copy). Both are read through the element strides given.

There is no CPU path: if the shared library is missing or no GPU is visible,
calls raise instead of computing anything on the host.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libuor_b200.so")

# enums (include/uor_b200.h)
OK, NONCONFORMANT, OUTPUT_ALIASES, DEVICE_ERROR, TIMEOUT, NCCL_ERROR, DOES_NOT_FIT, \
    INVALID_ARGUMENT, UNSUPPORTED = range(9)
NEAREST, TOWARD_ZERO, SATURATING, WRAPPING = range(4)
I8, I16, I32, I64, I128, F32, F64, TROP_I8, TROP_I16, TROP_I32, TROP_I64 = range(1, 12)
DEVICE_POINTERS, ASYNC, DIGIT_SLICES, MODULAR, CODEC_ON_CHIP = 1, 2, 4, 8, 16
KERNEL_NAMES = {0: "none", 1: "i8_tcgen05", 2: "limb_tcgen05", 3: "tropical",
                4: "coded_tcgen05", 5: "float_exact", 6: "epilogue_only", 7: "skinny_dp4a"}

DTYPE_SIZE = {I8: 1, I16: 2, I32: 4, I64: 8, I128: 16, F32: 4, F64: 8,
              TROP_I8: 2, TROP_I16: 4, TROP_I32: 8, TROP_I64: 16}


class UorError(RuntimeError):
    def __init__(self, status, what=""):
        self.status = status
        super().__init__(f"{what}: status {status} ({status_string(status)})")


class NotAProduct(UorError):
    """NotAProduct (error.rs:104-131): Nonconformant or OutputAliasesItself."""


class DoesNotFit(UorError):
    """A buffer shorter than its declared view (the slice face panics, slice.rs:104)."""


class View(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("len", ctypes.c_size_t), ("rows", ctypes.c_size_t),
                ("cols", ctypes.c_size_t), ("rs", ctypes.c_ssize_t), ("cs", ctypes.c_ssize_t)]


class Route(ctypes.Structure):
    _fields_ = [("kernel", ctypes.c_uint32), ("tile_m", ctypes.c_uint32),
                ("tile_n", ctypes.c_uint32), ("tile_k", ctypes.c_uint32),
                ("k_chunks", ctypes.c_uint32), ("a_layout", ctypes.c_uint32),
                ("b_layout", ctypes.c_uint32), ("ctas", ctypes.c_uint32),
                ("pairs", ctypes.c_uint32), ("fixups", ctypes.c_uint32),
                ("moduli", ctypes.c_uint32), ("crt", ctypes.c_uint32)]

    def as_dict(self):
        d = {f: getattr(self, f) for f, _ in self._fields_}
        d["kernel_name"] = KERNEL_NAMES.get(self.kernel, "?")
        return d


class Codec(ctypes.Structure):
    """uor_b200_codec: a fixed-width codec tier and its parameters."""
    _fields_ = [("tier", ctypes.c_uint32), ("per_byte", ctypes.c_uint32),
                ("block", ctypes.c_uint32), ("code_bytes", ctypes.c_uint32),
                ("table", ctypes.c_void_p), ("table_len", ctypes.c_size_t),
                ("zero", ctypes.c_int32)]


TIER_GRID, TIER_SIGN, TIER_TERNARY, TIER_BOOK = range(4)


class Call(ctypes.Structure):
    _fields_ = [("encode", ctypes.c_uint32), ("flags", ctypes.c_uint32),
                ("ctx", ctypes.c_void_p), ("route", ctypes.POINTER(Route))]


class Trop(ctypes.Structure):
    _fields_ = [("value", ctypes.c_int64), ("finite", ctypes.c_uint32)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise UorError(DEVICE_ERROR, f"{LIB_PATH} is not built (run __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        P, Z, D, I, L64, U32, U64 = (ctypes.c_void_p, ctypes.c_size_t, ctypes.c_ssize_t,
                                      ctypes.c_int, ctypes.c_int64, ctypes.c_uint32,
                                      ctypes.c_uint64)
        VP, CP = ctypes.POINTER(View), ctypes.POINTER(Call)
        sig = {
            "uor_b200_ctx_create": ([I], P),
            "uor_b200_ctx_destroy": ([P], None),
            "uor_b200_ctx_set_stream": ([P, P], I),
            "uor_b200_ctx_set_wait_budget_ns": ([P, U64], I),
            "uor_b200_ctx_sync": ([P], I),
            "uor_b200_gemm": ([I, I, VP, VP, VP, L64, L64, CP], I),
            "uor_b200_slice_gemm_ex": ([I, I, Z, Z, Z, L64, P, Z, Z, P, Z, Z, L64, P, Z, Z, P, Z,
                                        CP], I),
            "uor_b200_slice_gemm": ([I, I, Z, Z, Z, P, Z, P, Z, P, Z, P, Z, CP], I),
            "uor_b200_slice_gemm_ex_full": ([I, I, Z, Z, Z, L64, P, Z, Z, P, Z, Z, L64, P, Z, Z,
                                             P, Z, P, Z, CP], I),
            "uor_b200_gemm_i8_i32": ([Z, Z, Z, P, P, P, CP], I),
            "uor_b200_gemm_ex_i8_i32": ([Z, Z, Z, L64, P, Z, P, Z, L64, P, Z, CP], I),
            "uor_b200_gemm_float": ([I, I, VP, VP, VP, L64, L64, CP], I),
            "uor_b200_slice_gemm_float_ex": ([I, I, Z, Z, Z, L64, P, Z, Z, P, Z, Z, L64, P, Z, Z,
                                              P, Z, P, Z, CP], I),
            "uor_b200_sgemm": ([Z, Z, Z, L64, P, D, D, P, D, D, L64, P, D, D, CP], I),
            "uor_b200_dgemm": ([Z, Z, Z, L64, P, D, D, P, D, D, L64, P, D, D, CP], I),
            "uor_b200_gemm_tropical": ([I, I, VP, VP, VP, Trop, Trop, CP], I),
            "uor_b200_gemm_tropical_selected": ([I, I, VP, VP, VP, VP, Trop, Trop, CP], I),
            "uor_b200_coded_gemm": ([I, VP, P, Z, Z, Z, U32, P, Z, VP, L64, L64, CP], I),
            "uor_b200_tabulated_gemm": ([I, VP, P, Z, Z, Z, U32, P, Z, VP, L64, L64, CP], I),
            "uor_b200_codec_gemm": ([I, VP, ctypes.POINTER(Codec), P, Z, Z, Z, U32, VP, L64, L64,
                                     CP], I),
            "uor_b200_gemm_complex": ([I, I, VP, VP, VP, L64, L64, CP], I),
            "uor_b200_e8_table": ([U32, P, Z], I),
            "uor_b200_arena_gemm": ([I, I, VP, P, Z, P, Z, U32, Z, Z, U32, VP, L64, L64, CP], I),
            "uor_b200_arena_canonicalize": ([I, P, Z, ctypes.POINTER(Z)], I),
            "uor_b200_gemm_partial_limbs": ([I, VP, VP, P, Z, CP], I),
            "uor_b200_limbs_finish": ([I, I, P, Z, VP, L64, L64, CP], I),
            "uor_b200_trop_partial_keys": ([I, VP, VP, P, Z, CP], I),
            "uor_b200_trop_keys_finish": ([I, P, Z, VP, Trop, Trop, CP], I),
            "uor_b200_raw_gemm_trop_i8_i32": ([Z, Z, Z, Trop, P, D, D, P, D, D, Trop, P, D, D, CP],
                                              I),
            "uor_b200_raw_coded_grid16_i8_i32": ([Z, Z, Z, L64, P, D, D, P, P, L64, P, D, D, CP], I),
            "uor_b200_raw_tabulated_grid16_i8_i32": ([Z, Z, Z, L64, P, D, D, P, P, L64, P, D, D, CP],
                                                     I),
            "uor_b200_gemm_splitk_nccl": ([P, I, I, VP, VP, VP, L64, L64, CP], I),
            "uor_b200_gemm_tropical_splitk_nccl": ([P, I, I, VP, VP, VP, Trop, Trop, CP], I),
            "uor_b200_nccl_unique_id": ([P, Z], I),
            "uor_b200_nccl_comm_init": ([P, I, P, Z, I, ctypes.POINTER(P)], I),
            "uor_b200_nccl_comm_destroy": ([P], I),
            "uor_b200_status_string": ([I], ctypes.c_char_p),
            "uor_b200_version": ([], I),
            "uor_b200_selftest_wait_timeout": ([P, U64], I),
            "uor_b200_corpus_fill": ([U64, U32, Z, P], I),
        }
        for pair in ("i8_i32", "i8_i64", "i16_i64", "i32_i64", "i32_i128", "i64_i128"):
            sig["uor_b200_raw_gemm_" + pair] = ([Z, Z, Z, L64, P, D, D, P, D, D, L64, P, D, D, CP], I)
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def status_string(s: int) -> str:
    try:
        return lib().uor_b200_status_string(s).decode()
    except UorError:
        return "?"


def _check(status, what):
    if status == OK:
        return
    if status in (NONCONFORMANT, OUTPUT_ALIASES):
        raise NotAProduct(status, what)
    if status == DOES_NOT_FIT:
        raise DoesNotFit(status, what)
    raise UorError(status, what)


def exported_symbols():
    """Names the shared library exports (for the ABI check)."""
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    return sorted(line.split()[-1] for line in out.splitlines() if " T uor_b200" in line)


# ------------------------------------------------------------------ operands

def _is_torch(x):
    return type(x).__module__.startswith("torch")


def _buffer(x):
    """(pointer, length in elements, on_device) of a NumPy array or torch tensor.

    The pointer is the array's first element; the length counts elements of the
    underlying storage reachable from it (the whole flat array).
    """
    if _is_torch(x):
        return x.data_ptr(), x.numel(), x.is_cuda
    arr = np.asarray(x)
    return arr.ctypes.data, arr.size, False


class Context:
    """A device, a stream and device buffers (uor_b200_ctx)."""

    def __init__(self, device: int = 0):
        self.handle = lib().uor_b200_ctx_create(device)
        if not self.handle:
            raise UorError(DEVICE_ERROR, f"uor_b200_ctx_create({device})")
        self.device = device

    def set_stream(self, stream_ptr: int | None):
        _check(lib().uor_b200_ctx_set_stream(self.handle, stream_ptr), "set_stream")

    def set_wait_budget_ns(self, ns: int):
        _check(lib().uor_b200_ctx_set_wait_budget_ns(self.handle, ns), "set_wait_budget_ns")

    def sync(self):
        return lib().uor_b200_ctx_sync(self.handle)

    def close(self):
        if self.handle:
            lib().uor_b200_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def make_call(encode=NEAREST, device=False, ctx: Context | None = None, route: Route | None = None,
              asynchronous=False):
    flags = (DEVICE_POINTERS if device else 0) | (ASYNC if asynchronous else 0)
    c = Call(encode, flags, ctx.handle if ctx else None,
             ctypes.pointer(route) if route is not None else None)
    return c


def view(buf, rows, cols, rs=None, cs=1):
    """A MatView over a flat buffer (NumPy array or torch tensor)."""
    ptr, n, _ = _buffer(buf)
    return View(ptr, n, rows, cols, cols if rs is None else rs, cs)


def _on_device(*bufs):
    devs = {_buffer(b)[2] for b in bufs}
    if len(devs) != 1:
        raise ValueError("operands must all be host arrays or all be CUDA tensors")
    return devs.pop()


# ------------------------------------------------------------------ integer

def gemm(elem, out, a, av, b, bv, c, cv, alpha=1, beta=0, encode=NEAREST, ctx=None, route=None,
         asynchronous=False, digits=False, modular=False):
    """uor_matmul::gemm over views: av/bv/cv are (rows, cols, rs, cs) tuples over buffers a/b/c.
    digits=True keeps wide elements on the byte-slice route (the same bytes)."""
    dev = _on_device(a, b, c)
    A, B, C = view(a, *av), view(b, *bv), view(c, *cv)
    call = make_call(encode, dev, ctx, route, asynchronous)
    if digits:
        call.flags |= DIGIT_SLICES
    if modular:
        call.flags |= MODULAR
    _check(lib().uor_b200_gemm(elem, out, ctypes.byref(A), ctypes.byref(B), ctypes.byref(C),
                               alpha, beta, ctypes.byref(call)), "gemm")


def complex_view(buf, rows, cols, rs=None, cs=1):
    """A MatView of Complex<T> over a flat buffer of interleaved (re, im) parts; the
    length and strides count complex elements."""
    ptr, n, _ = _buffer(buf)
    return View(ptr, n // 2, rows, cols, cols if rs is None else rs, cs)


def gemm_complex(elem, out, a, av, b, bv, c, cv, alpha=1, beta=0, encode=NEAREST, ctx=None,
                 route=None, asynchronous=False, digits=False, modular=False):
    """driver::gemm over Complex<elem> (alphabet.rs:656-776) into Complex<out>.

    elem in {I32, I64} and out in {I8 .. I128} name the part types; a, b, c are flat
    buffers of interleaved parts and av/bv/cv are (rows, cols, rs, cs) in complex
    elements. Each part is encoded on its own (EncodeFrom<ComplexAcc>); alpha and beta
    scale each part as Linear scales a scalar accumulator."""
    dev = _on_device(a, b, c)
    A, B, C = complex_view(a, *av), complex_view(b, *bv), complex_view(c, *cv)
    call = make_call(encode, dev, ctx, route, asynchronous)
    if digits:
        call.flags |= DIGIT_SLICES
    if modular:
        call.flags |= MODULAR
    _check(lib().uor_b200_gemm_complex(elem, out, ctypes.byref(A), ctypes.byref(B),
                                       ctypes.byref(C), alpha, beta, ctypes.byref(call)),
           "gemm_complex")


def slice_gemm_ex(elem, out, m, k, n, alpha, a, lda, b, ldb, beta, c, ldc, encode=NEAREST,
                  ctx=None, route=None, scratch=None):
    """slice::gemm_ex (slice.rs:144-178)."""
    dev = _on_device(a, b, c)
    pa, la, _ = _buffer(a)
    pb, lb, _ = _buffer(b)
    pc, lc, _ = _buffer(c)
    ps, ls = (_buffer(scratch)[:2] if scratch is not None else (None, 0))
    call = make_call(encode, dev, ctx, route)
    _check(lib().uor_b200_slice_gemm_ex(elem, out, m, k, n, alpha, pa, la, lda, pb, lb, ldb, beta,
                                        pc, lc, ldc, ps, ls, ctypes.byref(call)), "slice_gemm_ex")


def slice_gemm(elem, out, m, k, n, a, b, c, encode=NEAREST, ctx=None, route=None):
    """slice::gemm (slice.rs:184-199)."""
    dev = _on_device(a, b, c)
    pa, la, _ = _buffer(a)
    pb, lb, _ = _buffer(b)
    pc, lc, _ = _buffer(c)
    call = make_call(encode, dev, ctx, route)
    _check(lib().uor_b200_slice_gemm(elem, out, m, k, n, pa, la, pb, lb, pc, lc, None, 0,
                                     ctypes.byref(call)), "slice_gemm")


def gemm_i8_i32(m, k, n, a, b, c, ctx=None, route=None, asynchronous=False):
    """slice::gemm::<i8, i32>, monomorphised (contiguous, alpha 1, beta 0)."""
    dev = _on_device(a, b, c)
    call = make_call(NEAREST, dev, ctx, route, asynchronous)
    _check(lib().uor_b200_gemm_i8_i32(m, k, n, _buffer(a)[0], _buffer(b)[0], _buffer(c)[0],
                                      ctypes.byref(call)), "gemm_i8_i32")


# ------------------------------------------------------------------ float

def gemm_float(elem, out, a, av, b, bv, c, cv, alpha=1, beta=0, encode=NEAREST, ctx=None,
               route=None, asynchronous=False, digits=False, modular=False):
    """gemm_float over views; digits=True takes the digit-slice route even where the
    modular route applies (the same bytes either way)."""
    dev = _on_device(a, b, c)
    A, B, C = view(a, *av), view(b, *bv), view(c, *cv)
    call = make_call(encode, dev, ctx, route, asynchronous)
    if digits:
        call.flags |= DIGIT_SLICES
    if modular:
        call.flags |= MODULAR
    _check(lib().uor_b200_gemm_float(elem, out, ctypes.byref(A), ctypes.byref(B),
                                     ctypes.byref(C), alpha, beta, ctypes.byref(call)),
           "gemm_float")


def slice_gemm_float_ex(elem, out, m, k, n, alpha, a, lda, b, ldb, beta, c, ldc, encode=NEAREST,
                        ctx=None, route=None):
    """slice::gemm_float_ex (slice.rs:304-356)."""
    dev = _on_device(a, b, c)
    pa, la, _ = _buffer(a)
    pb, lb, _ = _buffer(b)
    pc, lc, _ = _buffer(c)
    call = make_call(encode, dev, ctx, route)
    _check(lib().uor_b200_slice_gemm_float_ex(elem, out, m, k, n, alpha, pa, la, lda, pb, lb, ldb,
                                              beta, pc, lc, ldc, None, 0, None, 0,
                                              ctypes.byref(call)), "slice_gemm_float_ex")


def sgemm(m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc, origin=(0, 0, 0),
          ctx=None, route=None, encode=NEAREST):
    """raw::sgemm (raw.rs:45-64); `origin` gives the element index of (0,0) in each buffer."""
    dev = _on_device(a, b, c)
    pa, pb, pc = (_buffer(x)[0] + o * 4 for x, o in zip((a, b, c), origin))
    call = make_call(encode, dev, ctx, route)
    _check(lib().uor_b200_sgemm(m, k, n, alpha, pa, rsa, csa, pb, rsb, csb, beta, pc, rsc, csc,
                                ctypes.byref(call)), "sgemm")


def dgemm(m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc, origin=(0, 0, 0),
          ctx=None, route=None, encode=NEAREST):
    """raw::dgemm (raw.rs:72-90)."""
    dev = _on_device(a, b, c)
    pa, pb, pc = (_buffer(x)[0] + o * 8 for x, o in zip((a, b, c), origin))
    call = make_call(encode, dev, ctx, route)
    _check(lib().uor_b200_dgemm(m, k, n, alpha, pa, rsa, csa, pb, rsb, csb, beta, pc, rsc, csc,
                                ctypes.byref(call)), "dgemm")


# ------------------------------------------------------------------ tropical

def gemm_tropical(elem, out, a, av, b, bv, c, cv, alpha=(0, True), beta=(0, False),
                  encode=NEAREST, ctx=None, route=None, asynchronous=False):
    """driver::gemm over Trop<E> with MaxPlus{alpha, beta}; scalars are (value, finite)."""
    dev = _on_device(a, b, c)
    A, B, C = view(a, *av), view(b, *bv), view(c, *cv)
    call = make_call(encode, dev, ctx, route, asynchronous)
    _check(lib().uor_b200_gemm_tropical(elem, out, ctypes.byref(A), ctypes.byref(B),
                                        ctypes.byref(C), Trop(alpha[0], int(alpha[1])),
                                        Trop(beta[0], int(beta[1])), ctypes.byref(call)),
           "gemm_tropical")


def gemm_tropical_selected(elem, out, a, av, b, bv, c, cv, w, wv, alpha=(0, True),
                           beta=(0, False), encode=NEAREST, ctx=None, route=None):
    """driver::gemm_selected: the product and the least-index witness (u64 view w)."""
    dev = _on_device(a, b, c, w)
    A, B, C, W = view(a, *av), view(b, *bv), view(c, *cv), view(w, *wv)
    call = make_call(encode, dev, ctx, route)
    _check(lib().uor_b200_gemm_tropical_selected(elem, out, ctypes.byref(A), ctypes.byref(B),
                                                 ctypes.byref(C), ctypes.byref(W),
                                                 Trop(alpha[0], int(alpha[1])),
                                                 Trop(beta[0], int(beta[1])), ctypes.byref(call)),
           "gemm_tropical_selected")


# ------------------------------------------------------------------ codec

def coded_gemm(out, a, av, codes, k, n, per_byte, table, c, cv, alpha=1, beta=0,
               encode=NEAREST, ctx=None, route=None, tabulated=False, asynchronous=False,
               on_chip=False):
    """coded_gemm (k x n codes) or, with tabulated=True, gemm_tabulated's A W^T (n x k codes).
    on_chip=True never decodes the codes into a dense device copy (CODEC_ON_CHIP)."""
    dev = _on_device(a, codes, table, c)
    A, C = view(a, *av), view(c, *cv)
    pc, lc, _ = _buffer(codes)
    pt, lt, _ = _buffer(table)
    call = make_call(encode, dev, ctx, route, asynchronous)
    if on_chip:
        call.flags |= CODEC_ON_CHIP
    fn = lib().uor_b200_tabulated_gemm if tabulated else lib().uor_b200_coded_gemm
    _check(fn(out, ctypes.byref(A), pc, lc, k, n, per_byte, pt, lt, ctypes.byref(C), alpha, beta,
              ctypes.byref(call)), "coded_gemm")


def codec_gemm(out, a, av, tier, codes, k, n, c, cv, table=None, per_byte=0, block=0,
               code_bytes=1, zero=0, alpha=1, beta=0, encode=NEAREST, ctx=None, route=None,
               orientation=0, asynchronous=False):
    """coded_gemm (orientation 0, codes k x n) / gemm_tabulated (1, codes n x k) for any
    fixed-width tier: TIER_GRID (per_byte, table), TIER_SIGN / TIER_TERNARY (block,
    code_bytes), TIER_BOOK (block, code_bytes, table of N x block); zero is Offset's."""
    bufs = (a, codes, c) if table is None else (a, codes, table, c)
    dev = _on_device(*bufs)
    A, C = view(a, *av), view(c, *cv)
    pc, lc, _ = _buffer(codes)
    if table is not None:
        pt, lt, _ = _buffer(table)
        n_entries = lt if tier != TIER_BOOK else lt // max(block, 1)
    else:
        pt, n_entries = None, 0
    cod = Codec(tier, per_byte, block, code_bytes, pt, n_entries, zero)
    call = make_call(encode, dev, ctx, route, asynchronous)
    _check(lib().uor_b200_codec_gemm(out, ctypes.byref(A), ctypes.byref(cod), pc, lc, k, n,
                                     orientation, ctypes.byref(C), alpha, beta,
                                     ctypes.byref(call)), "codec_gemm")


E8_ENTRIES, E8_BLOCK = 256, 8


def e8_table(bound=0):
    """e8_table (e8.rs:295-307): the E8 codebook as a (256, 8) int8 array, for
    codec_gemm(tier=TIER_BOOK, block=8). bound = 0 is Full<i8>; a bound below 32
    has no table (UorError UNSUPPORTED, the reference's None)."""
    out = np.zeros((E8_ENTRIES, E8_BLOCK), np.int8)
    _check(lib().uor_b200_e8_table(bound, out.ctypes.data, out.size), "e8_table")
    return out


def arena_gemm(elem, out, a, av, table, codes, k, n, c, cv, code_bytes=1, orientation=0,
               alpha=1, beta=0, encode=NEAREST, ctx=None, route=None, asynchronous=False):
    """coded_gemm / gemm_tabulated over Arena<E, N, K> (codecs.rs:894-985): codes (u8 or
    u16) index `table`, N float symbols of elem's type (F32 / F64), modulo N; the product
    with the float A is gemm_float's. orientation 0: codes k x n, 1: n x k."""
    dev = _on_device(a, table, codes, c)
    A, C = view(a, *av), view(c, *cv)
    pt, lt, _ = _buffer(table)
    pc, _, _ = _buffer(codes)
    nbytes = codes.numel() * codes.element_size() if _is_torch(codes) else np.asarray(codes).nbytes
    call = make_call(encode, dev, ctx, route, asynchronous)
    _check(lib().uor_b200_arena_gemm(elem, out, ctypes.byref(A), pt, lt, pc, nbytes, code_bytes,
                                     k, n, orientation, ctypes.byref(C), alpha, beta,
                                     ctypes.byref(call)), "arena_gemm")


def arena_canonicalize(values):
    """canonicalize (codecs.rs:990-1003) in place on a float32 / float64 NumPy array;
    returns the count of distinct bit patterns now at the front."""
    elem = {np.dtype(np.float32): F32, np.dtype(np.float64): F64}[values.dtype]
    n = ctypes.c_size_t(0)
    _check(lib().uor_b200_arena_canonicalize(elem, values.ctypes.data, values.size,
                                             ctypes.byref(n)), "arena_canonicalize")
    return n.value


# ------------------------------------------------------------------ split-K exchange

SPLITK_LIMBS = 3


def gemm_partial_limbs(elem, a, av, b, bv, limbs, ctx=None, route=None, asynchronous=False):
    """Exact partial sum of A B as radix-2^40 int64 limbs [m][n][3] (device buffers)."""
    if not _on_device(a, b, limbs):
        raise UorError(INVALID_ARGUMENT, "gemm_partial_limbs takes device buffers")
    A, B = view(a, *av), view(b, *bv)
    pl, ll, _ = _buffer(limbs)
    call = make_call(NEAREST, True, ctx, route, asynchronous)
    _check(lib().uor_b200_gemm_partial_limbs(elem, ctypes.byref(A), ctypes.byref(B), pl,
                                             _int64_len(limbs, ll), ctypes.byref(call)),
           "gemm_partial_limbs")


def limbs_finish(elem, out, limbs, c, cv, alpha=1, beta=0, encode=NEAREST, ctx=None,
                 asynchronous=False):
    """C := encode(alpha X + beta C) from summed limbs (device buffers)."""
    if not _on_device(limbs, c):
        raise UorError(INVALID_ARGUMENT, "limbs_finish takes device buffers")
    C = view(c, *cv)
    pl, ll, _ = _buffer(limbs)
    call = make_call(encode, True, ctx, None, asynchronous)
    _check(lib().uor_b200_limbs_finish(elem, out, pl, _int64_len(limbs, ll), ctypes.byref(C),
                                       alpha, beta, ctypes.byref(call)), "limbs_finish")


def trop_partial_keys(elem, a, av, b, bv, keys, ctx=None, route=None, asynchronous=False):
    """One range of a Trop<E> reduction as int64 keys [m][n] (INT64_MIN: no finite term);
    the element-wise max of ranges' keys is the reduction of their union (device buffers)."""
    if not _on_device(a, b, keys):
        raise UorError(INVALID_ARGUMENT, "trop_partial_keys takes device buffers")
    A, B = view(a, *av), view(b, *bv)
    pk, lk, _ = _buffer(keys)
    call = make_call(NEAREST, True, ctx, route, asynchronous)
    _check(lib().uor_b200_trop_partial_keys(elem, ctypes.byref(A), ctypes.byref(B), pk,
                                            _int64_len(keys, lk), ctypes.byref(call)),
           "trop_partial_keys")


def trop_keys_finish(out, keys, c, cv, alpha=(0, True), beta=(0, False), encode=NEAREST, ctx=None,
                     asynchronous=False):
    """C := (alpha (x) X) (+) (beta (x) C), encoded, from keys X (device buffers)."""
    if not _on_device(keys, c):
        raise UorError(INVALID_ARGUMENT, "trop_keys_finish takes device buffers")
    C = view(c, *cv)
    pk, lk, _ = _buffer(keys)
    call = make_call(encode, True, ctx, None, asynchronous)
    _check(lib().uor_b200_trop_keys_finish(out, pk, _int64_len(keys, lk), ctypes.byref(C),
                                           Trop(alpha[0], int(alpha[1])),
                                           Trop(beta[0], int(beta[1])), ctypes.byref(call)),
           "trop_keys_finish")


# ------------------------------------------------------------------ split-K over NCCL

NCCL_ID_BYTES = 128


def nccl_unique_id() -> bytes:
    """A new NCCL unique id (rank 0 makes it; every rank joins with it)."""
    buf = (ctypes.c_uint8 * NCCL_ID_BYTES)()
    _check(lib().uor_b200_nccl_unique_id(ctypes.addressof(buf), NCCL_ID_BYTES), "nccl_unique_id")
    return bytes(buf)


class NcclComm:
    """An NCCL communicator made through the C ABI (uor_b200_nccl_comm_init) on the
    context's device; destroy() (or the context manager) releases it."""

    def __init__(self, nranks: int, uid: bytes, rank: int, ctx: "Context | None" = None):
        if len(uid) != NCCL_ID_BYTES:
            raise UorError(INVALID_ARGUMENT, "an NCCL id is 128 bytes")
        buf = (ctypes.c_uint8 * NCCL_ID_BYTES).from_buffer_copy(uid)
        out = ctypes.c_void_p()
        _check(lib().uor_b200_nccl_comm_init(ctx.handle if ctx else None, nranks,
                                             ctypes.addressof(buf), NCCL_ID_BYTES, rank,
                                             ctypes.byref(out)), "nccl_comm_init")
        self.handle = out.value

    def destroy(self):
        if self.handle:
            _check(lib().uor_b200_nccl_comm_destroy(self.handle), "nccl_comm_destroy")
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.destroy()


def gemm_splitk_nccl(comm, elem, out, a, av, b, bv, c, cv, alpha=1, beta=0, encode=NEAREST,
                     ctx=None, route=None, asynchronous=False):
    """This rank's range of the reduction (A's columns, B's rows) in, the whole exact C out
    on every rank: partial limbs, an NCCL all-reduce and the finish (device buffers)."""
    if not _on_device(a, b, c):
        raise UorError(INVALID_ARGUMENT, "gemm_splitk_nccl takes device buffers")
    A, B, C = view(a, *av), view(b, *bv), view(c, *cv)
    call = make_call(encode, True, ctx, route, asynchronous)
    _check(lib().uor_b200_gemm_splitk_nccl(comm.handle if isinstance(comm, NcclComm) else comm,
                                           elem, out, ctypes.byref(A), ctypes.byref(B),
                                           ctypes.byref(C), alpha, beta, ctypes.byref(call)),
           "gemm_splitk_nccl")


def gemm_tropical_splitk_nccl(comm, elem, out, a, av, b, bv, c, cv, alpha=(0, True),
                              beta=(0, False), encode=NEAREST, ctx=None, route=None,
                              asynchronous=False):
    """The same for Trop<E>: max-plus keys, an NCCL all-reduce with MAX, MaxPlus::finish."""
    if not _on_device(a, b, c):
        raise UorError(INVALID_ARGUMENT, "gemm_tropical_splitk_nccl takes device buffers")
    A, B, C = view(a, *av), view(b, *bv), view(c, *cv)
    call = make_call(encode, True, ctx, route, asynchronous)
    _check(lib().uor_b200_gemm_tropical_splitk_nccl(
        comm.handle if isinstance(comm, NcclComm) else comm, elem, out, ctypes.byref(A),
        ctypes.byref(B), ctypes.byref(C), Trop(alpha[0], int(alpha[1])),
        Trop(beta[0], int(beta[1])), ctypes.byref(call)), "gemm_tropical_splitk_nccl")


def _int64_len(limbs, count):
    if str(limbs.dtype) not in ("torch.int64", "int64"):
        raise UorError(INVALID_ARGUMENT, "limbs must be int64")
    return count


# ------------------------------------------------------------------ corpus

CORPUS_I8, CORPUS_I32_FULL, CORPUS_RAW, CORPUS_NIBBLES, CORPUS_TROP_I8, CORPUS_F32_WIDE = range(6)


def corpus(salt: int, kind: int, count: int) -> np.ndarray:
    """The reference's recorded fill (validate/tests/common/mod.rs:9-19), mapped by kind."""
    if kind == CORPUS_I8:
        out = np.empty(count, dtype=np.int8)
    elif kind == CORPUS_I32_FULL:
        out = np.empty(count, dtype=np.int32)
    elif kind == CORPUS_RAW:
        out = np.empty(count, dtype=np.uint64)
    elif kind == CORPUS_NIBBLES:
        out = np.empty((count + 1) // 2, dtype=np.uint8)
    elif kind == CORPUS_TROP_I8:
        out = np.empty(count * 2, dtype=np.uint8)
    elif kind == CORPUS_F32_WIDE:
        out = np.empty(count, dtype=np.float32)
    else:
        raise ValueError(kind)
    _check(lib().uor_b200_corpus_fill(salt, kind, count, out.ctypes.data), "corpus_fill")
    return out


def selftest_wait_timeout(ctx: Context, budget_ns: int) -> int:
    return lib().uor_b200_selftest_wait_timeout(ctx.handle, budget_ns)
