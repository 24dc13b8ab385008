"""CPU stand-ins for the device calls of uor_b200_dist, so that its host protocol
(ranges, limb format, exchange, gather) runs under gloo without a GPU. They are
restatements on top of the oracle, used only by the tests."""
import numpy as np

import uor_b200 as U
from oracle import oracle as orc

NP = {U.I8: np.int8, U.I16: np.int16, U.I32: np.int32, U.I64: np.int64}
OBITS = {U.I8: 8, U.I16: 16, U.I32: 32, U.I64: 64, U.I128: 128}
I128_MIN, I128_MAX = -(1 << 127), (1 << 127) - 1
MASK40 = (1 << 40) - 1


def _np(t, dtype):
    return t.numpy().view(dtype)


def partial_cpu(elem, a, av, b, bv, limbs, ctx=None, asynchronous=False):
    """Exact sum over the views (oracle, i128 out, Wrapping) written as radix-2^40 limbs."""
    m, k = av[0], av[1]
    n = bv[1]
    an, bn = _np(a, NP[elem]), _np(b, NP[elem])
    x = np.zeros(2 * m * n, np.int64)
    if k:
        orc.gemm_int(orc.View(an, m, k, av[2], av[3]), orc.View(bn, k, n, bv[2], bv[3]),
                     orc.View(x, m, n, n, 1), mode=orc.WRAPPING, out_bits=128)
    out = limbs.numpy()
    for idx in range(m * n):
        v = int(np.uint64(x[2 * idx])) + (int(x[2 * idx + 1]) << 64)
        out[3 * idx] = v & MASK40
        out[3 * idx + 1] = (v >> 40) & MASK40
        out[3 * idx + 2] = v >> 80


def _sat(v):
    return max(I128_MIN, min(I128_MAX, v))


def _wrap128(v):
    v &= (1 << 128) - 1
    return v - (1 << 128) if v >> 127 else v


def _encode(v, bits, mode):
    if bits >= 128:
        return v
    if mode == orc.WRAPPING:
        v &= (1 << bits) - 1
        return v - (1 << bits) if v >> (bits - 1) else v
    lo, hi = -(1 << (bits - 1)), (1 << (bits - 1)) - 1
    return max(lo, min(hi, v))


def finish_cpu(elem, out, limbs, c, cv, alpha=1, beta=0, encode=0, ctx=None, asynchronous=False):
    """Linear::finish over the i128 accumulator (epilogue.rs:79-93, 280-288)."""
    m, n, rs, cs = cv
    ln = limbs.numpy()
    bits = OBITS[out]
    cn = c.numpy()
    for i in range(m):
        for j in range(n):
            idx = i * n + j
            x = int(ln[3 * idx]) + (int(ln[3 * idx + 1]) << 40) + (int(ln[3 * idx + 2]) << 80)
            tot = x if alpha == 1 else _sat(x * alpha)
            off = i * rs + j * cs
            if beta != 0:
                if bits == 128:
                    prior = int(np.uint64(cn[2 * off])) + (int(cn[2 * off + 1]) << 64)
                    prior = prior - (1 << 128) if prior >> 127 else prior
                else:
                    prior = int(cn[off])
                tot = _wrap128(tot + _sat(prior * beta))
            r = _encode(tot, bits, encode)
            if bits == 128:
                r &= (1 << 128) - 1
                cn[2 * off] = np.int64(np.uint64(r & ((1 << 64) - 1)).view(np.int64))
                cn[2 * off + 1] = np.int64(np.uint64(r >> 64).view(np.int64))
            else:
                cn[off] = r


def gemm_cpu(elem, out, a, av, b, bv, c, cv, alpha=1, beta=0, encode=0, ctx=None):
    """The view-API call on host arrays, through the oracle."""
    an, bn = _np(a, NP[elem]), _np(b, NP[elem])
    cn = c.numpy()
    orc.gemm_int(orc.View(an, *av), orc.View(bn, *bv), orc.View(cn, *cv), alpha=alpha, beta=beta,
                 mode=encode, out_bits=OBITS[out])


# ---- tropical (driver::gemm over Trop<E>, MaxPlus, the clamp encode)

TBITS = {U.TROP_I8: 8, U.TROP_I16: 16, U.TROP_I32: 32, U.TROP_I64: 64}
INT64_MIN = -(1 << 63)


def trop_partial_cpu(elem, a, av, b, bv, keys, ctx=None, asynchronous=False):
    """One range's (max, +) reduction as int64 keys, through the oracle (Trop<i64> out,
    alpha the identity, no C read)."""
    m, k = av[0], av[1]
    n = bv[1]
    TD = orc.TROP_DTYPES
    eb = TBITS[elem]
    an, bn = a.numpy().view(TD[eb]), b.numpy().view(TD[eb])
    x = np.zeros(m * n, TD[64])
    orc.gemm_trop(orc.View(an, m, k, av[2], av[3]), orc.View(bn, k, n, bv[2], bv[3]),
                  orc.View(x, m, n, n, 1), ebits=eb, obits=64)
    kn = keys.numpy()
    kn[: m * n] = np.where(x["f"] != 0, x["v"], INT64_MIN)


def trop_finish_cpu(out, keys, c, cv, alpha=(0, True), beta=(0, False), encode=0, ctx=None,
                    asynchronous=False):
    """MaxPlus::finish (epilogue.rs:137-186) and the clamp encode (tropical.rs:336-351)."""
    m, n, rs, cs = cv
    ob = TBITS[out]
    cn = c.numpy().view(orc.TROP_DTYPES[ob])
    kn = keys.numpy()
    mx = (1 << (ob - 1)) - 2
    mn = -mx - 1
    for i in range(m):
        for j in range(n):
            key = int(kn[i * n + j])
            fin = key != INT64_MIN and alpha[1]
            tot = key + alpha[0] if fin else 0
            off = i * rs + j * cs
            if beta[1] and cn["f"][off]:
                s = int(cn["v"][off]) + beta[0]
                if not fin or s > tot:
                    tot, fin = s, True
            if fin:
                if encode == orc.WRAPPING:
                    span = mx - mn + 1
                    tot = ((tot - mn) % (1 << 128)) % span + mn
                    tot = tot - (1 << 128) if tot >= (1 << 127) else tot
                else:
                    tot = max(mn, min(mx, tot))
            cn["v"][off] = tot if fin else 0
            cn["f"][off] = 1 if fin else 0


def trop_gemm_cpu(elem, out, a, av, b, bv, c, cv, alpha=(0, True), beta=(0, False), encode=0,
                  ctx=None):
    """driver::gemm over Trop<E> on host byte tensors, through the oracle."""
    TD = orc.TROP_DTYPES
    an = a.numpy().view(TD[TBITS[elem]])
    bn = b.numpy().view(TD[TBITS[elem]])
    cn = c.numpy().view(TD[TBITS[out]])
    orc.gemm_trop(orc.View(an, *av), orc.View(bn, *bv), orc.View(cn, *cv), ebits=TBITS[elem],
                  obits=TBITS[out], alpha=alpha, beta=beta, mode=encode)

