"""The arithmetic the modular route's kernels rely on, checked on the host over the moduli
list exactly as csrc/modular.cu declares it:

* the balanced residue from one widening multiply-add (fm_balanced_v): with
  magic = ceil(2^32 / p) and half = (p - 1) / 2 (127 for 256),
  v - p * floor((v * magic + half * magic) / 2^32) == ((v + half) mod p) - half
  for every v a slicer can produce (below 2^20);
* the CRT's last base-256 column is zero from three moduli on: M / p_g < 256^(NM - 1);
* the moduli are pairwise coprime and at most 256 (int8 residues)."""
import math
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def moduli():
    src = open(os.path.join(ROOT, "uor-matmul_b200", "csrc", "modular.cu")).read()
    body = re.search(r"kModuli\[FM_MAX\]\s*=\s*\{([^}]*)\}", src).group(1)
    return [int(x) for x in re.findall(r"\d+", body)]


def half_of(p):
    return 127 if p == 256 else (p - 1) // 2


def test_moduli_list():
    ps = moduli()
    assert len(ps) == 40 and all(2 <= p <= 256 for p in ps)
    for i in range(len(ps)):
        for j in range(i):
            assert math.gcd(ps[i], ps[j]) == 1, (ps[i], ps[j])


def test_balanced_residue_by_one_multiply_add():
    v = np.arange(0, 1 << 20, dtype=np.uint64)
    for p in moduli():
        h = half_of(p)
        magic = ((1 << 32) + p - 1) // p
        q = (v * np.uint64(magic) + np.uint64(h * magic)) >> np.uint64(32)
        r = v.astype(np.int64) - q.astype(np.int64) * p
        want = (v.astype(np.int64) + h) % p - h
        assert np.array_equal(r, want), p
        # the low byte read as int8 is the same residue modulo p
        low = (r & 0xFF).astype(np.uint8).view(np.int8).astype(np.int64)
        assert np.all((low - want) % p == 0), p


def test_last_crt_column_is_zero():
    ps = moduli()
    for nm in range(4, 41, 2):
        m = math.prod(ps[:nm])
        for p in ps[:nm]:
            assert m // p < 256 ** (nm - 1), (nm, p)
    # with two moduli the column is needed: M / 255 = 256
    assert math.prod(ps[:2]) // 255 == 256
