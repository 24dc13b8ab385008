"""Config-3 operands: the wide-exponent f32 corpus with exact-cancellation columns."""
import numpy as np

import uor_b200 as U


def config3(m, k, n, salt_a=1, salt_b=2):
    """A, B as float32 arrays: entries +-m 2^(e-23), m in [2^23, 2^24), e in [-30, 30]
    (the reference generator, kind F32_WIDE); every tenth column j of B is
    B[p][j] = (-1)^p 2^s_j A[r][p ^ 1] with r = j mod m and s_j in [-4, 4], so that
    row r of column j cancels pairwise to exactly zero."""
    a = U.corpus(salt_a, U.CORPUS_F32_WIDE, m * k).reshape(m, k)
    b = U.corpus(salt_b, U.CORPUS_F32_WIDE, k * n).reshape(k, n)
    kk = k - (k % 2)
    sign = np.where(np.arange(k) % 2 == 0, 1.0, -1.0).astype(np.float32)
    for j in range(0, n, 10):
        r = j % m
        s = ((j // 10) % 9) - 4
        col = b[:, j].copy()
        col[:kk] = a[r, np.arange(kk) ^ 1] * sign[:kk] * np.float32(2.0 ** s)
        b[:, j] = col
    return np.ascontiguousarray(a), np.ascontiguousarray(b)
