"""The multi-device protocol on CPU: Partition, reduction ranges, and world-size-2
gloo runs of the split-K limb exchange and the column-block gather, with the device
calls replaced by oracle-backed stand-ins (tests/dist_standins.py)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import uor_b200 as U
import uor_b200_dist as D
from oracle import oracle as orc


def test_partition_covers_output_exactly_once():
    # partition.rs CD-02: every cell in exactly one tile, for every tile shape
    for m, n in [(0, 0), (1, 1), (5, 7), (13, 17), (64, 64), (97, 3)]:
        for tr, tc in [(0, 0), (1, 1), (2, 3), (8, 8), (64, 64), (1000, 1000)]:
            part = D.Partition(m, n, tr, tc)
            seen = np.zeros(m * n, np.int32)
            tiles = list(part)
            assert len(tiles) == len(part)
            for t in tiles:
                for i in range(t.row, t.row + t.rows):
                    for j in range(t.col, t.col + t.cols):
                        seen[i * n + j] += 1
            assert (seen == 1).all(), (m, n, tr, tc)


def test_partition_indexed_and_sequential_agree():
    part = D.Partition(13, 17, 4, 6)
    assert list(part) == [part.tile(i) for i in range(len(part))]
    assert part.tile(len(part)) is None


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_column_blocks_and_k_ranges_cover(world):
    for n in (1, 7, 256, 8192, 8193):
        part = D.column_blocks(5, n, world)
        assert len(part) <= world
        assert sum(t.cols for t in part) == n
    for k in (0, 1, 100, 128 * world, 65536, 65537):
        r = D.k_ranges(k, world)
        assert len(r) == world and r[0][0] == 0 and r[-1][1] == k
        assert all(a1 == b0 for (_, a1), (b0, _) in zip(r, r[1:]))
        if k >= 128 * world:
            assert all(k0 % 128 == 0 for k0, _ in r)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _trop_draw(salt, count, bits, lo=-64, hi=63):
    """Trop<E> values in [lo, hi] with about 5 % at the semiring zero (value stored 0)."""
    raw = U.corpus(salt, U.CORPUS_RAW, count)
    t = np.zeros(count, orc.TROP_DTYPES[bits])
    fin = (raw >> np.uint64(20)) % np.uint64(100) >= np.uint64(5)
    t["v"] = np.where(fin, (raw % np.uint64(hi - lo + 1)).astype(np.int64) + lo, 0)
    t["f"] = fin
    return t


def _worker(rank, world, port, case):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    import dist_standins as S
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        if case == "splitk":
            for elem, out, (m, k, n), alpha, beta, mode in [
                    (U.I32, U.I128, (5, 300, 7), 1, 0, U.NEAREST),
                    (U.I32, U.I64, (4, 257, 3), -3, 2, U.SATURATING),
                    (U.I16, U.I32, (6, 129, 5), 7, -1, U.WRAPPING),
                    (U.I8, U.I32, (3, 1000, 9), 2**40, 1, U.NEAREST),
                    (U.I32, U.I32, (2, 1, 2), 1, 0, U.NEAREST)]:   # one rank has no range
                dt = S.NP[elem]
                a = U.corpus(4, U.CORPUS_I32_FULL, m * k).astype(dt, casting="unsafe")
                b = U.corpus(5, U.CORPUS_I32_FULL, k * n).astype(dt, casting="unsafe")
                cw = 2 if out == U.I128 else 1
                prior = U.corpus(3, U.CORPUS_I32_FULL, m * n * cw).astype(np.int64)
                if out != U.I128:
                    prior = prior.astype(S.NP[out], casting="unsafe")
                c = torch.from_numpy(prior.copy())
                D.splitk_gemm(elem, out, torch.from_numpy(a), (m, k, k, 1), torch.from_numpy(b),
                              (k, n, n, 1), c, (m, n, n, 1), alpha, beta, mode,
                              partial=S.partial_cpu, finish=S.finish_cpu)
                want = prior.copy()
                orc.gemm_int(orc.View(a, m, k, k, 1), orc.View(b, k, n, n, 1),
                             orc.View(want, m, n, n, 1), alpha=alpha, beta=beta, mode=mode,
                             out_bits=S.OBITS[out])
                assert np.array_equal(c.numpy(), want), (rank, elem, out, m, k, n)
        elif case == "trop-splitk":
            # driver::gemm over Trop<E> with the reduction split across the two ranks:
            # int64 keys, an all-reduce of MAX, MaxPlus and the encode once
            TD = orc.TROP_DTYPES
            for elem, out, (m, k, n), alpha, beta, mode in [
                    (U.TROP_I8, U.TROP_I32, (5, 301, 7), (0, True), (0, False), U.NEAREST),
                    (U.TROP_I8, U.TROP_I8, (4, 260, 6), (100, True), (-3, True), U.NEAREST),
                    (U.TROP_I16, U.TROP_I16, (3, 129, 5), (2**14, True), (7, True), U.WRAPPING),
                    (U.TROP_I8, U.TROP_I32, (6, 40, 4), (5, False), (1, True), U.NEAREST),
                    (U.TROP_I8, U.TROP_I64, (2, 1, 3), (0, True), (0, False), U.NEAREST)]:
                eb, ob = S.TBITS[elem], S.TBITS[out]
                a = _trop_draw(11 + m, m * k, eb)
                b = _trop_draw(12 + n, k * n, eb)
                prior = _trop_draw(13, m * n, ob, lo=-100, hi=100)
                c = torch.from_numpy(prior.copy().view(np.uint8))
                D.splitk_gemm_tropical(elem, out, torch.from_numpy(a.view(np.uint8)),
                                       (m, k, k, 1), torch.from_numpy(b.view(np.uint8)),
                                       (k, n, n, 1), c, (m, n, n, 1), alpha, beta, mode,
                                       partial=S.trop_partial_cpu, finish=S.trop_finish_cpu)
                want = prior.copy()
                orc.gemm_trop(orc.View(a, m, k, k, 1), orc.View(b, k, n, n, 1),
                              orc.View(want, m, n, n, 1), ebits=eb, obits=ob, alpha=alpha,
                              beta=beta, mode=mode)
                got = c.numpy().view(TD[ob])
                assert np.array_equal(got["f"], want["f"]), (rank, elem, out)
                fin = want["f"] != 0
                assert np.array_equal(got["v"][fin], want["v"][fin]), (rank, elem, out)
        elif case == "trop-columns":
            TD = orc.TROP_DTYPES
            m, k, n = 6, 45, 11
            a = _trop_draw(21, m * k, 8)
            b = _trop_draw(22, k * n, 8)
            c = torch.zeros(m * n * 8, dtype=torch.uint8)
            t = D.column_block_gemm_tropical(U.TROP_I8, U.TROP_I32,
                                             torch.from_numpy(a.view(np.uint8)), (m, k, k, 1),
                                             torch.from_numpy(b.view(np.uint8)), (k, n, n, 1), c,
                                             (m, n, n, 1), (4, True), gather=True,
                                             gemm=S.trop_gemm_cpu)
            assert t is not None and t.cols > 0
            want = np.zeros(m * n, TD[32])
            orc.gemm_trop(orc.View(a, m, k, k, 1), orc.View(b, k, n, n, 1),
                          orc.View(want, m, n, n, 1), ebits=8, obits=32, alpha=(4, True))
            got = c.numpy().view(TD[32])
            assert np.array_equal(got["f"], want["f"]), rank
            fin = want["f"] != 0
            assert np.array_equal(got["v"][fin], want["v"][fin]), rank
        else:
            m, k, n = 7, 33, 13
            a = U.corpus(1, U.CORPUS_I8, m * k)
            b = U.corpus(2, U.CORPUS_I8, k * n)
            c = torch.zeros(m * n, dtype=torch.int32)
            t = D.column_block_gemm(U.I8, U.I32, torch.from_numpy(a), (m, k, k, 1),
                                    torch.from_numpy(b), (k, n, n, 1), c, (m, n, n, 1), 3, 0,
                                    gather=True, gemm=S.gemm_cpu)
            assert t is not None and t.cols > 0
            want = np.zeros(m * n, np.int32)
            orc.gemm_int(orc.View(a, m, k, k, 1), orc.View(b, k, n, n, 1),
                         orc.View(want, m, n, n, 1), alpha=3)
            assert np.array_equal(c.numpy(), want), rank
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", ["splitk", "columns", "trop-splitk", "trop-columns"])
def test_two_ranks_gloo(case):
    mp.spawn(_worker, args=(2, _free_port(), case), nprocs=2, join=True)
