"""The split-K exchange on the GPU: partial limbs and the finish kernel against the
single-device call (bit for bit), one GPU emulating the ranks' ranges; and, where the
box has two GPUs, two NCCL ranks through uor_b200_dist.splitk_gemm and through the C ABI's
own NCCL entry points (uor_b200_gemm_splitk_nccl, uor_b200_gemm_tropical_splitk_nccl)."""
import os
import socket

import numpy as np
import pytest

import uor_b200 as U
import uor_b200_dist as D
from gpu_util import needs_gpu, torch

pytestmark = [pytest.mark.gpu, needs_gpu]

NPT = {U.I8: np.int8, U.I16: np.int16, U.I32: np.int32}


def _operands(elem, m, k, n):
    dt = NPT[elem]
    a = U.corpus(4, U.CORPUS_I32_FULL, m * k).astype(dt, casting="unsafe")
    b = U.corpus(5, U.CORPUS_I32_FULL, k * n).astype(dt, casting="unsafe")
    return torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()


def _prior(out, m, n):
    w = 2 if out == U.I128 else 1
    p = U.corpus(3, U.CORPUS_I32_FULL, m * n * w).astype(np.int64)
    if out != U.I128:
        p = p.astype({U.I32: np.int32, U.I64: np.int64, U.I16: np.int16}[out], casting="unsafe")
    return torch.from_numpy(p).cuda()


@pytest.mark.parametrize("elem,out,shape,alpha,beta,mode", [
    (U.I32, U.I128, (64, 4096, 96), 1, 0, U.NEAREST),
    (U.I32, U.I64, (33, 1000, 17), -3, 2, U.SATURATING),
    (U.I16, U.I32, (40, 777, 50), 7, -1, U.WRAPPING),
    (U.I8, U.I32, (128, 300000, 8), 2**40, 1, U.NEAREST),
    (U.I32, U.I128, (5, 0, 7), 3, -1, U.NEAREST),
])
def test_ranges_summed_on_one_gpu_equal_the_whole(elem, out, shape, alpha, beta, mode):
    m, k, n = shape
    a, b = _operands(elem, m, k, n)
    prior = _prior(out, m, n)
    want = prior.clone()
    U.gemm(elem, out, a, (m, k, k, 1), b, (k, n, n, 1), want, (m, n, n, 1), alpha, beta, mode)
    for world in (1, 2, 3):
        total = torch.zeros(m * n * 3, dtype=torch.int64, device="cuda")
        for k0, k1 in D.k_ranges(k, world):
            limbs = torch.full((m * n * 3,), -7, dtype=torch.int64, device="cuda")
            U.gemm_partial_limbs(elem, a[k0:], (m, k1 - k0, k, 1), b[k0 * n:], (k1 - k0, n, n, 1),
                                 limbs)
            total += limbs
        got = prior.clone()
        U.limbs_finish(elem, out, total, got, (m, n, n, 1), alpha, beta, mode)
        assert torch.equal(got, want), (world, shape)


def _trop(salt, count, bits, lo=-64, hi=63):
    """Trop<E> values in [lo, hi], about 5 % the semiring zero (value 0), as bytes on the GPU."""
    from oracle import oracle as orc
    raw = U.corpus(salt, U.CORPUS_RAW, count)
    t = np.zeros(count, orc.TROP_DTYPES[bits])
    fin = (raw >> np.uint64(20)) % np.uint64(100) >= np.uint64(5)
    t["v"] = np.where(fin, (raw % np.uint64(hi - lo + 1)).astype(np.int64) + lo, 0)
    t["f"] = fin
    return t, torch.from_numpy(t.view(np.uint8).copy()).cuda()


@pytest.mark.parametrize("elem,out,shape,alpha,beta,mode", [
    (U.TROP_I8, U.TROP_I32, (64, 4096, 96), (0, True), (0, False), U.NEAREST),
    (U.TROP_I8, U.TROP_I8, (33, 1000, 17), (90, True), (-2, True), U.NEAREST),
    (U.TROP_I16, U.TROP_I16, (20, 300, 30), (2**14, True), (5, True), U.WRAPPING),
    (U.TROP_I32, U.TROP_I64, (9, 100, 11), (-7, True), (0, False), U.NEAREST),
    (U.TROP_I8, U.TROP_I32, (5, 0, 7), (3, True), (1, True), U.NEAREST),
])
def test_trop_ranges_maxed_on_one_gpu_equal_the_whole(elem, out, shape, alpha, beta, mode):
    """Trop<E> split-K: each range's keys, their element-wise max, MaxPlus and the encode
    once give the single call's bytes and the oracle's values."""
    from oracle import oracle as orc
    TD = orc.TROP_DTYPES
    bits = {U.TROP_I8: 8, U.TROP_I16: 16, U.TROP_I32: 32, U.TROP_I64: 64}
    m, k, n = shape
    eb, ob = bits[elem], bits[out]
    ah, a = _trop(31 + m, m * k, eb)
    bh, b = _trop(32 + n, k * n, eb)
    ph, prior = _trop(33, m * n, ob, -100, 100)
    want = prior.clone()
    U.gemm_tropical(elem, out, a, (m, k, k, 1), b, (k, n, n, 1), want, (m, n, n, 1), alpha, beta,
                    mode)
    ref = ph.copy()
    orc.gemm_trop(orc.View(ah, m, k, k, 1), orc.View(bh, k, n, n, 1), orc.View(ref, m, n, n, 1),
                  ebits=eb, obits=ob, alpha=alpha, beta=beta, mode=mode)
    w = want.cpu().numpy().view(TD[ob])
    assert np.array_equal(w["f"], ref["f"]) and np.array_equal(w["v"], ref["v"])
    esz = {8: 2, 16: 4, 32: 8}[eb]
    for world in (1, 2, 3):
        total = torch.full((m * n,), -(2**63), dtype=torch.int64, device="cuda")
        for k0, k1 in D.k_ranges(k, world):
            keys = torch.full((m * n,), 12345, dtype=torch.int64, device="cuda")
            U.trop_partial_keys(elem, a[k0 * esz:], (m, k1 - k0, k, 1), b[k0 * n * esz:],
                                (k1 - k0, n, n, 1), keys)
            total = torch.maximum(total, keys)
        got = prior.clone()
        U.trop_keys_finish(out, total, got, (m, n, n, 1), alpha, beta, mode)
        assert torch.equal(got, want), (world, shape)


def test_partial_limbs_validation():
    a, b = _operands(U.I32, 4, 8, 4)
    limbs = torch.zeros(4 * 4 * 3 - 1, dtype=torch.int64, device="cuda")
    with pytest.raises(U.DoesNotFit):
        U.gemm_partial_limbs(U.I32, a, (4, 8, 8, 1), b, (8, 4, 4, 1), limbs)
    limbs = torch.zeros(48, dtype=torch.int64, device="cuda")
    with pytest.raises(U.NotAProduct):
        U.gemm_partial_limbs(U.I32, a, (4, 8, 8, 1), b, (7, 4, 4, 1), limbs)
    with pytest.raises(U.UorError):
        U.gemm_partial_limbs(U.I64, a, (4, 8, 8, 1), b, (8, 4, 4, 1), limbs)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port):
    import datetime
    import torch.distributed as dist
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    try:
        ctx = U.Context(rank)
        m, k, n = 256, 65536, 128
        a, b = _operands(U.I32, m, k, n)
        prior = _prior(U.I128, m, n)
        got = prior.clone()
        D.splitk_gemm(U.I32, U.I128, a, (m, k, k, 1), b, (k, n, n, 1), got, (m, n, n, 1), 3, -1,
                      ctx=ctx)
        torch.cuda.synchronize()
        want = prior.clone()
        U.gemm(U.I32, U.I128, a, (m, k, k, 1), b, (k, n, n, 1), want, (m, n, n, 1), 3, -1,
               ctx=ctx)
        assert torch.equal(got, want), rank
        # column blocks with the gather
        c = torch.zeros(m * n, dtype=torch.int64, device="cuda")
        D.column_block_gemm(U.I32, U.I64, a, (m, k, k, 1), b, (k, n, n, 1), c, (m, n, n, 1),
                            ctx=ctx, gather=True)
        w2 = torch.zeros_like(c)
        U.gemm(U.I32, U.I64, a, (m, k, k, 1), b, (k, n, n, 1), w2, (m, n, n, 1), ctx=ctx)
        assert torch.equal(c, w2), rank
        # Trop<i8> split-K (all-reduce of MAX over keys) and column blocks
        ah, ta = _trop(41, m * k, 8)
        bh, tb = _trop(42, k * n, 8)
        tc = torch.zeros(m * n * 8, dtype=torch.uint8, device="cuda")
        D.splitk_gemm_tropical(U.TROP_I8, U.TROP_I32, ta, (m, k, k, 1), tb, (k, n, n, 1), tc,
                               (m, n, n, 1), (3, True), ctx=ctx)
        torch.cuda.synchronize()
        tw = torch.zeros_like(tc)
        U.gemm_tropical(U.TROP_I8, U.TROP_I32, ta, (m, k, k, 1), tb, (k, n, n, 1), tw,
                        (m, n, n, 1), (3, True), ctx=ctx)
        assert torch.equal(tc, tw), rank
        tc.zero_()
        D.column_block_gemm_tropical(U.TROP_I8, U.TROP_I32, ta, (m, k, k, 1), tb, (k, n, n, 1),
                                     tc, (m, n, n, 1), (3, True), ctx=ctx, gather=True)
        assert torch.equal(tc, tw), rank
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_nccl_ranks_match_one_device():
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)


def _abi_worker(rank, world, port):
    """The C ABI's collective entries: a communicator made with uor_b200_nccl_comm_init
    (the id passed through a TCP store), each rank its own range of the reduction, every
    rank's C equal to the single-device call's bytes."""
    import datetime
    import torch.distributed as dist
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=60))
    if rank == 0:
        store.set("uid", U.nccl_unique_id())
    uid = store.get("uid")
    ctx = U.Context(rank)
    comm = U.NcclComm(world, uid, rank, ctx)
    try:
        for elem, out, (m, k, n), alpha, beta, mode in [
                (U.I32, U.I128, (256, 65536, 128), 3, -1, U.NEAREST),
                (U.I8, U.I32, (130, 5000, 70), -2, 1, U.SATURATING),
                (U.I16, U.I64, (64, 777, 96), 1, 0, U.WRAPPING)]:
            a, b = _operands(elem, m, k, n)
            prior = _prior(out, m, n)
            want = prior.clone()
            U.gemm(elem, out, a, (m, k, k, 1), b, (k, n, n, 1), want, (m, n, n, 1), alpha, beta,
                   mode, ctx=ctx)
            k0, k1 = D.k_ranges(k, world)[rank]
            got = prior.clone()
            route = U.Route()
            U.gemm_splitk_nccl(comm, elem, out, a[k0:], (m, k1 - k0, k, 1), b[k0 * n:],
                               (k1 - k0, n, n, 1), got, (m, n, n, 1), alpha, beta, mode, ctx=ctx,
                               route=route)
            assert torch.equal(got, want), (rank, elem, out)
            assert route.kernel != 0
            # asynchronous: returns at once, the context's sync reports the status
            got = prior.clone()
            U.gemm_splitk_nccl(comm, elem, out, a[k0:], (m, k1 - k0, k, 1), b[k0 * n:],
                               (k1 - k0, n, n, 1), got, (m, n, n, 1), alpha, beta, mode, ctx=ctx,
                               asynchronous=True)
            ctx.sync()
            assert torch.equal(got, want), (rank, elem, out, "async")
        m, k, n = 96, 4000, 80
        ah, ta = _trop(43, m * k, 8)
        bh, tb = _trop(44, k * n, 8)
        ph, prior = _trop(45, m * n, 32, -100, 100)
        want = prior.clone()
        U.gemm_tropical(U.TROP_I8, U.TROP_I32, ta, (m, k, k, 1), tb, (k, n, n, 1), want,
                        (m, n, n, 1), (3, True), (-5, True), ctx=ctx)
        k0, k1 = D.k_ranges(k, world)[rank]
        got = prior.clone()
        U.gemm_tropical_splitk_nccl(comm, U.TROP_I8, U.TROP_I32, ta[2 * k0:], (m, k1 - k0, k, 1),
                                    tb[2 * k0 * n:], (k1 - k0, n, n, 1), got, (m, n, n, 1),
                                    (3, True), (-5, True), ctx=ctx)
        assert torch.equal(got, want), rank
        # a partial that fails on one rank only (its A one column short of B's rows): that
        # rank still joins the exchange and reports its own status, the other learns of it
        m2, k2, n2 = 16, 64, 24
        a2, b2 = _operands(U.I32, m2, k2, n2)
        c2 = torch.zeros(m2 * n2 * 2, dtype=torch.int64, device="cuda")
        kk = k2 - 1 if rank == 1 else k2
        with pytest.raises(U.UorError) as exc:
            U.gemm_splitk_nccl(comm, U.I32, U.I128, a2, (m2, kk, k2, 1), b2, (k2, n2, n2, 1), c2,
                               (m2, n2, n2, 1), ctx=ctx)
        assert exc.value.status == (U.NONCONFORMANT if rank == 1 else U.NCCL_ERROR), rank
        # and the communicator still serves the next call on both ranks
        got = prior.clone()
        U.gemm_tropical_splitk_nccl(comm, U.TROP_I8, U.TROP_I32, ta[2 * k0:], (m, k1 - k0, k, 1),
                                    tb[2 * k0 * n:], (k1 - k0, n, n, 1), got, (m, n, n, 1),
                                    (3, True), (-5, True), ctx=ctx)
        assert torch.equal(got, want), rank
        # a communicator of another device is refused before any work
        with pytest.raises(U.UorError):
            other = U.Context(1 - rank)
            try:
                U.gemm_splitk_nccl(comm, U.I8, U.I32, a, (4, 4, k, 1), b, (4, 4, n, 1), got,
                                   (4, 4, n, 1), ctx=other)
            finally:
                other.close()
    finally:
        comm.destroy()
        ctx.close()


@pytest.mark.skipif(not torch or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_through_the_c_abi_nccl_entries():
    import torch.multiprocessing as mp
    mp.spawn(_abi_worker, args=(2, _free_port()), nprocs=2, join=True)
