"""Calls from two contexts on two streams and two host threads run one after another
on the GPU (the library's device-wide order), and each gives the oracle's bytes.

Only K1 products run here: two K1 CTAs never fit on one SM (each takes more than half of
its shared memory), so even without the order they could not share an SM's tensor
memory; the test observes the order through the calls' completion times."""
import threading

import numpy as np
import pytest

import uor_b200 as U
from oracle import oracle as orc
from gpu_util import needs_gpu, torch

pytestmark = [pytest.mark.gpu, needs_gpu]


def test_two_contexts_on_two_streams_do_not_overlap():
    m = k = n = 4096
    a = U.corpus(61, U.CORPUS_I8, m * k)
    b = U.corpus(62, U.CORPUS_I8, k * n)
    ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    want = np.zeros(m * n, np.int32)
    orc.gemm_i8_blocked(a, b, want, m, k, n)
    ctxs = [U.Context(0), U.Context(0)]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [torch.zeros(m * n, dtype=torch.int32, device="cuda") for _ in range(2)]
    for c, s in zip(ctxs, streams):
        c.set_stream(s.cuda_stream)
    # one solo call to know a call's device time
    base = torch.cuda.Event(enable_timing=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(2):
        e0.record(streams[0])
        U.gemm_i8_i32(m, k, n, ta, tb, outs[0], ctx=ctxs[0], asynchronous=True)
        e1.record(streams[0])
    torch.cuda.synchronize()
    solo = e0.elapsed_time(e1)
    ends = {0: [], 1: []}
    base.record(torch.cuda.current_stream())
    torch.cuda.synchronize()

    def issue(i):
        for _ in range(6):
            U.gemm_i8_i32(m, k, n, ta, tb, outs[i], ctx=ctxs[i], asynchronous=True)
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(streams[i])
            ends[i].append(ev)
    threads = [threading.Thread(target=issue, args=(i,)) for i in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    torch.cuda.synchronize()
    times = sorted(base.elapsed_time(ev) for i in (0, 1) for ev in ends[i])
    gaps = np.diff(times)
    # one call at a time: completions at least most of a solo call apart
    assert gaps.min() > 0.6 * solo, (solo, gaps.tolist())
    for i in (0, 1):
        assert np.array_equal(outs[i].cpu().numpy(), want)
        assert ctxs[i].sync() == 0
        ctxs[i].close()
