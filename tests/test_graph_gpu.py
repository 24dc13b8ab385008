"""CUDA graph capture of asynchronous device-pointer calls, as the header promises for the
i8, narrow-side, wide-integer (byte-slice and modular routes, the latter with its side
stream and its reduction chunks) and tropical paths: a call captured on the context's
stream after one eager call of the same shape, replayed after the inputs change in place,
writes the bytes an eager call writes."""
import numpy as np
import pytest

import uor_b200 as U
from gpu_util import needs_gpu, torch

pytestmark = [pytest.mark.gpu, needs_gpu]


def _replayed_equals_eager(make_inputs, call, out_like):
    """Capture call(ins, out) once, refill the inputs, replay, and compare with an eager call
    on the new inputs."""
    s = torch.cuda.Stream()
    ctx = U.Context(0)
    ctx.set_stream(s.cuda_stream)
    try:
        ins = make_inputs(1)
        out = out_like()
        with torch.cuda.stream(s):
            call(ctx, ins, out)  # eager: grows the context's buffers to this shape
            assert ctx.sync() == 0
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                call(ctx, ins, out)
        for t, new in zip(ins, make_inputs(2)):
            t.copy_(new)
        out.zero_()
        g.replay()
        s.synchronize()
        want = out_like()
        with torch.cuda.stream(s):
            call(ctx, ins, want)
        assert ctx.sync() == 0
        assert torch.equal(out, want)
        del g
    finally:
        ctx.close()


def _ints(salt, count, dt, kind=U.CORPUS_I32_FULL):
    return torch.from_numpy(U.corpus(salt, kind, count).astype(dt, casting="unsafe")).cuda()


@pytest.mark.parametrize("m,k,n", [(1024, 1024, 512), (8, 4096, 640)])
def test_i8_and_narrow_side_replay(m, k, n):
    def ins(v):
        return [_ints(10 * v, m * k, np.int8, U.CORPUS_I8), _ints(10 * v + 1, k * n, np.int8, U.CORPUS_I8)]

    def call(ctx, x, c):
        U.gemm(U.I8, U.I32, x[0], (m, k, k, 1), x[1], (k, n, n, 1), c, (m, n, n, 1), 3, 0,
               ctx=ctx, asynchronous=True)
    _replayed_equals_eager(ins, call, lambda: torch.zeros(m * n, dtype=torch.int32, device="cuda"))


@pytest.mark.parametrize("modular", [True, False])
def test_wide_integer_replay(modular):
    m, k, n = 256, 20000, 256

    def ins(v):
        return [_ints(10 * v + 2, m * k, np.int32), _ints(10 * v + 3, k * n, np.int32)]

    def call(ctx, x, c):
        route = U.Route()
        U.gemm(U.I32, U.I128, x[0], (m, k, k, 1), x[1], (k, n, n, 1), c, (m, n, n, 1), ctx=ctx,
               route=route, asynchronous=True, modular=modular, digits=not modular)
        assert (route.moduli > 0) == modular
    _replayed_equals_eager(ins, call, lambda: torch.zeros(m * n * 2, dtype=torch.int64, device="cuda"))


def test_tropical_replay():
    m, k, n = 300, 2000, 260

    def ins(v):
        raw = U.corpus(10 * v + 4, U.CORPUS_RAW, m * k + k * n)
        vals = ((raw % np.uint64(128)).astype(np.int64) - 64).astype(np.int8)
        fin = ((raw >> np.uint64(20)) % np.uint64(100) >= np.uint64(5)).astype(np.int8)
        t = np.stack([np.where(fin == 1, vals, 0), fin], axis=1).astype(np.int8).reshape(-1)
        tt = torch.from_numpy(t.view(np.uint8).copy()).cuda()
        return [tt[:2 * m * k].clone(), tt[2 * m * k:].clone()]

    def call(ctx, x, c):
        U.gemm_tropical(U.TROP_I8, U.TROP_I32, x[0], (m, k, k, 1), x[1], (k, n, n, 1), c,
                        (m, n, n, 1), (2, True), ctx=ctx, asynchronous=True)
    _replayed_equals_eager(ins, call, lambda: torch.zeros(m * n * 8, dtype=torch.uint8, device="cuda"))
