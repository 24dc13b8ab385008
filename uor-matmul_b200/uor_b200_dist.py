"""uor_b200_dist -- the exact GEMM across devices, one process per GPU.

Two decompositions, both exact by construction:

* Column blocks (``column_block_gemm``): the reference's ``Partition`` of C into
  independent tiles (crates/uor-matmul-gemm/src/partition.rs:34-111), one tile of
  whole columns per rank. Every output element is one exact sum computed on one
  device, so there is no exchange on the data path; ``gather=True`` then shares the
  blocks (an all-gather of finished bytes, outside the arithmetic).
* Tropical (``column_block_gemm_tropical``, ``splitk_gemm_tropical``): the same two
  decompositions of driver::gemm over Trop<E> (driver.rs:67-182). Split-K exchanges
  each range's (max, +) reduction as int64 keys with one all-reduce of MAX (max is
  associative and commutative, so the union of ranges is their maximum) and applies
  MaxPlus and the encode once (uor_b200_trop_keys_finish).
* Split-K (``splitk_gemm``): each rank takes a contiguous range of the reduction,
  computes its exact partial sum as radix-2^40 int64 limbs (uor_b200_gemm_partial_limbs),
  the limbs are summed across ranks with one all-reduce, and every rank encodes the
  total once (uor_b200_limbs_finish) -- the reference's exact chunk fold
  (run_chunked_depth, kernel.rs:1431) with the chunks on different devices.

torch.distributed carries the exchange (NCCL on GPUs). All arithmetic runs in the
CUDA library through its C ABI; the ``partial``/``finish`` hooks exist so that the
host protocol can be exercised by CPU tests with stand-ins.
"""
from __future__ import annotations

from typing import Callable, NamedTuple

import uor_b200 as U


class Tile(NamedTuple):
    """One independently computable region of C (partition.rs:17-27)."""
    row: int
    col: int
    rows: int
    cols: int


class Partition:
    """C's shape cut into tiles of at most tile_rows x tile_cols (partition.rs:33-99).

    A zero tile dimension means the whole extent; tiles are numbered row-major over
    the tile grid, and ``tile(i)`` is None past the end."""

    def __init__(self, m: int, n: int, tile_rows: int = 0, tile_cols: int = 0):
        self.m, self.n = m, n
        self.tile_rows = tile_rows if tile_rows else max(m, 1)
        self.tile_cols = tile_cols if tile_cols else max(n, 1)

    def _rows_of_tiles(self):
        return -(-self.m // self.tile_rows)

    def _cols_of_tiles(self):
        return -(-self.n // self.tile_cols)

    def __len__(self):
        return self._rows_of_tiles() * self._cols_of_tiles()

    def tile(self, idx: int) -> Tile | None:
        if idx >= len(self):
            return None
        cot = self._cols_of_tiles()
        ti, tj = divmod(idx, cot)
        row, col = ti * self.tile_rows, tj * self.tile_cols
        return Tile(row, col, min(self.tile_rows, self.m - row), min(self.tile_cols, self.n - col))

    def __iter__(self):
        for i in range(len(self)):
            yield self.tile(i)


def column_blocks(m: int, n: int, world: int) -> Partition:
    """Whole-column tiles, one per rank (the last may be narrower; a rank past the end
    has none)."""
    return Partition(m, n, 0, -(-n // max(world, 1)) if n else 0)


def k_ranges(k: int, world: int, align: int = 128) -> list[tuple[int, int]]:
    """Contiguous reduction ranges, one per rank, in multiples of `align` where
    possible (whole tensor-core k-steps); trailing ranks may be empty."""
    if world <= 1:
        return [(0, k)]
    step = -(-k // world)
    step = -(-step // align) * align if k >= world * align else step
    out = []
    for r in range(world):
        k0 = min(r * step, k)
        out.append((k0, min(k0 + step, k)))
    return out


def _rank_world(group):
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def _nonneg(v):
    rows, cols, rs, cs = v
    if rs < 0 or cs < 0:
        raise ValueError("split views need non-negative strides")


def column_block_gemm(elem, out, a, av, b, bv, c, cv, alpha=1, beta=0, encode=U.NEAREST,
                      ctx=None, group=None, gather=False, gemm: Callable | None = None):
    """This rank's column block of C := encode(alpha A B + beta C).

    a, b, c are flat device tensors holding the full views av, bv, cv (tuples
    (rows, cols, rs, cs), non-negative strides). The rank writes only its block of C;
    with gather=True (C row-major and contiguous) every rank receives all blocks."""
    import torch
    import torch.distributed as dist
    rank, world = _rank_world(group)
    m, k = av[0], av[1]
    n = bv[1]
    for v in (av, bv, cv):
        _nonneg(v)
    t = column_blocks(m, n, world).tile(rank)
    ob = U.DTYPE_SIZE[out]
    per_b = U.DTYPE_SIZE[elem] // b.element_size()  # buffer entries per element
    per_c = ob // c.element_size()
    if t is not None and t.cols and m:
        b_off = t.col * bv[3] * per_b
        c_off = t.col * cv[3] * per_c
        (gemm or U.gemm)(elem, out, a, av, b[b_off:], (k, t.cols, bv[2], bv[3]), c[c_off:],
                         (m, t.cols, cv[2], cv[3]), alpha, beta, encode, ctx=ctx)
    if not gather or world == 1:
        return t
    if cv[3] != 1 or cv[2] != n:
        raise ValueError("gather needs a contiguous row-major C")
    part = column_blocks(m, n, world)
    width = part.tile_cols * ob
    cm = c.view(-1).view(torch.uint8)[: m * n * ob].view(m, n * ob)
    mine = torch.zeros(m, width, dtype=torch.uint8, device=c.device)
    if t is not None:
        mine[:, : t.cols * ob] = cm[:, t.col * ob: (t.col + t.cols) * ob]
    blocks = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(blocks, mine, group=group)
    for r, blk in enumerate(blocks):
        tr = part.tile(r)
        if tr is not None and r != rank:
            cm[:, tr.col * ob: (tr.col + tr.cols) * ob] = blk[:, : tr.cols * ob]
    return t


def splitk_gemm(elem, out, a, av, b, bv, c, cv, alpha=1, beta=0, encode=U.NEAREST, ctx=None,
                group=None, partial: Callable | None = None, finish: Callable | None = None):
    """C := encode(alpha A B + beta C) with the reduction split across ranks.

    Every rank passes the same full views (flat tensors on its own device, non-negative
    strides) and the same C prior; every rank ends with the same bytes of C, equal to
    the single-device call's. ctx is bound to torch's current stream, on which the
    all-reduce runs; the call returns with the work queued (ctx.sync() or a stream
    synchronize collects it). elem in {I8, I16, I32}."""
    import torch
    import torch.distributed as dist
    rank, world = _rank_world(group)
    m, k = av[0], av[1]
    n = bv[1]
    for v in (av, bv):
        _nonneg(v)
    partial = partial or U.gemm_partial_limbs
    finish = finish or U.limbs_finish
    if ctx is not None and a.is_cuda:
        ctx.set_stream(torch.cuda.current_stream(a.device).cuda_stream)
    k0, k1 = k_ranges(k, world)[rank]
    per_a = U.DTYPE_SIZE[elem] // a.element_size()
    per_b = U.DTYPE_SIZE[elem] // b.element_size()
    limbs = torch.zeros(m * n * U.SPLITK_LIMBS, dtype=torch.int64, device=a.device)
    if m and n:
        # Stream-ordered throughout: the partial, the all-reduce and the finish queue on
        # one stream without a host round trip between them.
        partial(elem, a[k0 * av[3] * per_a:], (m, k1 - k0, av[2], av[3]), b[k0 * bv[2] * per_b:],
                (k1 - k0, n, bv[2], bv[3]), limbs, ctx=ctx, asynchronous=True)
        if world > 1:
            dist.all_reduce(limbs, op=dist.ReduceOp.SUM, group=group)
        finish(elem, out, limbs, c, cv, alpha, beta, encode, ctx=ctx, asynchronous=True)
    return (k0, k1)


def column_block_gemm_tropical(elem, out, a, av, b, bv, c, cv, alpha=(0, True), beta=(0, False),
                               encode=U.NEAREST, ctx=None, group=None, gather=False,
                               gemm: Callable | None = None):
    """This rank's column block of driver::gemm over Trop<E> with MaxPlus{alpha, beta}
    (scalars are (value, finite) pairs); a, b, c are byte tensors of Trop<E> / Trop<O>
    structs holding the full views. As column_block_gemm, gather=True shares the blocks."""
    return column_block_gemm(elem, out, a, av, b, bv, c, cv, alpha, beta, encode, ctx=ctx,
                             group=group, gather=gather, gemm=gemm or U.gemm_tropical)


def splitk_gemm_tropical(elem, out, a, av, b, bv, c, cv, alpha=(0, True), beta=(0, False),
                         encode=U.NEAREST, ctx=None, group=None, partial: Callable | None = None,
                         finish: Callable | None = None):
    """driver::gemm over Trop<E> with the reduction split across ranks: every rank's range
    reduced to int64 keys, one all-reduce of MAX, MaxPlus and the encode on every rank.
    Every rank passes the same full views and C prior and ends with the single-device
    call's bytes. elem in {TROP_I8, TROP_I16, TROP_I32}; queued on torch's current stream."""
    import torch
    import torch.distributed as dist
    rank, world = _rank_world(group)
    m, k = av[0], av[1]
    n = bv[1]
    for v in (av, bv):
        _nonneg(v)
    partial = partial or U.trop_partial_keys
    finish = finish or U.trop_keys_finish
    if ctx is not None and a.is_cuda:
        ctx.set_stream(torch.cuda.current_stream(a.device).cuda_stream)
    k0, k1 = k_ranges(k, world)[rank]
    per_a = U.DTYPE_SIZE[elem] // a.element_size()
    per_b = U.DTYPE_SIZE[elem] // b.element_size()
    keys = torch.empty(m * n, dtype=torch.int64, device=a.device)
    if m and n:
        partial(elem, a[k0 * av[3] * per_a:], (m, k1 - k0, av[2], av[3]), b[k0 * bv[2] * per_b:],
                (k1 - k0, n, bv[2], bv[3]), keys, ctx=ctx, asynchronous=True)
        if world > 1:
            dist.all_reduce(keys, op=dist.ReduceOp.MAX, group=group)
        finish(out, keys, c, cv, alpha, beta, encode, ctx=ctx, asynchronous=True)
    return (k0, k1)


class HostStaging:
    """Device buffers (and a copy-out stream) that ``replicated_gemm_i8_host`` stages
    host operands through; allocate once and reuse across calls."""

    def __init__(self, a_bytes: int, b_bytes: int, c_bytes: int):
        import torch
        dev = torch.device("cuda", torch.cuda.current_device())
        self.a = torch.empty(a_bytes, dtype=torch.uint8, device=dev)
        self.b = torch.empty(b_bytes, dtype=torch.uint8, device=dev)
        self.c = torch.empty(c_bytes, dtype=torch.uint8, device=dev)
        self.out_stream = torch.cuda.Stream(dev)


def replicated_gemm_i8_host(m, k, n, a_host, b_host, c_host, work: HostStaging, ctx=None,
                            group=None, root=0, row_blocks=4):
    """C_r := A B_r (slice::gemm::<i8, i32>, row-major) on every rank from pinned HOST
    buffers, with A shared: the root uploads A once and it is broadcast over NCCL to
    every rank, instead of one host upload per GPU; each rank uploads its own B block
    and reads back its own C block (the column-block Partition, partition.rs:34).

    The product runs in row blocks of A: block i's upload and broadcast, its GEMM and
    its C copy-out queue behind one another, and block i's copy-out overlaps block
    i + 1's upload and GEMM. a_host is read on the root only (None elsewhere). Returns
    when c_host holds the result."""
    import torch
    import torch.distributed as dist
    rank, world = _rank_world(group)
    if m == 0 or n == 0:
        return
    stream = torch.cuda.current_stream()
    if ctx is not None:
        ctx.set_stream(stream.cuda_stream)
    a_all = work.a[: m * k].view(torch.int8)
    b = work.b[: k * n].view(torch.int8)
    c_all = work.c[: 4 * m * n].view(torch.int32)
    b.copy_(b_host.view(torch.int8)[: k * n], non_blocking=True)
    src = dist.get_global_rank(group, root) if (world > 1 and group is not None) else root
    step = -(-m // max(1, row_blocks))
    for i0 in range(0, m, step):
        rows = min(step, m - i0)
        a = a_all[i0 * k: (i0 + rows) * k]
        if rank == root and k:
            a.copy_(a_host.view(torch.int8)[i0 * k: (i0 + rows) * k], non_blocking=True)
        if world > 1 and k:
            dist.broadcast(a, src=src, group=group)
        c = c_all[i0 * n: (i0 + rows) * n]
        U.gemm_i8_i32(rows, k, n, a, b, c, ctx=ctx, asynchronous=True)
        done = torch.cuda.Event()
        done.record(stream)
        work.out_stream.wait_event(done)
        with torch.cuda.stream(work.out_stream):
            c_host.view(torch.int32)[i0 * n: (i0 + rows) * n].copy_(c, non_blocking=True)
    stream.wait_stream(work.out_stream)
    stream.synchronize()


def bind_to_local_cpus(device: int) -> int:
    """Restrict this process to the host cores NVML reports as closest to `device`
    (its NUMA node), so pinned host buffers it allocates afterwards sit in memory
    local to the GPU's PCIe root. Returns the number of cores kept (0: unchanged)."""
    import os
    try:
        import pynvml
        import torch
        p = torch.cuda.get_device_properties(device)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        words = pynvml.nvmlDeviceGetCpuAffinity(h, 16)
    except Exception:
        return 0
    cpus = {64 * w + b for w, word in enumerate(words) for b in range(64) if (word >> b) & 1}
    cpus &= set(os.sched_getaffinity(0))
    if not cpus:
        return 0
    os.sched_setaffinity(0, cpus)
    return len(cpus)
