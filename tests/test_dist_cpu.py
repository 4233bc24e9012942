"""Host logic of the M-row sharding on CPU: two gloo ranks, the per-shard
compute stood in by a float64 CPU product (no GPU, no kernels here)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from zengpu_b200.dist import ShardedGemm, chunk_range, row_range


@pytest.mark.parametrize("m,world", [(10, 3), (32768, 8), (7, 8), (0, 2), (8192, 1)])
def test_row_range_partitions(m, world):
    spans = [row_range(m, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == m
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("n,world", [(1 << 28, 8), (1001, 3), (3, 4), (65536, 2)])
def test_chunk_range_alignment(n, world):
    spans = [chunk_range(n, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0 and b0 % 4 == 0 or b0 == n


def _cpu_compute(a, b, alpha, bias, relu, mode, out):
    c = alpha * (a.double() @ b.double())
    if bias is not None:
        c = c + bias.double()
    if relu:
        c = torch.clamp_min(c, 0.0)
    return c.float()


def _worker(rank, world, port, m, n, k, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        a = torch.rand((m, k), generator=g) * 2 - 1
        b_full = torch.rand((k, n), generator=g) * 2 - 1
        # only rank 0 holds the real B; the others must receive it
        b = b_full.clone() if rank == 0 else torch.zeros_like(b_full)
        sg = ShardedGemm(mode=1, compute=_cpu_compute)
        r0, r1 = row_range(m, world, rank)
        c_rows = sg.sgemm_rows(a[r0:r1].contiguous(), b, src=0, alpha=0.5)
        c = sg.gather_rows(c_rows, m)
        ref = 0.5 * (a.double() @ b_full.double())
        q.put((rank, float((c.double() - ref).abs().max())))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_broadcast_and_gather():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, 37, 19, 23, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err in results:
        assert err < 1e-5, (rank, err)


class _CpuOps:
    """Stand-in for pack_a / pack_b / sgemm_packed on CPU tensors (float64
    product): exercises the panel bookkeeping and broadcast order only."""

    class P:
        def __init__(self, t):
            self.t = t.clone()
            self.buf = self.t

    def pack_a(self, a, mode, out=None):
        return self.P(a)

    def pack_b(self, b, mode, out=None):
        return self.P(b)

    def sgemm_packed(self, pa, pb, c, alpha=1.0, bias=None, relu=False):
        r = alpha * (pa.t.double() @ pb.t.double())
        if bias is not None:
            r = r + bias.double()
        if relu:
            r = torch.clamp_min(r, 0.0)
        c.copy_(r.float())
        return c


def _worker_pipelined(rank, world, port, m, n, k, panels, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(1)
        a = torch.rand((m, k), generator=g) * 2 - 1
        b_full = torch.rand((k, n), generator=g) * 2 - 1
        bias = torch.rand(n, generator=g) - 0.5
        b = b_full.clone() if rank == 1 else torch.zeros_like(b_full)
        sg = ShardedGemm(mode=1, ops=_CpuOps())
        r0, r1 = row_range(m, world, rank)
        c = sg.sgemm_rows_pipelined(a[r0:r1].contiguous(), b, src=1, panels=panels, alpha=2.0,
                                    bias=bias, relu=True)
        ref = torch.clamp_min(2.0 * (a[r0:r1].double() @ b_full.double()) + bias.double(), 0)
        q.put((rank, float((c.double() - ref).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("panels", [1, 3, 5])
def test_two_rank_pipelined_panels(panels):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_pipelined, args=(r, 2, port, 21, 37, 13, panels, q))
             for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err in results:
        assert err < 1e-5, (rank, err)


def test_panel_count():
    from zengpu_b200.dist import panel_count
    assert panel_count(8192, 8192) == 2      # 2 panels of 1024 tiles each
    assert panel_count(4096, 32768) == 4
    assert panel_count(1024, 8192) == 1      # too small to split
    assert panel_count(32768, 32768) == 8


# ---- chained copy-engine broadcast: host-side protocol ------------------------------
from zengpu_b200.dist import ChainedGemm, chain_neighbours, default_chunk_cols  # noqa: E402


@pytest.mark.parametrize("world,src", [(1, 0), (2, 0), (8, 0), (8, 3), (3, 2)])
def test_chain_neighbours_form_one_chain(world, src):
    order = [src]
    while True:
        _, nxt = chain_neighbours(order[-1], world, src)
        if nxt is None:
            break
        order.append(nxt)
    assert sorted(order) == list(range(world))
    for i, r in enumerate(order):
        prev, nxt = chain_neighbours(r, world, src)
        assert prev == (order[i - 1] if i > 0 else None)
        assert nxt == (order[i + 1] if i + 1 < world else None)


def test_default_chunk_cols():
    assert default_chunk_cols(8192, 8192) == 256          # 16 MiB packed at k = 8192
    assert default_chunk_cols(32768, 1024) == 2048
    assert default_chunk_cols(300, 16) == 512             # never more than n rounded to 256
    for n, k in [(8192, 8192), (32768, 8192), (1000, 77)]:
        assert default_chunk_cols(n, k) % 256 == 0


class _FakeStream:
    cuda_stream = 0

    def __init__(self, log=None, name="copy"):
        self.log, self.name = log, name

    def wait_stream(self, other):
        if self.log is not None:
            self.log.append(("wait_stream", other.name))


class _FakeBuf:
    def data_ptr(self):
        return 0x2000


class _FakePacked:
    buf = _FakeBuf()


class _FakeOps:
    def __init__(self, log):
        self.log = log

    def pack_a(self, a, mode, out=None):
        self.log.append(("pack_a", tuple(a.shape)))
        return _FakePacked()


class _FakeChainLib:
    """Records the C calls of one rank; the IPC handle is the rank number."""

    def __init__(self, rank, log):
        self.rank, self.log = rank, log

    def zg_bchain_create(self, mode, k, n, chunk, out, handle):
        out._obj.value = 0x1000 + self.rank
        for i in range(64):
            handle[i] = self.rank
        self.log.append(("create", mode, k, n, chunk))
        return 0

    def zg_bchain_connect(self, chain, prev, nxt):
        self.log.append(("connect", None if prev is None else prev[0],
                         None if nxt is None else nxt[0]))
        return 0

    def zg_bchain_source(self, chain, epoch, b, ldb, stream):
        self.log.append(("source", epoch))
        return 0

    def zg_bchain_forward(self, chain, epoch, stream):
        self.log.append(("forward", epoch))
        return 0

    def zg_bchain_gemm(self, chain, epoch, gated, m, alpha, pa, c, ldc, bias, relu, stream):
        self.log.append(("gemm", epoch, gated, m))
        return 0

    def zg_bchain_release(self, chain, epoch, stream):
        self.log.append(("release", epoch))
        return 0

    def zg_bchain_destroy(self, chain):
        self.log.append(("destroy",))
        return 0


def _worker_chain(rank, world, port, src, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        log = []
        torch.cuda.current_stream = lambda: _FakeStream(log, "compute")
        cg = ChainedGemm(k=64, n=512, mode=3, src=src, chunk_cols=256,
                         lib=_FakeChainLib(rank, log), ops=_FakeOps(log))
        cg.copy_stream = _FakeStream(log, "copy")
        a = torch.zeros((10, 64))
        b = torch.zeros((64, 512)) if rank == src else None
        out = torch.zeros((10, 512))
        for _ in range(3):
            cg.step(a, b, out)
        cg.close()
        q.put((rank, log))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,src", [(3, 0), (3, 1)])
def test_chained_gemm_call_protocol(world, src):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_chain, args=(r, world, port, src, q))
             for r in range(world)]
    for p in procs:
        p.start()
    logs = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, log in logs.items():
        prev, nxt = chain_neighbours(rank, world, src)
        assert log[0] == ("create", 3, 64, 512, 256)
        assert log[1] == ("connect", prev, nxt)   # neighbours' handles, by rank
        steps = log[2:-1]
        assert log[-1] == ("destroy",)
        per_step = 6 if rank == src else 5
        assert len(steps) == 3 * per_step
        for i in range(3):
            e = i + 1
            s = steps[i * per_step:(i + 1) * per_step]
            expect = ([("source", e)] if rank == src else []) + [
                ("forward", e), ("pack_a", (10, 64)), ("gemm", e, 0 if rank == src else 1, 10),
                ("wait_stream", "copy"), ("release", e)]
            assert s == expect


def _worker_chain_mismatch(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        log = []
        try:
            ChainedGemm(k=64, n=512 + 256 * rank, mode=3, chunk_cols=256,
                        lib=_FakeChainLib(rank, log), ops=_FakeOps(log))
            q.put((rank, "no error"))
        except ValueError as e:
            q.put((rank, "disagree" in str(e) and ("destroy",) in log))
    finally:
        dist.destroy_process_group()


def test_chained_gemm_rejects_mismatched_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_chain_mismatch, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}
