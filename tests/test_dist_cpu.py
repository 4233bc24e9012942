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
from zengpu_b200.dist import (  # noqa: E402
    ChainBroken, ChainedGemm, ChainGuard, chain_neighbours, default_chunk_cols, pid_alive)


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


class _FakeEvent:
    """Completion marker of one step: steps recorded while `complete_new` is
    set complete at once, the others only once an abort released them."""
    complete_new = True
    released = False

    def __init__(self):
        self.complete = _FakeEvent.complete_new

    def record(self, stream):
        pass

    def query(self):
        return self.complete or _FakeEvent.released


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

    def zg_bchain_abort(self, chain, epoch):
        self.log.append(("abort", epoch))
        _FakeEvent.released = True  # the aborted steps drain
        return 0

    def zg_kernel_status(self, code):
        self.log.append(("status",))
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
        cg._new_event = _FakeEvent
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


# ---- failure detection of the chain (host side, no GPU) -----------------------------
class _Ev:
    def __init__(self, done):
        self.done = done

    def query(self):
        return self.done


def test_chain_guard_deadline_and_pruning():
    g = ChainGuard(0, [11, 22], None, 1, deadline_s=0.2, alive=lambda pid: True)
    g.wait(5)  # never launched: nothing to wait for
    g.launched(1, _Ev(True))
    g.launched(2, _Ev(False))
    g.launched(3, _Ev(True))
    assert sorted(g.events) == [2, 3]  # only the last two steps are kept
    assert g.in_flight()
    g.wait(3)
    import time as _t
    t0 = _t.monotonic()
    with pytest.raises(ChainBroken, match="step 2 did not complete within 0.2 s"):
        g.wait(2)
    assert _t.monotonic() - t0 < 2.0


def test_chain_guard_neighbours():
    alive = {11: True, 22: True, 33: True}
    g = ChainGuard(1, [11, 22, 33], 0, 2, alive=lambda pid: alive[pid])
    g.check_neighbours()
    alive[33] = False
    assert g.gone_neighbours() == [2]
    with pytest.raises(ChainBroken, match="neighbour rank 2 \\(pid 33\\) has exited"):
        g.check_neighbours()


def test_pid_alive_sees_exit_and_zombies():
    import subprocess
    p = subprocess.Popen(["sleep", "30"])
    try:
        assert pid_alive(p.pid)
        p.kill()
        import time as _t
        _t.sleep(0.2)  # killed, not yet reaped: a zombie counts as exited
        assert not pid_alive(p.pid)
    finally:
        p.wait()
    assert not pid_alive(p.pid)
    assert pid_alive(os.getpid())


def _worker_chain_leave(rank, world, port, mode, q):
    """Two ranks run two steps; then rank 1 leaves (its process exits) or stops
    taking part (stays alive, steps no more).  Rank 0's next step must raise
    ChainBroken, and so must every step after it."""
    import time as _t
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    log = []
    torch.cuda.current_stream = lambda: _FakeStream(log, "compute")
    cg = ChainedGemm(k=64, n=512, mode=3, src=0, chunk_cols=256, deadline_s=0.5,
                     lib=_FakeChainLib(rank, log), ops=_FakeOps(log))
    cg.copy_stream = _FakeStream(log, "copy")
    cg._new_event = _FakeEvent
    a = torch.zeros((10, 64))
    b = torch.zeros((64, 512)) if rank == 0 else None
    out = torch.zeros((10, 512))
    for _ in range(2):
        cg.step(a, b, out)
    dist.barrier()
    if rank == 1:
        if mode == "stop":
            q.get(timeout=60)  # stays alive, steps no more, until rank 0 is done
        return
    peer = cg.guard.pids[1]
    if mode == "exit":
        t0 = _t.monotonic()
        while pid_alive(peer) and _t.monotonic() - t0 < 60:
            _t.sleep(0.05)
    else:
        _FakeEvent.complete_new = False  # from here on, steps do not complete
    results = []
    for _ in range(4):
        try:
            cg.step(a, b, out)
            results.append("ok")
        except ChainBroken as e:
            results.append(str(e))
    cg.close()  # a broken chain is not freed (no collective, no hang)
    if mode == "stop":
        q.put("done")  # lets rank 1 exit
    q.put((results, log))


@pytest.mark.parametrize("mode", ["exit", "stop"])
def test_chain_survivor_detects_a_peer_that_left(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_chain_leave, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    procs[0].join(timeout=120)
    got = [q.get(timeout=10)]
    while not isinstance(got[-1], tuple):
        got.append(q.get(timeout=10))
    results, log = got[-1]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    if mode == "exit":
        # found before step 3 was queued: nothing launched, no abort needed
        assert "neighbour rank 1" in results[0] and "has exited" in results[0]
        assert ("source", 3) not in log and not any(e[0] == "abort" for e in log)
    else:
        # steps 3 and 4 are queued; step 5 waits for step 3, which never
        # completes: the deadline expires, this rank's waits are opened
        assert results[:2] == ["ok", "ok"]
        assert "step 3 did not complete within 0.5 s" in results[2]
        assert ("abort", 4) in log and ("status",) in log
    assert results[-1] == results[-2]  # the chain stays broken
    assert ("destroy",) not in log     # and keeps its memory


def _worker_never_joins(rank, port, q):
    import datetime
    import time as _t
    if rank == 1:
        return  # this rank never joins the process group
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    t0 = _t.monotonic()
    try:
        dist.init_process_group("gloo", rank=0, world_size=2,
                                timeout=datetime.timedelta(seconds=3))
        q.put(("joined", _t.monotonic() - t0))
    except Exception as e:  # noqa: BLE001 - the expected failure
        q.put((type(e).__name__, _t.monotonic() - t0))


def test_rank_that_never_joins_ends_the_others_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_never_joins, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    what, seconds = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert what != "joined"
    assert seconds < 60
