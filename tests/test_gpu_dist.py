"""Row-sharded GEMM on several GPUs, one process per GPU (needs >= 2 GPUs).

ChainedGemm carries B from the source rank along the chain by the copy
engines while every rank's GEMM runs; each rank's rows of C must equal, bit
for bit, the single-GPU GEMM of the same rows (same packed operands, same
kernel).  B changes every step, so both chain buffers and the reuse
hand-shake between ranks are exercised."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, m_total, n, k, chunk, src, steps, q):
    import datetime

    import torch.distributed as dist

    from zengpu_b200 import kernels as K
    from zengpu_b200.dist import ChainedGemm, row_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    result = {"rank": rank, "ok": False}
    try:
        r0, r1 = row_range(m_total, world, rank)
        a_full = K.fill_uniform(torch.empty((m_total, k), device="cuda"), 7)
        a = a_full[r0:r1].contiguous()
        cg = ChainedGemm(k, n, mode=mode, src=src, chunk_cols=chunk)
        out = torch.empty((r1 - r0, n), device="cuda")
        bias = K.fill_uniform(torch.empty(n, device="cuda"), 9, -0.1, 0.1)
        mismatches = []
        for step in range(steps):
            # every rank can make the same B; only the source's copy is used
            b_full = K.fill_uniform(torch.empty((k, n), device="cuda"), 100 + step)
            relu = step % 2 == 1
            cg.step(a, b_full if rank == src else None, out, alpha=0.5,
                    bias=bias if relu else None, relu=relu)
            ref = K.sgemm(a, b_full, mode=mode, alpha=0.5, bias=bias if relu else None,
                          relu=relu)
            torch.cuda.synchronize()
            if not torch.equal(out.view(torch.int32), ref.view(torch.int32)):
                diff = (out - ref).abs().max().item()
                mismatches.append((step, diff))
        status = K.kernel_status()
        cg.close()
        result.update(ok=not mismatches and status == 0, mismatches=mismatches, status=status)
    except Exception as e:  # noqa: BLE001 - reported to the parent
        result["error"] = f"{type(e).__name__}: {e}"
    finally:
        q.put(result)
        dist.destroy_process_group()


def _run(world, **kw):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    args = (kw["mode"], kw["m_total"], kw["n"], kw["k"], kw["chunk"], kw.get("src", 0),
            kw.get("steps", 4))
    # daemonic: a rank left waiting on a peer that failed dies with the test
    procs = [ctx.Process(target=_worker, args=(r, world, port) + args + (q,), daemon=True)
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for r in sorted(results, key=lambda r: r["rank"]):
        assert r["ok"], r
    for p in procs:
        assert p.exitcode == 0


@pytest.mark.parametrize("mode", [3, 1, 2, 4], ids=["TF32_BF16X2", "TF32X3", "TF32", "BF16X3"])
def test_chained_gemm_two_ranks(mode):
    # 2 x 1024 rows: 64 tiles of 256 x 256 per rank (CTA-pair kernel); chunks of 256 columns
    _run(2, mode=mode, m_total=2048, n=4096, k=1024, chunk=256)


@pytest.mark.parametrize("mode", [4, 1], ids=["BF16X3", "TF32X3"])
def test_chained_gemm_single_cta_kernel(mode):
    # 2 x 256 rows, 1024 columns: 4 tiles of 256 x 256 per rank, below the pair
    # kernel's 8, so the gated GEMM runs one CTA per 128 x 256 tile
    _run(2, mode=mode, m_total=512, n=1024, k=768, chunk=256)


def test_chained_gemm_pair_kernel_ragged():
    # 2 x 2050 rows, n not a multiple of the chunk, k not a multiple of 16:
    # enough 256 x 256 tiles for the CTA-pair kernel
    _run(2, mode=3, m_total=4100, n=4000, k=2072, chunk=512)


def test_chained_gemm_source_not_rank0():
    # 2 x 512 rows: 16 tiles per rank, run as 32 half-width (256 x 128) units
    _run(2, mode=3, m_total=1024, n=2048, k=512, chunk=256, src=1)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs four GPUs")
def test_chained_gemm_four_ranks():
    _run(4, mode=3, m_total=4096, n=4096, k=1024, chunk=256, src=2)


def _worker_leave(rank, world, port, how, q, release):
    """Two ranks run two chained steps; then one rank leaves between steps
    (none of its work in flight): `exit` - its process ends; `stop` - it stays
    alive but takes no further step.  The survivor must find out on the host
    before it launches into the gone rank (pid check) or, for a rank that
    stopped, when a step misses its deadline (then its own waits are opened
    and its queued work drains), raise ChainBroken, and still compute a
    correct one-GPU GEMM afterwards."""
    import datetime
    import time

    import numpy as np
    import torch.distributed as dist

    import _oracle as O
    from zengpu_b200 import kernels as K
    from zengpu_b200.dist import ChainBroken, ChainedGemm, pid_alive, row_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    leaver = 1 if how in ("exit", "stop") else 0
    result = {"rank": rank, "ok": False}
    try:
        m_total, n, k = 2048, 2048, 1024
        r0, r1 = row_range(m_total, world, rank)
        a = K.fill_uniform(torch.empty((r1 - r0, k), device="cuda"), 7 + rank)
        cg = ChainedGemm(k, n, mode=4, src=0, chunk_cols=256, deadline_s=3.0)
        out = torch.empty((r1 - r0, n), device="cuda")
        b = K.fill_uniform(torch.empty((k, n), device="cuda"), 100)
        for _ in range(2):
            cg.step(a, b if rank == 0 else None, out)
        torch.cuda.synchronize()
        dist.barrier()  # every rank's two steps are complete
        if rank == leaver:
            result["ok"] = True
            if how == "stop":
                q.put(result)
                release.get(timeout=120)  # stays alive until the survivor is done
                return
            return  # exit: the process ends here
        peer = cg.guard.pids[leaver]
        if how in ("exit", "exit0"):
            t0 = time.monotonic()
            while pid_alive(peer) and time.monotonic() - t0 < 60:
                time.sleep(0.05)
        outcomes = []
        t0 = time.monotonic()
        for _ in range(6):
            try:
                cg.step(a, b if rank == 0 else None, out)
                outcomes.append("ok")
            except ChainBroken as e:
                outcomes.append(str(e))
        elapsed = time.monotonic() - t0
        torch.cuda.synchronize()
        broken = [o for o in outcomes if o != "ok"]
        # a fresh one-GPU GEMM on the survivor, on the same stream, is correct
        x = O.uniform(300 * 200, 31).reshape(300, 200)
        y = O.uniform(200 * 260, 32).reshape(200, 260)
        c = K.sgemm(torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda(), mode=4)
        torch.cuda.synchronize()
        err = O.rel_fro(c.cpu().numpy(), O.sgemm(x, y))
        result.update(outcomes=outcomes, elapsed=elapsed, err=err, status=K.kernel_status(),
                      ok=bool(broken) and err <= 1e-5 and np.isfinite(err))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        result["error"] = f"{type(e).__name__}: {e}"
    finally:
        gone = rank == leaver and how in ("exit", "exit0")
        if not gone and not (rank == leaver and how == "stop"):
            q.put(result)
        if how == "stop" and rank != leaver:
            release.put("done")  # lets the rank that stopped exit
        if not gone:
            dist.destroy_process_group()


@pytest.mark.parametrize("how", ["exit", "exit0", "stop"])
def test_chain_survivor_after_a_rank_leaves(how):
    """exit: the last rank leaves; exit0: the source leaves; stop: the last
    rank stays alive but stops stepping (the source's deadline expires)."""
    ctx = mp.get_context("spawn")
    q, release = ctx.Queue(), ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_leave, args=(r, 2, port, how, q, release), daemon=True)
             for r in range(2)]
    for p in procs:
        p.start()
    survivor = 0 if how in ("exit", "stop") else 1
    results = {}
    deadline = 300
    while survivor not in results:
        item = q.get(timeout=deadline)
        results[item["rank"]] = item
    for p in procs:
        p.join(timeout=120)
    r = results[survivor]
    assert r["ok"], r
    if how == "stop":
        # steps 3 to 6 are queued (3 and 4 complete: the stopped rank had
        # released steps 1 and 2); the fifth call waits for step 5, whose copy
        # to the stopped rank waits for it to release step 3: the deadline
        # expires
        assert r["outcomes"][:4] == ["ok"] * 4, r
        assert "did not complete within 3 s" in r["outcomes"][4], r
    else:
        assert "has exited" in r["outcomes"][0], r
        assert r["elapsed"] < 10, r
    assert r["status"] == 0, r
    for p in procs:
        assert p.exitcode == 0
