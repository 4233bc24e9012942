#!/usr/bin/env python
"""Benchmark of the ZenGPU compute hot path on B200.

Default workload (one JSON line on rank 0):
  f32 GEMM, BF16X3 tensor-core mode (each f32 operand split into bf16 hi +
  lo, three bf16 products; rel-Frobenius error ~4e-6 against float64, inside
  the 1e-5 bar of the fp32-class modes), M = N = K = 8192 per GPU.  With N
  GPUs each rank owns an 8192-row block of A and C (weak scaling, M = 8192 *
  N); every step B (8192 x 8192) is packed on rank 0 and carried rank to rank
  over NVLink by the copy engines while every rank's GEMM runs (--bcast nccl:
  an NCCL broadcast first) - the path's only exchange.

  value       whole-job useful TFLOP/s (2*M*N*K per step over all ranks),
              device-timed with CUDA events, max over ranks
  accuracy    sampled blocks against float64; at N > 1 also each rank's rows
              bit for bit against the same rows computed by that GPU alone
  e2e         the same GEMM through the drop-in API with host buffers on
              every rank (GemmKernel.sgemm_host: pinned H2D of A rows and B,
              GEMM, D2H of C rows, every step), host clock, max over ranks
  roofline    the tcgen05 kernel alone against its mode's tensor ceiling
  sustained   (N = 1) the same step back to back for >= 2.5 s, against the
              sustained (power-limited) bf16 peak, with the median SM clock
  strong      M = N = 32768, K = 8192 row-sharded over this run's N GPUs for
              >= 1.5 s, with the one-GPU time of the same problem measured in
              the same process (rank 0 alone) as its denominator
  mlp         (N = 1) the op_graph_lower MLP, fused vs unfused epilogue
  peer_copy   (N > 1) CudaDevice.copy_from_peer between neighbouring GPUs
  cpu_baseline the CPU backend's algorithm (the oracle's C restatement of
              zengpu-cpu's loop) on a bounded row sample, all host cores, and
              on one thread with CpuDevice's per-dispatch buffer clones
  elementwise add (z = x + y) and in-place ReLU on 2^28 f32 (1 GiB each)

--impl reference runs only the CPU backend's algorithm (rank 0; other ranks
exit at once) on the same metric and prints its own line.
--workload mlp / sharded run the op_graph_lower MLP chain or the
32768 x 32768 x 8192 strong-scaling GEMM instead.
"""
from __future__ import annotations

import argparse
import ctypes as C
import datetime
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "f32 GEMM TFLOP/s at 8192³ (1/2/4/8 B200); add/ReLU HBM GB/s; vs CPU backend"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the
# dominant kernel, from one ncu capture of the same workload on a B200:
#   BF16X3: --set full -k regex:sgemm_tc_pair -s 3 -c 1 on
#   `bench.py --steps 4 --warmup 3 --no-extras` (the current kernel; captures of
#   the same command on other boxes read 2.3-3.8 GB);
#   the other GEMM modes were captured with the earlier raster of 16 row-tiles;
#   --section MemoryWorkloadAnalysis -k regex:stream_vec_kernel on the elementwise workload
# Keyed by the kernel and the per-rank GEMM size (M = N = K) or element count.
NCU_TRAFFIC = {
    ("sgemm_tc_pair_kernel<4>", 8192): 2.687e9,
    ("sgemm_tc_pair_kernel<3>", 8192): 5.642e9,
    ("sgemm_tc_pair_kernel<2>", 8192): 5.999e9,
    ("sgemm_tc_pair_kernel<1>", 8192): 3.105e9,
    ("sgemm_tc_kernel<3>", 8192): 4.841e9,
    ("sgemm_tc_kernel<2>", 8192): 4.869e9,
    ("stream_vec_kernel<AddOp>", 1 << 28): 3.188e9,
}


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def env_ranks() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


# ---- clocks -------------------------------------------------------------------------
class ClockSampler:
    """SM clock, power and clock-event reasons of one GPU, sampled every 2 ms
    on a background thread while the `with` block (the timed region) runs.

    The GPU is found through NVML by the PCI bus id of the CUDA device, so the
    samples belong to the GPU this process runs on whatever CUDA_VISIBLE_DEVICES
    says.  `reader` (tests) replaces NVML: a callable returning
    (sm_mhz, sm_max_mhz, power_w, set of active reason names)."""

    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    PERIOD_S = 0.002

    def __init__(self, cuda_index: int = 0, reader=None):
        self.cuda_index = cuda_index
        self.reader = reader
        self.samples: list[tuple[float, float, float, frozenset]] = []
        self.error = None
        self._stop = threading.Event()
        self._thread = None

    def _nvml_reader(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.cuda_index)
        bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
        h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        bits = {"hw_slowdown": pynvml.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": pynvml.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": pynvml.nvmlClocksEventReasonSwPowerCap}
        sm_max = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))

        def read():
            sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
            power = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
            mask = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
            return sm, sm_max, power, frozenset(n for n, b in bits.items() if mask & b)
        return read

    def _run(self):
        while True:
            try:
                self.samples.append((time.monotonic(),) + tuple(self.reader()))
            except Exception as e:  # noqa: BLE001 - reported in the summary
                self.error = f"{type(e).__name__}: {e}"
                return
            if self._stop.wait(self.PERIOD_S):
                return

    def __enter__(self):
        if self.reader is None:
            try:
                self.reader = self._nvml_reader()
            except Exception as e:  # noqa: BLE001
                self.error = f"NVML unavailable: {type(e).__name__}: {e}"
                return self
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "source": "nvml", "error": self.error}
        sm = [s[1] for s in self.samples]
        reasons = sorted({r for s in self.samples for r in s[4]} & set(self.REASONS))
        out = {"sm_mhz": statistics.median(sm), "sm_min_mhz": min(sm),
               "sm_max_mhz": max(s[2] for s in self.samples),
               "power_w_max": round(max(s[3] for s in self.samples), 1),
               "reasons": reasons, "samples": len(self.samples),
               "source": f"nvml every {int(self.PERIOD_S * 1000)} ms over the timed region"}
        if self.error:
            out["error"] = self.error
        return out


def _oracle():
    sys.path.insert(0, str(ROOT / "tests"))
    import _oracle
    return _oracle


def cpu_gemm_sample(m: int, n: int, k: int, seconds: float, seed: int = 2,
                    threads: int | None = None) -> dict:
    """Times the CPU backend's row -> col -> k loop (zengpu-cpu via the oracle)
    on whole rows of C, about `seconds` of work, on `threads` host threads
    (default: all host cores)."""
    import numpy as np
    O = _oracle()
    threads = threads or os.cpu_count() or 1
    a = O.uniform(m * k, seed).reshape(m, k)
    b = O.uniform(k * n, seed + 1000).reshape(k, n)
    c = np.zeros((m, n), np.float32)
    L = O.lib()

    def run(rows: int) -> float:
        t0 = time.perf_counter()
        L.zgo_sgemm_ref(m, n, k, 1.0, C.c_void_p(a.ctypes.data), C.c_void_p(b.ctypes.data),
                        C.c_void_p(c.ctypes.data), 0, rows, threads)
        return time.perf_counter() - t0

    rows = threads
    dt = run(rows)
    if dt < seconds / 2:
        rows = min(m, max(rows, int(rows * seconds / max(dt, 1e-3))))
        rows = max(threads, rows // threads * threads)
        dt = run(rows)
    flops = 2.0 * rows * n * k
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": threads,
            "seconds": dt, "rows": rows,
            "sample": f"{rows} of {m} rows of C = A@B, {m}x{n}x{k} f32 (row,col,k loop of "
                      f"zengpu-cpu, unfused mul+add), {threads} threads, {dt:.1f} s"}


def cpu_dispatch_clone_cost(m: int, n: int, k: int) -> dict:
    """The reference CpuDevice's per-dispatch buffer handling for one GEMM
    (zengpu-cpu/src/lib.rs:322-365): every bound buffer (A, B, C) is cloned
    into a fresh Vec before the kernel runs, and every one is copied back into
    its buffer afterwards.  Timed here as a fresh copy of each array, then a
    copy back into the original, on one thread."""
    import numpy as np
    arrays = [np.ones((m, k), np.float32), np.ones((k, n), np.float32),
              np.zeros((m, n), np.float32)]
    t0 = time.perf_counter()
    snaps = [x.copy() for x in arrays]
    for x, s in zip(arrays, snaps):
        np.copyto(x, s)
    dt = time.perf_counter() - t0
    nbytes = sum(x.nbytes for x in arrays)
    return {"seconds_per_dispatch": dt, "bytes_cloned": nbytes, "bytes_written_back": nbytes}


def cpu_single_thread_line(m: int, n: int, k: int, seconds: float = 6.0) -> dict:
    """The reference semantics line: the CPU backend runs the GEMM on one host
    thread, as CpuDevice does, plus its per-dispatch clone / write-back of the
    bound buffers.  The loop is timed on a row sample; the full step is that
    rate over all of C plus one dispatch's clone cost."""
    s = cpu_gemm_sample(m, n, k, seconds=seconds, threads=1)
    clone = cpu_dispatch_clone_cost(m, n, k)
    loop_s = 2.0 * m * n * k / (s["value"] * 1e12)
    step_s = loop_s + clone["seconds_per_dispatch"]
    return {"value": s["value"], "unit": "TFLOP/s", "cores": 1, "kind": "port",
            "sample": s["sample"], "clone_per_dispatch": clone,
            "full_step_seconds_projected": step_s,
            "value_with_clone": 2.0 * m * n * k / step_s / 1e12}


# ---- GPU helpers ------------------------------------------------------------------------
def elementwise_bench(torch, K, peak_gbs: float, iters: int = 20) -> dict:
    n = 1 << 28
    x = torch.empty(n, device="cuda")
    y = torch.empty(n, device="cuda")
    z = torch.empty(n, device="cuda")
    K.fill_normal(x, 1)
    K.fill_normal(y, 2)
    s = torch.cuda.current_stream()
    out = {}
    for name, fn, bytes_per in (("add", lambda: K.add_f32(x, y, z), 12),
                                ("relu_inplace", lambda: K.relu_f32(z, z), 8)):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(s)
        for _ in range(iters):
            fn()
        e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / iters
        gbs = bytes_per * n / (ms * 1e-3) / 1e9
        out[name] = {"gbs": round(gbs, 1), "ms": round(ms, 4), "frac": round(gbs / peak_gbs, 3),
                     "bytes": bytes_per * n}
    out["elements"] = n
    out["peak_gbs"] = peak_gbs
    del x, y, z
    torch.cuda.empty_cache()
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["gemm", "mlp", "sharded", "elementwise"],
                    default="gemm")
    ap.add_argument("--mode", choices=["tf32x3", "tf32", "simt", "tf32bf16", "bf16x3"],
                    default="bf16x3",
                    help="GEMM arithmetic; bf16x3, tf32bf16 and tf32x3 are the fp32-accurate "
                         "(rel-Frobenius <= 1e-5) tensor-core modes, tf32 the fast one (5e-3)")
    ap.add_argument("--size", type=int, default=8192)
    ap.add_argument("--panels", type=int, default=1,
                    help="N > 1: column panels of the B broadcast (1 = whole B, overlapped "
                         "with packing A)")
    ap.add_argument("--bcast", choices=["chain", "nccl"], default="chain",
                    help="N > 1: how B reaches every rank - packed once on rank 0 and pushed "
                         "rank to rank by the copy engines under the running GEMMs (chain), or "
                         "an NCCL broadcast of raw B before each rank packs it (nccl)")
    ap.add_argument("--chunk-cols", type=int, default=0,
                    help="chain: columns of B per chunk (multiple of 256; 0 = ~16 MiB packed)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the e2e / elementwise / cpu-baseline legs")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    rank, local_rank, world = env_ranks()
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    return ours(args, rank, local_rank, world)


def reference_arm(args, rank: int, world: int) -> int:
    """The CPU backend's own algorithm, timed on the host cores (rank 0 only)."""
    if rank != 0:
        return 0
    m = n = k = args.size
    sample = None
    for _ in range(args.warmup):
        cpu_gemm_sample(m, n, k, seconds=2.0)
    vals, secs = [], 0.0
    for _ in range(args.steps):
        sample = cpu_gemm_sample(m, n, k, seconds=2.0)
        vals.append(sample["value"])
        secs += sample["seconds"]
    value = statistics.mean(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * secs / max(args.steps, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"sgemm f32 M=N=K={m}, CPU backend loop on a row sample",
                   "m": m, "n": n, "k": k},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": sample["cores"],
                         "kind": "port", "sample": sample["sample"]},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)
    return 0


def ours(args, rank: int, local_rank: int, world: int) -> int:
    import torch
    import torch.distributed as dist

    import zengpu_b200 as zg
    from zengpu_b200 import kernels as K

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=dev)
    peaks, peak_src = load_peaks()
    mode = {"tf32x3": zg.GemmMode.TF32X3, "tf32": zg.GemmMode.TF32,
            "simt": zg.GemmMode.SIMT_FP32, "tf32bf16": zg.GemmMode.TF32_BF16X2,
            "bf16x3": zg.GemmMode.BF16X3}[args.mode]
    try:
        if args.workload == "mlp":
            line = mlp_workload(args, torch, zg, K, mode, peaks, peak_src, world)
        elif args.workload == "elementwise":
            line = elementwise_workload(args, torch, dist, K, peaks, peak_src, rank, local_rank,
                                        world)
        else:
            line = gemm_workload(args, torch, dist, zg, K, mode, peaks, peak_src, rank,
                                 local_rank, world)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
    return 0


def _gather_floats(torch, dist, world, value: float) -> list[float]:
    if world == 1:
        return [value]
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    return [round(float(p.item()), 4) for p in parts]


def _max_over_ranks(torch, dist, world, value: float) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _event_pair(torch):
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def timed_steps(torch, dist, world, stream, step, warmup: int, local_rank: int,
                steps: int | None = None, min_seconds: float = 0.0, max_steps: int = 4000,
                kev=None) -> dict:
    """Runs `warmup` untimed steps, then times `steps` steps (or, when steps is
    None, enough steps for at least `min_seconds`, the same count on every
    rank) with CUDA events on `stream`, a barrier and a synchronize on both
    sides, and NVML clocks sampled meanwhile.  ms is this rank's mean step."""
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if steps is None:
        e0, e1 = _event_pair(torch)
        e0.record(stream)
        step()
        e1.record(stream)
        torch.cuda.synchronize()
        est = _max_over_ranks(torch, dist, world, e0.elapsed_time(e1))
        steps = int(min(max_steps, max(5, math.ceil(min_seconds * 1e3 / max(est, 1e-3)))))
    t0, t1 = _event_pair(torch)
    with ClockSampler(local_rank) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0.record(stream)
        for i in range(steps):
            if kev is not None and i < len(kev):
                step(*kev[i])
            else:
                step()
        t1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    return {"ms": t0.elapsed_time(t1) / steps, "steps": steps, "clocks": clocks.summary()}


class RowGemm:
    """C[rows] = A[rows] @ B on this rank: the row-sharded GEMM the path runs.

    A's row block of rank r is uniform[-1, 1) from seed seed_a + 7919 r (one
    fill of the block), B is uniform[-1, 1) from seed_b and lives on rank 0;
    with one GPU a step is the pre-pass plus the tcgen05 kernel, with several
    it is ChainedGemm (B packed on rank 0 and carried rank to rank by the copy
    engines under the running GEMMs) or, with bcast='nccl', ShardedGemm's
    pipelined NCCL broadcast."""

    def __init__(self, torch, dist, zg, K, mode, m_total: int, n: int, k: int, rank: int,
                 world: int, seed_a: int, seed_b: int, bcast: str = "chain",
                 chunk_cols: int | None = None, panels: int = 1):
        from zengpu_b200.dist import row_range
        self.torch, self.dist, self.zg, self.K = torch, dist, zg, K
        self.mode, self.n, self.k, self.rank, self.world = mode, n, k, rank, world
        self.m_total = m_total
        self.rows = row_range(m_total, world, rank)
        self.m = self.rows[1] - self.rows[0]
        self.seed_a, self.seed_b = seed_a, seed_b
        self.a = K.fill_uniform(torch.empty((self.m, k), device="cuda"), seed_a + 7919 * rank)
        self.b = torch.empty((k, n), device="cuda")
        if rank == 0 or world == 1:
            K.fill_uniform(self.b, seed_b)
        else:
            self.b.zero_()  # B reaches this rank only through the exchange
        self.c = torch.empty((self.m, n), device="cuda")
        self.lib = zg.load_library()
        self.stream = torch.cuda.current_stream()
        self.sp = C.c_void_p(self.stream.cuda_stream)
        self.ws = None
        self.chain = None
        self.sg = None
        self.panels = 1
        if world > 1 and bcast == "chain":
            from zengpu_b200.dist import ChainedGemm
            self.chain = ChainedGemm(k, n, mode=int(mode), src=0, chunk_cols=chunk_cols)
        elif world > 1:
            from zengpu_b200.dist import ShardedGemm
            self.sg = ShardedGemm(mode=int(mode))
            self.panels = max(1, panels)
        else:
            self._workspace()

    def _workspace(self):
        if self.ws is None:
            nb = self.K.workspace_bytes(self.mode, self.m, self.n, self.k)
            self.ws = self.torch.empty(max(nb, 256), dtype=self.torch.uint8, device="cuda")
        return self.ws

    def local(self, ev0=None, ev1=None, out=None):
        """This rank's rows on this GPU alone: pre-pass, then the kernel
        (bracketed by ev0 / ev1 when given)."""
        ws = self._workspace()
        out = self.c if out is None else out
        self.zg.api.check(self.lib.zg_sgemm_prepare(
            int(self.mode), self.m, self.n, self.k, self.a.data_ptr(), self.b.data_ptr(),
            ws.data_ptr(), ws.numel(), self.sp))
        if ev0 is not None:
            ev0.record(self.stream)
        self.zg.api.check(self.lib.zg_sgemm_compute(
            int(self.mode), self.m, self.n, self.k, 1.0, self.a.data_ptr(), self.b.data_ptr(),
            out.data_ptr(), None, 0, ws.data_ptr(), ws.numel(), self.sp))
        if ev1 is not None:
            ev1.record(self.stream)

    def step(self, ev0=None, ev1=None):
        if self.chain is not None:
            self.chain.step(self.a, self.b if self.rank == 0 else None, self.c)
        elif self.sg is not None:
            self.sg.sgemm_rows_pipelined(self.a, self.b, src=0, panels=self.panels, out=self.c)
        else:
            self.local(ev0, ev1)

    @property
    def launches_per_step(self) -> int:
        """This library's kernels per step: chain (rank 0) B pack with chunk
        flags, A pack, GEMM; NCCL: A pack + per panel B pack + GEMM; one GPU:
        the pre-pass kernels of the mode plus the GEMM (SIMT: A's transpose
        when n % 4 == 0, for its TMA-fed kernel)."""
        zg = self.zg
        if self.chain is not None:
            return 3
        if self.sg is not None:
            return 1 + 2 * self.panels
        return {zg.GemmMode.TF32X3: 3, zg.GemmMode.TF32: 2 + (self.k % 4 != 0),
                zg.GemmMode.SIMT_FP32: 1 + (self.n % 4 == 0), zg.GemmMode.TF32_BF16X2: 3,
                zg.GemmMode.BF16X3: 3}[self.mode]

    def finish_exchange(self):
        """After the timed steps: every rank regenerates B from its seed (the
        exchange delivered the same bytes), and the chain is released."""
        desc = None
        if self.chain is not None:
            desc = (self.chain.chunks, self.chain.chunk_cols)
            self.chain.close()
            self.chain = None
        if self.world > 1 and self.rank != 0:
            self.K.fill_uniform(self.b, self.seed_b)
        return desc

    def bit_equal_to_one_gpu(self) -> bool:
        """This rank's rows of C, as the exchange produced them, against the
        same rows computed by this GPU alone from the same A and B (same
        kernel, same packed operands): equal bit for bit."""
        got = self.c.clone()
        self.local()
        self.torch.cuda.synchronize()
        same = bool(self.torch.equal(got.view(self.torch.int32), self.c.view(self.torch.int32)))
        del got
        return same

    def accuracy(self, blocks: int = 4, size: int = 128) -> dict:
        """Relative Frobenius error of `blocks` size x size blocks of this rank's
        C against a float64 product on the host; max over ranks."""
        import numpy as np
        torch, dist, world = self.torch, self.dist, self.world
        rng = np.random.default_rng(1000 + self.rank)
        worst = 0.0
        picks = []
        for i in range(blocks):
            r0 = int(rng.integers(0, max(1, self.m - size + 1)))
            c0 = int(rng.integers(0, max(1, self.n - size + 1)))
            if i == 0:
                r0, c0 = 0, 0
            rows = self.a[r0:r0 + size].double().cpu().numpy()
            cols = self.b[:, c0:c0 + size].double().cpu().numpy()
            ref = rows @ cols
            got = self.c[r0:r0 + size, c0:c0 + size].double().cpu().numpy()
            worst = max(worst, float(np.linalg.norm(got - ref) / np.linalg.norm(ref)))
            picks.append([self.rows[0] + r0, c0])
        err = _max_over_ranks(torch, dist, world, worst)
        bar = 5e-3 if self.mode == self.zg.GemmMode.TF32 else 1e-5
        return {"rel_fro_vs_fp64": err, "bar": bar, "blocks_per_rank": blocks,
                "block": size, "rank0_blocks": picks, "ranks": world, "within_bar": err <= bar}

    def close(self):
        if self.chain is not None:
            self.chain.close()
            self.chain = None
        self.a = self.b = self.c = self.ws = None
        self.torch.cuda.synchronize()
        self.torch.cuda.empty_cache()


def gemm_workload(args, torch, dist, zg, K, mode, peaks, peak_src, rank, local_rank, world):
    """The default line (weak scaling, M = N = K = size per GPU) or, with
    --workload sharded, the 32768 x 32768 x 8192 strong-scaling GEMM."""
    s = args.size
    if args.workload == "sharded":
        m_total, n, k, seed_a, seed_b = 32768, 32768, 8192, 4, 1004
        scaling = "strong"
        workload = f"sgemm {args.mode} M=N=32768 K=8192 row-sharded over {world}"
    else:
        m_total, n, k, seed_a, seed_b = s * world, s, s, 2, 1002
        scaling = "weak"
        workload = f"sgemm {args.mode} M=N=K={s} per GPU (M={m_total} total, A/C row blocks)"
    g = RowGemm(torch, dist, zg, K, mode, m_total, n, k, rank, world, seed_a, seed_b,
                bcast=args.bcast, chunk_cols=args.chunk_cols or None, panels=args.panels)
    m_local = g.m
    kev = [_event_pair(torch) for _ in range(args.steps)]
    t = timed_steps(torch, dist, world, g.stream, g.step, args.warmup, local_rank,
                    steps=args.steps, kev=kev if world == 1 else None)
    if K.kernel_status() != 0:
        raise RuntimeError("bounded on-device wait expired during the timed steps")
    ms_local = t["ms"]
    chain_desc = g.finish_exchange()
    accuracy = g.accuracy()
    if world > 1:
        accuracy["bit_equal_to_1gpu"] = _gather_floats(
            torch, dist, world, 1.0 if g.bit_equal_to_one_gpu() else 0.0)
        accuracy["bit_equal_to_1gpu"] = [bool(v) for v in accuracy["bit_equal_to_1gpu"]]
        accuracy["bit_equal_check"] = ("each rank's rows of C from the exchange vs the same "
                                       "rows computed by that GPU alone (same kernel)")
        # the dominant kernel alone: one full-shard launch per rank, same stream
        for _ in range(2):
            g.local()
        nk = min(args.steps, 5)
        for i in range(nk):
            g.local(*kev[i])
        torch.cuda.synchronize()
        kern_ms_local = statistics.mean(e0.elapsed_time(e1) for e0, e1 in kev[:nk])
    else:
        kern_ms_local = statistics.mean(e0.elapsed_time(e1) for e0, e1 in kev)
    ms = _max_over_ranks(torch, dist, world, ms_local)
    ms_by_rank = _gather_floats(torch, dist, world, ms_local)
    kern_ms = _max_over_ranks(torch, dist, world, kern_ms_local)
    if K.kernel_status() != 0:
        raise RuntimeError("bounded on-device wait expired in the kernel-only timing")
    launches_per_step = g.launches_per_step
    lib, sp, stream = g.lib, g.sp, g.stream

    other = {}
    sustained = None
    fp32_class = {"tf32x3": zg.GemmMode.TF32X3, "tf32bf16": zg.GemmMode.TF32_BF16X2,
                  "bf16x3": zg.GemmMode.BF16X3}
    if not args.no_extras and args.workload == "gemm" and world == 1:
        if mode in fp32_class.values():
            # the other fp32-accurate modes' kernels on the same operands
            for name, other_mode in fp32_class.items():
                if other_mode != mode:
                    other[name] = kernel_only(torch, lib, other_mode, g.a, g.b, g.c, m_local, n,
                                              k, sp, stream, dist, world)
        sustained = sustained_gemm(torch, dist, g, mode, peaks, peak_src, local_rank)
    total_flops = 2.0 * m_total * n * k
    value = total_flops / (ms * 1e-3) / 1e12
    achieved = 2.0 * m_local * n * k / (kern_ms * 1e-3) / 1e12
    peak, peak_basis = mode_peak(zg, mode, peaks, peak_src)
    kname = tc_kernel_name(torch, int(mode), m_local, n, k)
    g.close()
    del g

    extras = {}
    e2e = cpu = None
    if not args.no_extras:
        if args.workload == "gemm":
            extras["strong"] = strong_scaling(args, torch, dist, zg, K, mode, peaks, rank,
                                              local_rank, world)
        e2e = gemm_e2e(args, torch, dist, zg, K, mode, m_local, n, k, m_total, world, local_rank)
        extras["elementwise"] = elementwise_bench(torch, K, peaks["hbm_gbs"])
        if world > 1:
            extras["peer_copy"] = peer_copy_check(torch, dist, zg, rank, local_rank, world)
        if world == 1:
            extras["mlp"] = mlp_measure(torch, K, mode, steps=5, warmup=3)
            extras["mlp"]["drop_in"] = mlp_drop_in(torch, zg, mode)
        if world == 1 and rank == 0:
            cpu = cpu_gemm_sample(m_total, n, k, seconds=12.0)
            cpu["single_thread"] = cpu_single_thread_line(m_total, n, k)
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic: A, B uniform[-1,1) from the splitmix64 generator (A block of "
                f"rank r: seed {seed_a} + 7919 r; B: seed {seed_b})",
        "config": {"workload": workload, "m": m_total, "n": n, "k": k, "mode": args.mode,
                   "parallelism": (f"dp{world} (A/C row blocks; B packed on rank 0 and pushed "
                                   f"rank to rank over NVLink by the copy engines in "
                                   f"{chain_desc[0]} chunks of {chain_desc[1]} columns, each "
                                   f"rank's GEMM gated per chunk)" if chain_desc is not None else
                                   f"dp{world} (A/C row blocks, B broadcast over NCCL in "
                                   f"{args.panels} column panels)" if world > 1 else
                                   "dp1 (one GPU, no exchange)"),
                   "l2": f"inputs larger than L2: A {m_local * k * 4 >> 20} MiB, B {k * n * 4 >> 20} MiB, "
                         f"packed operands {algorithmic_bytes(mode, m_local, n, k) - 4 * m_local * n >> 20} MiB"},
        "roofline": {"bound": "tensor" if mode != zg.GemmMode.SIMT_FP32 else "fp32",
                     "kernel": kname, "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak,
                     "traffic": NCU_TRAFFIC.get((kname, s)) if args.workload == "gemm" else None,
                     "algorithmic_bytes": algorithmic_bytes(mode, m_local, n, k),
                     "kernel_ms": kern_ms, "peak_basis": peak_basis},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": t["clocks"],
    }
    if world > 1:
        line["ms_per_step_by_rank"] = ms_by_rank
    line["accuracy"] = accuracy
    if other:
        line["other_modes"] = other
    if sustained is not None:
        line["sustained"] = sustained
    if e2e is not None:
        line["e2e"] = e2e
    if cpu is not None:
        line["cpu_baseline"] = {"value": cpu["value"], "unit": cpu["unit"], "cores": cpu["cores"],
                                "kind": "port", "sample": cpu["sample"],
                                "single_thread": cpu["single_thread"]}
    line.update(extras)
    return line


def mode_peak(zg, mode, peaks, peak_src, key: str = "bf16_tflops") -> tuple[float, str]:
    """The mode's tensor ceiling in useful TFLOP/s: bf16 peak / 3 for BF16X3,
    the tf32 rate (bf16 / 2) / 3 for TF32X3, / 2 for TF32_BF16X2 (one tf32 +
    two half-cost bf16 MMAs per product), tf32 for TF32; nominal FP32 SIMT."""
    bf16 = peaks[key]
    tf32 = bf16 / 2.0
    if mode == zg.GemmMode.SIMT_FP32:
        return 148 * 128 * 2 * 1.965e9 / 1e12, \
            "nominal FP32 SIMT: 148 SMs x 128 lanes x 2 flop x 1965 MHz"
    peak = {zg.GemmMode.TF32X3: tf32 / 3.0, zg.GemmMode.TF32: tf32,
            zg.GemmMode.TF32_BF16X2: tf32 / 2.0, zg.GemmMode.BF16X3: bf16 / 3.0}[mode]
    basis = (f"{peak_src} {key} {bf16} TFLOP/s / 3 (three bf16 MMAs per useful product)"
             if mode == zg.GemmMode.BF16X3 else
             f"{peak_src} {key} {bf16} TFLOP/s / 2 (tf32 rate)" +
             {zg.GemmMode.TF32X3: " / 3 (tf32 MMAs per useful product)",
              zg.GemmMode.TF32_BF16X2: " / 2 (one tf32 + two half-cost bf16 MMAs per useful "
                                       "product)"}.get(mode, ""))
    return peak, basis


def sustained_gemm(torch, dist, g, mode, peaks, peak_src, local_rank,
                   seconds: float = 2.5) -> dict:
    """The same one-GPU step (pre-pass + kernel) back to back for at least
    `seconds`, so the GPU settles at the clock its power limit allows; against
    the sustained bf16 peak.  ms_x_mhz (kilo-cycles per step at the median SM
    clock) compares it with the burst independently of the clock."""
    import zengpu_b200 as zg
    t = timed_steps(torch, dist, 1, g.stream, g.step, 2, local_rank, steps=None,
                    min_seconds=seconds)
    flops = 2.0 * g.m * g.n * g.k
    tflops = flops / (t["ms"] * 1e-3) / 1e12
    key = "bf16_tflops_sustained" if "bf16_tflops_sustained" in peaks else "bf16_tflops"
    peak, basis = mode_peak(zg, mode, peaks, peak_src, key)
    mhz = t["clocks"].get("sm_mhz")
    return {"tflops": tflops, "ms_per_step": t["ms"], "steps": t["steps"],
            "seconds": t["ms"] * t["steps"] / 1e3, "peak": peak, "peak_basis": basis,
            "frac_of_sustained_peak": tflops / peak, "sm_mhz_median": mhz,
            "ms_x_mhz": t["ms"] * mhz if mhz else None, "clocks": t["clocks"],
            "what": "pre-pass + tcgen05 kernel per step, back to back"}


def strong_scaling(args, torch, dist, zg, K, mode, peaks, rank, local_rank, world,
                   seconds: float = 1.5) -> dict:
    """The strong-scaling case of the sharded configuration, M = N = 32768,
    K = 8192, in the bench's mode, at this run's N: A's row blocks over the ranks, B from rank 0 along
    the copy-engine chain.  Every N times at least `seconds` of steps, long
    enough to reach the power-limited clock, so N = 1 and N > 1 compare in the
    same regime.  At N > 1 rank 0 also times the whole problem on its GPU alone
    in the same process (the measured one-GPU denominator)."""
    m_total, n, k = 32768, 32768, 8192
    g = RowGemm(torch, dist, zg, K, mode, m_total, n, k, rank, world, 4, 1004,
                bcast="chain", chunk_cols=args.chunk_cols or None)
    t = timed_steps(torch, dist, world, g.stream, g.step, 3, local_rank, steps=None,
                    min_seconds=seconds)
    if K.kernel_status() != 0:
        raise RuntimeError("bounded on-device wait expired in the strong-scaling steps")
    chain_desc = g.finish_exchange()
    ms = _max_over_ranks(torch, dist, world, t["ms"])
    by_rank = _gather_floats(torch, dist, world, t["ms"])
    mhz = t["clocks"].get("sm_mhz") or 0.0
    mhz_by_rank = _gather_floats(torch, dist, world, float(mhz))
    acc = g.accuracy()
    if world > 1:
        acc["bit_equal_to_1gpu"] = [bool(v) for v in _gather_floats(
            torch, dist, world, 1.0 if g.bit_equal_to_one_gpu() else 0.0)]
    g.close()
    del g
    flops = 2.0 * m_total * n * k
    out = {"m": m_total, "n": n, "k": k, "mode": args.mode, "n_gpus": world,
           "ms_per_step": ms, "ms_per_step_by_rank": by_rank, "steps": t["steps"],
           "tflops": flops / (ms * 1e-3) / 1e12, "sm_mhz_median_by_rank": mhz_by_rank,
           "accuracy": acc, "clocks_rank0": t["clocks"]}
    if chain_desc is not None:
        out["chain"] = {"chunks": chain_desc[0], "chunk_cols": chain_desc[1]}
    one = None
    if world == 1:
        one = {"ms_per_step": ms, "sm_mhz_median": mhz, "steps": t["steps"],
               "source": "this run"}
    else:
        if rank == 0:
            # the same problem on rank 0's GPU alone, same A (all row blocks, each
            # from its rank's seed) and B
            from zengpu_b200.dist import row_range
            g1 = RowGemm(torch, None, zg, K, mode, m_total, n, k, 0, 1, 4, 1004)
            for r in range(world):
                r0, r1 = row_range(m_total, world, r)
                K.fill_uniform(g1.a[r0:r1], 4 + 7919 * r)
            t1 = timed_steps(torch, None, 1, g1.stream, g1.step, 2, local_rank, steps=None,
                             min_seconds=seconds)
            g1.close()
            del g1
            one = {"ms_per_step": t1["ms"], "sm_mhz_median": t1["clocks"].get("sm_mhz"),
                   "steps": t1["steps"], "clocks": t1["clocks"],
                   "source": "rank 0 alone, same process, after the sharded run"}
        dist.barrier()
    if one is not None and rank == 0:
        out["one_gpu"] = one
        out["speedup_measured"] = one["ms_per_step"] / ms
        out["efficiency_measured"] = one["ms_per_step"] / (world * ms)
        # cycles, not seconds: each time at the median SM clock of its own run
        # (at N > 1 the clock of the rank whose step set the time)
        slowest = max(range(world), key=lambda r: by_rank[r])
        mhz_n = mhz_by_rank[slowest]
        if one.get("sm_mhz_median") and mhz_n:
            out["efficiency_clock_normalized"] = (one["ms_per_step"] * one["sm_mhz_median"]) / (
                world * ms * mhz_n)
            out["clock_normalized_with"] = {"one_gpu_mhz": one["sm_mhz_median"],
                                            "n_gpu_mhz": mhz_n, "n_gpu_rank": slowest}
    return out


def peer_copy_check(torch, dist, zg, rank, local_rank, world, nbytes: int = 64 << 20) -> dict:
    """GpuDevice::copy_from_peer through the drop-in API: each rank copies
    nbytes from a buffer on the next GPU into one on its own, over NVLink, and
    checks the bytes; GB/s of the copy (host clock, synchronous call)."""
    import numpy as np
    O = _oracle()
    res = {"ok": None, "gbs": None}
    if torch.cuda.device_count() < 2:
        res["skipped"] = "one visible GPU per process"
        return res
    peer = (local_rank + 1) % torch.cuda.device_count()
    mine = zg.CudaDevice(local_rank)
    other = zg.CudaDevice(peer)
    try:
        data = O.uniform(nbytes // 4, 300 + rank)
        src = other.create_buffer(nbytes)
        other.write_buffer(src, 0, data)
        dst = mine.create_buffer(nbytes)
        mine.copy_from_peer(dst, other, src, nbytes)
        t0 = time.perf_counter()
        reps = 5
        for _ in range(reps):
            mine.copy_from_peer(dst, other, src, nbytes)
        dt = (time.perf_counter() - t0) / reps
        got = np.frombuffer(mine.read_buffer(dst, 0, nbytes), np.uint32)
        ok = bool(np.array_equal(got, data.view(np.uint32)))
        other.destroy_buffer(src)
        mine.destroy_buffer(dst)
    finally:
        other.close()
        mine.close()
    torch.cuda.set_device(local_rank)
    oks = _gather_floats(torch, dist, world, 1.0 if ok else 0.0)
    gbs = _gather_floats(torch, dist, world, nbytes / dt / 1e9)
    return {"ok": [bool(v) for v in oks], "gbs": gbs, "bytes": nbytes,
            "what": "CudaDevice.copy_from_peer from GPU local_rank + 1, checked bit for bit"}


def tc_kernel_name(torch, mode: int, m: int, n: int, k: int = 8192) -> str:
    """The main GEMM kernel the library launches for this problem, as the
    library itself reports it."""
    import zengpu_b200 as zg
    return zg.load_library().zg_sgemm_kernel_name(int(mode), m, n, k).decode()


def sampled_accuracy(torch, dist, a, b, c, mode, world) -> dict:
    """Relative Frobenius error of a 256 x 256 block of each rank's C against a
    float64 product of the same operands (numpy on the host); max over ranks."""
    import numpy as np
    import zengpu_b200 as zg
    r0 = min(1000, max(a.shape[0] - 256, 0))
    c0 = min(3000, max(b.shape[1] - 256, 0))
    rows = a[r0:r0 + 256].double().cpu().numpy()
    cols = b[:, c0:c0 + 256].double().cpu().numpy()
    ref = rows @ cols
    got = c[r0:r0 + 256, c0:c0 + 256].double().cpu().numpy()
    err = _max_over_ranks(torch, dist, world,
                          float(np.linalg.norm(got - ref) / np.linalg.norm(ref)))
    bar = 5e-3 if mode == zg.GemmMode.TF32 else 1e-5
    return {"rel_fro_vs_fp64": err, "bar": bar, "block": [r0, c0, 256, 256],
            "ranks": world, "within_bar": err <= bar}


def kernel_only(torch, lib, mode, a, b, c, m, n, k, sp, stream, dist, world, reps: int = 5):
    """Device time of one more mode's tensor-core kernel on the same operands."""
    import zengpu_b200 as zg
    from zengpu_b200 import kernels as K
    ws = torch.empty(max(K.workspace_bytes(mode, m, n, k), 256), dtype=torch.uint8,
                     device="cuda")
    zg.api.check(lib.zg_sgemm_prepare(int(mode), m, n, k, a.data_ptr(), b.data_ptr(),
                                      ws.data_ptr(), ws.numel(), sp))
    evs = [_event_pair(torch) for _ in range(reps + 2)]
    for e0, e1 in evs:
        e0.record(stream)
        zg.api.check(lib.zg_sgemm_compute(int(mode), m, n, k, 1.0, a.data_ptr(), b.data_ptr(),
                                          c.data_ptr(), None, 0, ws.data_ptr(), ws.numel(), sp))
        e1.record(stream)
    torch.cuda.synchronize()
    ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs[2:])
    acc = sampled_accuracy(torch, None, a, b, c, mode, 1)
    del ws
    torch.cuda.empty_cache()
    return {"kernel_ms": ms, "kernel_tflops": 2.0 * m * n * k / (ms * 1e-3) / 1e12,
            "accuracy": acc}


def algorithmic_bytes(mode: int, m: int, n: int, k: int) -> int:
    """Bytes the GEMM kernel must move once: its operand planes in, C out."""
    if mode == 0:  # SIMT reads A and B directly
        return 4 * (m * k + k * n + m * n)
    per_elem = {1: 8, 2: 4, 3: 8, 4: 4}[int(mode)]  # tf32 hi+lo / f32 / tf32 + 2 bf16 / 2 bf16
    return per_elem * (m * k + n * k) + 4 * m * n


def gemm_e2e(args, torch, dist, zg, K, mode, m_local, n, k, m_total, world, local_rank):
    """The GEMM through the drop-in API with host buffers, every step: each
    rank calls GemmKernel.sgemm_host on its own GPU with pinned host A rows,
    host B and host C rows (B up, then row panels of A up / GEMM / C rows down
    on three streams), timed with the host clock around the synchronous calls,
    a barrier on both sides, max over ranks."""
    ha = torch.empty((m_local, k), pin_memory=True)
    hb = torch.empty((k, n), pin_memory=True)
    hc = torch.empty((m_local, n), pin_memory=True)
    rank = dist.get_rank() if world > 1 else 0
    tmp = torch.empty((m_local, k), device="cuda")
    K.fill_uniform(tmp, 2 + 7919 * rank)
    ha.copy_(tmp)
    tmp = torch.empty((k, n), device="cuda")
    K.fill_uniform(tmp, 1002)
    hb.copy_(tmp)
    del tmp
    torch.cuda.synchronize()
    steps = max(3, min(args.steps, 5))
    device = zg.CudaDevice(local_rank)
    gemm = zg.GemmKernel(device, mode)

    def step():
        gemm.sgemm_host(device, 1.0, ha, hb, hc, m_local, n, k)

    for _ in range(2):
        step()
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
    t = time.perf_counter()
    for _ in range(steps):
        step()
    dt_local = (time.perf_counter() - t) / steps
    dt = _max_over_ranks(torch, dist, world, dt_local)
    device.close()
    torch.cuda.set_device(local_rank)
    # the PCIe floor of one rank: its uploads alone at the measured H2D rate
    h2d_rank = ha.numel() * 4 + hb.numel() * 4
    d2h_rank = hc.numel() * 4
    floor = pcie_floor(torch, dist, world, h2d_rank)
    total_flops = 2.0 * m_total * n * k
    return {"value": total_flops / dt / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": h2d_rank * world, "d2h_bytes_per_step": d2h_rank * world,
            "ms_per_step": dt * 1e3, "steps": steps,
            "ms_by_rank": _gather_floats(torch, dist, world, dt_local * 1e3),
            "pcie_floor_ms": floor["ms"], "h2d_gbs": floor["gbs"],
            "clock": "host clock around GemmKernel.sgemm_host on every rank (synchronous; B up, "
                     "then row panels of A up / GEMM / C down overlapped on three streams), "
                     "barrier before, max over ranks"}


def pcie_floor(torch, dist, world: int, nbytes: int) -> dict:
    """Time of nbytes of pinned host -> device copies at the H2D rate this GPU
    reaches while every rank copies at once (256 MiB copies, CUDA events, max
    time over ranks): the floor of any step in which each rank must upload
    nbytes."""
    size = 256 << 20
    h = torch.empty(size // 4, pin_memory=True)
    d = torch.empty(size // 4, device="cuda")
    s = torch.cuda.current_stream()
    d.copy_(h, non_blocking=True)
    e0, e1 = _event_pair(torch)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record(s)
    for _ in range(3):
        d.copy_(h, non_blocking=True)
    e1.record(s)
    torch.cuda.synchronize()
    ms = _max_over_ranks(torch, dist, world, e0.elapsed_time(e1))
    gbs = 3 * size / (ms * 1e-3) / 1e9
    del h, d
    return {"gbs": gbs, "ms": nbytes / (gbs * 1e9) * 1e3}


def elementwise_workload(args, torch, dist, K, peaks, peak_src, rank, local_rank, world):
    """DeviceArray add (z = x + y) then in-place ReLU on 2^28 f32 per GPU
    (1 GiB per array, larger than L2); value = whole-job HBM GB/s of the pair
    (20 algorithmic bytes per element), chunks independent per rank."""
    n = 1 << 28
    x = torch.empty(n, device="cuda")
    y = torch.empty(n, device="cuda")
    z = torch.empty(n, device="cuda")
    K.fill_normal(x, 1 + 7919 * rank)
    K.fill_normal(y, 2 + 7919 * rank)
    stream = torch.cuda.current_stream()

    def step(ev=None):
        if ev:
            ev[0].record(stream)
        K.add_f32(x, y, z)
        if ev:
            ev[1].record(stream)
        K.relu_f32(z, z)
        if ev:
            ev[2].record(stream)

    for _ in range(args.warmup):
        step()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0.record(stream)
        for i in range(args.steps):
            step(evs[i])
        t1.record(stream)
        torch.cuda.synchronize()
    ms = _max_over_ranks(torch, dist, world, t0.elapsed_time(t1) / args.steps)
    add_ms = _max_over_ranks(torch, dist, world,
                             statistics.mean(e[0].elapsed_time(e[1]) for e in evs))
    relu_ms = _max_over_ranks(torch, dist, world,
                              statistics.mean(e[1].elapsed_time(e[2]) for e in evs))
    peak = peaks["hbm_gbs"]
    value = 20.0 * n * world / (ms * 1e-3) / 1e9
    add_gbs = 12.0 * n / (add_ms * 1e-3) / 1e9
    relu_gbs = 8.0 * n / (relu_ms * 1e-3) / 1e9
    # e2e: host arrays in pinned memory, H2D of x and y, add + relu, D2H of z
    hx = torch.empty(n, pin_memory=True)
    hy = torch.empty(n, pin_memory=True)
    hz = torch.empty(n, pin_memory=True)
    hx.copy_(x)
    hy.copy_(y)
    torch.cuda.synchronize()

    def e2e_step():
        x.copy_(hx, non_blocking=True)
        y.copy_(hy, non_blocking=True)
        K.add_f32(x, y, z)
        K.relu_f32(z, z)
        hz.copy_(z, non_blocking=True)

    e2e_step()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(3):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = _max_over_ranks(torch, dist, world, e0.elapsed_time(e1) / 3)
    cpu = None
    if world == 1 and rank == 0:
        cpu = cpu_elementwise(n)
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: x, y normal(0,1), splitmix64 + Box-Muller (seeds 1, 2)",
        "config": {"workload": "DeviceArray add z=x+y then in-place relu(z), 2^28 f32 per GPU",
                   "elements_per_gpu": n, "bytes_per_element": 20,
                   "l2": "inputs larger than L2 (1 GiB per array)",
                   "parallelism": f"{world} independent contiguous chunks, no collective"},
        "roofline": {"bound": "hbm", "kernel": "stream_vec_kernel<AddOp>", "achieved": add_gbs,
                     "peak": peak, "unit": "GB/s", "frac": add_gbs / peak,
                     "traffic": NCU_TRAFFIC.get(("stream_vec_kernel<AddOp>", n)),
                     "algorithmic_bytes": 12 * n,
                     "kernel_ms": add_ms, "peak_basis": f"{peak_src} hbm_gbs",
                     "relu_inplace": {"achieved": relu_gbs, "frac": relu_gbs / peak,
                                      "kernel_ms": relu_ms}},
        "e2e": {"value": 20.0 * n * world / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": 8 * n, "d2h_bytes_per_step": 4 * n,
                "ms_per_step": e2e_ms},
        "gpu_launches": 2 * args.steps,
        "clocks": clocks.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    return line


def cpu_elementwise(n: int) -> dict:
    """The CPU backend's add then relu over n elements, all host cores."""
    O = _oracle()
    threads = os.cpu_count() or 1
    x = O.normal(n, 1)
    y = O.normal(n, 2)
    reps = 0
    t = time.perf_counter()
    while time.perf_counter() - t < 10.0 or reps < 2:
        z = O.add(x, y, threads=threads)
        O.relu(z, threads=threads)
        reps += 1
    dt = (time.perf_counter() - t) / reps
    return {"value": 20.0 * n / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"add + relu over all {n} elements, {reps} repetitions, {threads} threads "
                      "(zengpu-cpu semantics, output buffers freshly allocated per call)"}


def mlp_measure(torch, K, mode, steps: int, warmup: int) -> dict:
    """op_graph_lower MLP: 4 x (Y = ReLU(X @ W + b)), batch 4096, hidden 4096
    (X normal(0,1) seed 3, W Kaiming-uniform seeds 100.., b uniform[-0.1, 0.1)
    seeds 200..); the fused epilogue vs the unfused gemm -> add(broadcast bias)
    -> relu chain, each timed over `steps` passes with CUDA events.  Also the
    fused chain with the weights packed once beforehand (packed-operand API:
    each layer packs only its activations), as a caller that reuses weights
    across passes would run it; it must give the fused chain's bits."""
    bsz = hid = 4096
    layers = 4
    x = torch.empty((bsz, hid), device="cuda")
    K.fill_normal(x, 3)
    bound = math.sqrt(6.0 / hid)
    ws = [K.fill_uniform(torch.empty((hid, hid), device="cuda"), 100 + i, -bound, bound)
          for i in range(layers)]
    bs = [K.fill_uniform(torch.empty(hid, device="cuda"), 200 + i, -0.1, 0.1)
          for i in range(layers)]
    bfull = [b.expand(bsz, hid).contiguous() for b in bs]
    acts = [torch.empty((bsz, hid), device="cuda") for _ in range(2)]
    tmp = torch.empty((bsz, hid), device="cuda")
    stream = torch.cuda.current_stream()

    def fused():
        h = x
        for i in range(layers):
            o = acts[i % 2]
            K.sgemm(h, ws[i], mode=mode, bias=bs[i], relu=True, out=o)
            h = o
        return h

    def unfused():
        h = x
        for i in range(layers):
            o = acts[i % 2]
            K.sgemm(h, ws[i], mode=mode, out=tmp)
            K.add_f32(tmp, bfull[i], o)
            K.relu_f32(o, o)
            h = o
        return h

    packed_w = [K.pack_b(w, mode) for w in ws]  # once, outside the timed region
    packed_x = [None]

    def fused_packed_weights():
        h = x
        for i in range(layers):
            o = acts[i % 2]
            pa = K.pack_a(h, mode, out=packed_x[0])
            packed_x[0] = pa.buf
            K.sgemm_packed(pa, packed_w[i], o, bias=bs[i], relu=True)
            h = o
        return h

    ref = fused().clone()
    same = bool(torch.equal(fused_packed_weights().view(torch.int32), ref.view(torch.int32)))
    del ref

    res = {}
    clock_summary = packed_clocks = None
    for name, fn in (("fused", fused), ("unfused", unfused),
                     ("fused_packed_weights", fused_packed_weights)):
        for _ in range(warmup):
            fn()
        e0, e1 = _event_pair(torch)
        torch.cuda.synchronize()
        with ClockSampler(torch.cuda.current_device()) as clocks:
            e0.record(stream)
            for _ in range(steps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize()
        res[name] = e0.elapsed_time(e1) / steps
        if name == "fused":
            clock_summary = clocks.summary()
        if name == "fused_packed_weights":
            packed_clocks = clocks.summary()
    flops = layers * 2.0 * bsz * hid * hid
    del x, ws, bs, bfull, acts, tmp, packed_w, packed_x
    torch.cuda.empty_cache()
    return {"fused_ms": res["fused"], "unfused_ms": res["unfused"],
            "tflops_fused": flops / (res["fused"] * 1e-3) / 1e12,
            "tflops_unfused": flops / (res["unfused"] * 1e-3) / 1e12,
            "speedup_fused_vs_unfused": res["unfused"] / res["fused"], "steps": steps,
            "fused_packed_weights_ms": res["fused_packed_weights"],
            "tflops_fused_packed_weights": flops / (res["fused_packed_weights"] * 1e-3) / 1e12,
            "packed_weights_bit_equal_to_fused": same,
            "packed_weights_clocks": packed_clocks,
            # per layer: the split modes pack A, pack B, kernel; TF32 transposes B then
            # runs the kernel; SIMT transposes A then runs the kernel; unfused adds add + relu
            "launches_fused": steps * layers * {0: 2, 1: 3, 2: 2, 3: 3, 4: 3}.get(int(mode), 1),
            "clocks": clock_summary,
            "workload": "op_graph_lower MLP 4 x relu(X@W+b), X 4096x4096, W 4096x4096"}


def mlp_drop_in(torch, zg, mode, steps: int = 5) -> dict:
    """The op_graph_lower MLP end to end through the drop-in API, host clock:
    each step writes X (4096 x 4096, from host memory) into a DeviceArray,
    runs the four fused layers (GemmKernel.gemm_bias_relu; weights and biases
    resident) and reads Y back.  Upload pool: the reference's flow, every op
    waits for the GPU; GpuOnly pool: the layers are queued and Y returns
    through one readback submission into pinned memory."""
    import numpy as np
    O = _oracle()
    bsz = hid = 4096
    layers = 4
    bound = math.sqrt(6.0 / hid)
    x = O.normal(bsz * hid, 3).reshape(bsz, hid)
    ws = [O.uniform(hid * hid, 100 + i, -bound, bound).reshape(hid, hid) for i in range(layers)]
    bs = [O.uniform(hid, 200 + i, -0.1, 0.1) for i in range(layers)]
    device = zg.CudaDevice(torch.cuda.current_device())
    gemm = zg.GemmKernel(device, mode)
    out = {}
    ys = {}
    try:
        for memory in (zg.MemoryUsage.Upload, zg.MemoryUsage.GpuOnly):
            pool = zg.BufferPool(device, memory)
            dws = [zg.upload(device, pool, w) for w in ws]
            dbs = [zg.upload(device, pool, b) for b in bs]
            dx = pool.alloc([bsz, hid])
            x_host = torch.from_numpy(x).pin_memory()
            y_host = torch.empty((bsz, hid), pin_memory=True)

            def step():
                device.write_buffer_ptr(dx.buffer, 0, x_host.data_ptr(), bsz * hid * 4)
                h, prev = dx, None
                for w, b in zip(dws, dbs):
                    h = gemm.gemm_bias_relu(device, pool, 1.0, h, w, b)
                    if prev is not None:
                        pool.free(prev)  # reused in stream order by the next layer
                    prev = h
                if memory == zg.MemoryUsage.GpuOnly:
                    _, sub = zg.download_async(device, h, y_host)
                    sub.wait(60.0)
                else:
                    device.read_buffer_ptr(h.buffer, 0, y_host.data_ptr(), bsz * hid * 4)
                pool.free(h)

            for _ in range(2):
                step()
            t = time.perf_counter()
            for _ in range(steps):
                step()
            dt = (time.perf_counter() - t) / steps
            ys[memory] = y_host.numpy().copy()
            out["gpu_only" if memory == zg.MemoryUsage.GpuOnly else "upload"] = {
                "ms_per_step": dt * 1e3,
                "tflops": layers * 2.0 * bsz * hid * hid / dt / 1e12}
            pool.close()
    finally:
        device.close()
        torch.cuda.set_device(torch.cuda.current_device())
    out["bit_identical"] = bool(np.array_equal(ys[zg.MemoryUsage.Upload].view(np.uint32),
                                               ys[zg.MemoryUsage.GpuOnly].view(np.uint32)))
    out["h2d_bytes_per_step"] = bsz * hid * 4
    out["d2h_bytes_per_step"] = bsz * hid * 4
    out["clock"] = "host clock around write X -> 4 x gemm_bias_relu -> read Y"
    return out


def mlp_workload(args, torch, zg, K, mode, peaks, peak_src, world):
    r = mlp_measure(torch, K, mode, args.steps, args.warmup)
    return {
        "metric": METRIC, "value": r["tflops_fused"], "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": r["fused_ms"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"op_graph_lower MLP 4 x relu(X@W+b), 4096x4096, {args.mode}",
                   "unfused_ms_per_step": r["unfused_ms"],
                   "speedup_fused_vs_unfused": r["speedup_fused_vs_unfused"]},
        "gpu_launches": r["launches_fused"],
        "clocks": r["clocks"],
        "packed_weights": {"ms_per_step": r["fused_packed_weights_ms"],
                           "tflops": r["tflops_fused_packed_weights"],
                           "bit_equal_to_fused": r["packed_weights_bit_equal_to_fused"],
                           "clocks": r["packed_weights_clocks"],
                           "what": "weights packed once beforehand (packed-operand API); "
                                   "each layer packs its activations and runs the kernel"},
    }


if __name__ == "__main__":
    sys.exit(main())
