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
  e2e         the same GEMM through the drop-in API (CudaDevice + BufferPool +
              GemmKernel at N=1; torch tensors + dist at N>1) with host
              buffers: pinned H2D of A and B, GEMM, D2H of C, every step
  roofline    the tcgen05 kernel alone against its mode's tensor ceiling
  cpu_baseline the CPU backend's algorithm (the oracle's C restatement of
              zengpu-cpu's loop) on a bounded row sample, all host cores
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
#   --set full -k regex:sgemm_tc_kernel on `bench.py --steps 1 --warmup 3 --no-extras`
#   --section MemoryWorkloadAnalysis -k regex:stream_vec_kernel on the elementwise workload
# Keyed by the kernel and the per-rank GEMM size (M = N = K) or element count.
NCU_TRAFFIC = {
    ("sgemm_tc_pair_kernel<4>", 8192): 4.179e9,
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


def cpu_gemm_sample(m: int, n: int, k: int, seconds: float, seed: int = 2) -> dict:
    """Times the CPU backend's row -> col -> k loop (zengpu-cpu via the oracle)
    on whole rows of C, all host cores, about `seconds` of work."""
    import numpy as np
    O = _oracle()
    threads = os.cpu_count() or 1
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


def gemm_workload(args, torch, dist, zg, K, mode, peaks, peak_src, rank, local_rank, world):
    s = args.size
    if args.workload == "sharded":
        m_total, n, k = 32768, 32768, 8192
        from zengpu_b200.dist import row_range
        r0, r1 = row_range(m_total, world, rank)
        m_local = r1 - r0
        scaling, workload = "strong", f"sgemm {args.mode} M=N=32768 K=8192 row-sharded over {world}"
    else:
        m_local, n, k = s, s, s
        m_total = s * world
        scaling = "weak"
        workload = f"sgemm {args.mode} M=N=K={s} per GPU (M={m_total} total, A/C row blocks)"

    a = torch.empty((m_local, k), device="cuda")
    b = torch.empty((k, n), device="cuda")
    c = torch.empty((m_local, n), device="cuda")
    K.fill_uniform(a, 2 + 7919 * rank)
    if rank == 0:
        K.fill_uniform(b, 1002)
    else:
        b.zero_()
    ws_bytes = K.workspace_bytes(mode, m_local, n, k)
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device="cuda")
    lib = zg.load_library()
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)

    def check(rc):
        zg.api.check(rc)

    def local_gemm(ev0=None, ev1=None):
        check(lib.zg_sgemm_prepare(int(mode), m_local, n, k, a.data_ptr(), b.data_ptr(),
                                   ws.data_ptr(), ws.numel(), sp))
        if ev0 is not None:
            ev0.record(stream)
        check(lib.zg_sgemm_compute(int(mode), m_local, n, k, 1.0, a.data_ptr(), b.data_ptr(),
                                   c.data_ptr(), None, 0, ws.data_ptr(), ws.numel(), sp))
        if ev1 is not None:
            ev1.record(stream)

    chain = None
    if world > 1 and args.bcast == "chain":
        # B is packed once on rank 0 and pushed rank to rank by the copy engines
        # while every rank's GEMM runs, gated per chunk (dist.ChainedGemm).
        from zengpu_b200.dist import ChainedGemm
        chain = ChainedGemm(k, n, mode=int(mode), src=0, chunk_cols=args.chunk_cols or None)
        panels = 1

        def step(ev0=None, ev1=None):
            chain.step(a, b if rank == 0 else None, c)
    elif world > 1:
        # B arrives from rank 0 in column panels; panel j+1 crosses NVLink while
        # panel j is multiplied (dist.ShardedGemm.sgemm_rows_pipelined).
        from zengpu_b200.dist import ShardedGemm
        sg = ShardedGemm(mode=int(mode))
        panels = max(1, args.panels)

        def step(ev0=None, ev1=None):
            sg.sgemm_rows_pipelined(a, b, src=0, panels=panels, out=c)
    else:
        panels = 1
        step = local_gemm

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if K.kernel_status() != 0:
        raise RuntimeError("bounded on-device wait expired during warm-up")

    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    with ClockSampler(local_rank) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0.record(stream)
        for i in range(args.steps):
            step(*kev[i])
        t1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms_local = t0.elapsed_time(t1) / args.steps
    if K.kernel_status() != 0:
        raise RuntimeError("bounded on-device wait expired during timing")
    if world > 1 and rank != 0:
        # B reached this rank only through the broadcast; the accuracy check and
        # the kernel-only timing use the same B, regenerated from its seed
        K.fill_uniform(b, 1002)
    # the last timed step's C of every rank, checked before anything rewrites it
    accuracy = sampled_accuracy(torch, dist, a, b, c, mode, world)
    chain_desc = None
    if chain is not None:
        chain_desc = (chain.chunks, chain.chunk_cols)
        chain.close()
    if world > 1:
        # the dominant kernel alone: one full-shard launch per rank, same stream
        for _ in range(2):
            local_gemm()
        for i in range(min(args.steps, 5)):
            local_gemm(*kev[i])
        torch.cuda.synchronize()
        kern_ms_local = statistics.mean(e0.elapsed_time(e1) for e0, e1 in kev[:min(args.steps, 5)])
    else:
        kern_ms_local = statistics.mean(e0.elapsed_time(e1) for e0, e1 in kev)
    ms = _max_over_ranks(torch, dist, world, ms_local)
    ms_by_rank = _gather_floats(torch, dist, world, ms_local)
    kern_ms = _max_over_ranks(torch, dist, world, kern_ms_local)
    if K.kernel_status() != 0:
        raise RuntimeError("bounded on-device wait expired in the kernel-only timing")
    other = {}
    fp32_class = {"tf32x3": zg.GemmMode.TF32X3, "tf32bf16": zg.GemmMode.TF32_BF16X2,
                  "bf16x3": zg.GemmMode.BF16X3}
    if not args.no_extras and args.workload == "gemm" and mode in fp32_class.values():
        # the other fp32-accurate modes' kernels on the same operands, for comparison
        for name, other_mode in fp32_class.items():
            if other_mode != mode:
                other[name] = kernel_only(torch, lib, other_mode, a, b, c, m_local, n, k, sp,
                                          stream, dist, world)
    total_flops = 2.0 * m_total * n * k
    value = total_flops / (ms * 1e-3) / 1e12
    rank_flops = 2.0 * m_local * n * k
    achieved = rank_flops / (kern_ms * 1e-3) / 1e12
    tf32_peak = peaks["bf16_tflops"] / 2.0
    fp32_simt_peak = 148 * 128 * 2 * 1.965e9 / 1e12  # SMs x FP32 lanes x FMA x max clock
    # TF32_BF16X2: one tf32 product + two bf16 products at twice the tf32 rate;
    # BF16X3: three bf16 products
    peak = {zg.GemmMode.TF32X3: tf32_peak / 3.0, zg.GemmMode.TF32: tf32_peak,
            zg.GemmMode.SIMT_FP32: fp32_simt_peak,
            zg.GemmMode.TF32_BF16X2: tf32_peak / 2.0,
            zg.GemmMode.BF16X3: peaks["bf16_tflops"] / 3.0}[mode]
    # N = 1: TF32X3 split(A) + transpose-split(B) + tcgen05 kernel; TF32:
    # transpose(B) (+ a pitched copy of A when k % 4 != 0) + kernel; SIMT: one.
    # N > 1, chain (rank 0): pack(B) in one launch that flags each chunk, then
    # pack(A) + kernel; nccl: pack(A) + per column panel pack(B panel) + kernel.
    if chain_desc is not None:
        launches_per_step = 3
    elif world > 1:
        launches_per_step = 1 + 2 * panels
    else:
        launches_per_step = {zg.GemmMode.TF32X3: 3, zg.GemmMode.TF32: 2 + (k % 4 != 0),
                             zg.GemmMode.SIMT_FP32: 1, zg.GemmMode.TF32_BF16X2: 3,
                             zg.GemmMode.BF16X3: 3}[mode]

    extras = {}
    e2e = None
    cpu = None
    if not args.no_extras:
        del ws
        torch.cuda.empty_cache()
        e2e = gemm_e2e(args, torch, dist, zg, K, mode, m_local, n, k, m_total, world, local_rank)
        extras["elementwise"] = elementwise_bench(torch, K, peaks["hbm_gbs"])
        if world == 1 and rank == 0:
            cpu = cpu_gemm_sample(m_total, n, k, seconds=12.0)
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: A, B uniform[-1,1) from the splitmix64 generator (seeds 2, 1002)",
        "config": {"workload": workload, "m": m_total, "n": n, "k": k, "mode": args.mode,
                   "parallelism": (f"dp{world} (A/C row blocks; B packed on rank 0 and pushed "
                                   f"rank to rank over NVLink by the copy engines in "
                                   f"{chain_desc[0]} chunks of {chain_desc[1]} columns, each "
                                   f"rank's GEMM gated per chunk)" if chain_desc is not None else
                                   f"dp{world} (A/C row blocks, B broadcast over NCCL in "
                                   f"{panels} column panels)" if world > 1 else
                                   "dp1 (one GPU, no exchange)"),
                   "l2": f"inputs larger than L2: A {m_local * k * 4 >> 20} MiB, B {k * n * 4 >> 20} MiB, "
                         f"packed operands {algorithmic_bytes(mode, m_local, n, k) - 4 * m_local * n >> 20} MiB"},
        "roofline": {"bound": "tensor" if mode != zg.GemmMode.SIMT_FP32 else "fp32",
                     "kernel": tc_kernel_name(torch, int(mode), m_local, n, k),
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak,
                     "traffic": NCU_TRAFFIC.get((tc_kernel_name(torch, int(mode), m_local, n, k), s))
                     if args.workload == "gemm" else None,
                     "algorithmic_bytes": algorithmic_bytes(mode, m_local, n, k),
                     "kernel_ms": kern_ms,
                     "peak_basis": (f"{peak_src} bf16 {peaks['bf16_tflops']} TFLOP/s / 3 "
                                    "(three bf16 MMAs per useful product)"
                                    if mode == zg.GemmMode.BF16X3 else
                                    f"{peak_src} bf16 {peaks['bf16_tflops']} TFLOP/s / 2 (tf32 "
                                    "rate)" + {zg.GemmMode.TF32X3: " / 3 (tf32 MMAs per useful "
                                               "product)",
                                               zg.GemmMode.TF32_BF16X2: " / 2 (one tf32 + two "
                                               "half-cost bf16 MMAs per useful product)"}
                                    .get(mode, ""))
                     if mode != zg.GemmMode.SIMT_FP32 else
                     "nominal FP32 SIMT: 148 SMs x 128 lanes x 2 flop x 1965 MHz"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks.summary(),
    }
    if world > 1:
        line["ms_per_step_by_rank"] = ms_by_rank
    line["accuracy"] = accuracy
    if other:
        line["other_modes"] = other
    if e2e is not None:
        line["e2e"] = e2e
    if cpu is not None:
        line["cpu_baseline"] = {"value": cpu["value"], "unit": cpu["unit"], "cores": cpu["cores"],
                                "kind": "port", "sample": cpu["sample"]}
    line.update(extras)
    return line


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
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(reps + 2)]
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
    """The GEMM through the drop-in API with host buffers, H2D + D2H every step."""
    ha = torch.empty((m_local, k), pin_memory=True)
    hb = torch.empty((k, n), pin_memory=True)
    hc = torch.empty((m_local, n), pin_memory=True)
    tmp = torch.empty((m_local, k), device="cuda")
    K.fill_uniform(tmp, 2)
    ha.copy_(tmp)
    tmp = torch.empty((k, n), device="cuda")
    K.fill_uniform(tmp, 1002)
    hb.copy_(tmp)
    del tmp
    torch.cuda.synchronize()
    steps = max(3, min(args.steps, 5))
    h2d = ha.numel() * 4 + hb.numel() * 4
    d2h = hc.numel() * 4
    if world == 1:
        device = zg.CudaDevice(local_rank)
        gemm = zg.GemmKernel(device, mode)

        def step():
            gemm.sgemm_host(device, 1.0, ha, hb, hc, m_local, n, k)

        for _ in range(2):
            step()
        t = time.perf_counter()
        for _ in range(steps):
            step()
        dt = (time.perf_counter() - t) / steps
        device.close()
        clock = ("host clock around GemmKernel.sgemm_host (synchronous; B up, then row "
                 "panels of A up / GEMM / C down overlapped on three streams)")
    else:
        a = torch.empty((m_local, k), device="cuda")
        b = torch.empty((k, n), device="cuda")
        c = torch.empty((m_local, n), device="cuda")
        rank = dist.get_rank()
        stream = torch.cuda.current_stream()
        chain = None
        if args.bcast == "chain":
            from zengpu_b200.dist import ChainedGemm
            chain = ChainedGemm(k, n, mode=int(mode), src=0, chunk_cols=args.chunk_cols or None)

            def gemm_rows():
                chain.step(a, b if rank == 0 else None, c)
        else:
            from zengpu_b200.dist import ShardedGemm
            sg = ShardedGemm(mode=int(mode))

            def gemm_rows():
                sg.sgemm_rows_pipelined(a, b, src=0, panels=max(1, args.panels), out=c)

        def step():
            a.copy_(ha, non_blocking=True)
            if rank == 0:
                b.copy_(hb, non_blocking=True)
            gemm_rows()
            hc.copy_(c, non_blocking=True)

        for _ in range(2):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        dt = _max_over_ranks(torch, dist, world, e0.elapsed_time(e1) / steps / 1e3)
        if chain is not None:
            chain.close()
        h2d = ha.numel() * 4 + (hb.numel() * 4 if rank == 0 else 0)
        clock = "CUDA events on the compute stream, max over ranks"
    total_flops = 2.0 * m_total * n * k
    return {"value": total_flops / dt / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": dt * 1e3, "steps": steps, "clock": clock}


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


def mlp_workload(args, torch, zg, K, mode, peaks, peak_src, world):
    """op_graph_lower MLP: 4 x (Y = ReLU(X @ W + b)), batch 4096, hidden 4096;
    fused epilogue vs the unfused gemm -> add(broadcast bias) -> relu chain."""
    import math
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

    res = {}
    clock_summary = None
    for name, fn in (("fused", fused), ("unfused", unfused)):
        for _ in range(args.warmup):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        with ClockSampler(torch.cuda.current_device()) as clocks:
            e0.record(stream)
            for _ in range(args.steps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize()
        res[name] = e0.elapsed_time(e1) / args.steps
        if name == "fused":
            clock_summary = clocks.summary()
    flops = layers * 2.0 * bsz * hid * hid
    return {
        "metric": METRIC, "value": flops / (res["fused"] * 1e-3) / 1e12, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["fused"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"op_graph_lower MLP 4 x relu(X@W+b), 4096x4096, {args.mode}",
                   "unfused_ms_per_step": res["unfused"],
                   "speedup_fused_vs_unfused": res["unfused"] / res["fused"]},
        # per layer: TF32X3 / TF32_BF16X2 / BF16X3 pack A, pack B, kernel; TF32 transpose B,
        # kernel; SIMT one kernel
        "gpu_launches": args.steps * layers * {1: 3, 2: 2, 3: 3, 4: 3}.get(int(mode), 1),
        "clocks": clock_summary,
    }


if __name__ == "__main__":
    sys.exit(main())
