"""Multi-GPU sharding of the hot path: one process per GPU.

The reference has no collective (its only multi-device op is a HIP peer
copy, zengpu-hip/src/lib.rs:609-710); large problems here shard naturally:

* GEMM: A and C are split into contiguous M-row blocks, one per rank; every
  rank needs all of B - the only exchange on the path.  By default
  (ChainedGemm) B is packed once on its owner and carried rank to rank over
  NVLink by the copy engines while every rank's GEMM already runs; ShardedGemm
  broadcasts it over NCCL instead.  C stays sharded; gather_rows() assembles
  it only when a caller asks for the whole matrix.
* elementwise add / ReLU: contiguous chunks, no collective at all.

torch.distributed supplies the process group (NCCL on GPUs, gloo for the CPU
tests); the per-shard compute is libzengpu_b200's own kernels.
"""
from __future__ import annotations

import os
import time
from typing import Callable

import torch
import torch.distributed as dist


def row_range(m: int, world: int, rank: int) -> tuple[int, int]:
    """[row0, row1) of rank's M-row block: sizes differ by at most one row,
    the larger blocks first."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(m, world)
    row0 = rank * base + min(rank, extra)
    return row0, row0 + base + (1 if rank < extra else 0)


def chunk_range(n: int, world: int, rank: int, align: int = 4) -> tuple[int, int]:
    """[i0, i1) of rank's chunk of an n-element vector, chunk starts aligned to
    `align` elements (16 bytes for f32) so every shard keeps vector loads."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    units = (n + align - 1) // align
    u0, u1 = row_range(units, world, rank)
    return min(u0 * align, n), min(u1 * align, n)


def panel_count(m: int, n: int, tile_m: int = 128, tile_n: int = 256,
                min_tiles: int = 900, max_panels: int = 8) -> int:
    """Column panels for the pipelined broadcast: as many as possible (up to
    max_panels) while each panel's GEMM still fills the GPU with at least
    min_tiles output tiles (about six waves of 148 SMs)."""
    tiles_m = (m + tile_m - 1) // tile_m
    best = 1
    for p in range(1, max_panels + 1):
        w = (n + p - 1) // p
        if tiles_m * ((w + tile_n - 1) // tile_n) >= min_tiles:
            best = p
    return best


def _default_compute(a, b, alpha, bias, relu, mode, out):
    from . import kernels
    return kernels.sgemm(a, b, mode=mode, alpha=alpha, bias=bias, relu=relu, out=out)


class ShardedGemm:
    """C[row0:row1] = epilogue(alpha * A[row0:row1] @ B) on every rank."""

    def __init__(self, group=None, mode: int = 1,
                 compute: Callable | None = None, ops=None):
        """compute: per-shard GEMM for sgemm_rows (default: the library's).
        ops: object with pack_a / pack_b / sgemm_packed for the pipelined path
        (default: zengpu_b200.kernels); the CPU tests pass a stand-in."""
        self.group = group
        self.mode = mode
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.compute = compute or _default_compute
        self.ops = ops

    def broadcast_b(self, b: torch.Tensor, src: int = 0) -> torch.Tensor:
        """Broadcasts B (same shape and dtype on every rank) from `src`."""
        dist.broadcast(b, src=src, group=self.group)
        return b

    def sgemm_rows(self, a_rows: torch.Tensor, b: torch.Tensor, src: int = 0,
                   alpha: float = 1.0, bias: torch.Tensor | None = None,
                   relu: bool = False, out: torch.Tensor | None = None,
                   broadcast: bool = True) -> torch.Tensor:
        if a_rows.dim() != 2 or b.dim() != 2 or a_rows.shape[1] != b.shape[0]:
            raise ValueError(f"sgemm_rows: bad shapes {tuple(a_rows.shape)} @ {tuple(b.shape)}")
        if broadcast:
            self.broadcast_b(b, src)
        return self.compute(a_rows, b, alpha, bias, relu, self.mode, out)

    def sgemm_rows_pipelined(self, a_rows: torch.Tensor, b: torch.Tensor, src: int = 0,
                             panels: int | None = None, alpha: float = 1.0,
                             bias: torch.Tensor | None = None, relu: bool = False,
                             out: torch.Tensor | None = None) -> torch.Tensor:
        """C[row0:row1] = epilogue(alpha * A[row0:row1] @ B) with B broadcast in
        column panels: the broadcast of panel j+1 runs on NCCL's stream while
        panel j is multiplied, so only the first panel's transfer is exposed.

        B must have its full shape on every rank (contents only on `src`).  A is
        packed once; each panel of B is packed as it arrives and multiplied
        into its column panel of C (row pitch n)."""
        if self.ops is None:
            from . import kernels as K
        else:
            K = self.ops

        k, n = b.shape
        m = a_rows.shape[0]
        if a_rows.dim() != 2 or a_rows.shape[1] != k:
            raise ValueError(f"bad shapes {tuple(a_rows.shape)} @ {tuple(b.shape)}")
        if panels is None:
            panels = panel_count(m, n)
        widths = [row_range(n, panels, j) for j in range(panels)]
        c = out if out is not None else torch.empty((m, n), dtype=torch.float32,
                                                    device=a_rows.device)
        # NCCL moves contiguous buffers: with one panel B itself is broadcast in
        # place; otherwise each column panel gets its own staging buffer
        # (together the size of B), so no panel waits for another's reuse.
        if panels == 1 and b.is_contiguous():
            bufs = [b]
        else:
            bufs = [torch.empty((k, j1 - j0), dtype=b.dtype, device=b.device)
                    for j0, j1 in widths]
        packed_b = None

        def issue(j):
            j0, j1 = widths[j]
            buf = bufs[j]
            if self.rank == src and buf is not b:
                buf.copy_(b[:, j0:j1])
            return dist.broadcast(buf, src=src, group=self.group, async_op=True), buf

        # The first transfer is issued before A is packed, so packing A (no
        # dependence on B) runs while panel 0 crosses NVLink.
        pending = issue(0)
        pa = K.pack_a(a_rows, self.mode)
        for j in range(panels):
            work, buf = pending
            work.wait()  # the compute stream waits for panel j
            if j + 1 < panels:
                pending = issue(j + 1)  # panel j+1 overlaps panel j's GEMM
            j0, j1 = widths[j]
            packed_b = K.pack_b(buf, self.mode,
                                out=packed_b.buf if packed_b is not None else None)
            K.sgemm_packed(pa, packed_b, c[:, j0:j1], alpha=alpha,
                           bias=bias[j0:j1] if bias is not None else None, relu=relu)
        return c

    def gather_rows(self, c_rows: torch.Tensor, m: int) -> torch.Tensor:
        """All-gathers the row blocks into the full [m, n] C on every rank."""
        n = c_rows.shape[1]
        counts = [row_range(m, self.world, r) for r in range(self.world)]
        rows_max = max(r1 - r0 for r0, r1 in counts)
        padded = torch.zeros((rows_max, n), dtype=c_rows.dtype, device=c_rows.device)
        padded[: c_rows.shape[0]] = c_rows
        parts = [torch.empty_like(padded) for _ in range(self.world)]
        dist.all_gather(parts, padded, group=self.group)
        return torch.cat([p[: r1 - r0] for p, (r0, r1) in zip(parts, counts)], dim=0)


def chain_neighbours(rank: int, world: int, src: int = 0) -> tuple[int | None, int | None]:
    """(previous, next) rank of `rank` in the broadcast chain src -> src+1 ->
    ... (mod world); None at the chain's two ends."""
    if world <= 0 or not 0 <= rank < world or not 0 <= src < world:
        raise ValueError(f"bad rank {rank} / src {src} of {world}")
    pos = (rank - src) % world
    prev = (rank - 1) % world if pos > 0 else None
    nxt = (rank + 1) % world if pos < world - 1 else None
    return prev, nxt


def default_chunk_cols(n: int, k: int, target_bytes: int = 16 << 20, bytes_per_elem: int = 8) -> int:
    """Columns of B per chunk of the chained broadcast: a multiple of 256 whose
    packed size is about `target_bytes` (large enough for a copy engine to run
    near NVLink speed, small enough that the last rank starts early)."""
    cols = max(256, (target_bytes // max(1, k * bytes_per_elem)) // 256 * 256)
    return min(cols, ((n + 255) // 256) * 256)


class ChainBroken(RuntimeError):
    """The B chain can no longer run steps: a neighbouring rank exited, or a
    step did not finish within the deadline."""


def pid_alive(pid: int) -> bool:
    """True while process `pid` runs on this host (a zombie counts as exited)."""
    try:
        os.kill(pid, 0)
    except ProcessLookupError:
        return False
    except PermissionError:
        return True
    try:
        with open(f"/proc/{pid}/stat", "rb") as f:
            state = f.read().rsplit(b")", 1)[1].split()[0]
        return state not in (b"Z", b"X")
    except (OSError, IndexError):
        return True


class ChainGuard:
    """Host-side failure detection of the B chain, checked before each step is
    launched so that no step is queued toward a rank that has gone.

    * Neighbours: the chain moves data only between neighbouring ranks of one
      host (CUDA IPC), so a neighbour that left is one whose process no longer
      runs (pids exchanged when the chain is built).
    * Deadline: step e is launched only after step e - 2 (the last step that
      used the same buffers) completed; a step that does not complete within
      `deadline_s` means a peer stopped taking part.
    `events[e]` is any object with query() -> bool (a CUDA event in use, a
    stand-in in the CPU tests)."""

    def __init__(self, rank: int, pids: list[int], prev: int | None, nxt: int | None,
                 deadline_s: float = 30.0, alive: Callable[[int], bool] = pid_alive):
        self.rank, self.pids, self.prev, self.next = rank, list(pids), prev, nxt
        self.deadline_s = deadline_s
        self.alive = alive
        self.events: dict[int, object] = {}

    def gone_neighbours(self) -> list[int]:
        return [r for r in (self.prev, self.next) if r is not None and not self.alive(self.pids[r])]

    def in_flight(self) -> bool:
        return any(not ev.query() for ev in self.events.values())

    def check_neighbours(self) -> None:
        gone = self.gone_neighbours()
        if gone:
            raise ChainBroken(f"rank {self.rank}: chain neighbour rank {gone[0]} "
                              f"(pid {self.pids[gone[0]]}) has exited")

    def wait(self, epoch: int, deadline_s: float | None = None) -> None:
        """Waits until step `epoch` (if it was launched) completed; raises
        ChainBroken after the deadline."""
        ev = self.events.get(epoch)
        if ev is None:
            return
        limit = time.monotonic() + (self.deadline_s if deadline_s is None else deadline_s)
        pause = 1e-5
        while not ev.query():
            if time.monotonic() > limit:
                raise ChainBroken(f"rank {self.rank}: step {epoch} did not complete within "
                                  f"{self.deadline_s:g} s (a peer stopped taking part)")
            time.sleep(pause)
            pause = min(pause * 2, 1e-3)

    def wait_all(self, deadline_s: float | None = None) -> None:
        for e in sorted(self.events):
            self.wait(e, deadline_s)

    def launched(self, epoch: int, ev) -> None:
        self.events[epoch] = ev
        for e in [e for e in self.events if e <= epoch - 2]:
            del self.events[e]


class ChainedGemm:
    """C[row0:row1] = epilogue(alpha * A[row0:row1] @ B) on every rank, with B
    carried from rank `src` along the chain src -> src+1 -> ... by the copy
    engines while every rank's GEMM already runs (zg_bchain_* in the C ABI).

    B is packed once, on `src`, into the tensor-core operand form; chunks of
    it hop rank to rank over NVLink, and each rank's GEMM waits per output
    tile only for the chunk that tile reads.  No SM is spent on the transfer,
    and no collective library is on the data path.  The process group is used
    once, to exchange the CUDA IPC handles of the chain buffers.

    Failures (ChainGuard): before each step, both chain neighbours must still
    run and step e - 2 must have completed within `deadline_s`.  A neighbour
    that exited with none of this rank's work in flight ends the chain at
    once.  A deadline that expires while the neighbours still run opens this
    rank's waits (zg_bchain_abort) so its queued work drains, then ends the
    chain.  Either way step() raises ChainBroken and every later step does
    too; the chain's device memory stays allocated until the process exits,
    since a neighbour that still runs may yet write into it.  If a neighbour
    exits while this rank's work is still in flight, that work is not
    released (it would copy into the exited rank's memory): its streams stay
    blocked and the process should exit."""

    def __init__(self, k: int, n: int, mode: int = 3, group=None, src: int = 0,
                 chunk_cols: int | None = None, lib=None, ops=None, deadline_s: float = 30.0):
        import ctypes as C

        from . import _lib as L
        from .api import check

        self._C, self._check = C, check
        self.lib = lib if lib is not None else L.load()
        if ops is None:
            from . import kernels as ops
        self.ops = ops
        self.group, self.src, self.mode, self.k, self.n = group, src, int(mode), k, n
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        bpe = 4 if self.mode in (2, 4) else 8  # packed bytes per element of B
        self.chunk_cols = chunk_cols or default_chunk_cols(n, k, bytes_per_elem=bpe)
        self.chunks = (n + self.chunk_cols - 1) // self.chunk_cols
        self.prev, self.next = chain_neighbours(self.rank, self.world, src)

        handle = (C.c_uint8 * 64)()
        ptr = C.c_void_p()
        check(self.lib.zg_bchain_create(self.mode, k, n, self.chunk_cols, C.byref(ptr), handle))
        self.chain = ptr
        everyone = [None] * self.world
        dist.all_gather_object(everyone, (bytes(handle), (self.mode, k, n, self.chunk_cols),
                                          os.getpid()), group=group)
        if any(cfg != everyone[self.rank][1] for _, cfg, _ in everyone):
            self.lib.zg_bchain_destroy(self.chain)
            raise ValueError(f"ChainedGemm: ranks disagree on (mode, k, n, chunk): "
                             f"{[cfg for _, cfg, _ in everyone]}")

        def buf(r):
            return None if r is None else (C.c_uint8 * 64).from_buffer_copy(everyone[r][0])

        check(self.lib.zg_bchain_connect(self.chain, buf(self.prev), buf(self.next)))
        dist.barrier(group=group)
        self.copy_stream = torch.cuda.Stream() if torch.cuda.is_available() else None
        self.epoch = 0
        self._packed_a = None
        self.guard = ChainGuard(self.rank, [p for _, _, p in everyone], self.prev, self.next,
                                deadline_s)
        self.broken: str | None = None
        self._new_event = torch.cuda.Event  # completion marker of each step

    def step(self, a_rows: torch.Tensor, b: torch.Tensor | None, out: torch.Tensor,
             alpha: float = 1.0, bias: torch.Tensor | None = None,
             relu: bool = False) -> torch.Tensor:
        """One sharded GEMM.  `b` [k, n] is read on `src` only (others may pass
        None); `out` [rows, n] (row pitch out.stride(0)) receives this rank's
        rows of C."""
        C = self._C
        if a_rows.dim() != 2 or a_rows.shape[1] != self.k:
            raise ValueError(f"ChainedGemm: A rows must be [m, {self.k}]")
        m = a_rows.shape[0]
        if tuple(out.shape) != (m, self.n) or out.stride(1) != 1:
            raise ValueError(f"ChainedGemm: out must be [{m}, {self.n}] with unit column stride")
        is_src = self.rank == self.src
        if is_src and (b is None or tuple(b.shape) != (self.k, self.n) or b.stride(1) != 1):
            raise ValueError(f"ChainedGemm: the source rank needs B [{self.k}, {self.n}]")
        if bias is not None and (bias.numel() != self.n or not bias.is_contiguous()):
            raise ValueError(f"ChainedGemm: bias must be a contiguous [{self.n}] vector")
        if self.broken:
            raise ChainBroken(self.broken)
        # before anything of step e is queued: both neighbours still run, and
        # step e - 2, the last user of this step's buffers, has completed
        try:
            self.guard.check_neighbours()
            self.guard.wait(self.epoch - 1)
        except ChainBroken as exc:
            self._fail(str(exc))
        # every check is done: from here on each rank enqueues the same step e
        self.epoch += 1
        e = self.epoch & 0xFFFFFFFF
        compute = torch.cuda.current_stream()
        cs = C.c_void_p(compute.cuda_stream)
        copy = C.c_void_p(self.copy_stream.cuda_stream)
        if is_src:
            # packs chunk by chunk; each chunk's flag lets the copy stream push it on
            self._check(self.lib.zg_bchain_source(self.chain, e, b.data_ptr(), b.stride(0), cs))
        self._check(self.lib.zg_bchain_forward(self.chain, e, copy))
        self._packed_a = self.ops.pack_a(
            a_rows, self.mode, out=self._packed_a.buf if self._packed_a is not None else None)
        self._check(self.lib.zg_bchain_gemm(
            self.chain, e, 0 if is_src else 1, m, float(alpha), self._packed_a.buf.data_ptr(),
            out.data_ptr(), out.stride(0), bias.data_ptr() if bias is not None else None,
            1 if relu else 0, cs))
        # this rank's buffer of step e is free once its GEMM and its forwarding are done
        compute.wait_stream(self.copy_stream)
        self._check(self.lib.zg_bchain_release(self.chain, e, cs))
        ev = self._new_event()
        ev.record(compute)
        self.guard.launched(self.epoch, ev)
        return out

    def _fail(self, reason: str) -> None:
        """Ends the chain after a failure found on the host and raises."""
        if self.guard.in_flight():
            if self.guard.gone_neighbours():
                self.broken = (reason + "; this rank's queued steps wait on the exited rank and "
                               "are not released (they would write into its memory): exit "
                               "this process")
                raise ChainBroken(self.broken)
            # the neighbours still run: open this rank's waits so its queued
            # work ends (results of those steps are invalid), bounded
            self._check(self.lib.zg_bchain_abort(self.chain, self.epoch & 0xFFFFFFFF))
            try:
                self.guard.wait_all()
            except ChainBroken as exc:
                self.broken = f"{reason}; after the abort: {exc}"
                raise ChainBroken(self.broken) from None
        # a gate that gave up on the device set the status word: clear it, the
        # failure is reported here
        code = self._C.c_uint32(0)
        self.lib.zg_kernel_status(self._C.byref(code))
        self.broken = reason
        raise ChainBroken(reason)

    def packed_b(self, epoch: int | None = None) -> tuple[int, int]:
        """(device pointer, bytes) of the packed B^T buffer of a step."""
        C = self._C
        p, nb = C.c_void_p(), C.c_uint64()
        e = (self.epoch if epoch is None else epoch) & 0xFFFFFFFF
        self._check(self.lib.zg_bchain_buffer(self.chain, e, C.byref(p), C.byref(nb)))
        return p.value, nb.value

    def close(self) -> None:
        """Frees the chain after every rank is done with every step (collective:
        every rank calls it).  A chain that failed keeps its memory (see the
        class docstring) and is not freed here."""
        if self.chain is None or self.broken:
            return
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self._check(self.lib.zg_bchain_destroy(self.chain))
        self.chain = None
