"""Multi-GPU sharding of the hot path: one process per GPU.

The reference has no collective (its only multi-device op is a HIP peer
copy, zengpu-hip/src/lib.rs:609-710); large problems here shard naturally:

* GEMM: A and C are split into contiguous M-row blocks, one per rank; every
  rank needs all of B, so B is broadcast from its owner over NCCL (NVLink /
  NVSwitch) - the only exchange on the path.  C stays sharded; gather_rows()
  assembles it only when a caller asks for the whole matrix.
* elementwise add / ReLU: contiguous chunks, no collective at all.

torch.distributed supplies the process group (NCCL on GPUs, gloo for the CPU
tests); the per-shard compute is libzengpu_b200's own kernels.
"""
from __future__ import annotations

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


def _default_compute(a, b, alpha, bias, relu, mode, out):
    from . import kernels
    return kernels.sgemm(a, b, mode=mode, alpha=alpha, bias=bias, relu=relu, out=out)


class ShardedGemm:
    """C[row0:row1] = epilogue(alpha * A[row0:row1] @ B) on every rank."""

    def __init__(self, group=None, mode: int = 1,
                 compute: Callable | None = None):
        self.group = group
        self.mode = mode
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.compute = compute or _default_compute

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
