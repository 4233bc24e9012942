"""Stream-level entry points on torch CUDA tensors (layer 3 of the C ABI).

Thin wrappers: shape / dtype / device checks in Python, then one call into
libzengpu_b200 with raw device pointers and torch's current CUDA stream.
torch only supplies device memory and streams here; every kernel that runs
is this library's own sm_100a code.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from .api import GemmMode, check

# One scratch tensor per (device, stream): GEMMs issued on different streams
# may overlap, and each stream reuses its own scratch in stream order.
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def _stream(t: torch.Tensor) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _f32_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
            raise ValueError("expected contiguous float32 CUDA tensors")


def add_f32(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out = a + b, elementwise (bit-exact f32)."""
    _f32_cuda(a, b)
    if a.shape != b.shape:
        raise ValueError(f"add: shape mismatch {tuple(a.shape)} vs {tuple(b.shape)}")
    out = torch.empty_like(a) if out is None else out
    _f32_cuda(out)
    check(L.load().zg_add_f32(a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(), _stream(a)))
    return out


def relu_f32(a: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out = relu(a); pass out=a for the in-place form."""
    _f32_cuda(a)
    out = torch.empty_like(a) if out is None else out
    _f32_cuda(out)
    check(L.load().zg_relu_f32(a.data_ptr(), out.data_ptr(), a.numel(), _stream(a)))
    return out


def saxpy_f32(alpha: float, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    _f32_cuda(x, y)
    check(L.load().zg_saxpy_f32(float(alpha), x.data_ptr(), y.data_ptr(), x.numel(), _stream(x)))
    return y


def sscal_f32(alpha: float, x: torch.Tensor) -> torch.Tensor:
    _f32_cuda(x)
    check(L.load().zg_sscal_f32(float(alpha), x.data_ptr(), x.numel(), _stream(x)))
    return x


def workspace_bytes(mode: int, m: int, n: int, k: int) -> int:
    return int(L.load().zg_sgemm_workspace_bytes(int(mode), m, n, k))


def workspace_for(device: torch.device, nbytes: int) -> torch.Tensor | None:
    """Scratch tensor of the current stream on `device`, grown on demand
    (reused in stream order, so only GEMMs on that stream share it)."""
    if nbytes == 0:
        return None
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, torch.cuda.current_stream(idx).cuda_stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def release_workspaces(device: torch.device | int | None = None) -> int:
    """Drops the cached GEMM scratch tensors (of one device, or of all) and
    returns how many were dropped.  The cache holds one tensor per (device,
    stream) that ever ran sgemm, each the size of that stream's largest GEMM,
    until this is called: code that creates short-lived streams should call it
    once those streams are done.  Dropping a tensor whose GEMM is still queued
    is safe: torch's caching allocator hands its memory out again only in the
    order of the stream it was allocated on (the stream it was cached for)."""
    if device is None:
        n = len(_workspaces)
        _workspaces.clear()
        return n
    idx = device if isinstance(device, int) else (
        device.index if device.index is not None else torch.cuda.current_device())
    keys = [key for key in _workspaces if key[0] == idx]
    for key in keys:
        del _workspaces[key]
    return len(keys)


def sgemm(a: torch.Tensor, b: torch.Tensor, mode: int = GemmMode.TF32X3, alpha: float = 1.0,
          bias: torch.Tensor | None = None, relu: bool = False,
          out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """C = epilogue(alpha * a @ b) for row-major f32 a [m,k], b [k,n]."""
    _f32_cuda(a, b)
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise ValueError(f"sgemm: bad shapes {tuple(a.shape)} @ {tuple(b.shape)}")
    m, k = a.shape
    n = b.shape[1]
    if bias is not None:
        _f32_cuda(bias)
        if bias.numel() != n:
            raise ValueError("sgemm: bias must have n elements")
    out = torch.empty((m, n), dtype=torch.float32, device=a.device) if out is None else out
    _f32_cuda(out)
    need = workspace_bytes(mode, m, n, k)
    ws = workspace if workspace is not None else workspace_for(a.device, need)
    ws_ptr = ws.data_ptr() if ws is not None else None
    ws_len = ws.numel() if ws is not None else 0
    check(L.load().zg_sgemm_f32(int(mode), m, n, k, float(alpha), a.data_ptr(), b.data_ptr(),
                                out.data_ptr(), bias.data_ptr() if bias is not None else None,
                                1 if relu else 0, ws_ptr, ws_len, _stream(a)))
    return out


def fill_uniform(t: torch.Tensor, seed: int, lo: float = -1.0, hi: float = 1.0) -> torch.Tensor:
    _f32_cuda(t)
    check(L.load().zg_fill_uniform_f32(t.data_ptr(), t.numel(), int(seed), float(lo), float(hi),
                                       _stream(t)))
    return t


def fill_normal(t: torch.Tensor, seed: int) -> torch.Tensor:
    _f32_cuda(t)
    check(L.load().zg_fill_normal_f32(t.data_ptr(), t.numel(), int(seed), _stream(t)))
    return t


def kernel_status() -> int:
    """Reads and clears the device status word (0 = every bounded wait finished)."""
    code = C.c_uint32(0)
    check(L.load().zg_kernel_status(C.byref(code)))
    return int(code.value)


# ---- packed operands (zg_sgemm_pack_*, zg_sgemm_packed) ----------------------------
class Packed:
    """An operand packed for one GEMM mode: the planes its kernel reads."""

    def __init__(self, mode: int, operand: int, outer: int, k: int, buf: torch.Tensor):
        self.mode, self.operand, self.outer, self.k, self.buf = int(mode), operand, outer, k, buf


def pack_bytes(mode: int, operand: int, outer: int, k: int) -> int:
    return int(L.load().zg_sgemm_pack_bytes(int(mode), operand, outer, k))


def _pack_buffer(nbytes: int, device, out: torch.Tensor | None) -> torch.Tensor:
    if out is not None and out.numel() >= nbytes and out.data_ptr() % 256 == 0:
        return out
    return torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)


def _pitch(t: torch.Tensor) -> int:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError("expected a 2-D float32 CUDA tensor with unit column stride")
    return t.stride(0)


def pack_a(a: torch.Tensor, mode: int = GemmMode.TF32X3, out: torch.Tensor | None = None) -> Packed:
    """Packs A [m, k] (any row pitch) for `mode`."""
    if a.dtype != torch.float32 or not a.is_cuda:
        raise ValueError("pack_a: float32 CUDA tensor expected")
    m, k = a.shape
    buf = _pack_buffer(pack_bytes(mode, 0, m, k), a.device, out)
    check(L.load().zg_sgemm_pack_a(int(mode), m, k, a.data_ptr(), _pitch(a), buf.data_ptr(),
                                   buf.numel(), _stream(a)))
    return Packed(mode, 0, m, k, buf)


def pack_b(b: torch.Tensor, mode: int = GemmMode.TF32X3, out: torch.Tensor | None = None) -> Packed:
    """Packs B [k, n] (any row pitch) for `mode`."""
    if b.dtype != torch.float32 or not b.is_cuda:
        raise ValueError("pack_b: float32 CUDA tensor expected")
    k, n = b.shape
    buf = _pack_buffer(pack_bytes(mode, 1, n, k), b.device, out)
    check(L.load().zg_sgemm_pack_b(int(mode), k, n, b.data_ptr(), _pitch(b), buf.data_ptr(),
                                   buf.numel(), _stream(b)))
    return Packed(mode, 1, n, k, buf)


def sgemm_packed(pa: Packed, pb: Packed, c: torch.Tensor | None = None, alpha: float = 1.0,
                 bias: torch.Tensor | None = None, relu: bool = False) -> torch.Tensor:
    """C = epilogue(alpha * A @ B) from packed operands; `c` may be a column
    panel view of a larger row-major matrix (row pitch = c.stride(0))."""
    if pa.mode != pb.mode or pa.k != pb.k or pa.operand != 0 or pb.operand != 1:
        raise ValueError("sgemm_packed: operands packed for different GEMMs")
    m, n, k = pa.outer, pb.outer, pa.k
    if c is None:
        c = torch.empty((m, n), dtype=torch.float32, device=pa.buf.device)
    if tuple(c.shape) != (m, n) or c.dtype != torch.float32:
        raise ValueError(f"sgemm_packed: C must be float32 [{m}, {n}]")
    if bias is not None:
        _f32_cuda(bias)
    check(L.load().zg_sgemm_packed(pa.mode, m, n, k, float(alpha), pa.buf.data_ptr(),
                                   pb.buf.data_ptr(), c.data_ptr(), _pitch(c),
                                   bias.data_ptr() if bias is not None else None,
                                   1 if relu else 0, _stream(c)))
    return c
