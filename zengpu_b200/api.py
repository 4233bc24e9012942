"""Python mirror of ZenGPU's compute API over libzengpu_b200.

Names, argument meaning and errors follow the reference crates:

* ``CudaDevice``          - GpuDevice compute subset (zengpu-hal/src/device.rs:20-277,
                            zengpu-cuda/src/lib.rs:472-1164)
* ``DeviceArray``         - zengpu-compute/src/lib.rs:21-85
* ``BufferPool``          - zengpu-compute/src/pool.rs:17-89
* ``ElementwiseKernels``  - zengpu-compute/src/elementwise.rs:51-146
* ``GemmKernel``          - zengpu-blas/src/level3.rs:101-182 (+ ``gemm_bias_relu``)
* ``Level1Kernels``, ``Blas`` - zengpu-blas/src/level1.rs:51-139, zengpu-blas/src/lib.rs:51-108

Every call goes through the C ABI; errors come back as ``GpuError`` subclasses
matching ``GpuError`` / ``UsageError`` variants (zengpu-hal/src/error.rs:15-58).
"""
from __future__ import annotations

import ctypes as C
import enum
from typing import Iterable, Sequence

import numpy as np

from . import _lib as L


# ---- errors -------------------------------------------------------------------
class GpuError(Exception):
    code = -1

    def __init__(self, message: str = ""):
        super().__init__(message)
        self.message = message


class DeviceLost(GpuError): code = 1
class Timeout(GpuError): code = 2
class OutOfMemory(GpuError): code = 3
class UnsupportedFeatures(GpuError): code = 4
class Unsupported(GpuError): code = 5
class InvalidUsage(GpuError): pass
class StaleHandle(InvalidUsage): code = 6
class MissingUsage(InvalidUsage): code = 7
class BindingMismatch(InvalidUsage): code = 8
class ShaderCompile(GpuError): code = 9
class PipelineCreation(GpuError): code = 10
class Dispatch(GpuError): code = 11
class Backend(GpuError): code = 12
class NoDevice(GpuError): code = 13
class KernelWait(GpuError): code = 14


_ERRORS = {cls.code: cls for cls in (
    DeviceLost, Timeout, OutOfMemory, UnsupportedFeatures, Unsupported, StaleHandle,
    MissingUsage, BindingMismatch, ShaderCompile, PipelineCreation, Dispatch, Backend,
    NoDevice, KernelWait)}


def check(rc: int) -> None:
    """Raises the GpuError subclass of a non-zero status, with the reference's
    structured fields where the variant has them (zg_last_error_detail):
    StaleHandle.index / expected_gen / actual_gen, MissingUsage.resource /
    needed, OutOfMemory.memory, UnsupportedFeatures.features."""
    if rc == 0:
        return
    err = _ERRORS.get(rc, GpuError)(L.last_error())
    d = L.last_error_detail()
    if d.status == rc:
        if rc == StaleHandle.code:
            err.index, err.expected_gen, err.actual_gen = (d.handle_index, d.expected_gen,
                                                           d.actual_gen)
        elif rc == MissingUsage.code:
            err.resource = (d.resource or b"").decode()
            err.needed = (d.needed or b"").decode()
        elif rc == OutOfMemory.code:
            err.memory = MemoryUsage(d.memory)
        elif rc == UnsupportedFeatures.code:
            err.features = int(d.features)
    raise err


# ---- enums ----------------------------------------------------------------------
class DType(enum.IntEnum):
    """zengpu-hal/src/types.rs:195-230"""
    F32 = 0
    F16 = 1
    Bf16 = 2
    F64 = 3
    I8 = 4
    I16 = 5
    I32 = 6
    I64 = 7
    U8 = 8
    U16 = 9
    U32 = 10
    U64 = 11
    Bool = 12

    def size_bytes(self) -> int:
        return {DType.F64: 8, DType.I64: 8, DType.U64: 8, DType.F32: 4, DType.I32: 4,
                DType.U32: 4, DType.F16: 2, DType.Bf16: 2, DType.I16: 2,
                DType.U16: 2}.get(self, 1)


class BufferUsage(enum.IntFlag):
    STORAGE = 1 << 0
    UNIFORM = 1 << 1
    TRANSFER_SRC = 1 << 5
    TRANSFER_DST = 1 << 6
    READBACK = 1 << 7


class MemoryUsage(enum.IntEnum):
    GpuOnly = 0
    Upload = 1
    Readback = 2


class GemmMode(enum.IntEnum):
    SIMT_FP32 = 0
    TF32X3 = 1
    TF32 = 2
    TF32_BF16X2 = 3
    BF16X3 = 4


class ShaderKind(enum.IntEnum):
    CUBIN = 0
    PTX = 1
    BUILTIN = 2


Handle = L.Handle


def u32(v: int) -> L.Scalar:
    return L.Scalar(0, int(v) & 0xFFFFFFFF)


def i32(v: int) -> L.Scalar:
    return L.Scalar(1, int(v) & 0xFFFFFFFF)


def f32(v: float) -> L.Scalar:
    return L.Scalar(2, int(np.array([v], dtype=np.float32).view(np.uint32)[0]))


def _as_bytes(data) -> tuple[C.c_void_p, int, object]:
    if isinstance(data, (bytes, bytearray)):
        buf = (C.c_char * len(data)).from_buffer_copy(data)
        return C.cast(buf, C.c_void_p), len(data), buf
    arr = np.ascontiguousarray(data)
    return C.c_void_p(arr.ctypes.data), arr.nbytes, arr


# ---- device ---------------------------------------------------------------------------
def device_count() -> int:
    n = C.c_int(0)
    rc = L.load().zg_device_count(C.byref(n))
    if rc == NoDevice.code:
        return 0
    check(rc)
    return n.value


class Submission:
    """GpuSubmission (zengpu-hal/src/submission.rs:22-63)."""

    def __init__(self, ptr: C.c_void_p):
        self._p = ptr

    def poll(self) -> bool:
        done = C.c_int(0)
        check(L.load().zg_submission_poll(self._p, C.byref(done)))
        return bool(done.value)

    def wait(self, timeout_s: float) -> None:
        check(L.load().zg_submission_wait(self._p, int(max(timeout_s, 0.0) * 1e9)))

    def __del__(self):
        if getattr(self, "_p", None):
            L.load().zg_submission_destroy(self._p)
            self._p = None


class CudaDevice:
    """One opened CUDA device (primary context, one non-blocking stream)."""

    def __init__(self, ordinal: int = 0):
        self._lib = L.load()
        p = C.c_void_p()
        check(self._lib.zg_device_open(int(ordinal), C.byref(p)))
        self._p = p

    @property
    def raw(self) -> C.c_void_p:
        return self._p

    def close(self) -> None:
        if self._p:
            self._lib.zg_device_close(self._p)
            self._p = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def device_ordinal(self) -> int:
        return self._lib.zg_device_ordinal(self._p)

    def stream(self) -> int:
        return self._lib.zg_device_stream(self._p) or 0

    def can_peer(self, peer: int) -> bool:
        out = C.c_int(0)
        check(self._lib.zg_device_can_peer(self._p, int(peer), C.byref(out)))
        return bool(out.value)

    # buffers
    def create_buffer(self, size: int, usage: int = BufferUsage.STORAGE | BufferUsage.READBACK,
                      memory: int = MemoryUsage.GpuOnly) -> Handle:
        h = Handle()
        check(self._lib.zg_buffer_create(self._p, int(size), int(usage), int(memory), C.byref(h)))
        return h

    def write_buffer(self, buffer: Handle, offset: int, data) -> None:
        ptr, n, keep = _as_bytes(data)
        check(self._lib.zg_buffer_write(self._p, buffer, int(offset), ptr, n))
        del keep

    def read_buffer(self, buffer: Handle, offset: int, length: int) -> bytes:
        out = (C.c_char * int(length))()
        check(self._lib.zg_buffer_read(self._p, buffer, int(offset), C.cast(out, C.c_void_p),
                                       int(length)))
        return bytes(out)

    def read_buffer_into(self, buffer: Handle, offset: int, dst: np.ndarray) -> None:
        if not dst.flags["C_CONTIGUOUS"]:
            raise ValueError("read_buffer_into needs a C-contiguous destination")
        check(self._lib.zg_buffer_read(self._p, buffer, int(offset), C.c_void_p(dst.ctypes.data),
                                       dst.nbytes))

    def read_buffer_ptr(self, buffer: Handle, offset: int, host_ptr: int, length: int) -> None:
        """read_buffer_into a caller-owned host pointer (e.g. pinned memory)."""
        check(self._lib.zg_buffer_read(self._p, buffer, int(offset), C.c_void_p(host_ptr),
                                       int(length)))

    def read_buffer_async(self, buffer: Handle, offset: int, dst, length: int | None = None
                          ) -> "Submission":
        """Queues a device -> host copy into `dst` (a host address, a numpy array
        or a pinned torch CPU tensor) after everything queued before it and
        returns the submission; `dst` holds the bytes once it completes
        (zg_buffer_read_async).  Needs READBACK or TRANSFER_SRC usage."""
        ptr, keep = _host_ptr_bytes(dst)
        nbytes = keep[1] if length is None else int(length)
        sub = C.c_void_p()
        check(self._lib.zg_buffer_read_async(self._p, buffer, int(offset), C.c_void_p(ptr),
                                             nbytes, C.byref(sub)))
        s = Submission(sub)
        s._keep = keep  # the destination must outlive the copy
        return s

    def write_buffer_ptr(self, buffer: Handle, offset: int, host_ptr: int, length: int) -> None:
        check(self._lib.zg_buffer_write(self._p, buffer, int(offset), C.c_void_p(host_ptr),
                                        int(length)))

    def copy_buffer(self, src: Handle, src_offset: int, dst: Handle, dst_offset: int,
                    length: int) -> None:
        check(self._lib.zg_buffer_copy(self._p, src, int(src_offset), dst, int(dst_offset),
                                       int(length)))

    def destroy_buffer(self, buffer: Handle) -> None:
        self._lib.zg_buffer_destroy(self._p, buffer)

    def buffer_info(self, buffer: Handle) -> tuple[int, int]:
        ptr, size = C.c_uint64(), C.c_uint64()
        check(self._lib.zg_buffer_info(self._p, buffer, C.byref(ptr), C.byref(size)))
        return ptr.value, size.value

    def copy_from_peer(self, dst: Handle, src_device: "CudaDevice", src: Handle,
                       nbytes: int) -> None:
        check(self._lib.zg_buffer_copy_from_peer(self._p, dst, src_device.raw, src, int(nbytes)))

    # shaders / pipelines / dispatch
    def create_shader(self, kind: int, code: bytes | None = None) -> Handle:
        h = Handle()
        if code is None:
            check(self._lib.zg_shader_create(self._p, int(kind), None, 0, C.byref(h)))
        else:
            buf = C.create_string_buffer(code, len(code))
            check(self._lib.zg_shader_create(self._p, int(kind), C.cast(buf, C.c_void_p),
                                             len(code), C.byref(h)))
        return h

    def destroy_shader(self, shader: Handle) -> None:
        self._lib.zg_shader_destroy(self._p, shader)

    def create_compute_pipeline(self, shader: Handle, entry: str,
                                block: Sequence[int] = (256, 1, 1), dynamic_smem: int = 0) -> Handle:
        h = Handle()
        blk = (C.c_uint32 * 3)(*block)
        check(self._lib.zg_pipeline_create(self._p, shader, entry.encode(), blk,
                                           int(dynamic_smem), C.byref(h)))
        return h

    def destroy_pipeline(self, pipeline: Handle) -> None:
        self._lib.zg_pipeline_destroy(self._p, pipeline)

    @staticmethod
    def _op(pipeline: Handle, buffers: Iterable[int], scalars: Iterable[L.Scalar],
            grid: Sequence[int]):
        bufs = list(buffers)
        scs = list(scalars)
        barr = (C.c_uint32 * max(len(bufs), 1))(*bufs)
        sarr = (L.Scalar * max(len(scs), 1))(*scs)
        op = L.DispatchOp(pipeline, C.cast(barr, C.POINTER(C.c_uint32)), len(bufs),
                          C.cast(sarr, C.POINTER(L.Scalar)), len(scs),
                          (C.c_uint32 * 3)(*grid))
        return op, (barr, sarr)

    def dispatch(self, pipeline: Handle, buffers: Iterable[int], scalars: Iterable[L.Scalar],
                 grid: Sequence[int] = (1, 1, 1)) -> None:
        op, keep = self._op(pipeline, buffers, scalars, grid)
        check(self._lib.zg_dispatch(self._p, C.byref(op)))

    def submit_batch(self, ops: Sequence[tuple]) -> Submission:
        built = [self._op(*o) for o in ops]
        arr = (L.DispatchOp * len(built))(*[b[0] for b in built])
        sub = C.c_void_p()
        check(self._lib.zg_submit_batch(self._p, arr, len(built), C.byref(sub)))
        return Submission(sub)

    def submit(self, pipeline: Handle, buffers, scalars, grid=(1, 1, 1)) -> Submission:
        return self.submit_batch([(pipeline, buffers, scalars, grid)])


# ---- DeviceArray / BufferPool ------------------------------------------------------------
class DeviceArray:
    """Resident buffer + u32 shape/stride + dtype (zengpu-compute/src/lib.rs:21-72)."""

    def __init__(self, c: L.CDeviceArray):
        self._c = c

    @property
    def buffer(self) -> Handle:
        return self._c.buffer

    @property
    def shape(self) -> list[int]:
        return list(self._c.shape[: self._c.rank])

    @property
    def stride(self) -> list[int]:
        return list(self._c.stride[: self._c.rank])

    @property
    def dtype(self) -> DType:
        return DType(self._c.dtype)

    def len(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n

    def is_empty(self) -> bool:
        return self.len() == 0

    def size_bytes(self) -> int:
        return self.len() * self.dtype.size_bytes()

    def allocation_size_bytes(self) -> int:
        return int(self._c.allocation_size)

    def __repr__(self) -> str:
        return f"DeviceArray(shape={self.shape}, dtype={self.dtype.name}, buffer={self.buffer})"


def size_class(size: int) -> int:
    return int(L.load().zg_size_class(int(size)))


class BufferPool:
    """Size-classed (pow2, min 256 B) free list over device buffers.

    memory=MemoryUsage.Upload is the reference's pool (STORAGE | READBACK,
    zengpu-compute/src/pool.rs:47-51).  MemoryUsage.GpuOnly gives device-resident
    arrays without READBACK: ops writing them are queued without a per-op
    synchronize, and they are read back with download_async (or copied)."""

    def __init__(self, device: CudaDevice, memory: MemoryUsage = MemoryUsage.Upload):
        self._lib = L.load()
        self.device = device
        p = C.c_void_p()
        check(self._lib.zg_pool_create_with(device.raw, int(memory), C.byref(p)))
        self._p = p

    @property
    def memory(self) -> MemoryUsage:
        return MemoryUsage(int(self._lib.zg_pool_memory(self._p)))

    @property
    def raw(self) -> C.c_void_p:
        return self._p

    def alloc(self, shape: Sequence[int], dtype: DType = DType.F32) -> DeviceArray:
        shp = (C.c_uint32 * max(len(shape), 1))(*shape)
        out = L.CDeviceArray()
        check(self._lib.zg_pool_alloc(self._p, shp, len(shape), int(dtype), C.byref(out)))
        return DeviceArray(out)

    def free(self, array: DeviceArray) -> None:
        self._lib.zg_pool_free(self._p, C.byref(array._c))

    def free_count(self, size_class_bytes: int) -> int:
        return int(self._lib.zg_pool_free_count(self._p, int(size_class_bytes)))

    def close(self) -> None:
        if self._p:
            self._lib.zg_pool_destroy(self._p)
            self._p = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def upload(device: CudaDevice, pool: BufferPool, data: np.ndarray) -> DeviceArray:
    """Allocates a DeviceArray of data's shape and writes data into it."""
    data = np.ascontiguousarray(data, dtype=np.float32)
    arr = pool.alloc(list(data.shape), DType.F32)
    device.write_buffer(arr.buffer, 0, data)
    return arr


def download(device: CudaDevice, array: DeviceArray) -> np.ndarray:
    out = np.empty(array.shape, dtype=np.float32)
    device.read_buffer_into(array.buffer, 0, out)
    return out


def download_async(device: CudaDevice, array: DeviceArray, out=None):
    """Queues the readback of `array` into `out` (a float32 numpy array of its
    shape, or a pinned torch CPU tensor; allocated when None) and returns
    (out, submission): `out` holds the values once the submission completes.
    Works for GpuOnly arrays."""
    if out is None:
        out = np.empty(array.shape, dtype=np.float32)
    return out, device.read_buffer_async(array.buffer, 0, out, array.size_bytes())


# ---- kernels -------------------------------------------------------------------------------
class ElementwiseKernels:
    """add / relu pipelines (zengpu-compute/src/elementwise.rs:51-146)."""

    def __init__(self, device: CudaDevice):
        self._lib = L.load()
        self._k = L.CElementwiseKernels()
        check(self._lib.zg_elementwise_new(device.raw, C.byref(self._k)))

    @property
    def add_pipeline(self) -> Handle:
        return self._k.add_pipeline

    @property
    def relu_pipeline(self) -> Handle:
        return self._k.relu_pipeline

    def destroy(self, device: CudaDevice) -> None:
        self._lib.zg_elementwise_destroy(device.raw, C.byref(self._k))

    def add(self, device: CudaDevice, pool: BufferPool, a: DeviceArray, b: DeviceArray) -> DeviceArray:
        out = L.CDeviceArray()
        check(self._lib.zg_elementwise_add(C.byref(self._k), device.raw, pool.raw, C.byref(a._c),
                                           C.byref(b._c), C.byref(out)))
        return DeviceArray(out)

    def relu(self, device: CudaDevice, pool: BufferPool, a: DeviceArray) -> DeviceArray:
        out = L.CDeviceArray()
        check(self._lib.zg_elementwise_relu(C.byref(self._k), device.raw, pool.raw, C.byref(a._c),
                                            C.byref(out)))
        return DeviceArray(out)

    def relu_inplace(self, device: CudaDevice, a: DeviceArray) -> None:
        check(self._lib.zg_elementwise_relu_inplace(C.byref(self._k), device.raw, C.byref(a._c)))


def _host_ptr_bytes(x) -> tuple[int, tuple]:
    """(address, (keep-alive, size in bytes)) of a host destination buffer: an
    int address (size unknown: 0), a C-contiguous numpy array, or a CPU tensor."""
    if isinstance(x, int):
        return x, (None, 0)
    if hasattr(x, "data_ptr"):
        if x.is_cuda or not x.is_contiguous():
            raise ValueError("host destination must be a contiguous CPU tensor")
        return int(x.data_ptr()), (x, x.numel() * x.element_size())
    if not isinstance(x, np.ndarray) or not x.flags["C_CONTIGUOUS"] or not x.flags["WRITEABLE"]:
        raise ValueError("host destination must be a writeable C-contiguous numpy array")
    return x.ctypes.data, (x, x.nbytes)


def _host_ptr(x) -> tuple[int, object]:
    """(address, keep-alive) of a host buffer: an int address, or a C-contiguous
    float32 numpy array (or anything exposing data_ptr(), e.g. a pinned torch
    CPU tensor)."""
    if x is None:
        return 0, None
    if isinstance(x, int):
        return x, None
    if hasattr(x, "data_ptr"):
        return int(x.data_ptr()), x
    arr = np.ascontiguousarray(x, dtype=np.float32)
    return arr.ctypes.data, arr


class GemmKernel:
    """f32 GEMM (zengpu-blas/src/level3.rs:101-182) with a selectable mode."""

    def __init__(self, device: CudaDevice, mode: GemmMode | None = None):
        self._lib = L.load()
        self._k = L.CGemmKernel()
        check(self._lib.zg_gemm_new(device.raw, C.byref(self._k)))
        if mode is not None:
            self._k.mode = int(mode)

    @property
    def pipeline(self) -> Handle:
        return self._k.pipeline

    @property
    def mode(self) -> GemmMode:
        return GemmMode(self._k.mode)

    @mode.setter
    def mode(self, m: GemmMode) -> None:
        self._k.mode = int(m)

    def destroy(self, device: CudaDevice) -> None:
        self._lib.zg_gemm_destroy(device.raw, C.byref(self._k))

    def sgemm(self, device: CudaDevice, pool: BufferPool, alpha: float, a: DeviceArray,
              b: DeviceArray) -> DeviceArray:
        out = L.CDeviceArray()
        check(self._lib.zg_gemm_sgemm(C.byref(self._k), device.raw, pool.raw, float(alpha),
                                      C.byref(a._c), C.byref(b._c), C.byref(out)))
        return DeviceArray(out)

    def gemm(self, device: CudaDevice, pool: BufferPool, a: DeviceArray, b: DeviceArray) -> DeviceArray:
        out = L.CDeviceArray()
        check(self._lib.zg_gemm_gemm(C.byref(self._k), device.raw, pool.raw, C.byref(a._c),
                                     C.byref(b._c), C.byref(out)))
        return DeviceArray(out)

    def gemm_bias_relu(self, device: CudaDevice, pool: BufferPool, alpha: float, a: DeviceArray,
                       b: DeviceArray, bias: DeviceArray) -> DeviceArray:
        out = L.CDeviceArray()
        check(self._lib.zg_gemm_bias_relu(C.byref(self._k), device.raw, pool.raw, float(alpha),
                                          C.byref(a._c), C.byref(b._c), C.byref(bias._c),
                                          C.byref(out)))
        return DeviceArray(out)


    def sgemm_host(self, device: CudaDevice, alpha: float, a, b, c, m: int, n: int, k: int,
                   bias=None, relu: bool = False) -> None:
        """C = epilogue(alpha * A @ B) on host arrays (zg_gemm_sgemm_host): B up,
        then row panels of A up / GEMM / C rows down, overlapped on three streams.
        a, b, c, bias: host addresses, float32 numpy arrays or pinned torch tensors."""
        pa, ka = _host_ptr(a)
        pb, kb = _host_ptr(b)
        pc, kc = _host_ptr(c)
        pbias, kbias = _host_ptr(bias)
        check(self._lib.zg_gemm_sgemm_host(C.byref(self._k), device.raw, float(alpha),
                                           C.c_void_p(pa), C.c_void_p(pb),
                                           C.c_void_p(pbias) if bias is not None else None,
                                           1 if relu else 0, C.c_void_p(pc), m, n, k))
        del ka, kb, kc, kbias


class Level1Kernels:
    """saxpy / sscal, in place (zengpu-blas/src/level1.rs:51-139)."""

    def __init__(self, device: CudaDevice):
        self._lib = L.load()

    def destroy(self, device: CudaDevice) -> None:
        pass

    def saxpy(self, device: CudaDevice, pool: BufferPool, alpha: float, x: DeviceArray,
              y: DeviceArray) -> None:
        check(self._lib.zg_level1_saxpy(device.raw, float(alpha), C.byref(x._c), C.byref(y._c)))

    def sscal(self, device: CudaDevice, pool: BufferPool, alpha: float, x: DeviceArray) -> None:
        check(self._lib.zg_level1_sscal(device.raw, float(alpha), C.byref(x._c)))


class Blas:
    """Level-1 + Level-3 pipelines for one device (zengpu-blas/src/lib.rs:51-108)."""

    def __init__(self, device: CudaDevice):
        self.level1 = Level1Kernels(device)
        self.gemm = GemmKernel(device)

    def destroy(self, device: CudaDevice) -> None:
        self.level1.destroy(device)
        self.gemm.destroy(device)

    def sgemm(self, device, pool, alpha, a, b) -> DeviceArray:
        return self.gemm.sgemm(device, pool, alpha, a, b)

    def saxpy(self, device, pool, alpha, x, y) -> None:
        self.level1.saxpy(device, pool, alpha, x, y)

    def sscal(self, device, pool, alpha, x) -> None:
        self.level1.sscal(device, pool, alpha, x)
