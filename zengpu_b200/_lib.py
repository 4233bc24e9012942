"""ctypes binding of libzengpu_b200.so (the C ABI in include/zengpu_b200.h).

Loading fails loudly: there is no CPU fallback anywhere in this package, so a
missing or unloadable library raises at import of any op.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libzengpu_b200.so"

MAX_RANK = 8


class Handle(C.Structure):
    _fields_ = [("index", C.c_uint32), ("generation", C.c_uint32)]

    def __repr__(self) -> str:
        return f"Handle({self.index}, gen={self.generation})"

    def __eq__(self, other) -> bool:
        return isinstance(other, Handle) and (self.index, self.generation) == (
            other.index, other.generation)

    def __hash__(self) -> int:
        return hash((self.index, self.generation))


class ErrorDetail(C.Structure):
    _fields_ = [
        ("status", C.c_int32),
        ("handle_index", C.c_uint32),
        ("expected_gen", C.c_uint32),
        ("actual_gen", C.c_uint32),
        ("memory", C.c_uint32),
        ("reserved", C.c_uint32),
        ("features", C.c_uint64),
        ("resource", C.c_char_p),
        ("needed", C.c_char_p),
    ]


class Scalar(C.Structure):
    _fields_ = [("kind", C.c_uint32), ("bits", C.c_uint32)]


class DispatchOp(C.Structure):
    _fields_ = [
        ("pipeline", Handle),
        ("buffers", C.POINTER(C.c_uint32)),
        ("num_buffers", C.c_uint32),
        ("scalars", C.POINTER(Scalar)),
        ("num_scalars", C.c_uint32),
        ("grid", C.c_uint32 * 3),
    ]


class CDeviceArray(C.Structure):
    _fields_ = [
        ("buffer", Handle),
        ("dtype", C.c_uint32),
        ("rank", C.c_uint32),
        ("shape", C.c_uint32 * MAX_RANK),
        ("stride", C.c_uint32 * MAX_RANK),
        ("allocation_size", C.c_uint64),
    ]


class CElementwiseKernels(C.Structure):
    _fields_ = [
        ("add_shader", Handle),
        ("add_pipeline", Handle),
        ("relu_shader", Handle),
        ("relu_pipeline", Handle),
    ]


class CGemmKernel(C.Structure):
    _fields_ = [
        ("shader", Handle),
        ("pipeline", Handle),
        ("fused_pipeline", Handle),
        ("mode", C.c_int32),
    ]


_vp = C.c_void_p
_i = C.c_int
_u32 = C.c_uint32
_u64 = C.c_uint64
_f = C.c_float
_fp = C.c_void_p  # device float pointers travel as integers

# name -> (restype, argtypes); mirrors include/zengpu_b200.h one to one.
SIGNATURES: dict[str, tuple] = {
    "zg_last_error": (C.c_char_p, []),
    "zg_last_error_detail": (_i, [C.POINTER(ErrorDetail)]),
    "zg_abi_version": (_i, []),
    "zg_device_count": (_i, [C.POINTER(_i)]),
    "zg_device_open": (_i, [_i, C.POINTER(_vp)]),
    "zg_device_close": (None, [_vp]),
    "zg_device_ordinal": (_i, [_vp]),
    "zg_device_stream": (_vp, [_vp]),
    "zg_device_can_peer": (_i, [_vp, _i, C.POINTER(_i)]),
    "zg_buffer_create": (_i, [_vp, _u64, _u32, _u32, C.POINTER(Handle)]),
    "zg_buffer_write": (_i, [_vp, Handle, _u64, _vp, _u64]),
    "zg_buffer_read": (_i, [_vp, Handle, _u64, _vp, _u64]),
    "zg_buffer_read_async": (_i, [_vp, Handle, _u64, _vp, _u64, C.POINTER(_vp)]),
    "zg_buffer_copy": (_i, [_vp, Handle, _u64, Handle, _u64, _u64]),
    "zg_buffer_destroy": (None, [_vp, Handle]),
    "zg_buffer_info": (_i, [_vp, Handle, C.POINTER(_u64), C.POINTER(_u64)]),
    "zg_buffer_copy_from_peer": (_i, [_vp, Handle, _vp, Handle, _u64]),
    "zg_shader_create": (_i, [_vp, _u32, _vp, _u64, C.POINTER(Handle)]),
    "zg_shader_destroy": (None, [_vp, Handle]),
    "zg_pipeline_create": (_i, [_vp, Handle, C.c_char_p, C.POINTER(_u32), _u32,
                                C.POINTER(Handle)]),
    "zg_pipeline_destroy": (None, [_vp, Handle]),
    "zg_dispatch": (_i, [_vp, C.POINTER(DispatchOp)]),
    "zg_submit_batch": (_i, [_vp, C.POINTER(DispatchOp), _u32, C.POINTER(_vp)]),
    "zg_submission_poll": (_i, [_vp, C.POINTER(_i)]),
    "zg_submission_wait": (_i, [_vp, _u64]),
    "zg_submission_destroy": (None, [_vp]),
    "zg_size_class": (_u64, [_u64]),
    "zg_pool_create": (_i, [_vp, C.POINTER(_vp)]),
    "zg_pool_create_with": (_i, [_vp, _u32, C.POINTER(_vp)]),
    "zg_pool_memory": (_u32, [_vp]),
    "zg_pool_destroy": (None, [_vp]),
    "zg_pool_alloc": (_i, [_vp, C.POINTER(_u32), _u32, _u32, C.POINTER(CDeviceArray)]),
    "zg_pool_free": (None, [_vp, C.POINTER(CDeviceArray)]),
    "zg_pool_free_count": (_u32, [_vp, _u64]),
    "zg_elementwise_new": (_i, [_vp, C.POINTER(CElementwiseKernels)]),
    "zg_elementwise_destroy": (None, [_vp, C.POINTER(CElementwiseKernels)]),
    "zg_elementwise_add": (_i, [C.POINTER(CElementwiseKernels), _vp, _vp,
                                C.POINTER(CDeviceArray), C.POINTER(CDeviceArray),
                                C.POINTER(CDeviceArray)]),
    "zg_elementwise_relu": (_i, [C.POINTER(CElementwiseKernels), _vp, _vp,
                                 C.POINTER(CDeviceArray), C.POINTER(CDeviceArray)]),
    "zg_elementwise_relu_inplace": (_i, [C.POINTER(CElementwiseKernels), _vp,
                                         C.POINTER(CDeviceArray)]),
    "zg_gemm_new": (_i, [_vp, C.POINTER(CGemmKernel)]),
    "zg_gemm_destroy": (None, [_vp, C.POINTER(CGemmKernel)]),
    "zg_gemm_sgemm": (_i, [C.POINTER(CGemmKernel), _vp, _vp, _f, C.POINTER(CDeviceArray),
                           C.POINTER(CDeviceArray), C.POINTER(CDeviceArray)]),
    "zg_gemm_gemm": (_i, [C.POINTER(CGemmKernel), _vp, _vp, C.POINTER(CDeviceArray),
                          C.POINTER(CDeviceArray), C.POINTER(CDeviceArray)]),
    "zg_gemm_bias_relu": (_i, [C.POINTER(CGemmKernel), _vp, _vp, _f, C.POINTER(CDeviceArray),
                               C.POINTER(CDeviceArray), C.POINTER(CDeviceArray),
                               C.POINTER(CDeviceArray)]),
    "zg_gemm_sgemm_host": (_i, [C.POINTER(CGemmKernel), _vp, _f, _vp, _vp, _vp, _i, _vp, _u32,
                                _u32, _u32]),
    "zg_level1_saxpy": (_i, [_vp, _f, C.POINTER(CDeviceArray), C.POINTER(CDeviceArray)]),
    "zg_level1_sscal": (_i, [_vp, _f, C.POINTER(CDeviceArray)]),
    "zg_add_f32": (_i, [_fp, _fp, _fp, _u64, _vp]),
    "zg_relu_f32": (_i, [_fp, _fp, _u64, _vp]),
    "zg_saxpy_f32": (_i, [_f, _fp, _fp, _u64, _vp]),
    "zg_sscal_f32": (_i, [_f, _fp, _u64, _vp]),
    "zg_sgemm_workspace_bytes": (_u64, [_i, _i, _i, _i]),
    "zg_sgemm_f32": (_i, [_i, _i, _i, _i, _f, _fp, _fp, _fp, _fp, _i, _vp, _u64, _vp]),
    "zg_sgemm_prepare": (_i, [_i, _i, _i, _i, _fp, _fp, _vp, _u64, _vp]),
    "zg_sgemm_compute": (_i, [_i, _i, _i, _i, _f, _fp, _fp, _fp, _fp, _i, _vp, _u64, _vp]),
    "zg_sgemm_pack_bytes": (_u64, [_i, _i, _i, _i]),
    "zg_sgemm_pack_a": (_i, [_i, _i, _i, _fp, C.c_int64, _vp, _u64, _vp]),
    "zg_sgemm_pack_b": (_i, [_i, _i, _i, _fp, C.c_int64, _vp, _u64, _vp]),
    "zg_sgemm_packed": (_i, [_i, _i, _i, _i, _f, _vp, _vp, _fp, C.c_int64, _fp, _i, _vp]),
    "zg_sgemm_f32_noalloc": (_i, [_i, _i, _i, _i, _f, _fp, _fp, _fp, _fp, _i, _vp]),
    "zg_fill_uniform_f32": (_i, [_fp, _u64, _u64, _f, _f, _vp]),
    "zg_fill_normal_f32": (_i, [_fp, _u64, _u64, _vp]),
    "zg_kernel_status": (_i, [C.POINTER(_u32)]),
    "zg_sgemm_kernel_name": (C.c_char_p, [_i, _i, _i, _i]),
    "zg_bchain_create": (_i, [_i, _i, _i, _i, C.POINTER(_vp), C.POINTER(C.c_uint8)]),
    "zg_bchain_connect": (_i, [_vp, C.POINTER(C.c_uint8), C.POINTER(C.c_uint8)]),
    "zg_bchain_source": (_i, [_vp, _u32, _fp, C.c_int64, _vp]),
    "zg_bchain_forward": (_i, [_vp, _u32, _vp]),
    "zg_bchain_gemm": (_i, [_vp, _u32, _i, _i, _f, _vp, _fp, C.c_int64, _fp, _i, _vp]),
    "zg_bchain_release": (_i, [_vp, _u32, _vp]),
    "zg_bchain_buffer": (_i, [_vp, _u32, C.POINTER(_vp), C.POINTER(_u64)]),
    "zg_bchain_abort": (_i, [_vp, _u32]),
    "zg_bchain_destroy": (_i, [_vp]),
}

_lib: C.CDLL | None = None


def load() -> C.CDLL:
    """Loads libzengpu_b200.so once; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("ZENGPU_B200_LIB", LIB_PATH))
    if not path.exists():
        raise ImportError(
            f"{path} is missing: build the CUDA library first "
            "(python -m zengpu_b200.build); there is no CPU fallback")
    lib = C.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    msg = load().zg_last_error()
    return msg.decode() if msg else ""


def last_error_detail() -> ErrorDetail:
    d = ErrorDetail()
    load().zg_last_error_detail(C.byref(d))
    return d
