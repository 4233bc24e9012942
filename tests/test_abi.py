"""The C-ABI library on a CPU-only machine: it loads, exports every symbol
include/zengpu_b200.h declares, and its host-side logic answers without a
GPU (no kernel is launched here)."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

import zengpu_b200 as zg
from zengpu_b200 import _lib as L

HEADER = Path(__file__).resolve().parents[1] / "include" / "zengpu_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(zg_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = zg.load_library()
    names = declared_functions()
    assert len(names) > 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # the ctypes signature table covers the same set
    assert set(L.SIGNATURES) == set(names)


def test_abi_version():
    assert zg.load_library().zg_abi_version() == 1


@pytest.mark.parametrize("size,cls", [(0, 256), (1, 256), (255, 256), (256, 256), (257, 512),
                                      (4097, 8192), (1 << 30, 1 << 30), ((1 << 30) + 1, 1 << 31)])
def test_size_class(size, cls):
    # zengpu-compute/src/pool.rs:91-104 plus the 1 GiB arrays of the bandwidth config
    assert zg.size_class(size) == cls


def test_no_device_is_reported_not_crashed():
    if zg.device_count() > 0:
        pytest.skip("a GPU is visible")
    with pytest.raises(zg.NoDevice):
        zg.CudaDevice(0)


def test_workspace_bytes():
    lib = zg.load_library()
    # SIMT (optional): A transposed, k rows of round_up(m, 4) floats
    assert lib.zg_sgemm_workspace_bytes(0, 1024, 1024, 1024) == 1024 * 1024 * 4
    assert lib.zg_sgemm_workspace_bytes(0, 17, 9, 33) == 256 * ((33 * 20 * 4 + 255) // 256)
    # TF32X3 / TF32_BF16X2: A (m rows) and B transposed (n rows), each 16-k block
    # one 128-byte row of interleaved terms (k padded to 16), 256-byte aligned
    assert lib.zg_sgemm_workspace_bytes(1, 8192, 8192, 8192) == 4 * 8192 * 8192 * 4
    assert lib.zg_sgemm_workspace_bytes(3, 8192, 8192, 8192) == 4 * 8192 * 8192 * 4
    assert lib.zg_sgemm_workspace_bytes(1, 17, 9, 33) == 256 * ((17 * 96 * 4 + 255) // 256) + \
        256 * ((9 * 96 * 4 + 255) // 256)
    # BF16X3: each 32-k block one 128-byte row (32 bf16 hi, 32 bf16 lo), k padded to 32
    assert lib.zg_sgemm_workspace_bytes(4, 8192, 8192, 8192) == 2 * 8192 * 8192 * 4
    assert lib.zg_sgemm_workspace_bytes(4, 17, 9, 33) == 256 * ((17 * 64 * 4 + 255) // 256) + \
        256 * ((9 * 64 * 4 + 255) // 256)
    # TF32: the K-major copy of B, plus a pitched copy of A when k % 4 != 0
    assert lib.zg_sgemm_workspace_bytes(2, 64, 64, 64) == 64 * 64 * 4
    assert lib.zg_sgemm_workspace_bytes(2, 17, 9, 33) == 256 * ((17 * 36 * 4 + 255) // 256) + \
        256 * ((9 * 36 * 4 + 255) // 256)
    assert lib.zg_sgemm_workspace_bytes(1, 0, 5, 5) == 0


def test_sgemm_argument_errors_are_dispatch():
    lib = zg.load_library()
    fake = C.c_void_p(0x1000)
    assert lib.zg_sgemm_f32(7, 4, 4, 4, 1.0, fake, fake, fake, None, 0, None, 0, None) == 11
    assert "unknown mode" in L.last_error()
    assert lib.zg_sgemm_f32(0, -1, 4, 4, 1.0, fake, fake, fake, None, 0, None, 0, None) == 11
    assert lib.zg_sgemm_f32(0, 0, 4, 4, 1.0, None, None, None, None, 0, None, 0, None) == 0
    assert lib.zg_sgemm_f32(0, 4, 4, 4, 1.0, None, fake, fake, None, 0, None, 0, None) == 11
    # TF32X3 needs its hi/lo workspace
    assert lib.zg_sgemm_f32(1, 64, 64, 64, 1.0, fake, fake, fake, None, 0, None, 0, None) == 11
    assert "workspace" in L.last_error()


def test_simt_workspace_is_optional():
    """SIMT states a workspace (A transposed, for its TMA-fed kernel) but runs
    without one: a call with none passes the argument checks, where every
    other fp32-class mode rejects it (no GPU here, so the SIMT call then fails
    at the launch, not at the checks)."""
    if zg.device_count() > 0:
        pytest.skip("a GPU is visible: the SIMT call would launch on placeholder pointers")
    lib = zg.load_library()
    fake = C.c_void_p(0x1000)
    assert lib.zg_sgemm_workspace_bytes(0, 64, 64, 64) > 0
    rc = lib.zg_sgemm_f32(0, 64, 64, 64, 1.0, fake, fake, fake, None, 0, None, 0, None)
    assert rc != zg.api.Dispatch.code and "workspace" not in L.last_error()
    for mode in (1, 3, 4):
        assert lib.zg_sgemm_f32(mode, 64, 64, 64, 1.0, fake, fake, fake, None, 0, None, 0,
                                None) == zg.api.Dispatch.code
        assert "workspace" in L.last_error()


def test_elementwise_argument_errors():
    lib = zg.load_library()
    assert lib.zg_add_f32(None, None, None, 0, None) == 0  # empty is a no-op
    assert lib.zg_add_f32(None, None, None, 16, None) == 11
    assert lib.zg_relu_f32(None, None, 16, None) == 11


def test_error_classes_cover_every_status():
    for code in range(1, 15):
        assert code in zg.api._ERRORS
    with pytest.raises(zg.Dispatch):
        zg.api.check(11)
    assert issubclass(zg.StaleHandle, zg.InvalidUsage)


def test_dtype_sizes():
    assert zg.DType.F32.size_bytes() == 4
    assert zg.DType.F64.size_bytes() == 8
    assert zg.DType.Bf16.size_bytes() == 2
    assert zg.DType.Bool.size_bytes() == 1


def test_product_path_does_not_reference_the_oracle():
    pkg = Path(zg.__file__).resolve().parent
    for p in list(pkg.rglob("*.py")) + list(pkg.rglob("*.cu")) + list(pkg.rglob("*.cpp")):
        assert "oracle" not in p.read_text().lower(), p


def test_bchain_argument_errors_need_no_gpu():
    """The chain's argument checks answer before any CUDA call."""
    lib = zg.load_library()
    out = C.c_void_p()
    handle = (C.c_uint8 * 64)()
    # SIMT has no chunked B^T form; chunks must be multiples of 256 columns
    assert lib.zg_bchain_create(0, 64, 512, 256, C.byref(out), handle) == zg.api.Dispatch.code
    assert lib.zg_bchain_create(3, 64, 512, 200, C.byref(out), handle) == zg.api.Dispatch.code
    assert lib.zg_bchain_create(3, 0, 512, 256, C.byref(out), handle) == zg.api.Dispatch.code
    assert out.value is None
    assert lib.zg_bchain_forward(None, 1, None) == zg.api.Dispatch.code
    assert lib.zg_bchain_gemm(None, 1, 1, 8, 1.0, None, None, 512, None, 0, None) == \
        zg.api.Dispatch.code
    assert lib.zg_bchain_destroy(None) == 0


def test_sgemm_kernel_name():
    """The launch rule as the library reports it (148 SMs when no GPU answers)."""
    lib = zg.load_library()
    name = lambda *a: lib.zg_sgemm_kernel_name(*a).decode()  # noqa: E731
    assert name(4, 8192, 8192, 8192) == "sgemm_tc_pair_kernel<4>"
    assert name(3, 8192, 8192, 8192) == "sgemm_tc_pair_kernel<3>"
    assert name(1, 256, 512, 64) == "sgemm_tc_kernel<2>"
    assert name(2, 256, 512, 64) == "sgemm_tc_kernel<1>"
    assert name(0, 8192, 8192, 8192) == "sgemm_simt_tma_kernel"
    assert name(3, 64, 64, 0) == "gemm_k0_kernel"
    assert name(9, 64, 64, 64) == "" and name(3, 0, 64, 64) == ""


def test_release_workspaces_drops_cached_scratch():
    """kernels.release_workspaces empties the per-(device, stream) GEMM scratch
    cache, per device or all at once (no GPU needed: the cache is a dict)."""
    import torch

    from zengpu_b200 import kernels as K
    saved = dict(K._workspaces)
    try:
        K._workspaces.clear()
        K._workspaces.update({(0, 11): torch.empty(4), (0, 12): torch.empty(4),
                              (1, 13): torch.empty(4)})
        assert K.release_workspaces(0) == 2
        assert list(K._workspaces) == [(1, 13)]
        assert K.release_workspaces() == 1
        assert not K._workspaces
    finally:
        K._workspaces.clear()
        K._workspaces.update(saved)


def test_last_error_detail_follows_the_last_status():
    """zg_last_error_detail carries the status of the last failure on this
    thread, with the structured fields empty for variants that have none."""
    import ctypes as C

    from zengpu_b200 import _lib as L
    lib = L.load()
    rc = lib.zg_sgemm_f32(99, 4, 4, 4, 1.0, None, None, None, None, 0, None, 0, None)
    assert rc == 11  # Dispatch: unknown mode
    d = L.last_error_detail()
    assert d.status == 11 and d.handle_index == 0 and d.resource == b"" and d.needed == b""
    assert lib.zg_pool_create_with(None, 0, C.byref(C.c_void_p())) == 12
    assert L.last_error_detail().status == 12
