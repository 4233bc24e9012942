"""GpuOnly residency and asynchronous readback in BufferPool.

The reference pool always creates STORAGE | READBACK buffers with
MemoryUsage::Upload (zengpu-compute/src/pool.rs:47-51), and every op waits for
the GPU before it returns.  A GpuOnly pool hands out device-resident arrays:
ops writing them are queued without that wait, and the result comes back
through one readback submission (zg_buffer_read_async).  The results must be
the same bits as the Upload path's."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import _oracle as O
import zengpu_b200 as zg

pytestmark = pytest.mark.gpu

MODES = [zg.GemmMode.BF16X3, zg.GemmMode.TF32X3, zg.GemmMode.TF32, zg.GemmMode.SIMT_FP32]


def bits(x) -> np.ndarray:
    return np.asarray(x, np.float32).view(np.uint32)


def test_gpu_only_pool_arrays(device):
    pool = zg.BufferPool(device, zg.MemoryUsage.GpuOnly)
    assert pool.memory == zg.MemoryUsage.GpuOnly
    assert zg.BufferPool(device).memory == zg.MemoryUsage.Upload
    data = O.uniform(1000, 1)
    arr = zg.upload(device, pool, data)
    assert arr.allocation_size_bytes() == 4096
    with pytest.raises(zg.MissingUsage):
        zg.download(device, arr)  # no READBACK: not host readable
    out, sub = zg.download_async(device, arr)
    sub.wait(10.0)
    assert sub.poll()
    np.testing.assert_array_equal(bits(out), bits(data))
    with pytest.raises(zg.Unsupported):
        zg.BufferPool(device, zg.MemoryUsage.Readback)
    pool.free(arr)
    assert pool.free_count(4096) == 1
    pool.close()


def test_read_async_in_flight_rules(device):
    """A readback submission is in flight until poll / wait observes it
    (zengpu-cuda/src/lib.rs:412-444): synchronous writes and reads are refused
    meanwhile; the destination holds the bytes once it completes."""
    pool = zg.BufferPool(device)
    a = zg.upload(device, pool, O.uniform(4096, 2))
    dst = torch.empty(4096).pin_memory()
    sub = device.read_buffer_async(a.buffer, 0, dst)
    with pytest.raises(zg.BindingMismatch, match="pending"):
        device.write_buffer(a.buffer, 0, b"\0" * 4)
    with pytest.raises(zg.BindingMismatch, match="pending"):
        zg.download(device, a)
    sub.wait(10.0)
    np.testing.assert_array_equal(bits(dst.numpy()), bits(O.uniform(4096, 2)))
    device.write_buffer(a.buffer, 0, b"\0" * 4)  # allowed again
    # partial range and range errors
    part = np.empty(10, np.float32)
    sub2 = device.read_buffer_async(a.buffer, 40, part, 40)
    sub2.wait(10.0)
    np.testing.assert_array_equal(bits(part), bits(O.uniform(4096, 2)[10:20]))
    with pytest.raises(zg.BindingMismatch, match="exceeds"):
        device.read_buffer_async(a.buffer, 16380, np.empty(2, np.float32), 8)
    pool.close()


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
def test_gpu_only_chain_matches_upload_path(device, mode):
    """C = A @ B, then C + U and ReLU (the op_graph_lower chain), and the fused
    relu(A @ B + bias) twice in a row, on GpuOnly arrays with one readback at
    the end: the same bits as the Upload path, which waits after every op."""
    m, n, k = 640, 520, 384
    a = O.uniform(m * k, 11).reshape(m, k)
    b = O.uniform(k * n, 12).reshape(k, n)
    u = O.uniform(m * n, 13).reshape(m, n)
    bias = O.uniform(n, 14, -0.1, 0.1)
    w2 = O.uniform(n * n, 15, -0.05, 0.05).reshape(n, n)
    gemm = zg.GemmKernel(device, mode)
    ew = zg.ElementwiseKernels(device)
    results = {}
    for memory in (zg.MemoryUsage.Upload, zg.MemoryUsage.GpuOnly):
        pool = zg.BufferPool(device, memory)
        da, db, du, dbias, dw2 = (zg.upload(device, pool, x) for x in (a, b, u, bias, w2))
        y = ew.relu(device, pool, ew.add(device, pool, gemm.gemm(device, pool, da, db), du))
        h = gemm.gemm_bias_relu(device, pool, 1.0, da, db, dbias)
        h2 = gemm.gemm_bias_relu(device, pool, 0.5, h, dw2, dbias)
        if memory == zg.MemoryUsage.GpuOnly:
            out_y, sub_y = zg.download_async(device, y)
            out_h, sub_h = zg.download_async(device, h2)
            sub_h.wait(30.0)  # ordered after sub_y on the device stream
            assert sub_y.poll()
        else:
            out_y, out_h = zg.download(device, y), zg.download(device, h2)
        results[memory] = (out_y, out_h)
        pool.close()
    (y_up, h_up), (y_go, h_go) = results[zg.MemoryUsage.Upload], results[zg.MemoryUsage.GpuOnly]
    np.testing.assert_array_equal(bits(y_go), bits(y_up))
    np.testing.assert_array_equal(bits(h_go), bits(h_up))
    tol = 5e-3 if mode == zg.GemmMode.TF32 else 1e-5
    assert O.rel_fro(y_go, O.relu(O.add(O.sgemm(a, b), u))) <= tol
    h_ref = O.sgemm_bias_relu(O.sgemm_bias_relu(a, b, bias), w2, bias, alpha=0.5)
    assert O.rel_fro(h_go, h_ref) <= tol


def test_gpu_only_inplace_and_level1(device):
    """In-place ReLU, saxpy and sscal on GpuOnly arrays are queued too; the
    readback sees all of them, bit-exact against the oracle."""
    pool = zg.BufferPool(device, zg.MemoryUsage.GpuOnly)
    ew = zg.ElementwiseKernels(device)
    blas = zg.Blas(device)
    x = O.normal(70001, 21)
    y = O.normal(70001, 22)
    dx, dy = zg.upload(device, pool, x), zg.upload(device, pool, y)
    blas.saxpy(device, pool, 0.75, dx, dy)  # y += 0.75 x
    blas.sscal(device, pool, -2.0, dy)      # y *= -2
    ew.relu_inplace(device, dy)
    out, sub = zg.download_async(device, dy)
    sub.wait(10.0)
    ref = O.relu(O.sscal(-2.0, O.saxpy(0.75, x, y)))
    np.testing.assert_array_equal(bits(out), bits(ref))
    pool.close()
