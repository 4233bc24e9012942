"""The GpuDevice compute subset on the B200: buffers, handles, pools,
caller PTX modules, dispatch and submissions, with the reference CUDA
backend's error behaviour (zengpu-cuda/src/lib.rs:1288-1975)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import _oracle as O
import zengpu_b200 as zg

pytestmark = pytest.mark.gpu

U = zg.BufferUsage

# A vec_add kernel written for this test in PTX (driver JIT to sm_100a).
VEC_ADD_PTX = b"""
.version 8.0
.target sm_90
.address_size 64
.visible .entry vec_add_f32(.param .u64 pa, .param .u64 pb, .param .u64 pc, .param .u32 pn)
{
    .reg .pred %p;
    .reg .b32 %r<6>;
    .reg .b64 %rd<8>;
    .reg .f32 %f<4>;
    ld.param.u64 %rd1, [pa];
    ld.param.u64 %rd2, [pb];
    ld.param.u64 %rd3, [pc];
    ld.param.u32 %r1, [pn];
    mov.u32 %r2, %ctaid.x;
    mov.u32 %r3, %ntid.x;
    mov.u32 %r4, %tid.x;
    mad.lo.u32 %r5, %r2, %r3, %r4;
    setp.ge.u32 %p, %r5, %r1;
    @%p bra DONE;
    mul.wide.u32 %rd4, %r5, 4;
    add.u64 %rd5, %rd1, %rd4;
    add.u64 %rd6, %rd2, %rd4;
    add.u64 %rd7, %rd3, %rd4;
    ld.global.f32 %f1, [%rd5];
    ld.global.f32 %f2, [%rd6];
    add.rn.f32 %f3, %f1, %f2;
    st.global.f32 [%rd7], %f3;
DONE:
    ret;
}
"""


def f32bytes(x) -> bytes:
    return np.asarray(x, np.float32).tobytes()


def test_buffer_roundtrip_and_errors(device):
    h = device.create_buffer(64, U.STORAGE | U.READBACK)
    device.write_buffer(h, 0, f32bytes(np.arange(16)))
    assert np.frombuffer(device.read_buffer(h, 0, 64), np.float32).tolist() == list(range(16))
    assert np.frombuffer(device.read_buffer(h, 32, 8), np.float32).tolist() == [8.0, 9.0]
    with pytest.raises(zg.Backend, match="write out of bounds"):
        device.write_buffer(h, 60, b"\0" * 8)
    with pytest.raises(zg.BindingMismatch, match="exceeds"):
        device.read_buffer(h, 60, 8)
    nr = device.create_buffer(16, U.STORAGE)
    with pytest.raises(zg.MissingUsage) as mu:
        device.read_buffer(nr, 0, 4)
    # UsageError::MissingUsage's fields as zengpu-cuda/src/lib.rs:539-542 sets them
    assert (mu.value.resource, mu.value.needed) == ("buffer", "READBACK")
    device.destroy_buffer(h)
    with pytest.raises(zg.StaleHandle) as st:
        device.write_buffer(h, 0, b"\0" * 4)
    assert st.value.index == h.index and st.value.expected_gen == h.generation
    assert st.value.actual_gen != h.generation
    device.destroy_buffer(h)  # stale destroy is a no-op
    device.destroy_buffer(nr)


def test_copy_buffer_rules(device):
    src = device.create_buffer(32, U.STORAGE | U.TRANSFER_SRC)
    dst = device.create_buffer(32, U.STORAGE | U.TRANSFER_DST | U.READBACK)
    plain = device.create_buffer(32, U.STORAGE | U.READBACK)
    device.write_buffer(src, 0, f32bytes([1, 2, 3, 4, 5, 6, 7, 8]))
    device.copy_buffer(src, 4, dst, 0, 12)
    assert np.frombuffer(device.read_buffer(dst, 0, 12), np.float32).tolist() == [2, 3, 4]
    with pytest.raises(zg.MissingUsage):
        device.copy_buffer(plain, 0, dst, 0, 4)
    with pytest.raises(zg.MissingUsage):
        device.copy_buffer(src, 0, plain, 0, 4)
    with pytest.raises(zg.BindingMismatch, match="copy ranges"):
        device.copy_buffer(src, 16, dst, 0, 32)
    device.copy_buffer(src, 0, dst, 0, 0)  # zero-length is a no-op
    for b in (src, dst, plain):
        device.destroy_buffer(b)


def test_pool_size_classes_and_reuse(device):
    pool = zg.BufferPool(device)
    a = pool.alloc([2, 3, 4], zg.DType.F32)
    assert a.shape == [2, 3, 4] and a.stride == [12, 4, 1]
    assert a.len() == 24 and a.size_bytes() == 96 and a.allocation_size_bytes() == 256
    pool.free(a)
    assert pool.free_count(256) == 1
    b = pool.alloc([50], zg.DType.F32)  # 200 B: same 256 B class, reuses the buffer
    assert b.buffer == a.buffer and pool.free_count(256) == 0
    c = pool.alloc([100], zg.DType.F32)  # 400 B -> 512 B class
    assert c.allocation_size_bytes() == 512 and c.buffer != a.buffer
    pool.close()


def test_ptx_module_dispatch(device):
    shader = device.create_shader(zg.ShaderKind.PTX, VEC_ADD_PTX)
    pipe = device.create_compute_pipeline(shader, "vec_add_f32", (256, 1, 1))
    n = 1024
    a = device.create_buffer(n * 4)
    b = device.create_buffer(n * 4)
    c = device.create_buffer(n * 4)
    device.write_buffer(a, 0, f32bytes(np.arange(n)))
    device.write_buffer(b, 0, f32bytes(100 * np.arange(n)))
    device.dispatch(pipe, [a.index, b.index, c.index], [zg.u32(n)], ((n + 255) // 256, 1, 1))
    out = np.frombuffer(device.read_buffer(c, 0, n * 4), np.float32)
    np.testing.assert_array_equal(out, 101 * np.arange(n, dtype=np.float32))
    with pytest.raises(zg.PipelineCreation):
        device.create_compute_pipeline(shader, "no_such_entry")
    with pytest.raises(zg.ShaderCompile):
        device.create_shader(zg.ShaderKind.PTX, b"this is not ptx")
    device.destroy_pipeline(pipe)
    with pytest.raises(zg.Dispatch, match="stale pipeline"):
        device.dispatch(pipe, [a.index, b.index, c.index], [zg.u32(n)], (4, 1, 1))
    device.destroy_shader(shader)
    for h in (a, b, c):
        device.destroy_buffer(h)


def test_builtin_pipelines_through_generic_dispatch(device):
    sh = device.create_shader(zg.ShaderKind.BUILTIN)
    add = device.create_compute_pipeline(sh, "add_f32")
    n = 1000
    a, b, c = (device.create_buffer(n * 4) for _ in range(3))
    device.write_buffer(a, 0, f32bytes(np.arange(n)))
    device.write_buffer(b, 0, f32bytes(np.ones(n)))
    device.dispatch(add, [a.index, b.index, c.index], [zg.u32(n)], (4, 1, 1))
    out = np.frombuffer(device.read_buffer(c, 0, n * 4), np.float32)
    np.testing.assert_array_equal(out, np.arange(n, dtype=np.float32) + 1)
    with pytest.raises(zg.BindingMismatch):
        device.dispatch(add, [a.index, b.index], [zg.u32(n)], (4, 1, 1))
    with pytest.raises(zg.BindingMismatch):
        device.dispatch(add, [a.index, b.index, c.index], [zg.f32(1.0)], (4, 1, 1))
    with pytest.raises(zg.PipelineCreation):
        device.create_compute_pipeline(sh, "not_a_builtin")


def test_submission_batch_chain_and_deferred_reuse(device):
    """zengpu-cuda/src/lib.rs:1860-1975 on this backend."""
    n = 256
    shader = device.create_shader(zg.ShaderKind.PTX, VEC_ADD_PTX)
    pipe = device.create_compute_pipeline(shader, "vec_add_f32", (256, 1, 1))
    bufs = [device.create_buffer(n * 4) for _ in range(4)]
    a, b, s, out = bufs
    device.write_buffer(a, 0, f32bytes(np.arange(n)))
    device.write_buffer(b, 0, f32bytes(10 * np.arange(n)))
    grid = (1, 1, 1)
    sub = device.submit_batch([
        (pipe, [a.index, b.index, s.index], [zg.u32(n)], grid),
        (pipe, [s.index, s.index, out.index], [zg.u32(n)], grid),
    ])
    second_out = device.create_buffer(n * 4)
    sub2 = device.submit(pipe, [a.index, b.index, second_out.index], [zg.u32(n)], grid)
    with pytest.raises(zg.BindingMismatch, match="pending"):
        device.write_buffer(a, 0, b"\0" * 4)
    retired = s.index
    device.destroy_buffer(s)
    device.destroy_pipeline(pipe)
    with pytest.raises(zg.StaleHandle):
        device.write_buffer(s, 0, b"\0" * 4)
    while_pending = device.create_buffer(n * 4)
    assert while_pending.index != retired
    try:
        sub.wait(0.0)
    except zg.Timeout:
        pass
    sub.wait(5.0)
    assert sub.poll()
    sub2.wait(5.0)
    assert sub2.poll()
    after = device.create_buffer(n * 4)
    assert after.index == retired
    got = np.frombuffer(device.read_buffer(out, 0, n * 4), np.float32)
    np.testing.assert_array_equal(got, 2 * 11 * np.arange(n, dtype=np.float32))
    for h in (a, b, out, second_out, while_pending, after):
        device.destroy_buffer(h)
    device.destroy_shader(shader)


def test_device_queries(device):
    assert device.device_ordinal() == 0
    assert device.can_peer(0)
    assert device.stream() != 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_copy_from_peer_two_devices(device):
    """GpuDevice::can_peer / copy_from_peer (zengpu-hal/src/device.rs:91-106):
    32 MiB + 12 bytes copied device 1 -> device 0 and back over NVLink, bit for
    bit, at NVLink speed (direct peer copy once can_peer enabled access); a
    copy longer than either buffer is rejected as the HIP backend does."""
    other = zg.CudaDevice(1)
    try:
        assert device.can_peer(1) and other.can_peer(0)
        n = (32 << 20) // 4 + 3
        data = O.uniform(n, 91)
        src = other.create_buffer(n * 4)
        other.write_buffer(src, 0, data)
        dst = device.create_buffer(n * 4)
        device.copy_from_peer(dst, other, src, n * 4)
        got = np.frombuffer(device.read_buffer(dst, 0, n * 4), np.float32)
        np.testing.assert_array_equal(got.view(np.uint32), data.view(np.uint32))
        back = other.create_buffer(n * 4)
        other.copy_from_peer(back, device, dst, n * 4)
        got2 = np.frombuffer(other.read_buffer(back, 0, n * 4), np.float32)
        np.testing.assert_array_equal(got2.view(np.uint32), data.view(np.uint32))
        import time
        t0 = time.perf_counter()
        for _ in range(5):
            device.copy_from_peer(dst, other, src, n * 4)
        gbs = 5 * n * 4 / (time.perf_counter() - t0) / 1e9
        assert gbs > 100, gbs  # NVLink, not a copy staged through the host
        with pytest.raises(zg.Backend, match="exceeds"):
            device.copy_from_peer(dst, other, src, n * 4 + 4)
        for h in (src, back):
            other.destroy_buffer(h)
        device.destroy_buffer(dst)
    finally:
        other.close()
