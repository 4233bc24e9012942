"""DeviceArray add / ReLU / Level-1 on the B200 against the oracle: bit-exact.

Mirrors zengpu-conformance/tests/devarray_elementwise.rs (KATs through the
ElementwiseKernels + BufferPool API), then seeded parity at the workload
sizes (256x256 and 2^28 elements), the edge sizes of the float4 path and the
pinned ReLU semantics."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import _oracle as O
import zengpu_b200 as zg
from zengpu_b200 import kernels as K

pytestmark = pytest.mark.gpu


def bits(x) -> np.ndarray:
    return np.asarray(x, np.float32).view(np.uint32)


@pytest.fixture(scope="module")
def ew(device):
    k = zg.ElementwiseKernels(device)
    yield k
    k.destroy(device)


@pytest.mark.parametrize("name", ["vec_add_1024", "vec_add_8", "add_quarter_1024"])
def test_add_kats(device, pool, ew, kats, name):
    a = zg.upload(device, pool, kats[f"{name}_a"])
    b = zg.upload(device, pool, kats[f"{name}_b"])
    out = ew.add(device, pool, a, b)
    assert out.shape == a.shape and out.dtype == zg.DType.F32
    np.testing.assert_array_equal(bits(zg.download(device, out)), bits(kats[f"{name}_out"]))
    for x in (a, b, out):
        pool.free(x)


def test_add_relu_conformance(device, pool, ew, kats):
    """zengpu-conformance/tests/devarray_elementwise.rs:59-143 on this backend."""
    a = zg.upload(device, pool, kats["add_relu_256_a"])
    b = zg.upload(device, pool, kats["add_relu_256_b"])
    s = ew.add(device, pool, a, b)
    r = ew.relu(device, pool, s)
    np.testing.assert_array_equal(bits(zg.download(device, s)), bits(kats["add_relu_256_sum"]))
    np.testing.assert_array_equal(bits(zg.download(device, r)), bits(kats["add_relu_256_relu"]))
    for x in (a, b, s, r):
        pool.free(x)


def test_config0_add_relu_seeded(device, pool, ew):
    """256x256 add of uniform[-1,1) (seeds 0 and 1) followed by ReLU."""
    x = O.uniform(256 * 256, 0).reshape(256, 256)
    y = O.uniform(256 * 256, 1).reshape(256, 256)
    a, b = zg.upload(device, pool, x), zg.upload(device, pool, y)
    s = ew.add(device, pool, a, b)
    ew.relu_inplace(device, s)
    np.testing.assert_array_equal(bits(zg.download(device, s)), bits(O.relu(O.add(x, y))))


def test_elementwise_errors(device, pool, ew):
    a = pool.alloc([4, 4], zg.DType.F32)
    b = pool.alloc([16], zg.DType.F32)
    c = pool.alloc([4, 4], zg.DType.I32)
    with pytest.raises(zg.Dispatch, match="shape mismatch"):
        ew.add(device, pool, a, b)
    with pytest.raises(zg.Dispatch, match="only DType::F32"):
        ew.add(device, pool, a, c)
    with pytest.raises(zg.Dispatch, match="only DType::F32"):
        ew.relu(device, pool, c)


@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 255, 1023, 1025, 65537, 1 << 20])
def test_stream_sizes_and_tails(n):
    x = O.normal(n, 10)
    y = O.normal(n, 11)
    tx, ty = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    np.testing.assert_array_equal(bits(K.add_f32(tx, ty).cpu()), bits(O.add(x, y)))
    np.testing.assert_array_equal(bits(K.relu_f32(tx).cpu()), bits(O.relu(x)))


def test_unaligned_views_take_scalar_path():
    base = torch.from_numpy(O.normal(4099, 3)).cuda()
    x = base[1:4098]  # data_ptr 4 bytes past a 16-byte boundary
    y = base[2:4099]
    out = torch.empty(4097, device="cuda")[0:4097]
    K.add_f32(x, y, out)
    np.testing.assert_array_equal(bits(out.cpu()), bits(O.add(x.cpu().numpy(), y.cpu().numpy())))
    r = K.relu_f32(x, torch.empty_like(x))
    np.testing.assert_array_equal(bits(r.cpu()), bits(O.relu(x.cpu().numpy())))


def test_relu_edge_cases(kats):
    t = torch.from_numpy(kats["relu_edge_in"].copy()).cuda()
    np.testing.assert_array_equal(bits(K.relu_f32(t).cpu()), bits(kats["relu_edge_out"]))
    K.relu_f32(t, t)  # in place
    np.testing.assert_array_equal(bits(t.cpu()), bits(kats["relu_edge_out"]))


def test_generators_match_host():
    for seed in range(5):
        t = torch.empty(100003, device="cuda")
        K.fill_uniform(t, seed)
        np.testing.assert_array_equal(bits(t.cpu()), bits(O.uniform(100003, seed)))
    t = torch.empty(4096, device="cuda")
    K.fill_uniform(t, 9, -0.1, 0.1)
    np.testing.assert_array_equal(bits(t.cpu()), bits(O.uniform(4096, 9, -0.1, 0.1)))
    z = torch.empty(100001, device="cuda")
    K.fill_normal(z, 1)
    np.testing.assert_allclose(z.cpu().numpy(), O.normal(100001, 1), rtol=1e-6, atol=1e-6)


def test_level1_bit_exact(device, pool):
    x = O.normal(10007, 4)
    y = O.normal(10007, 5)
    blas = zg.Blas(device)
    ax, ay = zg.upload(device, pool, x), zg.upload(device, pool, y)
    blas.saxpy(device, pool, 0.75, ax, ay)
    np.testing.assert_array_equal(bits(zg.download(device, ay)), bits(O.saxpy(0.75, x, y)))
    blas.sscal(device, pool, -2.5, ax)
    np.testing.assert_array_equal(bits(zg.download(device, ax)), bits(O.sscal(-2.5, x)))
    with pytest.raises(zg.Dispatch, match="shape mismatch"):
        blas.saxpy(device, pool, 1.0, ax, pool.alloc([3], zg.DType.F32))


def test_bandwidth_config_full_size():
    """2^28-element add and in-place ReLU of normal(0,1) data (1 GiB each):
    bit-exact against the oracle over every element."""
    n = 1 << 28
    x = torch.empty(n, device="cuda")
    y = torch.empty(n, device="cuda")
    K.fill_normal(x, 1)
    K.fill_normal(y, 2)
    z = K.add_f32(x, y)
    hx, hy, hz = x.cpu().numpy(), y.cpu().numpy(), z.cpu().numpy()
    np.testing.assert_array_equal(bits(hz), bits(O.add(hx, hy, threads=8)))
    K.relu_f32(z, z)
    np.testing.assert_array_equal(bits(z.cpu().numpy()), bits(O.relu(hz, threads=8)))
    del x, y, z
    torch.cuda.empty_cache()
