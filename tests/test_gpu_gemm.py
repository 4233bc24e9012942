"""f32 GEMM (SIMT, 3xTF32, TF32, the two bf16-assisted splits) and the fused
bias+ReLU epilogue on the B200 against the oracle.  Tolerances (relative
Frobenius error): SIMT, TF32X3, TF32_BF16X2 and BF16X3 <= 1e-5, TF32 <= 5e-3;
the integer KATs are exact in every mode."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import _oracle as O
import zengpu_b200 as zg
from zengpu_b200 import kernels as K

pytestmark = pytest.mark.gpu

MODES = [zg.GemmMode.SIMT_FP32, zg.GemmMode.TF32X3, zg.GemmMode.TF32, zg.GemmMode.TF32_BF16X2,
         zg.GemmMode.BF16X3]
TOL = {zg.GemmMode.SIMT_FP32: 1e-5, zg.GemmMode.TF32X3: 1e-5, zg.GemmMode.TF32: 5e-3,
       zg.GemmMode.TF32_BF16X2: 1e-5, zg.GemmMode.BF16X3: 1e-5}


def bits(x) -> np.ndarray:
    return np.asarray(x, np.float32).view(np.uint32)


def run(a: np.ndarray, b: np.ndarray, mode, alpha=1.0, bias=None, relu=False) -> np.ndarray:
    ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    tbias = torch.from_numpy(bias).cuda() if bias is not None else None
    c = K.sgemm(ta, tb, mode=mode, alpha=alpha, bias=tbias, relu=relu)
    torch.cuda.synchronize()
    assert K.kernel_status() == 0
    return c.cpu().numpy()


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
def test_gemm_17x33x9_kat_exact(device, pool, kats, mode):
    """zengpu-conformance/tests/devarray_matmul.rs:56-129 through GemmKernel."""
    gemm = zg.GemmKernel(device, mode)
    a = zg.upload(device, pool, kats["gemm_17x33x9_a"])
    b = zg.upload(device, pool, kats["gemm_17x33x9_b"])
    c = gemm.gemm(device, pool, a, b)
    assert c.shape == [17, 9]
    np.testing.assert_array_equal(bits(zg.download(device, c)), bits(kats["gemm_17x33x9_c"]))
    gemm.destroy(device)


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
def test_op_graph_chain(device, pool, kats, mode):
    """examples/op_graph_lower.rs: Matmul -> Add -> Relu as three dispatches."""
    gemm = zg.GemmKernel(device, mode)
    ew = zg.ElementwiseKernels(device)
    a = zg.upload(device, pool, kats["op_graph_8x4x6_a"])
    b = zg.upload(device, pool, kats["op_graph_8x4x6_b"])
    c = zg.upload(device, pool, kats["op_graph_8x4x6_c"])
    y = ew.relu(device, pool, ew.add(device, pool, gemm.gemm(device, pool, a, b), c))
    np.testing.assert_array_equal(bits(zg.download(device, y)), bits(kats["op_graph_8x4x6_y"]))


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
def test_tiled_and_heavy_patterns(kats, mode):
    c = run(kats["tiled_31x29x23_a"], kats["tiled_31x29x23_b"], mode)
    assert np.max(np.abs(c - kats["tiled_31x29x23_c64"])) < 1e-3
    h = run(kats["heavy_64x48x40_a"], kats["heavy_64x48x40_b"], mode)
    ref = kats["heavy_64x48x40_c64"]
    assert np.all(np.abs(h - ref) / np.maximum(np.abs(ref), 1.0) <= 0.01)


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
def test_config0_256_parity(mode):
    """M=N=K=256, A,B uniform[-1,1) seed 0 (one stream, A then B)."""
    ab = O.uniform(2 * 256 * 256, 0)
    a, b = ab[: 256 * 256].reshape(256, 256), ab[256 * 256:].reshape(256, 256)
    c = run(a, b, mode)
    assert O.rel_fro(c, O.sgemm_ref(a, b)) <= TOL[mode]


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
def test_1024_parity_vs_oracle(mode):
    a = O.uniform(1024 * 1024, 2).reshape(1024, 1024)
    b = O.uniform(1024 * 1024, 102).reshape(1024, 1024)
    c = run(a, b, mode)
    ref = O.sgemm(a, b)
    err = O.rel_fro(c, ref)
    assert err <= TOL[mode], err


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
@pytest.mark.parametrize("size", [2048, 4096])
def test_large_sampled_vs_fp64(mode, size):
    ta = torch.empty((size, size), device="cuda")
    tb = torch.empty((size, size), device="cuda")
    K.fill_uniform(ta, 2)
    K.fill_uniform(tb, 3)
    c = K.sgemm(ta, tb, mode=mode)
    torch.cuda.synchronize()
    assert K.kernel_status() == 0
    a, b = ta.cpu().numpy(), tb.cpu().numpy()
    for r0, c0 in [(0, 0), (size - 256, size - 256), (size // 2 - 100, 37)]:
        ref = O.dgemm_tile(a, b, r0, c0, 256, 256)
        got = c[r0:r0 + 256, c0:c0 + 256].cpu().numpy()
        assert O.rel_fro(got, ref) <= TOL[mode]


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (3, 5, 7), (129, 257, 33), (200, 300, 130),
                                   (130, 70, 1000), (257, 513, 31), (64, 8, 4096)])
def test_odd_shapes(mode, m, n, k):
    a = O.uniform(m * k, 21).reshape(m, k)
    b = O.uniform(k * n, 22).reshape(k, n)
    for alpha in (1.0, -0.5):
        c = run(a, b, mode, alpha=alpha)
        assert O.rel_fro(c, O.sgemm(a, b, alpha)) <= max(TOL[mode], 2e-6)


@pytest.mark.parametrize("m,n,k", [(300, 520, 72), (1000, 776, 1032), (128, 128, 16), (5, 3, 4)])
def test_simt_tma_and_register_staged_kernels_agree(m, n, k):
    """SIMT runs its TMA-fed kernel on A transposed in its workspace when B is
    16-byte aligned with n % 4 == 0, and the register-staged kernel on A
    itself otherwise: with the values one float past that boundary, or with
    no workspace at all.  All give the same bits (ragged M, N and K here)."""
    a = O.uniform(m * k, 31).reshape(m, k)
    b = O.uniform(k * n, 32).reshape(k, n)
    bias = O.uniform(n, 33)
    ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    buf_a = torch.empty(m * k + 1, device="cuda")
    buf_b = torch.empty(k * n + 1, device="cuda")
    buf_a[1:] = ta.reshape(-1)
    buf_b[1:] = tb.reshape(-1)
    ua, ub = buf_a[1:].view(m, k), buf_b[1:].view(k, n)
    assert ta.data_ptr() % 16 == 0 and ua.data_ptr() % 16 != 0
    tbias = torch.from_numpy(bias).cuda()
    for relu in (False, True):
        fast = K.sgemm(ta, tb, mode=zg.GemmMode.SIMT_FP32, alpha=-0.75, bias=tbias, relu=relu)
        slow = K.sgemm(ua, ub, mode=zg.GemmMode.SIMT_FP32, alpha=-0.75, bias=tbias, relu=relu)
        torch.cuda.synchronize()
        assert K.kernel_status() == 0
        np.testing.assert_array_equal(bits(fast.cpu().numpy()), bits(slow.cpu().numpy()))
        bare = torch.empty((m, n), device="cuda")
        zg.api.check(zg.load_library().zg_sgemm_f32(
            int(zg.GemmMode.SIMT_FP32), m, n, k, -0.75, ta.data_ptr(), tb.data_ptr(),
            bare.data_ptr(), tbias.data_ptr(), int(relu), None, 0,
            torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(bits(fast.cpu().numpy()), bits(bare.cpu().numpy()))
        ref = (O.sgemm_bias_relu(a, b, bias, -0.75) if relu
               else O.sgemm(a, b, -0.75) + bias[None, :])
        assert O.rel_fro(fast.cpu().numpy(), ref) <= 1e-5


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
def test_k_zero(mode):
    a = np.zeros((5, 0), np.float32)
    b = np.zeros((0, 7), np.float32)
    c = run(a, b, mode, alpha=-1.0)
    np.testing.assert_array_equal(bits(c), bits(O.sgemm_ref(a, b, -1.0)))


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
@pytest.mark.parametrize("m,n,k", [(256, 256, 256), (300, 520, 72)])
def test_fused_bias_relu(mode, m, n, k):
    a = O.normal(m * k, 3).reshape(m, k)
    b = O.uniform(k * n, 4, -0.038, 0.038).reshape(k, n)
    bias = O.uniform(n, 5, -0.1, 0.1)
    y = run(a, b, mode, alpha=1.0, bias=bias, relu=True)
    ref = O.sgemm_bias_relu(a, b, bias)
    assert O.rel_fro(y, ref) <= TOL[mode]
    assert (y >= 0).all() and not np.signbit(y).any()


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
def test_fused_api_matches_unfused_chain(device, pool, mode):
    m, n, k = 96, 160, 48
    a = O.normal(m * k, 8).reshape(m, k)
    b = O.uniform(k * n, 9).reshape(k, n)
    bias = O.uniform(n, 10, -0.1, 0.1)
    gemm = zg.GemmKernel(device, mode)
    ew = zg.ElementwiseKernels(device)
    da, db, dbias = (zg.upload(device, pool, x) for x in (a, b, bias))
    fused = zg.download(device, gemm.gemm_bias_relu(device, pool, 1.0, da, db, dbias))
    dbias_full = zg.upload(device, pool, np.broadcast_to(bias, (m, n)))
    unfused = ew.relu(device, pool, ew.add(device, pool, gemm.gemm(device, pool, da, db), dbias_full))
    np.testing.assert_array_equal(bits(fused), bits(zg.download(device, unfused)))


def test_gemm_api_errors(device, pool):
    gemm = zg.GemmKernel(device)
    a = pool.alloc([4, 8], zg.DType.F32)
    b = pool.alloc([7, 3], zg.DType.F32)
    v = pool.alloc([8], zg.DType.F32)
    i = pool.alloc([8, 3], zg.DType.I32)
    with pytest.raises(zg.Dispatch, match="inner dimensions mismatch"):
        gemm.gemm(device, pool, a, b)
    with pytest.raises(zg.Dispatch, match="expected 2D"):
        gemm.gemm(device, pool, a, v)
    with pytest.raises(zg.Dispatch, match="only f32"):
        gemm.gemm(device, pool, a, i)
    good_b = pool.alloc([8, 3], zg.DType.F32)
    with pytest.raises(zg.Dispatch, match="bias shape"):
        gemm.gemm_bias_relu(device, pool, 1.0, a, good_b, v)


def test_default_mode_is_tf32x3(device):
    assert zg.GemmKernel(device).mode == zg.GemmMode.TF32X3


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
def test_blas_sgemm_facade(device, pool, kats, mode):
    """Blas::sgemm (zengpu-blas/src/lib.rs:74-83) delegates to its GemmKernel:
    the 17 x 33 x 9 KAT exactly, a 300 x 260 x 190 product with alpha = -1.5
    against the oracle, and the reference's shape errors."""
    blas = zg.Blas(device)
    assert blas.gemm.mode == zg.GemmMode.TF32X3  # the library default
    blas.gemm.mode = mode
    a = zg.upload(device, pool, kats["gemm_17x33x9_a"])
    b = zg.upload(device, pool, kats["gemm_17x33x9_b"])
    c = blas.sgemm(device, pool, 1.0, a, b)
    np.testing.assert_array_equal(bits(zg.download(device, c)), bits(kats["gemm_17x33x9_c"]))
    x = O.uniform(300 * 190, 81).reshape(300, 190)
    y = O.uniform(190 * 260, 82).reshape(190, 260)
    z = blas.sgemm(device, pool, -1.5, zg.upload(device, pool, x), zg.upload(device, pool, y))
    assert z.shape == [300, 260]
    assert O.rel_fro(zg.download(device, z), O.sgemm_ref(x, y, -1.5)) <= TOL[mode]
    with pytest.raises(zg.Dispatch, match="inner dimensions mismatch"):
        blas.sgemm(device, pool, 1.0, a, a)
    blas.destroy(device)


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
def test_packed_operands_into_column_panels(mode):
    """pack_a once, pack_b per column panel, each GEMM written into its column
    panel of a row-major C (pitch n) - the multi-GPU pipelined path."""
    m, n, k = 384, 1000, 520
    a = O.uniform(m * k, 31).reshape(m, k)
    b = O.uniform(k * n, 32).reshape(k, n)
    bias = O.uniform(n, 33, -0.1, 0.1)
    ta, tb, tbias = (torch.from_numpy(x).cuda() for x in (a, b, bias))
    pa = K.pack_a(ta, mode)
    c = torch.full((m, n), float("nan"), device="cuda")
    for j0, j1 in [(0, 256), (256, 600), (600, 1000)]:
        pb = K.pack_b(tb[:, j0:j1].contiguous(), mode)
        K.sgemm_packed(pa, pb, c[:, j0:j1], alpha=0.5, bias=tbias[j0:j1], relu=True)
    torch.cuda.synchronize()
    assert K.kernel_status() == 0
    ref = O.sgemm_bias_relu(a, b, bias, alpha=0.5)
    assert O.rel_fro(c.cpu().numpy(), ref) <= TOL[mode]
    # packing a strided view (row pitch > k) gives the same result
    wide = torch.zeros((m, k + 12), device="cuda")
    wide[:, :k] = ta
    pa2 = K.pack_a(wide[:, :k], mode)
    c2 = K.sgemm_packed(pa2, K.pack_b(tb, mode), alpha=0.5, bias=tbias, relu=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(c2.cpu().numpy()), bits(c.cpu().numpy()))


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
@pytest.mark.parametrize("m,n,k", [(2500, 768, 1000), (77, 130, 65), (4096, 1024, 512)])
def test_sgemm_host_pipelined(device, mode, m, n, k):
    """GemmKernel.sgemm_host: host arrays in, row panels overlapped, host C out."""
    a = O.uniform(m * k, 41).reshape(m, k)
    b = O.uniform(k * n, 42).reshape(k, n)
    bias = O.uniform(n, 43, -0.1, 0.1)
    gemm = zg.GemmKernel(device, mode)
    c = np.full((m, n), np.nan, np.float32)
    gemm.sgemm_host(device, 1.0, a, b, c, m, n, k)
    assert O.rel_fro(c, O.sgemm(a, b)) <= TOL[mode]
    c2 = np.empty((m, n), np.float32)
    gemm.sgemm_host(device, -0.25, a, b, c2, m, n, k, bias=bias, relu=True)
    assert O.rel_fro(c2, O.sgemm_bias_relu(a, b, bias, alpha=-0.25)) <= TOL[mode]
    # pinned torch host tensors take the same path
    ha = torch.from_numpy(a).pin_memory()
    hb = torch.from_numpy(b).pin_memory()
    hc = torch.empty((m, n)).pin_memory()
    gemm.sgemm_host(device, 1.0, ha, hb, hc, m, n, k)
    np.testing.assert_array_equal(bits(hc.numpy()), bits(c))


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
def test_config0_chain_gemm_add_relu(device, pool, mode):
    """The CPU-runnable configuration end to end through the drop-in API:
    C = A @ B (256^3, seed 0), then C + U (uniform, seed 5) and ReLU."""
    ab = O.uniform(2 * 256 * 256, 0)
    a, b = ab[: 256 * 256].reshape(256, 256), ab[256 * 256:].reshape(256, 256)
    u = O.uniform(256 * 256, 5).reshape(256, 256)
    gemm = zg.GemmKernel(device, mode)
    ew = zg.ElementwiseKernels(device)
    da, db, du = (zg.upload(device, pool, x) for x in (a, b, u))
    y = ew.relu(device, pool, ew.add(device, pool, gemm.gemm(device, pool, da, db), du))
    ref = O.relu(O.add(O.sgemm_ref(a, b), u))
    assert O.rel_fro(zg.download(device, y), ref) <= TOL[mode]


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
def test_8192_sampled_vs_fp64(mode):
    """The square-sweep's largest size: 8192^3, sampled 256 x 256 blocks vs f64."""
    n = 8192
    ta = torch.empty((n, n), device="cuda")
    tb = torch.empty((n, n), device="cuda")
    K.fill_uniform(ta, 2)
    K.fill_uniform(tb, 102)
    c = K.sgemm(ta, tb, mode=mode)
    torch.cuda.synchronize()
    assert K.kernel_status() == 0
    a, b = ta.cpu().numpy(), tb.cpu().numpy()
    for r0, c0 in [(0, 0), (n - 256, n - 256), (3000, 5000)]:
        ref = O.dgemm_tile(a, b, r0, c0, 256, 256)
        assert O.rel_fro(c[r0:r0 + 256, c0:c0 + 256].cpu().numpy(), ref) <= TOL[mode]
    del ta, tb, c
    torch.cuda.empty_cache()


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
@pytest.mark.parametrize("m,n,k", [(2300, 2100, 1000), (4100, 4300, 72), (2176, 2432, 8200)])
def test_cta_pair_path_shapes(mode, m, n, k):
    """Shapes with enough 256 x 256 tiles to take the CTA-pair kernel, ragged in
    every dimension (rows and columns past the last full tile, k not a multiple
    of the stage depth)."""
    ta = torch.from_numpy(O.uniform(m * k, 51).reshape(m, k)).cuda()
    tb = torch.from_numpy(O.uniform(k * n, 52).reshape(k, n)).cuda()
    tbias = torch.from_numpy(O.uniform(n, 53, -0.1, 0.1)).cuda()
    c = K.sgemm(ta, tb, mode=mode, alpha=0.75, bias=tbias, relu=True)
    torch.cuda.synchronize()
    assert K.kernel_status() == 0
    a, b = ta.cpu().numpy(), tb.cpu().numpy()
    bias = tbias.cpu().numpy()
    for r0, c0 in [(0, 0), (m - 128, n - 128), (m // 2 + 5, n // 3)]:
        ref = np.maximum(0.75 * O.dgemm_tile(a, b, r0, c0, 128, 128) + bias[c0:c0 + 128], 0.0)
        got = c[r0:r0 + 128, c0:c0 + 128].cpu().numpy()
        assert O.rel_fro(got, ref) <= TOL[mode] * 1.5


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two visible GPUs")
@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
def test_second_device_in_one_process(mode):
    """The kernels' launch attributes are per device: the same process runs the
    GEMM on device 0, then on device 1, then on device 0 again, and all three
    agree bit for bit (same kernel, same inputs)."""
    m, n, k = 2048, 2304, 520
    a = O.uniform(m * k, 61).reshape(m, k)
    b = O.uniform(k * n, 62).reshape(k, n)
    outs = []
    for dev in (0, 1, 0):
        with torch.cuda.device(dev):
            ta = torch.from_numpy(a).to(f"cuda:{dev}")
            tb = torch.from_numpy(b).to(f"cuda:{dev}")
            c = K.sgemm(ta, tb, mode=mode)
            torch.cuda.synchronize(dev)
            assert K.kernel_status() == 0
            outs.append(c.cpu().numpy())
    assert np.array_equal(bits(outs[0]), bits(outs[1]))
    assert np.array_equal(bits(outs[0]), bits(outs[2]))
    ref = O.dgemm_tile(a, b, 0, 0, 128, 128)
    assert O.rel_fro(outs[1][:128, :128], ref) <= TOL[mode] * 1.5


_TAIL_SCRIPT = r"""
import sys, numpy as np, torch
import zengpu_b200 as zg
from zengpu_b200 import kernels as K
mode, m, n, k, out = int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]), int(sys.argv[4]), sys.argv[5]
a = K.fill_uniform(torch.empty((m, k), device="cuda"), 81)
b = K.fill_uniform(torch.empty((k, n), device="cuda"), 82)
bias = K.fill_uniform(torch.empty(n, device="cuda"), 83, -0.1, 0.1)
c = K.sgemm(a, b, mode=mode, alpha=0.5, bias=bias, relu=True)
torch.cuda.synchronize()
assert K.kernel_status() == 0
np.save(out, c.cpu().numpy())
"""


@pytest.mark.parametrize("mode", [zg.GemmMode.BF16X3, zg.GemmMode.TF32X3, zg.GemmMode.TF32,
                                  zg.GemmMode.TF32_BF16X2], ids=lambda m: m.name)
def test_tail_split_keeps_bits(mode, tmp_path):
    """4096 x 4096 output tiles: 256 CTA-pair tiles make 3 waves of 74 and a
    last wave of 34, which runs as 68 half-width (256 x 128) units.  The same
    GEMM with whole tiles only (ZENGPU_GEMM_TAIL_SPLIT=0, a fresh process)
    gives the same bits, and both meet the bar on sampled blocks."""
    import os
    import subprocess
    import sys
    m = n = 4096
    k = 1024
    outs = []
    for flag in ("1", "0"):
        path = tmp_path / f"c{flag}.npy"
        env = dict(os.environ, ZENGPU_GEMM_TAIL_SPLIT=flag)
        subprocess.run([sys.executable, "-c", _TAIL_SCRIPT, str(int(mode)), str(m), str(n),
                        str(k), str(path)], env=env, check=True, timeout=600)
        outs.append(np.load(path))
    np.testing.assert_array_equal(bits(outs[0]), bits(outs[1]))
    a = K.fill_uniform(torch.empty((m, k), device="cuda"), 81).cpu().numpy()
    b = K.fill_uniform(torch.empty((k, n), device="cuda"), 82).cpu().numpy()
    bias = K.fill_uniform(torch.empty(n, device="cuda"), 83, -0.1, 0.1).cpu().numpy()
    # a block of a whole tile and blocks of the last wave's tiles (columns of both halves)
    for r0, c0 in [(0, 0), (m - 128, n - 256), (m - 128, n - 128)]:
        ref = np.maximum(0.5 * O.dgemm_tile(a, b, r0, c0, 128, 128) + bias[c0:c0 + 128], 0)
        assert O.rel_fro(outs[0][r0:r0 + 128, c0:c0 + 128], ref) <= TOL[mode]
