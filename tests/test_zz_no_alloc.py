"""zg_sgemm_f32_noalloc: the GEMM entry point for callers that cannot
allocate device memory when they call (a framework that owns all of HBM in
its own pool, a latency-critical loop that cannot pay for cudaMalloc's
device-wide synchronisation, code inside an allocator callback).  It must
match zg_sgemm_f32 with a caller workspace, on two calls in a row, allocate
nothing, and reject shapes beyond its 64 MiB static scratch (except in SIMT,
whose workspace is optional).

This file is collected last on purpose, so that a stop-at-first-failure run
has already run every other test; it also passes alone in a fresh process."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

import _oracle as O
import zengpu_b200 as zg
from zengpu_b200 import _lib as L
from zengpu_b200 import kernels as K

pytestmark = pytest.mark.gpu

TOL = {zg.GemmMode.SIMT_FP32: 1e-5, zg.GemmMode.TF32X3: 1e-5, zg.GemmMode.TF32: 5e-3,
       zg.GemmMode.TF32_BF16X2: 1e-5, zg.GemmMode.BF16X3: 1e-5}


def _noalloc(a, b, c, mode, alpha=1.0, bias=None, relu=False) -> int:
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    m, k = a.shape
    n = b.shape[1]
    return L.load().zg_sgemm_f32_noalloc(int(mode), m, n, k, float(alpha), a.data_ptr(),
                                         b.data_ptr(), c.data_ptr(),
                                         bias.data_ptr() if bias is not None else None,
                                         1 if relu else 0, stream)


def _inputs(m, n, k, seed):
    a = torch.from_numpy(O.uniform(m * k, seed).reshape(m, k)).cuda()
    b = torch.from_numpy(O.uniform(k * n, seed + 1).reshape(k, n)).cuda()
    bias = torch.from_numpy(O.uniform(n, seed + 2, -0.1, 0.1)).cuda()
    return a, b, bias


MODES = [zg.GemmMode.BF16X3, zg.GemmMode.TF32_BF16X2, zg.GemmMode.TF32X3, zg.GemmMode.TF32,
         zg.GemmMode.SIMT_FP32]


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
def test_noalloc_matches_workspace_entry_point_twice(mode):
    torch.cuda.set_device(0)
    # two calls in a row with different shapes and data: the shared scratch
    # keeps the first call's contents, the second must not depend on them
    for (m, n, k, seed, relu) in [(1024, 768, 1000, 40, False), (333, 2048, 1536, 50, True)]:
        a, b, bias = _inputs(m, n, k, seed)
        c_ref = K.sgemm(a, b, mode=mode, alpha=0.5, bias=bias if relu else None, relu=relu)
        c = torch.full((m, n), float("nan"), device="cuda")
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        rc = _noalloc(a, b, c, mode, alpha=0.5, bias=bias if relu else None, relu=relu)
        assert rc == 0, L.last_error()
        torch.cuda.synchronize()
        assert K.kernel_status() == 0
        if seed == 50:  # scratch already looked up and loaded: nothing may allocate now
            assert torch.cuda.mem_get_info()[0] == free_before
        got = c.cpu().numpy()
        err = O.rel_fro(got, c_ref.cpu().numpy())
        assert err <= TOL[mode], err
        # and against the oracle (the reference CPU backend's arithmetic)
        an, bn = a.cpu().numpy(), b.cpu().numpy()
        ref = (O.sgemm_bias_relu(an, bn, bias.cpu().numpy(), alpha=0.5) if relu
               else O.sgemm(an, bn, 0.5))
        err = O.rel_fro(got, ref)
        assert err <= TOL[mode], err


def test_noalloc_bf16x3_largest_cube_that_fits():
    """BF16X3 needs 8 bytes of scratch per (m + n) * k: 2880^3 (63.3 MiB) is the
    largest multiple of 64 that fits, and takes the CTA-pair kernel."""
    torch.cuda.set_device(0)
    s = 2880
    mode = zg.GemmMode.BF16X3
    assert K.workspace_bytes(mode, s, s, s) <= 64 << 20 < K.workspace_bytes(mode, s + 64, s + 64, s + 64)
    for seed in (60, 61):
        a = K.fill_uniform(torch.empty((s, s), device="cuda"), seed)
        b = K.fill_uniform(torch.empty((s, s), device="cuda"), seed + 100)
        c = torch.full((s, s), float("nan"), device="cuda")
        assert _noalloc(a, b, c, mode) == 0, L.last_error()
        ref = K.sgemm(a, b, mode=mode)
        torch.cuda.synchronize()
        assert K.kernel_status() == 0
        assert torch.equal(c.view(torch.int32), ref.view(torch.int32))
        an, bn = a.cpu().numpy(), b.cpu().numpy()
        for r0, c0 in [(0, 0), (s - 128, s - 128)]:
            tile = O.dgemm_tile(an, bn, r0, c0, 128, 128)
            assert O.rel_fro(c[r0:r0 + 128, c0:c0 + 128].cpu().numpy(), tile) <= 1e-5


def test_noalloc_rejects_shapes_beyond_the_static_scratch():
    torch.cuda.set_device(0)
    m = n = k = 2056  # TF32X3 planes need more than 64 MiB
    assert K.workspace_bytes(zg.GemmMode.TF32X3, m, n, k) > 64 << 20
    a = torch.zeros((m, k), device="cuda")
    b = torch.zeros((k, n), device="cuda")
    c = torch.full((m, n), 7.0, device="cuda")
    rc = _noalloc(a, b, c, zg.GemmMode.TF32X3)
    assert rc == zg.Dispatch.code
    assert "static maximum" in L.last_error()
    torch.cuda.synchronize()
    assert bool((c == 7.0).all())  # nothing was launched
    # the largest cube that fits still runs
    a2, b2, _ = _inputs(2048, 2048, 2048, 60)
    c2 = torch.empty((2048, 2048), device="cuda")
    assert _noalloc(a2, b2, c2, zg.GemmMode.TF32X3) == 0, L.last_error()
    ref = K.sgemm(a2, b2, mode=zg.GemmMode.TF32X3)
    torch.cuda.synchronize()
    assert O.rel_fro(c2.cpu().numpy(), ref.cpu().numpy()) <= 1e-5


def test_noalloc_simt_beyond_the_scratch_runs_without_it():
    """SIMT's workspace (A transposed, 4 bytes per m * k element) is optional:
    a shape whose transposed A does not fit the 64 MiB array runs on the
    register-staged kernel instead of being rejected, with the same bits as the
    workspace path, twice in a row and without allocating."""
    torch.cuda.set_device(0)
    m, n, k = 4160, 256, 4096
    mode = zg.GemmMode.SIMT_FP32
    assert K.workspace_bytes(mode, m, n, k) > 64 << 20
    a, b, bias = _inputs(m, n, k, 70)
    ref = K.sgemm(a, b, mode=mode, alpha=-0.25, bias=bias, relu=True)
    for _ in range(2):
        c = torch.full((m, n), float("nan"), device="cuda")
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        assert _noalloc(a, b, c, mode, alpha=-0.25, bias=bias, relu=True) == 0, L.last_error()
        torch.cuda.synchronize()
        assert K.kernel_status() == 0
        assert torch.cuda.mem_get_info()[0] == free_before
        assert torch.equal(c.view(torch.int32), ref.view(torch.int32))
