"""Parity of the GEMM modes at the full benchmark configurations, on the B200.

* the sharded configuration: M = N = 32768, K = 8192 (seed 4), computed as two
  row shards the way the multi-GPU path splits it; 16 random 128 x 128 tiles
  against float64;
* the op_graph_lower MLP (examples/op_graph_lower.rs:39-68): X 4096 x 4096
  normal(0, 1) seed 3 through four layers Y = relu(X @ W + b), W Kaiming-uniform
  (bound sqrt(6 / 4096)), b uniform[-0.1, 0.1), fused epilogue and the unfused
  gemm -> add -> relu chain, compared with the oracle (zgo_sgemm_bias_relu, the
  reference's unfused f32 arithmetic) on sampled rows (rows of an MLP are
  independent).  Layer by layer, the oracle is given the GPU's input to that
  layer, so each layer is one GEMM held to its mode's bar; the whole chain is
  also compared with the oracle's own chain from X, where the errors of the
  four layers add up, at four times the bar;
* a margin case for the split modes: K = 32768 (64 TMEM accumulation chunks)
  with operands whose magnitudes span 2^-8 .. 2^8.

Tolerances (relative Frobenius error): SIMT, TF32X3, TF32_BF16X2 and BF16X3
<= 1e-5; TF32 <= 5e-3."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import _oracle as O
import zengpu_b200 as zg
from zengpu_b200 import kernels as K

pytestmark = pytest.mark.gpu

MODES = [zg.GemmMode.SIMT_FP32, zg.GemmMode.TF32X3, zg.GemmMode.TF32, zg.GemmMode.TF32_BF16X2,
         zg.GemmMode.BF16X3]
FP32_CLASS = [zg.GemmMode.BF16X3, zg.GemmMode.TF32_BF16X2, zg.GemmMode.TF32X3]
TOL = {zg.GemmMode.SIMT_FP32: 1e-5, zg.GemmMode.TF32X3: 1e-5, zg.GemmMode.TF32: 5e-3,
       zg.GemmMode.TF32_BF16X2: 1e-5, zg.GemmMode.BF16X3: 1e-5}


def bits(x) -> np.ndarray:
    return np.asarray(x, np.float32).view(np.uint32)


# ---- sharded configuration: 32768 x 32768 x 8192 ------------------------------------
@pytest.fixture(scope="module")
def sharded_operands():
    m = n = 32768
    k = 8192
    ta = K.fill_uniform(torch.empty((m, k), device="cuda"), 4)
    tb = K.fill_uniform(torch.empty((k, n), device="cuda"), 1004)
    torch.cuda.synchronize()
    yield ta, tb, ta.cpu().numpy(), tb.cpu().numpy()
    del ta, tb
    torch.cuda.empty_cache()


@pytest.mark.parametrize("mode", FP32_CLASS, ids=lambda m: m.name)
def test_sharded_config_tiles_vs_fp64(sharded_operands, mode):
    """Two row shards of 16384 rows each, as two GPUs would compute them."""
    ta, tb, a, b = sharded_operands
    m, k = ta.shape
    n = tb.shape[1]
    c = torch.empty((m, n), device="cuda")
    for r0, r1 in [(0, m // 2), (m // 2, m)]:
        K.sgemm(ta[r0:r1], tb, mode=mode, out=c[r0:r1])
    torch.cuda.synchronize()
    assert K.kernel_status() == 0
    rng = np.random.default_rng(4)
    worst = 0.0
    for _ in range(16):
        r0 = int(rng.integers(0, m // 128)) * 128
        c0 = int(rng.integers(0, n // 128)) * 128
        ref = O.dgemm_tile(a, b, r0, c0, 128, 128)
        worst = max(worst, O.rel_fro(c[r0:r0 + 128, c0:c0 + 128].cpu().numpy(), ref))
    del c
    torch.cuda.empty_cache()
    assert worst <= TOL[mode], worst


# ---- op_graph_lower MLP: 4 x relu(X @ W + b), 4096 x 4096 ----------------------------
MLP_ROWS = [(0, 128), (2000, 2128), (3968, 4096)]


@pytest.fixture(scope="module")
def mlp_operands():
    bsz = hid = 4096
    layers = 4
    bound = math.sqrt(6.0 / hid)
    x = O.normal(bsz * hid, 3).reshape(bsz, hid)
    ws = [O.uniform(hid * hid, 100 + i, -bound, bound).reshape(hid, hid) for i in range(layers)]
    bs = [O.uniform(hid, 200 + i, -0.1, 0.1) for i in range(layers)]
    # the oracle's own chain (unfused f32: fl(sum) -> + bias -> relu) from X
    h = np.concatenate([x[r0:r1] for r0, r1 in MLP_ROWS])
    chain = []
    for w, b in zip(ws, bs):
        h = O.sgemm_bias_relu(h, w, b)
        chain.append(h)
    return x, ws, bs, chain


def _sampled(t: torch.Tensor) -> np.ndarray:
    return np.concatenate([t[r0:r1].cpu().numpy() for r0, r1 in MLP_ROWS])


@pytest.mark.parametrize("mode", MODES, ids=lambda m: m.name)
def test_mlp_fused_and_unfused_vs_oracle(mlp_operands, mode):
    x, ws, bs, chain = mlp_operands
    tx = torch.from_numpy(x).cuda()
    tws = [torch.from_numpy(w).cuda() for w in ws]
    tbs = [torch.from_numpy(b).cuda() for b in bs]
    fused, unfused = [], []
    h = tx
    for w, b in zip(tws, tbs):
        h = K.sgemm(h, w, mode=mode, bias=b, relu=True)
        fused.append(h)
    h = tx
    for w, b in zip(tws, tbs):
        t = K.sgemm(h, w, mode=mode)
        h = K.relu_f32(K.add_f32(t, b.expand_as(t).contiguous()))
        unfused.append(h)
    torch.cuda.synchronize()
    assert K.kernel_status() == 0
    layer_in = np.concatenate([x[r0:r1] for r0, r1 in MLP_ROWS])
    for layer, (f, u, w, b) in enumerate(zip(fused, unfused, ws, bs)):
        # the fused epilogue rounds exactly as the unfused chain: same bits
        assert torch.equal(f.view(torch.int32), u.view(torch.int32)), layer
        got = _sampled(f)
        assert (got >= 0).all() and not np.signbit(got).any()
        err = O.rel_fro(got, O.sgemm_bias_relu(layer_in, w, b))
        assert err <= TOL[mode], (layer, err)
        layer_in = got
    err = O.rel_fro(_sampled(fused[-1]), chain[-1])
    assert err <= len(ws) * TOL[mode], err


# ---- split-mode margin: K = 32768, magnitudes over 17 binades ---------------------
def _wide(n: int, seed: int, span: int = 8) -> np.ndarray:
    """uniform[-1, 1) * 2^e, e a seeded integer in [-span, span]."""
    u = O.uniform(n, seed)
    e = np.floor((O.uniform(n, seed + 500) + 1.0) * 0.5 * (2 * span + 1)).astype(np.int32) - span
    return (u * np.ldexp(np.float32(1.0), e)).astype(np.float32)


@pytest.mark.parametrize("mode", FP32_CLASS, ids=lambda m: m.name)
@pytest.mark.parametrize("m,n", [(512, 512), (2560, 2304)])
def test_split_modes_margin_k32768_wide_magnitudes(mode, m, n):
    """512 x 512 takes the one-CTA kernel, 2560 x 2304 the CTA-pair kernel."""
    k = 32768
    a = _wide(m * k, 71).reshape(m, k)
    b = _wide(k * n, 72).reshape(k, n)
    c = K.sgemm(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), mode=mode)
    torch.cuda.synchronize()
    assert K.kernel_status() == 0
    got = c.cpu().numpy()
    for r0, c0 in [(0, 0), (m - 128, n - 128), (m // 2 - 64, n // 3)]:
        ref = a[r0:r0 + 128].astype(np.float64) @ b[:, c0:c0 + 128].astype(np.float64)
        err = O.rel_fro(got[r0:r0 + 128, c0:c0 + 128], ref)
        assert err <= TOL[mode], (r0, c0, err)
