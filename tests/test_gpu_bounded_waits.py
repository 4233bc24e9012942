"""Bounded on-device waits end with a status, not a hang.

A GEMM gated on a B chunk whose flag nothing ever raises (a chain with no
upstream rank) gives up after the 2 s wait limit, reports the gate bit
through zg_kernel_status, and leaves the context usable: an ordinary GEMM
right after it is correct.  zg_bchain_abort raises every local flag, so a
gated GEMM of a later step runs at once.  No GPU fault is involved: the wait
simply runs out, in the single-CTA and in the CTA-pair kernel."""
from __future__ import annotations

import ctypes as C
import time

import pytest
import torch

import _oracle as O
import zengpu_b200 as zg
from zengpu_b200 import _lib as L
from zengpu_b200 import kernels as K

pytestmark = pytest.mark.gpu

ERR_TC_GATE = 1 << 4  # status bit of the GEMM's arrival gate


@pytest.mark.parametrize("m,n,k", [(256, 512, 256), (2304, 2304, 128)],
                         ids=["single-cta", "cta-pair"])
def test_gate_that_never_opens_reports_and_recovers(m, n, k):
    mode = zg.GemmMode.BF16X3
    lib = L.load()
    K.kernel_status()  # start from a clear status word
    chain = C.c_void_p()
    handle = (C.c_uint8 * 64)()
    zg.api.check(lib.zg_bchain_create(int(mode), k, n, 256, C.byref(chain), handle))
    try:
        a = torch.from_numpy(O.uniform(m * k, 5).reshape(m, k)).cuda()
        pa = K.pack_a(a, mode)
        c = torch.empty((m, n), device="cuda")
        s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()

        t0 = time.time()
        zg.api.check(lib.zg_bchain_gemm(chain, 1, 1, m, 1.0, pa.buf.data_ptr(), c.data_ptr(), n,
                                        None, 0, s))
        torch.cuda.synchronize()
        waited = time.time() - t0
        status = K.kernel_status()
        assert status & ERR_TC_GATE, hex(status)
        assert 1.5 < waited < 30.0, waited

        # the context still works
        b = O.uniform(k * n, 6).reshape(k, n)
        got = K.sgemm(a, torch.from_numpy(b).cuda(), mode=mode)
        torch.cuda.synchronize()
        assert K.kernel_status() == 0
        ref = O.dgemm_tile(a.cpu().numpy(), b, 0, 0, 128, 128)
        assert O.rel_fro(got[:128, :128].cpu().numpy(), ref) <= 1e-5

        # abort opens every gate of the chain: the next step's gated GEMM runs at once
        zg.api.check(lib.zg_bchain_abort(chain, 2))
        t0 = time.time()
        zg.api.check(lib.zg_bchain_gemm(chain, 2, 1, m, 1.0, pa.buf.data_ptr(), c.data_ptr(), n,
                                        None, 0, s))
        torch.cuda.synchronize()
        assert time.time() - t0 < 1.0
        assert K.kernel_status() == 0
    finally:
        lib.zg_bchain_destroy(chain)
