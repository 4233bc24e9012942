"""The error budget of the split GEMM modes, emulated on the CPU in float64.

Each mode replaces an f32 product by a few tensor-core products of rounded
parts; the GPU tests measure the whole kernel against the 1e-5 bar.  This
checks the part of the error that the splitting alone causes, with exact
accumulation, on the bench's input distribution (uniform[-1, 1), K = 8192):
BF16X3 (x = bf16 hi + bf16 lo, three products) stays near 4e-6 and the
tf32-based splits are an order of magnitude below, so the modes keep their
margin under the bar once the f32 accumulation (about 2.5e-6) is added."""
from __future__ import annotations

import numpy as np
import pytest

import _oracle as O


def _round_bits(x: np.ndarray, drop: int) -> np.ndarray:
    """Rounds f32 values to nearest-even, keeping 23 - drop mantissa bits."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    half = (1 << (drop - 1)) - 1
    r = ((u + half + ((u >> drop) & 1)) >> drop) << drop
    return r.astype(np.uint32).view(np.float32)


def bf16(x):
    return _round_bits(x, 16)


def tf32(x):
    return _round_bits(x, 13)


@pytest.fixture(scope="module")
def operands():
    m, n, k = 64, 64, 8192
    a = O.uniform(m * k, 21).reshape(m, k)
    b = O.uniform(k * n, 22).reshape(k, n)
    return a, b, a.astype(np.float64) @ b.astype(np.float64)


def _err(parts, ref):
    c = sum(x.astype(np.float64) @ y.astype(np.float64) for x, y in parts)
    return float(np.linalg.norm(c - ref) / np.linalg.norm(ref))


def test_bf16_split_is_exact_in_two_parts_to_16_bits():
    x = O.uniform(1 << 16, 23)
    hi = bf16(x)
    lo = bf16(x - hi)
    # x - hi is exact in f32, and hi + lo keeps 16 of x's 24 mantissa bits
    assert np.all(np.abs((x.astype(np.float64) - hi - lo)) <= np.abs(x) * 2.0 ** -16)


def test_bf16x3_split_error(operands):
    a, b, ref = operands
    ah, bh = bf16(a), bf16(b)
    al, bl = bf16(a - ah), bf16(b - bh)
    err = _err([(ah, bh), (ah, bl), (al, bh)], ref)
    assert 1e-6 < err < 6e-6, err


def test_tf32_splits_error(operands):
    a, b, ref = operands
    ah, bh = tf32(a), tf32(b)
    # TF32X3: tf32 lo parts; TF32_BF16X2: the two corrections from bf16 operands
    x3 = _err([(ah, bh), (ah, tf32(b - bh)), (tf32(a - ah), bh)], ref)
    bx2 = _err([(ah, bh), (bf16(ah), bf16(b - bh)), (bf16(a - ah), bf16(bh))], ref)
    assert x3 < 1e-6, x3
    assert bx2 < 1e-6, bx2


def test_plain_tf32_error_is_far_above_the_split_modes(operands):
    a, b, ref = operands
    err = _err([(tf32(a), tf32(b))], ref)
    assert 1e-4 < err < 5e-3, err
