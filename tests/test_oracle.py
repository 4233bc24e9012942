"""The CPU oracle pinned against ZenGPU's own known-answer vectors
(tests/golden/kats.npz, generated independently by make_golden.py)."""
from __future__ import annotations

import numpy as np
import pytest

import _oracle as O


def bits(x) -> np.ndarray:
    return np.asarray(x, np.float32).view(np.uint32)


@pytest.mark.parametrize("name", ["vec_add_1024", "vec_add_8", "add_quarter_1024"])
def test_add_kats_bit_exact(kats, name):
    out = O.add(kats[f"{name}_a"], kats[f"{name}_b"])
    np.testing.assert_array_equal(bits(out), bits(kats[f"{name}_out"]))


def test_add_relu_256(kats):
    s = O.add(kats["add_relu_256_a"], kats["add_relu_256_b"])
    np.testing.assert_array_equal(bits(s), bits(kats["add_relu_256_sum"]))
    np.testing.assert_array_equal(bits(O.relu(s)), bits(kats["add_relu_256_relu"]))


def test_double_and_chain(kats):
    x = kats["double_64_in"]
    np.testing.assert_array_equal(bits(O.add(x, x)), bits(kats["double_64_out"]))
    s = O.add(kats["chain_256_a"], kats["chain_256_b"])
    np.testing.assert_array_equal(bits(O.add(s, s)), bits(kats["chain_256_out"]))


def test_relu_edge_cases(kats):
    out = O.relu(kats["relu_edge_in"])
    np.testing.assert_array_equal(bits(out), bits(kats["relu_edge_out"]))
    assert not np.signbit(out).any()


def test_gemm_17x33x9_exact(kats):
    c = O.sgemm_ref(kats["gemm_17x33x9_a"], kats["gemm_17x33x9_b"])
    np.testing.assert_array_equal(bits(c), bits(kats["gemm_17x33x9_c"]))


def test_op_graph_chain(kats):
    a, b, c = kats["op_graph_8x4x6_a"], kats["op_graph_8x4x6_b"], kats["op_graph_8x4x6_c"]
    y = O.relu(O.add(O.sgemm_ref(a, b), c))
    np.testing.assert_array_equal(bits(y), bits(kats["op_graph_8x4x6_y"]))


def test_tiled_31x29x23(kats):
    c = O.sgemm_ref(kats["tiled_31x29x23_a"], kats["tiled_31x29x23_b"])
    assert np.max(np.abs(c - kats["tiled_31x29x23_c64"])) < 1e-3


def test_heavy_pattern(kats):
    c = O.sgemm_ref(kats["heavy_64x48x40_a"], kats["heavy_64x48x40_b"])
    ref = kats["heavy_64x48x40_c64"]
    m, n = ref.shape
    for r, q in [(0, 0), (m // 3, n // 3), (m // 2, n // 2), (m - 1, n - 1)]:
        assert abs(c[r, q] - ref[r, q]) / max(abs(ref[r, q]), 1.0) <= 0.01
    assert O.rel_fro(c, ref) < 1e-5


def test_splitmix_and_uniform(kats):
    sm = kats["splitmix64_seed0to4_first16"]
    for seed in range(5):
        got = [O.lib().zgo_splitmix64_at(seed, t) for t in range(16)]
        assert got == [int(v) for v in sm[seed]]
        np.testing.assert_array_equal(bits(O.uniform(16, seed)),
                                      bits(kats["uniform_seed0to4_first16"][seed]))


def test_uniform_range_and_normal_statistics():
    u = O.uniform(1 << 16, 7)
    assert u.min() >= -1.0 and u.max() < 1.0 and abs(u.mean()) < 0.02
    w = O.uniform(1 << 16, 3, -0.5, 0.5)
    assert w.min() >= -0.5 and w.max() < 0.5
    z = O.normal(1 << 16, 1)
    assert abs(z.mean()) < 0.02 and abs(z.std() - 1.0) < 0.02
    z_odd = O.normal(7, 1)
    np.testing.assert_array_equal(bits(z_odd), bits(z[:7]))


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (7, 5, 3), (33, 17, 65), (64, 64, 64), (5, 130, 9)])
def test_fast_loop_order_is_bit_identical(m, n, k):
    a = O.uniform(m * k, 11).reshape(m, k)
    b = O.uniform(k * n, 12).reshape(k, n)
    for alpha in (1.0, -0.75):
        np.testing.assert_array_equal(bits(O.sgemm_ref(a, b, alpha)),
                                      bits(O.sgemm(a, b, alpha, threads=4)))


def test_sgemm_rows_subset_and_threads():
    a = O.uniform(40 * 24, 1).reshape(40, 24)
    b = O.uniform(24 * 16, 2).reshape(24, 16)
    full = O.sgemm_ref(a, b)
    part = O.sgemm_ref(a, b, rows=(8, 20), threads=3)
    np.testing.assert_array_equal(bits(part[8:20]), bits(full[8:20]))
    assert not part[:8].any() and not part[20:].any()


def test_k_zero_gives_alpha_times_zero():
    a = np.zeros((3, 0), np.float32)
    b = np.zeros((0, 4), np.float32)
    np.testing.assert_array_equal(bits(O.sgemm_ref(a, b, 1.0)), bits(np.zeros((3, 4), np.float32)))
    neg = O.sgemm_ref(a, b, -1.0)  # -1 * 0.0 = -0.0, as the Rust loop computes
    assert np.signbit(neg).all()


def test_bias_relu_matches_three_step_chain():
    m, n, k = 13, 21, 17
    a = O.uniform(m * k, 5).reshape(m, k)
    b = O.uniform(k * n, 6).reshape(k, n)
    bias = O.uniform(n, 7, -0.1, 0.1)
    y = O.sgemm_bias_relu(a, b, bias, alpha=0.5)
    c = O.sgemm_ref(a, b, 0.5)
    chain = O.relu(O.add(c, np.broadcast_to(bias, (m, n))))
    np.testing.assert_array_equal(bits(y), bits(chain))


def test_dgemm_tile_matches_numpy():
    a = O.uniform(50 * 30, 1).reshape(50, 30)
    b = O.uniform(30 * 40, 2).reshape(30, 40)
    t = O.dgemm_tile(a, b, 10, 5, 20, 30, alpha=2.0)
    ref = 2.0 * (a.astype(np.float64) @ b.astype(np.float64))[10:30, 5:35]
    np.testing.assert_allclose(t, ref, rtol=1e-12, atol=1e-12)


def test_level1():
    x = O.uniform(1000, 1)
    y = O.uniform(1000, 2)
    exp = (y + (np.float32(0.5) * x).astype(np.float32)).astype(np.float32)
    np.testing.assert_array_equal(bits(O.saxpy(0.5, x, y)), bits(exp))
    np.testing.assert_array_equal(bits(O.sscal(3.0, x)), bits((x * np.float32(3.0)).astype(np.float32)))


def test_multithreaded_elementwise_matches():
    a = O.normal(100003, 1)
    b = O.normal(100003, 2)
    np.testing.assert_array_equal(bits(O.add(a, b, threads=4)), bits(O.add(a, b)))
    np.testing.assert_array_equal(bits(O.relu(a, threads=4)), bits(O.relu(a)))
