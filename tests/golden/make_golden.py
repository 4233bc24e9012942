"""Generates tests/golden/kats.npz: the known-answer vectors of ZenGPU's own
tests for the compute hot path, with expected outputs computed here by
independent means (exact Python integers / float64 / numpy float32 single
operations), never by the oracle or the CUDA library.

Sources (paths relative to the ZenGPU repository):
  vec_add_1024      zengpu-conformance/src/lib.rs:320-343      a=i, b=100*i
  vec_add_8         zengpu-cpu/src/lib.rs:572-575             same pattern, N=8
  add_quarter_1024  zengpu-cuda/src/lib.rs:1537-1538          a=0.25*i, b=1000-0.5*i
  add_relu_256      zengpu-conformance/tests/devarray_elementwise.rs:74-78
  double_64         zengpu-cuda/src/lib.rs:1794-1848          values=i-31, out=2*values
  chain_256         zengpu-cuda/src/lib.rs:1862-1866          2*(a+b), a=i, b=10*i
  gemm_17x33x9      zengpu-conformance/tests/devarray_matmul.rs:72-87
  op_graph_8x4x6    examples/op_graph_lower.rs:97-102,126-141
  tiled_31x29x23    zengpu-zsl/src/lib.rs:654-676 (max_err < 1e-3)
  heavy_64x48x40    examples/heavy_compute.rs:98-103,162-173 (rel 1%)
plus the seeded generator's first outputs (splitmix64, uniform[-1,1)) and
the pinned ReLU edge cases.

Run: python tests/golden/make_golden.py   (rewrites kats.npz)
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "kats.npz"
MASK = (1 << 64) - 1


def splitmix64_at(seed: int, i: int) -> int:
    z = (seed + (i + 1) * 0x9E3779B97F4A7C15) & MASK
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK
    return z ^ (z >> 31)


def f32(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32)


def main() -> None:
    kat: dict[str, np.ndarray] = {}

    i = np.arange(1024)
    kat["vec_add_1024_a"] = f32(i)
    kat["vec_add_1024_b"] = f32(100 * i)
    kat["vec_add_1024_out"] = f32(101 * i)  # exact integers < 2^24

    i8 = np.arange(8)
    kat["vec_add_8_a"] = f32(i8)
    kat["vec_add_8_b"] = f32(100 * i8)
    kat["vec_add_8_out"] = f32(101 * i8)

    kat["add_quarter_1024_a"] = f32(0.25 * i)
    kat["add_quarter_1024_b"] = f32(1000.0 - 0.5 * i)
    kat["add_quarter_1024_out"] = f32(1000.0 - 0.25 * i)  # every value exact in f32

    i256 = np.arange(256)
    a = i256 - 128
    b = 100 - i256
    kat["add_relu_256_a"] = f32(a)
    kat["add_relu_256_b"] = f32(b)
    kat["add_relu_256_sum"] = f32(a + b)
    kat["add_relu_256_relu"] = f32(np.maximum(a + b, 0))

    i64 = np.arange(64)
    kat["double_64_in"] = f32(i64 - 31)
    kat["double_64_out"] = f32(2 * (i64 - 31))

    kat["chain_256_a"] = f32(i256)
    kat["chain_256_b"] = f32(10 * i256)
    kat["chain_256_out"] = f32(2 * (11 * i256))

    # GEMM 17x33x9 with small integers: exact in f32, TF32 and 3xTF32.
    M, K, N = 17, 33, 9
    A = [(t % 7) - 3 for t in range(M * K)]
    B = [(t % 5) - 2 for t in range(K * N)]
    Cm = [sum(A[r * K + q] * B[q * N + c] for q in range(K)) for r in range(M) for c in range(N)]
    kat["gemm_17x33x9_a"] = f32(A).reshape(M, K)
    kat["gemm_17x33x9_b"] = f32(B).reshape(K, N)
    kat["gemm_17x33x9_c"] = f32(Cm).reshape(M, N)

    # op_graph_lower: relu(A @ B + C), 8x4 @ 4x6 + 8x6.
    M, K, N = 8, 4, 6
    A = [(t % 5) - 2 for t in range(M * K)]
    B = [(t % 3) - 1 for t in range(K * N)]
    Cc = [(t % 7) - 3 for t in range(M * N)]
    Y = [max(sum(A[r * K + q] * B[q * N + c] for q in range(K)) + Cc[r * N + c], 0)
         for r in range(M) for c in range(N)]
    kat["op_graph_8x4x6_a"] = f32(A).reshape(M, K)
    kat["op_graph_8x4x6_b"] = f32(B).reshape(K, N)
    kat["op_graph_8x4x6_c"] = f32(Cc).reshape(M, N)
    kat["op_graph_8x4x6_y"] = f32(Y).reshape(M, N)

    # Tiled GEMM 31x29x23: a exact (multiples of 1/32), b rounded to f32.
    M, N, K = 31, 29, 23
    ta = (f32((np.arange(M * K) % 17) - 8) * np.float32(0.03125)).reshape(M, K)
    tb = (f32((np.arange(K * N) % 13) - 6) * np.float32(0.025)).reshape(K, N)
    kat["tiled_31x29x23_a"] = ta
    kat["tiled_31x29x23_b"] = tb
    kat["tiled_31x29x23_c64"] = ta.astype(np.float64) @ tb.astype(np.float64)

    # heavy_compute patterns, f32 arithmetic one rounding per operation.
    M, K, N = 64, 40, 48
    ha = (f32(((np.arange(M * K) * 17 + 3) % 31)) * np.float32(0.125) - np.float32(2.0)).reshape(M, K)
    hb = (f32(((np.arange(K * N) * 13 + 7) % 29)) * np.float32(0.1) - np.float32(1.4)).reshape(K, N)
    kat["heavy_64x48x40_a"] = ha.astype(np.float32)
    kat["heavy_64x48x40_b"] = hb.astype(np.float32)
    kat["heavy_64x48x40_c64"] = ha.astype(np.float64) @ hb.astype(np.float64)

    # Seeded generator: first outputs, computed with Python integers.
    sm = [[splitmix64_at(seed, t) for t in range(16)] for seed in range(5)]
    kat["splitmix64_seed0to4_first16"] = np.array(sm, dtype=np.uint64)
    uni = [[float((v >> 40) * 2.0 ** -23 - 1.0) for v in row] for row in sm]
    kat["uniform_seed0to4_first16"] = f32(uni)

    # ReLU edge cases: NaN -> +0, -0 -> +0, -inf -> +0, +inf stays, subnormals.
    edge = np.array([-0.0, 0.0, np.nan, -np.nan, np.inf, -np.inf, 1e-45, -1e-45,
                     1.17549435e-38, -1.0, 1.0, 3.4028235e38], dtype=np.float32)
    exp = np.where(edge > 0, edge, np.float32(0.0)).astype(np.float32)
    kat["relu_edge_in"] = edge
    kat["relu_edge_out"] = exp

    np.savez_compressed(OUT, **kat)
    print(f"wrote {OUT} ({len(kat)} arrays)")


if __name__ == "__main__":
    main()
