/*
 * zg_oracle.h - CPU oracle for the ZenGPU compute hot path (TEST INFRASTRUCTURE).
 *
 * This library is the checker, not the product.  Only the test suite, the
 * smoke check and the CPU-baseline leg of bench.py load it.  The product path
 * (libzengpu_b200.so) never links, loads or calls anything here.
 *
 * It restates, in plain C, the arithmetic of ZenGPU's deterministic CPU
 * backend for the three ops on the path:
 *   add   out[i] = a[i] + b[i]                 zengpu-conformance/tests/devarray_elementwise.rs:30-43
 *   relu  out[i] = max(a[i], 0)                zengpu-conformance/tests/devarray_elementwise.rs:44-56
 *   sgemm c[r,c] = alpha * sum_k a[r,k]*b[k,c] zengpu-conformance/tests/devarray_matmul.rs:22-53
 * The reference backend itself is Rust (zengpu-cpu) and cannot be built here
 * (no cargo/rustc), so the restatement is pinned on the reference's own
 * known-answer vectors instead (tests/golden/).
 *
 * Build with -O2 -ffp-contract=off and without -ffast-math: Rust never fuses
 * a*b+c into an FMA, and the oracle must round every product and every sum
 * exactly as the Rust loop does.
 */
#ifndef ZG_ORACLE_H
#define ZG_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- seeded synthetic inputs (shared with the device generator) ---------- */
/* splitmix64 output number i (0-based) of the stream that starts at `seed`. */
uint64_t zgo_splitmix64_at(uint64_t seed, uint64_t i);
/* x[i] = uniform[-1,1) with 24 random bits: (u24 * 2^-23) - 1, exact in f32. */
void zgo_fill_uniform(float *x, size_t n, uint64_t seed);
/* x[i] = lo + (hi-lo) * u, u = u24 * 2^-24 in [0,1), computed in f32. */
void zgo_fill_uniform_range(float *x, size_t n, uint64_t seed, float lo, float hi);
/* x[i] ~ normal(0,1): Box-Muller in f64 on pairs (2j, 2j+1), rounded to f32. */
void zgo_fill_normal(float *x, size_t n, uint64_t seed);

/* ---- elementwise (CPU backend semantics) --------------------------------- */
void zgo_add_f32(const float *a, const float *b, float *out, size_t n);
/* relu(v) = v > 0 ? v : +0.0  (NaN -> +0.0, -0.0 -> +0.0) */
void zgo_relu_f32(const float *in, float *out, size_t n);
void zgo_add_f32_mt(const float *a, const float *b, float *out, size_t n, int threads);
void zgo_relu_f32_mt(const float *in, float *out, size_t n, int threads);

/* ---- Level-1 (zengpu-blas/src/level1.rs:11-33) --------------------------- */
void zgo_saxpy_f32(float alpha, const float *x, float *y, size_t n); /* y += alpha*x */
void zgo_sscal_f32(float alpha, float *x, size_t n);                 /* x *= alpha   */

/* ---- GEMM ---------------------------------------------------------------- */
/* Faithful loop order: row, col, k; sum starts at 0.0f; unfused mul then add;
 * c = alpha * sum.  Rows [row0,row1) only; threads > 1 splits rows. */
void zgo_sgemm_ref(int m, int n, int k, float alpha, const float *a,
                   const float *b, float *c, int row0, int row1, int threads);
/* Same per-element arithmetic (same products, same k order, same roundings),
 * loop order row, k, col for cache locality: bit-identical to zgo_sgemm_ref. */
void zgo_sgemm_fast(int m, int n, int k, float alpha, const float *a,
                    const float *b, float *c, int threads);
/* The reference's unfused op_graph_lower chain with a row-broadcast bias:
 * y = relu( fl(alpha*sum) + bias[col] ), each step rounded to f32. */
void zgo_sgemm_bias_relu(int m, int n, int k, float alpha, const float *a,
                         const float *b, const float *bias, float *y, int threads);
/* f64 reference for a tile: out[(r-r0)*w + (c-c0)] = alpha * sum_k a*b in f64. */
void zgo_dgemm_tile(int m, int n, int k, double alpha, const float *a,
                    const float *b, int r0, int c0, int h, int w, double *out);

/* ---- error metrics -------------------------------------------------------- */
/* ||x - y||_F / ||y||_F in f64 (y is the reference). */
double zgo_rel_fro_f32(const float *x, const float *y, size_t n);
double zgo_rel_fro_f32_f64(const float *x, const double *y, size_t n);

#ifdef __cplusplus
}
#endif
#endif
