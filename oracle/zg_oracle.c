/*
 * zg_oracle.c - CPU oracle for the ZenGPU compute hot path (TEST INFRASTRUCTURE).
 *
 * Checker only: loaded by tests/, the smoke check and the CPU-baseline leg of
 * bench.py.  The product library never calls into it.  Each kernel cites the
 * reference lines whose arithmetic it restates; see zg_oracle.h.
 *
 * Compile: gcc -O2 -ffp-contract=off -fno-fast-math -fopenmp -shared -fPIC
 * (oracle/Makefile).  No FMA contraction anywhere: every product and every
 * partial sum is rounded to f32 separately, as in the Rust CPU backend.
 */
#include "zg_oracle.h"

#include <math.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ZGO_GOLDEN 0x9E3779B97F4A7C15ULL

/* splitmix64 (Steele, Lea, Flood 2014): state advances by the golden gamma,
 * output is the variant-13 finaliser of the new state.  Output i is a pure
 * function of (seed, i), so the device generator can produce it in parallel. */
uint64_t zgo_splitmix64_at(uint64_t seed, uint64_t i) {
    uint64_t z = seed + (i + 1) * ZGO_GOLDEN;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

void zgo_fill_uniform(float *x, size_t n, uint64_t seed) {
    for (size_t i = 0; i < n; ++i) {
        uint32_t u = (uint32_t)(zgo_splitmix64_at(seed, i) >> 40); /* 24 bits */
        x[i] = (float)u * 0x1p-23f - 1.0f; /* exact: spacing 2^-23 on [-1,1) */
    }
}

void zgo_fill_uniform_range(float *x, size_t n, uint64_t seed, float lo, float hi) {
    const float span = hi - lo;
    for (size_t i = 0; i < n; ++i) {
        uint32_t u24 = (uint32_t)(zgo_splitmix64_at(seed, i) >> 40);
        float u = (float)u24 * 0x1p-24f;
        float t = span * u; /* rounded product, then rounded sum: no FMA */
        x[i] = lo + t;
    }
}

void zgo_fill_normal(float *x, size_t n, uint64_t seed) {
    const double two_pi = 6.283185307179586476925286766559;
    for (size_t j = 0; 2 * j < n; ++j) {
        uint64_t s1 = zgo_splitmix64_at(seed, 2 * j);
        uint64_t s2 = zgo_splitmix64_at(seed, 2 * j + 1);
        double u1 = (double)((s1 >> 11) + 1) * 0x1p-53; /* (0,1] */
        double u2 = (double)(s2 >> 11) * 0x1p-53;       /* [0,1) */
        double r = sqrt(-2.0 * log(u1));
        double th = two_pi * u2;
        x[2 * j] = (float)(r * cos(th));
        if (2 * j + 1 < n) x[2 * j + 1] = (float)(r * sin(th));
    }
}

/* add: zengpu-conformance/tests/devarray_elementwise.rs:30-43 */
void zgo_add_f32(const float *a, const float *b, float *out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}

/* relu: zengpu-conformance/tests/devarray_elementwise.rs:44-56 (`v.max(0.0)`).
 * Rust's f32::max is IEEE maxNum: a NaN input yields the other operand, 0.0.
 * maxNum leaves the sign of a zero result open; this build pins it to +0.0
 * (relu never returns -0.0), and the device kernel uses the same select. */
static inline float zgo_relu1(float v) { return v > 0.0f ? v : 0.0f; }

void zgo_relu_f32(const float *in, float *out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = zgo_relu1(in[i]);
}

void zgo_add_f32_mt(const float *a, const float *b, float *out, size_t n, int threads) {
    long long nn = (long long)n;
#pragma omp parallel for num_threads(threads) schedule(static)
    for (long long i = 0; i < nn; ++i) out[i] = a[i] + b[i];
}

void zgo_relu_f32_mt(const float *in, float *out, size_t n, int threads) {
    long long nn = (long long)n;
#pragma omp parallel for num_threads(threads) schedule(static)
    for (long long i = 0; i < nn; ++i) out[i] = zgo_relu1(in[i]);
}

/* saxpy / sscal: zengpu-blas/src/level1.rs:11-33 */
void zgo_saxpy_f32(float alpha, const float *x, float *y, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        float t = alpha * x[i];
        y[i] = y[i] + t;
    }
}

void zgo_sscal_f32(float alpha, float *x, size_t n) {
    for (size_t i = 0; i < n; ++i) x[i] = x[i] * alpha;
}

/* GEMM: zengpu-conformance/tests/devarray_matmul.rs:38-49 and the shader it
 * mirrors, zengpu-blas/src/level3.rs:13-27.  for row, for col { sum = 0;
 * for i in 0..k { sum += a[row*k+i] * b[i*n+col] }; c = alpha * sum }. */
void zgo_sgemm_ref(int m, int n, int k, float alpha, const float *a,
                   const float *b, float *c, int row0, int row1, int threads) {
    (void)m;
#pragma omp parallel for num_threads(threads) schedule(dynamic, 1)
    for (int row = row0; row < row1; ++row) {
        for (int col = 0; col < n; ++col) {
            float sum = 0.0f;
            for (int i = 0; i < k; ++i) {
                float p = a[(size_t)row * k + i] * b[(size_t)i * n + col];
                sum = sum + p;
            }
            c[(size_t)row * n + col] = alpha * sum;
        }
    }
}

/* Same arithmetic as zgo_sgemm_ref element by element (each c[row,col] still
 * accumulates its products in increasing k from 0.0f, unfused); only the loop
 * nest is reordered so the inner loop walks B and the row accumulator
 * contiguously.  Bit-identical by construction; the tests also check it. */
void zgo_sgemm_fast(int m, int n, int k, float alpha, const float *a,
                    const float *b, float *c, int threads) {
#pragma omp parallel for num_threads(threads) schedule(dynamic, 1)
    for (int row = 0; row < m; ++row) {
        float *acc = c + (size_t)row * n;
        for (int col = 0; col < n; ++col) acc[col] = 0.0f;
        for (int i = 0; i < k; ++i) {
            const float av = a[(size_t)row * k + i];
            const float *brow = b + (size_t)i * n;
            for (int col = 0; col < n; ++col) {
                float p = av * brow[col];
                acc[col] = acc[col] + p;
            }
        }
        for (int col = 0; col < n; ++col) acc[col] = alpha * acc[col];
    }
}

/* op_graph_lower chain Matmul -> Add -> Relu (examples/op_graph_lower.rs:39-68,
 * host expectation :126-141) with the added operand a bias row broadcast over
 * the M rows: every stage rounds to f32 before the next. */
void zgo_sgemm_bias_relu(int m, int n, int k, float alpha, const float *a,
                         const float *b, const float *bias, float *y, int threads) {
    zgo_sgemm_fast(m, n, k, alpha, a, b, y, threads);
    long long mm = m;
#pragma omp parallel for num_threads(threads) schedule(static)
    for (long long row = 0; row < mm; ++row) {
        float *yr = y + (size_t)row * n;
        for (int col = 0; col < n; ++col) yr[col] = zgo_relu1(yr[col] + bias[col]);
    }
}

/* f64 reference used for sampled tiles of large GEMMs (examples/heavy_compute.rs:162-173
 * checks sampled elements the same way, at lower precision). */
void zgo_dgemm_tile(int m, int n, int k, double alpha, const float *a,
                    const float *b, int r0, int c0, int h, int w, double *out) {
    (void)m;
    for (int r = 0; r < h; ++r) {
        double *o = out + (size_t)r * w;
        for (int j = 0; j < w; ++j) o[j] = 0.0;
        for (int i = 0; i < k; ++i) {
            double av = (double)a[(size_t)(r0 + r) * k + i];
            const float *brow = b + (size_t)i * n + c0;
            for (int j = 0; j < w; ++j) o[j] += av * (double)brow[j];
        }
        for (int j = 0; j < w; ++j) o[j] *= alpha;
    }
}

double zgo_rel_fro_f32(const float *x, const float *y, size_t n) {
    double num = 0.0, den = 0.0;
    for (size_t i = 0; i < n; ++i) {
        double d = (double)x[i] - (double)y[i];
        num += d * d;
        den += (double)y[i] * (double)y[i];
    }
    return den > 0.0 ? sqrt(num / den) : sqrt(num);
}

double zgo_rel_fro_f32_f64(const float *x, const double *y, size_t n) {
    double num = 0.0, den = 0.0;
    for (size_t i = 0; i < n; ++i) {
        double d = (double)x[i] - y[i];
        num += d * d;
        den += y[i] * y[i];
    }
    return den > 0.0 ? sqrt(num / den) : sqrt(num);
}
