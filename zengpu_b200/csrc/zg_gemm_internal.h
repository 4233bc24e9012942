// zg_gemm_internal.h - host-side GEMM building blocks shared inside the
// library (not exported): the operand pre-pass for A and for B, and the GEMM
// kernel launch on prepared operands with a pitched C.  zg_sgemm_* and the
// runtime's pipelined host-buffer GEMM are built from these.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace zg {

// What the GEMM kernels read.  SIMT: a_hi = A (M x K, pitch lda), b_hi = B
// (K x N row-major, pitch ldb).  Tensor-core modes: A or its tf32 planes
// (M x K, K-major) and the K-major planes of B^T (N x K), pitches in floats.
struct GemmOperands {
    int mode;
    const float* a_hi;
    const float* a_lo;
    int64_t lda;
    const float* b_hi;
    const float* b_lo;
    int64_t ldb;
};

// True when the mode reads A (resp. B) through pre-pass planes.
bool gemm_a_needs_planes(int mode, int K);
bool gemm_b_needs_planes(int mode);
// Pitch (floats) of the pre-pass planes for inner dimension K.
int64_t gemm_plane_pitch(int K);

// Pre-pass of A (M x K, pitch lda) into planes of pitch ldp; `lo` only for TF32X3.
int gemm_prep_a(int mode, int M, int K, const float* A, int64_t lda, float* hi, float* lo,
                int64_t ldp, cudaStream_t s);
// Pre-pass of B (K x N, pitch ldb) into K-major B^T planes (N x K, pitch ldp).
int gemm_prep_b(int mode, int K, int N, const float* B, int64_t ldb, float* hi, float* lo,
                int64_t ldp, cudaStream_t s);
// C[M x N, pitch ldc] = epilogue(alpha * A @ B) on prepared operands.
int gemm_run(const GemmOperands& op, int M, int N, int K, float alpha, float* C, int64_t ldc,
             const float* bias, int relu, cudaStream_t s);

}  // namespace zg
