// zg_gemm_internal.h - host-side GEMM building blocks shared inside the
// library (not exported): the packed operand layout the tensor-core kernels
// read, the pre-pass that writes it, and the GEMM launch on prepared operands
// with a pitched C.  zg_sgemm_*, the packed-operand API and the runtime's
// pipelined host-buffer GEMM are built from these.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace zg {

// One operand as a kernel reads it: `rows` rows (A: m; B: n, i.e. B
// transposed so k is innermost), pitch `ld` in 4-byte units.
//   SIMT          the caller's f32 operand (B untransposed: k rows of n)
//   TF32          f32 (A: the caller's when k % 4 == 0), k innermost
//   TF32X3        per 16-k block one 128-byte row: 16 tf32 hi, 16 tf32 lo
//   TF32_BF16X2   per 16-k block one 128-byte row: 16 tf32 hi (64 B),
//                 16 bf16(hi) (32 B), 16 bf16(x - hi) (32 B)
//   BF16X3        per 32-k block one 128-byte row: 32 bf16(x) (64 B), then
//                 32 bf16(x - bf16(x)) (64 B); 4 bytes per element, the size
//                 of the f32 input
// The interleaved rows let one 128-byte-swizzled TMA box carry every term a
// stage needs; k beyond K inside the last block is zero.
struct OperandView {
    void* p = nullptr;
    int64_t ld = 0;
};

struct GemmOperands {
    int mode;
    OperandView a;
    OperandView b;
};

// True when the mode reads A (resp. B) through a pre-pass copy.
bool gemm_a_needs_planes(int mode, int K);
bool gemm_b_needs_planes(int mode);
// Bytes of the prepared form of one operand with `outer` rows and reduction
// K (256-byte aligned), and the view of such a buffer at `base`.
uint64_t gemm_planes_bytes(int mode, int outer, int K);
OperandView gemm_carve_planes(void* base, int mode, int outer, int K);
// The same view `rows` rows further down.
OperandView gemm_offset_rows(const OperandView& v, int64_t rows);
// A caller operand read directly.
OperandView gemm_raw_operand(const float* x, int64_t ld);

// Pre-pass of A (M x K, pitch lda) into `out` (carved for mode, M, K).
int gemm_prep_a(int mode, int M, int K, const float* A, int64_t lda, const OperandView& out,
                cudaStream_t s);
// Pre-pass of B (K x N, pitch ldb) into B^T form (carved for mode, N, K).
int gemm_prep_b(int mode, int K, int N, const float* B, int64_t ldb, const OperandView& out,
                cudaStream_t s);
// gemm_prep_b, in one launch that raises flags[c] = epoch (system-scope
// release) as soon as chunk c (columns [c * chunk_cols, ...) of B, rows of
// B^T) is fully written; chunks finish in order.  counters: one u32 per
// chunk, device memory, reset by the call.
int gemm_prep_b_signal(int mode, int K, int N, const float* B, int64_t ldb,
                       const OperandView& out, int chunk_cols, uint32_t* counters,
                       uint32_t* flags, uint32_t epoch, cudaStream_t s);

// Arrival gate of a GEMM whose B^T rows are still landing in its buffer
// (copied from another GPU while the GEMM runs): rows [c * rows, (c + 1) *
// rows) of B^T may be read once flags[c] has reached `epoch` (wrap-aware:
// (int32_t)(flags[c] - epoch) >= 0).  `rows` is a multiple of 256, so every
// output tile's B rows sit in one chunk.  The tensor-core kernels check the
// flag once per tile before loading its B rows.
struct GemmGate {
    const uint32_t* flags = nullptr;
    uint32_t epoch = 0;
    int rows = 0;
};

// C[M x N, pitch ldc] = epilogue(alpha * A @ B) on prepared operands; `gate`
// (tensor-core modes only) holds back B loads until their chunk has arrived.
int gemm_run(const GemmOperands& op, int M, int N, int K, float alpha, float* C, int64_t ldc,
             const float* bias, int relu, cudaStream_t s, const GemmGate* gate = nullptr);

}  // namespace zg
