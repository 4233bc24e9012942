/*
 * zengpu_b200.h - C ABI of the B200 (sm_100a) compute backend for ZenGPU's
 * hot path: DeviceArray add / ReLU, the f32 GEMM behind zengpu-blas, and a
 * fused GEMM -> bias -> ReLU epilogue.
 *
 * Plain C: pointers, sizes and integer status codes only, so the Rust crates
 * (zengpu-cuda, zengpu-compute, zengpu-blas) bind it with `extern "C"`.
 * Reference paths below are relative to the ZenGPU repository.
 *
 * Three layers, all exported from libzengpu_b200.so:
 *   1. Device runtime  - the GpuDevice compute subset (buffers, shaders,
 *      pipelines, dispatch, submissions) that zengpu-cuda's CudaDevice
 *      implements today (zengpu-cuda/src/lib.rs:472-1164).
 *   2. Array ops       - DeviceArray / BufferPool / ElementwiseKernels /
 *      GemmKernel / Level1Kernels with the reference's argument meaning and
 *      error behaviour (zengpu-compute/src/*.rs, zengpu-blas/src/*.rs).
 *   3. Stream kernels  - the same kernels on raw device pointers, ordered on a
 *      caller stream; used by the multi-GPU sharding and by callers that own
 *      their memory (torch tensors, cudaMalloc'd buffers).
 *
 * Every fallible call returns zg_status; ZG_OK is 0.  The message of the
 * last failure on the calling thread is available from zg_last_error().
 */
#ifndef ZENGPU_B200_H
#define ZENGPU_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Every declaration below is exported even when the library is built with
 * -fvisibility=hidden. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define ZG_ABI_VERSION 1

/* One code per GpuError / UsageError variant (zengpu-hal/src/error.rs:15-58);
 * CUresult mapping follows zengpu-cuda/src/error.rs:16-36. */
typedef enum zg_status {
    ZG_OK = 0,
    ZG_ERR_DEVICE_LOST = 1,          /* GpuError::DeviceLost                    */
    ZG_ERR_TIMEOUT = 2,              /* GpuError::Timeout (bounded host wait)   */
    ZG_ERR_OUT_OF_MEMORY = 3,        /* GpuError::OutOfMemory                   */
    ZG_ERR_UNSUPPORTED_FEATURES = 4, /* GpuError::UnsupportedFeatures           */
    ZG_ERR_UNSUPPORTED = 5,          /* GpuError::Unsupported                   */
    ZG_ERR_STALE_HANDLE = 6,         /* InvalidUsage(UsageError::StaleHandle)   */
    ZG_ERR_MISSING_USAGE = 7,        /* InvalidUsage(UsageError::MissingUsage)  */
    ZG_ERR_BINDING_MISMATCH = 8,     /* InvalidUsage(UsageError::BindingMismatch) */
    ZG_ERR_SHADER_COMPILE = 9,       /* GpuError::ShaderCompile                 */
    ZG_ERR_PIPELINE_CREATION = 10,   /* GpuError::PipelineCreation              */
    ZG_ERR_DISPATCH = 11,            /* GpuError::Dispatch (shape/dtype errors) */
    ZG_ERR_BACKEND = 12,             /* GpuError::Backend (any other driver error) */
    ZG_ERR_NO_DEVICE = 13,           /* cuInit / no CUDA device: callers skip   */
    ZG_ERR_KERNEL_WAIT = 14          /* a kernel's bounded on-device wait expired */
} zg_status;

/* Generational handle (zengpu-hal/src/handle.rs:15-19). */
typedef struct zg_handle {
    uint32_t index;
    uint32_t generation;
} zg_handle;

/* BufferUsage bits (zengpu-hal/src/types.rs:60-72). */
#define ZG_USAGE_STORAGE (1u << 0)
#define ZG_USAGE_UNIFORM (1u << 1)
#define ZG_USAGE_TRANSFER_SRC (1u << 5)
#define ZG_USAGE_TRANSFER_DST (1u << 6)
#define ZG_USAGE_READBACK (1u << 7)

/* MemoryUsage (zengpu-hal/src/types.rs:38-56). */
#define ZG_MEMORY_GPU_ONLY 0u
#define ZG_MEMORY_UPLOAD 1u
#define ZG_MEMORY_READBACK 2u

/* DType, in the order of zengpu-hal/src/types.rs:195-210. */
#define ZG_DTYPE_F32 0u
#define ZG_DTYPE_F16 1u
#define ZG_DTYPE_BF16 2u
#define ZG_DTYPE_F64 3u
#define ZG_DTYPE_I8 4u
#define ZG_DTYPE_I16 5u
#define ZG_DTYPE_I32 6u
#define ZG_DTYPE_I64 7u
#define ZG_DTYPE_U8 8u
#define ZG_DTYPE_U16 9u
#define ZG_DTYPE_U32 10u
#define ZG_DTYPE_U64 11u
#define ZG_DTYPE_BOOL 12u

/* GEMM arithmetic.  SIMT_FP32: exact-fp32 CUDA-core SGEMM (FMA, rel-Frobenius
 * <= 1e-5).  TF32X3: tcgen05 tensor cores, split-precision hi*hi + hi*lo +
 * lo*hi, three TF32 products (rel-Frobenius <= 1e-5).  TF32: one tcgen05 TF32
 * pass (<= 5e-3).  TF32_BF16X2: the same split with the two small correction
 * products in bf16 (twice the TF32 rate), 2/3 of TF32X3's tensor time
 * (rel-Frobenius <= 1e-5).  BF16X3: x = bf16 hi + bf16 lo for both operands,
 * hi*hi + hi*lo + lo*hi as three bf16 products, 1/2 of TF32X3's tensor time
 * and half its operand bytes (rel-Frobenius <= 1e-5). */
#define ZG_GEMM_SIMT_FP32 0
#define ZG_GEMM_TF32X3 1
#define ZG_GEMM_TF32 2
#define ZG_GEMM_TF32_BF16X2 3
#define ZG_GEMM_BF16X3 4

/* ======================================================================
 * 1. Device runtime
 * ====================================================================== */

typedef struct zg_device zg_device;
typedef struct zg_submission zg_submission;

/* Message of the last failed call on this thread ("" if none). */
const char *zg_last_error(void);

/* The fields of the last failure on this thread, so a binding can rebuild the
 * reference's error value exactly (zengpu-hal/src/error.rs:15-58):
 *   ZG_ERR_STALE_HANDLE     UsageError::StaleHandle { index, expected_gen, actual_gen }
 *   ZG_ERR_MISSING_USAGE    UsageError::MissingUsage { resource, needed }
 *                           (static strings, e.g. "buffer" / "READBACK")
 *   ZG_ERR_OUT_OF_MEMORY    GpuError::OutOfMemory(memory) (ZG_MEMORY_*)
 *   ZG_ERR_UNSUPPORTED_FEATURES  GpuError::UnsupportedFeatures(features)
 * Fields a status does not use are zero / "".  status is 0 before any failure. */
typedef struct zg_error_detail {
    int32_t status;
    uint32_t handle_index;
    uint32_t expected_gen;
    uint32_t actual_gen;
    uint32_t memory;
    uint32_t reserved;
    uint64_t features;
    const char *resource;
    const char *needed;
} zg_error_detail;
int zg_last_error_detail(zg_error_detail *out);
int zg_abi_version(void);

/* Number of CUDA devices; ZG_ERR_NO_DEVICE when the driver cannot init.
 * Replaces CudaInstance::new + enumerate (zengpu-cuda/src/lib.rs:107-162). */
int zg_device_count(int *count);
/* Open `ordinal`: primary context, one non-blocking stream.
 * Replaces CudaAdapter::open (zengpu-cuda/src/lib.rs:184-205). */
int zg_device_open(int ordinal, zg_device **out);
/* Waits for outstanding work, frees every buffer/module, releases the device. */
void zg_device_close(zg_device *dev);
/* GpuDevice::device_ordinal (zengpu-hal/src/device.rs:86-89). */
int zg_device_ordinal(const zg_device *dev);
/* The device's stream (a cudaStream_t), for interop with layer 3. */
void *zg_device_stream(zg_device *dev);
/* GpuDevice::can_peer (zengpu-hal/src/device.rs:91-94), as the HIP backend
 * implements it (zengpu-hip/src/lib.rs:613-631): 1 once `dev` can access
 * `peer_ordinal`'s memory (peer access is enabled on the first query and the
 * answer cached per peer), else 0; a device can always reach itself. */
int zg_device_can_peer(zg_device *dev, int peer_ordinal, int *out);

/* GpuDevice::create_buffer (zengpu-cuda/src/lib.rs:481-500). */
int zg_buffer_create(zg_device *dev, uint64_t size, uint32_t usage, uint32_t memory,
                     zg_handle *out);
/* GpuDevice::write_buffer (zengpu-cuda/src/lib.rs:502-527). */
int zg_buffer_write(zg_device *dev, zg_handle buf, uint64_t offset, const void *data,
                    uint64_t len);
/* GpuDevice::read_buffer_into (zengpu-cuda/src/lib.rs:560-615): needs READBACK. */
int zg_buffer_read(zg_device *dev, zg_handle buf, uint64_t offset, void *dst, uint64_t len);
/* Asynchronous counterpart of zg_buffer_read (new; the reference only has the
 * synchronous read_buffer_into, zengpu-cuda/src/lib.rs:560-615): queues a
 * device -> host copy of `len` bytes at `offset` into `dst` on the device
 * stream, after everything queued before it, and returns a submission whose
 * poll / wait report completion (like zg_submit_batch's).  Needs READBACK or
 * TRANSFER_SRC usage, so GpuOnly arrays (no READBACK) read back this way.
 * `dst` must stay valid and unread until the submission completes; page-locked
 * host memory makes the copy truly asynchronous.  While the submission is
 * pending the in-flight rules hold (no synchronous write / read / copy).  If a
 * GEMM queued before it without a synchronize had a bounded on-device wait
 * expire, the completing poll / wait returns ZG_ERR_KERNEL_WAIT. */
int zg_buffer_read_async(zg_device *dev, zg_handle buf, uint64_t offset, void *dst,
                         uint64_t len, zg_submission **out);
/* GpuDevice::copy_buffer (zengpu-cuda/src/lib.rs:617-691). */
int zg_buffer_copy(zg_device *dev, zg_handle src, uint64_t src_offset, zg_handle dst,
                   uint64_t dst_offset, uint64_t len);
/* GpuDevice::destroy_buffer (zengpu-cuda/src/lib.rs:693-723): stale handle is
 * a no-op; while a submission is in flight the free is deferred. */
void zg_buffer_destroy(zg_device *dev, zg_handle buf);
/* Device address and size of a live buffer (for layer 3 interop). */
int zg_buffer_info(zg_device *dev, zg_handle buf, uint64_t *device_ptr, uint64_t *size);
/* GpuDevice::copy_from_peer (zengpu-hal/src/device.rs:96-106; HIP backend
 * zengpu-hip/src/lib.rs:633-710): `bytes` from src (on src_dev) to dst (on
 * dst_dev), a direct copy over NVLink when can_peer holds, else staged through
 * host memory; synchronous.  A size beyond either buffer is ZG_ERR_BACKEND. */
int zg_buffer_copy_from_peer(zg_device *dst_dev, zg_handle dst, zg_device *src_dev,
                             zg_handle src, uint64_t bytes);

/* Shader kinds for zg_shader_create (ShaderDesc, zengpu-hal/src/desc.rs:63-126). */
#define ZG_SHADER_CUBIN 0u   /* sm_100a cubin or fatbin image */
#define ZG_SHADER_PTX 1u     /* NUL-terminated PTX text (driver JIT) */
#define ZG_SHADER_BUILTIN 2u /* this library's own kernels; code/len ignored */

/* GpuDevice::create_shader (zengpu-cuda/src/lib.rs:747-775). */
int zg_shader_create(zg_device *dev, uint32_t kind, const void *code, uint64_t len,
                     zg_handle *out);
void zg_shader_destroy(zg_device *dev, zg_handle shader);
/* GpuDevice::create_compute_pipeline (zengpu-cuda/src/lib.rs:803-832):
 * block {0,0,0} means 256x1x1. */
int zg_pipeline_create(zg_device *dev, zg_handle shader, const char *entry,
                       const uint32_t block[3], uint32_t dynamic_smem, zg_handle *out);
void zg_pipeline_destroy(zg_device *dev, zg_handle pipeline);

/* Scalar (zengpu-hal/src/command.rs:7-27): each occupies one 8-byte slot. */
#define ZG_SCALAR_U32 0u
#define ZG_SCALAR_I32 1u
#define ZG_SCALAR_F32 2u
typedef struct zg_scalar {
    uint32_t kind;
    uint32_t bits; /* the 4-byte value */
} zg_scalar;

/* One DispatchOp (zengpu-hal/src/command.rs:30-52).  `buffers` are buffer
 * slot indices (BufferHandle::index), as the reference binds them. */
typedef struct zg_dispatch_op {
    zg_handle pipeline;
    const uint32_t *buffers;
    uint32_t num_buffers;
    const zg_scalar *scalars;
    uint32_t num_scalars;
    uint32_t grid[3];
} zg_dispatch_op;

/* GpuDevice::dispatch - synchronous (zengpu-cuda/src/lib.rs:853-868). */
int zg_dispatch(zg_device *dev, const zg_dispatch_op *op);
/* GpuDevice::submit_batch - ops in order on the device stream, returns a
 * pollable submission (zengpu-cuda/src/lib.rs:870-993). */
int zg_submit_batch(zg_device *dev, const zg_dispatch_op *ops, uint32_t count,
                    zg_submission **out);
/* GpuSubmission::poll / wait(timeout) (zengpu-hal/src/submission.rs:22-38):
 * wait returns ZG_ERR_TIMEOUT without cancelling; *done is 1 once complete. */
int zg_submission_poll(zg_submission *sub, int *done);
int zg_submission_wait(zg_submission *sub, uint64_t timeout_ns);
/* Releases the submission; pending work keeps running and in-flight guards
 * drop once it completes. */
void zg_submission_destroy(zg_submission *sub);

/* ======================================================================
 * 2. Array ops (zengpu-compute, zengpu-blas)
 * ====================================================================== */

#define ZG_MAX_RANK 8

/* DeviceArray (zengpu-compute/src/lib.rs:21-72): row-major contiguous. */
typedef struct zg_device_array {
    zg_handle buffer;
    uint32_t dtype;
    uint32_t rank;
    uint32_t shape[ZG_MAX_RANK];
    uint32_t stride[ZG_MAX_RANK];
    uint64_t allocation_size;
} zg_device_array;

typedef struct zg_pool zg_pool;

/* size_class (zengpu-compute/src/pool.rs:75-78): next pow2, min 256 bytes. */
uint64_t zg_size_class(uint64_t size);
/* BufferPool::new / drop (zengpu-compute/src/pool.rs:17-89): Upload
 * residency, STORAGE | READBACK buffers, as the reference (:47-51). */
int zg_pool_create(zg_device *dev, zg_pool **out);
/* BufferPool with a chosen residency (new): ZG_MEMORY_UPLOAD as above, or
 * ZG_MEMORY_GPU_ONLY for device-resident arrays (STORAGE | TRANSFER_SRC |
 * TRANSFER_DST, no READBACK: read them back with zg_buffer_read_async or copy
 * them).  Ops whose output array comes from a GpuOnly pool (add, relu, sgemm,
 * gemm_bias_relu; in-place relu / saxpy / sscal on a GpuOnly array) are queued
 * on the device stream and return without the per-dispatch synchronize;
 * everything the host can do with those arrays is ordered after them on that
 * stream.  Other values: ZG_ERR_UNSUPPORTED. */
int zg_pool_create_with(zg_device *dev, uint32_t memory, zg_pool **out);
/* The residency a pool's buffers are created with (ZG_MEMORY_*). */
uint32_t zg_pool_memory(const zg_pool *pool);
void zg_pool_destroy(zg_pool *pool);
/* BufferPool::alloc (zengpu-compute/src/pool.rs:36-60). */
int zg_pool_alloc(zg_pool *pool, const uint32_t *shape, uint32_t rank, uint32_t dtype,
                  zg_device_array *out);
/* BufferPool::free (zengpu-compute/src/pool.rs:64-73). */
void zg_pool_free(zg_pool *pool, const zg_device_array *array);
/* Number of free pooled buffers in `size_class` (test introspection). */
uint32_t zg_pool_free_count(zg_pool *pool, uint64_t size_class);

/* ElementwiseKernels (zengpu-compute/src/elementwise.rs:51-146). */
typedef struct zg_elementwise_kernels {
    zg_handle add_shader;
    zg_handle add_pipeline;
    zg_handle relu_shader;
    zg_handle relu_pipeline;
} zg_elementwise_kernels;

int zg_elementwise_new(zg_device *dev, zg_elementwise_kernels *out);
void zg_elementwise_destroy(zg_device *dev, const zg_elementwise_kernels *k);
/* ElementwiseKernels::add: same shape, F32 only; `out` allocated from pool. */
int zg_elementwise_add(const zg_elementwise_kernels *k, zg_device *dev, zg_pool *pool,
                       const zg_device_array *a, const zg_device_array *b,
                       zg_device_array *out);
/* ElementwiseKernels::relu: F32 only; `out` allocated from pool. */
int zg_elementwise_relu(const zg_elementwise_kernels *k, zg_device *dev, zg_pool *pool,
                        const zg_device_array *a, zg_device_array *out);
/* In-place ReLU on `a` (the relu pipeline bound with out == in). */
int zg_elementwise_relu_inplace(const zg_elementwise_kernels *k, zg_device *dev,
                                const zg_device_array *a);

/* GemmKernel (zengpu-blas/src/level3.rs:101-182) plus a mode selector. */
typedef struct zg_gemm_kernel {
    zg_handle shader;
    zg_handle pipeline;       /* builtin "sgemm_f32": buffers [a,b,c], scalars [m,n,k,alpha] */
    zg_handle fused_pipeline; /* builtin "sgemm_bias_relu_f32": buffers [a,b,bias,c], same scalars */
    int32_t mode; /* ZG_GEMM_*; zg_gemm_new reads ZENGPU_GEMM_MODE, default TF32X3 */
} zg_gemm_kernel;

int zg_gemm_new(zg_device *dev, zg_gemm_kernel *out);
void zg_gemm_destroy(zg_device *dev, const zg_gemm_kernel *k);
/* GemmKernel::sgemm: C[m,n] = alpha * A[m,k] @ B[k,n]; C allocated from pool. */
int zg_gemm_sgemm(const zg_gemm_kernel *k, zg_device *dev, zg_pool *pool, float alpha,
                  const zg_device_array *a, const zg_device_array *b, zg_device_array *out);
/* GemmKernel::gemm: sgemm with alpha = 1. */
int zg_gemm_gemm(const zg_gemm_kernel *k, zg_device *dev, zg_pool *pool,
                 const zg_device_array *a, const zg_device_array *b, zg_device_array *out);
/* New fused op for the op_graph_lower Matmul->Add->Relu chain
 * (examples/op_graph_lower.rs:39-68): Y = relu(alpha * A@B + bias[n]),
 * bias a 1-D [n] array broadcast over rows; one kernel. */
int zg_gemm_bias_relu(const zg_gemm_kernel *k, zg_device *dev, zg_pool *pool, float alpha,
                      const zg_device_array *a, const zg_device_array *b,
                      const zg_device_array *bias, zg_device_array *out);

/* GemmKernel::sgemm on host arrays (new; the reference's callers write A and
 * B, dispatch and read C back, one synchronous step after the other):
 * C[m,n] = epilogue(alpha * A @ B) with a [m,k], b [k,n], c [m,n] row-major
 * host pointers and an optional host bias [n] (relu as in zg_sgemm_f32).
 * B is uploaded first, then row panels of A are uploaded, multiplied and
 * their C rows downloaded on three streams so the copies in both directions
 * overlap the tensor-core work.  Synchronous; device staging is cached per
 * device.  Pinned (page-locked) host memory gives full PCIe bandwidth. */
int zg_gemm_sgemm_host(const zg_gemm_kernel *k, zg_device *dev, float alpha, const float *a,
                       const float *b, const float *bias, int relu, float *c, uint32_t m,
                       uint32_t n, uint32_t kdim);

/* Level1Kernels (zengpu-blas/src/level1.rs:51-139): in place, no allocation. */
int zg_level1_saxpy(zg_device *dev, float alpha, const zg_device_array *x,
                    const zg_device_array *y);
int zg_level1_sscal(zg_device *dev, float alpha, const zg_device_array *x);

/* ======================================================================
 * 3. Stream kernels on raw device pointers (current device, caller stream;
 *    stream NULL = legacy default stream).  Asynchronous: errors found on
 *    the host are returned, launch errors are returned, device-side wait
 *    expiries are reported by zg_kernel_status().
 * ====================================================================== */

/* out[i] = a[i] + b[i]   (ADD_ZSL, zengpu-compute/src/elementwise.rs:17-26) */
int zg_add_f32(const float *a, const float *b, float *out, uint64_t n, void *stream);
/* out[i] = a[i] > 0 ? a[i] : +0  (RELU_ZSL, :29-38); out may equal a. */
int zg_relu_f32(const float *a, float *out, uint64_t n, void *stream);
/* y += alpha * x  (AXPY_ZSL, zengpu-blas/src/level1.rs:11-20) */
int zg_saxpy_f32(float alpha, const float *x, float *y, uint64_t n, void *stream);
/* x *= alpha  (SCAL_ZSL, zengpu-blas/src/level1.rs:23-32) */
int zg_sscal_f32(float alpha, float *x, uint64_t n, void *stream);

/* Scratch bytes zg_sgemm_f32 needs for (mode, m, n, k): the operand planes
 * the tensor-core kernel reads (tf32 / bf16 planes of A, and of B transposed
 * to K-major; TF32 reads A directly when k is a multiple of 4).  SIMT's is
 * optional: A transposed (k rows of round_up(m, 4) floats) for its TMA-fed
 * kernel, used when it is given and B is 16-byte aligned with n % 4 == 0;
 * otherwise SIMT runs its register-staged kernel on A (the same bits). */
uint64_t zg_sgemm_workspace_bytes(int mode, int m, int n, int k);
/* C[m,n] = epilogue(alpha * A[m,k] @ B[k,n]), all row-major f32.
 * epilogue: identity, or relu(x + bias[col]) when `bias` is non-NULL and
 * `relu` is 1, or x + bias[col] when `relu` is 0.  `workspace` must hold
 * zg_sgemm_workspace_bytes(...) bytes (may be NULL when that is 0, and for
 * SIMT, whose workspace is optional).
 * Replaces GEMM_PTX's entry `main(a,b,c,m,n,k,alpha)` (zengpu-blas/src/level3.rs:35-90). */
int zg_sgemm_f32(int mode, int m, int n, int k, float alpha, const float *a, const float *b,
                 float *c, const float *bias, int relu, void *workspace,
                 uint64_t workspace_bytes, void *stream);

/* The two halves of zg_sgemm_f32, for callers that reuse operands or time
 * the main kernel alone.  prepare: writes the operand planes of `mode` into
 * `workspace` (tf32 hi/lo of A and B for TF32X3, pitch-padded copies for
 * TF32 when k or n is not a multiple of 4; A transposed for SIMT when the
 * workspace and B allow its TMA-fed kernel).  compute: runs
 * the GEMM on planes a previous prepare wrote into the same workspace for the
 * same (mode, m, n, k, a, b); stream order makes the pair safe. */
int zg_sgemm_prepare(int mode, int m, int n, int k, const float *a, const float *b,
                     void *workspace, uint64_t workspace_bytes, void *stream);
int zg_sgemm_compute(int mode, int m, int n, int k, float alpha, const float *a, const float *b,
                     float *c, const float *bias, int relu, const void *workspace,
                     uint64_t workspace_bytes, void *stream);

/* Packed operands, for operands reused across GEMMs (a weight matrix, or the
 * row block of A multiplied by successive column panels of B).  A packed
 * operand holds exactly the planes the mode's kernel reads (TF32X3: tf32
 * hi/lo; TF32: f32; B K-major for the tensor-core modes), 256-byte aligned.
 * pack_bytes: size for operand 0 = A (outer = m) or 1 = B (outer = n).
 * sgemm_packed: C[m, n] (row pitch ldc >= n) = epilogue(alpha * A @ B) from
 * packed A and B of the same mode and k. */
uint64_t zg_sgemm_pack_bytes(int mode, int operand, int outer, int k);
int zg_sgemm_pack_a(int mode, int m, int k, const float *a, int64_t lda, void *packed,
                    uint64_t packed_bytes, void *stream);
int zg_sgemm_pack_b(int mode, int k, int n, const float *b, int64_t ldb, void *packed,
                    uint64_t packed_bytes, void *stream);
int zg_sgemm_packed(int mode, int m, int n, int k, float alpha, const void *a_packed,
                    const void *b_packed, float *c, int64_t ldc, const float *bias, int relu,
                    void *stream);

/* zg_sgemm_f32 for callers that cannot allocate device memory when they call
 * (no counterpart in the reference: ZenGPU's GemmKernel always allocates its
 * output from a BufferPool).  For example a host framework that owns all of
 * HBM in its own pool, a latency-critical loop that cannot pay for cudaMalloc's
 * device-wide synchronisation, or code inside an allocator callback.  The
 * caller still passes a, b, c (and bias); instead of a workspace this uses a
 * fixed 64 MiB scratch array in the library's device image, held on every GPU
 * that loads it until the process exits.  Shapes whose scratch need
 * (zg_sgemm_workspace_bytes) exceeds 64 MiB are rejected with ZG_ERR_DISPATCH
 * (TF32X3 fits up to 2048^3, BF16X3 up to 2880^3), except in SIMT, which then
 * runs without its optional workspace.  Allocates nothing.  The
 * first call on each device looks up the array's device address (make it
 * before any stream capture); a call under a new context of that device (after
 * cudaDeviceReset) looks it up again.  All calls share the array: calls that
 * overlap on the GPU race. */
int zg_sgemm_f32_noalloc(int mode, int m, int n, int k, float alpha, const float *a,
                         const float *b, float *c, const float *bias, int relu, void *stream);

/* Seeded synthetic inputs, bit-identical to the CPU generator:
 * uniform: x = lo + (hi - lo) * (u24 * 2^-24), or exactly u24*2^-23 - 1 when
 * lo = -1, hi = 1; normal: Box-Muller in f64 (may differ from a host libm in
 * the last bit, so parity tests feed identical bytes to both sides). */
int zg_fill_uniform_f32(float *x, uint64_t n, uint64_t seed, float lo, float hi, void *stream);
int zg_fill_normal_f32(float *x, uint64_t n, uint64_t seed, void *stream);

/* Name of the main kernel zg_sgemm_f32 / zg_sgemm_packed launch for
 * (mode, m, n, k) on the current device ("" for an unknown mode or an empty
 * output), for reports and profiler filters.  The tensor-core modes take the
 * CTA-pair kernel once there is a 256 x 256 tile for every SM pair (unless
 * the environment sets ZENGPU_GEMM_PAIRS=0).  SIMT names its TMA-fed kernel,
 * the one zg_sgemm_f32 runs with its workspace on 16-byte aligned B with
 * n % 4 == 0 (without them it runs sgemm_simt_kernel). */
const char *zg_sgemm_kernel_name(int mode, int m, int n, int k);

/* Reads and clears the device-side status word of the current device:
 * *code = 0 when every bounded on-device wait since the last call finished
 * in time, else a bitmask of the kernels whose wait expired.  Synchronises. */
int zg_kernel_status(uint32_t *code);

/* ---- B broadcast along a chain of GPUs (row-sharded GEMM, one process per
 * GPU).  No counterpart in the reference: ZenGPU has no collective; its only
 * multi-device operation is a HIP peer copy (zengpu-hip/src/lib.rs:609-710).
 *
 * Ranks 0 -> 1 -> ... -> W-1 each create a chain object (same mode, k, n,
 * chunk_cols on every rank), exchange the 64-byte CUDA IPC handles by any
 * means, and connect to their neighbours.  Each step e (1, 2, ..., the same
 * on every rank) then runs:
 *   rank 0      zg_bchain_source(e, B): packs B^T into the tensor-core operand
 *               form chunk by chunk (chunk_cols columns of B each, a multiple
 *               of 256), raising each chunk's flag;
 *   every rank  zg_bchain_forward(e) on a copy stream: pushes each chunk, once
 *               its flag is up, to the next rank with a copy-engine peer copy
 *               and raises the flag there (no SMs used);
 *               zg_bchain_gemm(e, gated): C = epilogue(alpha * A @ B) with A
 *               packed by zg_sgemm_pack_a; gated = 1 lets the kernel start at
 *               once and hold back the B loads of chunks not yet arrived (the
 *               rank that ran zg_bchain_source on the same stream passes 0);
 *               zg_bchain_release(e) on a stream ordered after both: tells the
 *               previous rank this rank's buffer of step e may be reused.
 * Two buffers alternate between steps.  A wait that can never end (a rank
 * that died) is ended by zg_bchain_abort on the waiting ranks; the GEMM's own
 * gate gives up after 2 s and reports ZG_ERR_KERNEL_WAIT through
 * zg_kernel_status.  After an abort the flags order nothing any more: the
 * results of the aborted steps are invalid and the chain is only destroyed.  Tensor-core modes only.  A chain object belongs to the
 * device current at create and is driven from one host thread. */
#define ZG_IPC_HANDLE_BYTES 64
typedef struct zg_bchain zg_bchain;
int zg_bchain_create(int mode, int k, int n, int chunk_cols, zg_bchain **out, uint8_t *handle);
int zg_bchain_connect(zg_bchain *chain, const uint8_t *prev_handle, const uint8_t *next_handle);
int zg_bchain_source(zg_bchain *chain, uint32_t epoch, const float *b, int64_t ldb, void *stream);
int zg_bchain_forward(zg_bchain *chain, uint32_t epoch, void *stream);
int zg_bchain_gemm(zg_bchain *chain, uint32_t epoch, int gated, int m, float alpha,
                   const void *a_packed, float *c, int64_t ldc, const float *bias, int relu,
                   void *stream);
int zg_bchain_release(zg_bchain *chain, uint32_t epoch, void *stream);
/* The packed B^T buffer step `epoch` uses, and its size in bytes. */
int zg_bchain_buffer(const zg_bchain *chain, uint32_t epoch, const void **ptr, uint64_t *bytes);
int zg_bchain_abort(zg_bchain *chain, uint32_t epoch);
int zg_bchain_destroy(zg_bchain *chain);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* ZENGPU_B200_H */
