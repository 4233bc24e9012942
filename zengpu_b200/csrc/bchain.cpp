// bchain.cpp - B broadcast along a chain of GPUs by the copy engines, for the
// row-sharded GEMM (one process per GPU).
//
// The reference has no collective (its only multi-device operation is a HIP
// peer copy, zengpu-hip/src/lib.rs:609-710).  Here the sharded GEMM's one
// exchange - every rank needs all of B - is done without taking SMs from the
// GEMM: rank 0 packs B into the tensor-core operand form chunk by chunk, and
// each rank r pushes every chunk it holds to rank r + 1 with cudaMemcpyAsync
// over NVLink (a copy engine), then raises that chunk's flag in rank r + 1's
// memory with a stream write.  Every rank's GEMM starts at once and holds back
// only the B loads of chunks whose flag has not arrived (GemmGate), so the
// transfer runs under the GEMM.  Stream waits (cuStreamWaitValue32) order the
// forwarding on each copy stream; no kernel waits on another kernel.
//
// Memory of one rank (one cudaMalloc, exported through CUDA IPC):
//   packed B buffer 0 | packed B buffer 1 | arrival flags [2][chunks] | done
// Epoch e (1, 2, ...) uses buffer e & 1.  flags[b][c] >= e: chunk c of epoch
// e is in buffer b.  done >= e: the downstream rank has finished epoch e (its
// GEMM and its own forwarding), so its buffer e & 1 may be overwritten by
// epoch e + 2.  All comparisons are wrap-aware ((int32_t)(x - e) >= 0).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <new>

#include "zengpu_b200.h"
#include "zg_gemm_internal.h"

namespace zg {
int set_error(int code, const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);
}  // namespace zg

using zg::cuda_status;
using zg::set_error;

namespace {

struct StreamOps {
    CUresult (*wait32)(CUstream, CUdeviceptr, cuuint32_t, unsigned int) = nullptr;
    CUresult (*write32)(CUstream, CUdeviceptr, cuuint32_t, unsigned int) = nullptr;
    bool ok = false;
};

const StreamOps& stream_ops() {
    static StreamOps ops;
    static std::once_flag once;
    std::call_once(once, [] {
        auto get = [](const char* name, void** fn) {
            cudaDriverEntryPointQueryResult q;
            return cudaGetDriverEntryPointByVersion(name, fn, 12000, cudaEnableDefault, &q) ==
                       cudaSuccess &&
                   q == cudaDriverEntryPointSuccess;
        };
        ops.ok = get("cuStreamWaitValue32", reinterpret_cast<void**>(&ops.wait32)) &&
                 get("cuStreamWriteValue32", reinterpret_cast<void**>(&ops.write32));
    });
    return ops;
}

int drv_status(CUresult r, const char* what) {
    if (r == CUDA_SUCCESS) return ZG_OK;
    return set_error(ZG_ERR_BACKEND, "%s failed (CUresult %d)", what, static_cast<int>(r));
}

// Stream write of `value` to a u32 (this GPU's or a peer's), after every
// earlier operation of the stream, with a system-wide memory barrier first.
int write_flag(uint32_t* addr, uint32_t value, cudaStream_t s) {
    const StreamOps& ops = stream_ops();
    if (!ops.ok) return set_error(ZG_ERR_BACKEND, "stream memory operations unavailable");
    return drv_status(ops.write32(reinterpret_cast<CUstream>(s),
                                  reinterpret_cast<CUdeviceptr>(addr), value, 0),
                      "cuStreamWriteValue32");
}

// The stream waits until (int32_t)(*addr - value) >= 0.
int wait_flag(const uint32_t* addr, uint32_t value, cudaStream_t s) {
    const StreamOps& ops = stream_ops();
    if (!ops.ok) return set_error(ZG_ERR_BACKEND, "stream memory operations unavailable");
    return drv_status(ops.wait32(reinterpret_cast<CUstream>(s),
                                 reinterpret_cast<CUdeviceptr>(addr), value,
                                 CU_STREAM_WAIT_VALUE_GEQ),
                      "cuStreamWaitValue32");
}

constexpr uint64_t round256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

}  // namespace

struct zg_bchain {
    int device = 0;
    int mode = 0, k = 0, n = 0, chunk_cols = 0, chunks = 0;
    int64_t ld = 0;               // packed B^T row pitch, 4-byte units
    uint64_t buf_bytes = 0;       // one packed B buffer
    uint64_t off_flags = 0, off_done = 0, off_count = 0, total = 0;
    uint8_t* base = nullptr;      // this rank's allocation
    uint8_t* prev = nullptr;      // upstream rank's allocation (IPC), or null
    uint8_t* next = nullptr;      // downstream rank's allocation (IPC), or null

    uint8_t* buf(uint8_t* b, uint32_t epoch) const { return b + (epoch & 1u) * buf_bytes; }
    uint32_t* flags(uint8_t* b, uint32_t epoch) const {
        return reinterpret_cast<uint32_t*>(b + off_flags) + (epoch & 1u) * chunks;
    }
    uint32_t* done(uint8_t* b) const { return reinterpret_cast<uint32_t*>(b + off_done); }
    uint32_t* counters() const { return reinterpret_cast<uint32_t*>(base + off_count); }
    int chunk_rows(int c) const {
        const int r0 = c * chunk_cols;
        return (n - r0 < chunk_cols) ? n - r0 : chunk_cols;
    }
    uint64_t chunk_offset(int c) const {
        return static_cast<uint64_t>(c) * chunk_cols * static_cast<uint64_t>(ld) * 4;
    }
};

namespace {

int check_chain(const zg_bchain* c, const char* what) {
    if (!c) return set_error(ZG_ERR_DISPATCH, "%s: null chain", what);
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != c->device)
        return set_error(ZG_ERR_DISPATCH, "%s: chain lives on device %d, current device is %d",
                         what, c->device, dev);
    return ZG_OK;
}

}  // namespace

extern "C" int zg_bchain_create(int mode, int k, int n, int chunk_cols, zg_bchain** out,
                                uint8_t* handle) {
    if (!out || !handle) return set_error(ZG_ERR_DISPATCH, "bchain_create: null output");
    *out = nullptr;
    if (mode != ZG_GEMM_TF32 && mode != ZG_GEMM_TF32X3 && mode != ZG_GEMM_TF32_BF16X2 &&
        mode != ZG_GEMM_BF16X3)
        return set_error(ZG_ERR_DISPATCH, "bchain_create: mode %d has no chunked B^T form", mode);
    if (k <= 0 || n <= 0 || chunk_cols <= 0 || chunk_cols % 256 != 0)
        return set_error(ZG_ERR_DISPATCH,
                         "bchain_create: bad shape k=%d n=%d chunk=%d (chunk: multiple of 256)", k,
                         n, chunk_cols);
    zg_bchain* c = new (std::nothrow) zg_bchain;
    if (!c) return set_error(ZG_ERR_OUT_OF_MEMORY, "bchain_create: host allocation");
    cudaGetDevice(&c->device);
    c->mode = mode;
    c->k = k;
    c->n = n;
    c->chunk_cols = chunk_cols;
    c->chunks = (n + chunk_cols - 1) / chunk_cols;
    c->ld = zg::gemm_carve_planes(nullptr, mode, n, k).ld;
    c->buf_bytes = round256(zg::gemm_planes_bytes(mode, n, k));
    c->off_flags = 2 * c->buf_bytes;
    c->off_done = c->off_flags + round256(2ull * c->chunks * sizeof(uint32_t));
    c->off_count = c->off_done + 256;
    c->total = c->off_count + round256(static_cast<uint64_t>(c->chunks) * sizeof(uint32_t));
    cudaError_t e = cudaMalloc(&c->base, c->total);
    if (e != cudaSuccess) {
        delete c;
        return cuda_status(e, "bchain_create: cudaMalloc");
    }
    // flags and done start at 0: no epoch has arrived, every buffer is free
    e = cudaMemset(c->base + c->off_flags, 0, c->total - c->off_flags);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->base);
    if (e != cudaSuccess) {
        cudaFree(c->base);
        delete c;
        return cuda_status(e, "bchain_create: flags / IPC handle");
    }
    static_assert(sizeof(h) == ZG_IPC_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle, &h, sizeof(h));
    *out = c;
    return ZG_OK;
}

extern "C" int zg_bchain_connect(zg_bchain* c, const uint8_t* prev_handle,
                                 const uint8_t* next_handle) {
    if (int rc = check_chain(c, "bchain_connect")) return rc;
    if (c->prev || c->next) return set_error(ZG_ERR_DISPATCH, "bchain_connect: already connected");
    auto open = [](const uint8_t* hb, uint8_t** ptr) {
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hb, sizeof(h));
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        *ptr = static_cast<uint8_t*>(p);
        return e;
    };
    if (prev_handle) {
        cudaError_t e = open(prev_handle, &c->prev);
        if (e != cudaSuccess) return cuda_status(e, "bchain_connect: open upstream");
    }
    if (next_handle) {
        cudaError_t e = open(next_handle, &c->next);
        if (e != cudaSuccess) {
            if (c->prev) cudaIpcCloseMemHandle(c->prev);
            c->prev = nullptr;
            return cuda_status(e, "bchain_connect: open downstream");
        }
    }
    return ZG_OK;
}

extern "C" int zg_bchain_source(zg_bchain* c, uint32_t epoch, const float* b, int64_t ldb,
                                void* stream) {
    if (int rc = check_chain(c, "bchain_source")) return rc;
    if (!b || ldb < c->n) return set_error(ZG_ERR_DISPATCH, "bchain_source: bad B");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const zg::OperandView view = zg::gemm_carve_planes(c->buf(c->base, epoch), c->mode, c->n, c->k);
    // one launch; its last CTA of each chunk raises that chunk's flag
    return zg::gemm_prep_b_signal(c->mode, c->k, c->n, b, ldb, view, c->chunk_cols,
                                  c->counters(), c->flags(c->base, epoch), epoch, s);
}

extern "C" int zg_bchain_forward(zg_bchain* c, uint32_t epoch, void* stream) {
    if (int rc = check_chain(c, "bchain_forward")) return rc;
    if (!c->next) return ZG_OK;  // last rank of the chain
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // the downstream rank is done with this buffer's previous epoch
    if (int rc = wait_flag(c->done(c->base), epoch - 2, s)) return rc;
    const uint32_t* mine = c->flags(c->base, epoch);
    uint32_t* theirs = c->flags(c->next, epoch);
    uint8_t* src = c->buf(c->base, epoch);
    uint8_t* dst = c->buf(c->next, epoch);
    for (int ch = 0; ch < c->chunks; ++ch) {
        const uint64_t off = c->chunk_offset(ch);
        const uint64_t bytes = static_cast<uint64_t>(c->chunk_rows(ch)) * c->ld * 4;
        if (int rc = wait_flag(mine + ch, epoch, s)) return rc;
        cudaError_t e = cudaMemcpyAsync(dst + off, src + off, bytes, cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return cuda_status(e, "bchain_forward: peer copy");
        if (int rc = write_flag(theirs + ch, epoch, s)) return rc;
    }
    return ZG_OK;
}

extern "C" int zg_bchain_gemm(zg_bchain* c, uint32_t epoch, int gated, int m, float alpha,
                              const void* a_packed, float* out, int64_t ldc, const float* bias,
                              int relu, void* stream) {
    if (int rc = check_chain(c, "bchain_gemm")) return rc;
    if (m < 0 || ldc < c->n) return set_error(ZG_ERR_DISPATCH, "bchain_gemm: bad shape");
    if (m == 0) return ZG_OK;
    if (!a_packed || !out) return set_error(ZG_ERR_DISPATCH, "bchain_gemm: null operand");
    zg::GemmOperands op{c->mode, zg::gemm_carve_planes(const_cast<void*>(a_packed), c->mode, m, c->k),
                        zg::gemm_carve_planes(c->buf(c->base, epoch), c->mode, c->n, c->k)};
    zg::GemmGate gate;
    if (gated) {
        gate.flags = c->flags(c->base, epoch);
        gate.epoch = epoch;
        gate.rows = c->chunk_cols;
    }
    return zg::gemm_run(op, m, c->n, c->k, alpha, out, ldc, bias, relu,
                        static_cast<cudaStream_t>(stream), gated ? &gate : nullptr);
}

extern "C" int zg_bchain_release(zg_bchain* c, uint32_t epoch, void* stream) {
    if (int rc = check_chain(c, "bchain_release")) return rc;
    if (!c->prev) return ZG_OK;  // rank 0 has no upstream
    return write_flag(c->done(c->prev), epoch, static_cast<cudaStream_t>(stream));
}

extern "C" int zg_bchain_buffer(const zg_bchain* c, uint32_t epoch, const void** ptr,
                                uint64_t* bytes) {
    if (int rc = check_chain(c, "bchain_buffer")) return rc;
    if (ptr) *ptr = c->buf(c->base, epoch);
    if (bytes) *bytes = zg::gemm_planes_bytes(c->mode, c->n, c->k);
    return ZG_OK;
}

extern "C" int zg_bchain_abort(zg_bchain* c, uint32_t epoch) {
    if (int rc = check_chain(c, "bchain_abort")) return rc;
    // Every local flag and the done word jump far past `epoch`, on a stream of
    // their own, so this rank's stream waits and arrival gates end.
    const uint32_t v = epoch + (1u << 30);
    const uint64_t words = (c->total - c->off_flags) / sizeof(uint32_t);
    uint32_t* host = new (std::nothrow) uint32_t[words];
    if (!host) return set_error(ZG_ERR_OUT_OF_MEMORY, "bchain_abort: host buffer");
    for (uint64_t i = 0; i < words; ++i) host[i] = v;
    cudaStream_t s = nullptr;
    cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    if (e == cudaSuccess) {
        e = cudaMemcpyAsync(c->base + c->off_flags, host, words * sizeof(uint32_t),
                            cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        cudaStreamDestroy(s);
    }
    delete[] host;
    return cuda_status(e, "bchain_abort");
}

extern "C" int zg_bchain_destroy(zg_bchain* c) {
    if (!c) return ZG_OK;
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != c->device) cudaSetDevice(c->device);
    cudaError_t e = cudaSuccess;
    if (c->prev) e = cudaIpcCloseMemHandle(c->prev);
    if (c->next) {
        cudaError_t e2 = cudaIpcCloseMemHandle(c->next);
        if (e == cudaSuccess) e = e2;
    }
    cudaError_t e3 = cudaFree(c->base);
    if (e == cudaSuccess) e = e3;
    if (dev != c->device && dev >= 0) cudaSetDevice(dev);
    delete c;
    return cuda_status(e, "bchain_destroy");
}
