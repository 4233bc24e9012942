// runtime.cpp - host side of libzengpu_b200: the GpuDevice compute subset
// (zengpu-cuda/src/lib.rs:472-1164), DeviceArray / BufferPool
// (zengpu-compute/src/lib.rs, pool.rs), ElementwiseKernels
// (zengpu-compute/src/elementwise.rs), GemmKernel (zengpu-blas/src/level3.rs)
// and Level1Kernels (zengpu-blas/src/level1.rs), exported as the C ABI in
// include/zengpu_b200.h.
//
// Semantics kept from the reference:
//  * generational handles; a stale handle is an error on use and a no-op on
//    destroy (zengpu-hal/src/handle.rs:72-243);
//  * one non-blocking stream per device; dispatch is synchronous, submit
//    returns a pollable submission whose wait(timeout) never cancels;
//  * buffer writes / reads / copies are refused while a submission is in
//    flight, and destroys are deferred until it completes;
//  * shape and dtype errors are GpuError::Dispatch with the reference text.
// Added: a BufferPool may hand out GpuOnly (device-resident, not host
// readable) arrays; ops whose output is such an array are queued on the device
// stream without the per-dispatch synchronize, and zg_buffer_read_async reads
// results back through a pollable submission.
// What changed: the CUDA backend now runs hand-written sm_100a kernels linked
// into this library ("builtin" shaders) instead of ZSL/SPIR-V, and can still
// load caller cubins / PTX through the driver API.
#include <cuda.h>
#include <cuda_runtime.h>

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "zengpu_b200.h"
#include "zg_gemm_internal.h"

namespace zg {

// ---- errors -------------------------------------------------------------------
namespace {
thread_local std::string g_last_error;
thread_local zg_error_detail g_detail{};
}

int set_error(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    g_detail = zg_error_detail{};
    g_detail.status = code;
    g_detail.memory = ZG_MEMORY_GPU_ONLY;  // a CUDA allocation (zengpu-cuda/src/error.rs:18)
    g_detail.resource = "";
    g_detail.needed = "";
    return code;
}

// UsageError::MissingUsage with the reference's field values
// (zengpu-cuda/src/lib.rs:539-542, 645-654).
int missing_usage(const char* resource, const char* needed, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    set_error(ZG_ERR_MISSING_USAGE, "%s", buf);
    g_detail.resource = resource;
    g_detail.needed = needed;
    return ZG_ERR_MISSING_USAGE;
}

// CUDA runtime error -> status, following zengpu-cuda/src/error.rs:16-36.
int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return ZG_OK;
    const char* name = cudaGetErrorName(e);
    int code = ZG_ERR_BACKEND;
    switch (e) {
        case cudaErrorMemoryAllocation: code = ZG_ERR_OUT_OF_MEMORY; break;
        case cudaErrorContextIsDestroyed:
        case cudaErrorCudartUnloading: code = ZG_ERR_DEVICE_LOST; break;
        case cudaErrorNoDevice:
        case cudaErrorInsufficientDriver: code = ZG_ERR_NO_DEVICE; break;
        case cudaErrorLaunchFailure:
        case cudaErrorLaunchOutOfResources:
        case cudaErrorLaunchTimeout:
        case cudaErrorCooperativeLaunchTooLarge:
        case cudaErrorInvalidConfiguration: code = ZG_ERR_DISPATCH; break;
        case cudaErrorInvalidPtx:
        case cudaErrorNoKernelImageForDevice:
        case cudaErrorUnsupportedPtxVersion:
        case cudaErrorInvalidSource: code = ZG_ERR_SHADER_COMPILE; break;
        default: break;
    }
    return set_error(code, "cuda: %s: %s (%s)", what, name ? name : "?", cudaGetErrorString(e));
}

int cu_status(CUresult r, const char* what) {
    if (r == CUDA_SUCCESS) return ZG_OK;
    int code = ZG_ERR_BACKEND;
    switch (r) {
        case CUDA_ERROR_OUT_OF_MEMORY: code = ZG_ERR_OUT_OF_MEMORY; break;
        case CUDA_ERROR_CONTEXT_IS_DESTROYED:
        case CUDA_ERROR_DEINITIALIZED: code = ZG_ERR_DEVICE_LOST; break;
        case CUDA_ERROR_LAUNCH_FAILED:
        case CUDA_ERROR_LAUNCH_OUT_OF_RESOURCES:
        case CUDA_ERROR_LAUNCH_TIMEOUT:
        case CUDA_ERROR_COOPERATIVE_LAUNCH_TOO_LARGE: code = ZG_ERR_DISPATCH; break;
        case CUDA_ERROR_INVALID_PTX:
        case CUDA_ERROR_NO_BINARY_FOR_GPU:
        case CUDA_ERROR_UNSUPPORTED_PTX_VERSION:
        case CUDA_ERROR_INVALID_SOURCE:
        case CUDA_ERROR_INVALID_IMAGE: code = ZG_ERR_SHADER_COMPILE; break;
        case CUDA_ERROR_NOT_FOUND: code = ZG_ERR_PIPELINE_CREATION; break;
        default: break;
    }
    return set_error(code, "cuda: %s failed (CUresult %d)", what, static_cast<int>(r));
}

// ---- driver entry points (no link-time dependency on libcuda) --------------------
struct Driver {
    CUresult (*moduleLoadData)(CUmodule*, const void*) = nullptr;
    CUresult (*moduleUnload)(CUmodule) = nullptr;
    CUresult (*moduleGetFunction)(CUfunction*, CUmodule, const char*) = nullptr;
    CUresult (*funcSetAttribute)(CUfunction, CUfunction_attribute, int) = nullptr;
    CUresult (*launchKernel)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned,
                             unsigned, unsigned, CUstream, void**, void**) = nullptr;
    bool ok = false;
};

const Driver& driver() {
    static Driver d;
    static std::once_flag once;
    std::call_once(once, [] {
        auto get = [](const char* name, void** fn) {
            cudaDriverEntryPointQueryResult q;
            return cudaGetDriverEntryPointByVersion(name, fn, 12000, cudaEnableDefault, &q) ==
                       cudaSuccess &&
                   q == cudaDriverEntryPointSuccess;
        };
        d.ok = get("cuModuleLoadData", reinterpret_cast<void**>(&d.moduleLoadData)) &&
               get("cuModuleUnload", reinterpret_cast<void**>(&d.moduleUnload)) &&
               get("cuModuleGetFunction", reinterpret_cast<void**>(&d.moduleGetFunction)) &&
               get("cuFuncSetAttribute", reinterpret_cast<void**>(&d.funcSetAttribute)) &&
               get("cuLaunchKernel", reinterpret_cast<void**>(&d.launchKernel));
    });
    return d;
}

// ---- generational slot map (zengpu-hal/src/handle.rs:72-243) ---------------------
template <class T>
class SlotMap {
  public:
    enum State : uint8_t { kFree = 0, kLive = 1, kRetired = 2 };
    struct Slot {
        T value{};
        uint32_t gen = 0;
        State state = kFree;
    };

    zg_handle insert(const T& v) {
        uint32_t idx;
        if (!free_.empty()) {
            idx = free_.back();
            free_.pop_back();
        } else {
            idx = static_cast<uint32_t>(slots_.size());
            slots_.emplace_back();
        }
        Slot& s = slots_[idx];
        s.value = v;
        s.state = kLive;
        return zg_handle{idx, s.gen};
    }
    // Live value for `h`, or null (stale generation, freed or out of range).
    T* get(zg_handle h) {
        if (h.index >= slots_.size()) return nullptr;
        Slot& s = slots_[h.index];
        return (s.state == kLive && s.gen == h.generation) ? &s.value : nullptr;
    }
    // Live value in slot `idx` regardless of generation (Bindings carry bare
    // slot indices, zengpu-hal/src/handle.rs:206-208).
    T* get_by_index(uint32_t idx) {
        if (idx >= slots_.size()) return nullptr;
        Slot& s = slots_[idx];
        return s.state == kLive ? &s.value : nullptr;
    }
    // Value in an occupied (live or retired) slot, else null.
    T* value_at(uint32_t idx) {
        if (idx >= slots_.size() || slots_[idx].state == kFree) return nullptr;
        return &slots_[idx].value;
    }
    uint32_t current_gen(uint32_t idx) const {
        return idx < slots_.size() ? slots_[idx].gen : 0;
    }
    bool remove(zg_handle h, T* out) {
        T* v = get(h);
        if (!v) return false;
        *out = *v;
        release(h.index);
        return true;
    }
    // Invalidate `h` now but keep the slot out of reuse until release().
    bool retire(zg_handle h, T* out) {
        T* v = get(h);
        if (!v) return false;
        *out = *v;
        Slot& s = slots_[h.index];
        s.state = kRetired;
        ++s.gen;
        return true;
    }
    void release(uint32_t idx) {
        Slot& s = slots_[idx];
        if (s.state == kLive) ++s.gen;
        s.state = kFree;
        s.value = T{};
        free_.push_back(idx);
    }
    template <class F>
    void for_each_occupied(F f) {
        for (uint32_t i = 0; i < slots_.size(); ++i)
            if (slots_[i].state != kFree) f(i, slots_[i].value);
    }

  private:
    std::vector<Slot> slots_;
    std::vector<uint32_t> free_;
};

// ---- device objects ----------------------------------------------------------------
struct Buffer {
    void* ptr = nullptr;
    uint64_t len = 0;
    uint32_t usage = 0;
    uint32_t memory = 0;
};

struct Shader {
    uint32_t kind = 0;
    CUmodule module = nullptr;
};

enum Builtin : int {
    kNotBuiltin = 0,
    kAddF32,
    kReluF32,
    kSaxpyF32,
    kSscalF32,
    kSgemmF32,
    kSgemmBiasReluF32,
};

struct Pipeline {
    zg_handle shader{};
    int builtin = kNotBuiltin;
    int gemm_mode = -1;  // builtin sgemm: -1 = device default
    CUfunction fn = nullptr;
    uint32_t block[3] = {256, 1, 1};
    uint32_t smem = 0;
};

int default_gemm_mode() {
    const char* e = std::getenv("ZENGPU_GEMM_MODE");
    if (!e) return ZG_GEMM_TF32X3;
    std::string s(e);
    if (s == "simt" || s == "simt_fp32" || s == "fp32") return ZG_GEMM_SIMT_FP32;
    if (s == "tf32") return ZG_GEMM_TF32;
    if (s == "tf32bf16" || s == "tf32_bf16x2") return ZG_GEMM_TF32_BF16X2;
    if (s == "bf16x3") return ZG_GEMM_BF16X3;
    return ZG_GEMM_TF32X3;
}

}  // namespace zg

using namespace zg;

struct zg_device {
    int ordinal = 0;
    cudaStream_t stream = nullptr;
    std::recursive_mutex mu;
    SlotMap<Buffer> buffers;
    SlotMap<Shader> shaders;
    SlotMap<Pipeline> pipelines;
    // Submissions not yet observed complete, and frees deferred until then.
    std::vector<cudaEvent_t> pending;
    std::vector<uint32_t> deferred_buffers;  // retired slot indices
    // A tensor-core GEMM was queued without a synchronize since the device
    // status word was last read: the next readback submission checks it.
    bool status_unchecked = false;
    void* workspace = nullptr;
    uint64_t workspace_bytes = 0;
    // Pipelined host-buffer GEMM: copy streams and device staging.
    cudaStream_t h2d = nullptr;
    cudaStream_t d2h = nullptr;
    void* staging = nullptr;
    uint64_t staging_bytes = 0;
    // can_peer results: peer ordinal -> usable (peer access enabled)
    std::unordered_map<int, bool> peer_access;
};

struct zg_submission {
    zg_device* dev = nullptr;
    cudaEvent_t event = nullptr;
    bool done = false;
    // read the device status word once complete (bounded on-device waits of
    // GEMMs queued without a synchronize before this submission)
    bool check_status = false;
};

struct zg_pool {
    zg_device* dev = nullptr;
    uint32_t memory = ZG_MEMORY_UPLOAD;  // residency of the buffers it creates
    std::mutex mu;
    std::unordered_map<uint64_t, std::vector<zg_handle>> free;
};

namespace zg {
namespace {

int set_device(zg_device* dev) { return cuda_status(cudaSetDevice(dev->ordinal), "cudaSetDevice"); }

// Releases one submission's in-flight token (zengpu-cuda/src/lib.rs:412-444):
// a submission counts as in flight until poll/wait observes it complete or it
// is destroyed, exactly as in the reference, even when the GPU finished
// earlier.  Deferred frees run once no submission is in flight.  Caller
// holds dev->mu.
void release_submission(zg_device* dev, cudaEvent_t ev) {
    auto& p = dev->pending;
    for (size_t i = 0; i < p.size(); ++i)
        if (p[i] == ev) {
            p[i] = p.back();
            p.pop_back();
            break;
        }
    cudaEventDestroy(ev);
    if (p.empty() && !dev->deferred_buffers.empty()) {
        for (uint32_t idx : dev->deferred_buffers) {
            Buffer* b = dev->buffers.value_at(idx);  // retired slots keep their value
            if (b && b->ptr) cudaFree(b->ptr);
            dev->buffers.release(idx);
        }
        dev->deferred_buffers.clear();
    }
}

bool in_flight(zg_device* dev) { return !dev->pending.empty(); }

int stale(const char* what, zg_handle h, uint32_t actual) {
    set_error(ZG_ERR_STALE_HANDLE, "%s: stale handle (index %u, generation %u, current %u)",
              what, h.index, h.generation, actual);
    g_detail.handle_index = h.index;
    g_detail.expected_gen = h.generation;
    g_detail.actual_gen = actual;
    return ZG_ERR_STALE_HANDLE;
}

int ensure_workspace(zg_device* dev, uint64_t bytes) {
    if (bytes <= dev->workspace_bytes) return ZG_OK;
    if (dev->workspace) {
        cudaStreamSynchronize(dev->stream);
        cudaFree(dev->workspace);
        dev->workspace = nullptr;
        dev->workspace_bytes = 0;
    }
    int rc = cuda_status(cudaMalloc(&dev->workspace, bytes), "workspace alloc");
    if (rc == ZG_OK) dev->workspace_bytes = bytes;
    return rc;
}

// Resolves binding slot i to a live buffer pointer.
int bound_ptr(zg_device* dev, const zg_dispatch_op* op, uint32_t i, void** out) {
    if (i >= op->num_buffers)
        return set_error(ZG_ERR_BINDING_MISMATCH, "dispatch: expected at least %u buffers, got %u",
                         i + 1, op->num_buffers);
    Buffer* b = dev->buffers.get_by_index(op->buffers[i]);
    if (!b)
        return set_error(ZG_ERR_BINDING_MISMATCH, "dispatch: buffer slot %u is not a live buffer",
                         op->buffers[i]);
    *out = b->ptr;
    return ZG_OK;
}

int scalar_u32(const zg_dispatch_op* op, uint32_t i, uint32_t* v) {
    if (i >= op->num_scalars || (op->scalars[i].kind != ZG_SCALAR_U32 &&
                                 op->scalars[i].kind != ZG_SCALAR_I32))
        return set_error(ZG_ERR_BINDING_MISMATCH, "dispatch: scalar %u must be a U32", i);
    *v = op->scalars[i].bits;
    return ZG_OK;
}

int scalar_f32(const zg_dispatch_op* op, uint32_t i, float* v) {
    if (i >= op->num_scalars || op->scalars[i].kind != ZG_SCALAR_F32)
        return set_error(ZG_ERR_BINDING_MISMATCH, "dispatch: scalar %u must be an F32", i);
    std::memcpy(v, &op->scalars[i].bits, 4);
    return ZG_OK;
}

// Launches one builtin op on the device stream (no synchronisation).
int launch_builtin(zg_device* dev, const Pipeline& p, const zg_dispatch_op* op, int mode_override) {
    int rc;
    void *b0 = nullptr, *b1 = nullptr, *b2 = nullptr, *b3 = nullptr;
    uint32_t n = 0, m = 0, k = 0;
    float alpha = 0.f;
    switch (p.builtin) {
        case kAddF32:  // buffers [a, b, out], scalars [U32 len]
            if ((rc = bound_ptr(dev, op, 0, &b0)) || (rc = bound_ptr(dev, op, 1, &b1)) ||
                (rc = bound_ptr(dev, op, 2, &b2)) || (rc = scalar_u32(op, 0, &n)))
                return rc;
            return zg_add_f32(static_cast<float*>(b0), static_cast<float*>(b1),
                              static_cast<float*>(b2), n, dev->stream);
        case kReluF32:  // buffers [in, out], scalars [U32 len]
            if ((rc = bound_ptr(dev, op, 0, &b0)) || (rc = bound_ptr(dev, op, 1, &b1)) ||
                (rc = scalar_u32(op, 0, &n)))
                return rc;
            return zg_relu_f32(static_cast<float*>(b0), static_cast<float*>(b1), n, dev->stream);
        case kSaxpyF32:  // buffers [x, y], scalars [U32 n, F32 alpha]
            if ((rc = bound_ptr(dev, op, 0, &b0)) || (rc = bound_ptr(dev, op, 1, &b1)) ||
                (rc = scalar_u32(op, 0, &n)) || (rc = scalar_f32(op, 1, &alpha)))
                return rc;
            return zg_saxpy_f32(alpha, static_cast<float*>(b0), static_cast<float*>(b1), n,
                                dev->stream);
        case kSscalF32:  // buffers [x], scalars [U32 n, F32 alpha]
            if ((rc = bound_ptr(dev, op, 0, &b0)) || (rc = scalar_u32(op, 0, &n)) ||
                (rc = scalar_f32(op, 1, &alpha)))
                return rc;
            return zg_sscal_f32(alpha, static_cast<float*>(b0), n, dev->stream);
        case kSgemmF32:          // buffers [a, b, c], scalars [m, n, k, alpha]
        case kSgemmBiasReluF32:  // buffers [a, b, bias, c], same scalars
        {
            const bool fused = p.builtin == kSgemmBiasReluF32;
            if ((rc = bound_ptr(dev, op, 0, &b0)) || (rc = bound_ptr(dev, op, 1, &b1)) ||
                (rc = bound_ptr(dev, op, 2, &b2)) ||
                (fused && (rc = bound_ptr(dev, op, 3, &b3))) || (rc = scalar_u32(op, 0, &m)) ||
                (rc = scalar_u32(op, 1, &n)) || (rc = scalar_u32(op, 2, &k)) ||
                (rc = scalar_f32(op, 3, &alpha)))
                return rc;
            int mode = mode_override >= 0 ? mode_override
                                          : (p.gemm_mode >= 0 ? p.gemm_mode : default_gemm_mode());
            if (m > 0x7fffffffu || n > 0x7fffffffu || k > 0x7fffffffu)
                return set_error(ZG_ERR_DISPATCH, "sgemm: dimension exceeds 2^31-1");
            const uint64_t ws = zg_sgemm_workspace_bytes(mode, m, n, k);
            if ((rc = ensure_workspace(dev, ws))) return rc;
            float* c = static_cast<float*>(fused ? b3 : b2);
            const float* bias = fused ? static_cast<float*>(b2) : nullptr;
            return zg_sgemm_f32(mode, m, n, k, alpha, static_cast<float*>(b0),
                                static_cast<float*>(b1), c, bias, fused ? 1 : 0, dev->workspace,
                                dev->workspace_bytes, dev->stream);
        }
        default:
            return set_error(ZG_ERR_DISPATCH, "dispatch: pipeline has no builtin kernel");
    }
}

// Launches a module kernel: params are 8-byte slots, buffer pointers then
// scalars in their low 4 bytes (zengpu-cuda/src/lib.rs:885-940).
int launch_module(zg_device* dev, const Pipeline& p, const zg_dispatch_op* op) {
    const uint32_t nparams = op->num_buffers + op->num_scalars;
    if (nparams > 32)
        return set_error(ZG_ERR_BINDING_MISMATCH, "dispatch: %u params exceed the 32-slot limit",
                         nparams);
    uint64_t slots[32] = {0};
    void* args[32];
    for (uint32_t i = 0; i < op->num_buffers; ++i) {
        void* ptr = nullptr;
        int rc = bound_ptr(dev, op, i, &ptr);
        if (rc) return rc;
        slots[i] = reinterpret_cast<uint64_t>(ptr);
    }
    for (uint32_t j = 0; j < op->num_scalars; ++j) slots[op->num_buffers + j] = op->scalars[j].bits;
    for (uint32_t i = 0; i < nparams; ++i) args[i] = &slots[i];
    const Driver& d = driver();
    if (!d.ok) return set_error(ZG_ERR_BACKEND, "cuda: driver entry points unavailable");
    return cu_status(d.launchKernel(p.fn, op->grid[0], op->grid[1], op->grid[2], p.block[0],
                                    p.block[1], p.block[2], p.smem,
                                    reinterpret_cast<CUstream>(dev->stream), args, nullptr),
                     "cuLaunchKernel");
}

int launch_op(zg_device* dev, const zg_dispatch_op* op, int mode_override) {
    if (!op) return set_error(ZG_ERR_DISPATCH, "dispatch: null op");
    Pipeline* p = dev->pipelines.get(op->pipeline);
    if (!p) return set_error(ZG_ERR_DISPATCH, "stale pipeline handle");
    if ((op->num_buffers && !op->buffers) || (op->num_scalars && !op->scalars))
        return set_error(ZG_ERR_BINDING_MISMATCH, "dispatch: null binding array");
    return p->builtin != kNotBuiltin ? launch_builtin(dev, *p, op, mode_override)
                                     : launch_module(dev, *p, op);
}

// Waits for the device stream and surfaces device-side wait expiries.
int finish_sync(zg_device* dev, bool check_status) {
    int rc = cuda_status(cudaStreamSynchronize(dev->stream), "synchronize");
    if (rc) return rc;
    if (check_status || dev->status_unchecked) {
        dev->status_unchecked = false;
        uint32_t code = 0;
        if ((rc = zg_kernel_status(&code))) return rc;
        if (code)
            return set_error(ZG_ERR_KERNEL_WAIT,
                             "kernel bounded wait expired (status 0x%x); results are invalid",
                             code);
    }
    return ZG_OK;
}

bool is_gemm_pipeline(zg_device* dev, zg_handle pipeline) {
    Pipeline* p = dev->pipelines.get(pipeline);
    return p && (p->builtin == kSgemmF32 || p->builtin == kSgemmBiasReluF32);
}

int dispatch_sync(zg_device* dev, const zg_dispatch_op* op, int mode_override) {
    int rc = launch_op(dev, op, mode_override);
    if (rc) {
        cudaStreamSynchronize(dev->stream);
        return rc;
    }
    return finish_sync(dev, is_gemm_pipeline(dev, op->pipeline));
}

// Queues the op on the device stream and returns without waiting: for ops
// whose output is a GpuOnly array, which the host can only observe through
// stream-ordered calls (copy, readback submission, synchronous write / read
// of other buffers), so the reference's per-dispatch wait buys nothing.  Host
// errors and launch errors are still returned here; a bounded on-device wait
// that expires is reported by the next readback submission.
int dispatch_deferred(zg_device* dev, const zg_dispatch_op* op, int mode_override) {
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    int rc = set_device(dev);
    if (rc) return rc;
    if ((rc = launch_op(dev, op, mode_override))) {
        cudaStreamSynchronize(dev->stream);
        return rc;
    }
    if (is_gemm_pipeline(dev, op->pipeline)) dev->status_unchecked = true;
    return ZG_OK;
}

// The residency of a live buffer (ZG_MEMORY_UPLOAD when the handle is stale;
// the op that uses it reports the stale handle).
uint32_t buffer_memory(zg_device* dev, zg_handle h) {
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    Buffer* b = dev->buffers.get(h);
    return b ? b->memory : ZG_MEMORY_UPLOAD;
}

}  // namespace
}  // namespace zg

// ======================================================================
// 1. Device runtime
// ======================================================================

extern "C" const char* zg_last_error(void) { return g_last_error.c_str(); }
extern "C" int zg_last_error_detail(zg_error_detail* out) {
    if (!out) return ZG_ERR_BACKEND;
    *out = g_detail;
    if (!out->resource) out->resource = "";
    if (!out->needed) out->needed = "";
    return ZG_OK;
}
extern "C" int zg_abi_version(void) { return ZG_ABI_VERSION; }

extern "C" int zg_device_count(int* count) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (count) *count = (e == cudaSuccess) ? n : 0;
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(ZG_ERR_NO_DEVICE, "cuda: no device (%s)", cudaGetErrorString(e));
    }
    return ZG_OK;
}

extern "C" int zg_device_open(int ordinal, zg_device** out) {
    if (!out) return set_error(ZG_ERR_BACKEND, "zg_device_open: null out");
    *out = nullptr;
    int n = 0;
    int rc = zg_device_count(&n);
    if (rc) return rc;
    if (ordinal < 0 || ordinal >= n)
        return set_error(ZG_ERR_BACKEND, "cuda: invalid device ordinal %d (%d devices)", ordinal, n);
    if ((rc = cuda_status(cudaSetDevice(ordinal), "cudaSetDevice"))) return rc;
    if ((rc = cuda_status(cudaFree(nullptr), "context init"))) return rc;
    auto* dev = new zg_device();
    dev->ordinal = ordinal;
    if ((rc = cuda_status(cudaStreamCreateWithFlags(&dev->stream, cudaStreamNonBlocking),
                          "stream create"))) {
        delete dev;
        return rc;
    }
    *out = dev;
    return ZG_OK;
}

extern "C" void zg_device_close(zg_device* dev) {
    if (!dev) return;
    {
        std::lock_guard<std::recursive_mutex> lk(dev->mu);
        cudaSetDevice(dev->ordinal);
        cudaStreamSynchronize(dev->stream);
        for (cudaEvent_t e : dev->pending) cudaEventDestroy(e);
        dev->pending.clear();
        dev->buffers.for_each_occupied([](uint32_t, Buffer& b) {
            if (b.ptr) cudaFree(b.ptr);
        });
        const Driver& d = driver();
        dev->shaders.for_each_occupied([&](uint32_t, Shader& s) {
            if (s.module && d.ok) d.moduleUnload(s.module);
        });
        if (dev->workspace) cudaFree(dev->workspace);
        if (dev->staging) cudaFree(dev->staging);
        if (dev->h2d) cudaStreamDestroy(dev->h2d);
        if (dev->d2h) cudaStreamDestroy(dev->d2h);
        cudaStreamDestroy(dev->stream);
    }
    delete dev;
}

extern "C" int zg_device_ordinal(const zg_device* dev) { return dev ? dev->ordinal : -1; }
extern "C" void* zg_device_stream(zg_device* dev) { return dev ? dev->stream : nullptr; }

// GpuDevice::can_peer as the HIP backend implements it (zengpu-hip/src/lib.rs:
// 613-631): true once this device can access the peer's memory, enabling that
// access on first use; the answer is cached per peer.
bool peer_usable(zg_device* dev, int peer_ordinal) {
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    if (peer_ordinal == dev->ordinal) return true;
    auto it = dev->peer_access.find(peer_ordinal);
    if (it != dev->peer_access.end()) return it->second;
    int can = 0;
    bool usable = cudaDeviceCanAccessPeer(&can, dev->ordinal, peer_ordinal) == cudaSuccess && can &&
                  cudaSetDevice(dev->ordinal) == cudaSuccess;
    if (usable) {
        const cudaError_t e = cudaDeviceEnablePeerAccess(peer_ordinal, 0);
        usable = e == cudaSuccess || e == cudaErrorPeerAccessAlreadyEnabled;
    }
    cudaGetLastError();  // a refused query or an already-enabled peer is not an error
    dev->peer_access[peer_ordinal] = usable;
    return usable;
}

extern "C" int zg_device_can_peer(zg_device* dev, int peer_ordinal, int* out) {
    if (!dev || !out) return set_error(ZG_ERR_BACKEND, "zg_device_can_peer: null argument");
    *out = peer_usable(dev, peer_ordinal) ? 1 : 0;
    return ZG_OK;
}

extern "C" int zg_buffer_create(zg_device* dev, uint64_t size, uint32_t usage, uint32_t memory,
                                zg_handle* out) {
    if (!dev || !out) return set_error(ZG_ERR_BACKEND, "zg_buffer_create: null argument");
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    int rc = set_device(dev);
    if (rc) return rc;
    Buffer b;
    b.len = size;
    b.usage = usage;
    b.memory = memory;
    if (size > 0) {
        cudaError_t e = cudaMalloc(&b.ptr, size);
        if (e != cudaSuccess) {
            cudaGetLastError();
            if (e == cudaErrorMemoryAllocation) {
                set_error(ZG_ERR_OUT_OF_MEMORY, "out of memory allocating %llu bytes",
                          (unsigned long long)size);
                g_detail.memory = memory;
                return ZG_ERR_OUT_OF_MEMORY;
            }
            return cuda_status(e, "cudaMalloc");
        }
    }
    *out = dev->buffers.insert(b);
    return ZG_OK;
}

extern "C" int zg_buffer_info(zg_device* dev, zg_handle h, uint64_t* device_ptr, uint64_t* size) {
    if (!dev) return set_error(ZG_ERR_BACKEND, "zg_buffer_info: null device");
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    Buffer* b = dev->buffers.get(h);
    if (!b) return stale("buffer", h, dev->buffers.current_gen(h.index));
    if (device_ptr) *device_ptr = reinterpret_cast<uint64_t>(b->ptr);
    if (size) *size = b->len;
    return ZG_OK;
}

extern "C" int zg_buffer_write(zg_device* dev, zg_handle h, uint64_t offset, const void* data,
                               uint64_t len) {
    if (!dev) return set_error(ZG_ERR_BACKEND, "zg_buffer_write: null device");
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    Buffer* b = dev->buffers.get(h);
    if (!b) return stale("write_buffer", h, dev->buffers.current_gen(h.index));
    if (in_flight(dev))
        return set_error(ZG_ERR_BINDING_MISMATCH,
                         "write_buffer cannot mutate buffers while an asynchronous submission "
                         "is pending");
    if (offset > b->len || len > b->len - offset)
        return set_error(ZG_ERR_BACKEND, "cuda: write out of bounds");
    if (len == 0) return ZG_OK;
    if (!data) return set_error(ZG_ERR_BACKEND, "write_buffer: null data");
    int rc = set_device(dev);
    if (rc) return rc;
    rc = cuda_status(cudaMemcpyAsync(static_cast<uint8_t*>(b->ptr) + offset, data, len,
                                     cudaMemcpyHostToDevice, dev->stream),
                     "write_buffer");
    if (rc) return rc;
    return cuda_status(cudaStreamSynchronize(dev->stream), "write_buffer sync");
}

extern "C" int zg_buffer_read(zg_device* dev, zg_handle h, uint64_t offset, void* dst,
                              uint64_t len) {
    if (!dev) return set_error(ZG_ERR_BACKEND, "zg_buffer_read: null device");
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    Buffer* b = dev->buffers.get(h);
    if (!b) return stale("read_buffer", h, dev->buffers.current_gen(h.index));
    if (!(b->usage & ZG_USAGE_READBACK))
        return missing_usage("buffer", "READBACK", "buffer needs READBACK usage");
    if (in_flight(dev))
        return set_error(ZG_ERR_BINDING_MISMATCH,
                         "read_buffer_into cannot observe buffers while an asynchronous "
                         "submission is pending");
    if (offset > b->len || len > b->len - offset)
        return set_error(ZG_ERR_BINDING_MISMATCH, "cuda: read range %llu..%llu exceeds %llu",
                         (unsigned long long)offset, (unsigned long long)(offset + len),
                         (unsigned long long)b->len);
    if (len == 0) return ZG_OK;
    if (!dst) return set_error(ZG_ERR_BACKEND, "read_buffer: null destination");
    int rc = set_device(dev);
    if (rc) return rc;
    rc = cuda_status(cudaMemcpyAsync(dst, static_cast<uint8_t*>(b->ptr) + offset, len,
                                     cudaMemcpyDeviceToHost, dev->stream),
                     "read_buffer");
    if (rc) return rc;
    return cuda_status(cudaStreamSynchronize(dev->stream), "read_buffer sync");
}

extern "C" int zg_buffer_read_async(zg_device* dev, zg_handle h, uint64_t offset, void* dst,
                                    uint64_t len, zg_submission** out) {
    if (!dev || !out) return set_error(ZG_ERR_BACKEND, "zg_buffer_read_async: null argument");
    *out = nullptr;
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    Buffer* b = dev->buffers.get(h);
    if (!b) return stale("read_buffer_async", h, dev->buffers.current_gen(h.index));
    if (!(b->usage & (ZG_USAGE_READBACK | ZG_USAGE_TRANSFER_SRC)))
        return missing_usage("buffer", "READBACK", "buffer needs READBACK or TRANSFER_SRC usage");
    if (offset > b->len || len > b->len - offset)
        return set_error(ZG_ERR_BINDING_MISMATCH, "cuda: read range %llu..%llu exceeds %llu",
                         (unsigned long long)offset, (unsigned long long)(offset + len),
                         (unsigned long long)b->len);
    if (len && !dst) return set_error(ZG_ERR_BACKEND, "read_buffer_async: null destination");
    int rc = set_device(dev);
    if (rc) return rc;
    if (len)
        rc = cuda_status(cudaMemcpyAsync(dst, static_cast<uint8_t*>(b->ptr) + offset, len,
                                         cudaMemcpyDeviceToHost, dev->stream),
                         "read_buffer_async");
    if (rc) return rc;
    cudaEvent_t ev;
    if ((rc = cuda_status(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "event create")))
        return rc;
    if ((rc = cuda_status(cudaEventRecord(ev, dev->stream), "event record"))) {
        cudaEventDestroy(ev);
        return rc;
    }
    dev->pending.push_back(ev);
    auto* sub = new zg_submission();
    sub->dev = dev;
    sub->event = ev;
    sub->check_status = dev->status_unchecked;
    dev->status_unchecked = false;
    *out = sub;
    return ZG_OK;
}

extern "C" int zg_buffer_copy(zg_device* dev, zg_handle src, uint64_t src_offset, zg_handle dst,
                              uint64_t dst_offset, uint64_t len) {
    if (!dev) return set_error(ZG_ERR_BACKEND, "zg_buffer_copy: null device");
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    if (in_flight(dev))
        return set_error(ZG_ERR_BINDING_MISMATCH,
                         "copy_buffer cannot run while an asynchronous submission is pending");
    Buffer* s = dev->buffers.get(src);
    if (!s) return set_error(ZG_ERR_BACKEND, "cuda: invalid source buffer handle");
    Buffer* d = dev->buffers.get(dst);
    if (!d) return set_error(ZG_ERR_BACKEND, "cuda: invalid destination buffer handle");
    if (!(s->usage & ZG_USAGE_TRANSFER_SRC))
        return missing_usage("source buffer", "TRANSFER_SRC",
                             "source buffer needs TRANSFER_SRC usage");
    if (!(d->usage & ZG_USAGE_TRANSFER_DST))
        return missing_usage("destination buffer", "TRANSFER_DST",
                             "destination buffer needs TRANSFER_DST usage");
    if (src.index == dst.index)
        return set_error(ZG_ERR_BINDING_MISMATCH,
                         "copy_buffer requires distinct source and destination buffers");
    if (src_offset > UINT64_MAX - len)
        return set_error(ZG_ERR_BINDING_MISMATCH, "source copy range overflows u64");
    if (dst_offset > UINT64_MAX - len)
        return set_error(ZG_ERR_BINDING_MISMATCH, "destination copy range overflows u64");
    if (src_offset + len > s->len || dst_offset + len > d->len)
        return set_error(ZG_ERR_BINDING_MISMATCH, "copy ranges src %llu..%llu/%llu dst %llu..%llu/%llu",
                         (unsigned long long)src_offset, (unsigned long long)(src_offset + len),
                         (unsigned long long)s->len, (unsigned long long)dst_offset,
                         (unsigned long long)(dst_offset + len), (unsigned long long)d->len);
    if (len == 0) return ZG_OK;
    int rc = set_device(dev);
    if (rc) return rc;
    rc = cuda_status(cudaMemcpyAsync(static_cast<uint8_t*>(d->ptr) + dst_offset,
                                     static_cast<uint8_t*>(s->ptr) + src_offset, len,
                                     cudaMemcpyDeviceToDevice, dev->stream),
                     "copy_buffer");
    if (rc) return rc;
    return cuda_status(cudaStreamSynchronize(dev->stream), "copy_buffer sync");
}

extern "C" void zg_buffer_destroy(zg_device* dev, zg_handle h) {
    if (!dev) return;
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    Buffer b;
    if (in_flight(dev)) {
        if (dev->buffers.retire(h, &b)) dev->deferred_buffers.push_back(h.index);
        return;
    }
    if (dev->buffers.remove(h, &b) && b.ptr) {
        cudaSetDevice(dev->ordinal);
        // ops queued without a synchronize (GpuOnly outputs) may still read it
        cudaStreamSynchronize(dev->stream);
        cudaFree(b.ptr);
    }
}

// GpuDevice::copy_from_peer (zengpu-hal/src/device.rs:96-106), as the HIP
// backend does it (zengpu-hip/src/lib.rs:633-710): a direct peer copy over
// NVLink when can_peer holds, else staged through host memory; synchronous.
extern "C" int zg_buffer_copy_from_peer(zg_device* dst_dev, zg_handle dst, zg_device* src_dev,
                                        zg_handle src, uint64_t bytes) {
    if (!dst_dev || !src_dev) return set_error(ZG_ERR_BACKEND, "copy_from_peer: null device");
    void *dptr = nullptr, *sptr = nullptr;
    uint64_t dlen = 0, slen = 0;
    {
        std::lock_guard<std::recursive_mutex> lk(dst_dev->mu);
        Buffer* d = dst_dev->buffers.get(dst);
        if (!d) return stale("copy_from_peer destination", dst, dst_dev->buffers.current_gen(dst.index));
        if (in_flight(dst_dev))
            return set_error(ZG_ERR_BINDING_MISMATCH,
                             "copy_from_peer cannot run while a submission is pending");
        dptr = d->ptr;
        dlen = d->len;
    }
    {
        std::lock_guard<std::recursive_mutex> lk(src_dev->mu);
        Buffer* s = src_dev->buffers.get(src);
        if (!s) return stale("copy_from_peer source", src, src_dev->buffers.current_gen(src.index));
        if (in_flight(src_dev))
            return set_error(ZG_ERR_BINDING_MISMATCH,
                             "copy_from_peer cannot run while the source device has pending work");
        sptr = s->ptr;
        slen = s->len;
        // work queued on the source device without a synchronize (GpuOnly
        // outputs) completes before its buffer is read
        cudaSetDevice(src_dev->ordinal);
        int rc = cuda_status(cudaStreamSynchronize(src_dev->stream), "copy_from_peer source sync");
        if (rc) return rc;
    }
    if (bytes > slen || bytes > dlen)
        return set_error(ZG_ERR_BACKEND,
                         "cuda: peer copy of %llu bytes exceeds source (%llu) or destination (%llu) "
                         "buffer",
                         (unsigned long long)bytes, (unsigned long long)slen,
                         (unsigned long long)dlen);
    if (bytes == 0) return ZG_OK;
    std::lock_guard<std::recursive_mutex> lk(dst_dev->mu);
    int rc;
    if (peer_usable(dst_dev, src_dev->ordinal)) {
        if ((rc = set_device(dst_dev))) return rc;
        rc = cuda_status(cudaMemcpyPeerAsync(dptr, dst_dev->ordinal, sptr, src_dev->ordinal, bytes,
                                             dst_dev->stream),
                         "cudaMemcpyPeerAsync");
        if (rc) return rc;
        return cuda_status(cudaStreamSynchronize(dst_dev->stream), "copy_from_peer sync");
    }
    std::vector<uint8_t> staging(bytes);
    if ((rc = cuda_status(cudaSetDevice(src_dev->ordinal), "cudaSetDevice peer source")) ||
        (rc = cuda_status(cudaMemcpy(staging.data(), sptr, bytes, cudaMemcpyDeviceToHost),
                          "peer copy staging D2H")))
        return rc;
    if ((rc = set_device(dst_dev))) return rc;
    rc = cuda_status(cudaMemcpyAsync(dptr, staging.data(), bytes, cudaMemcpyHostToDevice,
                                     dst_dev->stream),
                     "peer copy staging H2D");
    if (rc) return rc;
    return cuda_status(cudaStreamSynchronize(dst_dev->stream), "copy_from_peer sync");
}

extern "C" int zg_shader_create(zg_device* dev, uint32_t kind, const void* code, uint64_t len,
                                zg_handle* out) {
    if (!dev || !out) return set_error(ZG_ERR_BACKEND, "zg_shader_create: null argument");
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    Shader s;
    s.kind = kind;
    if (kind == ZG_SHADER_BUILTIN) {
        *out = dev->shaders.insert(s);
        return ZG_OK;
    }
    if (kind != ZG_SHADER_CUBIN && kind != ZG_SHADER_PTX)
        return set_error(ZG_ERR_SHADER_COMPILE,
                         "cuda backend accepts only cubin, PTX or builtin shaders");
    if (!code || len == 0) return set_error(ZG_ERR_SHADER_COMPILE, "empty shader code");
    const Driver& d = driver();
    if (!d.ok) return set_error(ZG_ERR_BACKEND, "cuda: driver entry points unavailable");
    int rc = set_device(dev);
    if (rc) return rc;
    std::vector<uint8_t> image;
    const void* img = code;
    if (kind == ZG_SHADER_PTX) {  // the driver wants NUL-terminated text
        image.assign(static_cast<const uint8_t*>(code), static_cast<const uint8_t*>(code) + len);
        if (image.back() != 0) image.push_back(0);
        img = image.data();
    }
    if ((rc = cu_status(d.moduleLoadData(&s.module, img), "cuModuleLoadData")) != ZG_OK) {
        if (rc == ZG_ERR_BACKEND) g_last_error = "cuda: PTX/module error: " + g_last_error;
        return rc == ZG_ERR_BACKEND ? set_error(ZG_ERR_SHADER_COMPILE, "%s", g_last_error.c_str())
                                    : rc;
    }
    *out = dev->shaders.insert(s);
    return ZG_OK;
}

extern "C" void zg_shader_destroy(zg_device* dev, zg_handle h) {
    if (!dev) return;
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    Shader s;
    if (dev->shaders.remove(h, &s) && s.module) {
        const Driver& d = driver();
        cudaSetDevice(dev->ordinal);
        if (d.ok) d.moduleUnload(s.module);
    }
}

extern "C" int zg_pipeline_create(zg_device* dev, zg_handle shader, const char* entry,
                                  const uint32_t block[3], uint32_t dynamic_smem, zg_handle* out) {
    if (!dev || !out || !entry)
        return set_error(ZG_ERR_PIPELINE_CREATION, "zg_pipeline_create: null argument");
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    Shader* s = dev->shaders.get(shader);
    if (!s) return set_error(ZG_ERR_PIPELINE_CREATION, "stale shader handle");
    Pipeline p;
    p.shader = shader;
    if (block && (block[0] | block[1] | block[2]) != 0) {
        p.block[0] = block[0] ? block[0] : 1;
        p.block[1] = block[1] ? block[1] : 1;
        p.block[2] = block[2] ? block[2] : 1;
    }
    p.smem = dynamic_smem;
    if (s->kind == ZG_SHADER_BUILTIN) {
        const std::string e(entry);
        struct {
            const char* name;
            int id;
            int mode;
        } table[] = {
            {"add_f32", kAddF32, -1},
            {"relu_f32", kReluF32, -1},
            {"saxpy_f32", kSaxpyF32, -1},
            {"sscal_f32", kSscalF32, -1},
            {"sgemm_f32", kSgemmF32, -1},
            {"sgemm_f32.simt", kSgemmF32, ZG_GEMM_SIMT_FP32},
            {"sgemm_f32.tf32x3", kSgemmF32, ZG_GEMM_TF32X3},
            {"sgemm_f32.tf32", kSgemmF32, ZG_GEMM_TF32},
            {"sgemm_f32.tf32bf16", kSgemmF32, ZG_GEMM_TF32_BF16X2},
            {"sgemm_f32.bf16x3", kSgemmF32, ZG_GEMM_BF16X3},
            {"sgemm_bias_relu_f32", kSgemmBiasReluF32, -1},
        };
        for (auto& t : table)
            if (e == t.name) {
                p.builtin = t.id;
                p.gemm_mode = t.mode;
                *out = dev->pipelines.insert(p);
                return ZG_OK;
            }
        return set_error(ZG_ERR_PIPELINE_CREATION, "no builtin kernel named '%s'", entry);
    }
    const Driver& d = driver();
    if (!d.ok) return set_error(ZG_ERR_BACKEND, "cuda: driver entry points unavailable");
    int rc = set_device(dev);
    if (rc) return rc;
    if ((rc = cu_status(d.moduleGetFunction(&p.fn, s->module, entry), "cuModuleGetFunction")))
        return set_error(ZG_ERR_PIPELINE_CREATION, "entry '%s' not found in module", entry);
    if (dynamic_smem > 48 * 1024 &&
        (rc = cu_status(d.funcSetAttribute(p.fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                           static_cast<int>(dynamic_smem)),
                        "cuFuncSetAttribute")))
        return set_error(ZG_ERR_PIPELINE_CREATION, "%s", g_last_error.c_str());
    *out = dev->pipelines.insert(p);
    return ZG_OK;
}

extern "C" void zg_pipeline_destroy(zg_device* dev, zg_handle h) {
    if (!dev) return;
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    Pipeline p;
    dev->pipelines.remove(h, &p);
}

extern "C" int zg_dispatch(zg_device* dev, const zg_dispatch_op* op) {
    if (!dev) return set_error(ZG_ERR_BACKEND, "zg_dispatch: null device");
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    int rc = set_device(dev);
    if (rc) return rc;
    return dispatch_sync(dev, op, -1);
}

extern "C" int zg_submit_batch(zg_device* dev, const zg_dispatch_op* ops, uint32_t count,
                               zg_submission** out) {
    if (!dev || !out || (count && !ops))
        return set_error(ZG_ERR_BACKEND, "zg_submit_batch: null argument");
    *out = nullptr;
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    int rc = set_device(dev);
    if (rc) return rc;
    for (uint32_t i = 0; i < count; ++i) {
        if ((rc = launch_op(dev, &ops[i], -1)) != ZG_OK) {
            // A failed launch after partial enqueue drains what was queued
            // (zengpu-cuda/src/lib.rs:968-982).
            cudaStreamSynchronize(dev->stream);
            return rc;
        }
    }
    cudaEvent_t ev;
    if ((rc = cuda_status(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "event create")))
        return rc;
    if ((rc = cuda_status(cudaEventRecord(ev, dev->stream), "event record"))) {
        cudaEventDestroy(ev);
        return rc;
    }
    dev->pending.push_back(ev);
    auto* sub = new zg_submission();
    sub->dev = dev;
    sub->event = ev;
    sub->check_status = dev->status_unchecked;
    for (uint32_t i = 0; i < count; ++i)
        if (is_gemm_pipeline(dev, ops[i].pipeline)) sub->check_status = true;
    dev->status_unchecked = false;
    *out = sub;
    return ZG_OK;
}

extern "C" int zg_submission_poll(zg_submission* sub, int* done) {
    if (!sub || !done) return set_error(ZG_ERR_BACKEND, "zg_submission_poll: null argument");
    int status_rc = ZG_OK;
    if (!sub->done) {
        std::lock_guard<std::recursive_mutex> lk(sub->dev->mu);
        cudaSetDevice(sub->dev->ordinal);
        cudaError_t e = cudaEventQuery(sub->event);
        if (e == cudaSuccess) {
            sub->done = true;
            release_submission(sub->dev, sub->event);
            sub->event = nullptr;
            if (sub->check_status) {
                // GEMMs queued before this submission without a synchronize
                sub->check_status = false;
                uint32_t code = 0;
                status_rc = zg_kernel_status(&code);
                if (!status_rc && code)
                    status_rc = set_error(ZG_ERR_KERNEL_WAIT,
                                          "kernel bounded wait expired (status 0x%x); results of "
                                          "the work before this submission are invalid",
                                          code);
            }
        } else if (e == cudaErrorNotReady) {
            cudaGetLastError();
        } else {
            return cuda_status(e, "submission poll");
        }
    }
    *done = sub->done ? 1 : 0;
    return status_rc;
}

extern "C" int zg_submission_wait(zg_submission* sub, uint64_t timeout_ns) {
    if (!sub) return set_error(ZG_ERR_BACKEND, "zg_submission_wait: null submission");
    // Bounded poll (the reference busy-polls cuEventQuery + yield,
    // zengpu-cuda/src/lib.rs:378-391); Timeout leaves the work running.
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        int done = 0;
        int rc = zg_submission_poll(sub, &done);
        if (rc) return rc;
        if (done) return ZG_OK;
        const auto dt = std::chrono::duration_cast<std::chrono::nanoseconds>(
                            std::chrono::steady_clock::now() - t0)
                            .count();
        if (static_cast<uint64_t>(dt) >= timeout_ns)
            return set_error(ZG_ERR_TIMEOUT, "operation timed out");
        std::this_thread::yield();
    }
}

// Dropping a pending submission waits for its stream position first, then
// releases its in-flight token (the reference's Drop for CudaSubmission).
extern "C" void zg_submission_destroy(zg_submission* sub) {
    if (!sub) return;
    if (!sub->done && sub->event) {
        std::lock_guard<std::recursive_mutex> lk(sub->dev->mu);
        cudaSetDevice(sub->dev->ordinal);
        cudaEventSynchronize(sub->event);
        release_submission(sub->dev, sub->event);
    }
    delete sub;
}

// ======================================================================
// 2. Array ops
// ======================================================================

namespace zg {
namespace {

uint32_t dtype_size(uint32_t dt) {
    switch (dt) {
        case ZG_DTYPE_F64: case ZG_DTYPE_I64: case ZG_DTYPE_U64: return 8;
        case ZG_DTYPE_F32: case ZG_DTYPE_I32: case ZG_DTYPE_U32: return 4;
        case ZG_DTYPE_F16: case ZG_DTYPE_BF16: case ZG_DTYPE_I16: case ZG_DTYPE_U16: return 2;
        case ZG_DTYPE_I8: case ZG_DTYPE_U8: case ZG_DTYPE_BOOL: return 1;
        default: return 0;
    }
}

const char* dtype_name(uint32_t dt) {
    static const char* names[] = {"F32", "F16", "Bf16", "F64", "I8", "I16", "I32",
                                  "I64", "U8",  "U16",  "U32", "U64", "Bool"};
    return dt < 13 ? names[dt] : "?";
}

std::string shape_str(const zg_device_array* a) {
    std::string s = "[";
    for (uint32_t i = 0; i < a->rank; ++i) {
        if (i) s += ", ";
        s += std::to_string(a->shape[i]);
    }
    return s + "]";
}

bool same_shape(const zg_device_array* a, const zg_device_array* b) {
    if (a->rank != b->rank) return false;
    for (uint32_t i = 0; i < a->rank; ++i)
        if (a->shape[i] != b->shape[i]) return false;
    return true;
}

// Element count as the reference's u32 product; false on overflow.
bool array_len(const zg_device_array* a, uint32_t* out) {
    uint64_t n = 1;
    for (uint32_t i = 0; i < a->rank; ++i) {
        n *= a->shape[i];
        if (n > 0xffffffffull) return false;
    }
    *out = static_cast<uint32_t>(n);
    return true;
}

int check_f32(uint32_t dt, const char* op) {
    if (dt != ZG_DTYPE_F32)
        return set_error(ZG_ERR_DISPATCH, "%s: only DType::F32 is supported in this version, got %s",
                         op, dtype_name(dt));
    return ZG_OK;
}

int check_array(const zg_device_array* a, const char* op) {
    if (!a) return set_error(ZG_ERR_DISPATCH, "%s: null array", op);
    if (a->rank > ZG_MAX_RANK) return set_error(ZG_ERR_DISPATCH, "%s: rank above %d", op, ZG_MAX_RANK);
    return ZG_OK;
}

zg_dispatch_op make_op(zg_handle pipeline, const uint32_t* bufs, uint32_t nb,
                       const zg_scalar* sc, uint32_t ns, uint32_t gx, uint32_t gy) {
    zg_dispatch_op op;
    op.pipeline = pipeline;
    op.buffers = bufs;
    op.num_buffers = nb;
    op.scalars = sc;
    op.num_scalars = ns;
    op.grid[0] = gx;
    op.grid[1] = gy;
    op.grid[2] = 1;
    return op;
}

zg_scalar u32s(uint32_t v) { return zg_scalar{ZG_SCALAR_U32, v}; }
zg_scalar f32s(float v) {
    zg_scalar s{ZG_SCALAR_F32, 0};
    std::memcpy(&s.bits, &v, 4);
    return s;
}

int builtin_pipeline(zg_device* dev, zg_handle shader, const char* entry, uint32_t bx, uint32_t by,
                     zg_handle* out) {
    const uint32_t block[3] = {bx, by, 1};
    return zg_pipeline_create(dev, shader, entry, block, 0, out);
}

}  // namespace
}  // namespace zg

extern "C" uint64_t zg_size_class(uint64_t size) {
    const uint64_t kMin = 256;
    uint64_t s = size < 1 ? 1 : size;
    uint64_t p = 1;
    while (p < s) p <<= 1;
    return p < kMin ? kMin : p;
}

extern "C" int zg_pool_create(zg_device* dev, zg_pool** out) {
    return zg_pool_create_with(dev, ZG_MEMORY_UPLOAD, out);
}

extern "C" int zg_pool_create_with(zg_device* dev, uint32_t memory, zg_pool** out) {
    if (!dev || !out) return set_error(ZG_ERR_BACKEND, "zg_pool_create: null argument");
    if (memory != ZG_MEMORY_UPLOAD && memory != ZG_MEMORY_GPU_ONLY)
        return set_error(ZG_ERR_UNSUPPORTED, "BufferPool: memory usage %u (Upload or GpuOnly)",
                         memory);
    auto* p = new zg_pool();
    p->dev = dev;
    p->memory = memory;
    *out = p;
    return ZG_OK;
}

extern "C" uint32_t zg_pool_memory(const zg_pool* pool) {
    return pool ? pool->memory : ZG_MEMORY_UPLOAD;
}

extern "C" void zg_pool_destroy(zg_pool* pool) {
    if (!pool) return;
    {
        std::lock_guard<std::mutex> lk(pool->mu);
        for (auto& kv : pool->free)
            for (zg_handle h : kv.second) zg_buffer_destroy(pool->dev, h);
        pool->free.clear();
    }
    delete pool;
}

extern "C" int zg_pool_alloc(zg_pool* pool, const uint32_t* shape, uint32_t rank, uint32_t dtype,
                             zg_device_array* out) {
    if (!pool || !out || (rank && !shape))
        return set_error(ZG_ERR_DISPATCH, "pool alloc: null argument");
    if (rank > ZG_MAX_RANK) return set_error(ZG_ERR_DISPATCH, "pool alloc: rank above %d", ZG_MAX_RANK);
    const uint32_t es = dtype_size(dtype);
    if (!es) return set_error(ZG_ERR_DISPATCH, "pool alloc: unknown dtype %u", dtype);
    zg_device_array a;
    std::memset(&a, 0, sizeof(a));
    a.rank = rank;
    a.dtype = dtype;
    for (uint32_t i = 0; i < rank; ++i) a.shape[i] = shape[i];
    // contiguous_strides (zengpu-compute/src/lib.rs:79-85)
    if (rank) {
        a.stride[rank - 1] = 1;
        for (int i = static_cast<int>(rank) - 2; i >= 0; --i)
            a.stride[i] = a.stride[i + 1] * a.shape[i + 1];
    }
    uint32_t len = 0;
    if (!array_len(&a, &len))
        return set_error(ZG_ERR_DISPATCH, "pool alloc: element count of %s overflows u32",
                         shape_str(&a).c_str());
    const uint64_t cls = zg_size_class(static_cast<uint64_t>(len) * es);
    zg_handle h{0, 0};
    bool have = false;
    {
        std::lock_guard<std::mutex> lk(pool->mu);
        auto it = pool->free.find(cls);
        if (it != pool->free.end() && !it->second.empty()) {
            h = it->second.back();
            it->second.pop_back();
            have = true;
        }
    }
    if (!have) {
        // Upload (the reference's pool): host-readable STORAGE | READBACK.
        // GpuOnly: device resident, read back only through a copy or a
        // readback submission.
        const uint32_t usage = pool->memory == ZG_MEMORY_GPU_ONLY
                                   ? ZG_USAGE_STORAGE | ZG_USAGE_TRANSFER_SRC | ZG_USAGE_TRANSFER_DST
                                   : ZG_USAGE_STORAGE | ZG_USAGE_READBACK;
        int rc = zg_buffer_create(pool->dev, cls, usage, pool->memory, &h);
        if (rc) return rc;
    }
    a.buffer = h;
    a.allocation_size = cls;
    *out = a;
    return ZG_OK;
}

extern "C" void zg_pool_free(zg_pool* pool, const zg_device_array* array) {
    if (!pool || !array) return;
    std::lock_guard<std::mutex> lk(pool->mu);
    pool->free[array->allocation_size].push_back(array->buffer);
}

extern "C" uint32_t zg_pool_free_count(zg_pool* pool, uint64_t size_class) {
    if (!pool) return 0;
    std::lock_guard<std::mutex> lk(pool->mu);
    auto it = pool->free.find(size_class);
    return it == pool->free.end() ? 0u : static_cast<uint32_t>(it->second.size());
}

extern "C" int zg_elementwise_new(zg_device* dev, zg_elementwise_kernels* out) {
    if (!dev || !out) return set_error(ZG_ERR_BACKEND, "zg_elementwise_new: null argument");
    std::memset(out, 0, sizeof(*out));
    int rc;
    if ((rc = zg_shader_create(dev, ZG_SHADER_BUILTIN, nullptr, 0, &out->add_shader))) return rc;
    if ((rc = builtin_pipeline(dev, out->add_shader, "add_f32", 256, 1, &out->add_pipeline)))
        return rc;
    if ((rc = zg_shader_create(dev, ZG_SHADER_BUILTIN, nullptr, 0, &out->relu_shader))) return rc;
    return builtin_pipeline(dev, out->relu_shader, "relu_f32", 256, 1, &out->relu_pipeline);
}

extern "C" void zg_elementwise_destroy(zg_device* dev, const zg_elementwise_kernels* k) {
    if (!dev || !k) return;
    zg_pipeline_destroy(dev, k->add_pipeline);
    zg_shader_destroy(dev, k->add_shader);
    zg_pipeline_destroy(dev, k->relu_pipeline);
    zg_shader_destroy(dev, k->relu_shader);
}

extern "C" int zg_elementwise_add(const zg_elementwise_kernels* k, zg_device* dev, zg_pool* pool,
                                  const zg_device_array* a, const zg_device_array* b,
                                  zg_device_array* out) {
    int rc;
    if (!k || !dev || !pool || !out) return set_error(ZG_ERR_DISPATCH, "elementwise::add: null argument");
    if ((rc = check_array(a, "elementwise::add")) || (rc = check_array(b, "elementwise::add")))
        return rc;
    if ((rc = check_f32(a->dtype, "elementwise::add")) || (rc = check_f32(b->dtype, "elementwise::add")))
        return rc;
    if (!same_shape(a, b))
        return set_error(ZG_ERR_DISPATCH, "elementwise::add: shape mismatch %s vs %s",
                         shape_str(a).c_str(), shape_str(b).c_str());
    if ((rc = zg_pool_alloc(pool, a->shape, a->rank, ZG_DTYPE_F32, out))) return rc;
    uint32_t n = 0;
    array_len(a, &n);
    const uint32_t bufs[3] = {a->buffer.index, b->buffer.index, out->buffer.index};
    const zg_scalar sc[1] = {u32s(n)};
    zg_dispatch_op op = make_op(k->add_pipeline, bufs, 3, sc, 1, (n + 255) / 256, 1);
    return pool->memory == ZG_MEMORY_GPU_ONLY ? dispatch_deferred(dev, &op, -1)
                                              : zg_dispatch(dev, &op);
}

extern "C" int zg_elementwise_relu(const zg_elementwise_kernels* k, zg_device* dev, zg_pool* pool,
                                   const zg_device_array* a, zg_device_array* out) {
    int rc;
    if (!k || !dev || !pool || !out) return set_error(ZG_ERR_DISPATCH, "elementwise::relu: null argument");
    if ((rc = check_array(a, "elementwise::relu")) || (rc = check_f32(a->dtype, "elementwise::relu")))
        return rc;
    if ((rc = zg_pool_alloc(pool, a->shape, a->rank, ZG_DTYPE_F32, out))) return rc;
    uint32_t n = 0;
    array_len(a, &n);
    const uint32_t bufs[2] = {a->buffer.index, out->buffer.index};
    const zg_scalar sc[1] = {u32s(n)};
    zg_dispatch_op op = make_op(k->relu_pipeline, bufs, 2, sc, 1, (n + 255) / 256, 1);
    return pool->memory == ZG_MEMORY_GPU_ONLY ? dispatch_deferred(dev, &op, -1)
                                              : zg_dispatch(dev, &op);
}

extern "C" int zg_elementwise_relu_inplace(const zg_elementwise_kernels* k, zg_device* dev,
                                           const zg_device_array* a) {
    int rc;
    if (!k || !dev) return set_error(ZG_ERR_DISPATCH, "elementwise::relu: null argument");
    if ((rc = check_array(a, "elementwise::relu")) || (rc = check_f32(a->dtype, "elementwise::relu")))
        return rc;
    uint32_t n = 0;
    if (!array_len(a, &n)) return set_error(ZG_ERR_DISPATCH, "elementwise::relu: length overflows u32");
    const uint32_t bufs[2] = {a->buffer.index, a->buffer.index};
    const zg_scalar sc[1] = {u32s(n)};
    zg_dispatch_op op = make_op(k->relu_pipeline, bufs, 2, sc, 1, (n + 255) / 256, 1);
    return buffer_memory(dev, a->buffer) == ZG_MEMORY_GPU_ONLY ? dispatch_deferred(dev, &op, -1)
                                                               : zg_dispatch(dev, &op);
}

extern "C" int zg_gemm_new(zg_device* dev, zg_gemm_kernel* out) {
    if (!dev || !out) return set_error(ZG_ERR_BACKEND, "zg_gemm_new: null argument");
    std::memset(out, 0, sizeof(*out));
    int rc;
    if ((rc = zg_shader_create(dev, ZG_SHADER_BUILTIN, nullptr, 0, &out->shader))) return rc;
    if ((rc = builtin_pipeline(dev, out->shader, "sgemm_f32", 16, 16, &out->pipeline))) return rc;
    if ((rc = builtin_pipeline(dev, out->shader, "sgemm_bias_relu_f32", 16, 16, &out->fused_pipeline)))
        return rc;
    out->mode = default_gemm_mode();
    return ZG_OK;
}

extern "C" void zg_gemm_destroy(zg_device* dev, const zg_gemm_kernel* k) {
    if (!dev || !k) return;
    zg_pipeline_destroy(dev, k->pipeline);
    zg_pipeline_destroy(dev, k->fused_pipeline);
    zg_shader_destroy(dev, k->shader);
}

namespace zg {
namespace {
// Validation of zengpu-blas/src/level3.rs:137-153.
int gemm_shapes(const zg_device_array* a, const zg_device_array* b, uint32_t* m, uint32_t* n,
                uint32_t* k) {
    int rc;
    if ((rc = check_array(a, "sgemm")) || (rc = check_array(b, "sgemm"))) return rc;
    if (a->dtype != ZG_DTYPE_F32 || b->dtype != ZG_DTYPE_F32)
        return set_error(ZG_ERR_DISPATCH, "sgemm: only f32 is supported, got %s and %s",
                         dtype_name(a->dtype), dtype_name(b->dtype));
    if (a->rank != 2 || b->rank != 2)
        return set_error(ZG_ERR_DISPATCH, "sgemm: expected 2D arrays, got shapes %s and %s",
                         shape_str(a).c_str(), shape_str(b).c_str());
    if (a->shape[1] != b->shape[0])
        return set_error(ZG_ERR_DISPATCH, "sgemm: inner dimensions mismatch (%u vs %u)", a->shape[1],
                         b->shape[0]);
    *m = a->shape[0];
    *k = a->shape[1];
    *n = b->shape[1];
    return ZG_OK;
}

int gemm_dispatch(const zg_gemm_kernel* kern, zg_device* dev, zg_pool* pool, float alpha,
                  const zg_device_array* a, const zg_device_array* b, const zg_device_array* bias,
                  zg_device_array* out) {
    if (!kern || !dev || !pool || !out) return set_error(ZG_ERR_DISPATCH, "sgemm: null argument");
    uint32_t m = 0, n = 0, k = 0;
    int rc = gemm_shapes(a, b, &m, &n, &k);
    if (rc) return rc;
    if (bias) {
        if ((rc = check_array(bias, "gemm_bias_relu"))) return rc;
        if (bias->dtype != ZG_DTYPE_F32)
            return set_error(ZG_ERR_DISPATCH, "gemm_bias_relu: bias must be f32, got %s",
                             dtype_name(bias->dtype));
        if (bias->rank != 1 || bias->shape[0] != n)
            return set_error(ZG_ERR_DISPATCH, "gemm_bias_relu: bias shape %s, expected [%u]",
                             shape_str(bias).c_str(), n);
    }
    const uint32_t shape[2] = {m, n};
    if ((rc = zg_pool_alloc(pool, shape, 2, ZG_DTYPE_F32, out))) return rc;
    const zg_scalar sc[4] = {u32s(m), u32s(n), u32s(k), f32s(alpha)};
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    if ((rc = set_device(dev))) return rc;
    const bool deferred = pool->memory == ZG_MEMORY_GPU_ONLY;
    if (bias) {
        const uint32_t bufs[4] = {a->buffer.index, b->buffer.index, bias->buffer.index,
                                  out->buffer.index};
        zg_dispatch_op op = make_op(kern->fused_pipeline, bufs, 4, sc, 4, (n + 15) / 16, (m + 15) / 16);
        return deferred ? dispatch_deferred(dev, &op, kern->mode)
                        : dispatch_sync(dev, &op, kern->mode);
    }
    const uint32_t bufs[3] = {a->buffer.index, b->buffer.index, out->buffer.index};
    zg_dispatch_op op = make_op(kern->pipeline, bufs, 3, sc, 4, (n + 15) / 16, (m + 15) / 16);
    return deferred ? dispatch_deferred(dev, &op, kern->mode) : dispatch_sync(dev, &op, kern->mode);
}
}  // namespace
}  // namespace zg

extern "C" int zg_gemm_sgemm(const zg_gemm_kernel* k, zg_device* dev, zg_pool* pool, float alpha,
                             const zg_device_array* a, const zg_device_array* b,
                             zg_device_array* out) {
    return gemm_dispatch(k, dev, pool, alpha, a, b, nullptr, out);
}

extern "C" int zg_gemm_gemm(const zg_gemm_kernel* k, zg_device* dev, zg_pool* pool,
                            const zg_device_array* a, const zg_device_array* b,
                            zg_device_array* out) {
    return gemm_dispatch(k, dev, pool, 1.0f, a, b, nullptr, out);
}

extern "C" int zg_gemm_bias_relu(const zg_gemm_kernel* k, zg_device* dev, zg_pool* pool,
                                 float alpha, const zg_device_array* a, const zg_device_array* b,
                                 const zg_device_array* bias, zg_device_array* out) {
    if (!bias) return set_error(ZG_ERR_DISPATCH, "gemm_bias_relu: null bias");
    return gemm_dispatch(k, dev, pool, alpha, a, b, bias, out);
}

namespace zg {
namespace {
int level1_ptr(zg_device* dev, const zg_device_array* a, float** p) {
    Buffer* b = dev->buffers.get(a->buffer);
    if (!b) return stale("level1", a->buffer, dev->buffers.current_gen(a->buffer.index));
    *p = static_cast<float*>(b->ptr);
    return ZG_OK;
}
}  // namespace
}  // namespace zg

extern "C" int zg_level1_saxpy(zg_device* dev, float alpha, const zg_device_array* x,
                               const zg_device_array* y) {
    int rc;
    if (!dev) return set_error(ZG_ERR_DISPATCH, "saxpy: null device");
    if ((rc = check_array(x, "saxpy")) || (rc = check_array(y, "saxpy"))) return rc;
    // check_f32_shape (zengpu-blas/src/level1.rs:35-48)
    if (x->dtype != ZG_DTYPE_F32 || y->dtype != ZG_DTYPE_F32)
        return set_error(ZG_ERR_DISPATCH, "saxpy: only f32 supported, got %s and %s",
                         dtype_name(x->dtype), dtype_name(y->dtype));
    if (!same_shape(x, y))
        return set_error(ZG_ERR_DISPATCH, "saxpy: shape mismatch %s vs %s", shape_str(x).c_str(),
                         shape_str(y).c_str());
    uint32_t n = 0;
    if (!array_len(x, &n)) return set_error(ZG_ERR_DISPATCH, "saxpy: length overflows u32");
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    float *px, *py;
    if ((rc = level1_ptr(dev, x, &px)) || (rc = level1_ptr(dev, y, &py))) return rc;
    if ((rc = set_device(dev))) return rc;
    if ((rc = zg_saxpy_f32(alpha, px, py, n, dev->stream))) return rc;
    if (buffer_memory(dev, y->buffer) == ZG_MEMORY_GPU_ONLY) return ZG_OK;  // queued, see dispatch_deferred
    return finish_sync(dev, false);
}

extern "C" int zg_level1_sscal(zg_device* dev, float alpha, const zg_device_array* x) {
    int rc;
    if (!dev) return set_error(ZG_ERR_DISPATCH, "sscal: null device");
    if ((rc = check_array(x, "sscal"))) return rc;
    if (x->dtype != ZG_DTYPE_F32)
        return set_error(ZG_ERR_DISPATCH, "sscal: only f32 supported, got %s", dtype_name(x->dtype));
    uint32_t n = 0;
    if (!array_len(x, &n)) return set_error(ZG_ERR_DISPATCH, "sscal: length overflows u32");
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    float* px;
    if ((rc = level1_ptr(dev, x, &px))) return rc;
    if ((rc = set_device(dev))) return rc;
    if ((rc = zg_sscal_f32(alpha, px, n, dev->stream))) return rc;
    if (buffer_memory(dev, x->buffer) == ZG_MEMORY_GPU_ONLY) return ZG_OK;  // queued, see dispatch_deferred
    return finish_sync(dev, false);
}

// ======================================================================
// Pipelined GEMM on host arrays
// ======================================================================

namespace zg {
namespace {

uint64_t align256(uint64_t x) { return (x + 255) / 256 * 256; }

int ensure_staging(zg_device* dev, uint64_t bytes) {
    if (bytes <= dev->staging_bytes) return ZG_OK;
    if (dev->staging) {
        cudaDeviceSynchronize();
        cudaFree(dev->staging);
        dev->staging = nullptr;
        dev->staging_bytes = 0;
    }
    int rc = cuda_status(cudaMalloc(&dev->staging, bytes), "host-gemm staging alloc");
    if (rc == ZG_OK) dev->staging_bytes = bytes;
    return rc;
}

int ensure_copy_streams(zg_device* dev) {
    int rc = ZG_OK;
    if (!dev->h2d)
        rc = cuda_status(cudaStreamCreateWithFlags(&dev->h2d, cudaStreamNonBlocking), "h2d stream");
    if (!rc && !dev->d2h)
        rc = cuda_status(cudaStreamCreateWithFlags(&dev->d2h, cudaStreamNonBlocking), "d2h stream");
    return rc;
}

}  // namespace
}  // namespace zg

extern "C" int zg_gemm_sgemm_host(const zg_gemm_kernel* kern, zg_device* dev, float alpha,
                                  const float* a, const float* b, const float* bias, int relu,
                                  float* c, uint32_t m, uint32_t n, uint32_t k) {
    if (!kern || !dev) return set_error(ZG_ERR_DISPATCH, "sgemm_host: null kernel or device");
    if (m > 0x7fffffffu || n > 0x7fffffffu || k > 0x7fffffffu)
        return set_error(ZG_ERR_DISPATCH, "sgemm_host: dimension exceeds 2^31-1");
    if (m == 0 || n == 0) return ZG_OK;
    if (!c || (k > 0 && (!a || !b))) return set_error(ZG_ERR_DISPATCH, "sgemm_host: null host pointer");
    const int mode = kern->mode;
    if (mode != ZG_GEMM_SIMT_FP32 && mode != ZG_GEMM_TF32X3 && mode != ZG_GEMM_TF32 &&
        mode != ZG_GEMM_TF32_BF16X2 && mode != ZG_GEMM_BF16X3)
        return set_error(ZG_ERR_DISPATCH, "sgemm: unknown mode %d", mode);
    std::lock_guard<std::recursive_mutex> lk(dev->mu);
    int rc = set_device(dev);
    if (rc) return rc;
    if (in_flight(dev))
        return set_error(ZG_ERR_BINDING_MISMATCH,
                         "sgemm_host cannot run while an asynchronous submission is pending");
    if ((rc = ensure_copy_streams(dev))) return rc;
    const int M = static_cast<int>(m), N = static_cast<int>(n), K = static_cast<int>(k);
    const bool a_planes = K > 0 && gemm_a_needs_planes(mode, K);
    const bool b_planes = K > 0 && gemm_b_needs_planes(mode);
    // Staging layout: A, B, C, bias, A planes, B^T planes.
    uint64_t off = 0;
    const uint64_t o_a = off; off += align256(uint64_t(M) * K * 4);
    const uint64_t o_b = off; off += align256(uint64_t(K) * N * 4);
    const uint64_t o_c = off; off += align256(uint64_t(M) * N * 4);
    const uint64_t o_bias = off; off += align256(uint64_t(N) * 4);
    const uint64_t o_ap = off; off += a_planes ? gemm_planes_bytes(mode, M, K) : 0;
    const uint64_t o_bp = off; off += b_planes ? gemm_planes_bytes(mode, N, K) : 0;
    if ((rc = ensure_staging(dev, off))) return rc;
    uint8_t* base = static_cast<uint8_t*>(dev->staging);
    float* dA = reinterpret_cast<float*>(base + o_a);
    float* dB = reinterpret_cast<float*>(base + o_b);
    float* dC = reinterpret_cast<float*>(base + o_c);
    float* dBias = reinterpret_cast<float*>(base + o_bias);
    const OperandView a_ps = a_planes ? gemm_carve_planes(base + o_ap, mode, M, K) : OperandView{};
    const OperandView b_ps = b_planes ? gemm_carve_planes(base + o_bp, mode, N, K)
                                      : gemm_raw_operand(dB, N);

    // Row panels of A / C (16, of at least 512 rows): the host links, not the
    // GEMM, bound this call, so panels only need to keep the GPU busy enough
    // to hide under the uploads; smaller panels shorten the tail (the last
    // panel's GEMM and C download) that nothing overlaps.
    const int rows = M <= 1024 ? M : std::max(512, (((M + 15) / 16 + 127) / 128) * 128);
    const int panels = (M + rows - 1) / rows;
    std::vector<cudaEvent_t> ev(2 * panels + 1, nullptr);
    for (auto& e : ev)
        if ((rc = cuda_status(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event")))
            break;
    cudaStream_t comp = dev->stream;
    if (!rc && K > 0) rc = cuda_status(cudaMemcpyAsync(dB, b, uint64_t(K) * N * 4,
                                                       cudaMemcpyHostToDevice, dev->h2d), "H2D B");
    if (!rc && bias)
        rc = cuda_status(cudaMemcpyAsync(dBias, bias, uint64_t(N) * 4, cudaMemcpyHostToDevice,
                                         dev->h2d), "H2D bias");
    if (!rc) rc = cuda_status(cudaEventRecord(ev[0], dev->h2d), "event");
    for (int p = 0; p < panels && !rc; ++p) {
        const int r0 = p * rows, nr = std::min(rows, M - r0);
        if (K > 0)
            rc = cuda_status(cudaMemcpyAsync(dA + int64_t(r0) * K, a + int64_t(r0) * K,
                                             uint64_t(nr) * K * 4, cudaMemcpyHostToDevice, dev->h2d),
                             "H2D A panel");
        if (!rc) rc = cuda_status(cudaEventRecord(ev[1 + p], dev->h2d), "event");
    }
    if (!rc) rc = cuda_status(cudaStreamWaitEvent(comp, ev[0], 0), "wait B");
    if (!rc && b_planes) rc = gemm_prep_b(mode, K, N, dB, N, b_ps, comp);
    for (int p = 0; p < panels && !rc; ++p) {
        const int r0 = p * rows, nr = std::min(rows, M - r0);
        if ((rc = cuda_status(cudaStreamWaitEvent(comp, ev[1 + p], 0), "wait A panel"))) break;
        float* cp = dC + int64_t(r0) * N;
        if (K == 0) {
            rc = zg_sgemm_f32(mode, nr, N, 0, alpha, nullptr, nullptr, cp, bias ? dBias : nullptr,
                              relu, nullptr, 0, comp);
        } else {
            const float* ap = dA + int64_t(r0) * K;
            const OperandView panel_ps = a_planes ? gemm_offset_rows(a_ps, r0) : OperandView{};
            if (a_planes && (rc = gemm_prep_a(mode, nr, K, ap, K, panel_ps, comp))) break;
            GemmOperands op{mode, a_planes ? panel_ps : gemm_raw_operand(ap, K), b_ps};
            rc = gemm_run(op, nr, N, K, alpha, cp, N, bias ? dBias : nullptr, relu, comp);
        }
        if (!rc) rc = cuda_status(cudaEventRecord(ev[1 + panels + p], comp), "event");
        if (!rc) rc = cuda_status(cudaStreamWaitEvent(dev->d2h, ev[1 + panels + p], 0), "wait C");
        if (!rc)
            rc = cuda_status(cudaMemcpyAsync(c + int64_t(r0) * N, cp, uint64_t(nr) * N * 4,
                                             cudaMemcpyDeviceToHost, dev->d2h),
                             "D2H C panel");
    }
    // Drain all three streams whatever happened, then report.
    cudaStreamSynchronize(dev->h2d);
    cudaStreamSynchronize(comp);
    const int sync_rc = cuda_status(cudaStreamSynchronize(dev->d2h), "sgemm_host sync");
    for (auto& e : ev)
        if (e) cudaEventDestroy(e);
    if (rc) return rc;
    if (sync_rc) return sync_rc;
    uint32_t code = 0;
    if ((rc = zg_kernel_status(&code))) return rc;
    if (code)
        return set_error(ZG_ERR_KERNEL_WAIT,
                         "kernel bounded wait expired (status 0x%x); results are invalid", code);
    return ZG_OK;
}
