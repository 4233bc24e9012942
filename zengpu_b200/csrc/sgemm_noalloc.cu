// sgemm_noalloc.cu - zg_sgemm_f32_noalloc: the f32 GEMM for callers that
// cannot allocate device memory at the point of the call.
//
// Who needs it: a caller whose device memory is owned by someone else (a host
// framework that reserves nearly all of HBM in its own pool and forbids
// outside allocations), a latency-critical loop that cannot afford
// cudaMalloc / cudaFree and the device-wide synchronisation they imply, or
// code running inside an allocator callback, where re-entering the allocator
// would deadlock.  zg_sgemm_f32 needs a caller-provided workspace for the
// tensor-core modes' operand planes; this entry point instead uses a fixed
// scratch array that lives in this library's own device image.
//
// The scratch array below is kNoAllocScratchBytes (64 MiB) on every GPU where
// this file's module is loaded, held until the process exits.  It bounds the
// shapes the entry point accepts: zg_sgemm_workspace_bytes(mode, m, n, k)
// must not exceed it (TF32X3 fits up to 2048 x 2048 x 2048).  Larger shapes
// are rejected with ZG_ERR_DISPATCH and nothing is launched, except in SIMT,
// whose workspace (A transposed, up to 4096 x 4096) is optional: beyond the
// array it runs without one, on the register-staged kernel.
//
// Host code must not pass the array's name to a kernel: on the host it is
// only a stand-in symbol, not a device address.  The first call on each
// device (with that device current) looks up the real device address with
// cudaGetSymbolAddress and caches it together with the CUDA context it belongs
// to; a later call under a different context (the primary context torn down by
// cudaDeviceReset and created again, which reloads the module) looks it up
// again.  Make the first call before any stream capture.  All calls share the
// one array and it keeps the last call's contents; nothing in it needs to
// start at zero (the pre-pass writes every element the GEMM kernel then
// reads).  Calls whose work overlaps on the GPU (different streams, or several
// host threads) race on the array: serialise them, e.g. on one stream.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "zg_common.cuh"

namespace zg {
namespace {

constexpr uint64_t kNoAllocScratchBytes = 64ull << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};

// The CUDA context current on this thread, or null when none is (cuCtxGetCurrent,
// found through the runtime so the library keeps no link-time dependency on
// libcuda).
int current_context(CUcontext* ctx) {
    using Fn = CUresult (*)(CUcontext*);
    static Fn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault,
                                             &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<Fn>(p);
    });
    *ctx = nullptr;
    if (!fn) return set_error(ZG_ERR_BACKEND, "zg_sgemm_f32_noalloc: cuCtxGetCurrent unavailable");
    if (fn(ctx) != CUDA_SUCCESS)
        return set_error(ZG_ERR_BACKEND, "zg_sgemm_f32_noalloc: cuCtxGetCurrent failed");
    return ZG_OK;
}

// Device address of the scratch array on the current device; looked up with
// that device current, once per (device, context).  A thread with no context
// current yet gets the runtime's primary context from the lookup itself.
int scratch_for_current_device(void** out) {
    int dev = 0;
    int rc = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
    if (rc) return rc;
    if (dev < 0 || dev >= kMaxDevices)
        return set_error(ZG_ERR_UNSUPPORTED, "zg_sgemm_f32_noalloc: device ordinal %d above %d",
                         dev, kMaxDevices - 1);
    CUcontext ctx = nullptr;
    if ((rc = current_context(&ctx))) return rc;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!ctx || !g_scratch_ptr[dev] || g_scratch_ctx[dev] != ctx) {
        void* p = nullptr;
        rc = cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                         "cudaGetSymbolAddress(scratch)");
        if (rc) return rc;
        if (!p) return set_error(ZG_ERR_BACKEND, "zg_sgemm_f32_noalloc: null scratch address");
        if ((rc = current_context(&ctx))) return rc;
        g_scratch_ptr[dev] = p;
        g_scratch_ctx[dev] = ctx;
    }
    *out = g_scratch_ptr[dev];
    return ZG_OK;
}

}  // namespace
}  // namespace zg

using namespace zg;

extern "C" int zg_sgemm_f32_noalloc(int mode, int m, int n, int k, float alpha, const float* a,
                                    const float* b, float* c, const float* bias, int relu,
                                    void* stream) {
    if (m < 0 || n < 0 || k < 0)
        return set_error(ZG_ERR_DISPATCH, "zg_sgemm_f32_noalloc: negative shape %d x %d x %d", m,
                         n, k);
    uint64_t need = zg_sgemm_workspace_bytes(mode, m, n, k);
    // SIMT's workspace (A transposed) is optional: without it, it runs the
    // register-staged kernel on A itself
    if (mode == ZG_GEMM_SIMT_FP32 && need > kNoAllocScratchBytes) need = 0;
    if (need > kNoAllocScratchBytes)
        return set_error(ZG_ERR_DISPATCH,
                         "zg_sgemm_f32_noalloc: %d x %d x %d (mode %d) needs %llu bytes of "
                         "scratch, above the %llu-byte static maximum; call zg_sgemm_f32 "
                         "with a caller workspace instead",
                         m, n, k, mode, (unsigned long long)need,
                         (unsigned long long)kNoAllocScratchBytes);
    void* scratch = nullptr;
    if (need > 0) {
        int rc = scratch_for_current_device(&scratch);
        if (rc) return rc;
    }
    return zg_sgemm_f32(mode, m, n, k, alpha, a, b, c, bias, relu, scratch,
                        need > 0 ? kNoAllocScratchBytes : 0, stream);
}
