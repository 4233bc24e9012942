// elementwise.cu - HBM-streaming f32 kernels for ZenGPU's DeviceArray ops:
// add (ADD_ZSL, zengpu-compute/src/elementwise.rs:17-26), ReLU (RELU_ZSL,
// :29-38), Level-1 saxpy/sscal (zengpu-blas/src/level1.rs:11-33) and the
// seeded input generators.
//
// Each kernel is grid-stride over 16-byte float4 lanes with streaming cache
// hints (the data is touched once), eight independent 16-byte loads in flight
// per thread (four from each input for binary ops, eight from the one input
// for unary ops), and a scalar tail.  Arithmetic is plain IEEE f32 with no
// contraction (__fadd_rn / __fmul_rn), so results are bit-identical to the
// Rust CPU backend.
#include <cstdint>

#include "zg_common.cuh"

namespace zg {
namespace {

constexpr int kThreads = 256;
// float4 loads in flight per thread and input: 128 bytes per thread either way
template <bool kBinary>
constexpr int kUnroll = kBinary ? 4 : 8;

int sm_count() {
    static thread_local int cached_dev = -1, cached = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != cached_dev) {
        cudaDeviceGetAttribute(&cached, cudaDevAttrMultiProcessorCount, dev);
        if (cached <= 0) cached = 148;
        cached_dev = dev;
    }
    return cached;
}

// Grid: enough CTAs to fill every SM (8 x 256 threads resident per SM), never
// more than the work needs.
unsigned grid_for(uint64_t units) {
    uint64_t want = (units + kThreads - 1) / kThreads;
    uint64_t cap = static_cast<uint64_t>(sm_count()) * 8;
    if (want > cap) want = cap;
    return static_cast<unsigned>(want < 1 ? 1 : want);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct AddOp {
    __device__ static float apply(float a, float b, float) { return __fadd_rn(a, b); }
};
struct ReluOp {
    __device__ static float apply(float a, float, float) { return relu1(a); }
};
struct AxpyOp {  // y + alpha * x, rounded product then rounded sum
    __device__ static float apply(float x, float y, float alpha) {
        return __fadd_rn(y, __fmul_rn(alpha, x));
    }
};
struct ScalOp {
    __device__ static float apply(float x, float, float alpha) { return __fmul_rn(x, alpha); }
};

__device__ __forceinline__ float4 ld_stream(const float4* p) { return __ldcs(p); }

template <class Op>
__device__ __forceinline__ float4 apply4(float4 a, float4 b, float s) {
    return make_float4(Op::apply(a.x, b.x, s), Op::apply(a.y, b.y, s), Op::apply(a.z, b.z, s),
                       Op::apply(a.w, b.w, s));
}

// out[i] = Op(a[i], b[i]) over n4 float4 lanes plus `tail` trailing scalars.
// `b` may be null for unary ops; `out` may alias `a` (in-place ReLU/scal) or
// `b` (saxpy writes y), so no __restrict__ here.
template <class Op, bool kBinary>
__global__ void __launch_bounds__(kThreads)
    stream_vec_kernel(const float4* a, const float4* b, float4* out, uint64_t n4,
                      const float* a_s, const float* b_s, float* out_s, uint32_t tail,
                      float scalar) {
    constexpr int U = kUnroll<kBinary>;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kThreads;
    uint64_t i = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
    for (; i + (U - 1) * stride < n4; i += U * stride) {
        float4 va[U], vb[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            va[u] = ld_stream(a + i + u * stride);
            vb[u] = kBinary ? ld_stream(b + i + u * stride) : va[u];
        }
#pragma unroll
        for (int u = 0; u < U; ++u) __stcs(out + i + u * stride, apply4<Op>(va[u], vb[u], scalar));
    }
    for (; i < n4; i += stride) {
        float4 va = ld_stream(a + i);
        float4 vb = kBinary ? ld_stream(b + i) : va;
        __stcs(out + i, apply4<Op>(va, vb, scalar));
    }
    if (blockIdx.x == 0 && threadIdx.x < tail) {
        const uint64_t j = n4 * 4 + threadIdx.x;
        out_s[j] = Op::apply(a_s[j], kBinary ? b_s[j] : 0.0f, scalar);
    }
}

// Scalar path for pointers that are not 16-byte aligned.
template <class Op, bool kBinary>
__global__ void __launch_bounds__(kThreads)
    stream_scalar_kernel(const float* a, const float* b, float* out, uint64_t n, float scalar) {
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kThreads;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n;
         i += stride)
        out[i] = Op::apply(a[i], kBinary ? b[i] : 0.0f, scalar);
}

template <class Op, bool kBinary>
int launch_stream(const float* a, const float* b, float* out, uint64_t n, float scalar,
                  void* stream, const char* name) {
    if (n == 0) return ZG_OK;
    if (!a || !out || (kBinary && !b))
        return set_error(ZG_ERR_DISPATCH, "%s: null pointer for %llu elements", name,
                         (unsigned long long)n);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool vec = aligned16(a) && aligned16(out) && (!kBinary || aligned16(b));
    if (vec) {
        const uint64_t n4 = n / 4;
        const uint32_t tail = static_cast<uint32_t>(n - n4 * 4);
        stream_vec_kernel<Op, kBinary><<<grid_for(n4 > 0 ? n4 : 1), kThreads, 0, s>>>(
            reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b),
            reinterpret_cast<float4*>(out), n4, a, b, out, tail, scalar);
    } else {
        stream_scalar_kernel<Op, kBinary><<<grid_for(n), kThreads, 0, s>>>(a, b, out, n, scalar);
    }
    return cuda_status(cudaGetLastError(), name);
}

// ---- seeded generators: splitmix64 counter stream, bit-identical to the host one
__device__ __forceinline__ uint64_t splitmix64_at(uint64_t seed, uint64_t i) {
    uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void __launch_bounds__(kThreads)
    fill_uniform_kernel(float* x, uint64_t n, uint64_t seed, float lo, float hi, int exact_pm1) {
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kThreads;
    const float span = __fsub_rn(hi, lo);
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n;
         i += stride) {
        const uint32_t u24 = static_cast<uint32_t>(splitmix64_at(seed, i) >> 40);
        if (exact_pm1) {
            x[i] = __fsub_rn(__fmul_rn(static_cast<float>(u24), 0x1p-23f), 1.0f);
        } else {
            const float u = __fmul_rn(static_cast<float>(u24), 0x1p-24f);
            x[i] = __fadd_rn(lo, __fmul_rn(span, u));
        }
    }
}

__global__ void __launch_bounds__(kThreads)
    fill_normal_kernel(float* x, uint64_t n, uint64_t seed) {
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kThreads;
    const uint64_t pairs = (n + 1) / 2;
    for (uint64_t j = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x; j < pairs;
         j += stride) {
        const uint64_t s1 = splitmix64_at(seed, 2 * j), s2 = splitmix64_at(seed, 2 * j + 1);
        const double u1 = static_cast<double>((s1 >> 11) + 1) * 0x1p-53;
        const double u2 = static_cast<double>(s2 >> 11) * 0x1p-53;
        const double r = sqrt(-2.0 * log(u1));
        const double th = 6.283185307179586476925286766559 * u2;
        double sn, cs;
        sincos(th, &sn, &cs);
        x[2 * j] = static_cast<float>(r * cs);
        if (2 * j + 1 < n) x[2 * j + 1] = static_cast<float>(r * sn);
    }
}

}  // namespace
}  // namespace zg

using namespace zg;

extern "C" int zg_add_f32(const float* a, const float* b, float* out, uint64_t n, void* stream) {
    return launch_stream<AddOp, true>(a, b, out, n, 0.0f, stream, "zg_add_f32");
}

extern "C" int zg_relu_f32(const float* a, float* out, uint64_t n, void* stream) {
    return launch_stream<ReluOp, false>(a, nullptr, out, n, 0.0f, stream, "zg_relu_f32");
}

extern "C" int zg_saxpy_f32(float alpha, const float* x, float* y, uint64_t n, void* stream) {
    return launch_stream<AxpyOp, true>(x, y, y, n, alpha, stream, "zg_saxpy_f32");
}

extern "C" int zg_sscal_f32(float alpha, float* x, uint64_t n, void* stream) {
    return launch_stream<ScalOp, false>(x, nullptr, x, n, alpha, stream, "zg_sscal_f32");
}

extern "C" int zg_fill_uniform_f32(float* x, uint64_t n, uint64_t seed, float lo, float hi,
                                   void* stream) {
    if (n == 0) return ZG_OK;
    if (!x) return set_error(ZG_ERR_DISPATCH, "zg_fill_uniform_f32: null pointer");
    const int exact = (lo == -1.0f && hi == 1.0f) ? 1 : 0;
    fill_uniform_kernel<<<grid_for(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        x, n, seed, lo, hi, exact);
    return cuda_status(cudaGetLastError(), "zg_fill_uniform_f32");
}

extern "C" int zg_fill_normal_f32(float* x, uint64_t n, uint64_t seed, void* stream) {
    if (n == 0) return ZG_OK;
    if (!x) return set_error(ZG_ERR_DISPATCH, "zg_fill_normal_f32: null pointer");
    fill_normal_kernel<<<grid_for((n + 1) / 2), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        x, n, seed);
    return cuda_status(cudaGetLastError(), "zg_fill_normal_f32");
}
