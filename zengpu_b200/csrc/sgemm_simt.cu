// sgemm_simt.cu - exact-fp32 CUDA-core SGEMM, the accuracy anchor of the GEMM
// family.  Replaces the one-thread-per-element GEMM_PTX / GEMM_ZSL kernels
// (zengpu-blas/src/level3.rs:13-90): same contract, C = alpha * A @ B with
// row-major f32 operands, plus the optional fused bias/ReLU epilogue.
//
// Design: 128x128 CTA tile, 256 threads, each thread an 8x8 register
// tile laid out as 2x2 blocks of 4x4 so every shared-memory read is a
// conflict-free 128-bit load, with A k-major in shared memory.  Products are
// accumulated with IEEE fma (round to nearest, as GEMM_PTX's fma.rn.f32), two
// accumulators per instruction with sm_100's packed fma.rn.f32x2: the
// accumulators are kept as pairs of rows (acc[2p][j], acc[2p+1][j]), A's
// fragments load straight into such pairs, and each b[j] is broadcast into a
// pair before its four packed FMAs.  Every element still sees the same fma
// sequence in k order, so the result is bit-identical to scalar fmaf, and the
// FFMA issue slots halve.
//
// Two kernels share that inner loop.  sgemm_simt_tma_kernel (the fast one)
// reads A transposed by a pre-pass into the caller's workspace, so both
// operands arrive by TMA as k rows into a ring of mbarrier-guarded stages.
// sgemm_simt_kernel needs no workspace: it double-buffers tiles through
// registers, transposing A as it stores it, at the cost of a block barrier
// and the load / store instructions per tile.  They give the same bits.
#include <atomic>
#include <cstdint>
#include <cstring>

#include "zg_common.cuh"

namespace zg {

// Device status word of the SIMT SGEMM's bounded waits (read by zg_kernel_status).
__device__ uint32_t g_simt_status = 0;

namespace {

// d (pair) += a (pair) * b (pair), lane-wise IEEE fma.rn.
__device__ __forceinline__ void ffma2(uint64_t& d, uint64_t a, uint64_t b) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(a), "l"(b));
}
__device__ __forceinline__ uint64_t pair_of(float x) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(x));
    return r;
}
// Two adjacent pairs of floats from shared memory (the clobber keeps the load
// after the barrier that publishes the tile).
__device__ __forceinline__ void lds_pairs(uint32_t addr, uint64_t& p0, uint64_t& p1) {
    asm("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(p0), "=l"(p1) : "r"(addr) : "memory");
}
__device__ __forceinline__ float pair_lo(uint64_t p) {
    return __uint_as_float(static_cast<uint32_t>(p));
}
__device__ __forceinline__ float pair_hi(uint64_t p) {
    return __uint_as_float(static_cast<uint32_t>(p >> 32));
}
// Four floats from global memory, or zeros when !ok: the registers are zeroed
// and the load is predicated, so no select waits on the load before the tile's
// shared-memory store uses it (1 % faster than `ok ? __ldg(p) : 0`).
__device__ __forceinline__ float4 ldg4_or_zero(const float* p, bool ok) {
    float4 v;
    asm("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t"
        "mov.b32 %0, 0;\n\tmov.b32 %1, 0;\n\tmov.b32 %2, 0;\n\tmov.b32 %3, 0;\n\t"
        "@q ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];\n\t}"
        : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
        : "l"(p), "r"(static_cast<int>(ok)));
    return v;
}

constexpr int BM = 128, BN = 128, BK = 16;
constexpr int kThreads = 256;
constexpr int kPadA = 4;  // As row pitch 132 floats: 16-byte aligned rows

template <bool kVecA, bool kVecB>
__global__ void __launch_bounds__(kThreads, 2)
    sgemm_simt_kernel(int M, int N, int K, float alpha, const float* __restrict__ A, int64_t lda,
                      const float* __restrict__ B, int64_t ldb, float* __restrict__ C,
                      int64_t ldc, const float* __restrict__ bias, int relu, int vec_c) {
    __shared__ __align__(16) float As[2][BK][BM + kPadA];
    __shared__ __align__(16) float Bs[2][BK][BN];

    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;

    // Global-load mapping.  A: 2 x (row, 4 k) per thread.  B: 2 x (k, 4 n).
    const int a_row = tid >> 2, a_kq = (tid & 3) * 4;
    const int b_k = tid >> 5, b_nq = (tid & 31) * 4;

    float4 ra[2], rb[2];

    auto load_tile = [&](int k0) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int row = m0 + a_row + 64 * j;
            const int kk = k0 + a_kq;
            if (kVecA) {
                const bool ok = row < M && kk < K;
                ra[j] = ldg4_or_zero(A + (ok ? row * lda + kk : 0), ok);
            } else {
                float v[4];
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    v[c] = (row < M && kk + c < K) ? __ldg(A + row * lda + kk + c) : 0.f;
                ra[j] = make_float4(v[0], v[1], v[2], v[3]);
            }
            const int krow = k0 + b_k + 8 * j;
            const int col = n0 + b_nq;
            if (kVecB) {
                const bool ok = krow < K && col < N;
                rb[j] = ldg4_or_zero(B + (ok ? krow * ldb + col : 0), ok);
            } else {
                float v[4];
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    v[c] = (krow < K && col + c < N) ? __ldg(B + krow * ldb + col + c) : 0.f;
                rb[j] = make_float4(v[0], v[1], v[2], v[3]);
            }
        }
    };
    auto store_tile = [&](int buf) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int row = a_row + 64 * j;
            As[buf][a_kq + 0][row] = ra[j].x;
            As[buf][a_kq + 1][row] = ra[j].y;
            As[buf][a_kq + 2][row] = ra[j].z;
            As[buf][a_kq + 3][row] = ra[j].w;
            *reinterpret_cast<float4*>(&Bs[buf][b_k + 8 * j][b_nq]) = rb[j];
        }
    };

    // acc2[p][j] = (acc[2p][j], acc[2p + 1][j]); acc rows i: 4ty + i (i < 4),
    // 64 + 4ty + i - 4 (i >= 4); columns j: 4tx + j (j < 4), 64 + 4tx + j - 4
    uint64_t acc2[4][8];
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc2[p][j] = 0ull;

    const int nk = (K + BK - 1) / BK;
    if (nk > 0) {
        load_tile(0);
        store_tile(0);
    }
    __syncthreads();
    for (int kt = 0; kt < nk; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < nk) load_tile((kt + 1) * BK);
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            uint64_t a2[4];
            lds_pairs(smem_u32(&As[buf][k][ty * 4]), a2[0], a2[1]);
            lds_pairs(smem_u32(&As[buf][k][64 + ty * 4]), a2[2], a2[3]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][k][64 + tx * 4]);
            const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint64_t bb = pair_of(b[j]);
#pragma unroll
                for (int p = 0; p < 4; ++p) ffma2(acc2[p][j], a2[p], bb);
            }
        }
        if (kt + 1 < nk) store_tile(buf ^ 1);
        __syncthreads();
    }

    // Epilogue: c = alpha*acc, then + bias[col], then ReLU, each rounded.
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int row = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (row >= M) continue;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int col = n0 + h * 64 + tx * 4;
            float v[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint64_t pr = acc2[i >> 1][h * 4 + c];
                float x = __fmul_rn(alpha, (i & 1) ? pair_hi(pr) : pair_lo(pr));
                if (bias && col + c < N) x = __fadd_rn(x, __ldg(bias + col + c));
                if (relu) x = relu1(x);
                v[c] = x;
            }
            float* dst = C + row * ldc + col;
            if (vec_c && col + 3 < N) {
                *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
            } else {
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    if (col + c < N) dst[c] = v[c];
            }
        }
    }
}

// ---- TMA-fed kernel (A transposed by a pre-pass) ------------------------------------
// The same 128 x 128 tile, 8 x 8 thread tile and inner loop, but both operands
// arrive by TMA as 32 k rows of 128 floats: B as it lies in global memory and
// A from its transposed copy (A^T: k rows of m, written by the caller's
// pre-pass), so A's stage has the k-major layout the inner loop reads without
// any transposing store.  Stages (32 KB) sit in a three-deep ring, two
// blocks per SM (measured at 8192^3: 0.829 of the FP32 peak against 0.800
// with 16-k stages four deep, whose per-tile waits and votes cost more);
// consumer warps wait on a stage's mbarrier, multiply it and release it, and
// thread 0 refills each stage one tile after every warp is done with it, so
// there is no block barrier, no register staging and no global load in the
// multiply loop.  TMA writes zeros beyond the matrix (rows, columns, k), as
// the register-staged kernel does, so every element sees the same fma
// sequence and both kernels give the same bits.
constexpr int kTStages = 3;
constexpr int TBK = 32;
constexpr int kTThreads = 256;
constexpr int kTStageFloats = TBK * BM;                     // per operand per stage
constexpr uint32_t kTStageBytes = 2 * kTStageFloats * 4;   // A^T and B: 32 KB
constexpr int kTSmemBytes = kTStages * kTStageBytes + 1024 /*align*/ + 2 * kTStages * 8;
static_assert(BM == BN, "A^T and B stages share one shape");

struct SimtMaps {
    CUtensorMap at;  // A^T: M columns x K rows, box 128 x 16
    CUtensorMap b;   // B:   N columns x K rows, box 128 x 16
};

__global__ void __launch_bounds__(kTThreads, 2)
    sgemm_simt_tma_kernel(const __grid_constant__ SimtMaps maps, int M, int N, int K, float alpha,
                          float* __restrict__ C, int64_t ldc, const float* __restrict__ bias,
                          int relu, int vec_c) {
    uint32_t* status = &g_simt_status;
    extern __shared__ uint8_t smem_raw[];
    float* smem = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~uintptr_t(1023));
    float* As = smem;                                  // [stage][TBK][BM]
    float* Bs = smem + kTStages * kTStageFloats;       // [stage][TBK][BN]
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * kTStages * kTStageFloats);
    uint64_t* empty = full + kTStages;

    const int tid = threadIdx.x, lane = tid & 31;
    const int tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int nk = (K + TBK - 1) / TBK;
    const bool producer = tid == 0;

    auto issue = [&](int t) {
        const int s = t % kTStages;
        mbar_arrive_expect_tx(&full[s], kTStageBytes);
        tma_load_2d(As + s * kTStageFloats, &maps.at, m0, t * TBK, &full[s]);
        tma_load_2d(Bs + s * kTStageFloats, &maps.b, n0, t * TBK, &full[s]);
    };
    int issued = 0;
    if (producer) {
        for (int s = 0; s < kTStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kTThreads / 32);  // one arrive per warp
        }
        fence_mbar_init();
        prefetch_tensormap(&maps.at);
        prefetch_tensormap(&maps.b);
        for (; issued < kTStages - 1 && issued < nk; ++issued) issue(issued);
    }
    __syncthreads();

    // acc2[p][j] = (acc[2p][j], acc[2p + 1][j]); acc rows i: 4ty + i (i < 4),
    // 64 + 4ty + i - 4 (i >= 4); columns j: 4tx + j (j < 4), 64 + 4tx + j - 4
    uint64_t acc2[4][8];
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc2[p][j] = 0ull;

    bool ok = true;
    for (int kt = 0; kt < nk; ++kt) {
        const int s = kt % kTStages;
        // the warp gives up together, so no lane multiplies a stage that never came
        const bool got =
            mbar_wait_bounded(&full[s], (kt / kTStages) & 1, status, kErrSimtConsumer);
        if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
        }
        const float* as = As + s * kTStageFloats;
        const float* bs = Bs + s * kTStageFloats;
#pragma unroll
        for (int k = 0; k < TBK; ++k) {
            uint64_t a2[4];
            lds_pairs(smem_u32(as + k * BM + ty * 4), a2[0], a2[1]);
            lds_pairs(smem_u32(as + k * BM + 64 + ty * 4), a2[2], a2[3]);
            const float4 b0 = *reinterpret_cast<const float4*>(bs + k * BN + tx * 4);
            const float4 b1 = *reinterpret_cast<const float4*>(bs + k * BN + 64 + tx * 4);
            const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint64_t bb = pair_of(b[j]);
#pragma unroll
                for (int p = 0; p < 4; ++p) ffma2(acc2[p][j], a2[p], bb);
            }
        }
        // every lane's reads of the stage come before the warp frees it
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        // thread 0: tile kt + 2 goes into the stage of tile kt - 1 once every
        // warp has released that stage
        bool pok = true;
        if (producer && issued < nk) {
            const int t = issued;
            if (t >= kTStages)
                pok = mbar_wait_bounded(&empty[t % kTStages], ((t / kTStages) - 1) & 1, status,
                                        kErrSimtProducer);
            if (pok) {
                issue(t);
                ++issued;
            }
        }
        if (!__all_sync(0xffffffffu, pok)) {
            ok = false;
            break;
        }
    }
    // No copy of this block may still be landing when it exits.
    if (producer)
        for (int i = issued > kTStages ? issued - kTStages : 0; i < issued; ++i)
            mbar_wait_bounded(&full[i % kTStages], (i / kTStages) & 1, status, kErrSimtDrain);
    if (!ok) return;

    // Epilogue: c = alpha*acc, then + bias[col], then ReLU, each rounded.
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int row = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (row >= M) continue;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int col = n0 + h * 64 + tx * 4;
            float v[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint64_t pr = acc2[i >> 1][h * 4 + c];
                float x = __fmul_rn(alpha, (i & 1) ? pair_hi(pr) : pair_lo(pr));
                if (bias && col + c < N) x = __fadd_rn(x, __ldg(bias + col + c));
                if (relu) x = relu1(x);
                v[c] = x;
            }
            float* dst = C + row * ldc + col;
            if (vec_c && col + 3 < N) {
                *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
            } else {
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    if (col + c < N) dst[c] = v[c];
            }
        }
    }
}

}  // namespace

cudaError_t take_simt_status(uint32_t* v) {
    uint32_t zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(v, g_simt_status, sizeof(*v));
    if (e == cudaSuccess && *v) e = cudaMemcpyToSymbol(g_simt_status, &zero, sizeof(zero));
    return e;
}

// Launches the register-staged SIMT SGEMM on `stream`; shapes already
// validated by the caller.
int launch_sgemm_simt(int M, int N, int K, float alpha, const float* A, int64_t lda,
                      const float* B, int64_t ldb, float* C, int64_t ldc, const float* bias,
                      int relu, cudaStream_t stream) {
    const bool va = (lda % 4 == 0) && ((reinterpret_cast<uintptr_t>(A) & 15u) == 0);
    const bool vb = (ldb % 4 == 0) && ((reinterpret_cast<uintptr_t>(B) & 15u) == 0);
    const int vc = (ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(C) & 15u) == 0);
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    if (va && vb)
        sgemm_simt_kernel<true, true><<<grid, kThreads, 0, stream>>>(M, N, K, alpha, A, lda, B, ldb, C, ldc,
                                                                     bias, relu, vc);
    else if (va)
        sgemm_simt_kernel<true, false><<<grid, kThreads, 0, stream>>>(M, N, K, alpha, A, lda, B, ldb, C,
                                                                      ldc, bias, relu, vc);
    else if (vb)
        sgemm_simt_kernel<false, true><<<grid, kThreads, 0, stream>>>(M, N, K, alpha, A, lda, B, ldb, C,
                                                                      ldc, bias, relu, vc);
    else
        sgemm_simt_kernel<false, false><<<grid, kThreads, 0, stream>>>(M, N, K, alpha, A, lda, B, ldb, C,
                                                                       ldc, bias, relu, vc);
    return cuda_status(cudaGetLastError(), "sgemm_simt");
}

// Launches the TMA-fed SIMT SGEMM on A^T (K rows of M floats, pitch ldat) and
// B (K rows of N floats, pitch ldb): both 16-byte aligned with pitches of a
// multiple of 4 floats, K > 0 (the caller checks).
int launch_sgemm_simt_at(int M, int N, int K, float alpha, const float* At, int64_t ldat,
                         const float* B, int64_t ldb, float* C, int64_t ldc, const float* bias,
                         int relu, cudaStream_t stream) {
    const int vc = (ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(C) & 15u) == 0);
    SimtMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    int rc = encode_f32_map(&maps.at, At, M, K, ldat, BM, TBK, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!rc) rc = encode_f32_map(&maps.b, B, N, K, ldb, BN, TBK, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    // the dynamic shared-memory opt-in, once per device
    static std::atomic<uint64_t> attr_done{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_done.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(
            sgemm_simt_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTSmemBytes);
        if (e != cudaSuccess) return cuda_status(e, "sgemm_simt_tma smem attribute");
        attr_done.fetch_or(bit);
    }
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    sgemm_simt_tma_kernel<<<grid, kTThreads, kTSmemBytes, stream>>>(maps, M, N, K, alpha, C, ldc,
                                                                    bias, relu, vc);
    return cuda_status(cudaGetLastError(), "sgemm_simt_tma");
}

}  // namespace zg
