// sgemm_tc.cu - tcgen05 / TMEM tensor-core SGEMM for sm_100a, and the GEMM
// dispatcher behind zg_sgemm_f32 (the kernel contract of GEMM_PTX's entry
// `main(a, b, c, m, n, k, alpha)`, zengpu-blas/src/level3.rs:35-90).
//
// Two tensor-core modes share one kernel template:
//   TF32    one kind::tf32 MMA per k-step on the raw f32 operands;
//   TF32X3  split precision: x = hi + lo with hi = tf32(x), lo = tf32(x - hi)
//           (round-to-nearest both), D += A_lo*B_hi + A_hi*B_lo + A_hi*B_hi;
//           the dropped lo*lo term is ~2^-22 relative, so the result keeps
//           fp32-class accuracy.  A pre-pass writes the hi/lo planes.
//
// Kernel layout (one 128 x 256 output tile per CTA, 320 threads):
//   warp 0      TMA producer: A tile [128 x BK] and B^T tile [256 x BK], both
//               K-major and swizzled (B is transposed to K-major planes by the
//               pre-pass), into a STAGES-deep mbarrier ring;
//   warp 1      allocates 512 TMEM columns (two 128 x 256 f32 accumulators,
//               lane = row) and one thread issues tcgen05.mma, committing each
//               stage back to the producer and each finished k-chunk to the
//               epilogue;
//   warps 2-9   epilogue: two warps per TMEM lane quarter, one per 128-column
//               half.  The tensor core's f32 accumulation truncates, so its
//               error grows with k; the epilogue therefore drains the TMEM
//               accumulator every kChunkK of k into f32 registers (round to
//               nearest) while the MMA fills the other accumulator, then
//               applies alpha / bias / ReLU and stores with 128-bit writes.
// Every mbarrier wait is bounded (zg_common.cuh); an expiry sets a bit in the
// device status word, the kernel drains its in-flight copies and MMAs, frees
// TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <algorithm>
#include <cstring>
#include <mutex>

#include "zg_common.cuh"
#include "zg_gemm_internal.h"

namespace zg {

__device__ uint32_t g_status = 0;

int launch_sgemm_simt(int M, int N, int K, float alpha, const float* A, int64_t lda,
                      const float* B, int64_t ldb, float* C, int64_t ldc, const float* bias,
                      int relu, cudaStream_t stream);

namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int kEpiWarps = 8;
constexpr int kTcThreads = 64 + 32 * kEpiWarps;  // producer, MMA, 8 epilogue warps
constexpr uint32_t kTmemCols = 512;              // two BN-column accumulators

template <int kPlanes>
struct TcCfg {
    static constexpr int BK = kPlanes == 1 ? 32 : 16;  // k per stage
    static constexpr int STAGES = 4;                   // 48 KB per stage
    static constexpr int A_BYTES = BM * BK * 4;        // one plane
    static constexpr int B_BYTES = BN * BK * 4;        // one plane
    static constexpr int STAGE_BYTES = kPlanes * (A_BYTES + B_BYTES);
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*bars*/;
    // Both operands K-major, rows of BK*4 bytes, swizzled at that width.
    static constexpr uint32_t LAYOUT = BK == 32 ? 2u : 4u;  // SWIZZLE_128B : SWIZZLE_64B
    static constexpr uint32_t SBO = 8 * BK * 4;             // 8-row core-matrix group
    // k-blocks per TMEM accumulation chunk: 512 of k for TF32X3 (keeps the
    // truncation error of the tensor-core accumulator near 3e-6 relative);
    // TF32 (tolerance 5e-3) accumulates the whole k range in TMEM.
    static constexpr int KB_PER_CHUNK = kPlanes == 2 ? 512 / BK : (1 << 30);
};

struct TcMaps {
    CUtensorMap a[2];  // hi, lo (TF32 uses a[0] only)
    CUtensorMap b[2];
};

// UMMA shared-memory descriptor (sm100): start, leading / stride byte
// offsets (16-byte units), version 1, layout type in bits 61-63.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) |
           (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) |
           (static_cast<uint64_t>(layout) << 61);
}

// Instruction descriptor, kind::tf32: D f32, A/B tf32, both K-major,
// M = 128, N = 256.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (0u << 15) | (0u << 16) |
                            (static_cast<uint32_t>(BN >> 3) << 17) |
                            (static_cast<uint32_t>(BM >> 4) << 24);

// Grouped raster: consecutive CTAs walk down kGroupM row-tiles before moving
// right, so CTAs resident together share A row-blocks and B column-blocks in L2.
constexpr int kGroupM = 16;
__device__ __forceinline__ void tile_coords(int tile, int mt, int nt, int& m_tile, int& n_tile) {
    const int group_size = kGroupM * nt;
    const int group = tile / group_size;
    const int first_m = group * kGroupM;
    const int gm = min(mt - first_m, kGroupM);
    const int r = tile - group * group_size;
    m_tile = first_m + r % gm;
    n_tile = r / gm;
}

template <int kPlanes>
__global__ void __launch_bounds__(kTcThreads, 1)
    sgemm_tc_kernel(const __grid_constant__ TcMaps maps, int M, int N, int K, float alpha,
                    float* __restrict__ C, int64_t ldc, const float* __restrict__ bias, int relu,
                    int vec_c) {
    using Cfg = TcCfg<kPlanes>;
    constexpr int BK = Cfg::BK, STAGES = Cfg::STAGES;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;  // [2]: chunk in TMEM buffer b is complete
    uint64_t* acc_empty = acc_full + 2;   // [2]: epilogue has drained TMEM buffer b
    uint64_t* drain = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = (M + BM - 1) / BM, nt = (N + BN - 1) / BN;
    const int num_tiles = mt * nt;
    const int nkb = (K + BK - 1) / BK;
    const int nchunks = (nkb + Cfg::KB_PER_CHUNK - 1) / Cfg::KB_PER_CHUNK;
    // Persistent: CTA b owns tiles b, b + gridDim.x, ... in grouped raster order.
    auto tile_origin = [&](int t, int& m0, int& n0) {
        int mi, ni;
        tile_coords(t, mt, nt, mi, ni);
        m0 = mi * BM;
        n0 = ni * BN;
    };

    auto a_plane = [&](int s, int p) { return smem + s * Cfg::STAGE_BYTES + p * Cfg::A_BYTES; };
    auto b_plane = [&](int s, int p) {
        return smem + s * Cfg::STAGE_BYTES + kPlanes * Cfg::A_BYTES + p * Cfg::B_BYTES;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 32 * kEpiWarps);
        }
        mbar_init(drain, 1);
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        for (int p = 0; p < kPlanes; ++p) {
            prefetch_tensormap(&maps.a[p]);
            prefetch_tensormap(&maps.b[p]);
        }
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int it = 0;  // k-blocks issued by this CTA over all its tiles
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                int m0, n0;
                tile_origin(t, m0, n0);
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait_bounded(&empty[s], ph ^ 1, &g_status, kErrTcProducer)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
                    const int k0 = kb * BK;
                    for (int p = 0; p < kPlanes; ++p) {
                        tma_load_2d(a_plane(s, p), &maps.a[p], k0, m0, &full[s]);
                        tma_load_2d(b_plane(s, p), &maps.b[p], k0, n0, &full[s]);
                    }
                }
            }
            // Make sure no copy is still landing in shared memory at exit.
            const int first = it > STAGES ? it - STAGES : 0;
            for (int i = first; i < it; ++i)
                mbar_wait_bounded(&full[i % STAGES], (i / STAGES) & 1, &g_status, kErrTcDrain);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            bool ok = true;
            int it = 0;  // k-blocks consumed
            int cj = 0;  // accumulation chunks issued (alternating TMEM buffers)
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                for (int j = 0; j < nchunks && ok; ++j, ++cj) {
                    const int buf = cj & 1;
                    const uint32_t d_tmem = tmem_base + buf * BN;
                    if (cj >= 2 && !mbar_wait_bounded(&acc_empty[buf], ((cj >> 1) - 1) & 1,
                                                      &g_status, kErrTcMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const int kb0 = j * Cfg::KB_PER_CHUNK;
                    const int kb1 = min(nkb, kb0 + Cfg::KB_PER_CHUNK);
                    for (int kb = kb0; kb < kb1; ++kb, ++it) {
                        const int s = it % STAGES;
                        const uint32_t ph = (it / STAGES) & 1;
                        if (!mbar_wait_bounded(&full[s], ph, &g_status, kErrTcMma)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a0 = smem_u32(a_plane(s, 0));
                        const uint32_t b0 = smem_u32(b_plane(s, 0));
#pragma unroll
                        for (int kk = 0; kk < BK / 8; ++kk) {
                            // Advance 8 f32 (32 bytes) inside the swizzled K row.
                            const uint64_t ahi =
                                umma_desc(a0 + kk * 32, 16, Cfg::SBO, Cfg::LAYOUT);
                            const uint64_t bhi =
                                umma_desc(b0 + kk * 32, 16, Cfg::SBO, Cfg::LAYOUT);
                            const uint32_t acc0 = (kb != kb0 || kk != 0) ? 1u : 0u;
                            if (kPlanes == 2) {
                                const uint32_t a1 = smem_u32(a_plane(s, 1));
                                const uint32_t b1 = smem_u32(b_plane(s, 1));
                                const uint64_t alo =
                                    umma_desc(a1 + kk * 32, 16, Cfg::SBO, Cfg::LAYOUT);
                                const uint64_t blo =
                                    umma_desc(b1 + kk * 32, 16, Cfg::SBO, Cfg::LAYOUT);
                                mma_tf32_ss(d_tmem, alo, bhi, kIdesc, acc0);
                                mma_tf32_ss(d_tmem, ahi, blo, kIdesc, 1u);
                                mma_tf32_ss(d_tmem, ahi, bhi, kIdesc, 1u);
                            } else {
                                mma_tf32_ss(d_tmem, ahi, bhi, kIdesc, acc0);
                            }
                        }
                        mma_commit(&empty[s]);  // stage s free once these MMAs finish
                    }
                    if (ok) mma_commit(&acc_full[buf]);  // chunk complete in buffer buf
                }
            }
            if (!ok) {
                mma_commit(drain);
                mbar_wait_bounded(drain, 0, &g_status, kErrTcDrain);
            }
        }
    } else {
        // ---------------- epilogue (warps 2..9) ----------------
        const int q = warp & 3;             // TMEM lane quarter this warp may access
        const int half = (warp - 2) >> 2;   // 128-column half of the tile
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + half * 128;
        bool ok = true;
        int cj = 0;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            int m0, n0;
            tile_origin(t, m0, n0);
            const int row = m0 + q * 32 + lane;
            float acc[128];
#pragma unroll
            for (int i = 0; i < 128; ++i) acc[i] = 0.0f;
            for (int j = 0; j < nchunks; ++j, ++cj) {
                const int buf = cj & 1;
                if (!mbar_wait_bounded(&acc_full[buf], (cj >> 1) & 1, &g_status,
                                       kErrTcEpilogue)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(lane_base + buf * BN + cc * 32, r);
#pragma unroll
                    for (int u = 0; u < 32; ++u) acc[cc * 32 + u] += __uint_as_float(r[u]);
                }
                tc_fence_before();
                mbar_arrive(&acc_empty[buf]);
            }
            if (ok && row < M) {
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    const int col0 = n0 + half * 128 + cc * 32;
                    if (col0 < N) {
                        float v[32];
#pragma unroll
                        for (int u = 0; u < 32; ++u) {
                            float x = __fmul_rn(alpha, acc[cc * 32 + u]);
                            if (bias) x = __fadd_rn(x, col0 + u < N ? __ldg(bias + col0 + u) : 0.0f);
                            if (relu) x = relu1(x);
                            v[u] = x;
                        }
                        float* dst = C + static_cast<int64_t>(row) * ldc + col0;
                        if (vec_c && col0 + 32 <= N) {
#pragma unroll
                            for (int u = 0; u < 32; u += 4)
                                *reinterpret_cast<float4*>(dst + u) =
                                    make_float4(v[u], v[u + 1], v[u + 2], v[u + 3]);
                        } else {
#pragma unroll
                            for (int u = 0; u < 32; ++u)
                                if (col0 + u < N) dst[u] = v[u];
                        }
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ---- split / pad pre-pass ---------------------------------------------------
// dst_hi[r, c] = tf32(src[r, c]); dst_lo[r, c] = tf32(src - hi) (when non-null);
// rows of `cols` elements, source pitch `lds`, destination pitch `ldd`.
// With dst_lo == null and round == 0 it is a plain pitched copy.
__global__ void __launch_bounds__(256)
    split_planes_kernel(const float* __restrict__ src, int rows, int cols, int64_t lds,
                        float* __restrict__ hi, float* __restrict__ lo, int64_t ldd, int round) {
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
        const float* s = src + r * lds;
        float* h = hi + r * ldd;
        float* l = lo ? lo + r * ldd : nullptr;
        for (int c = threadIdx.x; c < cols; c += blockDim.x) {
            const float x = __ldcs(s + c);
            const float xh = round ? to_tf32(x) : x;
            h[c] = xh;
            if (l) l[c] = to_tf32(__fsub_rn(x, xh));
        }
    }
}

__global__ void __launch_bounds__(256)
    split_planes_vec_kernel(const float4* __restrict__ src, int rows, int cols4, int64_t lds4,
                            float4* __restrict__ hi, float4* __restrict__ lo, int64_t ldd4) {
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
        const float4* s = src + r * lds4;
        float4* h = hi + r * ldd4;
        float4* l = lo + r * ldd4;
        for (int c = threadIdx.x; c < cols4; c += blockDim.x) {
            const float4 x = __ldcs(s + c);
            const float4 xh = make_float4(to_tf32(x.x), to_tf32(x.y), to_tf32(x.z), to_tf32(x.w));
            h[c] = xh;
            l[c] = make_float4(to_tf32(__fsub_rn(x.x, xh.x)), to_tf32(__fsub_rn(x.y, xh.y)),
                               to_tf32(__fsub_rn(x.z, xh.z)), to_tf32(__fsub_rn(x.w, xh.w)));
        }
    }
}

// Transposing variant for B: dst[n, k] = f(src[k, n]) from a K x N source
// (pitch lds) into N x K planes (pitch ldd), through a 32 x 33 shared tile so
// both the reads and the writes are coalesced.  hi = tf32(x) (round) or x;
// lo = tf32(x - hi) when `lo` is non-null.
__global__ void __launch_bounds__(256)
    transpose_planes_kernel(const float* __restrict__ src, int K, int N, int64_t lds,
                            float* __restrict__ hi, float* __restrict__ lo, int64_t ldd,
                            int round) {
    __shared__ float tile[32][33];
    const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
#pragma unroll
    for (int j = ty; j < 32; j += 8) {
        const int k = k0 + j, n = n0 + tx;
        tile[j][tx] = (k < K && n < N) ? __ldcs(src + static_cast<int64_t>(k) * lds + n) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int j = ty; j < 32; j += 8) {
        const int n = n0 + j, k = k0 + tx;
        if (n < N && k < K) {
            const float x = tile[tx][j];
            const float h = round ? to_tf32(x) : x;
            const int64_t o = static_cast<int64_t>(n) * ldd + k;
            hi[o] = h;
            if (lo) lo[o] = to_tf32(__fsub_rn(x, h));
        }
    }
}

// C = epilogue(alpha * 0) for K == 0 (an empty sum, as the reference loop).
__global__ void gemm_k0_kernel(int M, int N, float alpha, float* C, const float* bias, int relu) {
    const int64_t total = static_cast<int64_t>(M) * N;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float x = __fmul_rn(alpha, 0.0f);
        if (bias) x = __fadd_rn(x, bias[i % N]);
        if (relu) x = relu1(x);
        C[i] = x;
    }
}

// ---- host side ----------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D row-major f32 map: inner extent `cols`, outer `rows`, pitch `ld`
// elements, box {box_x, box_y}.
int encode_map(CUtensorMap* map, const float* base, uint64_t cols, uint64_t rows, uint64_t ld,
               uint32_t box_x, uint32_t box_y, CUtensorMapSwizzle swz) {
    auto fn = get_encode_fn();
    if (!fn) return set_error(ZG_ERR_BACKEND, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 4};
    cuuint32_t box[2] = {box_x, box_y};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(ZG_ERR_BACKEND, "cuTensorMapEncodeTiled failed (%d): %llux%llu ld=%llu",
                         static_cast<int>(r), (unsigned long long)rows, (unsigned long long)cols,
                         (unsigned long long)ld);
    return ZG_OK;
}

uint64_t round_up(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct WsLayout {
    uint64_t a_hi, a_lo, b_hi, b_lo, total;  // byte offsets; ~0 = unused
};

constexpr uint64_t kNone = ~0ull;

WsLayout ws_layout(int mode, int m, int n, int k) {
    WsLayout w{kNone, kNone, kNone, kNone, 0};
    // A planes M x kp, B planes (transposed, K-major) N x kp.
    const uint64_t kp = round_up(k, 4);
    const uint64_t a_bytes = round_up(static_cast<uint64_t>(m) * kp * 4, 256);
    const uint64_t b_bytes = round_up(static_cast<uint64_t>(n) * kp * 4, 256);
    uint64_t off = 0;
    if (mode == ZG_GEMM_TF32X3) {
        w.a_hi = off; off += a_bytes;
        w.a_lo = off; off += a_bytes;
        w.b_hi = off; off += b_bytes;
        w.b_lo = off; off += b_bytes;
    } else if (mode == ZG_GEMM_TF32) {
        if (k % 4 != 0) { w.a_hi = off; off += a_bytes; }
        w.b_hi = off; off += b_bytes;
    }
    w.total = off;
    return w;
}

unsigned split_grid(int rows) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int cap = sms * 8;
    return static_cast<unsigned>(rows < cap ? (rows < 1 ? 1 : rows) : cap);
}

// Writes the tf32 hi (and lo) planes of a rows x cols matrix into pitch-ldd
// buffers; a plain pitched copy when lo == null and round == 0.
int launch_split(const float* src, int rows, int cols, int64_t lds, float* hi, float* lo,
                 int64_t ldd, int round, cudaStream_t s) {
    if (rows == 0 || cols == 0) return ZG_OK;
    if (lo && round && cols % 4 == 0 && lds % 4 == 0 && ldd % 4 == 0 && aligned16(src) &&
        aligned16(hi) && aligned16(lo)) {
        split_planes_vec_kernel<<<split_grid(rows), 256, 0, s>>>(
            reinterpret_cast<const float4*>(src), rows, cols / 4, lds / 4,
            reinterpret_cast<float4*>(hi), reinterpret_cast<float4*>(lo), ldd / 4);
    } else {
        split_planes_kernel<<<split_grid(rows), 256, 0, s>>>(src, rows, cols, lds, hi, lo, ldd,
                                                             round);
    }
    return cuda_status(cudaGetLastError(), "sgemm split pre-pass");
}

// Writes the K-major (transposed) planes of B: N x K, pitch ldd.
int launch_transpose(const float* src, int K, int N, int64_t lds, float* hi, float* lo,
                     int64_t ldd, int round, cudaStream_t s) {
    if (K == 0 || N == 0) return ZG_OK;
    dim3 grid((N + 31) / 32, (K + 31) / 32);
    if (grid.y > 65535u) return set_error(ZG_ERR_DISPATCH, "sgemm: k too large for the pre-pass");
    transpose_planes_kernel<<<grid, 256, 0, s>>>(src, K, N, lds, hi, lo, ldd, round);
    return cuda_status(cudaGetLastError(), "sgemm transpose pre-pass");
}

template <int kPlanes>
int launch_tc(const TcMaps& maps, int M, int N, int K, float alpha, float* C, int64_t ldc,
              const float* bias, int relu, cudaStream_t s) {
    using Cfg = TcCfg<kPlanes>;
    static std::once_flag attr_once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(attr_once, [] {
        attr_err = cudaFuncSetAttribute(sgemm_tc_kernel<kPlanes>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        Cfg::SMEM_BYTES);
    });
    if (attr_err != cudaSuccess) return cuda_status(attr_err, "sgemm_tc smem attribute");
    const int mt = (M + BM - 1) / BM, nt = (N + BN - 1) / BN;
    const int vec_c = (ldc % 4 == 0) && aligned16(C);
    // Persistent grid: one CTA per SM (the smem footprint allows no more).
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int grid = std::min(mt * nt, std::max(sms, 1));
    sgemm_tc_kernel<kPlanes><<<grid, kTcThreads, Cfg::SMEM_BYTES, s>>>(maps, M, N, K, alpha, C,
                                                                      ldc, bias, relu, vec_c);
    return cuda_status(cudaGetLastError(), "sgemm_tc");
}

}  // namespace

// ---- GEMM building blocks (shared with the runtime's pipelined host GEMM) ----
bool gemm_a_needs_planes(int mode, int K) {
    return mode == ZG_GEMM_TF32X3 || (mode == ZG_GEMM_TF32 && K % 4 != 0);
}
bool gemm_b_needs_planes(int mode) { return mode == ZG_GEMM_TF32X3 || mode == ZG_GEMM_TF32; }
int64_t gemm_plane_pitch(int K) { return static_cast<int64_t>(round_up(K, 4)); }

int gemm_prep_a(int mode, int M, int K, const float* A, int64_t lda, float* hi, float* lo,
                int64_t ldp, cudaStream_t s) {
    if (mode == ZG_GEMM_TF32X3) return launch_split(A, M, K, lda, hi, lo, ldp, 1, s);
    if (mode == ZG_GEMM_TF32 && K % 4 != 0)
        return launch_split(A, M, K, lda, hi, nullptr, ldp, 0, s);
    return ZG_OK;
}

int gemm_prep_b(int mode, int K, int N, const float* B, int64_t ldb, float* hi, float* lo,
                int64_t ldp, cudaStream_t s) {
    if (mode == ZG_GEMM_TF32X3) return launch_transpose(B, K, N, ldb, hi, lo, ldp, 1, s);
    if (mode == ZG_GEMM_TF32) return launch_transpose(B, K, N, ldb, hi, nullptr, ldp, 0, s);
    return ZG_OK;
}

int gemm_run(const GemmOperands& op, int M, int N, int K, float alpha, float* C, int64_t ldc,
             const float* bias, int relu, cudaStream_t s) {
    if (op.mode == ZG_GEMM_SIMT_FP32)
        return launch_sgemm_simt(M, N, K, alpha, op.a_hi, op.lda, op.b_hi, op.ldb, C, ldc, bias,
                                 relu, s);
    TcMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    int rc;
    if (!aligned16(op.a_hi) || !aligned16(op.b_hi) || op.lda % 4 != 0 || op.ldb % 4 != 0)
        return set_error(ZG_ERR_DISPATCH,
                         "sgemm (tensor-core mode): operand planes must be 16-byte aligned with a "
                         "pitch that is a multiple of 4 floats");
    if (op.mode == ZG_GEMM_TF32X3) {
        using Cfg = TcCfg<2>;
        const CUtensorMapSwizzle swz =
            Cfg::BK == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
        if ((rc = encode_map(&maps.a[0], op.a_hi, K, M, op.lda, Cfg::BK, BM, swz))) return rc;
        if ((rc = encode_map(&maps.a[1], op.a_lo, K, M, op.lda, Cfg::BK, BM, swz))) return rc;
        if ((rc = encode_map(&maps.b[0], op.b_hi, K, N, op.ldb, Cfg::BK, BN, swz))) return rc;
        if ((rc = encode_map(&maps.b[1], op.b_lo, K, N, op.ldb, Cfg::BK, BN, swz))) return rc;
        return launch_tc<2>(maps, M, N, K, alpha, C, ldc, bias, relu, s);
    }
    using Cfg = TcCfg<1>;
    if ((rc = encode_map(&maps.a[0], op.a_hi, K, M, op.lda, Cfg::BK, BM,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if ((rc = encode_map(&maps.b[0], op.b_hi, K, N, op.ldb, Cfg::BK, BN,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    return launch_tc<1>(maps, M, N, K, alpha, C, ldc, bias, relu, s);
}

namespace {

// The operands zg_sgemm_compute reads for (mode, m, n, k) in workspace `ws`.
GemmOperands operands_in_workspace(int mode, int M, int N, int K, const float* A,
                                   const float* B, const uint8_t* ws) {
    const WsLayout w = ws_layout(mode, M, N, K);
    const int64_t kp = gemm_plane_pitch(K);
    auto plane = [&](uint64_t off) {
        return off == kNone ? nullptr : reinterpret_cast<const float*>(ws + off);
    };
    GemmOperands op{mode, A, nullptr, K, B, nullptr, N};
    if (mode == ZG_GEMM_SIMT_FP32) return op;
    if (w.a_hi != kNone) {
        op.a_hi = plane(w.a_hi);
        op.a_lo = plane(w.a_lo);
        op.lda = kp;
    }
    op.b_hi = plane(w.b_hi);
    op.b_lo = plane(w.b_lo);
    op.ldb = kp;
    return op;
}

int prepare_planes(int mode, int M, int N, int K, const float* A, const float* B, uint8_t* ws,
                   cudaStream_t s) {
    const WsLayout w = ws_layout(mode, M, N, K);
    const int64_t kp = gemm_plane_pitch(K);
    auto plane = [&](uint64_t off) {
        return off == kNone ? nullptr : reinterpret_cast<float*>(ws + off);
    };
    int rc = ZG_OK;
    if (gemm_a_needs_planes(mode, K) &&
        (rc = gemm_prep_a(mode, M, K, A, K, plane(w.a_hi), plane(w.a_lo), kp, s)) != ZG_OK)
        return rc;
    if (gemm_b_needs_planes(mode))
        rc = gemm_prep_b(mode, K, N, B, N, plane(w.b_hi), plane(w.b_lo), kp, s);
    return rc;
}

// Shared argument checks of the three GEMM entry points.  Returns ZG_OK and
// sets *trivial when there is nothing (m or n is 0) to compute.
int check_gemm_args(int mode, int m, int n, int k, const float* a, const float* b,
                    const void* workspace, uint64_t workspace_bytes, bool need_c, const float* c,
                    bool* trivial) {
    *trivial = false;
    if (mode != ZG_GEMM_SIMT_FP32 && mode != ZG_GEMM_TF32X3 && mode != ZG_GEMM_TF32)
        return set_error(ZG_ERR_DISPATCH, "sgemm: unknown mode %d", mode);
    if (m < 0 || n < 0 || k < 0)
        return set_error(ZG_ERR_DISPATCH, "sgemm: negative shape %d x %d x %d", m, n, k);
    if (m == 0 || n == 0) {
        *trivial = true;
        return ZG_OK;
    }
    if ((need_c && !c) || (k > 0 && (!a || !b)))
        return set_error(ZG_ERR_DISPATCH, "sgemm: null operand pointer");
    const uint64_t need = k > 0 ? ws_layout(mode, m, n, k).total : 0;
    if (need > 0 && (!workspace || workspace_bytes < need))
        return set_error(ZG_ERR_DISPATCH,
                         "sgemm: workspace of %llu bytes needed for %d x %d x %d, got %llu",
                         (unsigned long long)need, m, n, k, (unsigned long long)workspace_bytes);
    if (need > 0 && (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return set_error(ZG_ERR_DISPATCH, "sgemm: workspace must be 256-byte aligned");
    return ZG_OK;
}

}  // namespace
}  // namespace zg

using namespace zg;

extern "C" uint64_t zg_sgemm_workspace_bytes(int mode, int m, int n, int k) {
    if (m <= 0 || n <= 0 || k <= 0) return 0;
    return ws_layout(mode, m, n, k).total;
}

extern "C" int zg_sgemm_prepare(int mode, int m, int n, int k, const float* a, const float* b,
                                void* workspace, uint64_t workspace_bytes, void* stream) {
    bool trivial;
    int rc = check_gemm_args(mode, m, n, k, a, b, workspace, workspace_bytes, false, nullptr,
                             &trivial);
    if (rc || trivial || k == 0 || mode == ZG_GEMM_SIMT_FP32) return rc;
    return prepare_planes(mode, m, n, k, a, b, static_cast<uint8_t*>(workspace),
                          static_cast<cudaStream_t>(stream));
}

extern "C" int zg_sgemm_compute(int mode, int m, int n, int k, float alpha, const float* a,
                                const float* b, float* c, const float* bias, int relu,
                                const void* workspace, uint64_t workspace_bytes, void* stream) {
    bool trivial;
    int rc = check_gemm_args(mode, m, n, k, a, b, workspace, workspace_bytes, true, c, &trivial);
    if (rc || trivial) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (k == 0) {
        gemm_k0_kernel<<<split_grid(m), 256, 0, s>>>(m, n, alpha, c, bias, relu);
        return cuda_status(cudaGetLastError(), "sgemm k=0");
    }
    const GemmOperands op =
        operands_in_workspace(mode, m, n, k, a, b, static_cast<const uint8_t*>(workspace));
    return gemm_run(op, m, n, k, alpha, c, n, bias, relu, s);
}

extern "C" int zg_sgemm_f32(int mode, int m, int n, int k, float alpha, const float* a,
                            const float* b, float* c, const float* bias, int relu,
                            void* workspace, uint64_t workspace_bytes, void* stream) {
    int rc = zg_sgemm_prepare(mode, m, n, k, a, b, workspace, workspace_bytes, stream);
    if (rc) return rc;
    return zg_sgemm_compute(mode, m, n, k, alpha, a, b, c, bias, relu, workspace,
                            workspace_bytes, stream);
}

// ---- packed operands ----------------------------------------------------------
// A packed operand is the plane(s) the GEMM kernel of `mode` reads, each
// 256-byte aligned, row pitch kp = k rounded up to 4 floats:
//   A (m x k):  TF32X3 hi, lo;  TF32 one f32 copy;  SIMT one f32 copy.
//   B (k x n):  TF32X3 B^T hi, lo (n x kp, K-major);  TF32 B^T;  SIMT B itself
//               (k rows, pitch round_up(n, 4)).
namespace zg {
namespace {
uint64_t packed_plane_bytes(int mode, int operand, int outer, int k) {
    if (mode == ZG_GEMM_SIMT_FP32 && operand == 1)
        return round_up(static_cast<uint64_t>(k) * round_up(outer, 4) * 4, 256);
    return round_up(static_cast<uint64_t>(outer) * round_up(k, 4) * 4, 256);
}
int packed_planes(int mode) { return mode == ZG_GEMM_TF32X3 ? 2 : 1; }
bool valid_mode(int mode) {
    return mode == ZG_GEMM_SIMT_FP32 || mode == ZG_GEMM_TF32X3 || mode == ZG_GEMM_TF32;
}
}  // namespace
}  // namespace zg

extern "C" uint64_t zg_sgemm_pack_bytes(int mode, int operand, int outer, int k) {
    if (!valid_mode(mode) || (operand != 0 && operand != 1) || outer <= 0 || k <= 0) return 0;
    return packed_planes(mode) * packed_plane_bytes(mode, operand, outer, k);
}

extern "C" int zg_sgemm_pack_a(int mode, int m, int k, const float* a, int64_t lda, void* packed,
                               uint64_t packed_bytes, void* stream) {
    if (!valid_mode(mode)) return set_error(ZG_ERR_DISPATCH, "sgemm pack: unknown mode %d", mode);
    if (m < 0 || k < 0 || lda < k) return set_error(ZG_ERR_DISPATCH, "sgemm pack_a: bad shape");
    if (m == 0 || k == 0) return ZG_OK;
    const uint64_t need = zg_sgemm_pack_bytes(mode, 0, m, k);
    if (!a || !packed || packed_bytes < need || (reinterpret_cast<uintptr_t>(packed) & 255u))
        return set_error(ZG_ERR_DISPATCH,
                         "sgemm pack_a: needs a 256-byte aligned buffer of %llu bytes",
                         (unsigned long long)need);
    float* hi = static_cast<float*>(packed);
    float* lo = mode == ZG_GEMM_TF32X3
                    ? reinterpret_cast<float*>(static_cast<uint8_t*>(packed) +
                                               packed_plane_bytes(mode, 0, m, k))
                    : nullptr;
    return launch_split(a, m, k, lda, hi, lo, gemm_plane_pitch(k), mode == ZG_GEMM_TF32X3 ? 1 : 0,
                        static_cast<cudaStream_t>(stream));
}

extern "C" int zg_sgemm_pack_b(int mode, int k, int n, const float* b, int64_t ldb, void* packed,
                               uint64_t packed_bytes, void* stream) {
    if (!valid_mode(mode)) return set_error(ZG_ERR_DISPATCH, "sgemm pack: unknown mode %d", mode);
    if (n < 0 || k < 0 || ldb < n) return set_error(ZG_ERR_DISPATCH, "sgemm pack_b: bad shape");
    if (n == 0 || k == 0) return ZG_OK;
    const uint64_t need = zg_sgemm_pack_bytes(mode, 1, n, k);
    if (!b || !packed || packed_bytes < need || (reinterpret_cast<uintptr_t>(packed) & 255u))
        return set_error(ZG_ERR_DISPATCH,
                         "sgemm pack_b: needs a 256-byte aligned buffer of %llu bytes",
                         (unsigned long long)need);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* hi = static_cast<float*>(packed);
    if (mode == ZG_GEMM_SIMT_FP32)
        return launch_split(b, k, n, ldb, hi, nullptr, static_cast<int64_t>(round_up(n, 4)), 0, s);
    float* lo = mode == ZG_GEMM_TF32X3
                    ? reinterpret_cast<float*>(static_cast<uint8_t*>(packed) +
                                               packed_plane_bytes(mode, 1, n, k))
                    : nullptr;
    return gemm_prep_b(mode, k, n, b, ldb, hi, lo, gemm_plane_pitch(k), s);
}

extern "C" int zg_sgemm_packed(int mode, int m, int n, int k, float alpha, const void* a_packed,
                               const void* b_packed, float* c, int64_t ldc, const float* bias,
                               int relu, void* stream) {
    if (!valid_mode(mode)) return set_error(ZG_ERR_DISPATCH, "sgemm: unknown mode %d", mode);
    if (m < 0 || n < 0 || k < 0 || ldc < n)
        return set_error(ZG_ERR_DISPATCH, "sgemm_packed: bad shape %d x %d x %d, ldc %lld", m, n,
                         k, (long long)ldc);
    if (m == 0 || n == 0) return ZG_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!c) return set_error(ZG_ERR_DISPATCH, "sgemm_packed: null C");
    if (k == 0) {
        if (ldc != n) return set_error(ZG_ERR_DISPATCH, "sgemm_packed: k = 0 needs ldc = n");
        gemm_k0_kernel<<<split_grid(m), 256, 0, s>>>(m, n, alpha, c, bias, relu);
        return cuda_status(cudaGetLastError(), "sgemm k=0");
    }
    if (!a_packed || !b_packed) return set_error(ZG_ERR_DISPATCH, "sgemm_packed: null operand");
    const uint8_t* pa = static_cast<const uint8_t*>(a_packed);
    const uint8_t* pb = static_cast<const uint8_t*>(b_packed);
    GemmOperands op{mode, reinterpret_cast<const float*>(pa), nullptr, gemm_plane_pitch(k),
                    reinterpret_cast<const float*>(pb), nullptr, gemm_plane_pitch(k)};
    if (mode == ZG_GEMM_TF32X3) {
        op.a_lo = reinterpret_cast<const float*>(pa + packed_plane_bytes(mode, 0, m, k));
        op.b_lo = reinterpret_cast<const float*>(pb + packed_plane_bytes(mode, 1, n, k));
    }
    if (mode == ZG_GEMM_SIMT_FP32) op.ldb = static_cast<int64_t>(round_up(n, 4));
    return gemm_run(op, m, n, k, alpha, c, ldc, bias, relu, s);
}

extern "C" int zg_kernel_status(uint32_t* code) {
    uint32_t v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_status, &zero, sizeof(zero));
    if (code) *code = v;
    return cuda_status(e, "zg_kernel_status");
}
