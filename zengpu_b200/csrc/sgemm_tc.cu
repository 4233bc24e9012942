// sgemm_tc.cu - tcgen05 / TMEM tensor-core SGEMM for sm_100a, and the GEMM
// dispatcher behind zg_sgemm_f32 (the kernel contract of GEMM_PTX's entry
// `main(a, b, c, m, n, k, alpha)`, zengpu-blas/src/level3.rs:35-90).
//
// Four tensor-core modes share one kernel template (S = operand scheme):
//   TF32 (S=1)         one kind::tf32 MMA per k-step on f32 operands;
//   TF32X3 (S=2)       split precision: x = hi + lo, hi = tf32(x),
//                      lo = tf32(x - hi) (round to nearest both);
//                      D += A_lo*B_hi + A_hi*B_lo + A_hi*B_hi, three
//                      kind::tf32 MMAs; the dropped lo*lo term is ~2^-22;
//   TF32_BF16X2 (S=3)  the same split, but the two correction products, which
//                      only need ~2^-19 relative precision, run as one
//                      kind::f16 bf16 MMA each (twice the tf32 rate):
//                      D += bf16(A_lo)*bf16(B_hi) + bf16(A_hi)*bf16(B_lo)
//                         + A_hi*B_hi (tf32): 2/3 of TF32X3's MMA time;
//   BF16X3 (S=4)       x = hi + lo with hi = bf16(x), lo = bf16(x - hi);
//                      D += A_lo*B_hi + A_hi*B_lo + A_hi*B_hi as three
//                      kind::f16 bf16 MMAs (products exact in f32; the
//                      dropped lo*lo and the residue below lo are ~2^-16):
//                      1/2 of TF32X3's MMA time and half its operand bytes.
// A pre-pass writes the operands in the layout the kernel reads: A with k
// innermost, B transposed to K-major, and for the split modes every block of
// k of a row packed into one 128-byte row holding all of that block's terms
// (TF32X3, 16 k: 16 tf32 hi | 16 tf32 lo; TF32_BF16X2, 16 k: 16 tf32 hi | 16
// bf16 hi | 16 bf16 lo; BF16X3, 32 k: 32 bf16 hi | 32 bf16 lo).  Full
// 128-byte rows keep the TMA engine at full rate: one box per operand per
// stage, one 128-byte swizzle for every term, and each MMA descriptor is an
// offset into the same swizzled rows.
//
// Kernel layout (persistent, one CTA per SM, 128 x 256 output tiles, 320
// threads):
//   warp 0      TMA producer: per stage one 2-D load of A [128 rows x 128 B]
//               and one of B^T [256 rows x 128 B], 128-byte swizzled, into a
//               4-stage mbarrier ring (48 KB per stage);
//   warp 1      allocates 512 TMEM columns (two 128 x 256 f32 accumulators,
//               lane = row) and one thread issues the MMAs, committing each
//               stage back to the producer and each finished k-chunk to the
//               epilogue;
//   warps 2-9   epilogue, two warps per TMEM lane quarter (one per 128-column
//               half).  The tensor core's f32 accumulation truncates, so its
//               error grows with k; for the split modes the epilogue drains
//               the TMEM accumulator every 512 of k into f32 registers (round
//               to nearest) while the MMA fills the other accumulator, then
//               applies alpha / bias / ReLU and stores with 128-bit writes.
//               The chunk pipeline runs on across tiles, so a tile's final
//               drain and store overlap the next tile's MMAs.
// Problems with a 256 x 256 tile for every SM pair run the CTA-pair variant
// (sgemm_tc_pair_kernel: tcgen05 cta_group::2, M = 256, six 32 KB stages per
// CTA); when its last wave would occupy at most half of the pairs, that wave's
// tiles run as 256 x 128 halves (N = 128 MMAs), one per pair.  A GemmGate lets a GEMM start while its B^T rows are still arriving
// from another GPU: the producer waits for the chunk flag of each tile's B
// rows before loading them.
// Every mbarrier and flag wait is bounded (zg_common.cuh); an expiry sets a
// bit in the device status word, the kernel drains its in-flight copies and
// MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "zg_common.cuh"
#include "zg_gemm_internal.h"

namespace zg {

__device__ uint32_t g_status = 0;

int launch_sgemm_simt(int M, int N, int K, float alpha, const float* A, int64_t lda,
                      const float* B, int64_t ldb, float* C, int64_t ldc, const float* bias,
                      int relu, cudaStream_t stream);
int launch_sgemm_simt_at(int M, int N, int K, float alpha, const float* At, int64_t ldat,
                         const float* B, int64_t ldb, float* C, int64_t ldc, const float* bias,
                         int relu, cudaStream_t stream);

namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int kEpiWarps = 8;
constexpr int kTcThreads = 64 + 32 * kEpiWarps;  // producer, MMA, 8 epilogue warps
constexpr uint32_t kTmemCols = 512;              // two BN-column accumulators

// Per-scheme stage geometry: every operand row of a stage is 128 bytes (BK
// values of k: 32 f32 for TF32, 16 interleaved split values otherwise).
template <int S>
struct TcCfg {
    static constexpr int BK = (S == 1 || S == 4) ? 32 : 16;  // k per stage
    static constexpr int STAGES = 4;
    static constexpr int ROW = 128;              // bytes per operand row per stage
    static constexpr int A_BYTES = BM * ROW;
    static constexpr int B_BYTES = BN * ROW;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 48 KB
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*bars*/;
    // k-blocks per TMEM accumulation chunk: 512 of k for the split modes
    // (keeps the accumulator's truncation error near 3e-6 relative); TF32
    // (tolerance 5e-3) accumulates the whole k range in TMEM.
    static constexpr int KB_PER_CHUNK = S >= 2 ? 512 / BK : (1 << 30);
};

struct TcMaps {
    CUtensorMap a;
    CUtensorMap b;
    CUtensorMap b_half;  // CTA pairs: B^T in 64-row boxes, for the half-width tail units
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

// Instruction descriptors, M = 128, N = 256, D f32, both operands K-major:
// kind::tf32 (A, B format 2 = TF32) and kind::f16 with bf16 (format 1).
constexpr uint32_t kIdescShape =
    (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);
constexpr uint32_t kIdescTf32 = (1u << 4) | (2u << 7) | (2u << 10) | kIdescShape;
constexpr uint32_t kIdescBf16 = (1u << 4) | (1u << 7) | (1u << 10) | kIdescShape;

// Grouped raster: consecutive tiles walk down kGroupM row-tiles before moving
// right, so tiles in flight together share A row-blocks and B column-blocks in L2.
// Measured at 8192^3 (BF16X3, CTA pairs, DRAM bytes per launch by ncu): groups of
// 4 / 8 / 16 / 32 row-tiles read 4.37 / 3.42 / 3.79 / 6.10 GB; 8 is also the fastest.
constexpr int kGroupM = 8;
__device__ __forceinline__ void tile_coords(int tile, int mt, int nt, int& m_tile, int& n_tile) {
    const int group_size = kGroupM * nt;
    const int group = tile / group_size;
    const int first_m = group * kGroupM;
    const int gm = min(mt - first_m, kGroupM);
    const int r = tile - group * group_size;
    m_tile = first_m + r % gm;
    n_tile = r / gm;
}

// Issues the MMAs of one smem stage into d_tmem; `first` starts a fresh
// accumulation (the first MMA overwrites D).  Every operand is K-major with
// 128-byte swizzled rows (SBO = 8 rows = 1024 B); a term is selected by its
// byte offset inside the row: TF32 k-steps at 32 B apart; TF32X3 hi at +0,
// lo at +64; TF32_BF16X2 tf32 hi at +0, bf16 hi at +64, bf16 lo at +96.
template <int S>
__device__ __forceinline__ void issue_stage(uint32_t d_tmem, uint32_t stage_base, bool first) {
    using Cfg = TcCfg<S>;
    const uint32_t a = stage_base, b = stage_base + Cfg::A_BYTES;
    auto d = [](uint32_t addr) { return umma_desc(addr, 16, 1024, 2); };
    uint32_t acc = first ? 0u : 1u;
    if (S == 4) {
        // BF16X3: per 16 of k (32 bytes of the row) lo*hi, hi*lo, then hi*hi;
        // hi at +0 / +32, lo at +64 / +96
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            const uint32_t ko = kk * 32;
            mma_f16_ss(d_tmem, d(a + 64 + ko), d(b + ko), kIdescBf16, acc);
            acc = 1u;
            mma_f16_ss(d_tmem, d(a + ko), d(b + 64 + ko), kIdescBf16, 1u);
            mma_f16_ss(d_tmem, d(a + ko), d(b + ko), kIdescBf16, 1u);
        }
        return;
    }
    if (S == 3) {
        // bf16 corrections first (small terms into the accumulator first),
        // one K = 16 MMA each covering the whole stage
        mma_f16_ss(d_tmem, d(a + 96), d(b + 64), kIdescBf16, acc);
        acc = 1u;
        mma_f16_ss(d_tmem, d(a + 64), d(b + 96), kIdescBf16, 1u);
    }
#pragma unroll
    for (int kk = 0; kk < (S == 1 ? 4 : 2); ++kk) {
        // K = 8 per tf32 MMA: 32 bytes along the swizzled row
        const uint32_t ko = kk * 32;
        if (S == 2) {
            mma_tf32_ss(d_tmem, d(a + 64 + ko), d(b + ko), kIdescTf32, acc);
            acc = 1u;
            mma_tf32_ss(d_tmem, d(a + ko), d(b + 64 + ko), kIdescTf32, 1u);
        }
        mma_tf32_ss(d_tmem, d(a + ko), d(b + ko), kIdescTf32, acc);
        acc = 1u;
    }
}

template <int S>
__global__ void __launch_bounds__(kTcThreads, 1)
    sgemm_tc_kernel(const __grid_constant__ TcMaps maps, int M, int N, int K, float alpha,
                    float* __restrict__ C, int64_t ldc, const float* __restrict__ bias, int relu,
                    int vec_c, const GemmGate gate) {
    using Cfg = TcCfg<S>;
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
        prefetch_tensormap(&maps.a);
        prefetch_tensormap(&maps.b);
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
                if (gate.flags && !flag_wait_bounded(gate.flags + n0 / gate.rows, gate.epoch,
                                                     &g_status, kErrTcGate)) {
                    ok = false;
                    break;
                }
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait_bounded(&empty[s], ph ^ 1, &g_status, kErrTcProducer)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
                    uint8_t* st = smem + s * Cfg::STAGE_BYTES;
                    // k-block kb is 32 four-byte units into every row (TF32: 32
                    // f32 of k; split modes: one interleaved 128-byte block)
                    tma_load_2d(st, &maps.a, kb * 32, m0, &full[s]);
                    tma_load_2d(st + Cfg::A_BYTES, &maps.b, kb * 32, n0, &full[s]);
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
                        issue_stage<S>(d_tmem, smem_u32(smem + s * Cfg::STAGE_BYTES), kb == kb0);
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
        const int q = warp & 3;            // TMEM lane quarter this warp may access
        const int half = (warp - 2) >> 2;  // 128-column half of the tile
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
                // the whole warp gives up together: the TMEM loads below are
                // warp-collective, so no lane may go on alone
                const bool got = mbar_wait_bounded(&acc_full[buf], (cj >> 1) & 1, &g_status,
                                                   kErrTcEpilogue);
                if (!__all_sync(0xffffffffu, got)) {
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

// ---- CTA-pair kernel (tcgen05 cta_group::2) -----------------------------------------
// Two CTAs of a cluster compute one 256 x 256 tile: CTA r loads rows
// [128r, 128r + 128) of the tile's A rows and of its B^T rows, and the leader
// (r = 0) issues M = 256, N = 256 MMAs whose A and B halves come from both
// CTAs' shared memory; each CTA's TMEM holds its 128 rows of D.  Per SM a stage
// is 32 KB instead of 48 KB for the same MMA work, so six stages fit and the
// L2 -> SM operand traffic per flop drops by a third.  Loads signal the
// leader's full barrier (no multicast); the leader's commits arrive on both
// CTAs' barriers; every epilogue warp of both CTAs frees a TMEM buffer on the
// leader's barrier.
constexpr int PBM = 256, PBN = 256;

template <int S>
struct PairCfg {
    static constexpr int BK = (S == 1 || S == 4) ? 32 : 16;
    static constexpr int STAGES = 6;
    static constexpr int A_BYTES = 128 * 128;  // this CTA's 128 rows x 128 B
    static constexpr int B_BYTES = 128 * 128;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 32 KB
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*bars*/;
    static constexpr int KB_PER_CHUNK = S >= 2 ? 512 / BK : (1 << 30);
};

constexpr uint32_t kIdescShapePair =
    (static_cast<uint32_t>(PBN >> 3) << 17) | (static_cast<uint32_t>(PBM >> 4) << 24);
constexpr uint32_t kIdescTf32Pair = (1u << 4) | (2u << 7) | (2u << 10) | kIdescShapePair;
constexpr uint32_t kIdescBf16Pair = (1u << 4) | (1u << 7) | (1u << 10) | kIdescShapePair;
// N = 128: the halves of the tiles of the last, partial wave (see launch_tc_pair).
constexpr uint32_t kIdescShapePairHalf =
    (static_cast<uint32_t>((PBN / 2) >> 3) << 17) | (static_cast<uint32_t>(PBM >> 4) << 24);
constexpr uint32_t kIdescTf32PairHalf = (1u << 4) | (2u << 7) | (2u << 10) | kIdescShapePairHalf;
constexpr uint32_t kIdescBf16PairHalf = (1u << 4) | (1u << 7) | (1u << 10) | kIdescShapePairHalf;

template <int S>
__device__ __forceinline__ void issue_stage_pair(uint32_t d_tmem, uint32_t stage_base,
                                                 bool first, bool half) {
    const uint32_t a = stage_base, b = stage_base + PairCfg<S>::A_BYTES;
    auto d = [](uint32_t addr) { return umma_desc(addr, 16, 1024, 2); };
    const uint32_t idesc_bf16 = half ? kIdescBf16PairHalf : kIdescBf16Pair;
    const uint32_t idesc_tf32 = half ? kIdescTf32PairHalf : kIdescTf32Pair;
    uint32_t acc = first ? 0u : 1u;
    if (S == 4) {
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            const uint32_t ko = kk * 32;
            mma_f16_ss_pair(d_tmem, d(a + 64 + ko), d(b + ko), idesc_bf16, acc);
            acc = 1u;
            mma_f16_ss_pair(d_tmem, d(a + ko), d(b + 64 + ko), idesc_bf16, 1u);
            mma_f16_ss_pair(d_tmem, d(a + ko), d(b + ko), idesc_bf16, 1u);
        }
        return;
    }
    if (S == 3) {
        mma_f16_ss_pair(d_tmem, d(a + 96), d(b + 64), idesc_bf16, acc);
        acc = 1u;
        mma_f16_ss_pair(d_tmem, d(a + 64), d(b + 96), idesc_bf16, 1u);
    }
#pragma unroll
    for (int kk = 0; kk < (S == 1 ? 4 : 2); ++kk) {
        const uint32_t ko = kk * 32;
        if (S == 2) {
            mma_tf32_ss_pair(d_tmem, d(a + 64 + ko), d(b + ko), idesc_tf32, acc);
            acc = 1u;
            mma_tf32_ss_pair(d_tmem, d(a + ko), d(b + 64 + ko), idesc_tf32, 1u);
        }
        mma_tf32_ss_pair(d_tmem, d(a + ko), d(b + ko), idesc_tf32, acc);
        acc = 1u;
    }
}

template <int S>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTcThreads, 1)
    sgemm_tc_pair_kernel(const __grid_constant__ TcMaps maps, int M, int N, int K, float alpha,
                         float* __restrict__ C, int64_t ldc, const float* __restrict__ bias,
                         int relu, int vec_c, const GemmGate gate, int full_units,
                         int split) {
    using Cfg = PairCfg<S>;
    constexpr int BK = Cfg::BK, STAGES = Cfg::STAGES;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int mt = (M + PBM - 1) / PBM, nt = (N + PBN - 1) / PBN;
    const int num_tiles = mt * nt;
    const int nkb = (K + BK - 1) / BK;
    const int nchunks = (nkb + Cfg::KB_PER_CHUNK - 1) / Cfg::KB_PER_CHUNK;
    auto tile_origin = [&](int t, int& m0, int& n0) {
        int mi, ni;
        tile_coords(t, mt, nt, mi, ni);
        m0 = mi * PBM;
        n0 = ni * PBN;
    };
    // Unit u: tile u while u < full_units; after that (split == 2) the column
    // halves of the remaining tiles, tile full_units + (u - full_units) / 2,
    // columns [n0 + 128 h, n0 + 128 h + 128) for h = (u - full_units) % 2.
    const int num_units = full_units + (num_tiles - full_units) * split;
    auto unit_half = [&](int u) { return split > 1 && u >= full_units; };
    auto unit_origin = [&](int u, int& m0, int& n0) {
        if (!unit_half(u)) {
            tile_origin(u, m0, n0);
            return;
        }
        tile_origin(full_units + (u - full_units) / split, m0, n0);
        n0 += ((u - full_units) % split) * (PBN / 2);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 2 * kEpiWarps);  // one arrive per epilogue warp, both CTAs
        }
        mbar_init(drain, 1);
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tensormap(&maps.a);
        prefetch_tensormap(&maps.b);
    }
    if (warp == 1) tmem_alloc_pair(tmem_slot, kTmemCols);
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers initialised, TMEM allocated in both
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int t = pair; t < num_units && ok; t += npairs) {
                int m0, n0;
                unit_origin(t, m0, n0);
                const bool half = unit_half(t);
                // both CTAs' B rows lie in the chunk of n0 (chunks are 256-row multiples)
                if (gate.flags && !flag_wait_bounded(gate.flags + n0 / gate.rows, gate.epoch,
                                                     &g_status, kErrTcGate)) {
                    ok = false;
                    break;
                }
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait_bounded(&empty[s], ph ^ 1, &g_status, kErrTcProducer)) {
                        ok = false;
                        break;
                    }
                    // The leader's full barrier counts both CTAs' bytes.
                    if (leader)
                        mbar_arrive_expect_tx(&full[s], 2 * (half ? Cfg::A_BYTES + Cfg::B_BYTES / 2
                                                                  : Cfg::STAGE_BYTES));
                    const uint32_t bar = mapa_shared(&full[s], 0);
                    uint8_t* st = smem + s * Cfg::STAGE_BYTES;
                    tma_load_2d_pair(st, &maps.a, kb * 32, m0 + 128 * rank, bar);
                    if (half)
                        tma_load_2d_pair(st + Cfg::A_BYTES, &maps.b_half, kb * 32, n0 + 64 * rank,
                                         bar);
                    else
                        tma_load_2d_pair(st + Cfg::A_BYTES, &maps.b, kb * 32, n0 + 128 * rank,
                                         bar);
                }
            }
            // No copy of this CTA may still be landing when it exits: wait until
            // the leader's MMAs have consumed the last stages issued.
            const int first = it > STAGES ? it - STAGES : 0;
            for (int i = first; i < it; ++i)
                mbar_wait_bounded(&empty[i % STAGES], (i / STAGES) & 1, &g_status, kErrTcDrain);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (leader only) ----------------
        if (leader && lane == 0) {
            bool ok = true;
            int it = 0, cj = 0;
            for (int t = pair; t < num_units && ok; t += npairs) {
                const bool half = unit_half(t);
                for (int j = 0; j < nchunks && ok; ++j, ++cj) {
                    const int buf = cj & 1;
                    const uint32_t d_tmem = tmem_base + buf * PBN;
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
                        issue_stage_pair<S>(d_tmem, smem_u32(smem + s * Cfg::STAGE_BYTES),
                                            kb == kb0, half);
                        mma_commit_pair(&empty[s], 0x3);  // frees stage s in both CTAs
                    }
                    if (ok) mma_commit_pair(&acc_full[buf], 0x3);
                }
            }
            if (!ok) {
                mma_commit_pair(drain, 0x1);
                mbar_wait_bounded(drain, 0, &g_status, kErrTcDrain);
            }
        }
    } else {
        // ---------------- epilogue (warps 2..9, both CTAs) ----------------
        const int q = warp & 3;
        const int half = (warp - 2) >> 2;
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + half * 128;
        const uint32_t leader_empty0 = mapa_shared(&acc_empty[0], 0);
        const uint32_t leader_empty1 = mapa_shared(&acc_empty[1], 0);
        bool ok = true;
        int cj = 0;
        for (int t = pair; t < num_units && ok; t += npairs) {
            int m0, n0;
            unit_origin(t, m0, n0);
            // a half-width unit has 128 columns: the second column half's warps
            // keep in step with the barriers but load and store nothing
            const bool cols = !unit_half(t) || half == 0;
            const int row = m0 + 128 * static_cast<int>(rank) + q * 32 + lane;
            float acc[128];
#pragma unroll
            for (int i = 0; i < 128; ++i) acc[i] = 0.0f;
            for (int j = 0; j < nchunks; ++j, ++cj) {
                const int buf = cj & 1;
                // the whole warp gives up together: the TMEM loads below are
                // warp-collective, so no lane may go on alone
                const bool got = mbar_wait_bounded(&acc_full[buf], (cj >> 1) & 1, &g_status,
                                                   kErrTcEpilogue);
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (cols) {
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) {
                        uint32_t r[32];
                        tmem_ld_32x32b_x32(lane_base + buf * PBN + cc * 32, r);
#pragma unroll
                        for (int u = 0; u < 32; ++u) acc[cc * 32 + u] += __uint_as_float(r[u]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(buf ? leader_empty1 : leader_empty0);
            }
            if (ok && cols && row < M) {
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
    cluster_sync();  // no CTA leaves while its peer may still signal its barriers
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}

// ---- operand pre-pass ------------------------------------------------------------
// Layout of one operand view row: TF32 (S = 1): f32 copy; TF32X3 (S = 2):
// block kb = k / 16 holds tf32(x) at [kb*32 + j] and tf32(x - hi) at
// [kb*32 + 16 + j]; TF32_BF16X2 (S = 3): tf32(x) at [kb*32 + j], then 16
// bf16(hi) and 16 bf16(x - hi) in the block's last 64 bytes; j = k % 16.
// BF16X3 (S = 4): 32-k blocks of 32 bf16(x) then 32 bf16(x - hi).  x = 0 for
// padding k, so the padding is zero.
// Four consecutive k (k % 4 == 0) of one row with vector stores.
template <int S>
__device__ __forceinline__ void put_value4(float* base, int64_t ld, int64_t r, int k, float4 x) {
    float* row = base + r * ld;
    if (S == 1) {
        *reinterpret_cast<float4*>(row + k) = x;
        return;
    }
    if (S == 4) {
        const float xs[4] = {x.x, x.y, x.z, x.w};
        float hf[4], lf[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            hf[u] = __bfloat162float(__float2bfloat16_rn(xs[u]));
            lf[u] = __fsub_rn(xs[u], hf[u]);
        }
        __nv_bfloat162 bh[2] = {__floats2bfloat162_rn(hf[0], hf[1]),
                                __floats2bfloat162_rn(hf[2], hf[3])};
        __nv_bfloat162 bl[2] = {__floats2bfloat162_rn(lf[0], lf[1]),
                                __floats2bfloat162_rn(lf[2], lf[3])};
        __nv_bfloat16* bb = reinterpret_cast<__nv_bfloat16*>(row + (k >> 5) * 32);
        const int j = k & 31;
        *reinterpret_cast<uint2*>(bb + j) = *reinterpret_cast<uint2*>(bh);
        *reinterpret_cast<uint2*>(bb + 32 + j) = *reinterpret_cast<uint2*>(bl);
        return;
    }
    const float xs[4] = {x.x, x.y, x.z, x.w};
    float h[4], l[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        h[u] = to_tf32(xs[u]);
        l[u] = __fsub_rn(xs[u], h[u]);
    }
    float* blk = row + (k >> 4) * 32;
    const int j = k & 15;
    *reinterpret_cast<float4*>(blk + j) = make_float4(h[0], h[1], h[2], h[3]);
    if (S == 2) {
        *reinterpret_cast<float4*>(blk + 16 + j) =
            make_float4(to_tf32(l[0]), to_tf32(l[1]), to_tf32(l[2]), to_tf32(l[3]));
    } else {
        __nv_bfloat162 bh[2] = {__floats2bfloat162_rn(h[0], h[1]), __floats2bfloat162_rn(h[2], h[3])};
        __nv_bfloat162 bl[2] = {__floats2bfloat162_rn(l[0], l[1]), __floats2bfloat162_rn(l[2], l[3])};
        __nv_bfloat16* bb = reinterpret_cast<__nv_bfloat16*>(blk + 16);
        *reinterpret_cast<uint2*>(bb + j) = *reinterpret_cast<uint2*>(bh);
        *reinterpret_cast<uint2*>(bb + 16 + j) = *reinterpret_cast<uint2*>(bl);
    }
}

// Row-wise pre-pass: rows x K source (pitch lds) -> view with kpad k per row
// (kpad a multiple of 4; k >= K written as zero).  blockIdx.y strides rows.
template <int S>
__global__ void __launch_bounds__(256)
    prep_rows_kernel(const float* __restrict__ src, int rows, int K, int64_t lds, float* dst,
                     int64_t ldd, int kpad, int vec) {
    const int k = (blockIdx.x * 256 + threadIdx.x) * 4;
    if (k >= kpad) return;
    for (int r = blockIdx.y; r < rows; r += gridDim.y) {
        const float* s = src + static_cast<int64_t>(r) * lds;
        float4 x;
        if (vec && k + 3 < K) {
            x = __ldcs(reinterpret_cast<const float4*>(s + k));
        } else {
            x.x = k + 0 < K ? s[k + 0] : 0.f;
            x.y = k + 1 < K ? s[k + 1] : 0.f;
            x.z = k + 2 < K ? s[k + 2] : 0.f;
            x.w = k + 3 < K ? s[k + 3] : 0.f;
        }
        put_value4<S>(dst, ldd, r, k, x);
    }
}

// Transposing pre-pass for B: view row n, k from a K x N source (pitch lds).
// A CTA takes a 32-column strip of B over kTransposeTiles tiles of 64 k
// (blockIdx.x = group of k tiles, blockIdx.y = strip): each tile passes
// through a 64 x 33 shared tile so reads and writes are both coalesced.  Each
// thread keeps eight loads in flight, and the next tile's loads are issued
// before the current tile is stored (the shared tile is double buffered, one
// barrier per tile).  k in [K, kpad) is written as zero.
constexpr int kTransposeTileK = 64;
constexpr int kTransposeTiles = 4;

template <int S>
__device__ __forceinline__ void transpose_strip(const float* __restrict__ src, int K, int N,
                                                int64_t lds, float* dst, int64_t ldd, int kpad,
                                                int n0, int kt0, int kt1) {
    constexpr int TK = kTransposeTileK;
    __shared__ float tile[2][TK][33];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    float r[TK / 8];
    auto load = [&](int kt) {
#pragma unroll
        for (int j = 0; j < TK / 8; ++j) {
            const int k = kt * TK + ty + 8 * j, n = n0 + tx;
            r[j] = (k < K && n < N) ? __ldcs(src + static_cast<int64_t>(k) * lds + n) : 0.f;
        }
    };
    if (kt0 < kt1) load(kt0);
    for (int kt = kt0; kt < kt1; ++kt) {
        const int b = (kt - kt0) & 1;
#pragma unroll
        for (int j = 0; j < TK / 8; ++j) tile[b][ty + 8 * j][tx] = r[j];
        __syncthreads();
        if (kt + 1 < kt1) load(kt + 1);
        // 32 rows n x 64 k: each thread packs four consecutive k of one row n
        // (two such groups) and writes them with the row pre-pass's vector
        // stores; the 16 threads of a row cover its 64 k, so a row's output
        // lines are written whole
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int nl = (threadIdx.x >> 4) + 16 * i, kl = (threadIdx.x & 15) * 4;
            const int n = n0 + nl, k = kt * TK + kl;
            if (n < N && k < kpad)  // kpad is a multiple of 4: k + 3 < kpad too
                put_value4<S>(dst, ldd, n, k,
                              make_float4(tile[b][kl][nl], tile[b][kl + 1][nl],
                                          tile[b][kl + 2][nl], tile[b][kl + 3][nl]));
        }
    }
}

template <int S>
__global__ void __launch_bounds__(256)
    prep_transpose_kernel(const float* __restrict__ src, int K, int N, int64_t lds, float* dst,
                          int64_t ldd, int kpad) {
    const int kt_total = (kpad + kTransposeTileK - 1) / kTransposeTileK;
    const int kt0 = blockIdx.x * kTransposeTiles;
    transpose_strip<S>(src, K, N, lds, dst, ldd, kpad, blockIdx.y * 32, kt0,
                       min(kt_total, kt0 + kTransposeTiles));
}

// The transpose pre-pass for a chunked hand-off: the k-tile groups of a strip
// are the fastest grid dimension, so column strips (and chunks of chunk_cols
// columns) finish in order, and the last CTA of chunk c publishes flags[c] =
// epoch with a system-scope release (the copy engine and other GPUs read the
// chunk after seeing it).  counters[] (one per chunk) start at zero.
template <int S>
__global__ void __launch_bounds__(256)
    prep_transpose_signal_kernel(const float* __restrict__ src, int K, int N, int64_t lds,
                                 float* dst, int64_t ldd, int kpad, int chunk_cols,
                                 uint32_t* counters, uint32_t* flags, uint32_t epoch) {
    const int kt_total = (kpad + kTransposeTileK - 1) / kTransposeTileK;
    const int kt0 = blockIdx.x * kTransposeTiles;
    const int n0 = blockIdx.y * 32;
    transpose_strip<S>(src, K, N, lds, dst, ldd, kpad, n0, kt0,
                       min(kt_total, kt0 + kTransposeTiles));
    __threadfence();  // this thread's part of the chunk, before the CTA is counted
    __syncthreads();
    if (threadIdx.x == 0) {
        const int c = n0 / chunk_cols;
        const int c_end = min(N, (c + 1) * chunk_cols);
        const uint32_t expected =
            static_cast<uint32_t>((c_end - c * chunk_cols + 31) / 32) * gridDim.x;
        uint32_t prev;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                     : "=r"(prev)
                     : "l"(counters + c)
                     : "memory");
        if (prev + 1 == expected)
            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flags + c), "r"(epoch)
                         : "memory");
    }
}

// Plain pitched copy (SIMT packing of B).
__global__ void __launch_bounds__(256)
    copy_rows_kernel(const float* __restrict__ src, int rows, int cols, int64_t lds,
                     float* __restrict__ dst, int64_t ldd) {
    for (int r = blockIdx.x; r < rows; r += gridDim.x)
        for (int c = threadIdx.x; c < cols; c += blockDim.x) dst[r * ldd + c] = src[r * lds + c];
}

// C = epilogue(alpha * 0) for K == 0 (an empty sum, as the reference loop).
__global__ void gemm_k0_kernel(int M, int N, float alpha, float* C, int64_t ldc,
                               const float* bias, int relu) {
    const int64_t total = static_cast<int64_t>(M) * N;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / N, c = i - r * N;
        float x = __fmul_rn(alpha, 0.0f);
        if (bias) x = __fadd_rn(x, bias[c]);
        if (relu) x = relu1(x);
        C[r * ldc + c] = x;
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

uint64_t round_up(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
int sm_count() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms > 0 ? sms : 148;
}

// 2-D map over `rows` rows of `cols` 4-byte units, pitch `ld` units, box
// {32 units (128 B), box_rows}, 128-byte swizzle.
int encode_map(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t ld,
               uint32_t box_rows) {
    return encode_f32_map(map, base, cols, rows, ld, 32, box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

unsigned row_grid(int rows) {
    const int cap = sm_count() * 8;
    return static_cast<unsigned>(rows < cap ? (rows < 1 ? 1 : rows) : cap);
}

bool valid_mode(int mode) {
    return mode == ZG_GEMM_SIMT_FP32 || mode == ZG_GEMM_TF32X3 || mode == ZG_GEMM_TF32 ||
           mode == ZG_GEMM_TF32_BF16X2 || mode == ZG_GEMM_BF16X3;
}

// Kernel scheme of a tensor-core mode (0: SIMT).
int scheme_of(int mode) {
    return mode == ZG_GEMM_TF32 ? 1 : mode == ZG_GEMM_TF32X3 ? 2
                                  : mode == ZG_GEMM_TF32_BF16X2 ? 3
                                  : mode == ZG_GEMM_BF16X3 ? 4 : 0;
}

// k values stored per row of a prepared operand and its pitch (4-byte units).
int64_t view_kpad(int mode, int K) {
    const int sch = scheme_of(mode);
    return sch == 1 ? static_cast<int64_t>(round_up(K, 4))
                    : static_cast<int64_t>(round_up(K, sch == 4 ? 32 : 16));
}
// TF32: one f32 per k; TF32X3 / TF32_BF16X2: 8 bytes per k; BF16X3: 4.
int64_t view_pitch(int mode, int K) {
    const int sch = scheme_of(mode);
    return (sch == 1 || sch == 4) ? view_kpad(mode, K) : view_kpad(mode, K) * 2;
}
// 4-byte units of the global inner dimension the tensor map covers.
uint64_t map_cols(int mode, int K) {
    return scheme_of(mode) == 1 ? static_cast<uint64_t>(K) : static_cast<uint64_t>(view_pitch(mode, K));
}

int launch_prep_rows(int mode, const float* src, int rows, int K, int64_t lds,
                     const OperandView& v, cudaStream_t s) {
    if (rows == 0 || K == 0) return ZG_OK;
    const int kpad = static_cast<int>(view_kpad(mode, K));
    const int vec = lds % 4 == 0 && aligned16(src);
    dim3 grid((kpad / 4 + 255) / 256, static_cast<unsigned>(std::min(rows, 65535)));
    float* dst = static_cast<float*>(v.p);
    switch (scheme_of(mode)) {
        case 1: prep_rows_kernel<1><<<grid, 256, 0, s>>>(src, rows, K, lds, dst, v.ld, kpad, vec); break;
        case 2: prep_rows_kernel<2><<<grid, 256, 0, s>>>(src, rows, K, lds, dst, v.ld, kpad, vec); break;
        case 3: prep_rows_kernel<3><<<grid, 256, 0, s>>>(src, rows, K, lds, dst, v.ld, kpad, vec); break;
        case 4: prep_rows_kernel<4><<<grid, 256, 0, s>>>(src, rows, K, lds, dst, v.ld, kpad, vec); break;
        default: return set_error(ZG_ERR_DISPATCH, "sgemm pre-pass: no planes for mode %d", mode);
    }
    return cuda_status(cudaGetLastError(), "sgemm split pre-pass");
}

int launch_prep_transpose(int mode, const float* src, int K, int N, int64_t lds,
                          const OperandView& v, cudaStream_t s) {
    if (K == 0 || N == 0) return ZG_OK;
    const int kpad = static_cast<int>(view_kpad(mode, K));
    const int kgroups =
        ((kpad + kTransposeTileK - 1) / kTransposeTileK + kTransposeTiles - 1) / kTransposeTiles;
    dim3 grid(kgroups, (N + 31) / 32);
    if (grid.y > 65535u) return set_error(ZG_ERR_DISPATCH, "sgemm: n too large for the pre-pass");
    float* dst = static_cast<float*>(v.p);
    switch (scheme_of(mode)) {
        case 1: prep_transpose_kernel<1><<<grid, 256, 0, s>>>(src, K, N, lds, dst, v.ld, kpad); break;
        case 2: prep_transpose_kernel<2><<<grid, 256, 0, s>>>(src, K, N, lds, dst, v.ld, kpad); break;
        case 3: prep_transpose_kernel<3><<<grid, 256, 0, s>>>(src, K, N, lds, dst, v.ld, kpad); break;
        case 4: prep_transpose_kernel<4><<<grid, 256, 0, s>>>(src, K, N, lds, dst, v.ld, kpad); break;
        default: return set_error(ZG_ERR_DISPATCH, "sgemm pre-pass: no planes for mode %d", mode);
    }
    return cuda_status(cudaGetLastError(), "sgemm transpose pre-pass");
}

int launch_prep_transpose_signal(int mode, const float* src, int K, int N, int64_t lds,
                                 const OperandView& v, int chunk_cols, uint32_t* counters,
                                 uint32_t* flags, uint32_t epoch, cudaStream_t s) {
    if (K == 0 || N == 0) return ZG_OK;
    const int kpad = static_cast<int>(view_kpad(mode, K));
    const int chunks = (N + chunk_cols - 1) / chunk_cols;
    const int kgroups =
        ((kpad + kTransposeTileK - 1) / kTransposeTileK + kTransposeTiles - 1) / kTransposeTiles;
    dim3 grid(kgroups, (N + 31) / 32);
    if (grid.y > 65535u) return set_error(ZG_ERR_DISPATCH, "sgemm: n too large for the pre-pass");
    cudaError_t e = cudaMemsetAsync(counters, 0, static_cast<size_t>(chunks) * sizeof(uint32_t), s);
    if (e != cudaSuccess) return cuda_status(e, "sgemm chunked pre-pass: counters");
    float* dst = static_cast<float*>(v.p);
    switch (scheme_of(mode)) {
        case 1: prep_transpose_signal_kernel<1><<<grid, 256, 0, s>>>(src, K, N, lds, dst, v.ld, kpad, chunk_cols, counters, flags, epoch); break;
        case 2: prep_transpose_signal_kernel<2><<<grid, 256, 0, s>>>(src, K, N, lds, dst, v.ld, kpad, chunk_cols, counters, flags, epoch); break;
        case 3: prep_transpose_signal_kernel<3><<<grid, 256, 0, s>>>(src, K, N, lds, dst, v.ld, kpad, chunk_cols, counters, flags, epoch); break;
        case 4: prep_transpose_signal_kernel<4><<<grid, 256, 0, s>>>(src, K, N, lds, dst, v.ld, kpad, chunk_cols, counters, flags, epoch); break;
        default: return set_error(ZG_ERR_DISPATCH, "sgemm pre-pass: no planes for mode %d", mode);
    }
    return cuda_status(cudaGetLastError(), "sgemm chunked transpose pre-pass");
}

// The opt-in shared-memory size is a per-device attribute of a kernel: it is
// set the first time the kernel is launched on each device of the process.
template <typename Kern>
cudaError_t ensure_smem_attr(Kern* kern, int bytes, std::atomic<uint64_t>& done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev < 64 ? (uint64_t{1} << dev) : 0;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_release);
    return e;
}

template <int S>
int launch_tc(const TcMaps& maps, int M, int N, int K, float alpha, float* C, int64_t ldc,
              const float* bias, int relu, cudaStream_t s, const GemmGate& gate) {
    using Cfg = TcCfg<S>;
    static std::atomic<uint64_t> attr_done{0};
    const cudaError_t attr_err = ensure_smem_attr(sgemm_tc_kernel<S>, Cfg::SMEM_BYTES, attr_done);
    if (attr_err != cudaSuccess) return cuda_status(attr_err, "sgemm_tc smem attribute");
    const int mt = (M + BM - 1) / BM, nt = (N + BN - 1) / BN;
    const int vec_c = (ldc % 4 == 0) && aligned16(C);
    // Persistent grid: one CTA per SM (the smem footprint allows no more).
    const int grid = std::min(mt * nt, sm_count());
    sgemm_tc_kernel<S><<<grid, kTcThreads, Cfg::SMEM_BYTES, s>>>(maps, M, N, K, alpha, C, ldc,
                                                                bias, relu, vec_c, gate);
    return cuda_status(cudaGetLastError(), "sgemm_tc");
}

// ZENGPU_GEMM_TAIL_SPLIT=0 keeps whole tiles in the last wave (same bits either way).
bool tail_split_enabled() {
    static const bool enabled = [] {
        const char* e = std::getenv("ZENGPU_GEMM_TAIL_SPLIT");
        return !(e && e[0] == '0');
    }();
    return enabled;
}

template <int S>
int launch_tc_pair(const TcMaps& maps, int M, int N, int K, float alpha, float* C, int64_t ldc,
                   const float* bias, int relu, cudaStream_t s, const GemmGate& gate) {
    using Cfg = PairCfg<S>;
    static std::atomic<uint64_t> attr_done{0};
    const cudaError_t attr_err =
        ensure_smem_attr(sgemm_tc_pair_kernel<S>, Cfg::SMEM_BYTES, attr_done);
    if (attr_err != cudaSuccess) return cuda_status(attr_err, "sgemm_tc_pair smem attribute");
    const int tiles = ((M + PBM - 1) / PBM) * ((N + PBN - 1) / PBN);
    const int vec_c = (ldc % 4 == 0) && aligned16(C);
    const int pairs_max = std::max(sm_count() / 2, 1);
    // Tail split: when the last wave would keep at most half of the pairs busy,
    // its tiles run as 256 x 128 halves, one per pair (4096^3: 3 waves of 74
    // tiles, then 34 tiles as 68 halves; 1024^3: 16 tiles as 32 halves).  The
    // column width does not change any element's arithmetic.
    const int rem = tiles % pairs_max;
    const bool split = tail_split_enabled() && rem > 0 && 2 * rem <= pairs_max;
    const int full_units = split ? tiles - rem : tiles;
    const int units = full_units + (tiles - full_units) * (split ? 2 : 1);
    // Persistent grid: one CTA pair per two SMs, at most one per unit.
    const int pairs = std::min(units, pairs_max);
    sgemm_tc_pair_kernel<S><<<2 * pairs, kTcThreads, Cfg::SMEM_BYTES, s>>>(
        maps, M, N, K, alpha, C, ldc, bias, relu, vec_c, gate, full_units, split ? 2 : 1);
    return cuda_status(cudaGetLastError(), "sgemm_tc_pair");
}

// CTA pairs from 8 tiles of 256 x 256 up (with fewer tiles than SM pairs, the
// tail split turns up to 37 tiles into twice as many half tiles): measured
// against one CTA per 128 x 256 tile, 1024^3 and 1536^3 run 12-14 % faster
// and 2048^3 the same.  Below 8 tiles, one CTA per 128 x 256 tile.
bool use_pairs(int M, int N) {
    static const bool enabled = [] {
        const char* e = std::getenv("ZENGPU_GEMM_PAIRS");
        return !(e && e[0] == '0');
    }();
    const int tiles = ((M + PBM - 1) / PBM) * ((N + PBN - 1) / PBN);
    return enabled && tiles >= 8;
}

template <int S>
int run_tc(const GemmOperands& op, int M, int N, int K, float alpha, float* C, int64_t ldc,
           const float* bias, int relu, cudaStream_t s, const GemmGate* gate) {
    const GemmGate g = gate ? *gate : GemmGate{};
    if (g.flags && (g.rows <= 0 || g.rows % 256 != 0))
        return set_error(ZG_ERR_DISPATCH, "sgemm: gate chunk of %d rows is not a multiple of 256",
                         g.rows);
    for (const OperandView* v : {&op.a, &op.b})
        if (!v->p || !aligned16(v->p) || v->ld % 4 != 0)
            return set_error(ZG_ERR_DISPATCH,
                             "sgemm (tensor-core mode): operands must be 16-byte aligned with a "
                             "pitch of a multiple of 16 bytes");
    TcMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    const uint64_t cols = map_cols(op.mode, K);
    // TF32's A may be the caller's operand: its map covers exactly K columns
    const uint64_t acols = S == 1 ? static_cast<uint64_t>(K) : cols;
    const bool pairs = use_pairs(M, N);
    // Boxes: 128 rows of A per CTA; B^T 256 rows (one CTA) or 128 (each CTA of a
    // pair; 64 for the half-width tail units).
    int rc = encode_map(&maps.a, op.a.p, acols, M, op.a.ld, BM);
    if (!rc) rc = encode_map(&maps.b, op.b.p, cols, N, op.b.ld, pairs ? 128 : BN);
    if (!rc && pairs) rc = encode_map(&maps.b_half, op.b.p, cols, N, op.b.ld, 64);
    if (rc) return rc;
    if (pairs) return launch_tc_pair<S>(maps, M, N, K, alpha, C, ldc, bias, relu, s, g);
    return launch_tc<S>(maps, M, N, K, alpha, C, ldc, bias, relu, s, g);
}

}  // namespace

int encode_f32_map(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t ld,
                   uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
    auto fn = get_encode_fn();
    if (!fn) return set_error(ZG_ERR_BACKEND, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 4};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(ZG_ERR_BACKEND, "cuTensorMapEncodeTiled failed (%d): %llux%llu ld=%llu",
                         static_cast<int>(r), (unsigned long long)rows, (unsigned long long)cols,
                         (unsigned long long)ld);
    return ZG_OK;
}

// ---- GEMM building blocks (shared with the packed API and the host GEMM) -----------
bool gemm_a_needs_planes(int mode, int K) {
    return mode == ZG_GEMM_TF32X3 || mode == ZG_GEMM_TF32_BF16X2 || mode == ZG_GEMM_BF16X3 ||
           (mode == ZG_GEMM_TF32 && K % 4 != 0);
}
bool gemm_b_needs_planes(int mode) { return scheme_of(mode) > 0; }

uint64_t gemm_planes_bytes(int mode, int outer, int K) {
    if (scheme_of(mode) == 0 || outer <= 0 || K <= 0) return 0;
    return round_up(static_cast<uint64_t>(outer) * view_pitch(mode, K) * 4, 256);
}

OperandView gemm_carve_planes(void* base, int mode, int outer, int K) {
    (void)outer;
    OperandView v;
    v.p = base;
    v.ld = view_pitch(mode, K);
    return v;
}

OperandView gemm_offset_rows(const OperandView& v, int64_t rows) {
    OperandView o = v;
    o.p = static_cast<float*>(v.p) + rows * v.ld;
    return o;
}

OperandView gemm_raw_operand(const float* x, int64_t ld) {
    OperandView v;
    v.p = const_cast<float*>(x);
    v.ld = ld;
    return v;
}

int gemm_prep_a(int mode, int M, int K, const float* A, int64_t lda, const OperandView& out,
                cudaStream_t s) {
    if (!gemm_a_needs_planes(mode, K)) return ZG_OK;
    return launch_prep_rows(mode, A, M, K, lda, out, s);
}

int gemm_prep_b(int mode, int K, int N, const float* B, int64_t ldb, const OperandView& out,
                cudaStream_t s) {
    if (!gemm_b_needs_planes(mode)) return ZG_OK;
    return launch_prep_transpose(mode, B, K, N, ldb, out, s);
}

int gemm_prep_b_signal(int mode, int K, int N, const float* B, int64_t ldb,
                       const OperandView& out, int chunk_cols, uint32_t* counters,
                       uint32_t* flags, uint32_t epoch, cudaStream_t s) {
    if (!gemm_b_needs_planes(mode))
        return set_error(ZG_ERR_DISPATCH, "sgemm: mode %d has no B^T pre-pass", mode);
    if (chunk_cols <= 0 || chunk_cols % 32 != 0)
        return set_error(ZG_ERR_DISPATCH, "sgemm: chunk of %d columns", chunk_cols);
    return launch_prep_transpose_signal(mode, B, K, N, ldb, out, chunk_cols, counters, flags,
                                        epoch, s);
}

int gemm_run(const GemmOperands& op, int M, int N, int K, float alpha, float* C, int64_t ldc,
             const float* bias, int relu, cudaStream_t s, const GemmGate* gate) {
    if (gate && gate->flags && op.mode == ZG_GEMM_SIMT_FP32)
        return set_error(ZG_ERR_DISPATCH, "sgemm: the arrival gate needs a tensor-core mode");
    switch (op.mode) {
        case ZG_GEMM_SIMT_FP32:
            return launch_sgemm_simt(M, N, K, alpha, static_cast<const float*>(op.a.p), op.a.ld,
                                     static_cast<const float*>(op.b.p), op.b.ld, C, ldc, bias,
                                     relu, s);
        case ZG_GEMM_TF32: return run_tc<1>(op, M, N, K, alpha, C, ldc, bias, relu, s, gate);
        case ZG_GEMM_TF32X3: return run_tc<2>(op, M, N, K, alpha, C, ldc, bias, relu, s, gate);
        case ZG_GEMM_TF32_BF16X2:
            return run_tc<3>(op, M, N, K, alpha, C, ldc, bias, relu, s, gate);
        case ZG_GEMM_BF16X3: return run_tc<4>(op, M, N, K, alpha, C, ldc, bias, relu, s, gate);
        default: return set_error(ZG_ERR_DISPATCH, "sgemm: unknown mode %d", op.mode);
    }
}

namespace {

// Workspace of zg_sgemm_f32 / prepare / compute: A's prepared form, then B's.
struct WsLayout {
    uint64_t b_off, total;
    bool a_planes, b_planes;
};

// SIMT's workspace is optional: A transposed (k rows of round_up(m, 4)
// floats) for the TMA-fed kernel.  Without it, or with B not 16-byte aligned
// or n % 4 != 0, SIMT runs the register-staged kernel on A itself (same bits).
uint64_t simt_at_bytes(int m, int k) {
    return round_up(static_cast<uint64_t>(k) * round_up(m, 4) * 4, 256);
}
bool simt_uses_at(int m, int n, int k, const float* b, const void* ws, uint64_t ws_bytes) {
    return m > 0 && n > 0 && k > 0 && ws && ws_bytes >= simt_at_bytes(m, k) &&
           (reinterpret_cast<uintptr_t>(ws) & 255u) == 0 && n % 4 == 0 && aligned16(b) &&
           k <= 65535 * 32;  // the transposing pre-pass grid
}

WsLayout ws_layout(int mode, int m, int n, int k) {
    WsLayout w{0, 0, false, false};
    if (m <= 0 || n <= 0 || k <= 0 || !valid_mode(mode)) return w;
    if (mode == ZG_GEMM_SIMT_FP32) {
        w.total = simt_at_bytes(m, k);
        return w;
    }
    w.a_planes = gemm_a_needs_planes(mode, k);
    w.b_planes = gemm_b_needs_planes(mode);
    w.b_off = w.a_planes ? gemm_planes_bytes(mode, m, k) : 0;
    w.total = w.b_off + (w.b_planes ? gemm_planes_bytes(mode, n, k) : 0);
    return w;
}

GemmOperands operands_in_workspace(int mode, int M, int N, int K, const float* A,
                                   const float* B, uint8_t* ws) {
    const WsLayout w = ws_layout(mode, M, N, K);
    GemmOperands op{mode, gemm_raw_operand(A, K), gemm_raw_operand(B, N)};
    if (w.a_planes) op.a = gemm_carve_planes(ws, mode, M, K);
    if (w.b_planes) op.b = gemm_carve_planes(ws + w.b_off, mode, N, K);
    return op;
}

// Shared argument checks of the workspace entry points.  Returns ZG_OK and
// sets *trivial when there is nothing (m or n is 0) to compute.
int check_gemm_args(int mode, int m, int n, int k, const float* a, const float* b,
                    const void* workspace, uint64_t workspace_bytes, bool need_c, const float* c,
                    bool* trivial) {
    *trivial = false;
    if (!valid_mode(mode)) return set_error(ZG_ERR_DISPATCH, "sgemm: unknown mode %d", mode);
    if (m < 0 || n < 0 || k < 0)
        return set_error(ZG_ERR_DISPATCH, "sgemm: negative shape %d x %d x %d", m, n, k);
    if (m == 0 || n == 0) {
        *trivial = true;
        return ZG_OK;
    }
    if ((need_c && !c) || (k > 0 && (!a || !b)))
        return set_error(ZG_ERR_DISPATCH, "sgemm: null operand pointer");
    const uint64_t need = mode == ZG_GEMM_SIMT_FP32 ? 0 : ws_layout(mode, m, n, k).total;
    if (need > 0 && (!workspace || workspace_bytes < need))
        return set_error(ZG_ERR_DISPATCH,
                         "sgemm: workspace of %llu bytes needed for %d x %d x %d, got %llu",
                         (unsigned long long)need, m, n, k, (unsigned long long)workspace_bytes);
    if (need > 0 && (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return set_error(ZG_ERR_DISPATCH, "sgemm: workspace must be 256-byte aligned");
    return ZG_OK;
}

int launch_k0(int m, int n, float alpha, float* c, int64_t ldc, const float* bias, int relu,
              cudaStream_t s) {
    gemm_k0_kernel<<<row_grid(m), 256, 0, s>>>(m, n, alpha, c, ldc, bias, relu);
    return cuda_status(cudaGetLastError(), "sgemm k=0");
}

// ---- packed operands ----------------------------------------------------------
// A packed operand holds exactly what the mode's kernel reads (OperandView);
// for SIMT, A is an f32 copy with pitch round_up(k, 4) and B an f32 copy of
// its k rows with pitch round_up(n, 4); TF32's A is an f32 copy.
uint64_t simt_packed_bytes(int operand, int outer, int k) {
    return operand == 0 ? round_up(static_cast<uint64_t>(outer) * round_up(k, 4) * 4, 256)
                        : round_up(static_cast<uint64_t>(k) * round_up(outer, 4) * 4, 256);
}

OperandView packed_view(int mode, int operand, const void* packed, int outer, int k) {
    if (mode == ZG_GEMM_SIMT_FP32)
        return gemm_raw_operand(static_cast<const float*>(packed),
                                static_cast<int64_t>(round_up(operand == 0 ? k : outer, 4)));
    return gemm_carve_planes(const_cast<void*>(packed), mode, outer, k);
}

int check_pack(int mode, int outer, int k, int64_t ld, int64_t min_ld, const float* src,
               void* packed, uint64_t bytes, uint64_t need, const char* what) {
    if (!valid_mode(mode)) return set_error(ZG_ERR_DISPATCH, "sgemm pack: unknown mode %d", mode);
    if (outer < 0 || k < 0 || ld < min_ld)
        return set_error(ZG_ERR_DISPATCH, "sgemm %s: bad shape", what);
    if (outer == 0 || k == 0) return ZG_OK;
    if (!src || !packed || bytes < need || (reinterpret_cast<uintptr_t>(packed) & 255u))
        return set_error(ZG_ERR_DISPATCH,
                         "sgemm %s: needs a 256-byte aligned buffer of %llu bytes", what,
                         (unsigned long long)need);
    return ZG_OK;
}

}  // namespace
}  // namespace zg

using namespace zg;

extern "C" uint64_t zg_sgemm_workspace_bytes(int mode, int m, int n, int k) {
    return ws_layout(mode, m, n, k).total;
}

extern "C" int zg_sgemm_prepare(int mode, int m, int n, int k, const float* a, const float* b,
                                void* workspace, uint64_t workspace_bytes, void* stream) {
    bool trivial;
    int rc = check_gemm_args(mode, m, n, k, a, b, workspace, workspace_bytes, false, nullptr,
                             &trivial);
    if (rc || trivial || k == 0) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (mode == ZG_GEMM_SIMT_FP32) {
        if (!simt_uses_at(m, n, k, b, workspace, workspace_bytes)) return ZG_OK;
        // A^T: the f32 transposing pre-pass with A's m rows as its k
        OperandView at;
        at.p = workspace;
        at.ld = round_up(m, 4);
        return launch_prep_transpose(ZG_GEMM_TF32, a, m, k, k, at, s);
    }
    const GemmOperands op =
        operands_in_workspace(mode, m, n, k, a, b, static_cast<uint8_t*>(workspace));
    if ((rc = gemm_prep_a(mode, m, k, a, k, op.a, s))) return rc;
    return gemm_prep_b(mode, k, n, b, n, op.b, s);
}

extern "C" int zg_sgemm_compute(int mode, int m, int n, int k, float alpha, const float* a,
                                const float* b, float* c, const float* bias, int relu,
                                const void* workspace, uint64_t workspace_bytes, void* stream) {
    bool trivial;
    int rc = check_gemm_args(mode, m, n, k, a, b, workspace, workspace_bytes, true, c, &trivial);
    if (rc || trivial) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (k == 0) return launch_k0(m, n, alpha, c, n, bias, relu, s);
    if (mode == ZG_GEMM_SIMT_FP32 && simt_uses_at(m, n, k, b, workspace, workspace_bytes))
        return launch_sgemm_simt_at(m, n, k, alpha, static_cast<const float*>(workspace),
                                    round_up(m, 4), b, n, c, n, bias, relu, s);
    const GemmOperands op = operands_in_workspace(
        mode, m, n, k, a, b, static_cast<uint8_t*>(const_cast<void*>(workspace)));
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

extern "C" uint64_t zg_sgemm_pack_bytes(int mode, int operand, int outer, int k) {
    if (!valid_mode(mode) || (operand != 0 && operand != 1) || outer <= 0 || k <= 0) return 0;
    if (mode == ZG_GEMM_SIMT_FP32) return simt_packed_bytes(operand, outer, k);
    return gemm_planes_bytes(mode, outer, k);
}

extern "C" int zg_sgemm_pack_a(int mode, int m, int k, const float* a, int64_t lda, void* packed,
                               uint64_t packed_bytes, void* stream) {
    int rc = check_pack(mode, m, k, lda, k, a, packed, packed_bytes,
                        zg_sgemm_pack_bytes(mode, 0, m, k), "pack_a");
    if (rc || m == 0 || k == 0) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const OperandView v = packed_view(mode, 0, packed, m, k);
    // SIMT and TF32 store an f32 copy (the TF32 row pre-pass writes exactly that)
    return launch_prep_rows(mode == ZG_GEMM_SIMT_FP32 ? ZG_GEMM_TF32 : mode, a, m, k, lda, v, s);
}

extern "C" int zg_sgemm_pack_b(int mode, int k, int n, const float* b, int64_t ldb, void* packed,
                               uint64_t packed_bytes, void* stream) {
    int rc = check_pack(mode, n, k, ldb, n, b, packed, packed_bytes,
                        zg_sgemm_pack_bytes(mode, 1, n, k), "pack_b");
    if (rc || n == 0 || k == 0) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const OperandView v = packed_view(mode, 1, packed, n, k);
    if (mode == ZG_GEMM_SIMT_FP32) {
        copy_rows_kernel<<<row_grid(k), 256, 0, s>>>(b, k, n, ldb, static_cast<float*>(v.p), v.ld);
        return cuda_status(cudaGetLastError(), "sgemm pack_b");
    }
    return launch_prep_transpose(mode, b, k, n, ldb, v, s);
}

extern "C" int zg_sgemm_packed(int mode, int m, int n, int k, float alpha, const void* a_packed,
                               const void* b_packed, float* c, int64_t ldc, const float* bias,
                               int relu, void* stream) {
    if (!valid_mode(mode)) return set_error(ZG_ERR_DISPATCH, "sgemm: unknown mode %d", mode);
    if (m < 0 || n < 0 || k < 0 || ldc < n)
        return set_error(ZG_ERR_DISPATCH, "sgemm_packed: bad shape %d x %d x %d, ldc %lld", m, n,
                         k, (long long)ldc);
    if (m == 0 || n == 0) return ZG_OK;
    if (!c) return set_error(ZG_ERR_DISPATCH, "sgemm_packed: null C");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (k == 0) return launch_k0(m, n, alpha, c, ldc, bias, relu, s);
    if (!a_packed || !b_packed) return set_error(ZG_ERR_DISPATCH, "sgemm_packed: null operand");
    const GemmOperands op{mode, packed_view(mode, 0, a_packed, m, k),
                          packed_view(mode, 1, b_packed, n, k)};
    return gemm_run(op, m, n, k, alpha, c, ldc, bias, relu, s);
}

extern "C" const char* zg_sgemm_kernel_name(int mode, int m, int n, int k) {
    if (!valid_mode(mode) || m <= 0 || n <= 0 || k < 0) return "";
    if (k == 0) return "gemm_k0_kernel";
    if (mode == ZG_GEMM_SIMT_FP32) return "sgemm_simt_tma_kernel";
    static const char* const pair[] = {"", "sgemm_tc_pair_kernel<1>", "sgemm_tc_pair_kernel<2>",
                                       "sgemm_tc_pair_kernel<3>", "sgemm_tc_pair_kernel<4>"};
    static const char* const single[] = {"", "sgemm_tc_kernel<1>", "sgemm_tc_kernel<2>",
                                         "sgemm_tc_kernel<3>", "sgemm_tc_kernel<4>"};
    const int sch = scheme_of(mode);
    return use_pairs(m, n) ? pair[sch] : single[sch];
}

extern "C" int zg_kernel_status(uint32_t* code) {
    uint32_t v = 0, zero = 0, simt = 0;
    // clear only a word that is set: the common case is two 4-byte reads
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
    if (e == cudaSuccess && v) e = cudaMemcpyToSymbol(g_status, &zero, sizeof(zero));
    if (e == cudaSuccess) e = take_simt_status(&simt);
    if (code) *code = v | simt;
    return cuda_status(e, "zg_kernel_status");
}
