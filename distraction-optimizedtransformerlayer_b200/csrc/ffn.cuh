// The whole MLP of the layer in one kernel, the hidden activation kept on chip:
//
//   h      = GELU(a W1^T + b1)                      a = LN2 output, fp16 [M, D]; never stored
//   x_new  = resid-mode epilogue(h W2^T + b2)       fp32, as gemm_tc_kernel's residual modes
//   normed = LayerNorm(x_new) * ln_w + ln_b          0 on rows norm_row_valid marks 0
//
// Replaces the sequence linear_gelu -> linear_bias -> fused_add_layernorm of
// the reference layer (optimized/layers.py:241-261; linear_gelu.cuh:598-756,
// add_layernorm.cuh:663-692), and is the sm_100a successor of its fused FFN
// kernel (ffn_block.cuh:270-311), which declines every shape above d = 64.
// Covers D = 128 and D = 256 (the GEMM2 accumulator is one TMEM row block of
// D fp32 columns), F any multiple of 128.
//
// Per 128-row block of a (persistent CTAs, one per SM, 320 threads):
//   warp 0      TMA: the block's a (D/64 k-blocks, resident for the block), then
//               W1 / W2 k-blocks of 128 rows x 64 into a ring, in the MMA order;
//   warp 1      tcgen05.mma, for F/128 hidden chunks j, buffer b = j & 1:
//                 G1(j): acc1[b] = a W1[j]^T             (TMEM, 128 fp32 columns)
//                 G2(j): acc2   += H[b] W2[:, j]^T       (A operand read from TMEM)
//               issued G1(0), G1(1), G2(0), G1(2), G2(1), ...; G1(j+2)
//               overwrites acc1[b], where H(j) lives, with no wait: G2(j) was
//               issued before it, and tcgen05 MMAs run in issue order;
//   warps 2-9   per chunk: acc1 -> + b1 -> GELU -> fp16, written back into the
//               columns of acc1[b] it was read from (two fp16 per column), so
//               H never touches shared memory; per block: acc2 -> + b2 +
//               residual -> LayerNorm (two-pass statistics per thread, merged
//               across the two warps of a lane quarter by Chan et al.'s
//               pairwise update) -> direct stores.
// The hidden [M, F] never reaches HBM: per row, D fp16 in and D fp32 (+ D
// normed) out. Weights stream from L2 (F x D x 4 bytes per 128 rows).
//
// Every wait is bounded (2 s): a CTA that gives up sets the device error word,
// drains its copies and MMAs, frees its tensor memory and returns.

#pragma once

#include "gemm_ln.cuh"

namespace dotl {

constexpr int kFfnChunk = 128;            // hidden columns per chunk
constexpr int kFfnThreads = 320;
constexpr uint32_t kFfnTileBytes = kGemmBM * kGemmBK * 2;   // one [128 x 64] fp16 block, 16 KB

struct FfnParams {
    int M, D, F;
    int num_m_tiles;
    const float* b1;              // [F]
    const float* b2;              // [D]
    const float* resid;           // [M, ldr] fp32, or null (resid_mode NONE)
    int64_t ldr;
    const uint8_t* row_valid;
    int resid_mode;               // kResidNone / kResidAdd / kResidAddMaskSub / kResidAddMaskAll
    float* x_out;                 // [M, ldx], or null: x_new not stored
    int64_t ldx;
    const float* ln_w;
    const float* ln_b;
    float eps;
    void* normed;                 // [M, ldn] fp16 or fp32
    int64_t ldn;
    const uint8_t* norm_row_valid;
};

template <int D>
struct FfnSmem {
    static constexpr int kKb = D / kGemmBK;                       // k-blocks of a (and of W1 per chunk)
    static constexpr int kStages = D == 256 ? 6 : 8;              // W ring, 16 KB each
    static constexpr uint32_t kOffA = 0;
    static constexpr uint32_t kOffW = kOffA + kKb * kFfnTileBytes;
    static constexpr uint32_t kOffStats = kOffW + kStages * kFfnTileBytes;   // [2 parity][2 half][128] float2
    // per epilogue warp: a 32 x 32 fp32 block (128B swizzle; residual in,
    // x_new / fp32 normed out) and a 32 x 32 fp16 block (64B swizzle, normed out)
    static constexpr uint32_t kStageWarpBytes = 4096 + 2048;
    static constexpr uint32_t kOffStage = kOffStats + 2 * 2 * kGemmBM * 8;
    static constexpr uint32_t kOffBar = kOffStage + 8 * kStageWarpBytes;
    // a_full, a_empty, w_full[S], w_empty[S], acc1_full[2], h_full[2],
    // acc2_full, acc2_empty, stats[2 parity][4 quarters], drain, resid_full[8 warps]
    static constexpr int kNumBars = 2 + 2 * kStages + 4 + 2 + 8 + 1 + 8;
    static constexpr uint32_t kOffSlot = kOffBar + kNumBars * 8;
    static constexpr uint32_t kOffAbort = kOffSlot + 4;
    static constexpr uint32_t kBytes = kOffAbort + 4;
    static constexpr uint32_t kAlloc = kBytes + 1024;
    static constexpr uint32_t kTmemCols = 512;                    // acc1 x 2 (256) + acc2 (D)
    static constexpr uint32_t kColAcc2 = 2 * kFfnChunk;
};

template <int D>
struct FfnBars {
    using L = FfnSmem<D>;
    uint32_t bar0;
    __device__ __forceinline__ uint32_t a_full() const { return bar0; }
    __device__ __forceinline__ uint32_t a_empty() const { return bar0 + 8; }
    __device__ __forceinline__ uint32_t w_full(int s) const { return bar0 + 8u * (2 + s); }
    __device__ __forceinline__ uint32_t w_empty(int s) const { return bar0 + 8u * (2 + L::kStages + s); }
    __device__ __forceinline__ uint32_t acc1_full(int b) const { return bar0 + 8u * (2 + 2 * L::kStages + b); }
    __device__ __forceinline__ uint32_t h_full(int b) const { return bar0 + 8u * (4 + 2 * L::kStages + b); }
    __device__ __forceinline__ uint32_t acc2_full() const { return bar0 + 8u * (6 + 2 * L::kStages); }
    __device__ __forceinline__ uint32_t acc2_empty() const { return bar0 + 8u * (7 + 2 * L::kStages); }
    __device__ __forceinline__ uint32_t stats(int par, int q) const {
        return bar0 + 8u * (8 + 2 * L::kStages + par * 4 + q);
    }
    __device__ __forceinline__ uint32_t drain() const { return bar0 + 8u * (16 + 2 * L::kStages); }
    __device__ __forceinline__ uint32_t resid_full(int w) const { return bar0 + 8u * (17 + 2 * L::kStages + w); }
};

// The W ring in consumption order: per 128-row block, G1(0), G1(1) [W1 chunk
// j, k-blocks 0..kKb-1], then for j = 0..n-1: G2(j) [W2 k-block h = 0, 1 of
// chunk j, row halves r = 0..D/128-1], G1(j+2) if any. Both sides walk the
// ring with this visitor so producer and MMA cannot disagree on the order.
template <int D, typename G1Fn, typename G2Fn>
__device__ __forceinline__ bool ffn_walk(int n_chunks, G1Fn g1, G2Fn g2) {
    if (!g1(0)) return false;
    if (n_chunks > 1 && !g1(1)) return false;
    for (int j = 0; j < n_chunks; ++j) {
        if (!g2(j)) return false;
        if (j + 2 < n_chunks && !g1(j + 2)) return false;
    }
    return true;
}

template <int D, bool NORM_F16>
__global__ void __launch_bounds__(kFfnThreads, 1)
    ffn_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w1,
               const __grid_constant__ CUtensorMap tmap_w2, const __grid_constant__ CUtensorMap tmap_r,
               const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_n,
               const FfnParams p) {
    using L = FfnSmem<D>;
    constexpr int kS = L::kStages;
    constexpr int kRh = D / 128;                  // 128-row halves of a W2 k-block
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    const FfnBars<D> bars{sbase + L::kOffBar};
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffAbort);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffSlot);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n_chunks = p.F / kFfnChunk;

    if (threadIdx.x == 0) {
        mbar_init(bars.a_full(), 1);
        mbar_init(bars.a_empty(), 1);
        for (int s = 0; s < kS; ++s) {
            mbar_init(bars.w_full(s), 1);
            mbar_init(bars.w_empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bars.acc1_full(b), 1);
            mbar_init(bars.h_full(b), 256);
        }
        mbar_init(bars.acc2_full(), 1);
        mbar_init(bars.acc2_empty(), 256);
        for (int i = 0; i < 8; ++i) mbar_init(bars.stats(i >> 2, i & 3), 64);
        mbar_init(bars.drain(), 1);
        for (int w = 0; w < 8; ++w) mbar_init(bars.resid_full(w), 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_map(&tmap_a);
        tma_prefetch_map(&tmap_w1);
        tma_prefetch_map(&tmap_w2);
        if (p.resid_mode != kResidNone) tma_prefetch_map(&tmap_r);
        if (p.x_out != nullptr) tma_prefetch_map(&tmap_x);
        tma_prefetch_map(&tmap_n);
    }
    pdl_wait();
    pdl_launch_dependents();
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ TMA --
        int stage = 0;
        uint32_t phase = 0;
        int issued[kS];
        for (int s = 0; s < kS; ++s) issued[s] = -1;
        int a_issued = -1;
        uint32_t it = 0;
        for (int t = blockIdx.x; t < p.num_m_tiles; t += gridDim.x, ++it) {
            // a: the previous block's last G1 has completed
            if (!mbar_wait(bars.a_empty(), (it & 1u) ^ 1u, abort_flag)) break;
            mbar_arrive_expect_tx(bars.a_full(), L::kKb * kFfnTileBytes);
            for (int kb = 0; kb < L::kKb; ++kb)
                tma_load_2d(sbase + L::kOffA + kb * kFfnTileBytes, &tmap_a, bars.a_full(), kb * kGemmBK,
                            t * kGemmBM);
            a_issued = static_cast<int>(it & 1u);
            auto put = [&](const CUtensorMap* map, int c0, int c1) -> bool {
                if (!mbar_wait(bars.w_empty(stage), phase ^ 1u, abort_flag)) return false;
                mbar_arrive_expect_tx(bars.w_full(stage), kFfnTileBytes);
                tma_load_2d(sbase + L::kOffW + stage * kFfnTileBytes, map, bars.w_full(stage), c0, c1);
                issued[stage] = static_cast<int>(phase);
                if (++stage == kS) {
                    stage = 0;
                    phase ^= 1u;
                }
                return true;
            };
            const bool ok = ffn_walk<D>(
                n_chunks,
                [&](int j) {   // W1 rows [128 j, 128 j + 128), k-block kb
                    for (int kb = 0; kb < L::kKb; ++kb)
                        if (!put(&tmap_w1, kb * kGemmBK, j * kFfnChunk)) return false;
                    return true;
                },
                [&](int j) {   // W2 columns [128 j + 64 h, +64), rows [128 r, +128)
                    for (int h = 0; h < 2; ++h)
                        for (int r = 0; r < kRh; ++r)
                            if (!put(&tmap_w2, j * kFfnChunk + h * kGemmBK, r * 128)) return false;
                    return true;
                });
            if (!ok) break;
        }
        if (*abort_flag) {
            for (int s = 0; s < kS; ++s)
                if (issued[s] >= 0) mbar_wait_drain(bars.w_full(s), static_cast<uint32_t>(issued[s]));
            if (a_issued >= 0) mbar_wait_drain(bars.a_full(), static_cast<uint32_t>(a_issued));
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------ MMA --
        constexpr uint32_t idesc = idesc_f16_f32(kGemmBM, 128, false, false);
        constexpr uint32_t idesc_n256 = idesc_f16_f32(kGemmBM, 256, false, false);
        static_assert(kRh != 2 || (kS % 2 == 0 && L::kKb % 2 == 0), "W2 half pairs must not wrap the ring");
        int stage = 0;
        uint32_t phase = 0;
        uint32_t c1 = 0, c2 = 0, it = 0;
        for (int t = blockIdx.x; t < p.num_m_tiles; t += gridDim.x, ++it) {
            if (!mbar_wait(bars.a_full(), it & 1u, abort_flag)) break;
            tc_fence_after();
            auto take = [&]() -> bool {
                if (!mbar_wait(bars.w_full(stage), phase, abort_flag)) return false;
                tc_fence_after();
                return true;
            };
            auto give = [&]() {
                tc_commit(bars.w_empty(stage));
                if (++stage == kS) {
                    stage = 0;
                    phase ^= 1u;
                }
            };
            const bool ok = ffn_walk<D>(
                n_chunks,
                [&](int j) {
                    const int b = static_cast<int>(c1 & 1u);
                    // acc1[b] last held H of chunk j-2, which its G2 reads from
                    // TMEM. That G2 was issued before this G1 from this thread,
                    // and tcgen05 MMAs run in issue order, so no wait: the
                    // tensor pipe stays fed while G2(j-2) executes.
                    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * kFfnChunk);
                    for (int kb = 0; kb < L::kKb; ++kb) {
                        if (!take()) return false;
                        const uint32_t a_addr = sbase + L::kOffA + kb * kFfnTileBytes;
                        const uint32_t w_addr = sbase + L::kOffW + stage * kFfnTileBytes;
#pragma unroll
                        for (int kk = 0; kk < kGemmBK / 16; ++kk)
                            mma_f16_ss(d_tmem, smem_desc(a_addr + kk * 32, 16, 1024, kSwizzle128),
                                       smem_desc(w_addr + kk * 32, 16, 1024, kSwizzle128), idesc,
                                       (kb != 0 || kk != 0) ? 1u : 0u);
                        give();
                    }
                    tc_commit(bars.acc1_full(b));
                    ++c1;
                    if (j == n_chunks - 1) tc_commit(bars.a_empty());   // a is free once this G1 completes
                    return true;
                },
                [&](int j) {
                    const int b = static_cast<int>(c2 & 1u);
                    if (!mbar_wait(bars.h_full(b), (c2 >> 1) & 1u, abort_flag)) return false;
                    if (j == 0 && !mbar_wait(bars.acc2_empty(), (it & 1u) ^ 1u, abort_flag)) return false;
                    tc_fence_after();
                    for (int h = 0; h < 2; ++h) {
                        // hidden columns [64 h, 64 h + 64) of the chunk: packed fp16
                        // pairs in TMEM columns [b 128 + 64 h, + 32), 8 per K=16 step
                        const uint32_t h_tmem = tmem_base + static_cast<uint32_t>(b * kFfnChunk + h * 64);
                        if constexpr (kRh == 2) {
                            // The two 128-row halves of this W2 k-block sit in
                            // consecutive ring stages (every block of the walk takes
                            // an even number of stages, and the ring's count is even,
                            // so a pair never wraps): one N=256 MMA per K step reads
                            // both, half the MMA instructions of two N=128 ones.
                            const int s0 = stage;
                            if (!take()) return false;
                            if (!mbar_wait(bars.w_full(s0 + 1), phase, abort_flag)) return false;
                            tc_fence_after();
                            const uint32_t w_addr = sbase + L::kOffW + s0 * kFfnTileBytes;
                            const uint32_t d_tmem = tmem_base + L::kColAcc2;
#pragma unroll
                            for (int kk = 0; kk < kGemmBK / 16; ++kk)
                                mma_f16_ts(d_tmem, h_tmem + kk * 8, smem_desc(w_addr + kk * 32, 16, 1024, kSwizzle128),
                                           idesc_n256, (j != 0 || h != 0 || kk != 0) ? 1u : 0u);
                            give();
                            give();
                        } else {
                            for (int r = 0; r < kRh; ++r) {
                                if (!take()) return false;
                                const uint32_t w_addr = sbase + L::kOffW + stage * kFfnTileBytes;
                                const uint32_t d_tmem = tmem_base + L::kColAcc2 + static_cast<uint32_t>(r * 128);
#pragma unroll
                                for (int kk = 0; kk < kGemmBK / 16; ++kk)
                                    mma_f16_ts(d_tmem, h_tmem + kk * 8,
                                               smem_desc(w_addr + kk * 32, 16, 1024, kSwizzle128), idesc,
                                               (j != 0 || h != 0 || kk != 0) ? 1u : 0u);
                                give();
                            }
                        }
                    }
                    ++c2;
                    if (j == n_chunks - 1) tc_commit(bars.acc2_full());
                    return true;
                });
            if (!ok) break;
        }
        tc_commit(bars.drain());
        mbar_wait_drain(bars.drain(), 0);
    } else if (warp >= 2) {
        // ------------------------------------------------------- epilogue --
        // Thread = one row of the block (its warp's TMEM lane quarter); the two
        // warps of a quarter split the columns in halves.
        constexpr int kCW = 32;
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row_in_tile = quarter * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        const bool has_resid = p.resid_mode != kResidNone;
        float2* stats = reinterpret_cast<float2*>(smem + L::kOffStats);
        const uint32_t st32 = sbase + L::kOffStage + static_cast<uint32_t>(warp - 2) * L::kStageWarpBytes;
        const uint32_t st16 = st32 + 4096;
        uint8_t* s32 = smem + L::kOffStage + (warp - 2) * L::kStageWarpBytes;
        uint8_t* s16 = s32 + 4096;
        const uint32_t rbar = bars.resid_full(warp - 2);
        uint32_t ce = 0, it = 0, rcount = 0, rissued = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < p.num_m_tiles && ok; t += gridDim.x, ++it) {
            const int row = t * kGemmBM + row_in_tile;
            const bool row_ok = row < p.M;
            // ---- hidden chunks: acc1 -> GELU -> H
            for (int j = 0; j < n_chunks; ++j, ++ce) {
                const int b = static_cast<int>(ce & 1u);
                const float4* b1v = reinterpret_cast<const float4*>(p.b1 + j * kFfnChunk + half * 64);
                ok = mbar_wait(bars.acc1_full(b), (ce >> 1) & 1u, abort_flag);
                if (!__all_sync(0xffffffffu, ok)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t t_acc = tmem_base + lane_off + static_cast<uint32_t>(b * kFfnChunk + half * 64);
                uint32_t r2[2][32];
                tmem_ld_32x32b_x32(t_acc, r2[0]);
                tmem_ld_32x32b_x32(t_acc + kCW, r2[1]);
                tmem_ld_wait(r2[0]);
                tmem_ld_wait(r2[1]);
                uint32_t pk[32];
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    float v[kCW];
                    // the same 32 biases for every lane: uniform 16-byte loads (L1 broadcast)
#pragma unroll
                    for (int i = 0; i < kCW / 4; ++i) {
                        const float4 bb = __ldg(b1v + q * (kCW / 4) + i);
                        v[4 * i] = __uint_as_float(r2[q][4 * i]) + bb.x;
                        v[4 * i + 1] = __uint_as_float(r2[q][4 * i + 1]) + bb.y;
                        v[4 * i + 2] = __uint_as_float(r2[q][4 * i + 2]) + bb.z;
                        v[4 * i + 3] = __uint_as_float(r2[q][4 * i + 3]) + bb.w;
                    }
#pragma unroll
                    for (int i = 0; i < kCW; i += 2) {
                        gelu_fast_pair(v[i], v[i + 1]);
                        pk[q * 16 + i / 2] = pack_half2(v[i], v[i + 1]);
                    }
                }
                // hidden k = 64 half + 2c, +1 into column c of the span just read
                tmem_st_32x32b_x32(t_acc, pk);
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(bars.h_full(b));
            }
            if (!ok) break;

            // ---- the block's output: acc2 -> x_new -> LayerNorm
            ok = mbar_wait(bars.acc2_full(), it & 1u, abort_flag);
            if (!__all_sync(0xffffffffu, ok)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const bool valid = (p.row_valid == nullptr) || !row_ok || (p.row_valid[row] != 0);
            const bool nvalid = (p.norm_row_valid == nullptr) || !row_ok || (p.norm_row_valid[row] != 0);
            const int c_lo = half * (D / 2);
            const int row0 = t * kGemmBM + quarter * 32;        // first row of this warp's blocks
            const uint32_t t_out = tmem_base + lane_off + L::kColAcc2;
            // the warp's 32 x 32 blocks move by TMA through its staging buffers:
            // lane l's row is 128 B (fp32, granule g at g ^ (l & 7)) or 64 B (fp16,
            // granule g at g ^ ((l >> 1) & 3)), so every smem access is conflict-free
            // and every global access is a full-line bulk copy
            auto stage_resid = [&](int c) {
                __syncwarp();
                if (lane == 0) {
                    bulk_wait_read<0>();                 // stores still reading s32
                    fence_proxy_async_smem();
                    mbar_arrive_expect_tx(rbar, 4096);
                    tma_load_2d(st32, &tmap_r, rbar, c, row0);
                }
                ++rissued;
            };
            float mean_t = 0.0f, m2_t = 0.0f;
            if (has_resid) stage_resid(c_lo);
#pragma unroll 1
            for (int k = 0; k < D / 2 / kCW; ++k) {
                const int c = c_lo + k * kCW;
                const float4* b2v = reinterpret_cast<const float4*>(p.b2 + c);
                uint32_t r[32];
                tmem_ld_32x32b_x32(t_out + c, r);
                tmem_ld_wait(r);
                float v[kCW];
#pragma unroll
                for (int i = 0; i < kCW / 4; ++i) {
                    const float4 bb = __ldg(b2v + i);
                    v[4 * i] = __uint_as_float(r[4 * i]) + bb.x;
                    v[4 * i + 1] = __uint_as_float(r[4 * i + 1]) + bb.y;
                    v[4 * i + 2] = __uint_as_float(r[4 * i + 2]) + bb.z;
                    v[4 * i + 3] = __uint_as_float(r[4 * i + 3]) + bb.w;
                }
                if (has_resid) {
                    ok = mbar_wait(rbar, rcount & 1u, abort_flag);
                    if (!__all_sync(0xffffffffu, ok)) {
                        ok = false;
                        break;
                    }
                    ++rcount;
                    const bool keep_sub = valid || p.resid_mode == kResidAdd;
                    const bool keep_all = valid || p.resid_mode != kResidAddMaskAll;
#pragma unroll
                    for (int g = 0; g < 8; ++g) {
                        const float4 rr = *reinterpret_cast<const float4*>(s32 + lane * 128 + ((g ^ (lane & 7)) << 4));
                        v[4 * g] = keep_all ? rr.x + (keep_sub ? v[4 * g] : 0.0f) : 0.0f;
                        v[4 * g + 1] = keep_all ? rr.y + (keep_sub ? v[4 * g + 1] : 0.0f) : 0.0f;
                        v[4 * g + 2] = keep_all ? rr.z + (keep_sub ? v[4 * g + 2] : 0.0f) : 0.0f;
                        v[4 * g + 3] = keep_all ? rr.w + (keep_sub ? v[4 * g + 3] : 0.0f) : 0.0f;
                    }
                }
                if (p.x_out != nullptr) {
                    if (!has_resid) {
                        if (lane == 0) bulk_wait_read<0>();
                        __syncwarp();
                    }
#pragma unroll
                    for (int g = 0; g < 8; ++g)
                        *reinterpret_cast<uint4*>(s32 + lane * 128 + ((g ^ (lane & 7)) << 4)) =
                            make_uint4(__float_as_uint(v[4 * g]), __float_as_uint(v[4 * g + 1]),
                                       __float_as_uint(v[4 * g + 2]), __float_as_uint(v[4 * g + 3]));
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmap_x, st32, c, row0);
                        bulk_commit();
                    }
                }
                if (has_resid && k + 1 < D / 2 / kCW) stage_resid(c + kCW);   // in flight meanwhile
#pragma unroll
                for (int i = 0; i < kCW; ++i) r[i] = __float_as_uint(v[i]);
                tmem_st_32x32b_x32(t_out + c, r);
                float sum = 0.0f;
#pragma unroll
                for (int i = 0; i < kCW; ++i) sum += v[i];
                const float mean_c = sum * (1.0f / kCW);
                float m2_c = 0.0f;
#pragma unroll
                for (int i = 0; i < kCW; ++i) {
                    const float d = v[i] - mean_c;
                    m2_c = fmaf(d, d, m2_c);
                }
                if (k == 0) {
                    mean_t = mean_c;
                    m2_t = m2_c;
                } else {
                    chan_merge(mean_t, m2_t, static_cast<float>(k * kCW), mean_c, m2_c, static_cast<float>(kCW));
                }
            }
            if (!ok) break;
            tmem_st_wait();
            // both warps of the quarter publish their half, then merge half 0 +
            // half 1 in that order (the same bits in both)
            const int par = static_cast<int>(it & 1u);
            stats[(par * 2 + half) * kGemmBM + row_in_tile] = make_float2(mean_t, m2_t);
            mbar_arrive(bars.stats(par, quarter));
            ok = mbar_wait(bars.stats(par, quarter), (it >> 1) & 1u, abort_flag);
            if (!__all_sync(0xffffffffu, ok)) {
                ok = false;
                break;
            }
            const float2 s0 = stats[(par * 2 + 0) * kGemmBM + row_in_tile];
            const float2 s1 = stats[(par * 2 + 1) * kGemmBM + row_in_tile];
            float mean = s0.x, m2 = s0.y;
            chan_merge(mean, m2, static_cast<float>(D / 2), s1.x, s1.y, static_cast<float>(D / 2));
            const float rstd = rsqrtf(m2 / static_cast<float>(D) + p.eps);
#pragma unroll 1
            for (int k = 0; k < D / 2 / kCW; ++k) {
                const int c = c_lo + k * kCW;
                const float4* gv = reinterpret_cast<const float4*>(p.ln_w + c);
                const float4* ev = reinterpret_cast<const float4*>(p.ln_b + c);
                uint32_t r[32];
                tmem_ld_32x32b_x32(t_out + c, r);
                tmem_ld_wait(r);
                float v[kCW];
#pragma unroll
                for (int i = 0; i < kCW / 4; ++i) {
                    const float4 g = __ldg(gv + i);
                    const float4 e = __ldg(ev + i);
                    v[4 * i] = nvalid ? fmaf((__uint_as_float(r[4 * i]) - mean) * rstd, g.x, e.x) : 0.0f;
                    v[4 * i + 1] = nvalid ? fmaf((__uint_as_float(r[4 * i + 1]) - mean) * rstd, g.y, e.y) : 0.0f;
                    v[4 * i + 2] = nvalid ? fmaf((__uint_as_float(r[4 * i + 2]) - mean) * rstd, g.z, e.z) : 0.0f;
                    v[4 * i + 3] = nvalid ? fmaf((__uint_as_float(r[4 * i + 3]) - mean) * rstd, g.w, e.w) : 0.0f;
                }
                if (lane == 0) bulk_wait_read<0>();
                __syncwarp();
                if constexpr (NORM_F16) {
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        uint4 w;
                        w.x = pack_half2(v[8 * g], v[8 * g + 1]);
                        w.y = pack_half2(v[8 * g + 2], v[8 * g + 3]);
                        w.z = pack_half2(v[8 * g + 4], v[8 * g + 5]);
                        w.w = pack_half2(v[8 * g + 6], v[8 * g + 7]);
                        *reinterpret_cast<uint4*>(s16 + lane * 64 + ((g ^ ((lane >> 1) & 3)) << 4)) = w;
                    }
                } else {
#pragma unroll
                    for (int g = 0; g < 8; ++g)
                        *reinterpret_cast<uint4*>(s32 + lane * 128 + ((g ^ (lane & 7)) << 4)) =
                            make_uint4(__float_as_uint(v[4 * g]), __float_as_uint(v[4 * g + 1]),
                                       __float_as_uint(v[4 * g + 2]), __float_as_uint(v[4 * g + 3]));
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tmap_n, NORM_F16 ? st16 : st32, c, row0);
                    bulk_commit();
                }
            }
            tc_fence_before();
            mbar_arrive(bars.acc2_empty());
        }
        // after an abort a residual block may still be landing in staging memory
        if (lane == 0 && rissued != rcount) mbar_wait_drain(rbar, rcount & 1u);
    }

    if (warp >= 2 && lane == 0) bulk_wait_all();   // staging reads done before the CTA exits

    // ------------------------------------------------------------ teardown --
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, L::kTmemCols);
    }
}

}  // namespace dotl
