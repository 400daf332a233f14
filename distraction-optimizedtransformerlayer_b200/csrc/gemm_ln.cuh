// GEMM with a residual + LayerNorm epilogue, the row statistics exchanged
// between the CTAs of a thread-block cluster.
//
// Replaces, in one kernel, the reference's linear_bias (linear_gelu.cuh:
// 598-756) followed by fused_add_layernorm / fused_layernorm (add_layernorm.cuh:
// 663-692), the out_proj -> norm2 and ffn_out -> next-norm pairs of the layer:
//
//   x_new  = resid-mode epilogue(A W^T + bias)          (as gemm_tc_kernel)
//   normed = (x_new - mean) * rstd * ln_w + ln_b         over the row's N columns
//   normed = 0 on rows with norm_row_valid == 0          (the final masked fill)
//
// A LayerNorm needs the whole row, but a CTA owns BN columns of it. A cluster
// of CS = N / BN CTAs (CS <= 8) shares every 128-row block: CTA r computes
// columns [r BN, (r+1) BN), so the cluster walks the M blocks together. The
// epilogue makes two passes over the accumulator:
//   pass 1: x_new per 32-column chunk (the residual block arriving by TMA in
//           one of two per-warp staging buffers while the previous chunk is
//           processed; x_new stored by TMA from that buffer when requested,
//           and written back into TMEM), with the chunk's exact two-pass mean and
//           M2; chunks, then the CTA's two column halves, merge by Chan et al.'s
//           pairwise update; each CTA then writes its (mean, M2) for every row
//           into every peer's shared memory and arrives on the peer's barrier;
//   pass 2: once all CS contributions are in, every CTA merges them in rank
//           order (so all CTAs derive bit-identical mean and rstd), reads x_new
//           back from TMEM and stores the normalised chunk.
// Stats buffers alternate between two parities (a CTA cannot be two tiles
// ahead of a peer: each tile's exchange needs everyone's arrival). Every wait
// is bounded; on teardown each CTA tells every peer it is done with their
// shared memory and waits (bounded) for the same before it exits.
//
// N must be CS * BN exactly (the layer's d_model); BN in {64, 128, 256}.

#pragma once

#include "gemm.cuh"

namespace dotl {

constexpr int kLnMaxCluster = 8;

struct GemmLnParams {
    int M, N, K;
    int num_m_tiles;
    int cs;                      // cluster size = N / BN
    const float* bias;           // [N]
    const float* resid;          // [M, ldr] fp32, or null
    int64_t ldr;
    const uint8_t* row_valid;    // residual-mode row mask, or null
    int resid_mode;              // GemmResidMode (kMaskRows / act are not used here)
    int store_x;                 // write x_new through tmap_x
    const float* ln_w;           // [N]
    const float* ln_b;           // [N]
    float eps;
    const uint8_t* norm_row_valid;   // rows with 0 get normed = 0, or null
    int x3_nkb;                  // three-product mode (X3Pass): k-blocks per pass, 0 = one pass
    int a_lo_row, w_lo_row;
    int norm_lo;                 // fp16 normed: also store its lo half through tmap_nl
};

template <int BN, int STAGES>
struct GemmLnSmem {
    using G = GemmSmem<BN, STAGES>;
    static constexpr uint32_t kOffStage = G::kOffStage;              // 8 x 4 KB staging
    static constexpr uint32_t kStageBufBytes = G::kStageBufBytes;
    static constexpr uint32_t kOffStage2 = kOffStage + 8 * kStageBufBytes;  // 8 x 4 KB, residual double buffer
    static constexpr uint32_t kOffStats = kOffStage2 + 8 * kStageBufBytes;  // [2][8][128] (mean, M2)
    static constexpr uint32_t kStatsParityBytes = kLnMaxCluster * kGemmBM * 8;
    static constexpr uint32_t kOffHalf = kOffStats + 2 * kStatsParityBytes;  // [128] (mean, M2) of half 1
    static constexpr uint32_t kOffBar = kOffHalf + kGemmBM * 8;
    // GemmBars, then stats_full[2], half_ready[4] (one per lane quarter), exit,
    // resid_full[8 warps][2 buffers]
    static constexpr int kBarStats = GemmBars<STAGES>::kCount;
    static constexpr int kBarHalf = kBarStats + 2;
    static constexpr int kBarExit = kBarHalf + 4;
    static constexpr int kBarResid = kBarExit + 1;
    static constexpr uint32_t kNumBars = kBarResid + 16;
    static constexpr uint32_t kOffSlot = kOffBar + kNumBars * 8;
    static constexpr uint32_t kOffAbort = kOffSlot + 4;
    static constexpr uint32_t kBytes = kOffAbort + 4;
    static constexpr uint32_t kAlloc = kBytes + 1024;
    static constexpr uint32_t kTmemCols = 2 * BN;
    static_assert(kAlloc <= 232448, "dynamic shared memory over the 227 KB an sm_100a CTA may use");
};

// (mean_a, m2_a) over n_a values merged with (mean_b, m2_b) over n_b.
__device__ __forceinline__ void chan_merge(float& mean_a, float& m2_a, float n_a, float mean_b, float m2_b,
                                           float n_b) {
    const float n = n_a + n_b;
    const float delta = mean_b - mean_a;
    const float fb = n_b / n;
    mean_a = fmaf(delta, fb, mean_a);
    m2_a = m2_a + m2_b + delta * delta * n_a * fb;
}

template <int BN, int STAGES, bool NORM_F16>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_ln_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_n,
                   const __grid_constant__ CUtensorMap tmap_r, const __grid_constant__ CUtensorMap tmap_nl,
                   const GemmLnParams p) {
    using L = GemmLnSmem<BN, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + L::kOffBar;
    const GemmBars<STAGES> bars{bar0};
    auto stats_full = [&](int par) { return bar0 + 8u * (L::kBarStats + par); };
    auto half_ready = [&](int q) { return bar0 + 8u * (L::kBarHalf + q); };
    const uint32_t exit_bar = bar0 + 8u * L::kBarExit;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffAbort);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffSlot);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int cs = p.cs;
    const uint32_t rank = cluster_ctarank();

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(bars.full(s), 1);
            mbar_init(bars.empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bars.accf(b), 1);
            mbar_init(bars.acce(b), 256);
            mbar_init(stats_full(b), 128 * cs);   // the half-0 lanes of every CTA
        }
        for (int q = 0; q < 4; ++q) mbar_init(half_ready(q), 32);
        for (int i = 0; i < 16; ++i) mbar_init(bar0 + 8u * (L::kBarResid + i), 1);
        mbar_init(bars.drain(), 1);
        mbar_init(exit_bar, cs);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_map(&tmap_a);
        tma_prefetch_map(&tmap_w);
        tma_prefetch_map(&tmap_x);
        tma_prefetch_map(&tmap_n);
        if (p.resid_mode != kResidNone) tma_prefetch_map(&tmap_r);
    }
    cluster_sync_after_init();
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

    const int num_kb = p.x3_nkb > 0 ? 3 * p.x3_nkb : (p.K + kGemmBK - 1) / kGemmBK;
    const X3Pass x3{p.x3_nkb, p.a_lo_row, p.w_lo_row};
    const int cluster_id = static_cast<int>(blockIdx.x) / cs;
    const int num_clusters = static_cast<int>(gridDim.x) / cs;
    const TileSched ts{cluster_id, num_clusters, p.num_m_tiles, 1, static_cast<int>(rank)};

    if (warp == 0 && lane == 0) {
        gemm_produce<BN, STAGES>(&tmap_a, &tmap_w, sbase, bars, abort_flag, ts, 0, num_kb, x3);
    } else if (warp == 1 && lane == 0) {
        gemm_mma<BN, STAGES>(sbase, tmem_base, bars, abort_flag, ts, 0, num_kb);
    } else if (warp >= 2) {
        // -------------------------------------------------------- epilogue --
        // Thread = one row of the tile (lane quarter of its warp) and the
        // 32-column chunks half, half + 2, ... of the CTA's BN columns.
        constexpr int kCW = 32;
        constexpr int kChunks = BN / (2 * kCW);           // per thread
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row_in_tile = quarter * 32 + lane;
        const uint32_t stage_addr = sbase + L::kOffStage + static_cast<uint32_t>(warp - 2) * L::kStageBufBytes;
        uint8_t* stage_ptr = smem + L::kOffStage + (warp - 2) * L::kStageBufBytes;
        float2* half_buf = reinterpret_cast<float2*>(smem + L::kOffHalf);
        const float2* stats = reinterpret_cast<const float2*>(smem + L::kOffStats);
        const bool has_resid = p.resid_mode != kResidNone && p.resid_mode != kMaskRows;
        const int n_cta0 = static_cast<int>(rank) * BN;   // first column of this CTA
        // Residual 32 x 32 blocks arrive by TMA, alternating between the warp's
        // two staging buffers (128B swizzle: lane l's row at l * 128, granule g
        // at g ^ (l & 7)); the next block is in flight while this one is used,
        // and x_new leaves from the buffer its residual arrived in.
        uint8_t* sbuf[2] = {stage_ptr, smem + L::kOffStage2 + (warp - 2) * L::kStageBufBytes};
        const uint32_t saddr[2] = {stage_addr, sbase + L::kOffStage2 + static_cast<uint32_t>(warp - 2) * L::kStageBufBytes};
        const uint32_t rbar[2] = {bar0 + 8u * (L::kBarResid + 2 * (warp - 2)),
                                  bar0 + 8u * (L::kBarResid + 2 * (warp - 2) + 1)};
        uint32_t ruse[2] = {0u, 0u};                      // completed waits per buffer
        uint32_t rissued[2] = {0u, 0u};
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t it = 0;                                  // tiles done by this CTA
        for (int t = ts.first; t < ts.count; t += ts.stride, ++it) {
            const uint32_t par = it & 1u;
            const int m_blk = t;
            const int row = m_blk * kGemmBM + row_in_tile;
            const bool row_ok = row < p.M;
            const bool valid = (p.row_valid == nullptr) || !row_ok || (p.row_valid[row] != 0);
            const bool nvalid = (p.norm_row_valid == nullptr) || !row_ok || (p.norm_row_valid[row] != 0);
            auto issue_resid = [&](int nc, int slot) {
                __syncwarp();
                if (lane == 0) {
                    bulk_wait_read<0>();                  // stores still reading the buffer
                    fence_proxy_async_smem();
                    mbar_arrive_expect_tx(rbar[slot], 4096);
                    tma_load_2d(saddr[slot], &tmap_r, rbar[slot], nc, m_blk * kGemmBM + quarter * 32);
                }
                ++rissued[slot];
            };
            float b_cur = __ldg(p.bias + n_cta0 + half * kCW + lane);
            if (has_resid) issue_resid(n_cta0 + half * kCW, 0);
            bool ok = mbar_wait(bars.accf(acc), acc_phase, abort_flag);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc_fence_after();
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                   static_cast<uint32_t>(acc * BN);

            // ---- pass 1: x_new, written back to TMEM; per-thread (mean, M2)
            float mean_t = 0.0f, m2_t = 0.0f;
#pragma unroll 1
            for (int k = 0; k < kChunks; ++k) {
                const int c = half * kCW + k * 2 * kCW;
                const int nc = n_cta0 + c;
                const int slot = k & 1;
                if (has_resid && k + 1 < kChunks) issue_resid(nc + 2 * kCW, slot ^ 1);
                const float b_next = k + 1 < kChunks ? __ldg(p.bias + nc + 2 * kCW + lane) : 0.0f;
                uint32_t r[32];
                tmem_ld_32x32b_x32(t_row + c, r);
                tmem_ld_wait(r);
                float v[kCW];
#pragma unroll
                for (int j = 0; j < kCW; ++j) v[j] = __uint_as_float(r[j]) + __shfl_sync(0xffffffffu, b_cur, j);
                if (has_resid) {
                    ok = mbar_wait(rbar[slot], ruse[slot] & 1u, abort_flag);
                    if (!__all_sync(0xffffffffu, ok)) {
                        ok = false;
                        break;
                    }
                    ++ruse[slot];
                    const bool keep_sub = valid || p.resid_mode == kResidAdd;
                    const bool keep_all = valid || p.resid_mode != kResidAddMaskAll;
                    const uint8_t* rrow = sbuf[slot] + lane * 128;
#pragma unroll
                    for (int j = 0; j < kCW; j += 4) {
                        const float4 rr = *reinterpret_cast<const float4*>(rrow + (((j >> 2) ^ (lane & 7)) << 4));
                        v[j] = keep_all ? rr.x + (keep_sub ? v[j] : 0.0f) : 0.0f;
                        v[j + 1] = keep_all ? rr.y + (keep_sub ? v[j + 1] : 0.0f) : 0.0f;
                        v[j + 2] = keep_all ? rr.z + (keep_sub ? v[j + 2] : 0.0f) : 0.0f;
                        v[j + 3] = keep_all ? rr.w + (keep_sub ? v[j + 3] : 0.0f) : 0.0f;
                    }
                }
                if (p.store_x) {
                    if (!has_resid) {
                        if (lane == 0) bulk_wait_read<0>();
                        __syncwarp();
                    }
                    uint8_t* srow = sbuf[slot] + lane * 128;
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        *reinterpret_cast<uint4*>(srow + ((q ^ (lane & 7)) << 4)) =
                            make_uint4(__float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]),
                                       __float_as_uint(v[4 * q + 2]), __float_as_uint(v[4 * q + 3]));
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmap_x, saddr[slot], nc, m_blk * kGemmBM + quarter * 32);
                        bulk_commit();
                    }
                }
#pragma unroll
                for (int j = 0; j < kCW; ++j) r[j] = __float_as_uint(v[j]);
                tmem_st_32x32b_x32(t_row + c, r);
                // the chunk's exact two-pass statistics, merged into the thread's
                float s = 0.0f;
#pragma unroll
                for (int j = 0; j < kCW; ++j) s += v[j];
                const float mean_c = s * (1.0f / kCW);
                float m2_c = 0.0f;
#pragma unroll
                for (int j = 0; j < kCW; ++j) {
                    const float d = v[j] - mean_c;
                    m2_c = fmaf(d, d, m2_c);
                }
                if (k == 0) {
                    mean_t = mean_c;
                    m2_t = m2_c;
                } else {
                    chan_merge(mean_t, m2_t, static_cast<float>(k * kCW), mean_c, m2_c, static_cast<float>(kCW));
                }
                b_cur = b_next;
            }
            if (!ok) break;
            tmem_st_wait();

            // ---- the CTA's two halves, then the cluster exchange
            // half 1 hands its rows' (mean, M2) to the half-0 warp of its
            // quarter, which merges and publishes the CTA's statistics
            if (half == 1) {
                half_buf[row_in_tile] = make_float2(mean_t, m2_t);
                mbar_arrive(half_ready(quarter));
            } else {
                ok = mbar_wait(half_ready(quarter), it & 1u, abort_flag);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                const float2 o = half_buf[row_in_tile];
                chan_merge(mean_t, m2_t, static_cast<float>(BN / 2), o.x, o.y, static_cast<float>(BN / 2));
                const uint32_t slot = sbase + L::kOffStats + par * L::kStatsParityBytes +
                                      (rank * kGemmBM + row_in_tile) * 8;
                for (int r = 0; r < cs; ++r) st_cluster_v2f32(mapa_shared(slot, r), mean_t, m2_t);
                for (int r = 0; r < cs; ++r) mbar_arrive_cluster(mapa_shared(stats_full(par), r));
            }
            ok = mbar_wait_cluster(stats_full(par), (it >> 1) & 1u, abort_flag);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            float mean = 0.0f, m2 = 0.0f;
            {
                const float2* st = stats + par * (kLnMaxCluster * kGemmBM);
                for (int r = 0; r < cs; ++r) {
                    const float2 e = st[r * kGemmBM + row_in_tile];
                    if (r == 0) {
                        mean = e.x;
                        m2 = e.y;
                    } else {
                        chan_merge(mean, m2, static_cast<float>(r * BN), e.x, e.y, static_cast<float>(BN));
                    }
                }
            }
            const float rstd = rsqrtf(m2 / static_cast<float>(p.N) + p.eps);

            // ---- pass 2: normalise from TMEM and store
            float g_cur = __ldg(p.ln_w + n_cta0 + half * kCW + lane);
            float e_cur = __ldg(p.ln_b + n_cta0 + half * kCW + lane);
#pragma unroll 1
            for (int k = 0; k < kChunks; ++k) {
                const int c = half * kCW + k * 2 * kCW;
                const int nc = n_cta0 + c;
                const float g_next = k + 1 < kChunks ? __ldg(p.ln_w + nc + 2 * kCW + lane) : 0.0f;
                const float e_next = k + 1 < kChunks ? __ldg(p.ln_b + nc + 2 * kCW + lane) : 0.0f;
                uint32_t r[32];
                tmem_ld_32x32b_x32(t_row + c, r);
                tmem_ld_wait(r);
                float v[kCW];
#pragma unroll
                for (int j = 0; j < kCW; ++j) {
                    // shuffles outside the row-mask select: every lane must take part
                    const float g = __shfl_sync(0xffffffffu, g_cur, j);
                    const float e = __shfl_sync(0xffffffffu, e_cur, j);
                    const float y = (__uint_as_float(r[j]) - mean) * rstd;
                    v[j] = nvalid ? fmaf(y, g, e) : 0.0f;
                }
                if (lane == 0) bulk_wait_read<0>();
                __syncwarp();
                uint8_t* srow = stage_ptr + lane * (NORM_F16 ? 64 : 128);
                if constexpr (NORM_F16) {
                    // the lo half of the fp16 pair (three-product mode) goes
                    // to the second half of the 4 KB buffer
                    if (p.norm_lo) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            uint4 w, l;
                            split_half2(v[8 * q], v[8 * q + 1], w.x, l.x);
                            split_half2(v[8 * q + 2], v[8 * q + 3], w.y, l.y);
                            split_half2(v[8 * q + 4], v[8 * q + 5], w.z, l.z);
                            split_half2(v[8 * q + 6], v[8 * q + 7], w.w, l.w);
                            *reinterpret_cast<uint4*>(srow + ((q ^ ((lane >> 1) & 3)) << 4)) = w;
                            *reinterpret_cast<uint4*>(srow + 2048 + ((q ^ ((lane >> 1) & 3)) << 4)) = l;
                        }
                    } else {
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            *reinterpret_cast<uint4*>(srow + ((q ^ ((lane >> 1) & 3)) << 4)) =
                                make_uint4(pack_half2(v[8 * q], v[8 * q + 1]), pack_half2(v[8 * q + 2], v[8 * q + 3]),
                                           pack_half2(v[8 * q + 4], v[8 * q + 5]), pack_half2(v[8 * q + 6], v[8 * q + 7]));
                    }
                } else {
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        *reinterpret_cast<uint4*>(srow + ((q ^ (lane & 7)) << 4)) =
                            make_uint4(__float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]),
                                       __float_as_uint(v[4 * q + 2]), __float_as_uint(v[4 * q + 3]));
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tmap_n, stage_addr, nc, m_blk * kGemmBM + quarter * 32);
                    if (NORM_F16 && p.norm_lo) tma_store_2d(&tmap_nl, stage_addr + 2048, nc, m_blk * kGemmBM + quarter * 32);
                    bulk_commit();
                }
                g_cur = g_next;
                e_cur = e_next;
            }
            tc_fence_before();
            mbar_arrive(bars.acce(acc));
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (lane == 0) {
            bulk_wait_all();
            // after an abort a residual block may still be landing in staging memory
            for (int sl = 0; sl < 2; ++sl)
                if (rissued[sl] != ruse[sl]) mbar_wait_drain(rbar[sl], ruse[sl] & 1u);
        }
    }

    // ------------------------------------------------------------ teardown --
    // No peer may still be writing into this CTA's shared memory (or arriving
    // on its barriers) when it exits: every CTA tells every peer it is done,
    // then waits (bounded) for all of them.
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int r = 0; r < cs; ++r) mbar_arrive_cluster(mapa_shared(exit_bar, r));
        mbar_wait_cluster(exit_bar, 0, nullptr, 4 * kWaitLimitNs);
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, L::kTmemCols);
    }
}

}  // namespace dotl
