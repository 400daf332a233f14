// Flash attention forward on the 5th-generation tensor cores.
//
// Replaces the reference's wmma flash-attention kernel
// (csrc/attention_wmma.cuh:874-1770) and its launcher
// (attention_dispatch.cuh:332-519). Same contract: softmax(q k^T * scale +
// masks) v per (batch, head), fp16 operands, fp32 softmax and accumulation in
// the exp2 domain, causal and key-padding masks combinable, fully masked rows
// written as 0, output in [B,H,S,hd] (layout 0) or [B,S,H*hd] (layout 1).
//
// Design (sm_100a), one CTA per SM, persistent over work items
// (head, 128-row query tile), largest causal tiles first:
//   warp 0      TMA producer: the Q tile once per item, then K and V tiles
//               (128 keys each) into a STAGES-deep ring, 128B/64B swizzled;
//   warp 1      MMA issuer: S(j) = Q K(j)^T into one of two TMEM S buffers
//               (M=128, N=128, K=hd), then PV(j) = P(j) V(j) into one of two
//               TMEM partial-O buffers (M=128, N=hd, K=128 keys);
//   warps 2-5   softmax: each thread owns one query row, reads its 128 scores
//               from TMEM, applies scale, causal / segment / key masks,
//               online max and sum in the exp2 domain, writes P(j) as fp16
//               into swizzled smem for the PV MMA, and folds PV(j-1) into its
//               register-resident O with the running correction factor.
// The score matrix never leaves TMEM/SMEM. Key tiles past the causal
// diagonal or past a query tile's segment are never loaded.
//
// "Packed" mode runs the query/key tiles over the flat token axis
// (b * S + s), so short sequences (S < 128) share one 128-row tile; a row's
// keys are confined to its own sequence by an interval test. It needs
// batch stride == S * sequence stride, which the fused QKV buffer has.

#pragma once

#include "dotl_common.cuh"

namespace dotl {

constexpr int kAttnThreads = 192;
constexpr int kAttnTile = 128;   // query rows per tile and keys per key tile

struct AttnParams {
    int B, H, S;
    int packed;          // tiles over the flat token axis
    int rows_total;      // packed: B*S; else S
    int num_q_tiles;     // per (head[, batch]) stream
    int num_streams;     // packed: H; else B*H
    int causal;
    float scale_log2;    // scale * log2(e)
    int mask_kind;       // 0 none, 1 per-key mask, 2 general [B,H,S,S] mask
    const uint8_t* mask;
    int64_t ms0, ms1, ms2, ms3;   // mask strides (elements) for b, h, query, key
    void* out;
    int out_layout;      // 0: [B,H,S,hd]; 1: [B,S,H*hd]
    int head_inner;      // bit t (q=0,k=1,v=2): tensor map dims are {hd, H, rows, B}
};

// Loads one 128-row box of `map` at (col, row, head, batch), in whichever
// dimension order the map was encoded with.
__device__ __forceinline__ void attn_tma(uint32_t dst, const CUtensorMap* map, uint32_t bar, int col, int row,
                                         int h, int b, bool head_inner) {
    if (head_inner)
        tma_load_4d(dst, map, bar, col, h, row, b);
    else
        tma_load_4d(dst, map, bar, col, row, h, b);
}

template <int HD, int STAGES>
struct AttnSmem {
    static constexpr int kBlkCols = HD < 64 ? HD : 64;          // fp16 columns per TMA box
    static constexpr int kRowBytes = kBlkCols * 2;              // 128 or 64
    static constexpr int kNumBlk = HD / kBlkCols;
    static constexpr uint32_t kBlkBytes = kAttnTile * kRowBytes;
    static constexpr uint32_t kTileBytes = kNumBlk * kBlkBytes; // one Q/K/V tile
    static constexpr uint32_t kSwz = kRowBytes == 128 ? kSwizzle128 : kSwizzle64;
    static constexpr uint32_t kPBytes = kAttnTile * kAttnTile * 2;
    static constexpr uint32_t kOffQ = 0;
    static constexpr uint32_t kOffK = kOffQ + kTileBytes;
    static constexpr uint32_t kOffV = kOffK + STAGES * kTileBytes;
    static constexpr uint32_t kOffP = kOffV + STAGES * kTileBytes;
    static constexpr uint32_t kOffBar = kOffP + 2 * kPBytes;
    // q_full, q_empty, k_full[ST], v_full[ST], kv_empty[ST], s_full[2],
    // s_empty[2], p_full[2], o_full[2], o_empty[2], drain
    static constexpr uint32_t kNumBars = 2 + 3 * STAGES + 10 + 1;
    static constexpr uint32_t kOffSlot = kOffBar + kNumBars * 8;
    static constexpr uint32_t kOffAbort = kOffSlot + 4;
    static constexpr uint32_t kBytes = kOffAbort + 4;
    static constexpr uint32_t kAlloc = kBytes + 1024;
    static constexpr uint32_t kTmemCols = 512;    // S[2] at 0/128, O[2] at 256/256+HD
};

// Item -> (stream, query tile) with the query-tile index descending in the
// slowest position: under causal masking the longest tiles go first.
__device__ __forceinline__ void attn_item(const AttnParams& p, int item, int& stream, int& qt) {
    const int tile_rank = item / p.num_streams;
    stream = item - tile_rank * p.num_streams;
    qt = p.num_q_tiles - 1 - tile_rank;
}

// Key range [k_lo, k_hi) in map coordinates that query tile qt can see.
__device__ __forceinline__ void attn_key_range(const AttnParams& p, int qt, int& k_lo, int& k_hi) {
    const int r0 = qt * kAttnTile;
    const int r1 = min(r0 + kAttnTile, p.rows_total) - 1;
    if (p.packed) {
        k_lo = (r0 / p.S) * p.S;
        k_hi = p.causal ? r1 + 1 : (r1 / p.S + 1) * p.S;
    } else {
        k_lo = 0;
        k_hi = p.causal ? r1 + 1 : p.S;
    }
}

template <int HD, int STAGES>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                   const __grid_constant__ CUtensorMap tmap_v, const AttnParams p) {
    using L = AttnSmem<HD, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + L::kOffBar;
    const uint32_t q_full = bar0, q_empty = bar0 + 8;
    auto k_full = [&](int s) { return bar0 + 8u * (2 + s); };
    auto v_full = [&](int s) { return bar0 + 8u * (2 + STAGES + s); };
    auto kv_empty = [&](int s) { return bar0 + 8u * (2 + 2 * STAGES + s); };
    auto s_full = [&](int b) { return bar0 + 8u * (2 + 3 * STAGES + b); };
    auto s_empty = [&](int b) { return bar0 + 8u * (4 + 3 * STAGES + b); };
    auto p_full = [&](int b) { return bar0 + 8u * (6 + 3 * STAGES + b); };
    auto o_full = [&](int b) { return bar0 + 8u * (8 + 3 * STAGES + b); };
    auto o_empty = [&](int b) { return bar0 + 8u * (10 + 3 * STAGES + b); };
    const uint32_t drain_bar = bar0 + 8u * (12 + 3 * STAGES);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffAbort);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffSlot);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(k_full(s), 1);
            mbar_init(v_full(s), 1);
            mbar_init(kv_empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(s_full(b), 1);
            mbar_init(s_empty(b), 128);
            mbar_init(p_full(b), 128);
            mbar_init(o_full(b), 1);
            mbar_init(o_empty(b), 128);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_map(&tmap_q);
        tma_prefetch_map(&tmap_k);
        tma_prefetch_map(&tmap_v);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int num_items = p.num_streams * p.num_q_tiles;

    if (warp == 0 && lane == 0) {
        // ---------------------------------------------------- TMA producer --
        uint32_t tcount = 0;     // key tiles issued, across items
        uint32_t icount = 0;     // items issued
        int k_issued_phase[STAGES];
        for (int s = 0; s < STAGES; ++s) k_issued_phase[s] = -1;
        int q_issued = -1;
        for (int item = blockIdx.x; item < num_items; item += gridDim.x, ++icount) {
            int stream, qt, k_lo, k_hi;
            attn_item(p, item, stream, qt);
            attn_key_range(p, qt, k_lo, k_hi);
            const int h = p.packed ? stream : stream % p.H;
            const int bq = p.packed ? 0 : stream / p.H;
            if (!mbar_wait(q_empty, (icount & 1u) ^ 1u, abort_flag)) goto producer_done;
            mbar_arrive_expect_tx(q_full, L::kTileBytes);
#pragma unroll
            for (int cb = 0; cb < L::kNumBlk; ++cb)
                attn_tma(sbase + L::kOffQ + cb * L::kBlkBytes, &tmap_q, q_full, cb * L::kBlkCols,
                         qt * kAttnTile, h, bq, p.head_inner & 1);
            q_issued = static_cast<int>(icount & 1u);
            const int n_kt = (k_hi - k_lo + kAttnTile - 1) / kAttnTile;
            for (int j = 0; j < n_kt; ++j, ++tcount) {
                const int st = static_cast<int>(tcount % STAGES);
                const uint32_t ph = (tcount / STAGES) & 1u;
                const int kc0 = k_lo + j * kAttnTile;
                if (!mbar_wait(kv_empty(st), ph ^ 1u, abort_flag)) goto producer_done;
                mbar_arrive_expect_tx(k_full(st), L::kTileBytes);
#pragma unroll
                for (int cb = 0; cb < L::kNumBlk; ++cb)
                    attn_tma(sbase + L::kOffK + st * L::kTileBytes + cb * L::kBlkBytes, &tmap_k,
                             k_full(st), cb * L::kBlkCols, kc0, h, bq, p.head_inner & 2);
                mbar_arrive_expect_tx(v_full(st), L::kTileBytes);
#pragma unroll
                for (int cb = 0; cb < L::kNumBlk; ++cb)
                    attn_tma(sbase + L::kOffV + st * L::kTileBytes + cb * L::kBlkBytes, &tmap_v,
                             v_full(st), cb * L::kBlkCols, kc0, h, bq, p.head_inner & 4);
                k_issued_phase[st] = static_cast<int>(ph);
            }
        }
    producer_done:
        if (*abort_flag) {
            if (q_issued >= 0) mbar_wait_drain(q_full, static_cast<uint32_t>(q_issued));
            for (int s = 0; s < STAGES; ++s) {
                if (k_issued_phase[s] >= 0) {
                    mbar_wait_drain(k_full(s), static_cast<uint32_t>(k_issued_phase[s]));
                    mbar_wait_drain(v_full(s), static_cast<uint32_t>(k_issued_phase[s]));
                }
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------ MMA issuer --
        constexpr uint32_t idesc_s = idesc_f16_f32(kAttnTile, kAttnTile, false, false);
        constexpr uint32_t idesc_o = idesc_f16_f32(kAttnTile, HD, false, true);
        constexpr int kStepsPerBlk = L::kBlkCols / 16;
        uint32_t tcount = 0;
        uint32_t icount = 0;
        for (int item = blockIdx.x; item < num_items; item += gridDim.x, ++icount) {
            int stream, qt, k_lo, k_hi;
            attn_item(p, item, stream, qt);
            attn_key_range(p, qt, k_lo, k_hi);
            const int n_kt = (k_hi - k_lo + kAttnTile - 1) / kAttnTile;
            if (!mbar_wait(q_full, icount & 1u, abort_flag)) goto mma_done;
            tc_fence_after();
            // S(j) = Q K(j)^T for global tile index t
            auto issue_s = [&](uint32_t t) -> bool {
                const int st = static_cast<int>(t % STAGES);
                const int sb = static_cast<int>(t & 1u);
                if (!mbar_wait(k_full(st), (t / STAGES) & 1u, abort_flag)) return false;
                if (!mbar_wait(s_empty(sb), ((t >> 1) & 1u) ^ 1u, abort_flag)) return false;
                tc_fence_after();
                const uint32_t d = tmem_base + static_cast<uint32_t>(sb * kAttnTile);
                const uint32_t qa = sbase + L::kOffQ;
                const uint32_t ka = sbase + L::kOffK + st * L::kTileBytes;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk) {
                    const uint32_t off = (kk / kStepsPerBlk) * L::kBlkBytes + (kk % kStepsPerBlk) * 32;
                    const uint64_t ad = smem_desc(qa + off, 16, 8 * L::kRowBytes, L::kSwz);
                    const uint64_t bd = smem_desc(ka + off, 16, 8 * L::kRowBytes, L::kSwz);
                    mma_f16_ss(d, ad, bd, idesc_s, kk != 0 ? 1u : 0u);
                }
                tc_commit(s_full(sb));
                return true;
            };
            if (!issue_s(tcount)) goto mma_done;
            if (n_kt == 1) tc_commit(q_empty);
            for (int j = 0; j < n_kt; ++j) {
                const uint32_t t = tcount + j;
                if (j + 1 < n_kt) {
                    if (!issue_s(t + 1)) goto mma_done;
                    if (j + 2 == n_kt) tc_commit(q_empty);   // Q is no longer read
                }
                const int st = static_cast<int>(t % STAGES);
                const int b = static_cast<int>(t & 1u);
                const uint32_t use = (t >> 1) & 1u;
                if (!mbar_wait(p_full(b), use, abort_flag)) goto mma_done;
                if (!mbar_wait(v_full(st), (t / STAGES) & 1u, abort_flag)) goto mma_done;
                if (!mbar_wait(o_empty(b), use ^ 1u, abort_flag)) goto mma_done;
                tc_fence_after();
                const uint32_t d = tmem_base + 2u * kAttnTile + static_cast<uint32_t>(b * HD);
                const uint32_t pa = sbase + L::kOffP + b * L::kPBytes;
                const uint32_t va = sbase + L::kOffV + st * L::kTileBytes;
#pragma unroll
                for (int kk = 0; kk < kAttnTile / 16; ++kk) {
                    const uint64_t ad = smem_desc(pa + (kk / 4) * (kAttnTile * 128) + (kk % 4) * 32, 16,
                                                  1024, kSwizzle128);
                    const uint64_t bd = smem_desc(va + kk * 16 * L::kRowBytes, L::kBlkBytes,
                                                  8 * L::kRowBytes, L::kSwz);
                    mma_f16_ss(d, ad, bd, idesc_o, kk != 0 ? 1u : 0u);
                }
                tc_commit(o_full(b));
                tc_commit(kv_empty(st));
            }
            tcount += n_kt;
        }
    mma_done:
        tc_commit(drain_bar);
        mbar_wait_drain(drain_bar, 0);
    } else if (warp >= 2) {
        // --------------------------------------------- softmax + epilogue --
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;           // query row within the tile
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        uint32_t tcount = 0;
        for (int item = blockIdx.x; item < num_items; item += gridDim.x) {
            int stream, qt, k_lo, k_hi;
            attn_item(p, item, stream, qt);
            attn_key_range(p, qt, k_lo, k_hi);
            const int n_kt = (k_hi - k_lo + kAttnTile - 1) / kAttnTile;
            const int h = p.packed ? stream : stream % p.H;
            const int rq = qt * kAttnTile + row;       // map row coordinate
            const bool q_ok = rq < p.rows_total;
            int b, s, klo_r, khi_r;
            if (p.packed) {
                b = rq / p.S;
                s = rq - b * p.S;
                klo_r = b * p.S;
                khi_r = p.causal ? rq : klo_r + p.S - 1;
            } else {
                b = stream / p.H;
                s = rq;
                klo_r = 0;
                khi_r = p.causal ? rq : p.S - 1;
            }
            if (!q_ok) {
                klo_r = 1;
                khi_r = 0;
            }
            const uint8_t* mrow = nullptr;
            if (p.mask_kind == 2 && q_ok)
                mrow = p.mask + b * p.ms0 + h * p.ms1 + static_cast<int64_t>(s) * p.ms2;

            float o[HD];
#pragma unroll
            for (int i = 0; i < HD; ++i) o[i] = 0.0f;
            float m_run = -INFINITY, l_run = 0.0f, alpha_prev = 1.0f;

            // Folds PV(t) into o with the correction factor of its step.
            auto accumulate = [&](uint32_t t, float alpha) -> bool {
                const int ob = static_cast<int>(t & 1u);
                bool ok = mbar_wait(o_full(ob), (t >> 1) & 1u, abort_flag);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) return false;
                tc_fence_after();
                const uint32_t ta = tmem_base + lane_off + 2u * kAttnTile + static_cast<uint32_t>(ob * HD);
#pragma unroll
                for (int c = 0; c < HD; c += 32) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(ta + c, r);
                    tmem_ld_wait(r);
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[c + i] = fmaf(o[c + i], alpha, __uint_as_float(r[i]));
                }
                tc_fence_before();
                mbar_arrive(o_empty(ob));
                return true;
            };

            bool alive = true;
            for (int j = 0; j < n_kt && alive; ++j) {
                const uint32_t t = tcount + j;
                const int sb = static_cast<int>(t & 1u);
                const int kc0 = k_lo + j * kAttnTile;
                // Per-key mask bits for this tile, identical for every row:
                // bits[q] bit i  <->  key kc0 + 4 i + q.
                uint32_t kbits[4] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu};
                if (p.mask_kind == 1) {
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const int kc = kc0 + 4 * lane + q4;
                        bool allowed = false;
                        if (kc < p.rows_total) {
                            int bk = b, sk = kc;
                            if (p.packed) {
                                bk = kc / p.S;
                                sk = kc - bk * p.S;
                            } else {
                                bk = stream / p.H;
                            }
                            allowed = p.mask[bk * p.ms0 + static_cast<int64_t>(sk) * p.ms3] != 0;
                        }
                        kbits[q4] = __ballot_sync(0xffffffffu, allowed);
                    }
                }
                const bool interior = p.mask_kind == 0 && kc0 >= klo_r && kc0 + kAttnTile - 1 <= khi_r;

                bool ok = mbar_wait(s_full(sb), (t >> 1) & 1u, abort_flag);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) { alive = false; break; }
                tc_fence_after();
                const uint32_t ts = tmem_base + lane_off + static_cast<uint32_t>(sb * kAttnTile);

                auto allowed_at = [&](int c) -> bool {
                    if (interior) return true;
                    const int kc = kc0 + c;
                    bool a = kc >= klo_r && kc <= khi_r;
                    if (p.mask_kind == 1) a = a && ((kbits[c & 3] >> (c >> 2)) & 1u);
                    if (p.mask_kind == 2) a = a && mrow[static_cast<int64_t>(kc - klo_r) * p.ms3] != 0;
                    return a;
                };

                // pass 1: row max of the allowed raw scores
                float mx = -INFINITY;
#pragma unroll
                for (int c0 = 0; c0 < kAttnTile; c0 += 32) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(ts + c0, r);
                    tmem_ld_wait(r);
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (allowed_at(c0 + i)) mx = fmaxf(mx, __uint_as_float(r[i]));
                }
                const float m_new = fmaxf(m_run, mx);
                const float m_scaled = (m_new == -INFINITY) ? 0.0f : m_new * p.scale_log2;
                const float alpha = (m_run == -INFINITY) ? 0.0f : fast_exp2(m_run * p.scale_log2 - m_scaled);

                // pass 2: p = exp2(s*c - m*c), row sum, P as fp16 into swizzled smem
                uint8_t* prow = smem + L::kOffP + sb * L::kPBytes + (row >> 3) * 1024 + (row & 7) * 128;
                float rsum = 0.0f;
#pragma unroll
                for (int c0 = 0; c0 < kAttnTile; c0 += 32) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(ts + c0, r);
                    tmem_ld_wait(r);
                    uint32_t packed[16];
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        const float p0 = allowed_at(c0 + i)
                                             ? fast_exp2(fmaf(__uint_as_float(r[i]), p.scale_log2, -m_scaled))
                                             : 0.0f;
                        const float p1 = allowed_at(c0 + i + 1)
                                             ? fast_exp2(fmaf(__uint_as_float(r[i + 1]), p.scale_log2, -m_scaled))
                                             : 0.0f;
                        rsum += p0 + p1;
                        packed[i / 2] = pack_half2(p0, p1);
                    }
                    // keys [c0, c0+32): block c0/64, 16-byte chunks (c0%64)/8 .. +3
                    uint8_t* blk = prow + (c0 / 64) * (kAttnTile * 128);
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const int chunk = ((c0 % 64) / 8 + q4) ^ (row & 7);
                        *reinterpret_cast<uint4*>(blk + chunk * 16) =
                            make_uint4(packed[4 * q4], packed[4 * q4 + 1], packed[4 * q4 + 2], packed[4 * q4 + 3]);
                    }
                }
                l_run = l_run * alpha + rsum;
                m_run = m_new;
                tc_fence_before();
                mbar_arrive(s_empty(sb));
                fence_proxy_async_smem();     // P stores -> visible to the tensor core
                mbar_arrive(p_full(sb));

                if (j > 0 && !accumulate(t - 1, alpha_prev)) { alive = false; break; }
                alpha_prev = alpha;
            }
            if (alive && !accumulate(tcount + n_kt - 1, alpha_prev)) alive = false;
            if (!alive) break;
            tcount += n_kt;

            if (q_ok) {
                const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
                int64_t off;
                if (p.out_layout == 1)
                    off = ((static_cast<int64_t>(b) * p.S + s) * p.H + h) * HD;
                else
                    off = ((static_cast<int64_t>(b) * p.H + h) * p.S + s) * HD;
                __half* op = reinterpret_cast<__half*>(p.out) + off;
#pragma unroll
                for (int i = 0; i < HD; i += 8) {
                    uint4 v;
                    v.x = pack_half2(o[i] * inv, o[i + 1] * inv);
                    v.y = pack_half2(o[i + 2] * inv, o[i + 3] * inv);
                    v.z = pack_half2(o[i + 4] * inv, o[i + 5] * inv);
                    v.w = pack_half2(o[i + 6] * inv, o[i + 7] * inv);
                    *reinterpret_cast<uint4*>(op + i) = v;
                }
            }
        }
    }

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
