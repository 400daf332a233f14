// Flash attention forward on the 5th-generation tensor cores.
//
// Replaces the reference's wmma flash-attention kernel
// (csrc/attention_wmma.cuh:874-1770), its split-KV combine (:1783-1826) and its
// launcher (attention_dispatch.cuh:332-519). Same contract: softmax(q k^T *
// scale + masks) v per (batch, head), fp16 operands, fp32 softmax and
// accumulation in the exp2 domain, causal and key masks combinable, fully
// masked rows written as 0, output [B,H,S,hd] (layout 0) or [B,S,H*hd]
// (layout 1).
//
// Design (sm_100a): one CTA per SM, persistent over work items (stream, 128-row
// query tile), largest causal tiles first. Twelve warps:
//   warps 0-3   softmax group 0, warps 4-7 softmax group 1: each thread owns
//               one query row of the tile, reads its 128 scores of a key tile
//               from TMEM, masks (only on boundary tiles), takes the row max,
//               rescales its O row in TMEM only when the max grew by more than
//               2^8 (the stale max is exact: numerator and denominator share
//               it), writes P = exp2(s*c - m*c) as fp16 over the S columns it
//               has read, and keeps the row sum. The groups take alternate key
//               tiles of an item; group 1 hands (max, sum) to the group that
//               merges the two partial outputs and stores the row;
//   warp 8      producer: publishes each item's key-tile count (after scanning
//               a per-key mask for its last valid key) and loads by TMA the Q
//               tile (two slots, so the next item's Q lands during this one)
//               and the K and V tiles (128 keys each) into two rings;
//   warp 9      MMA issuer: S(t) = Q K(t)^T into S/P buffer t mod NS, then
//               O_g += P(t) V(t) with P read from TMEM (the tcgen05 "TS" form).
// With NS = 3 S/P buffers (head_dim <= 64: 3 x 128 S columns plus two O
// accumulators fit TMEM's 512 columns), S(t+3) is issued right after PV(t),
// so a group's next scores are ready while it finishes the current tile;
// head_dim 128 has room for two buffers. Splitting one query tile's keys
// between two groups interleaves their softmax phases on each SM
// sub-partition while the tensor core runs the other group's MMAs. The score
// matrix never leaves TMEM.
//
// "Packed" mode runs the tiles over the flat token axis (b * S + s), so short
// sequences share one 128-row tile; a row's keys are confined to its own
// sequence by an interval test. It needs batch stride == S * sequence stride,
// which the fused QKV buffer has.
//
// Split-KV (splits > 1; the reference's split-KV path, attention_wmma.cuh:
// 662-759, with its combine :1783-1826): when there are too few (stream, query
// tile) items to fill the SMs and the sequences are long, each item's key
// range is cut into `splits` runs of kt_per_split key tiles, each run its own
// work item. A run writes its unnormalised fp32 O rows and their (max, sum)
// into a workspace slot instead of the output, and attn_combine_kernel folds a
// query tile's runs: O = sum_s 2^(c (m_s - M)) O_s / sum_s 2^(c (m_s - M)) l_s,
// in run order (the same bits on every call).

#pragma once

#include "dotl_common.cuh"

namespace dotl {

constexpr int kAttnThreads = 384;        // softmax warpgroups 0-1, producer/MMA warpgroup 2
constexpr int kAttnRegsSoftmax = 192;    // setmaxnreg of the two softmax warpgroups
constexpr int kAttnRegsOther = 104;      // and of the producer/MMA warpgroup
constexpr int kAttnRegSplit = 256 * kAttnRegsSoftmax + 128 * kAttnRegsOther;
constexpr int kAttnTile = 128;          // query rows per tile and keys per key tile
constexpr float kRescaleLog2 = 8.0f;    // lazy-rescale threshold, in log2 units

struct AttnParams {
    int B, H, S;
    int packed;          // tiles over the flat token axis
    int rows_total;      // packed: B*S; else S
    int num_q_tiles;     // per stream
    int num_streams;     // packed: H; else B*H
    int causal;
    float scale_log2;    // scale * log2(e)
    int mask_kind;       // 0 none, 1 per-key mask, 2 general [B,H,S,S] mask
    const uint8_t* mask;
    int64_t ms0, ms1, ms2, ms3;   // mask strides (elements) for b, h, query, key
    void* out;
    int out_layout;      // 0: [B,H,S,hd]; 1: [B,S,H*hd]
    int head_inner;      // bit t (q=0,k=1,v=2): tensor map dims are {hd, H, rows, B}
    int64_t out_lo;      // 0, or the element offset from `out` of a plane receiving
                         // fp16(o - fp16(o)) (the fp16 pair of the three-product GEMM mode)
    int splits;          // key runs per query tile (1: no split-KV)
    int kt_per_split;    // key tiles per run
    float* ws_o;         // split-KV: [slot][128][HD] unnormalised fp32 O
    float2* ws_ml;       // split-KV: [slot][128] (row max in score units, row sum)
};

// Workspace slot of (stream, query tile, run).
__device__ __forceinline__ int64_t attn_slot(const AttnParams& p, int stream, int qt, int split) {
    return (static_cast<int64_t>(stream) * p.num_q_tiles + qt) * p.splits + split;
}

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
    static constexpr int kNS = 3 * kAttnTile + 2 * HD <= 512 ? 3 : 2;   // S/P buffers in TMEM
    static constexpr int kBlkCols = HD < 64 ? HD : 64;          // fp16 columns per TMA box
    static constexpr int kRowBytes = kBlkCols * 2;              // 128 or 64
    static constexpr int kNumBlk = HD / kBlkCols;
    static constexpr uint32_t kBlkBytes = kAttnTile * kRowBytes;
    static constexpr uint32_t kTileBytes = kNumBlk * kBlkBytes; // one Q/K/V tile
    static constexpr uint32_t kSwz = kRowBytes == 128 ? kSwizzle128 : kSwizzle64;
    static constexpr uint32_t kOffQ = 0;                                  // 2 slots
    static constexpr uint32_t kOffK = kOffQ + 2 * kTileBytes;
    static constexpr uint32_t kOffV = kOffK + STAGES * kTileBytes;
    static constexpr uint32_t kOffComb = kOffV + STAGES * kTileBytes;   // 128 x (max, sum) of group 1
    static constexpr uint32_t kOffInfo = kOffComb + kAttnTile * 8;      // 2 item slots
    static constexpr uint32_t kOffBar = kOffInfo + 16;   // 2 slots x {n_kt, hole}
    // mbarrier indices
    static constexpr int kBarQFull = 0, kBarQEmpty = 2;                  // [2] each
    static constexpr int kBarKFull = 4, kBarKEmpty = kBarKFull + STAGES; // [STAGES] each
    static constexpr int kBarVFull = kBarKEmpty + STAGES, kBarVEmpty = kBarVFull + STAGES;
    // S ready per (softmax group, buffer): a buffer's uses alternate between
    // the groups, and each group must wait on its own uses' phases in order
    static constexpr int kBarSFull = kBarVEmpty + STAGES, kBarPFull = kBarSFull + 2 * kNS;   // [2][NS], [NS]
    static constexpr int kBarODone = kBarPFull + kNS, kBarOFree = kBarODone + 2;             // [2] each
    static constexpr int kBarCombFull = kBarOFree + 2, kBarCombEmpty = kBarCombFull + 1;
    static constexpr int kBarInfoFull = kBarCombEmpty + 1, kBarInfoEmpty = kBarInfoFull + 2;
    // O final per group: committed after the group's last PV of an item, so
    // it completes only when every PV of the group in that item has
    static constexpr int kBarOFinal = kBarInfoEmpty + 2;                                     // [2]
    static constexpr int kBarDrain = kBarOFinal + 2;
    static constexpr uint32_t kNumBars = kBarDrain + 1;
    static constexpr uint32_t kOffSlot = kOffBar + kNumBars * 8;
    static constexpr uint32_t kOffAbort = kOffSlot + 4;
    static constexpr uint32_t kBytes = kOffAbort + 4;
    static constexpr uint32_t kAlloc = kBytes + 1024;
    static constexpr uint32_t kTmemCols = 512;
    // TMEM columns: S/P buffer i at 128 i, O of group g at 128 NS + HD g.
    static constexpr uint32_t kColS = 0;
    static constexpr uint32_t kColO = kNS * kAttnTile;
};

// Item -> (stream, query tile, key run), query-tile index descending in the
// slowest position: under causal masking the longest tiles go first.
__device__ __forceinline__ void attn_item(const AttnParams& p, int item, int& stream, int& qt, int& split) {
    const int per_rank = p.num_streams * p.splits;
    const int tile_rank = item / per_rank;
    const int rem = item - tile_rank * per_rank;
    split = rem / p.num_streams;
    stream = rem - split * p.num_streams;
    qt = p.num_q_tiles - 1 - tile_rank;
}

// Key range [k_lo, k_hi) in map coordinates that query tile qt can see, cut
// to key run `split` (k_lo >= k_hi: nothing to do).
__device__ __forceinline__ void attn_key_range(const AttnParams& p, int qt, int split, int& k_lo, int& k_hi) {
    const int r0 = qt * kAttnTile;
    const int r1 = min(r0 + kAttnTile, p.rows_total) - 1;
    if (p.packed) {
        k_lo = (r0 / p.S) * p.S;
        k_hi = p.causal ? r1 + 1 : (r1 / p.S + 1) * p.S;
    } else {
        k_lo = 0;
        k_hi = p.causal ? r1 + 1 : p.S;
    }
    if (p.splits > 1) {
        const int run_lo = k_lo + split * p.kt_per_split * kAttnTile;
        k_hi = min(k_hi, run_lo + p.kt_per_split * kAttnTile);
        k_lo = run_lo;
    }
}

// Scans sequence b's per-key mask once: `end` = one past its last allowed key
// (0 if none), `hole` = its first masked key (S if none). Keys below `hole`
// are all allowed, so tiles there need no per-key mask reads. Warp-collective.
__device__ __forceinline__ void attn_scan_keys(const AttnParams& p, int b, int lane, int& end, int& hole) {
    const uint8_t* base = p.mask + static_cast<int64_t>(b) * p.ms0;
    int first_zero = p.S, last_one = -1;
    const bool vec = p.ms3 == 1 && (reinterpret_cast<uintptr_t>(base) & 15u) == 0 && (p.S & 15) == 0;
    if (vec) {
        for (int k0 = 16 * lane; k0 < p.S; k0 += 512) {
            const uint4 v = *reinterpret_cast<const uint4*>(base + k0);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
#pragma unroll
                for (int byte = 0; byte < 4; ++byte) {
                    const int k = k0 + 4 * q + byte;
                    if ((w[q] >> (8 * byte)) & 0xffu) last_one = max(last_one, k);
                    else first_zero = min(first_zero, k);
                }
            }
        }
    } else {
        for (int k = lane; k < p.S; k += 32) {
            if (base[static_cast<int64_t>(k) * p.ms3]) last_one = max(last_one, k);
            else first_zero = min(first_zero, k);
        }
    }
    end = __reduce_max_sync(0xffffffffu, last_one) + 1;
    hole = __reduce_min_sync(0xffffffffu, first_zero);
}

// SINGLE: every item has one key tile and CTAs take several items (the host
// decides); the MMA thread then overlaps consecutive items (see below).
template <int HD, int STAGES, bool SINGLE>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                   const __grid_constant__ CUtensorMap tmap_v, const AttnParams p) {
    using L = AttnSmem<HD, STAGES>;
    // Every barrier has one consumer (a thread, or one softmax group) that
    // steps through its phases in order and never falls two behind: an
    // mbarrier parity wait cannot tell phase k from phase k + 2.
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + L::kOffBar;
    auto bar = [&](int i) { return bar0 + 8u * static_cast<uint32_t>(i); };
    auto q_full = [&](int i) { return bar(L::kBarQFull + i); };
    auto q_empty = [&](int i) { return bar(L::kBarQEmpty + i); };
    auto k_full = [&](int s) { return bar(L::kBarKFull + s); };
    auto k_empty = [&](int s) { return bar(L::kBarKEmpty + s); };
    auto v_full = [&](int s) { return bar(L::kBarVFull + s); };
    auto v_empty = [&](int s) { return bar(L::kBarVEmpty + s); };
    auto s_full = [&](int g, int i) { return bar(L::kBarSFull + g * L::kNS + i); };
    auto p_full = [&](int i) { return bar(L::kBarPFull + i); };
    auto o_done = [&](int g) { return bar(L::kBarODone + g); };
    auto o_final = [&](int g) { return bar(L::kBarOFinal + g); };
    auto o_free = [&](int g) { return bar(L::kBarOFree + g); };
    const uint32_t comb_full = bar(L::kBarCombFull);
    const uint32_t comb_empty = bar(L::kBarCombEmpty);
    auto info_full = [&](int s) { return bar(L::kBarInfoFull + s); };
    auto info_empty = [&](int s) { return bar(L::kBarInfoEmpty + s); };
    const uint32_t drain_bar = bar(L::kBarDrain);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffAbort);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffSlot);
    volatile int* info = reinterpret_cast<volatile int*>(smem + L::kOffInfo);   // {n_kt, hole} x 2
    float2* comb = reinterpret_cast<float2*>(smem + L::kOffComb);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(k_full(s), 1);
            mbar_init(k_empty(s), 1);
            mbar_init(v_full(s), 1);
            mbar_init(v_empty(s), 1);
        }
        for (int i = 0; i < L::kNS; ++i) {
            mbar_init(s_full(0, i), 1);
            mbar_init(s_full(1, i), 1);
            mbar_init(p_full(i), 128);
        }
        for (int g = 0; g < 2; ++g) {
            mbar_init(q_full(g), 1);
            mbar_init(q_empty(g), 1);
            mbar_init(o_done(g), 1);
            mbar_init(o_final(g), 1);
            mbar_init(o_free(g), 128);
            mbar_init(info_full(g), 1);
            mbar_init(info_empty(g), 1 + 8);
        }
        mbar_init(comb_full, 128);
        mbar_init(comb_empty, 128);
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_map(&tmap_q);
        tma_prefetch_map(&tmap_k);
        tma_prefetch_map(&tmap_v);
    }
    pdl_wait();
    pdl_launch_dependents();
    if (warp == 9) {
        tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int num_items = p.num_streams * p.num_q_tiles * p.splits;
    const bool scan_mask = p.mask_kind == 1 && !p.packed;

    // Which group takes an item's first key tile. Items with several tiles
    // alternate tiles between the groups (group 0 merges and writes); items
    // with a single tile alternate whole items between the groups.
    auto first_group = [](int n_kt, uint32_t& singles) -> int {
        if (n_kt != 1) return 0;
        return static_cast<int>(singles++ & 1u);
    };

    if (warp >= 8) {
        regs_dec<kAttnRegsOther>();
        if (warp == 8) {
            // --------------------------------------------------- producer --
            // Loads follow the MMA issuer's order: K(0..NS-1), then V(j) and
            // K(j+NS) for each j, so each ring runs independently.
            uint32_t kcount = 0, vcount = 0, qcount = 0, icount = 0;
            int k_issued_phase[STAGES], v_issued_phase[STAGES], q_issued_phase[2] = {-1, -1};
            for (int s = 0; s < STAGES; ++s) k_issued_phase[s] = v_issued_phase[s] = -1;
            for (int item = blockIdx.x; item < num_items; item += gridDim.x, ++icount) {
                int stream, qt, split, k_lo, k_hi;
                attn_item(p, item, stream, qt, split);
                attn_key_range(p, qt, split, k_lo, k_hi);
                const int h = p.packed ? stream : stream % p.H;
                const int bq = p.packed ? 0 : stream / p.H;
                int hole = 0;
                if (scan_mask) {
                    int end;
                    attn_scan_keys(p, bq, lane, end, hole);
                    k_hi = min(k_hi, end);
                }
                const int n_kt = k_hi > k_lo ? (k_hi - k_lo + kAttnTile - 1) / kAttnTile : 0;
                bool ok = true;
                if (lane == 0) {
                    const int slot = static_cast<int>(icount & 1u);
                    ok = mbar_wait(info_empty(slot), ((icount >> 1) & 1u) ^ 1u, abort_flag);
                    if (ok) {
                        info[2 * slot] = n_kt;
                        info[2 * slot + 1] = hole;
                        mbar_arrive(info_full(slot));
                    }
                    if (ok && n_kt > 0) {
                        const int qs = static_cast<int>(qcount & 1u);
                        const uint32_t qph = (qcount >> 1) & 1u;
                        ok = mbar_wait(q_empty(qs), qph ^ 1u, abort_flag);
                        if (ok) {
                            mbar_arrive_expect_tx(q_full(qs), L::kTileBytes);
#pragma unroll
                            for (int cb = 0; cb < L::kNumBlk; ++cb)
                                attn_tma(sbase + L::kOffQ + qs * L::kTileBytes + cb * L::kBlkBytes, &tmap_q,
                                         q_full(qs), cb * L::kBlkCols, qt * kAttnTile, h, bq, p.head_inner & 1);
                            q_issued_phase[qs] = static_cast<int>(qph);
                        }
                    }
                    auto load_k = [&](int j) -> bool {
                        const int st = static_cast<int>(kcount % STAGES);
                        const uint32_t ph = (kcount / STAGES) & 1u;
                        if (!mbar_wait(k_empty(st), ph ^ 1u, abort_flag)) return false;
                        mbar_arrive_expect_tx(k_full(st), L::kTileBytes);
#pragma unroll
                        for (int cb = 0; cb < L::kNumBlk; ++cb)
                            attn_tma(sbase + L::kOffK + st * L::kTileBytes + cb * L::kBlkBytes, &tmap_k,
                                     k_full(st), cb * L::kBlkCols, k_lo + j * kAttnTile, h, bq, p.head_inner & 2);
                        k_issued_phase[st] = static_cast<int>(ph);
                        ++kcount;
                        return true;
                    };
                    auto load_v = [&](int j) -> bool {
                        const int st = static_cast<int>(vcount % STAGES);
                        const uint32_t ph = (vcount / STAGES) & 1u;
                        if (!mbar_wait(v_empty(st), ph ^ 1u, abort_flag)) return false;
                        mbar_arrive_expect_tx(v_full(st), L::kTileBytes);
#pragma unroll
                        for (int cb = 0; cb < L::kNumBlk; ++cb)
                            attn_tma(sbase + L::kOffV + st * L::kTileBytes + cb * L::kBlkBytes, &tmap_v,
                                     v_full(st), cb * L::kBlkCols, k_lo + j * kAttnTile, h, bq, p.head_inner & 4);
                        v_issued_phase[st] = static_cast<int>(ph);
                        ++vcount;
                        return true;
                    };
                    for (int j = 0; ok && j < min(n_kt, L::kNS); ++j) ok = load_k(j);
                    for (int j = 0; ok && j < n_kt; ++j) {
                        ok = load_v(j);
                        if (ok && j + L::kNS < n_kt) ok = load_k(j + L::kNS);
                    }
                }
                if (n_kt > 0) ++qcount;
                ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                if (!ok) break;
            }
            if (lane == 0 && *abort_flag) {
                // no TMA write may still be in flight when the CTA exits
                for (int i = 0; i < 2; ++i)
                    if (q_issued_phase[i] >= 0) mbar_wait_drain(q_full(i), static_cast<uint32_t>(q_issued_phase[i]));
                for (int s = 0; s < STAGES; ++s) {
                    if (k_issued_phase[s] >= 0) mbar_wait_drain(k_full(s), static_cast<uint32_t>(k_issued_phase[s]));
                    if (v_issued_phase[s] >= 0) mbar_wait_drain(v_full(s), static_cast<uint32_t>(v_issued_phase[s]));
                }
            }
        } else if (warp == 9 && lane == 0) {
            // ------------------------------------------------- MMA issuer --
            constexpr uint32_t idesc_s = idesc_f16_f32(kAttnTile, kAttnTile, false, false);
            constexpr uint32_t idesc_o = idesc_f16_f32(kAttnTile, HD, false, true);
            constexpr int kStepsPerBlk = L::kBlkCols / 16;
            uint32_t tcount = 0, qcount = 0, icount = 0, singles = 0;
            uint32_t pcount[2] = {0, 0};
            if constexpr (SINGLE) {
                // Items of one key tile each, which the softmax groups take in
                // turn: S of item i+1 is issued before PV of item i, so both
                // groups run their softmax at once. S(t+1) refills the buffer
                // of item t+1-NS, whose PV this thread issued earlier (in the
                // previous iteration at the latest), and MMAs run in issue order.
                bool ok = true, pend = false;
                int pend_g = 0;
                uint32_t pend_t = 0;
                auto issue_pv = [&](int g, uint32_t t) -> bool {
                    const int st = static_cast<int>(t % STAGES);
                    const int sb = static_cast<int>(t % L::kNS);
                    // the group's previous item has read its O accumulator
                    if (!mbar_wait(o_free(g), (pcount[g] & 1u) ^ 1u, abort_flag)) return false;
                    if (!mbar_wait(p_full(sb), (t / L::kNS) & 1u, abort_flag)) return false;
                    if (!mbar_wait(v_full(st), (t / STAGES) & 1u, abort_flag)) return false;
                    tc_fence_after();
                    const uint32_t d = tmem_base + L::kColO + static_cast<uint32_t>(g * HD);
                    const uint32_t pa = tmem_base + L::kColS + static_cast<uint32_t>(sb * kAttnTile);
                    const uint32_t va = sbase + L::kOffV + st * L::kTileBytes;
#pragma unroll
                    for (int kk = 0; kk < kAttnTile / 16; ++kk)
                        mma_f16_ts(d, pa + kk * 8,
                                   smem_desc(va + kk * 16 * L::kRowBytes, L::kBlkBytes, 8 * L::kRowBytes, L::kSwz),
                                   idesc_o, kk != 0 ? 1u : 0u);
                    tc_commit(o_done(g));
                    tc_commit(v_empty(st));
                    tc_commit(o_final(g));
                    ++pcount[g];
                    return true;
                };
                for (int item = blockIdx.x; item < num_items; item += gridDim.x, ++icount) {
                    const int slot = static_cast<int>(icount & 1u);
                    if (!mbar_wait(info_full(slot), (icount >> 1) & 1u, abort_flag)) { ok = false; break; }
                    const int n_kt = info[2 * slot];
                    mbar_arrive(info_empty(slot));
                    if (n_kt == 0) continue;
                    const int g0 = first_group(n_kt, singles);
                    const int qs = static_cast<int>(qcount & 1u);
                    if (!mbar_wait(q_full(qs), (qcount >> 1) & 1u, abort_flag)) { ok = false; break; }
                    const uint32_t t = tcount;
                    const int st = static_cast<int>(t % STAGES);
                    const int sb = static_cast<int>(t % L::kNS);
                    if (!mbar_wait(k_full(st), (t / STAGES) & 1u, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d = tmem_base + L::kColS + static_cast<uint32_t>(sb * kAttnTile);
                    const uint32_t qa = sbase + L::kOffQ + qs * L::kTileBytes;
                    const uint32_t ka = sbase + L::kOffK + st * L::kTileBytes;
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk) {
                        const uint32_t off = (kk / kStepsPerBlk) * L::kBlkBytes + (kk % kStepsPerBlk) * 32;
                        mma_f16_ss(d, smem_desc(qa + off, 16, 8 * L::kRowBytes, L::kSwz),
                                   smem_desc(ka + off, 16, 8 * L::kRowBytes, L::kSwz), idesc_s, kk != 0 ? 1u : 0u);
                    }
                    tc_commit(s_full(g0, sb));
                    tc_commit(k_empty(st));
                    tc_commit(q_empty(qs));
                    if (pend && !issue_pv(pend_g, pend_t)) { ok = false; break; }
                    pend = true;
                    pend_g = g0;
                    pend_t = t;
                    ++tcount;
                    ++qcount;
                }
                if (ok && pend) issue_pv(pend_g, pend_t);
            }
            for (int item = blockIdx.x; !SINGLE && item < num_items; item += gridDim.x, ++icount) {
                const int slot = static_cast<int>(icount & 1u);
                if (!mbar_wait(info_full(slot), (icount >> 1) & 1u, abort_flag)) break;
                const int n_kt = info[2 * slot];
                mbar_arrive(info_empty(slot));
                if (n_kt == 0) continue;
                const int g0 = first_group(n_kt, singles);
                const int qs = static_cast<int>(qcount & 1u);
                if (!mbar_wait(q_full(qs), (qcount >> 1) & 1u, abort_flag)) break;
                tc_fence_after();
                // S(t) = Q K(t)^T into S/P buffer t mod NS (t counts this CTA's
                // key tiles). The buffer's previous P was read by a PV issued
                // earlier from this thread, and tcgen05 MMAs run in issue order.
                auto issue_s = [&](int j) -> bool {
                    const uint32_t t = tcount + j;
                    const int st = static_cast<int>(t % STAGES);
                    const int sb = static_cast<int>(t % L::kNS);
                    if (!mbar_wait(k_full(st), (t / STAGES) & 1u, abort_flag)) return false;
                    tc_fence_after();
                    const uint32_t d = tmem_base + L::kColS + static_cast<uint32_t>(sb * kAttnTile);
                    const uint32_t qa = sbase + L::kOffQ + qs * L::kTileBytes;
                    const uint32_t ka = sbase + L::kOffK + st * L::kTileBytes;
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk) {
                        const uint32_t off = (kk / kStepsPerBlk) * L::kBlkBytes + (kk % kStepsPerBlk) * 32;
                        mma_f16_ss(d, smem_desc(qa + off, 16, 8 * L::kRowBytes, L::kSwz),
                                   smem_desc(ka + off, 16, 8 * L::kRowBytes, L::kSwz), idesc_s,
                                   kk != 0 ? 1u : 0u);
                    }
                    tc_commit(s_full((g0 + j) & 1, sb));
                    tc_commit(k_empty(st));
                    if (j == n_kt - 1) tc_commit(q_empty(qs));   // this Q slot is no longer read
                    return true;
                };
                bool ok = true;
                for (int j = 0; ok && j < min(n_kt, L::kNS); ++j) ok = issue_s(j);
                for (int j = 0; ok && j < n_kt; ++j) {
                    const int g = (g0 + j) & 1;
                    const uint32_t t = tcount + j;
                    const int st = static_cast<int>(t % STAGES);
                    const int sb = static_cast<int>(t % L::kNS);
                    // the group's previous item has read its O accumulator
                    if (j < 2 && !mbar_wait(o_free(g), (pcount[g] & 1u) ^ 1u, abort_flag)) { ok = false; break; }
                    if (!mbar_wait(p_full(sb), (t / L::kNS) & 1u, abort_flag)) { ok = false; break; }
                    if (!mbar_wait(v_full(st), (t / STAGES) & 1u, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d = tmem_base + L::kColO + static_cast<uint32_t>(g * HD);
                    const uint32_t pa = tmem_base + L::kColS + static_cast<uint32_t>(sb * kAttnTile);
                    const uint32_t va = sbase + L::kOffV + st * L::kTileBytes;
#pragma unroll
                    for (int kk = 0; kk < kAttnTile / 16; ++kk)
                        mma_f16_ts(d, pa + kk * 8,
                                   smem_desc(va + kk * 16 * L::kRowBytes, L::kBlkBytes, 8 * L::kRowBytes, L::kSwz),
                                   idesc_o, (j >= 2 || kk != 0) ? 1u : 0u);
                    tc_commit(o_done(g));
                    tc_commit(v_empty(st));
                    if (j + 2 >= n_kt) tc_commit(o_final(g));   // the group's last PV of this item
                    if (j + L::kNS < n_kt && !issue_s(j + L::kNS)) { ok = false; break; }
                }
                if (!ok) break;
                ++pcount[g0];
                if (n_kt > 1) ++pcount[g0 ^ 1];
                tcount += n_kt;
                ++qcount;
            }
            tc_commit(drain_bar);
            mbar_wait_drain(drain_bar, 0);
        }
    } else {
        // -------------------------------------------- softmax warpgroups --
        regs_inc<kAttnRegsSoftmax>();
        const int grp = warp >> 2;                     // warpgroup 0 or 1
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;            // query row within the tile
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t t_s0 = tmem_base + lane_off + L::kColS;
        const uint32_t t_o0 = tmem_base + lane_off + L::kColO;
        const uint32_t t_o = t_o0 + static_cast<uint32_t>(grp * HD);
        const float c = p.scale_log2;
        uint32_t gtiles = 0, icount = 0, ccount = 0, singles = 0, tbase = 0, fcount = 0;
        uint32_t s_par = 0;   // bit b = phase parity of this group's next S in buffer b
        bool alive = true;
        for (int item = blockIdx.x; item < num_items && alive; item += gridDim.x, ++icount) {
            const int slot = static_cast<int>(icount & 1u);
            bool ok = mbar_wait(info_full(slot), (icount >> 1) & 1u, abort_flag);
            if (!__all_sync(0xffffffffu, ok)) { alive = false; break; }
            const int n_kt = info[2 * slot];
            const int hole = info[2 * slot + 1];
            __syncwarp();
            if (lane == 0) mbar_arrive(info_empty(slot));
            const int g0 = n_kt > 0 ? first_group(n_kt, singles) : 0;
            const uint32_t t_item = tbase;      // this CTA's index of the item's first key tile
            tbase += static_cast<uint32_t>(n_kt);

            int stream, qt, split, k_lo, k_hi;
            attn_item(p, item, stream, qt, split);
            attn_key_range(p, qt, split, k_lo, k_hi);
            const int h = p.packed ? stream : stream % p.H;
            const bool split_out = p.splits > 1;
            const int64_t ws_slot = split_out ? attn_slot(p, stream, qt, split) : 0;
            const int rq = qt * kAttnTile + row;
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
            // keys [kin_lo, kin_hi] are in range for every row of this warp
            const int kin_lo = __reduce_max_sync(0xffffffffu, klo_r);
            const int kin_hi = __reduce_min_sync(0xffffffffu, khi_r);
            auto out_row = [&]() -> __half* {
                const int64_t off = (p.out_layout == 1) ? ((static_cast<int64_t>(b) * p.S + s) * p.H + h) * HD
                                                        : ((static_cast<int64_t>(b) * p.H + h) * p.S + s) * HD;
                return reinterpret_cast<__half*>(p.out) + off;
            };
            if (n_kt == 0) {
                if (grp == 0 && q_ok && split_out) {
                    p.ws_ml[ws_slot * kAttnTile + row] = make_float2(-INFINITY, 0.0f);   // an empty run
                } else if (grp == 0 && q_ok) {
                    __half* op = out_row();
#pragma unroll
                    for (int i = 0; i < HD; i += 8) {
                        *reinterpret_cast<uint4*>(op + i) = make_uint4(0, 0, 0, 0);
                        if (p.out_lo != 0) *reinterpret_cast<uint4*>(op + p.out_lo + i) = make_uint4(0, 0, 0, 0);
                    }
                }
                continue;
            }
            const bool two = n_kt >= 2;
            if (!two && grp != g0) continue;           // the other group owns this single-tile item

            float m_used = -INFINITY, l_run = 0.0f;
            // Folds this tile's row max into the running (lazily rescaled) max:
            // rescales O in TMEM only when the max grew by more than
            // 2^kRescaleLog2. Returns m_used * c, the exp2 offset for this tile.
            auto softmax_rescale = [&](float mx) -> float {
                const float m_new = fmaxf(m_used, mx);
                float alpha = 1.0f;
                bool rescale = false;
                if (m_used == -INFINITY) {
                    m_used = m_new;          // no O yet (or O is all zero): nothing to scale
                } else if ((m_new - m_used) * c > kRescaleLog2) {
                    alpha = fast_exp2((m_used - m_new) * c);
                    rescale = true;
                }
                if (__any_sync(0xffffffffu, rescale)) {
                    // O holds the previous tiles of this group: wait for the last PV
                    const bool ok2 = mbar_wait(o_done(grp), (gtiles - 1) & 1u, abort_flag);
                    if (!__all_sync(0xffffffffu, ok2)) {
                        alive = false;
                        return 0.0f;
                    }
                    tc_fence_after();
#pragma unroll 1
                    for (int cc = 0; cc < HD; cc += 32) {
                        uint32_t orr[32];
                        tmem_ld_32x32b_x32(t_o + cc, orr);
                        tmem_ld_wait(orr);
#pragma unroll
                        for (int i = 0; i < 32; ++i) orr[i] = __float_as_uint(__uint_as_float(orr[i]) * alpha);
                        tmem_st_32x32b_x32(t_o + cc, orr);
                    }
                    tmem_st_wait();
                    if (rescale) {
                        l_run *= alpha;
                        m_used = m_new;
                    }
                }
                return (m_used == -INFINITY) ? 0.0f : m_used * c;
            };
            for (int j = (grp - g0) & 1; j < n_kt; j += 2, ++gtiles) {
                const int kc0 = k_lo + j * kAttnTile;
                // Interior tile: every key allowed for every row of the warp
                // (warp-uniform, so the branches below may hold .sync.aligned
                // TMEM loads). Other tiles build per-row allow masks.
                const bool interior = p.mask_kind != 2 && kc0 >= kin_lo && kc0 + (kAttnTile - 1) <= kin_hi &&
                                      (p.mask_kind == 0 || kc0 + kAttnTile <= hole);
                uint32_t allow[4] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu};
                if (!interior) {
                    // Allowed keys of this row in this tile as a 128-bit mask:
                    // bit i of allow[w] <-> key column 32 w + i.
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        const int lo = max(klo_r - kc0 - 32 * w, 0);
                        const int hi = min(khi_r - kc0 - 32 * w, 31);
                        uint32_t bits = 0u;
                        if (lo <= hi) bits = (hi == 31 ? 0xffffffffu : ((1u << (hi + 1)) - 1u)) & ~((1u << lo) - 1u);
                        allow[w] = bits;
                    }
                    if (p.mask_kind == 1 && kc0 + kAttnTile > hole) {
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            const int kc = kc0 + 32 * w + lane;
                            bool allowed = false;
                            if (kc < p.rows_total) {
                                int bk, sk;
                                if (p.packed) {
                                    bk = kc / p.S;
                                    sk = kc - bk * p.S;
                                } else {
                                    bk = stream / p.H;
                                    sk = kc;
                                }
                                allowed = p.mask[bk * p.ms0 + static_cast<int64_t>(sk) * p.ms3] != 0;
                            }
                            allow[w] &= __ballot_sync(0xffffffffu, allowed);
                        }
                    } else if (p.mask_kind == 2 && q_ok) {
                        const uint8_t* mrow = p.mask + b * p.ms0 + h * p.ms1 + static_cast<int64_t>(s) * p.ms2;
#pragma unroll 1
                        for (int i = 0; i < kAttnTile; ++i) {
                            const int kc = kc0 + i;
                            if (((allow[i >> 5] >> (i & 31)) & 1u) && mrow[static_cast<int64_t>(kc - klo_r) * p.ms3] == 0)
                                allow[i >> 5] &= ~(1u << (i & 31));
                        }
                    }
                }
                const uint32_t t = t_item + static_cast<uint32_t>(j);
                const int sb = static_cast<int>(t % L::kNS);
                const uint32_t t_s = t_s0 + static_cast<uint32_t>(sb * kAttnTile);
                ok = mbar_wait(s_full(grp, sb), (s_par >> sb) & 1u, abort_flag);
                s_par ^= 1u << sb;
                if (!__all_sync(0xffffffffu, ok)) { alive = false; break; }
                tc_fence_after();
                float sum8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                if (interior) {
                    // Every key allowed: the row max from all 128 scores in one
                    // TMEM round trip (four loads, one wait), then the
                    // exponentials over two reads of 64 (s c - m c as paired
                    // fp32 FMAs), P stored over the columns already read.
                    float mx8[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) mx8[k] = -INFINITY;
                    {
                        uint32_t sr[4][32];
#pragma unroll
                        for (int q = 0; q < 4; ++q) tmem_ld_32x32b_x32(t_s + q * 32, sr[q]);
                        tmem_ld_wait(sr[0]);
                        tmem_ld_wait(sr[1]);
                        tmem_ld_wait(sr[2]);
                        tmem_ld_wait(sr[3]);
#pragma unroll
                        for (int q = 0; q < 4; ++q)
#pragma unroll
                            for (int i = 0; i < 32; i += 2)
                                mx8[(i >> 1) & 7] = fmax3(mx8[(i >> 1) & 7], __uint_as_float(sr[q][i]),
                                                          __uint_as_float(sr[q][i + 1]));
                    }
                    const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                           fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
                    const float mc = softmax_rescale(mx);
                    if (!alive) break;
                    const unsigned long long c2 = f32x2(c, c), nmc2 = f32x2(-mc, -mc);
#pragma unroll 1
                    for (int h = 0; h < 2; ++h) {
                        uint32_t sr[2][32];
                        tmem_ld_32x32b_x32(t_s + h * 64, sr[0]);
                        tmem_ld_32x32b_x32(t_s + h * 64 + 32, sr[1]);
                        tmem_ld_wait(sr[0]);
                        tmem_ld_wait(sr[1]);
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            uint32_t pk[16];
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                float a0, a1;
                                f32x2_split(fma_x2(f32x2(__uint_as_float(sr[u][2 * i]),
                                                         __uint_as_float(sr[u][2 * i + 1])), c2, nmc2),
                                            a0, a1);
                                const float p0 = fast_exp2(a0);
                                const float p1 = fast_exp2(a1);
                                sum8[i & 7] += p0 + p1;
                                pk[i] = pack_half2(p0, p1);
                            }
                            tmem_st_32x32b_x16(t_s + h * 32 + u * 16, pk);
                        }
                    }
                } else {
                    // Some keys masked: two passes of 32 columns (compact code).
                    // A 32-key block no row of the warp may see (other sequences
                    // of a packed tile, keys above a causal diagonal) is skipped:
                    // no scores read, no exponentials, its P written as zeros.
                    float mx8[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) mx8[k] = -INFINITY;
#pragma unroll 1
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const uint32_t wq = q4 == 0 ? allow[0] : q4 == 1 ? allow[1] : q4 == 2 ? allow[2] : allow[3];
                        if (!__any_sync(0xffffffffu, wq != 0u)) continue;
                        uint32_t sr[32];
                        tmem_ld_32x32b_x32(t_s + q4 * 32, sr);
                        tmem_ld_wait(sr);
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            mx8[i & 7] = fmaxf(mx8[i & 7], ((wq >> i) & 1u) ? __uint_as_float(sr[i]) : -INFINITY);
                    }
                    const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                           fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
                    const float mc = softmax_rescale(mx);
                    if (!alive) break;
#pragma unroll 1
                    for (int q4 = 0; q4 < 4; ++q4) {
                        uint32_t sr[32], pk[16];
                        const uint32_t wq = q4 == 0 ? allow[0] : q4 == 1 ? allow[1] : q4 == 2 ? allow[2] : allow[3];
                        if (!__any_sync(0xffffffffu, wq != 0u)) {
#pragma unroll
                            for (int i = 0; i < 16; ++i) pk[i] = 0u;
                            tmem_st_32x32b_x16(t_s + q4 * 16, pk);
                            continue;
                        }
                        tmem_ld_32x32b_x32(t_s + q4 * 32, sr);
                        tmem_ld_wait(sr);
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            float p0 = fast_exp2(fmaf(__uint_as_float(sr[2 * i]), c, -mc));
                            float p1 = fast_exp2(fmaf(__uint_as_float(sr[2 * i + 1]), c, -mc));
                            p0 = ((wq >> (2 * i)) & 1u) ? p0 : 0.0f;
                            p1 = ((wq >> (2 * i + 1)) & 1u) ? p1 : 0.0f;
                            sum8[i & 7] += p0 + p1;
                            pk[i] = pack_half2(p0, p1);
                        }
                        tmem_st_32x32b_x16(t_s + q4 * 16, pk);
                    }
                }
                l_run += ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(p_full(sb));
            }
            if (!alive) break;
            // every PV of this group in this item has landed in O. A per-item
            // barrier: the phase of the last PV on o_done would alias an
            // earlier one if the group's previous PV were still in flight.
            ok = mbar_wait(o_final(grp), fcount & 1u, abort_flag);
            ++fcount;
            if (!__all_sync(0xffffffffu, ok)) { alive = false; break; }
            tc_fence_after();
            if (two && grp == 1) {
                // hand (max, sum) to group 0, which merges both accumulators
                ok = mbar_wait(comb_empty, (ccount & 1u) ^ 1u, abort_flag);
                if (!__all_sync(0xffffffffu, ok)) { alive = false; break; }
                comb[row] = make_float2(m_used, l_run);
                mbar_arrive(comb_full);
                ++ccount;
                continue;
            }
            float a0 = 1.0f, a1 = 0.0f, l_tot = l_run, m_tot = m_used;
            if (two) {
                ok = mbar_wait(comb_full, ccount & 1u, abort_flag);
                if (!__all_sync(0xffffffffu, ok)) { alive = false; break; }
                const float2 other = comb[row];
                mbar_arrive(comb_empty);
                ++ccount;
                const float m = fmaxf(m_used, other.x);
                a0 = (m_used == -INFINITY) ? 0.0f : fast_exp2((m_used - m) * c);
                a1 = (other.x == -INFINITY) ? 0.0f : fast_exp2((other.x - m) * c);
                l_tot = l_run * a0 + other.y * a1;
                m_tot = m;
            }
            if (split_out) {
                // this key run's unnormalised rows and their (max, sum)
                float* wo = p.ws_o + (ws_slot * kAttnTile + row) * HD;
#pragma unroll 1
                for (int cc = 0; cc < HD; cc += 16) {
                    uint32_t o0[16], o1[16];
                    tmem_ld_32x32b_x16(t_o + cc, o0);
                    if (two) tmem_ld_32x32b_x16(t_o0 + HD + cc, o1);
                    tmem_ld_wait16(o0);
                    if (two) tmem_ld_wait16(o1);
                    float v[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        v[i] = two ? fmaf(__uint_as_float(o0[i]), a0, __uint_as_float(o1[i]) * a1)
                                   : __uint_as_float(o0[i]) * a0;
                    if (q_ok) {
#pragma unroll
                        for (int i = 0; i < 16; i += 4)
                            *reinterpret_cast<float4*>(wo + cc + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
                    }
                }
                if (q_ok) p.ws_ml[ws_slot * kAttnTile + row] = make_float2(m_tot, l_tot);
                tc_fence_before();
                mbar_arrive(o_free(grp));
                if (two) mbar_arrive(o_free(1));
                continue;
            }
            const float inv = l_tot > 0.0f ? 1.0f / l_tot : 0.0f;
            a0 *= inv;
            a1 *= inv;
            __half* op = out_row();
#pragma unroll 1
            for (int cc = 0; cc < HD; cc += 16) {
                uint32_t o0[16], o1[16];
                tmem_ld_32x32b_x16(t_o + cc, o0);
                if (two) tmem_ld_32x32b_x16(t_o0 + HD + cc, o1);
                tmem_ld_wait16(o0);
                if (two) tmem_ld_wait16(o1);
                float v[16];
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    v[i] = two ? fmaf(__uint_as_float(o0[i]), a0, __uint_as_float(o1[i]) * a1)
                               : __uint_as_float(o0[i]) * a0;
                uint32_t w[8];
                if (p.out_lo != 0) {
                    // the fp16 pair's lo plane too (three-product mode)
                    uint32_t wl[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) split_half2(v[2 * i], v[2 * i + 1], w[i], wl[i]);
                    if (q_ok) {
                        *reinterpret_cast<uint4*>(op + p.out_lo + cc) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
                        *reinterpret_cast<uint4*>(op + p.out_lo + cc + 8) = make_uint4(wl[4], wl[5], wl[6], wl[7]);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i) w[i] = pack_half2(v[2 * i], v[2 * i + 1]);
                }
                if (q_ok) {
                    *reinterpret_cast<uint4*>(op + cc) = make_uint4(w[0], w[1], w[2], w[3]);
                    *reinterpret_cast<uint4*>(op + cc + 8) = make_uint4(w[4], w[5], w[6], w[7]);
                }
            }
            tc_fence_before();
            mbar_arrive(o_free(grp));
            if (two) mbar_arrive(o_free(1));
        }
    }

    // ------------------------------------------------------------ teardown --
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem_base, L::kTmemCols);
    }
}

// Split-KV combine: one warp per query row folds the row's key runs, in run
// order, and stores the normalised fp16 row (and its fp16 pair's lo plane
// when out_lo is set). Runs with no allowed key (sum 0) add nothing; a row
// with none at all is written as 0. Not packed (split-KV needs tiles of one
// sequence). Lane l owns head-dim columns [l * HD/32, (l+1) * HD/32).
constexpr int kCombineWarps = 8;

template <int HD>
__global__ void __launch_bounds__(kCombineWarps * 32) attn_combine_kernel(const AttnParams p) {
    pdl_wait();
    pdl_launch_dependents();
    constexpr int kPer = HD / 32;
    const int lane = threadIdx.x & 31;
    const int64_t gw = static_cast<int64_t>(blockIdx.x) * kCombineWarps + (threadIdx.x >> 5);
    const int64_t tiles = static_cast<int64_t>(p.num_streams) * p.num_q_tiles;
    if (gw >= tiles * kAttnTile) return;
    const int row = static_cast<int>(gw % kAttnTile);
    const int64_t tile = gw / kAttnTile;
    const int qt = static_cast<int>(tile % p.num_q_tiles);
    const int stream = static_cast<int>(tile / p.num_q_tiles);
    const int s = qt * kAttnTile + row;
    if (s >= p.rows_total) return;
    const float c = p.scale_log2;
    float m_all = -INFINITY;
    for (int r = 0; r < p.splits; ++r) {
        const float2 ml = p.ws_ml[attn_slot(p, stream, qt, r) * kAttnTile + row];
        if (ml.y > 0.0f) m_all = fmaxf(m_all, ml.x);
    }
    float acc[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) acc[i] = 0.0f;
    float l_all = 0.0f;
    for (int r = 0; r < p.splits; ++r) {
        const int64_t sl = attn_slot(p, stream, qt, r);
        const float2 ml = p.ws_ml[sl * kAttnTile + row];
        if (!(ml.y > 0.0f)) continue;
        const float wgt = fast_exp2((ml.x - m_all) * c);
        l_all = fmaf(ml.y, wgt, l_all);
        const float* o = p.ws_o + (sl * kAttnTile + row) * HD + lane * kPer;
#pragma unroll
        for (int i = 0; i < kPer; ++i) acc[i] = fmaf(o[i], wgt, acc[i]);
    }
    const float inv = l_all > 0.0f ? 1.0f / l_all : 0.0f;
    const int b = stream / p.H, h = stream % p.H;
    const int64_t off = (p.out_layout == 1) ? ((static_cast<int64_t>(b) * p.S + s) * p.H + h) * HD
                                            : ((static_cast<int64_t>(b) * p.H + h) * p.S + s) * HD;
    __half* op = reinterpret_cast<__half*>(p.out) + off + lane * kPer;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const float y = acc[i] * inv;
        const __half hi = __float2half_rn(y);
        op[i] = hi;
        if (p.out_lo != 0) op[p.out_lo + i] = __float2half_rn(y - __half2float(hi));
    }
}

}  // namespace dotl
