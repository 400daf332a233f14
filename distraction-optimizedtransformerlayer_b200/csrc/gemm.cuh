// C = epilogue(A[M,K] * W[N,K]^T + bias) on the 5th-generation tensor cores.
//
// Replaces the reference's csrc/linear_gelu.cuh (gemm_bias_act_kernel
// :186-462, wmma fp16 fragments on sm_80). Same arithmetic contract: fp16
// operands, fp32 accumulation, bias added in fp32, exact erf GELU.
//
// Design (sm_100a):
//   * persistent: one CTA per SM walks the output tiles with a stride of
//     gridDim.x; tile (m, n) with n fastest, so CTAs running together share
//     the same A row-block and the weight matrix stays L2 resident;
//   * warp-specialised: warp 0 issues TMA loads into a STAGES-deep ring of
//     128B-swizzled smem tiles, warp 1 issues tcgen05.mma (M=128, N=BN, K=16)
//     into one of two TMEM accumulators, warps 2-9 drain the other
//     accumulator through tcgen05.ld, run the fused epilogue and TMA-store
//     the result through swizzled smem, so the epilogue of tile i overlaps
//     the main loop of tile i+1;
//   * epilogues: bias, bias+GELU (fp16 out, the FFN hidden), bias + residual
//     with an optional padded-row mask (fp32 out, the residual stream);
//   * SPLIT2: two CTAs of a cluster split K for long-K problems with too few
//     tiles, exchanging partial halves through distributed shared memory;
//   * PEER: each 128-row output tile is TMA-stored into the receive slot of
//     the tensor-parallel rank that owns those rows (over NVLink), the
//     reduce-scatter of the row-parallel GEMMs done inside the GEMM;
//   * three-product mode (runtime, X3Pass): A and W each come as an fp16 pair
//     of planes (hi = fp16(v), lo = fp16(v - hi)), and the k loop runs three
//     passes into one accumulator, A_hi W_hi + A_lo W_hi + A_hi W_lo, which
//     carries the operands to about 22 bits instead of 11 (for stacks of
//     layers whose error would otherwise pass the harness's bound). The fp16
//     epilogue can likewise write its output as such a pair.
//
// A and W are K-major (rows contiguous along K), which is both nn.Linear's
// weight layout and the activations' row layout: no transpose anywhere.

#pragma once

#include "dotl_common.cuh"

namespace dotl {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;                  // one 128-byte swizzle atom of fp16
constexpr int kGemmThreads = 320;            // producer, MMA, 8 epilogue warps
constexpr uint32_t kGemmATileBytes = kGemmBM * kGemmBK * 2;

enum GemmResidMode : int {
    kResidNone = 0,       // out = acc + bias (+ GELU)
    kResidAdd = 1,        // out = resid + (acc + bias)
    kResidAddMaskSub = 2, // out = resid + (row valid ? acc + bias : 0)
    kResidAddMaskAll = 3, // out = row valid ? resid + acc + bias : 0
    kMaskRows = 4,        // out = row valid ? acc + bias : 0 (no residual)
};

struct GemmParams {
    int M, N, K;
    int num_m_tiles, num_n_tiles;
    const float* bias;       // [N]
    const float* resid;      // [M, ldr] fp32, or null
    int64_t ldr;
    const uint8_t* row_valid;  // [M] (nonzero = valid) or null
    int resid_mode;
    int act;                 // 0 = none, 1 = exact GELU
    void* out;               // [M, ldo], fp16 or fp32
    int64_t ldo;
    int x3_nkb;              // three-product mode: k-blocks per pass (0: one fp16 pass)
    int a_lo_row, w_lo_row;  // three-product mode: rows of the lo planes in the A and W maps
    int out_lo;              // fp16 out: also store the lo half through po.map[0]
};

// The three passes of the three-product mode: k-block kb of the combined loop
// reads A plane (pass == 1 ? lo : hi) and W plane (pass == 2 ? lo : hi) at
// k-block kb mod nkb. The planes sit in one tensor map each, the lo plane
// a_lo / w_lo rows below the hi plane. A tile that reaches past the hi plane's
// last row reads lo rows (or zeros) into accumulator rows or columns that are
// never stored.
struct X3Pass {
    int nkb;                 // 0: a single pass
    int a_lo, w_lo;
};

// Output tiles scattered over the ranks of a tensor-parallel group: row block
// m (rows [128 m, 128 m + 128)) belongs to rank (128 m) / rows, which receives
// it at row 128 m - rank * rows of map[rank] (its receive slot for this rank,
// in its own memory, reached over NVLink). Plain TMA stores, one destination each.
constexpr int kGemmPeerMax = 8;
struct GemmPeerOut {
    CUtensorMap map[kGemmPeerMax];
    int rows;                // rows per rank; 0: the ordinary output map
};

// BROWS: the W rows a CTA stages per k-block (BN, or BN / 2 for a CTA pair,
// which splits the tile's W rows between its two CTAs).
template <int BN, int STAGES, int BROWS = BN>
struct GemmSmem {
    static constexpr uint32_t kBTileBytes = BROWS * kGemmBK * 2;
    static constexpr uint32_t kStageBytes = kGemmATileBytes + kBTileBytes;
    static constexpr uint32_t kOffA = 0;
    static constexpr uint32_t kOffB = STAGES * kGemmATileBytes;
    // per epilogue warp: one 32-row x 128-byte staging buffer for TMA stores
    // (an fp32 chunk, or two fp16 chunks of 64-byte rows used alternately)
    static constexpr uint32_t kOffStage = kOffB + STAGES * kBTileBytes;
    static constexpr uint32_t kStageBufBytes = 32 * 128;
    static constexpr uint32_t kOffBar = kOffStage + 8 * kStageBufBytes;
    // full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], drain (GemmBars),
    // then the split-K pair's peer_ready, recv_full and exit, then one
    // residual-block barrier per epilogue warp
    static constexpr uint32_t kNumBars = 2 * STAGES + 16;
    static constexpr uint32_t kOffSlot = kOffBar + kNumBars * 8;
    static constexpr uint32_t kOffAbort = kOffSlot + 4;
    static constexpr uint32_t kBytes = kOffAbort + 4;
    static constexpr uint32_t kAlloc = kBytes + 1024;   // room to align the base to 1024
    // Two accumulators of BN fp32 columns, the second at column kAccStride.
    // tcgen05.alloc takes a power of two, so widths between the powers (160,
    // 192, 224) allocate 512 columns and put the second accumulator at 256.
    static constexpr uint32_t kTmemCols = 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;
    static constexpr uint32_t kAccStride = kTmemCols / 2;
    static_assert(kAlloc <= 232448, "dynamic shared memory over the 227 KB an sm_100a CTA may use");
    static_assert(BN % 32 == 0 && BN <= 256, "the epilogue walks 32-column chunks of at most 256 columns");
};

// Which output tiles a CTA visits: t = first, first + stride, ... < count.
// With n_fixed < 0, t enumerates (m, n) with n fastest; otherwise t is the M
// block and every tile is in N block n_fixed (the cluster-row schedule of the
// LayerNorm epilogue kernel).
struct TileSched {
    int first, stride, count, n_tiles, n_fixed;
    __device__ __forceinline__ void decode(int t, int& m_blk, int& n_blk) const {
        if (n_fixed >= 0) {
            m_blk = t;
            n_blk = n_fixed;
        } else {
            m_blk = t / n_tiles;
            n_blk = t - m_blk * n_tiles;
        }
    }
};

// Barriers every GEMM kernel keeps at the start of its barrier block:
// full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], drain.
template <int STAGES>
struct GemmBars {
    uint32_t bar0;
    __device__ __forceinline__ uint32_t full(int s) const { return bar0 + 8u * s; }
    __device__ __forceinline__ uint32_t empty(int s) const { return bar0 + 8u * (STAGES + s); }
    __device__ __forceinline__ uint32_t accf(int b) const { return bar0 + 8u * (2 * STAGES + b); }
    __device__ __forceinline__ uint32_t acce(int b) const { return bar0 + 8u * (2 * STAGES + 2 + b); }
    __device__ __forceinline__ uint32_t drain() const { return bar0 + 8u * (2 * STAGES + 4); }
    static constexpr int kCount = 2 * STAGES + 5;
};

// TMA producer (one thread): A and W k-blocks [kb0, kb1) of every scheduled
// tile into the STAGES-deep ring. On abort, waits out the copies in flight.
template <int BN, int STAGES>
__device__ __forceinline__ void gemm_produce(const CUtensorMap* tmap_a, const CUtensorMap* tmap_w, uint32_t sbase,
                                             GemmBars<STAGES> bars, volatile int* abort_flag, const TileSched& ts,
                                             int kb0, int kb1, X3Pass x3 = {0, 0, 0}) {
    using L = GemmSmem<BN, STAGES>;
    int stage = 0;
    uint32_t phase = 0;
    int issued_phase[STAGES];
    for (int s = 0; s < STAGES; ++s) issued_phase[s] = -1;
    for (int t = ts.first; t < ts.count; t += ts.stride) {
        int m_blk, n_blk;
        ts.decode(t, m_blk, n_blk);
        for (int kb = kb0; kb < kb1; ++kb) {
            if (!mbar_wait(bars.empty(stage), phase ^ 1u, abort_flag)) goto producer_done;
            mbar_arrive_expect_tx(bars.full(stage), L::kStageBytes);
            int ka = kb, arow = m_blk * kGemmBM, wrow = n_blk * BN;
            if (x3.nkb > 0) {
                const int pass = kb / x3.nkb;
                ka = kb - pass * x3.nkb;
                if (pass == 1) arow += x3.a_lo;
                if (pass == 2) wrow += x3.w_lo;
            }
            tma_load_2d(sbase + L::kOffA + stage * kGemmATileBytes, tmap_a, bars.full(stage), ka * kGemmBK, arow);
            tma_load_2d(sbase + L::kOffB + stage * L::kBTileBytes, tmap_w, bars.full(stage), ka * kGemmBK, wrow);
            issued_phase[stage] = static_cast<int>(phase);
            if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
            }
        }
    }
producer_done:
    if (*abort_flag) {
        // Copies still in flight land in this CTA's smem: wait them out.
        for (int s = 0; s < STAGES; ++s)
            if (issued_phase[s] >= 0) mbar_wait_drain(bars.full(s), static_cast<uint32_t>(issued_phase[s]));
    }
}

// MMA issuer (one thread): k-blocks [kb0, kb1) of each scheduled tile into
// TMEM accumulator 0, 1, 0, ... (BN columns each); every issued MMA has
// completed on return.
template <int BN, int STAGES>
__device__ __forceinline__ void gemm_mma(uint32_t sbase, uint32_t tmem_base, GemmBars<STAGES> bars,
                                         volatile int* abort_flag, const TileSched& ts, int kb0, int kb1) {
    using L = GemmSmem<BN, STAGES>;
    constexpr uint32_t idesc = idesc_f16_f32(kGemmBM, BN, false, false);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = ts.first; t < ts.count; t += ts.stride) {
        if (!mbar_wait(bars.acce(acc), acc_phase ^ 1u, abort_flag)) goto mma_done;
        tc_fence_after();
        {
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc) * L::kAccStride;
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(bars.full(stage), phase, abort_flag)) goto mma_done;
                tc_fence_after();
                const uint32_t a_addr = sbase + L::kOffA + stage * kGemmATileBytes;
                const uint32_t b_addr = sbase + L::kOffB + stage * L::kBTileBytes;
#pragma unroll
                for (int kk = 0; kk < kGemmBK / 16; ++kk) {
                    const uint64_t ad = smem_desc(a_addr + kk * 32, 16, 1024, kSwizzle128);
                    const uint64_t bd = smem_desc(b_addr + kk * 32, 16, 1024, kSwizzle128);
                    mma_f16_ss(d_tmem, ad, bd, idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
                }
                tc_commit(bars.empty(stage));
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        tc_commit(bars.accf(acc));
        if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
        }
    }
mma_done:
    // Every MMA this thread issued has completed once drain fires.
    tc_commit(bars.drain());
    mbar_wait_drain(bars.drain(), 0);
}

// CTA-pair producer (PAIR, one thread in each CTA): per k-block this CTA's
// 128 rows of the pair's 256-row A block and its half of the tile's W rows,
// both counted on the leader's full barrier, which the leader arms for the
// pair's bytes. The stage is free again when the leader's MMA commit arrives
// on this CTA's empty barrier.
template <int BN, int STAGES>
__device__ __forceinline__ void gemm_produce_pair(const CUtensorMap* tmap_a, const CUtensorMap* tmap_w,
                                                  uint32_t sbase, GemmBars<STAGES> bars, volatile int* abort_flag,
                                                  const TileSched& ts, int nkb, X3Pass x3, uint32_t rank) {
    using L = GemmSmem<BN, STAGES, BN / 2>;
    int stage = 0;
    uint32_t phase = 0;
    int issued_phase[STAGES];
    for (int s = 0; s < STAGES; ++s) issued_phase[s] = -1;
    for (int t = ts.first; t < ts.count; t += ts.stride) {
        int m_blk, n_blk;
        ts.decode(t, m_blk, n_blk);
        for (int kb = 0; kb < nkb; ++kb) {
            if (!mbar_wait(bars.empty(stage), phase ^ 1u, abort_flag)) goto pair_producer_done;
            if (rank == 0) mbar_arrive_expect_tx(bars.full(stage), 2 * L::kStageBytes);
            int ka = kb;
            int arow = m_blk * 2 * kGemmBM + static_cast<int>(rank) * kGemmBM;
            int wrow = n_blk * BN + static_cast<int>(rank) * (BN / 2);
            if (x3.nkb > 0) {
                const int pass = kb / x3.nkb;
                ka = kb - pass * x3.nkb;
                if (pass == 1) arow += x3.a_lo;
                if (pass == 2) wrow += x3.w_lo;
            }
            const uint32_t fbar = mapa_shared(bars.full(stage), 0);
            tma_load_2d_pair(sbase + L::kOffA + stage * kGemmATileBytes, tmap_a, fbar, ka * kGemmBK, arow);
            tma_load_2d_pair(sbase + L::kOffB + stage * L::kBTileBytes, tmap_w, fbar, ka * kGemmBK, wrow);
            issued_phase[stage] = static_cast<int>(phase);
            if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
            }
        }
    }
pair_producer_done:
    if (*abort_flag && rank == 0) {
        // the leader's full barriers count both CTAs' copies: wait them out
        for (int s = 0; s < STAGES; ++s)
            if (issued_phase[s] >= 0) mbar_wait_drain(bars.full(s), static_cast<uint32_t>(issued_phase[s]));
    }
}

// CTA-pair MMA issuer (the leader's one thread): M = 256 MMAs over both CTAs'
// operands into both CTAs' TMEM; each commit arrives on the barrier in both
// CTAs (one commit per CTA, no fan-out form). The accumulator is free again
// once all 16 epilogue warps of the pair have arrived on the leader's acce.
template <int BN, int STAGES>
__device__ __forceinline__ void gemm_mma_pair(uint32_t sbase, uint32_t tmem_base, GemmBars<STAGES> bars,
                                              volatile int* abort_flag, const TileSched& ts, int nkb) {
    using L = GemmSmem<BN, STAGES, BN / 2>;
    constexpr uint32_t idesc = idesc_f16_f32(2 * kGemmBM, BN, false, false);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = ts.first; t < ts.count; t += ts.stride) {
        if (!mbar_wait_cluster(bars.acce(acc), acc_phase ^ 1u, abort_flag)) goto pair_mma_done;
        tc_fence_after();
        {
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc) * L::kAccStride;
            for (int kb = 0; kb < nkb; ++kb) {
                if (!mbar_wait(bars.full(stage), phase, abort_flag)) goto pair_mma_done;
                tc_fence_after();
                const uint32_t a_addr = sbase + L::kOffA + stage * kGemmATileBytes;
                const uint32_t b_addr = sbase + L::kOffB + stage * L::kBTileBytes;
#pragma unroll
                for (int kk = 0; kk < kGemmBK / 16; ++kk) {
                    const uint64_t ad = smem_desc(a_addr + kk * 32, 16, 1024, kSwizzle128);
                    const uint64_t bd = smem_desc(b_addr + kk * 32, 16, 1024, kSwizzle128);
                    mma_f16_ss_pair(d_tmem, ad, bd, idesc, (kb != 0 || kk != 0) ? 1u : 0u);
                }
                tc_commit_pair(mapa_shared(bars.empty(stage), 0));
                tc_commit_pair(mapa_shared(bars.empty(stage), 1));
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        tc_commit_pair(mapa_shared(bars.accf(acc), 0));
        tc_commit_pair(mapa_shared(bars.accf(acc), 1));
        if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
        }
    }
pair_mma_done:
    tc_commit_pair(mapa_shared(bars.drain(), 0));
    mbar_wait_drain(bars.drain(), 0);
}

// SPLIT2: a cluster of two CTAs shares each output tile, CTA r running
// k-blocks [r nkb/2, (r+1) nkb/2). After the main loop each sends the other's
// column half of its partial accumulator into the other's shared memory (the
// stage ring, idle by then: every CTA has exactly one tile) and finishes its
// own half as partial_0 + partial_1 (one fp32 add, which commutes: both CTAs
// and every run give the same bits). Used when a problem has too few tiles
// to fill the SMs with long K.
//
// PAIR: a cluster of two CTAs computes each 256 x BN output tile with M = 256
// MMAs (tcgen05 cta_group::2): CTA r stages rows [128 r, 128 r + 128) of the
// tile's A block and W rows [r BN/2, (r+1) BN/2) of its N block, so per MMA each
// SM's shared memory feeds half the W operand it would alone; CTA r's TMEM
// holds output rows [128 r, 128 r + 128), drained by its own epilogue.
template <int BN, int STAGES, bool OUT_F16, bool SPLIT2 = false, bool PEER = false, bool PAIR = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ CUtensorMap tmap_out, const __grid_constant__ CUtensorMap tmap_r,
                   const GemmParams p, const __grid_constant__ GemmPeerOut po) {
    static_assert(!(PAIR && (SPLIT2 || PEER)), "a CTA pair is neither split-K nor peer-scattered");
    using L = GemmSmem<BN, STAGES, PAIR ? BN / 2 : BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + L::kOffBar;
    const GemmBars<STAGES> bars{bar0};
    const uint32_t peer_ready = bar0 + 8u * (GemmBars<STAGES>::kCount);
    const uint32_t recv_full = bar0 + 8u * (GemmBars<STAGES>::kCount + 1);
    const uint32_t exit_bar = bar0 + 8u * (GemmBars<STAGES>::kCount + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffAbort);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffSlot);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = (SPLIT2 || PAIR) ? cluster_ctarank() : 0u;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(bars.full(s), 1);
            mbar_init(bars.empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bars.accf(b), 1);
            mbar_init(bars.acce(b), PAIR ? 16 : 256);   // pair: one arrival per epilogue warp of both CTAs
        }
        mbar_init(bars.drain(), 1);
        mbar_init(peer_ready, 256);
        mbar_init(recv_full, 256);
        mbar_init(exit_bar, 2);
        for (int w = 0; w < 8; ++w) mbar_init(bar0 + 8u * (GemmBars<STAGES>::kCount + 3 + w), 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_map(&tmap_a);
        tma_prefetch_map(&tmap_w);
        tma_prefetch_map(&tmap_out);
        tma_prefetch_map(&tmap_r);
        if constexpr (PEER)
            for (int r = 0; r * po.rows < p.M && r < kGemmPeerMax; ++r) tma_prefetch_map(&po.map[r]);
    }
    if constexpr (SPLIT2 || PAIR) cluster_sync_after_init();
    pdl_wait();
    pdl_launch_dependents();
    if (warp == 1) {
        if constexpr (PAIR) {
            tmem_alloc_pair(smem_u32(tmem_slot), L::kTmemCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    if constexpr (PAIR) {
        cluster_sync_after_init();   // both CTAs' TMEM exists before the leader's first MMA
    } else {
        __syncthreads();
    }
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int num_tiles = p.num_m_tiles * p.num_n_tiles;
    const int num_kb = p.x3_nkb > 0 ? 3 * p.x3_nkb : (p.K + kGemmBK - 1) / kGemmBK;
    const X3Pass x3{p.x3_nkb, p.a_lo_row, p.w_lo_row};

    const int cta_unit = (SPLIT2 || PAIR) ? static_cast<int>(blockIdx.x) / 2 : static_cast<int>(blockIdx.x);
    const int units = (SPLIT2 || PAIR) ? static_cast<int>(gridDim.x) / 2 : static_cast<int>(gridDim.x);
    const TileSched ts{cta_unit, units, num_tiles, p.num_n_tiles, -1};
    const int kb0 = SPLIT2 ? static_cast<int>(rank) * (num_kb / 2) : 0;
    const int kb1 = SPLIT2 ? (rank == 0 ? num_kb / 2 : num_kb) : num_kb;
    if (warp == 0 && lane == 0) {
        if constexpr (PAIR) gemm_produce_pair<BN, STAGES>(&tmap_a, &tmap_w, sbase, bars, abort_flag, ts, num_kb, x3, rank);
        else gemm_produce<BN, STAGES>(&tmap_a, &tmap_w, sbase, bars, abort_flag, ts, kb0, kb1, x3);
    } else if (warp == 1 && lane == 0) {
        if constexpr (PAIR) {
            if (rank == 0) gemm_mma_pair<BN, STAGES>(sbase, tmem_base, bars, abort_flag, ts, num_kb);
        } else {
            gemm_mma<BN, STAGES>(sbase, tmem_base, bars, abort_flag, ts, kb0, kb1);
        }
    } else if (warp >= 2) {
        // -------------------------------------------------------- epilogue --
        // Eight warps, two per TMEM lane quarter (the 32 rows a warp may
        // read); the two split the tile's 32-column chunks alternately. Per
        // chunk a warp reads the accumulator, applies bias / GELU / residual /
        // row mask, writes the 32-row block into a swizzled smem buffer
        // (128 B rows for fp32, 64 B for fp16; conflict-free) and one lane
        // TMA-stores it, so every store is a full-line bulk copy.
        constexpr int kCW = 32;
        constexpr int kRowB = OUT_F16 ? 64 : 128;       // staged bytes per row
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row_in_tile = quarter * 32 + lane;
        const uint32_t stage_addr = sbase + L::kOffStage + static_cast<uint32_t>(warp - 2) * L::kStageBufBytes;
        uint8_t* stage_ptr = smem + L::kOffStage + (warp - 2) * L::kStageBufBytes;
        const bool has_resid = p.resid_mode != kResidNone && p.resid_mode != kMaskRows;
        // fp32 out with a residual: each 32 x 32 residual block comes in by TMA
        // (through tmap_r) into the warp's staging buffer, and the result
        // leaves from the same buffer, so every global access is a full-line
        // bulk copy (a lane per row reading its own 128 bytes touched 32 lines
        // per load instruction)
        const bool resid_tma = !OUT_F16 && has_resid;
        const uint32_t rbar = bar0 + 8u * (GemmBars<STAGES>::kCount + 3 + (warp - 2));
        uint32_t r_issued = 0, r_waited = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t nstore = 0;                              // chunks this warp has staged
        for (int t = ts.first; t < ts.count; t += ts.stride) {
            int m_blk, n_blk;
            ts.decode(t, m_blk, n_blk);
            // first output row of this CTA's accumulator rows
            const int row0 = PAIR ? m_blk * 2 * kGemmBM + static_cast<int>(rank) * kGemmBM : m_blk * kGemmBM;
            const int row = row0 + row_in_tile;
            const int n0 = n_blk * BN;
            const bool row_ok = row < p.M;
            const bool valid = (p.row_valid == nullptr) || !row_ok || (p.row_valid[row] != 0);
            // Global reads are issued ahead of the accumulator: the bias as
            // one coalesced float per lane (column nc + lane, broadcast by
            // shuffles), one chunk ahead; the residual row of a full chunk at
            // the top of the chunk (for the first chunk while the main loop
            // still runs).
            float4 rr[kCW / 4];
            auto load_bias = [&](int nc) -> float {
                return (p.bias != nullptr && nc + lane < p.N) ? __ldg(p.bias + nc + lane) : 0.0f;
            };
            // where this tile's rows go: the output map, or the owning rank's
            const CUtensorMap* omap = &tmap_out;
            int orow = row0;
            if constexpr (PEER) {
                const int owner = orow / po.rows;
                omap = &po.map[owner];
                orow -= owner * po.rows;
            }
            auto issue_resid = [&](int nc) {
                __syncwarp();
                if (lane == 0) {
                    bulk_wait_read<0>();              // the last store has read the buffer
                    fence_proxy_async_smem();
                    mbar_arrive_expect_tx(rbar, 4096);
                    tma_load_2d(stage_addr, &tmap_r, rbar, nc, row0 + quarter * 32);
                }
                ++r_issued;
            };
            auto load_resid = [&](int nc) {
                if (!resid_tma && has_resid && row_ok && nc + kCW <= p.N) {
                    const float4* rp = reinterpret_cast<const float4*>(p.resid + static_cast<int64_t>(row) * p.ldr + nc);
#pragma unroll
                    for (int j = 0; j < kCW / 4; ++j) rr[j] = rp[j];
                }
            };
            // Columns this CTA finishes: all BN, or its half of a split-K pair.
            const int c_lo = SPLIT2 ? static_cast<int>(rank) * (BN / 2) : 0;
            const int c_hi = SPLIT2 ? c_lo + BN / 2 : BN;
            const int c_first = c_lo + half * kCW;
            float b_cur = load_bias(n0 + c_first);
            if (resid_tma && n0 + c_first < p.N) issue_resid(n0 + c_first);
            load_resid(n0 + c_first);
            bool ok = mbar_wait(bars.accf(acc), acc_phase, abort_flag);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc_fence_after();
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                   static_cast<uint32_t>(acc) * L::kAccStride;
            // Split-K exchange buffer: [128 rows][BN/2 fp32] in the stage ring,
            // 16-byte granule g of row r at g ^ (r & mask) (conflict-free).
            constexpr int kHalfGranules = BN / 8;
            const uint32_t recv_row = static_cast<uint32_t>(row_in_tile) * (BN / 2) * 4;
            auto recv_pos = [&](int col) -> uint32_t {
                return recv_row + static_cast<uint32_t>(((col >> 2) ^ (row_in_tile & (kHalfGranules - 1))) << 4);
            };
            if constexpr (SPLIT2) {
                // This CTA's only tile is accumulated, so its ring is idle: the
                // partner may write there. Send the partner's half, receive ours.
                const uint32_t partner = rank ^ 1u;
                mbar_arrive_cluster(mapa_shared(peer_ready, partner));
                bool ok2 = mbar_wait_cluster(peer_ready, 0, abort_flag);
                if (!__all_sync(0xffffffffu, ok2)) break;
                const int p_lo = static_cast<int>(partner) * (BN / 2);
                const uint32_t recv_remote = mapa_shared(sbase + L::kOffA, partner);
#pragma unroll 1
                for (int c = p_lo + half * kCW; c < p_lo + BN / 2; c += 2 * kCW) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + c, r);
                    tmem_ld_wait(r);
#pragma unroll
                    for (int q = 0; q < kCW / 4; ++q)
                        st_cluster_v4f32(recv_remote + recv_pos(c - p_lo + 4 * q), __uint_as_float(r[4 * q]),
                                         __uint_as_float(r[4 * q + 1]), __uint_as_float(r[4 * q + 2]),
                                         __uint_as_float(r[4 * q + 3]));
                }
                mbar_arrive_cluster(mapa_shared(recv_full, partner));
                ok2 = mbar_wait_cluster(recv_full, 0, abort_flag);
                if (!__all_sync(0xffffffffu, ok2)) break;
            }
            bool tile_aborted = false;
#pragma unroll 1
            for (int c = c_first; c < c_hi; c += 2 * kCW) {
                const int nc = n0 + c;
                if (c != c_first) {
                    if (resid_tma && nc < p.N) issue_resid(nc);
                    load_resid(nc);
                }
                const float b_next = c + 2 * kCW < c_hi ? load_bias(nc + 2 * kCW) : 0.0f;
                float v[kCW];
                {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + c, r);
                    tmem_ld_wait(r);
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
                }
                if constexpr (SPLIT2) {
                    // partial_0 + partial_1 (a single add: the same bits in either order)
#pragma unroll
                    for (int q = 0; q < kCW / 4; ++q) {
                        const float4 f = *reinterpret_cast<const float4*>(smem + L::kOffA + recv_pos(c - c_lo + 4 * q));
                        v[4 * q] += f.x;
                        v[4 * q + 1] += f.y;
                        v[4 * q + 2] += f.z;
                        v[4 * q + 3] += f.w;
                    }
                }
                if (nc < p.N) {
                    const bool full = nc + kCW <= p.N;
#pragma unroll
                    for (int j = 0; j < kCW; ++j) v[j] += __shfl_sync(0xffffffffu, b_cur, j);
                    if (p.act == 1) {
#pragma unroll
                        for (int j = 0; j < kCW; j += 2) gelu_fast_pair(v[j], v[j + 1]);
                    }
                    if (p.resid_mode == kMaskRows && !valid) {
#pragma unroll
                        for (int j = 0; j < kCW; ++j) v[j] = 0.0f;
                    }
                    if (resid_tma) {
                        // the block's wait is warp-wide (rows past M included)
                        const bool okr = mbar_wait(rbar, r_waited & 1u, abort_flag);
                        if (!__all_sync(0xffffffffu, okr)) {
                            tile_aborted = true;
                            break;
                        }
                        ++r_waited;
                        const bool keep_sub = valid || p.resid_mode == kResidAdd;
                        const bool keep_all = valid || p.resid_mode != kResidAddMaskAll;
                        const uint8_t* rrow = stage_ptr + lane * 128;
#pragma unroll
                        for (int j = 0; j < kCW; j += 4) {
                            const float4 rq = *reinterpret_cast<const float4*>(rrow + (((j >> 2) ^ (lane & 7)) << 4));
                            v[j] = keep_all ? rq.x + (keep_sub ? v[j] : 0.0f) : 0.0f;
                            v[j + 1] = keep_all ? rq.y + (keep_sub ? v[j + 1] : 0.0f) : 0.0f;
                            v[j + 2] = keep_all ? rq.z + (keep_sub ? v[j + 2] : 0.0f) : 0.0f;
                            v[j + 3] = keep_all ? rq.w + (keep_sub ? v[j + 3] : 0.0f) : 0.0f;
                        }
                    } else if (has_resid && row_ok) {
                        const bool keep_sub = valid || p.resid_mode == kResidAdd;
                        const bool keep_all = valid || p.resid_mode != kResidAddMaskAll;
                        if (full) {
#pragma unroll
                            for (int j = 0; j < kCW; j += 4) {
                                v[j] = keep_all ? rr[j / 4].x + (keep_sub ? v[j] : 0.0f) : 0.0f;
                                v[j + 1] = keep_all ? rr[j / 4].y + (keep_sub ? v[j + 1] : 0.0f) : 0.0f;
                                v[j + 2] = keep_all ? rr[j / 4].z + (keep_sub ? v[j + 2] : 0.0f) : 0.0f;
                                v[j + 3] = keep_all ? rr[j / 4].w + (keep_sub ? v[j + 3] : 0.0f) : 0.0f;
                            }
                        } else {
                            const float* rp = p.resid + static_cast<int64_t>(row) * p.ldr + nc;
#pragma unroll
                            for (int j = 0; j < kCW; ++j)
                                if (nc + j < p.N) v[j] = keep_all ? rp[j] + (keep_sub ? v[j] : 0.0f) : 0.0f;
                        }
                    }
                }
                // Chunks past N (the unused columns of a partial tile) stage and
                // store nothing. fp16 chunks alternate between the two halves of
                // the buffer, so before writing a half wait until the store that
                // last read it is done: it is at most the one before the newest.
                if (nc < p.N) {
                    // with the lo half the chunk takes both halves of the buffer
                    const bool lo_out = OUT_F16 && p.out_lo != 0;
                    const uint32_t sb = (OUT_F16 && !lo_out) ? (nstore & 1u) * 2048u : 0u;
                    if (lane == 0) {
                        if (OUT_F16 && !lo_out) bulk_wait_read<1>();
                        else bulk_wait_read<0>();
                    }
                    __syncwarp();
                    uint8_t* srow = stage_ptr + sb + lane * kRowB;
                    if constexpr (OUT_F16) {
                        // 64 B rows, 64B swizzle: granule q of row r at q ^ ((r >> 1) & 3).
                        // The lo half is computed only when its plane is stored
                        // (a warp-uniform branch outside the loop).
                        if (lo_out) {
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
                                               pack_half2(v[8 * q + 4], v[8 * q + 5]),
                                               pack_half2(v[8 * q + 6], v[8 * q + 7]));
                        }
                    } else {
                        // 128 B rows, 128B swizzle: granule q of row r at q ^ (r & 7)
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            *reinterpret_cast<uint4*>(srow + ((q ^ (lane & 7)) << 4)) =
                                make_uint4(__float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]),
                                           __float_as_uint(v[4 * q + 2]), __float_as_uint(v[4 * q + 3]));
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(omap, stage_addr + sb, nc, orow + quarter * 32);
                        if (OUT_F16 && lo_out) tma_store_2d(&po.map[0], stage_addr + 2048, nc, orow + quarter * 32);
                        bulk_commit();
                    }
                    ++nstore;
                }
                b_cur = b_next;
            }
            if (tile_aborted) break;
            tc_fence_before();
            if constexpr (PAIR) {
                // the leader's MMA may refill this CTA's TMEM rows
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(mapa_shared(bars.acce(acc), 0));
            } else {
                mbar_arrive(bars.acce(acc));
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        // a residual block still in flight after an abort lands before exit
        if (lane == 0 && r_issued != r_waited) mbar_wait_drain(rbar, r_waited & 1u);
        if (lane == 0) bulk_wait_all();
    }

    // ------------------------------------------------------------ teardown --
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if constexpr (SPLIT2 || PAIR) {
        // neither CTA of the pair exits while the other may still write into it
        if (threadIdx.x == 0) {
            mbar_arrive_cluster(mapa_shared(exit_bar, 0));
            mbar_arrive_cluster(mapa_shared(exit_bar, 1));
            mbar_wait_cluster(exit_bar, 0, nullptr, 4 * kWaitLimitNs);
        }
        __syncthreads();
    }
    if (warp == 1) {
        tc_fence_after();
        if constexpr (PAIR) tmem_dealloc_pair(tmem_base, L::kTmemCols);
        else tmem_dealloc(tmem_base, L::kTmemCols);
    }
}

}  // namespace dotl
