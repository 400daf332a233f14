// All-reduce of per-rank partial sums + bias + residual + LayerNorm in one
// kernel, over peer memory (NVLink / NVSwitch), for the tensor-parallel layer.
//
// Replaces, on each rank, the sequence
//     all_reduce(part)            (NCCL, sum over the ranks)
//     x_new = x + part            }
//     normed = LN(x_new)          } fused_add_layernorm (add_layernorm.cuh:663-672)
// that follows each row-parallel GEMM of the layer (the reference's single-GPU
// pair is optimized/layers.py:241-243 and :258-261; it has no tensor
// parallelism, so the reduction itself has no counterpart there).
//
// Every rank's partial-sum buffer and signal area are mapped into every other
// rank's address space (CUDA IPC). Plain loads and stores only (one address each),
// no NVLS. Per call, on every rank, with the same grid on every rank:
//   1. start barrier: CTA b tells CTA b of every peer that it has started, and
//      waits until every peer's CTA b has (so every peer's partial sums, which
//      its previous kernel wrote, are complete and visible);
//   2. rows: sum = part_0 + part_1 + ... + part_{P-1} in rank order (the same
//      bits on every rank), then + bias, x_new = x + (valid ? sum : 0), and
//      normed = LN(x_new) * w + b (0 on rows that normed_row_valid marks);
//      one-shot mode: every rank does every row and writes only locally;
//      push mode: rank r does rows [r C, (r+1) C) and stores x_new / normed
//      into every rank's output buffers; with parts_local, the row-parallel
//      GEMMs have already scattered their tiles to the row owners
//      (dotl_linear_peer), so rank r's partial sums of its rows are read
//      from slots in its own memory and only the results cross NVLink;
//   3. end barrier: the same handshake again, after which no peer still reads
//      this rank's partial sums or still writes into its outputs.
// Flags carry a per-CTA call counter (kept in the rank's own signal area), so
// the same launch can be replayed from a CUDA graph. Every wait is bounded: on
// timeout the CTA or-s kDevErrPeerTimeout into the device error word and
// returns; after that the ranks' counters disagree and the peer group must be
// rebuilt.
//
// Roofline: NVLink-bound. One-shot at P ranks reads (P-1) remote rows per row;
// push mode reads (P-1)/P remote and writes (P-1)/P of x_new + normed remotely.

#pragma once

#include "dotl_common.cuh"
#include "layernorm.cuh"

namespace dotl {

constexpr int kPeerMax = 8;
constexpr int kPeerWarps = 8;
constexpr int kPeerBlocksPerSm = 2;   // every CTA of the grid resident at once
constexpr unsigned int kDevErrPeerTimeout = 4u;

// Signal area of one rank, in 32-bit words, for a grid of G CTAs:
//   [0, G)                      call counter of CTA b (only this rank's CTA b touches it)
//   [G + b*kPeerMax + src]      start flag written by rank src's CTA b
//   [G + G*kPeerMax + ...]      end flag, same layout
__host__ __device__ constexpr int64_t peer_signal_words(int blocks) {
    return static_cast<int64_t>(blocks) * (1 + 2 * kPeerMax);
}

struct PeerLnParams {
    const float* part[kPeerMax];   // rank i's partial sums [rows, D]
    unsigned int* signal[kPeerMax];
    float* x_new[kPeerMax];        // where x_new goes on rank i (push), [rank] only otherwise
    void* normed[kPeerMax];
    const float* x;                // residual, this rank's copy [rows, D]
    const float* bias;             // [D] or null
    const uint8_t* sum_row_valid;  // rows with 0 keep x (x_new = x); null = all valid
    const float* ln_w;
    const float* ln_b;
    const uint8_t* normed_row_valid;
    int64_t rows;
    int D;
    float eps;
    int world;
    int rank;
    int push;
    int parts_local;               // part[i]: rows [lo, hi) of rank i's partial sums, in this rank's memory
    unsigned long long timeout_ns;
    unsigned int* status;          // optional caller word (e.g. host-mapped) that a timeout also sets
};

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One thread per CTA: publish `val` into slot [b][rank] of every peer's area
// at word offset `off`, then wait for every peer's slot [b][peer] here.
__device__ __forceinline__ bool peer_handshake(const PeerLnParams& p, int64_t off, unsigned int val) {
    const int b = blockIdx.x;
    for (int src = 0; src < p.world; ++src)
        if (src != p.rank) st_release_sys(p.signal[src] + off + b * kPeerMax + p.rank, val);
    const unsigned int* mine = p.signal[p.rank] + off + b * kPeerMax;
    const unsigned long long t0 = global_ns();
    for (int src = 0; src < p.world; ++src) {
        if (src == p.rank) continue;
        while (static_cast<int>(ld_acquire_sys(mine + src) - val) < 0) {
            if (global_ns() - t0 > p.timeout_ns) {
                atomicOr(&g_dotl_dev_error, kDevErrPeerTimeout);
                if (p.status != nullptr) {
                    // a plain store: the word may be host memory, where
                    // device atomics are not guaranteed
                    *reinterpret_cast<volatile unsigned int*>(p.status) = kDevErrPeerTimeout;
                    __threadfence_system();
                }
                return false;
            }
        }
    }
    return true;
}

// EPL = elements per lane (D <= 32 * EPL, D % 4 == 0): lane owns the float4
// chunks at column (i * 32 + lane) * 4 that fall below D.
template <int EPL, typename NormT>
__global__ void __launch_bounds__(kPeerWarps * 32, kPeerBlocksPerSm) allreduce_ln_kernel(const PeerLnParams p) {
    pdl_wait();
    __shared__ int s_ok;
    const int G = gridDim.x;
    unsigned int* my_sig = p.signal[p.rank];
    unsigned int val = 0;
    if (threadIdx.x == 0) {
        val = my_sig[blockIdx.x] + 1u;
        my_sig[blockIdx.x] = val;
        s_ok = peer_handshake(p, G, val) ? 1 : 0;
    }
    __syncthreads();
    if (!s_ok) return;
    pdl_launch_dependents();

    const int lane = threadIdx.x & 31;
    const int D = p.D;
    int64_t lo = 0, hi = p.rows;
    if (p.push) {
        const int64_t chunk = (p.rows + p.world - 1) / p.world;
        lo = min(p.rows, chunk * p.rank);
        hi = min(p.rows, lo + chunk);
    }
    const int64_t warp0 = static_cast<int64_t>(blockIdx.x) * kPeerWarps + (threadIdx.x >> 5);
    const int64_t nwarps = static_cast<int64_t>(G) * kPeerWarps;
    const float inv_d = 1.0f / static_cast<float>(D);
    for (int64_t row = lo + warp0; row < hi; row += nwarps) {
        const int64_t base = row * D;
        // rank src's partial sums of this row: its buffer over NVLink, or (when
        // the GEMMs scattered their tiles to the row owners) this rank's slot
        const int64_t pbase = p.parts_local ? (row - lo) * D : base;
        float4 s[EPL / 4];
        // partial sums in rank order (L2-only loads: peer data is never
        // cached in L1)
#pragma unroll
        for (int i = 0; i < EPL / 4; ++i) {
            const int c = (i * 32 + lane) * 4;
            s[i] = c < D ? __ldcg(reinterpret_cast<const float4*>(p.part[0] + pbase + c))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        for (int src = 1; src < p.world; ++src) {
#pragma unroll
            for (int i = 0; i < EPL / 4; ++i) {
                const int c = (i * 32 + lane) * 4;
                if (c < D) {
                    const float4 t = __ldcg(reinterpret_cast<const float4*>(p.part[src] + pbase + c));
                    s[i].x += t.x; s[i].y += t.y; s[i].z += t.z; s[i].w += t.w;
                }
            }
        }
        const bool add = p.sum_row_valid == nullptr || p.sum_row_valid[row] != 0;
        float v[EPL];
#pragma unroll
        for (int i = 0; i < EPL / 4; ++i) {
            const int c = (i * 32 + lane) * 4;
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
            if (c < D) {
                a = *reinterpret_cast<const float4*>(p.x + base + c);
                if (add) {
                    float4 t = s[i];
                    if (p.bias != nullptr) {
                        const float4 bb = *reinterpret_cast<const float4*>(p.bias + c);
                        t.x += bb.x; t.y += bb.y; t.z += bb.z; t.w += bb.w;
                    }
                    a.x += t.x; a.y += t.y; a.z += t.z; a.w += t.w;
                }
            }
            v[4 * i] = a.x; v[4 * i + 1] = a.y; v[4 * i + 2] = a.z; v[4 * i + 3] = a.w;
        }
        // two-pass statistics over the registers, as the LayerNorm kernel
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < EPL; ++i) sum += v[i];
        const float mean = warp_sum(sum) * inv_d;
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < EPL / 4; ++i) {
            if ((i * 32 + lane) * 4 < D) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float c = v[4 * i + j] - mean;
                    ss += c * c;
                }
            }
        }
        const float rstd = rsqrtf(warp_sum(ss) * inv_d + p.eps);
        const bool keep = p.normed_row_valid == nullptr || p.normed_row_valid[row] != 0;
        const int d0 = p.push ? 0 : p.rank;
        const int d1 = p.push ? p.world : p.rank + 1;
#pragma unroll
        for (int i = 0; i < EPL / 4; ++i) {
            const int c = (i * 32 + lane) * 4;
            if (c >= D) continue;
            const float4 ww = *reinterpret_cast<const float4*>(p.ln_w + c);
            const float4 bb = *reinterpret_cast<const float4*>(p.ln_b + c);
            float o0 = (v[4 * i] - mean) * rstd * ww.x + bb.x;
            float o1 = (v[4 * i + 1] - mean) * rstd * ww.y + bb.y;
            float o2 = (v[4 * i + 2] - mean) * rstd * ww.z + bb.z;
            float o3 = (v[4 * i + 3] - mean) * rstd * ww.w + bb.w;
            if (!keep) o0 = o1 = o2 = o3 = 0.0f;
            const float4 xn = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            for (int dst = d0; dst < d1; ++dst) {
                if (p.x_new[dst] != nullptr) *reinterpret_cast<float4*>(p.x_new[dst] + base + c) = xn;
                if constexpr (sizeof(NormT) == 4) {
                    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.normed[dst]) + base + c) =
                        make_float4(o0, o1, o2, o3);
                } else {
                    uint2 h;
                    h.x = pack_half2(o0, o1);
                    h.y = pack_half2(o2, o3);
                    *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(p.normed[dst]) + base + c) = h;
                }
            }
        }
    }

    // End barrier: this CTA's stores (remote ones included) are ordered before
    // its flag; afterwards every peer's CTA b has finished reading and writing.
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) peer_handshake(p, G + static_cast<int64_t>(G) * kPeerMax, val);
}

}  // namespace dotl
