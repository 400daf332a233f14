// Attention for the head dims the tcgen05 kernel does not take (a multiple of
// 8 up to 256, other than 32, 64 and 128), on the CUDA cores.
//
// Replaces, for those shapes, the reference's scalar and wmma attention
// kernels (attention_scalar.cuh, attention_wmma.cuh; dispatch
// attention_dispatch.cuh:332-519): the reference's official dashboard shapes 7
// and 11 have head_dim 8 and shape 8 has head_dim 256. Same contract as
// attn_tc_kernel: softmax(q k^T * scale + masks) v per (batch, head), key-mask
// kinds 1 and 2, causal, fully masked query rows written as 0, output layouts
// [B,H,S,hd] and [B,S,H*hd].
//
// Head dims 40 to 256: one warp per query row, the head dims spread over the
// lanes (hd <= 32 HPL),
// fp32 scores through an online softmax (running max, running sum, rescaled
// accumulator; P rounded to fp16 before it multiplies V, as the tensor-core
// kernels do), fp16 output. The block's 16 query rows share every key/value
// tile, staged in shared memory (32 keys at a time, rows zero-padded to
// 32 HPL) with 16-byte loads. Head dims 8, 16 and 24 run attn_rows_kernel
// below, a thread per query row. Not tensor-core kernels: these shapes are
// small (the largest, dashboard shape 8, is 1 GFLOP per layer).

#pragma once

#include "dotl_common.cuh"
#include "layernorm.cuh"

namespace dotl {

constexpr int kGenRows = 16;   // query rows (warps) per block
constexpr int kGenKeys = 32;   // keys per shared-memory tile

struct AttnGenericParams {
    const __half* q;
    const __half* k;
    const __half* v;
    int64_t qs[3], ks[3], vs[3];   // batch, head, sequence strides in elements (head dim stride 1)
    int B, H, S, hd;
    int causal;
    float scale;
    int mask_kind;
    const uint8_t* mask;
    int64_t ms0, ms1, ms2, ms3;
    __half* out;
    int out_layout;
    int64_t out_lo;                // 0, or the element offset of the fp16 pair's lo plane
};

template <int HPL>
__global__ void __launch_bounds__(kGenRows * 32) attn_generic_kernel(const AttnGenericParams p) {
    constexpr int kRow = 32 * HPL;   // staged row length in halves
    __shared__ __align__(16) __half k_s[kGenKeys][kRow];
    __shared__ __align__(16) __half v_s[kGenKeys][kRow];
    pdl_wait();
    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.y / p.H;
    const int h = blockIdx.y - b * p.H;
    const int qi = blockIdx.x * kGenRows + warp;
    const bool q_ok = qi < p.S;

    float q[HPL], o[HPL];
#pragma unroll
    for (int i = 0; i < HPL; ++i) {
        const int d = lane + 32 * i;
        q[i] = (q_ok && d < p.hd) ? __half2float(p.q[b * p.qs[0] + h * p.qs[1] + qi * p.qs[2] + d]) : 0.0f;
        o[i] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    // under the causal rule no row of this block sees keys past its last row
    const int k_end = p.causal ? min(p.S, blockIdx.x * kGenRows + kGenRows) : p.S;
    const int chunks = kRow / 8;     // 16-byte pieces per staged row
    for (int k0 = 0; k0 < k_end; k0 += kGenKeys) {
        __syncthreads();             // the previous tile is no longer read
        for (int idx = threadIdx.x; idx < kGenKeys * chunks; idx += blockDim.x) {
            const int j = idx / chunks;
            const int d = (idx - j * chunks) * 8;
            uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = make_uint4(0u, 0u, 0u, 0u);
            if (k0 + j < k_end && d < p.hd) {
                kv = *reinterpret_cast<const uint4*>(p.k + b * p.ks[0] + h * p.ks[1] + (k0 + j) * p.ks[2] + d);
                vv = *reinterpret_cast<const uint4*>(p.v + b * p.vs[0] + h * p.vs[1] + (k0 + j) * p.vs[2] + d);
            }
            *reinterpret_cast<uint4*>(&k_s[j][d]) = kv;
            *reinterpret_cast<uint4*>(&v_s[j][d]) = vv;
        }
        __syncthreads();
        const int n = min(kGenKeys, k_end - k0);
        for (int j = 0; j < n; ++j) {
            const int kj = k0 + j;
            // the same decision for every lane of the warp (one query row)
            bool allowed = q_ok && (!p.causal || kj <= qi);
            if (allowed && p.mask_kind == 1) allowed = p.mask[b * p.ms0 + kj * p.ms3] != 0;
            else if (allowed && p.mask_kind == 2)
                allowed = p.mask[b * p.ms0 + h * p.ms1 + static_cast<int64_t>(qi) * p.ms2 + kj * p.ms3] != 0;
            if (!allowed) continue;
            float s = 0.0f;
#pragma unroll
            for (int i = 0; i < HPL; ++i) s = fmaf(q[i], __half2float(k_s[j][lane + 32 * i]), s);
            s = warp_sum(s) * p.scale;
            const float m_new = fmaxf(m, s);
            const float corr = __expf(m - m_new);   // 0 on the first allowed key
            const float pj = __expf(s - m_new);
            l = fmaf(l, corr, pj);
            // P meets V as fp16, the row sum takes the unrounded value: the
            // arithmetic of the reference's fp16 kernels and of attn_tc_kernel
            const float ph = __half2float(__float2half_rn(pj));
#pragma unroll
            for (int i = 0; i < HPL; ++i) o[i] = fmaf(o[i], corr, ph * __half2float(v_s[j][lane + 32 * i]));
            m = m_new;
        }
    }
    if (!q_ok) return;
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;   // no allowed key: the row is 0
    const int64_t base = p.out_layout == 1 ? ((static_cast<int64_t>(b) * p.S + qi) * p.H + h) * p.hd
                                           : ((static_cast<int64_t>(b) * p.H + h) * p.S + qi) * p.hd;
#pragma unroll
    for (int i = 0; i < HPL; ++i) {
        const int d = lane + 32 * i;
        if (d < p.hd) {
            const float y = o[i] * inv;
            const __half hi = __float2half_rn(y);
            p.out[base + d] = hi;
            if (p.out_lo != 0) p.out[p.out_lo + base + d] = __float2half_rn(y - __half2float(hi));
        }
    }
}

// Head dims 8, 16 and 24: one THREAD per query row (q and the output row in
// registers), 128 rows of one (batch, head) stream per block. The 32-key K/V
// tiles are staged in shared memory as fp32 and read as broadcasts (every
// thread of the block reads the same key). Per tile a row takes its 32
// scores, their max, one rescale of its running output and sum, and then
// P = exp2(s c - m c) per key: exponentials in the exp2 domain as in
// attn_tc_kernel, P rounded to fp16 before it multiplies V, the row sum over
// the unrounded P. One warp per row (attn_generic_kernel) would spend 32
// lanes on 8-24 products and repeat each exponential 32 times.
constexpr int kRowsBlock = 128;   // query rows (threads) per block
constexpr int kRowsKeys = 32;     // keys per staged tile

template <int HD>
__global__ void __launch_bounds__(kRowsBlock) attn_rows_kernel(const AttnGenericParams p) {
    static_assert(HD % 8 == 0 && HD <= 24, "attn_rows_kernel: head dims 8, 16, 24");
    __shared__ __align__(16) float k_s[kRowsKeys][HD];
    __shared__ __align__(16) float v_s[kRowsKeys][HD];
    __shared__ uint8_t key_ok[kRowsKeys];
    pdl_wait();
    pdl_launch_dependents();
    const int b = blockIdx.y / p.H;
    const int h = blockIdx.y - b * p.H;
    const int qi = blockIdx.x * kRowsBlock + threadIdx.x;
    const bool q_ok = qi < p.S;
    const float c = p.scale * 1.4426950408889634f;   // scores into the exp2 domain

    float q[HD], o[HD];
    {
        const __half* qrow = p.q + b * p.qs[0] + h * p.qs[1] + static_cast<int64_t>(q_ok ? qi : 0) * p.qs[2];
#pragma unroll
        for (int d = 0; d < HD; d += 8) {
            uint4 raw = q_ok ? *reinterpret_cast<const uint4*>(qrow + d) : make_uint4(0u, 0u, 0u, 0u);
            const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(h2[i]);
                q[d + 2 * i] = f.x;
                q[d + 2 * i + 1] = f.y;
            }
        }
#pragma unroll
        for (int d = 0; d < HD; ++d) o[d] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;   // m in the exp2 domain (max of s c)
    // under the causal rule no row of this block sees keys past its last row
    const int k_end = p.causal ? min(p.S, blockIdx.x * kRowsBlock + kRowsBlock) : p.S;
    constexpr int kChunks = HD / 8;   // 16-byte pieces per key row
    for (int k0 = 0; k0 < k_end; k0 += kRowsKeys) {
        __syncthreads();   // the previous tile is no longer read
        for (int idx = threadIdx.x; idx < kRowsKeys * kChunks; idx += kRowsBlock) {
            const int j = idx / kChunks;
            const int d = (idx - j * kChunks) * 8;
            uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = make_uint4(0u, 0u, 0u, 0u);
            if (k0 + j < k_end) {
                kv = *reinterpret_cast<const uint4*>(p.k + b * p.ks[0] + h * p.ks[1] +
                                                     static_cast<int64_t>(k0 + j) * p.ks[2] + d);
                vv = *reinterpret_cast<const uint4*>(p.v + b * p.vs[0] + h * p.vs[1] +
                                                     static_cast<int64_t>(k0 + j) * p.vs[2] + d);
            }
            const __half2* k2 = reinterpret_cast<const __half2*>(&kv);
            const __half2* v2 = reinterpret_cast<const __half2*>(&vv);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 kf = __half22float2(k2[i]);
                const float2 vf = __half22float2(v2[i]);
                k_s[j][d + 2 * i] = kf.x;
                k_s[j][d + 2 * i + 1] = kf.y;
                v_s[j][d + 2 * i] = vf.x;
                v_s[j][d + 2 * i + 1] = vf.y;
            }
        }
        if (threadIdx.x < kRowsKeys) {
            const int kj = k0 + threadIdx.x;
            bool ok = kj < k_end;
            if (ok && p.mask_kind == 1) ok = p.mask[b * p.ms0 + static_cast<int64_t>(kj) * p.ms3] != 0;
            key_ok[threadIdx.x] = ok ? 1 : 0;
        }
        __syncthreads();
        float s[kRowsKeys];
        float mt = -INFINITY;
#pragma unroll
        for (int j = 0; j < kRowsKeys; ++j) {
            const int kj = k0 + j;
            bool allowed = q_ok && key_ok[j] && (!p.causal || kj <= qi);
            if (allowed && p.mask_kind == 2)
                allowed = p.mask[b * p.ms0 + h * p.ms1 + static_cast<int64_t>(qi) * p.ms2 +
                                 static_cast<int64_t>(kj) * p.ms3] != 0;
            float acc = 0.0f;
#pragma unroll
            for (int d = 0; d < HD; d += 4) {
                const float4 kk = *reinterpret_cast<const float4*>(&k_s[j][d]);
                acc = fmaf(q[d], kk.x, acc);
                acc = fmaf(q[d + 1], kk.y, acc);
                acc = fmaf(q[d + 2], kk.z, acc);
                acc = fmaf(q[d + 3], kk.w, acc);
            }
            s[j] = allowed ? acc * c : -INFINITY;
            mt = fmaxf(mt, s[j]);
        }
        if (mt == -INFINITY) continue;   // nothing allowed in this tile for this row
        const float m_new = fmaxf(m, mt);
        const float corr = fast_exp2(m - m_new);   // 0 while nothing was accumulated
        l *= corr;
#pragma unroll
        for (int d = 0; d < HD; ++d) o[d] *= corr;
        m = m_new;
#pragma unroll
        for (int j = 0; j < kRowsKeys; ++j) {
            const float pj = fast_exp2(s[j] - m_new);   // -inf -> 0
            l += pj;
            const float ph = __half2float(__float2half_rn(pj));
#pragma unroll
            for (int d = 0; d < HD; d += 4) {
                const float4 vv = *reinterpret_cast<const float4*>(&v_s[j][d]);
                o[d] = fmaf(ph, vv.x, o[d]);
                o[d + 1] = fmaf(ph, vv.y, o[d + 1]);
                o[d + 2] = fmaf(ph, vv.z, o[d + 2]);
                o[d + 3] = fmaf(ph, vv.w, o[d + 3]);
            }
        }
    }
    if (!q_ok) return;
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;   // no allowed key: the row is 0
    const int64_t base = p.out_layout == 1 ? ((static_cast<int64_t>(b) * p.S + qi) * p.H + h) * HD
                                           : ((static_cast<int64_t>(b) * p.H + h) * p.S + qi) * HD;
#pragma unroll
    for (int d = 0; d < HD; d += 8) {
        uint4 hi, lo;
        uint32_t* hw = reinterpret_cast<uint32_t*>(&hi);
        uint32_t* lw = reinterpret_cast<uint32_t*>(&lo);
        if (p.out_lo != 0) {
#pragma unroll
            for (int i = 0; i < 4; ++i) split_half2(o[d + 2 * i] * inv, o[d + 2 * i + 1] * inv, hw[i], lw[i]);
            *reinterpret_cast<uint4*>(p.out + p.out_lo + base + d) = lo;
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) hw[i] = pack_half2(o[d + 2 * i] * inv, o[d + 2 * i + 1] * inv);
        }
        *reinterpret_cast<uint4*>(p.out + base + d) = hi;
    }
}

}  // namespace dotl
