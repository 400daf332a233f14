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
// One warp per query row, the head dims spread over the lanes (hd <= 32 HPL),
// fp32 scores through an online softmax (running max, running sum, rescaled
// accumulator; P rounded to fp16 before it multiplies V, as the tensor-core
// kernels do), fp16 output. The block's 16 query rows share every key/value
// tile, staged in shared memory (32 keys at a time, rows zero-padded to
// 32 HPL) with 16-byte loads. Not a tensor-core kernel: these shapes are small
// (the largest, dashboard shape 8, is 1 GFLOP per layer).

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

}  // namespace dotl
