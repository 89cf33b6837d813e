// The q|k|v epilogue of one rotation pair (bias, RoPE, q / K / V stores), shared by the per-layer kernels and the
// tensor-core matmul's q|k|v epilogue.
#pragma once

#include "kernels.cuh"
#include "layer_kernels.h"

namespace qb {

// Fused q|k|v rows are stored pair-interleaved per head: fused row 2i / 2i+1 of head unit u is original row i / i+half,
// units ordered q heads, k heads, v heads.  Applies bias, RoPE to q/k units and stores q (f32) and K/V (f16).
struct PairIn {
    float ba, bb;  // bias of the two rows
    float c, s;    // RoPE cos / sin at (pos, i)
};

__device__ __forceinline__ void pair_bias(const QkvArgs& a, int fused_row, PairIn& p) {
    p.ba = a.bias[fused_row];
    p.bb = a.bias[fused_row + 1];
}
__device__ __forceinline__ void pair_rope(const QkvArgs& a, int fused_row, int pos, PairIn& p) {
    const int hd = a.head_dim, half = hd / 2, u = fused_row / hd, i = (fused_row - u * hd) >> 1;
    p.c = 1.f;
    p.s = 0.f;
    if (u < a.n_heads + a.n_kv) {
        p.c = a.rope_cos[size_t(pos) * half + i];
        p.s = a.rope_sin[size_t(pos) * half + i];
    }
}

__device__ __forceinline__ void qkv_pair_store(const QkvArgs& a, int fused_row, float va, float vb, int pos, const PairIn& p,
                                               float* Qt) {
    const int hd = a.head_dim, half = hd / 2;
    const int u = fused_row / hd, i = (fused_row - u * hd) >> 1;
    va = fadd(va, p.ba);
    vb = fadd(vb, p.bb);
    if (u < a.n_heads + a.n_kv) rope_pair(va, vb, p.c, p.s);
    if (u < a.n_heads) {
        Qt[u * hd + i] = va;
        Qt[u * hd + i + half] = vb;
    } else {
        const bool is_k = u < a.n_heads + a.n_kv;
        const int kvh = is_k ? u - a.n_heads : u - a.n_heads - a.n_kv;
        __half* C = (is_k ? a.kcache : a.vcache) + size_t(pos) * a.kv_dim + kvh * hd;
        C[i] = __float2half_rn(va);
        C[i + half] = __float2half_rn(vb);
    }
}

__device__ __forceinline__ void qkv_pair_out(const QkvArgs& a, int fused_row, float va, float vb, int pos, float* Qt) {
    PairIn p;
    pair_bias(a, fused_row, p);
    pair_rope(a, fused_row, pos, p);
    qkv_pair_store(a, fused_row, va, vb, pos, p, Qt);
}

}  // namespace qb
