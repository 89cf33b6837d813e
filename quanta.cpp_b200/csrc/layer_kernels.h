// Launchers for the per-layer kernels (layer_kernels.cu).
#pragma once

#include <algorithm>

#include "common.cuh"
#include "exp_table.h"
#include "ops.h"

namespace qb {

struct QkvArgs {
    DMat W;                  // fused q|k|v, pair-interleaved rows
    const float* bias;       // fused, same row order
    const float* rope_cos;   // [ctx][head_dim/2]
    const float* rope_sin;
    __half* kcache;          // this layer's [ctx][kv_dim]
    __half* vcache;
    int n_heads, n_kv, head_dim, kv_dim;
};

// o_proj folded into the decode attention: T [W.rows][W.cols / 32] receives each row's block terms
// (float(s_b) * dw_b) * dx_b; the gate|up kernel adds them in block order onto the residual.
struct OArgs {
    DMat W;
    float* T = nullptr;
};

struct AttnArgs {
    const __half* kcache;    // this layer's [ctx][kv_dim]
    const __half* vcache;
    int n_heads, n_kv, head_dim, kv_dim;
    float scale;             // 1/sqrt(head_dim)
    int max_chunks;          // ceil(ctx / 64): the KV cache holds max_chunks * 64 >= ctx positions of room
    ExpTab exptab;           // host libm expf exceptions (exp_table.h)
    float neg_zero = -0.0f;  // -0.0 as a runtime value: the addend of the exact f32x2 products (common.cuh)
    int8_t* xq = nullptr;    // decode (one token): the output also quantized (quantize_q8) for the next matvec,
    float* dx = nullptr;     //   xq[n_heads * head_dim] int8 and dx[n_heads * head_dim / 32] block scales
};

// Multi-token launches over tokens of different sequences: token t sits at position pos[t] and its sequence's KV cache
// starts off[t] elements after the layer's cache pointer.  pos == nullptr: one sequence, token t at pos_dev[0] + t.
struct TokMap {
    const int* pos = nullptr;
    const long long* off = nullptr;
};

struct SlicePlan {
    int rows_per_cta = 0, grid = 0, u = 0;
    unsigned magic = 0;
    size_t smem = 0;
};

SlicePlan plan_rows(int dtype, int rows, int cols, int target_ctas, int row_multiple);

cudaError_t launch_embed(const DMat& E, const int* tokens, int n_tok, float* X, unsigned* status, cudaStream_t st, bool pdl);
cudaError_t launch_qkv_dec(const QkvArgs& a, const SlicePlan& p, const float* X, const float* norm_w, float eps,
                           const int* pos_dev, float* Q, cudaStream_t st, bool pdl);
cudaError_t launch_resid_dec(const DMat& W, const SlicePlan& p, const float* xin, const int8_t* qin, const float* din,
                             float* X, cudaStream_t st, bool pdl, const float* Xres = nullptr);
cudaError_t launch_gateup_dec(const DMat& W, const SlicePlan& p, const float* X, const float* norm_w, float eps,
                              int8_t* HQ, float* HD, const ExpTab& tab, cudaStream_t st, bool pdl,
                              const float* T = nullptr, int nbo = 0, float* X2 = nullptr, float* Hf = nullptr);
// residual-terms form of gate|up (T != nullptr): clusters of 8 CTAs first form X2 = X + (o_proj terms T summed in block
// order), the o_proj residual, then norm it; launched only where gateup_rt_supported.
bool gateup_rt_supported(const DMat& W, const SlicePlan& p, int nbo);
cudaError_t launch_attn(const AttnArgs& a, const float* Q, const int* pos_dev, int n_tok, float* out, cudaStream_t st, bool pdl);
// n_tok > 1 consecutive tokens whose positions stay below pos_bound (known on the host): one CTA per (kv head, token).
// Decode (one token): the layer's q|k|v matvec (with its rmsnorm prologue, bias, RoPE and K/V store) fused into the
// attention; cudaErrorNotSupported for shapes the fused form does not cover (then k_qkv_dec + launch_attn).
// With `o` (o_proj Q8_0, [dim][n_heads * 64]), the kernel also forms the o_proj block terms of its head into o->T
// (o_proj then runs inside launch_gateup_dec's residual-terms form).  qkv_attn_supported: whether the shapes allow it.
bool qkv_attn_supported(const QkvArgs& qa, const AttnArgs& a, const DMat* o);
cudaError_t launch_qkv_attn(const QkvArgs& qa, const AttnArgs& a, const float* X, const float* norm_w, float eps,
                            const int* pos_dev, float* Qout, float* out, cudaStream_t st, bool pdl, const OArgs* o = nullptr);
// The attention output quantized for o_proj (quantize_q8 of each token's n_heads * 64 outputs): xq [t][dim], dx [t][dim / 32]
// and, when dxt is set, dxt[b * ldt + t].
struct QuantOut {
    int8_t* xq = nullptr;
    float* dx = nullptr;
    float* dxt = nullptr;
    int ldt = 0;
};
// With qo, the outputs go to qo (quantized in the kernel, the same bits as launch_norm_quant_rows without a norm) instead
// of out; out is then scratch for the long-context fallback.
cudaError_t launch_attn_prefill(const AttnArgs& a, const float* Q, const int* pos_dev, int n_tok, int pos_bound, float* out,
                                cudaStream_t st, bool pdl, TokMap tm = TokMap{}, const QuantOut* qo = nullptr);
// DXT (optional): the block scales also block-major, DXT[b * ldt + t] (the tensor-core matmul's layout).
cudaError_t launch_norm_quant_rows(const float* X, const float* norm_w, int n_tok, int dim, float eps, int8_t* XQ, float* DX,
                                   float* DXT, int ldt, cudaStream_t st, bool pdl);
cudaError_t launch_qkv_epilogue(const QkvArgs& a, const float* R, int n_tok, const int* pos_dev, float* Q, cudaStream_t st,
                                bool pdl, TokMap tm = TokMap{});
cudaError_t launch_residual(float* X, const float* R, long long n, cudaStream_t st, bool pdl);
cudaError_t launch_swiglu_quant(const float* R, int n_tok, int ffn, int8_t* HQ, float* HD, float* HDT, int ldt, const ExpTab& tab,
                                cudaStream_t st, bool pdl, float* Hf = nullptr);
// FLAG_HADAMARD_DOWN: the block-256 Walsh-Hadamard transform of Hf[n_tok][ffn] (ffn % 256 == 0), then its quantization
// into HQ / HD (and HDT[b * ldt + t] when given) for the down projection.
cudaError_t launch_fwht_quant(const float* Hf, int n_tok, int ffn, int8_t* HQ, float* HD, float* HDT, int ldt, cudaStream_t st,
                              bool pdl);

}  // namespace qb
