// tcgen05 int8 matmul (gemm_tc.cu): TMA tensor maps and the launcher.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "exp_table.h"
#include "layer_kernels.h"

namespace qb {

// Token count from which qnt_matmul's automatic choice takes the tensor cores.
constexpr int kTcMinTokens = 1 << 30;

// A weight matrix as the kernel's TMA sources: m its int8 rows (two 128B-swizzled 128 x 128-byte tiles per load),
// s its block scales in K-step-major order (4 f16 per row and K-step).
struct alignas(64) TcMap {
    CUtensorMap m, s;
};

struct GemmTcArgs {
    int r0, r1;        // weight rows [r0, r1)
    int nb;            // 32-blocks per row
    int n;             // tokens
    float* out;        // out[t * ldo + r]
    int ldo;
    unsigned* status;  // device status word (ERR_WAIT_TIMEOUT)
    int n_valid;       // argmax epilogue: rows >= n_valid never win
    void* cand;        // argmax epilogue: Cand [row tiles * 4][n], each 32-row group's best (value, id) per token
    unsigned nzero;    // 0x80000000 (-0.0f): the addend that turns an fma into the exact product (see the kernel)
    int8_t* hq;        // SwiGLU epilogue: h quantized, hq [n][ffn], hd [n][ffn / 32], hdt[b * ldt + t] (optional)
    float* hd;
    float* hdt;
    int ldt;
    ExpTab tab;
    QkvArgs qa;            // q|k|v epilogue: bias, RoPE, the caches (this layer's), q out [n][n_heads * head_dim]
    TokMap tm;             // per-token positions / cache offsets (batched sequences), else position *pos_dev + t
    const int* pos_dev;
    float* qout;
};

bool gemm_tc_supported(const DMat& W);
// Device bytes the tensor-core path keeps beside W: a K-step-major copy of its block scales and, for Q4_0, an int8
// copy of q - 8 (the kernel reads int8 rows only; Q8_0 rows are read where they are).
size_t tc_weight_bytes(const DMat& W);
// Writes those copies into buf (tc_weight_bytes(W) bytes, 256-byte aligned) on st and encodes the TMA sources.
cudaError_t tc_prepare_weights(const DMat& W, void* buf, TcMap* out, cudaStream_t st);
// Quantized activations as TMA sources: q [rows][cols] int8 and the block scales in block-major order,
// dxt[b * ldt + t] = scale of block b of token t (ldt >= rows, a multiple of 32); boxes of 32 tokens (q, d) and of 16
// (q16, d16) for the two token-tile widths.
struct TcActMap {
    CUtensorMap m;
};
struct TcAct {
    TcActMap q, d, q16, d16;
};
bool make_act_maps(const int8_t* qx, const float* dxt, int rows, int ldt, int cols, TcAct* out);
// dxt[b * ldt + t] = dx[t * nb + b] for t < n (the block-major scales from the token-major ones).
cudaError_t launch_transpose_scales(const float* dx, int n, int nb, float* dxt, int ldt, cudaStream_t st);
// residual: out[t * ldo + r] = out[t * ldo + r] + row value (the residual add fused into the store).  pdl: launched as a
// programmatic dependent of the previous kernel on st (the weight loads start before that kernel ends).
cudaError_t launch_matmul_tc(const DMat& W, const TcMap& wmap, const TcAct& act, int n, int r0, int r1, float* out, int ldo,
                             unsigned* status, cudaStream_t st, bool pdl = false, bool residual = false);

// gate|up (rows interleaved per 32-row block, W.rows = 2 ffn, a multiple of 128) with the SwiGLU and its quantize_q8 in
// the epilogue: the same bits as the matmul followed by launch_swiglu_quant, without the f32 rows leaving the kernel.
cudaError_t launch_matmul_tc_swiglu(const DMat& W, const TcMap& wmap, const TcAct& act, int n, int8_t* hq, float* hd,
                                    float* hdt, int ldt, const ExpTab& tab, unsigned* status, cudaStream_t st, bool pdl);

// Fused q|k|v (pair-interleaved rows) with the bias, RoPE and the q / K / V stores in the epilogue: the same bits as
// the matmul followed by launch_qkv_epilogue.
cudaError_t launch_matmul_tc_qkv(const DMat& W, const TcMap& wmap, const TcAct& act, int n, const QkvArgs& qa,
                                 const int* pos_dev, TokMap tm, float* qout, unsigned* status, cudaStream_t st, bool pdl);

// Greedy head: the exact logits of rows [0, W.rows) for n tokens never leave the kernel; each 32-row group's best
// (value desc, id asc) per token goes to cand, and launch_argmax_reduce picks each token's winner (the first maximum
// over rows < n_valid, as std::max_element).  cand holds argmax_parts(W.rows) * n entries.
int argmax_parts(int rows);
cudaError_t launch_matmul_tc_argmax(const DMat& W, const TcMap& wmap, const TcAct& act, int n, int n_valid, void* cand,
                                    unsigned* status, cudaStream_t st, bool pdl = false);
cudaError_t launch_argmax_reduce(const void* cand, int n_parts, int n, int* ids, float* vals, cudaStream_t st);

// Dense int8 tensor-core peak of this GPU: every SM issues 4 * iters back-to-back tcgen05.mma.kind::i8 of
// M = 128, N = 256, K = 32 from shared memory; *tops = 2 M N K * MMAs / the slowest SM's time (synchronous).
cudaError_t bench_mma_i8(int iters, double* tops, unsigned* status);

// One bounded mbarrier wait that nothing completes, with `limit` tries (each may suspend up to 20 us): sets
// ERR_WAIT_TIMEOUT in *status and returns -- the error path of the matmul's waits, exercised on its own.
cudaError_t launch_wait_probe(unsigned limit, unsigned* status, cudaStream_t st);

}  // namespace qb
