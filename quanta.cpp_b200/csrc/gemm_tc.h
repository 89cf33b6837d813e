// tcgen05 int8 matmul (gemm_tc.cu): TMA tensor maps and the launcher.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace qb {

// Token count from which qnt_matmul's automatic choice takes the tensor cores.
constexpr int kTcMinTokens = 1 << 30;

struct alignas(64) TcMap {
    CUtensorMap m;
};

struct GemmTcArgs {
    int r0, r1;        // weight rows [r0, r1)
    int nb;            // 32-blocks per row
    int n;             // tokens
    const __half* wd;  // weight block scales [rows][nb]
    float* out;        // out[t * ldo + r]
    int ldo;
    unsigned* status;  // device status word (ERR_WAIT_TIMEOUT)
    int n_valid;       // argmax epilogue: rows >= n_valid never win
    void* cand;        // argmax epilogue: Cand [row tiles * 4][n], each 32-row group's best (value, id) per token
};

bool gemm_tc_supported(const DMat& W);
// The kernel reads int8 weight rows: Q8_0 matrices as stored, Q4_0 through an int8 copy of q - 8 (rows x cols
// bytes, tc_weight_copy_bytes; 0 for Q8_0) that unpack_q4_i8 writes once.
size_t tc_weight_copy_bytes(const DMat& W);
cudaError_t unpack_q4_i8(const DMat& W, int8_t* dst, cudaStream_t st);
// The int8 weights as the kernel's TMA source (128B-swizzled 128 x 128-byte tiles): W.q for Q8_0, i8 for Q4_0.
bool make_weight_map(const DMat& W, const int8_t* i8, TcMap* out);
// Quantized activations q [rows_alloc][cols] int8 and their block scales d [rows_alloc][cols / 32] f32, as TMA sources.
struct TcAct {
    TcMap q, d;
};
size_t gemm_tc_smem();
bool make_act_maps(const int8_t* qx, const float* dx, int rows_alloc, int cols, TcAct* out);
cudaError_t launch_matmul_tc(const DMat& W, const TcMap& wmap, const TcAct& act, int n, int r0, int r1, float* out, int ldo,
                             unsigned* status, cudaStream_t st);

// Greedy head: the exact logits of rows [0, W.rows) for n tokens never leave the kernel; each 32-row group's best
// (value desc, id asc) per token goes to cand, and launch_argmax_reduce picks each token's winner (the first maximum
// over rows < n_valid, as std::max_element).  cand holds argmax_parts(W.rows) * n entries.
int argmax_parts(int rows);
cudaError_t launch_matmul_tc_argmax(const DMat& W, const TcMap& wmap, const TcAct& act, int n, int n_valid, void* cand,
                                    unsigned* status, cudaStream_t st);
cudaError_t launch_argmax_reduce(const void* cand, int n_parts, int n, int* ids, float* vals, cudaStream_t st);

}  // namespace qb
