// Host-side launchers for the ops-level kernels (ops.cu) and the tensor-core matmul (gemm_tc.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace qb {

inline int row_bytes_host(int dtype, int cols) { return dtype == DT_Q4_0 ? cols / 2 : cols; }

cudaError_t launch_quantize_q8(const float* x, int n_tok, int n, int8_t* q, float* d, cudaStream_t st);
cudaError_t launch_matvec(const DMat& W, const int8_t* qx, const float* dx, int r0, int r1, float* out, cudaStream_t st);
cudaError_t launch_matmul_simt(const DMat& W, const int8_t* qx, const float* dx, int n, int r0, int r1, float* out, int ldo,
                               cudaStream_t st);
size_t matvec_smem(int dtype, int cols);

}  // namespace qb
