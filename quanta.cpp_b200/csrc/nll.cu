// Negative log-likelihood of one target token under the full-vocabulary softmax of the logits (the `ppl` command of
// tools/cli/main.cpp:261-282): nll += (log(sum_i exp(double(l_i - max))) + max) - l_target over ids < n_valid, with
// the reference's precisions: the difference l_i - max in f32, the exponentials and their sum in f64.  The f64 sum is a
// tree here (the reference adds in id order); at f64 the two differ far below the perplexity's printed digits.
#include "head_kernels.h"
#include "kernels.cuh"

namespace qb {

namespace {

constexpr int kNllThreads = 1024;

__global__ void __launch_bounds__(kNllThreads) k_token_nll(const float* __restrict__ logits, int n_valid, int target,
                                                           double* __restrict__ acc) {
    __shared__ float s_max[kNllThreads / 32];
    __shared__ double s_sum[kNllThreads / 32];
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < n_valid; i += kNllThreads) mx = fmaxf(mx, __ldcg(logits + i));
    mx = warp_max(mx);
    if (lane == 0) s_max[warp] = mx;
    __syncthreads();
    mx = s_max[0];
    for (int w = 1; w < kNllThreads / 32; ++w) mx = fmaxf(mx, s_max[w]);
    double sum = 0.0;
    for (int i = threadIdx.x; i < n_valid; i += kNllThreads) sum += exp(double(fsub(__ldcg(logits + i), mx)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) s_sum[warp] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        double total = 0.0;
        for (int w = 0; w < kNllThreads / 32; ++w) total += s_sum[w];
        const float lt = target >= 0 && target < n_valid ? __ldcg(logits + target) : -INFINITY;
        *acc += (log(total) + double(mx)) - double(lt);
    }
}

}  // namespace

cudaError_t launch_token_nll(const float* logits, int n_valid, int target, double* acc, cudaStream_t st, bool pdl) {
    if (n_valid <= 0) return cudaErrorInvalidValue;
    return launch_pdl(k_token_nll, dim3(1), dim3(kNllThreads), 0, st, pdl, logits, n_valid, target, acc);
}

}  // namespace qb
