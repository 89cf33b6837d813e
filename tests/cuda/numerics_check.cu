// Exhaustive checks of the exact arithmetic shortcuts in quanta.cpp_b200/csrc/common.cuh against the CUDA
// operations they stand in for (each compared bit for bit over its whole input range):
//   div127(a)        == __fdiv_rn(a, 127.0f)   every non-negative, non-NaN float a (the quantizer's scale)
//   __frcp_rn(d)     == __fdiv_rn(1.0f, d)     every non-negative, non-NaN float d (the scale's reciprocal)
//   round_away(y)    == lroundf(y)             every float with |y| < 2^22 (the quantizer's rounding)
// Prints one line "mismatches div127=... frcp=... round=..." and exits 0 when it ran.
#include <cmath>
#include <cstdio>

#include "common.cuh"

using namespace qb;

__global__ void k_check(unsigned long long* bad) {
    const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
    for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < (1ull << 32); i += stride) {
        const float x = __uint_as_float(unsigned(i));
        if (i < (1ull << 31) && x == x) {  // non-negative, non-NaN
            if (__float_as_uint(div127(x)) != __float_as_uint(__fdiv_rn(x, 127.0f))) atomicAdd(&bad[0], 1ull);
            if (__float_as_uint(__frcp_rn(x)) != __float_as_uint(__fdiv_rn(1.0f, x))) atomicAdd(&bad[1], 1ull);
        }
        if (fabsf(x) < 4194304.0f && long(round_away(x)) != lroundf(x)) atomicAdd(&bad[2], 1ull);
    }
}

int main() {
    unsigned long long* bad = nullptr;
    if (cudaMalloc(&bad, 3 * sizeof(unsigned long long)) != cudaSuccess) return 2;
    cudaMemset(bad, 0, 3 * sizeof(unsigned long long));
    k_check<<<148 * 8, 256>>>(bad);
    unsigned long long h[3];
    const cudaError_t e = cudaMemcpy(h, bad, sizeof(h), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        std::printf("cuda error %s\n", cudaGetErrorString(e));
        return 2;
    }
    std::printf("mismatches div127=%llu frcp=%llu round=%llu\n", h[0], h[1], h[2]);
    return 0;
}
