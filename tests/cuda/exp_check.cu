// Exhaustive check of exp_ref (quanta.cpp_b200/csrc/exp_table.h) against the host libm: for every float x in
// (-104, 89) -- the inputs that can give a finite, nonzero expf -- the device's exp_ref(x) must have the bits of the
// host's std::exp(float) (glibc expf, what the reference calls in softmax, SwiGLU and the sampler).
//
// The device side rounds its double-precision exp once and consults the exception table only near a rounding
// midpoint.  CUDA's double exp is not correctly rounded, so this also catches an input where the device's double
// and the host's double fall on opposite sides of a float midpoint.
//
// Prints "exp_ref checked=N mismatches=M" (and the first mismatching inputs) and exits 0 when it ran.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

#include "exp_table.h"

using namespace qb;

__global__ void k_exp(uint32_t b0, uint32_t n, ExpTab tab, float* out) {
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = exp_ref(__uint_as_float(b0 + i), tab);
}

int main() {
    const std::vector<uint64_t>& slots = expf_exception_slots(nullptr);
    unsigned long long* dslots = nullptr;
    if (cudaMalloc(&dslots, slots.size() * 8) != cudaSuccess) return 2;
    cudaMemcpy(dslots, slots.data(), slots.size() * 8, cudaMemcpyHostToDevice);
    const ExpTab tab{dslots, unsigned(slots.size() - 1)};

    // bit ranges of the floats in (-104, 89): [+0, 89) and [-0, -104)
    uint32_t pos_end, neg_end;
    const float p89 = 89.f, m104 = -104.f;
    std::memcpy(&pos_end, &p89, 4);
    std::memcpy(&neg_end, &m104, 4);
    const uint32_t ranges[2][2] = {{0u, pos_end}, {0x80000000u, neg_end}};

    const uint32_t chunk = 1u << 26;
    float* dout = nullptr;
    float* hout = nullptr;
    if (cudaMalloc(&dout, size_t(chunk) * 4) != cudaSuccess || cudaMallocHost(&hout, size_t(chunk) * 4) != cudaSuccess)
        return 2;
    unsigned nt = std::thread::hardware_concurrency();
    if (nt == 0) nt = 4;
    unsigned long long checked = 0, bad = 0;
    std::vector<uint32_t> first_bad;
    for (const auto& r : ranges) {
        for (uint64_t b0 = r[0]; b0 < r[1]; b0 += chunk) {
            const uint32_t n = uint32_t(std::min<uint64_t>(chunk, r[1] - b0));
            k_exp<<<148 * 8, 256>>>(uint32_t(b0), n, tab, dout);
            const cudaError_t e = cudaMemcpy(hout, dout, size_t(n) * 4, cudaMemcpyDeviceToHost);
            if (e != cudaSuccess) {
                std::printf("cuda error %s\n", cudaGetErrorString(e));
                return 2;
            }
            std::vector<unsigned long long> nbad(nt, 0);
            std::vector<std::vector<uint32_t>> firsts(nt);
            std::vector<std::thread> ts;
            for (unsigned t = 0; t < nt; ++t)
                ts.emplace_back([&, t] {
                    const uint32_t i0 = uint32_t(uint64_t(n) * t / nt), i1 = uint32_t(uint64_t(n) * (t + 1) / nt);
                    for (uint32_t i = i0; i < i1; ++i) {
                        const uint32_t bits = uint32_t(b0) + i;
                        float x;
                        std::memcpy(&x, &bits, 4);
                        const float want = std::exp(x);
                        uint32_t wb, gb;
                        std::memcpy(&wb, &want, 4);
                        std::memcpy(&gb, &hout[i], 4);
                        if (wb != gb) {
                            ++nbad[t];
                            if (firsts[t].size() < 4) firsts[t].push_back(bits);
                        }
                    }
                });
            for (auto& th : ts) th.join();
            for (unsigned t = 0; t < nt; ++t) {
                bad += nbad[t];
                for (uint32_t b : firsts[t])
                    if (first_bad.size() < 16) first_bad.push_back(b);
            }
            checked += n;
        }
    }
    std::printf("exp_ref checked=%llu mismatches=%llu\n", checked, bad);
    for (uint32_t b : first_bad) {
        float x;
        std::memcpy(&x, &b, 4);
        std::printf("  mismatch x=%.9g (0x%08x) host=%a\n", x, b, std::exp(x));
    }
    return 0;
}
