// Shared device helpers for the sm_100a kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qb {

constexpr int QK = 32;  // quantization block (engine/src/model_file.h:17)

enum DType : int { DT_F32 = 0, DT_F16 = 1, DT_Q8_0 = 2, DT_Q4_0 = 3 };

// Error bits written by kernels into the device status word (read by the host after a step).
enum : unsigned {
    ERR_WAIT_TIMEOUT = 1u,   // a bounded spin (mbarrier / flag) gave up
    ERR_BAD_TOKEN = 2u,      // token id outside the embedding
    ERR_BAD_POS = 4u,        // position outside the KV cache
    ERR_CAPACITY = 8u,       // a fixed-size device list overflowed
};

// Device view of a quantized (or float) matrix in HBM.  Quants are row-major, scales are [rows][cols/32] fp16,
// exactly the .qnt section order (quants then scales), each array 256-byte aligned.
struct DMat {
    int dtype;
    int rows, cols;
    const uint8_t* q;      // Q8_0: int8 [rows][cols]; Q4_0: packed nibbles [rows][cols/2]; F32/F16: values
    const __half* d;       // fp16 block scales [rows][cols/32] (quantized types only)
};

__device__ __forceinline__ int row_bytes(int dtype, int cols) { return dtype == DT_Q4_0 ? cols / 2 : cols; }

// int8 x int8 dot of four lanes, signed x signed (dp4a.s32.s32).
__device__ __forceinline__ int dp4a_ss(int a, int b, int c) { return __dp4a(a, b, c); }
// unsigned bytes (0..255) x signed bytes (dp4a.u32.s32).
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Round-to-nearest float ops with no FMA contraction: the reference evaluates `acc += float(s) * dw * dx`
// (engine/src/ops_ref.cpp:98) as two products then a sum, and these keep the same rounding sequence.
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

// One block term of the integer matvec: (float(s) * dw) * dx.
__device__ __forceinline__ float block_term(int s, float dw, float dx) { return fmul(fmul(float(s), dw), dx); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fadd(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Programmatic dependent launch: let the next kernel in the stream start its prologue (weight prefetch) now,
// and wait here until every kernel this one depends on has finished and its writes are visible.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void set_error(unsigned* status, unsigned bit) {
    if (status) atomicOr(status, bit);
}

// Quantize 32 consecutive floats held one per lane of a warp (engine/src/ops_ref.cpp:69-83):
// d = amax/127, inv = d > 0 ? 1/d : 0, q = lround(x * inv).  Returns q for this lane; *d_out gets d.
// Two f32 lanes in one 64-bit register: each lane rounds to nearest like fmaf / fmul / fadd, no flush to zero.
// ptxas contracts a mul.rn.f32x2 that feeds an add.rn.f32x2 into one fma (a single rounding), so the products are
// taken as fma(a, b, -0.0) with the -0.0 a kernel argument: round(a * b) exactly, and nothing left to contract.
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ unsigned long long f2_pack_bits(int lo, int hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ float2 f2_unpack(unsigned long long v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// a / 127 correctly rounded, for a >= 0 (the quantizer's scale): one correction step of the product with RN(1/127)
// (Markstein), infinity passed through.  Checked equal to a / 127.0f for every non-negative float bit pattern.  The
// reciprocal of the scale is __frcp_rn (IEEE round to nearest, equal to 1.0f / d for every d >= 0, checked the same way).
__device__ __forceinline__ float div127(float a) {
    const float r127 = 7.8740157186985015869140625e-3f;  // RN(1 / 127)
    const float q0 = __fmul_rn(a, r127);
    const float q1 = __fmaf_rn(__fmaf_rn(-q0, 127.0f, a), r127, q0);
    return isinf(a) ? a : q1;
}

// lroundf (half away from zero) for |y| < 2^22 with two round-toward-zero adds: floor(|y| + 0.5) + 2^23 lands in the
// low mantissa bits.  Checked equal to lroundf for every float of that range.
__device__ __forceinline__ int round_away(float y) {
    const float s = __fadd_rz(__fadd_rz(fabsf(y), 0.5f), 8388608.0f);
    const int q = __float_as_int(s) - 0x4B000000;
    return y < 0.f ? -q : q;
}

__device__ __forceinline__ int8_t quantize_lane(float x, float* d_out) {
    const float amax = warp_max(fabsf(x));
    const float d = div127(amax);
    const float inv = d > 0.f ? __frcp_rn(d) : 0.0f;
    *d_out = d;
    return (int8_t)round_away(fmul(x, inv));  // |x * inv| <= 127 (plus rounding)
}

// Launches `kernel`, optionally as a programmatic dependent of the previous launch on the stream (the kernel then
// calls griddepcontrol.launch_dependents / .wait); raises the dynamic shared memory limit when it needs more than 48 KB.
template <class... KArgs, class... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return e;
    }
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace qb

#define QB_CUDA_OK(expr)                                                         \
    do {                                                                         \
        cudaError_t e_ = (expr);                                                 \
        if (e_ != cudaSuccess) return qb::fail_cuda(e_, #expr, __FILE__, __LINE__); \
    } while (0)
