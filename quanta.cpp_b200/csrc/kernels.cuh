// Device building blocks shared by the decode (M=1) and prefill/batched kernels, so that every path evaluates
// each output with the same sequence of float operations.
#pragma once

#include "common.cuh"

namespace qb {

constexpr int kThreads = 256;  // threads per CTA for the matvec-family kernels
constexpr int kWarps = kThreads / 32;

// Exact quotient n / d for n, d < 2^16 from m = ceil(2^32 / d) (host-computed).
__device__ __forceinline__ unsigned fast_div(unsigned n, unsigned m) { return __umulhi(n, m); }
inline unsigned div_magic(unsigned d) { return unsigned((0x100000000ULL + d - 1) / d); }

// Streaming 16-byte load that does not allocate in L1 (weights are read once per step).
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Partial integer dot of one 16-byte weight chunk with the activation.
//   Q8_0: chunk c of a row covers elements [16c, 16c+16) -> half a block (two chunks per block).
//   Q4_0: chunk c covers block c (32 elements; byte j = q[j] | q[j+16] << 4, value q-8); the -8 offset is applied
//         by the caller as -8 * sum(x_block) so that the partial is the exact int sum of (q-8)*x.
template <int DT>
__device__ __forceinline__ int chunk_dot(const uint4 w, const int8_t* __restrict__ sx, int c) {
    if (DT == DT_Q8_0) {
        const int4 x = *reinterpret_cast<const int4*>(sx + c * 16);
        int s = dp4a_ss(int(w.x), x.x, 0);
        s = dp4a_ss(int(w.y), x.y, s);
        s = dp4a_ss(int(w.z), x.z, s);
        return dp4a_ss(int(w.w), x.w, s);
    } else {
        const int4 xl = *reinterpret_cast<const int4*>(sx + c * 32);
        const int4 xh = *reinterpret_cast<const int4*>(sx + c * 32 + 16);
        const unsigned m = 0x0F0F0F0Fu;
        int s = dp4a_us(w.x & m, xl.x, 0);
        s = dp4a_us(w.y & m, xl.y, s);
        s = dp4a_us(w.z & m, xl.z, s);
        s = dp4a_us(w.w & m, xl.w, s);
        s = dp4a_us((w.x >> 4) & m, xh.x, s);
        s = dp4a_us((w.y >> 4) & m, xh.y, s);
        s = dp4a_us((w.z >> 4) & m, xh.z, s);
        return dp4a_us((w.w >> 4) & m, xh.w, s);
    }
}

// Sum of the 32 int8 activations of each block, needed for the Q4_0 -8 offset.
__device__ __forceinline__ void block_sums_i8(const int8_t* sx, int n, int* ssum) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int b = warp; b < n / QK; b += blockDim.x / 32) {
        const int s = warp_sum_i(int(sx[b * QK + lane]));
        if (lane == 0) ssum[b] = s;
    }
}

// Row-range layout handed to the term/sum helpers.
struct RowSlice {
    const uint8_t* wq;  // first quant byte of row0
    const __half* wd;   // first scale of row0
    int nrows;
    int nb;             // blocks per row
    int cpr;            // 16-byte chunks per row
    unsigned cpr_magic; // div_magic(cpr)
    int tstride;        // smem term row stride (nb rounded up to odd)
};

__device__ __forceinline__ int term_stride(int nb) { return nb | 1; }

// Block terms (float(s) * dw) * dx for a CTA's contiguous rows, written to sterm[row * tstride + b].
// All threads of the CTA take part; U = chunks each thread handles (the whole slice must fit in
// blockDim * U chunks).  The weight chunks are loaded before `before_compute` runs, so a caller can overlap its
// activation prologue (and the programmatic-launch wait) with the weight loads in flight.
template <int DT, int U, class Prologue>
__device__ __forceinline__ void slice_terms(const RowSlice& S, const int8_t* sx, const float* sdx, const int* ssum,
                                            float* sterm, Prologue&& before_compute) {
    const int tid = threadIdx.x, T = blockDim.x;
    const int total = S.nrows * S.cpr;
    const uint4* src = reinterpret_cast<const uint4*>(S.wq);
    uint4 w[U];
    __half dw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int f = u * T + tid;
        if (f < total) {
            w[u] = ld_stream(src + f);
            const unsigned r = fast_div(unsigned(f), S.cpr_magic);
            const int c = f - int(r) * S.cpr;
            const int b = DT == DT_Q8_0 ? (c >> 1) : c;
            dw[u] = S.wd[size_t(r) * S.nb + b];
        } else {
            w[u] = make_uint4(0, 0, 0, 0);
            dw[u] = __float2half(0.f);
        }
    }
    before_compute();
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int f = u * T + tid;
        // Q8_0 pairs (f, f^1) always share validity: total and T are even.
        if (DT == DT_Q8_0) {
            if (u * T >= total) break;  // uniform across the CTA
            const unsigned r = fast_div(unsigned(f), S.cpr_magic);
            const int c = f - int(r) * S.cpr;
            int s = f < total ? chunk_dot<DT>(w[u], sx, c) : 0;
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            if (f < total && !(c & 1)) {
                const int b = c >> 1;
                sterm[int(r) * S.tstride + b] = block_term(s, __half2float(dw[u]), sdx[b]);
            }
        } else {
            if (f < total) {
                const unsigned r = fast_div(unsigned(f), S.cpr_magic);
                const int c = f - int(r) * S.cpr;
                const int s = chunk_dot<DT>(w[u], sx, c) - 8 * ssum[c];
                sterm[int(r) * S.tstride + c] = block_term(s, __half2float(dw[u]), sdx[c]);
            }
        }
    }
}

// Row sums acc = ((0 + t_0) + t_1) + ... in block order (the reference's sequential accumulation).
__device__ __forceinline__ float row_sum(const float* t, int nb) {
    float acc = 0.f;
    int b = 0;
    for (; b + 8 <= nb; b += 8) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = t[b + k];
#pragma unroll
        for (int k = 0; k < 8; ++k) acc = fadd(acc, v[k]);
    }
    for (; b < nb; ++b) acc = fadd(acc, t[b]);
    return acc;
}

// ---- activation prologues (one token; every thread of the CTA participates)

// rmsnorm (engine/src/ops_ref.cpp:194-199) then quantize_q8 (:69-83) of x[dim] into sx / sdx (and block sums).
// The sum of squares uses a fixed tree order (per-thread strided partials, warp butterfly, then warps in order),
// so every kernel that normalizes the same vector gets the same bits.
__device__ __forceinline__ void norm_quant(const float* __restrict__ x, const float* __restrict__ w, int dim, float eps,
                                           int8_t* sx, float* sdx, int* ssum, float* sred) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    float ss = 0.f;
    for (int i = tid; i < dim; i += blockDim.x) ss = fadd(ss, fmul(x[i], x[i]));
    ss = warp_sum(ss);
    if (lane == 0) sred[warp] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int k = 0; k < nw; ++k) tot = fadd(tot, sred[k]);
    const float scale = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(tot, float(dim)), eps)));
    for (int b = warp; b < dim / QK; b += nw) {
        const int i = b * QK + lane;
        const float v = fmul(fmul(x[i], scale), w[i]);
        float d;
        const int8_t q = quantize_lane(v, &d);
        sx[i] = q;
        if (ssum) {
            const int s = warp_sum_i(int(q));
            if (lane == 0) ssum[b] = s;
        }
        if (lane == 0) sdx[b] = d;
    }
    __syncthreads();
}

// quantize_q8 of x[n] (no norm) into sx / sdx (and block sums).
__device__ __forceinline__ void quant_only(const float* __restrict__ x, int n, int8_t* sx, float* sdx, int* ssum) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int b = warp; b < n / QK; b += nw) {
        const int i = b * QK + lane;
        float d;
        const int8_t q = quantize_lane(x[i], &d);
        sx[i] = q;
        if (ssum) {
            const int s = warp_sum_i(int(q));
            if (lane == 0) ssum[b] = s;
        }
        if (lane == 0) sdx[b] = d;
    }
    __syncthreads();
}

// Copies an already-quantized activation (int8 + block scales) into shared memory (and its block sums).
__device__ __forceinline__ void load_quant(const int8_t* __restrict__ q, const float* __restrict__ d, int n, int8_t* sx,
                                           float* sdx, int* ssum) {
    const int4* src = reinterpret_cast<const int4*>(q);
    int4* dst = reinterpret_cast<int4*>(sx);
    for (int i = threadIdx.x; i < n / 16; i += blockDim.x) dst[i] = src[i];
    for (int b = threadIdx.x; b < n / QK; b += blockDim.x) sdx[b] = d[b];
    __syncthreads();
    if (ssum) {
        block_sums_i8(sx, n, ssum);
        __syncthreads();
    }
}

// ---- elementwise pieces

// NeoX rotate-half RoPE on one pair (i, i + half) with host-computed cos/sin (engine/src/ops_ref.cpp:201-214).
__device__ __forceinline__ void rope_pair(float& a, float& b, float c, float s) {
    const float na = fsub(fmul(a, c), fmul(b, s));
    const float nb = fadd(fmul(b, c), fmul(a, s));
    a = na;
    b = nb;
}

// silu(g) * u (engine/src/ops_ref.cpp:243-248).
__device__ __forceinline__ float swiglu1(float g, float u) { return fmul(fdiv(g, fadd(1.0f, expf(-g))), u); }

}  // namespace qb
