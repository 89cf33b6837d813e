// Device building blocks shared by the decode (M=1) and prefill/batched kernels, so that every path evaluates
// each output with the same sequence of float operations.
#pragma once

#include "common.cuh"
#include "exp_table.h"

namespace qb {

constexpr int kThreads = 256;  // threads per CTA for the matvec-family kernels
constexpr int kWarps = kThreads / 32;

// Exact quotient n / d for n, d < 2^16 from m = ceil(2^32 / d) (host-computed).
__device__ __forceinline__ unsigned fast_div(unsigned n, unsigned m) { return __umulhi(n, m); }
inline unsigned div_magic(unsigned d) { return unsigned((0x100000000ULL + d - 1) / d); }

// cp.async: 16-byte (L2 only) and 4-byte asynchronous copies global -> shared, grouped and awaited per thread
// (cp.async.wait_group, then a CTA barrier, before other threads read the data).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

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
// ssum[b] = sum of the 32 int8 of block b, one thread per block (two 16-byte loads, eight byte-sum dp4a); sx 16-byte
// aligned.
__device__ __forceinline__ void block_sums_i8(const int8_t* sx, int n, int* ssum) {
    for (int b = threadIdx.x; b < n / QK; b += blockDim.x) {
        const int4* p = reinterpret_cast<const int4*>(sx + b * QK);
        const int4 u = p[0], v = p[1];
        int s = __dp4a(u.x, 0x01010101, 0);
        s = __dp4a(u.y, 0x01010101, s);
        s = __dp4a(u.z, 0x01010101, s);
        s = __dp4a(u.w, 0x01010101, s);
        s = __dp4a(v.x, 0x01010101, s);
        s = __dp4a(v.y, 0x01010101, s);
        s = __dp4a(v.z, 0x01010101, s);
        ssum[b] = __dp4a(v.w, 0x01010101, s);
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
//
// Element i of an activation belongs to thread i % blockDim in "round" i / blockDim; with blockDim a multiple of 32
// warp w of round k holds exactly block w + k * nwarps, so each block is quantized by one warp.  All of a thread's
// loads are issued before any dependent math (a decode step is a chain of these prologues).
constexpr int kMaxRounds = 8;  // vectors up to kMaxRounds * blockDim elements take the register path

// Norm weights in registers (constant: loaded before the programmatic-launch wait).
struct NormW {
    float w[kMaxRounds];
};
__device__ __forceinline__ void load_norm_w(const float* __restrict__ w, int dim, NormW& nw) {
#pragma unroll
    for (int k = 0; k < kMaxRounds; ++k) {
        const int i = threadIdx.x + k * blockDim.x;
        nw.w[k] = i < dim ? w[i] : 0.f;
    }
}

// quantize_q8 of a whole activation held in registers, v[k] = element k * blockDim + tid (0 past n): the rounds'
// warp reductions, divisions and roundings are interleaved (independent per round), which keeps the dependent
// latency of a decode prologue to about one round's.  Same results as quant_round on every round.
template <int NR>
__device__ __forceinline__ void quant_rounds_n(const float* v, int n, int8_t* sx, float* sdx, int* ssum) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, T = blockDim.x;
    float amax[NR];
#pragma unroll
    for (int k = 0; k < NR; ++k) amax[k] = fabsf(v[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int k = 0; k < NR; ++k) amax[k] = fmaxf(amax[k], __shfl_xor_sync(0xffffffffu, amax[k], o));
    }
    int q[NR];
#pragma unroll
    for (int k = 0; k < NR; ++k) {
        const float d = div127(amax[k]);
        const float inv = d > 0.f ? __frcp_rn(d) : 0.0f;
        q[k] = int((int8_t)round_away(fmul(v[k], inv)));
        if (k * T + warp * 32 < n) {
            sx[k * T + tid] = int8_t(q[k]);
            if (lane == 0) sdx[(k * T + tid) / QK] = d;
        }
    }
    if (ssum) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
            for (int k = 0; k < NR; ++k) q[k] += __shfl_xor_sync(0xffffffffu, q[k], o);
        }
#pragma unroll
        for (int k = 0; k < NR; ++k)
            if (k * T + warp * 32 < n && lane == 0) ssum[(k * T + tid) / QK] = q[k];
    }
}
__device__ __forceinline__ void quant_rounds(const float (&v)[kMaxRounds], int n, int8_t* sx, float* sdx, int* ssum) {
    if (n <= 4 * int(blockDim.x)) quant_rounds_n<4>(v, n, sx, sdx, ssum);
    else quant_rounds_n<kMaxRounds>(v, n, sx, sdx, ssum);
}

// Sum of squares in element order, ((x0*x0 + x1*x1) + x2*x2) + ..., the reference's sequential loop
// (engine/src/ops_ref.cpp:195-196): the squares are formed in parallel into sq[], one thread runs the add chain.
// Any other order changes the last bits of the scale, and those flip int8 activations and f16 cache entries
// downstream, so this order is kept although the chain costs ~4 cycles per element.
// s = ((s0 + v_0) + v_1) + ... + v_{n-1}: the reference's sequential float sum, on one thread.  The chain of adds is
// the latency floor, so the loads run one 16-value group ahead of the adds (v 16-byte aligned for the vector path).
__device__ __forceinline__ float ordered_sum(const float* v, int n, float s = 0.f) {
    int i = 0;
    if (n >= 16 && (reinterpret_cast<uintptr_t>(v) & 15) == 0) {
        const float4* v4 = reinterpret_cast<const float4*>(v);
        float4 cur[4], nxt[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) cur[k] = v4[k];
        for (i = 16; i + 16 <= n; i += 16) {
#pragma unroll
            for (int k = 0; k < 4; ++k) nxt[k] = v4[i / 4 + k];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                s = fadd(s, cur[k].x);
                s = fadd(s, cur[k].y);
                s = fadd(s, cur[k].z);
                s = fadd(s, cur[k].w);
                cur[k] = nxt[k];
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            s = fadd(s, cur[k].x);
            s = fadd(s, cur[k].y);
            s = fadd(s, cur[k].z);
            s = fadd(s, cur[k].w);
        }
    }
    for (; i < n; ++i) s = fadd(s, v[i]);
    return s;
}

// rmsnorm (engine/src/ops_ref.cpp:194-199) then quantize_q8 (:69-83) of x[dim] into sx / sdx (and block sums).
// sred: scratch of >= dim + 32 floats.  Bit-identical to the reference.  dim <= kMaxRounds * blockDim.
// norm_quant_v: the same on values already in registers, xv[k] = element tid + k * blockDim (0 past dim).
__device__ __forceinline__ void norm_quant_v(const float (&xv)[kMaxRounds], const NormW& nw, int dim, float eps, int8_t* sx,
                                             float* sdx, int* ssum, float* sred) {
    const int tid = threadIdx.x, T = blockDim.x;
    float* sq = sred + 32;
#pragma unroll
    for (int k = 0; k < kMaxRounds; ++k)
        if (tid + k * T < dim) sq[tid + k * T] = fmul(xv[k], xv[k]);
    __syncthreads();
    if (tid == 0) sred[0] = ordered_sum(sq, dim);
    __syncthreads();
    const float tot = sred[0];
    const float scale = __frcp_rn(__fsqrt_rn(fadd(fdiv(tot, float(dim)), eps)));  // 1.0f / sqrt(...), IEEE round to nearest
    float y[kMaxRounds];
#pragma unroll
    for (int k = 0; k < kMaxRounds; ++k) y[k] = fmul(fmul(xv[k], scale), nw.w[k]);  // 0 past dim
    quant_rounds(y, dim, sx, sdx, ssum);
    __syncthreads();
}
__device__ __forceinline__ void norm_quant(const float* __restrict__ x, const NormW& nw, int dim, float eps, int8_t* sx,
                                           float* sdx, int* ssum, float* sred) {
    const int tid = threadIdx.x, T = blockDim.x;
    float xv[kMaxRounds];
#pragma unroll
    for (int k = 0; k < kMaxRounds; ++k) xv[k] = tid + k * T < dim ? __ldcg(x + tid + k * T) : 0.f;
    norm_quant_v(xv, nw, dim, eps, sx, sdx, ssum, sred);
}

// quantize_q8 of x[n] (no norm) into sx / sdx (and block sums); n <= kMaxRounds * blockDim.
__device__ __forceinline__ void quant_only(const float* __restrict__ x, int n, int8_t* sx, float* sdx, int* ssum) {
    const int tid = threadIdx.x, T = blockDim.x;
    float xv[kMaxRounds];
#pragma unroll
    for (int k = 0; k < kMaxRounds; ++k) xv[k] = tid + k * T < n ? __ldcg(x + tid + k * T) : 0.f;
    quant_rounds(xv, n, sx, sdx, ssum);
    __syncthreads();
}

// Copies an already-quantized activation (int8 + block scales) into shared memory (and its block sums).
__device__ __forceinline__ void load_quant(const int8_t* __restrict__ q, const float* __restrict__ d, int n, int8_t* sx,
                                           float* sdx, int* ssum) {
    const int4* src = reinterpret_cast<const int4*>(q);
    int4* dst = reinterpret_cast<int4*>(sx);
    const int T = blockDim.x;
    int4 v[4];
    float dv[2];
    for (int base = 0; base < n / 16; base += 4 * T) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i = base + threadIdx.x + k * T;
            if (i < n / 16) v[k] = __ldcg(src + i);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i = base + threadIdx.x + k * T;
            if (i < n / 16) dst[i] = v[k];
        }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) dv[k] = threadIdx.x + k * T < n / QK ? __ldcg(d + threadIdx.x + k * T) : 0.f;
#pragma unroll
    for (int k = 0; k < 2; ++k)
        if (threadIdx.x + k * T < n / QK) sdx[threadIdx.x + k * T] = dv[k];
    for (int b = threadIdx.x + 2 * T; b < n / QK; b += T) sdx[b] = __ldcg(d + b);
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

// silu(g) * u (engine/src/ops_ref.cpp:243-248), e^-g with the host libm's bits (exp_table.h).
__device__ __forceinline__ float swiglu1(float g, float u, const ExpTab& tab) {
    return fmul(fdiv(g, fadd(1.0f, exp_ref(-g, tab))), u);
}

}  // namespace qb
