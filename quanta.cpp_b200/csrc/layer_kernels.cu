// Per-layer kernels of the Qwen2 forward (engine/src/model.cpp:165-228 decode, :363-433 prefill chunk).
//
// Decode (one token) runs, in its separate form, five kernels per layer, each fusing its neighbours:
//   k_qkv_dec     rmsnorm + quantize (prologue) -> fused q|k|v integer matvec -> bias + RoPE -> q, f16 K/V store
//   k_attn        GQA attention over the f16 KV cache (attention.cu)
//   k_resid_dec   quantize(attn) -> o_proj matvec -> residual add
//   k_gateup_dec  rmsnorm + quantize -> gate|up matvec (rows interleaved per 32-block) -> SwiGLU -> quantize
//   k_resid_dec   down_proj matvec -> residual add
// Where the shapes allow, the default is three: attention.cu's launch_qkv_attn takes q|k|v in front of the attention
// and the o_proj block terms behind it, k_gateup_dec<.., RT = true> adds those terms onto the residual before its
// norm, and k_resid_dec does down.  Files with FLAG_HADAMARD_DOWN add k_fwht_quant between gate|up and down.
// Every kernel first loads its weight slice, then waits for the previous kernel (programmatic dependent launch), and
// only then lets the next kernel launch: weight traffic overlaps the launch gap and the previous kernel's tail, and at
// most one kernel ahead is resident, so early launches never fill the SMs with CTAs that cannot run yet.
// A kernel launched early this way may run on an SM whose L1 still holds lines that earlier kernels of the chain
// have since rewritten (L1 is not coherent, and the wait does not invalidate it), so every read of data produced by
// another kernel goes through L2 (__ldcg / ld.global.cg); only constant weights use L1 or the non-coherent path.
//
// Prefill runs the matmul (tensor-core or CUDA-core) on whole chunks and the same elementwise helpers as the
// decode kernels' epilogues, so batched and token-by-token give the same bits.
#include <cooperative_groups.h>

#include "kernels.cuh"
#include "layer_kernels.h"
#include "qkv_pair.cuh"
#include "phase_stamps.cuh"

namespace qb {

namespace cg = cooperative_groups;
constexpr int kRtMaxNb = 32;  // o_proj blocks per row that the gate|up residual-terms form takes (o_proj cols <= 1024)

// ---------------------------------------------------------------- embedding (engine/src/ops_ref.cpp:162-192 get_row)

__global__ void k_embed(DMat E, const int* __restrict__ tokens, int n_tok, float* __restrict__ X, unsigned* status) {
    PhaseProbe probe;
    probe.begin(4);
    pdl_wait();
    pdl_launch_dependents();
    probe.mark();
    const int t = blockIdx.x;
    if (t >= n_tok) return;
    int tok = __ldcg(tokens + t);
    if (tok < 0 || tok >= E.rows) {
        if (threadIdx.x == 0) set_error(status, ERR_BAD_TOKEN);
        tok = 0;
    }
    const int dim = E.cols;
    const int8_t* q = reinterpret_cast<const int8_t*>(E.q) + size_t(tok) * dim;
    const __half* d = E.d + size_t(tok) * (dim / QK);
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
        X[size_t(t) * dim + i] = fmul(float(q[i]), __half2float(d[i / QK]));
    probe.end();
}

// ---------------------------------------------------------------- shared epilogues

// ---------------------------------------------------------------- decode kernels

struct SliceSmem {
    int8_t* sx;
    float* sdx;
    int* ssum;
    float* sterm;
    float* sval;  // row results
    float* sred;
};

__device__ __forceinline__ SliceSmem carve(unsigned char* smem, int cols, int rows, int tstride) {
    SliceSmem s;
    const int nb = cols / QK;
    s.sx = reinterpret_cast<int8_t*>(smem);
    s.sdx = reinterpret_cast<float*>(smem + cols);
    s.ssum = reinterpret_cast<int*>(s.sdx + nb);
    s.sred = reinterpret_cast<float*>(s.ssum + nb);  // 32 + cols floats (norm_quant's squares)
    s.sval = s.sred + 32 + cols;
    s.sterm = s.sval + ((rows + 3) & ~3);
    return s;
}

size_t slice_smem_bytes(int cols, int rows) {
    const int nb = cols / QK;
    return size_t(cols) + size_t(nb) * 8 + size_t(32 + cols) * 4 + size_t((rows + 3) & ~3) * 4 + size_t(rows) * (nb | 1) * 4;
}

__device__ __forceinline__ RowSlice make_slice(const DMat& W, int dt, int row0, int nrows, unsigned magic) {
    RowSlice S;
    const int rb = row_bytes(dt, W.cols);
    S.wq = W.q + size_t(row0) * rb;
    S.wd = W.d + size_t(row0) * (W.cols / QK);
    S.nrows = nrows;
    S.nb = W.cols / QK;
    S.cpr = rb / 16;
    S.cpr_magic = magic;
    S.tstride = term_stride(S.nb);
    return S;
}

template <int DT, int U>
__global__ void __launch_bounds__(kThreads) k_qkv_dec(QkvArgs a, const float* __restrict__ X, const float* __restrict__ norm_w,
                                                      float eps, const int* __restrict__ pos_dev, float* __restrict__ Q,
                                                      int rows_per_cta, unsigned magic) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int dim = a.W.cols;
    const int row0 = blockIdx.x * rows_per_cta, nrows = min(rows_per_cta, a.W.rows - row0);
    SliceSmem s = carve(smem, dim, rows_per_cta, term_stride(dim / QK));
    RowSlice S = make_slice(a.W, DT, row0, nrows, magic);
    NormW nw;
    load_norm_w(norm_w, dim, nw);
    const bool has_pair = int(threadIdx.x) < nrows / 2;  // one pair per thread (rows_per_cta <= 2 * blockDim)
    const int pr = row0 + 2 * threadIdx.x;
    PairIn pin{0.f, 0.f, 1.f, 0.f};
    if (has_pair) pair_bias(a, pr, pin);
    int pos = 0;
    slice_terms<DT, U>(S, s.sx, s.sdx, s.ssum, s.sterm, [&] {
        pdl_wait();
        pdl_launch_dependents();
        pos = __ldcg(pos_dev);
        if (has_pair) pair_rope(a, pr, pos, pin);
        norm_quant(X, nw, dim, eps, s.sx, s.sdx, DT == DT_Q4_0 ? s.ssum : nullptr, s.sred);
    });
    __syncthreads();
    for (int r = threadIdx.x; r < nrows; r += blockDim.x) s.sval[r] = row_sum(s.sterm + r * S.tstride, S.nb);
    __syncthreads();
    if (has_pair) qkv_pair_store(a, pr, s.sval[2 * threadIdx.x], s.sval[2 * threadIdx.x + 1], pos, pin, Q);
}

// out rows -> X[row] += value (residual).  mode 0: input is f32 attn output to quantize; mode 1: pre-quantized.
template <int DT, int U, int MODE>
// Xres: where the residual is read (X itself when null; the gate|up kernel's X2 after an o_proj folded into it).
__global__ void __launch_bounds__(kThreads) k_resid_dec(DMat W, const float* __restrict__ xin, const int8_t* __restrict__ qin,
                                                        const float* __restrict__ din, float* __restrict__ X,
                                                        int rows_per_cta, unsigned magic, const float* __restrict__ Xres) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int cols = W.cols;
    const int row0 = blockIdx.x * rows_per_cta, nrows = min(rows_per_cta, W.rows - row0);
    SliceSmem s = carve(smem, cols, rows_per_cta, term_stride(cols / QK));
    RowSlice S = make_slice(W, DT, row0, nrows, magic);
    float xres = 0.f;  // this thread's residual row (rows_per_cta <= blockDim)
    PhaseProbe probe;
    probe.begin(3);
    slice_terms<DT, U>(S, s.sx, s.sdx, s.ssum, s.sterm, [&] {
        pdl_wait();
        pdl_launch_dependents();
        probe.mark();  // 1: the previous kernel is done
        if (int(threadIdx.x) < nrows) xres = __ldcg((Xres ? Xres : X) + row0 + threadIdx.x);
        if (MODE == 0) quant_only(xin, cols, s.sx, s.sdx, DT == DT_Q4_0 ? s.ssum : nullptr);
        else load_quant(qin, din, cols, s.sx, s.sdx, DT == DT_Q4_0 ? s.ssum : nullptr);
        probe.mark();  // 2: the input activation in shared memory
    });
    __syncthreads();
    probe.mark();  // 3: the block terms of the matvec
    if (int(threadIdx.x) < nrows) X[row0 + threadIdx.x] = fadd(xres, row_sum(s.sterm + threadIdx.x * S.tstride, S.nb));
    probe.end();  // 4: the row chains and the residual
}

// gate|up rows interleaved per 32-block: fused row 64j + i = gate row 32j + i, 64j + 32 + i = up row 32j + i.
// Each CTA owns whole ffn blocks, so it finishes SwiGLU and the block's int8 quantization itself.
//
// RT (residual terms, decode with o_proj folded into the attention): launched in clusters of 8.  After the wait, CTA c
// of each cluster forms rows [c R, c R + R) (R = dim / 8) of the o_proj residual, X + ((0 + T_r0) + T_r1) + ... in
// block order (k_resid_dec's arithmetic on the attention's terms), posts them into all 8 CTAs (distributed shared
// memory) and the first cluster stores them into X2; every CTA then norms the whole vector from shared memory.
template <int DT, int U, bool RT>
__global__ void __launch_bounds__(kThreads) k_gateup_dec(DMat W, const float* __restrict__ X, const float* __restrict__ norm_w,
                                                         float eps, int8_t* __restrict__ HQ, float* __restrict__ HD,
                                                         int blocks_per_cta, unsigned magic, ExpTab tab,
                                                         const float* __restrict__ T, int nbo, float* __restrict__ X2,
                                                         int xn_off, float* __restrict__ Hf) {
    extern __shared__ __align__(16) unsigned char smem[];
    // every CTA of the cluster has started before the first remote store (the wait comes before it)
    if constexpr (RT) asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
    const int dim = W.cols;
    const int rows_per_cta = blocks_per_cta * 64;
    const int row0 = blockIdx.x * rows_per_cta, nrows = min(rows_per_cta, W.rows - row0);
    SliceSmem s = carve(smem, dim, rows_per_cta, term_stride(dim / QK));
    RowSlice S = make_slice(W, DT, row0, nrows, magic);
    NormW nw;
    load_norm_w(norm_w, dim, nw);
    PhaseProbe probe;
    probe.begin(2);
    slice_terms<DT, U>(S, s.sx, s.sdx, s.ssum, s.sterm, [&] {
        pdl_wait();
        pdl_launch_dependents();
        probe.mark();  // 1: the previous kernel is done
        if constexpr (RT) {
            cg::cluster_group cl = cg::this_cluster();
            const int cr = int(cl.block_rank()), rpc = (dim + 7) / 8, rr0 = cr * rpc, nr = min(rpc, dim - rr0);
            float* sxn = reinterpret_cast<float*>(smem + xn_off);
            const int i = threadIdx.x;
            float xn = 0.f;
            if (i < nr) {
                const int row = rr0 + i;
                const float xo = __ldcg(X + row);
                const float4* t4 = reinterpret_cast<const float4*>(T + size_t(row) * nbo);
                float4 tv[kRtMaxNb / 4];
#pragma unroll
                for (int j = 0; j < kRtMaxNb / 4; ++j)
                    if (j < nbo / 4) tv[j] = __ldcg(t4 + j);
                float acc = 0.f;
#pragma unroll
                for (int j = 0; j < kRtMaxNb / 4; ++j) {
                    if (j < nbo / 4) {
                        acc = fadd(acc, tv[j].x);
                        acc = fadd(acc, tv[j].y);
                        acc = fadd(acc, tv[j].z);
                        acc = fadd(acc, tv[j].w);
                    }
                }
                xn = fadd(xo, acc);
                if (blockIdx.x < 8) X2[row] = xn;  // the first cluster stores the residual for the down kernel
            }
            asm volatile("barrier.cluster.wait;" ::: "memory");
            if (i < nr) {
#pragma unroll
                for (int q = 0; q < 8; ++q) cl.map_shared_rank(sxn, q)[rr0 + i] = xn;
            }
            asm volatile("barrier.cluster.arrive.release;" ::: "memory");
            asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
            probe.mark();  // 2: the o_proj residual rows and their exchange
            float xv[kMaxRounds];
#pragma unroll
            for (int k = 0; k < kMaxRounds; ++k) xv[k] = i + k * int(blockDim.x) < dim ? sxn[i + k * blockDim.x] : 0.f;
            norm_quant_v(xv, nw, dim, eps, s.sx, s.sdx, DT == DT_Q4_0 ? s.ssum : nullptr, s.sred);
            probe.mark();  // 3: rmsnorm + quantize
        } else {
            norm_quant(X, nw, dim, eps, s.sx, s.sdx, DT == DT_Q4_0 ? s.ssum : nullptr, s.sred);
        }
    });
    __syncthreads();
    probe.mark();  // 4: the block terms of the gate|up matvec
    for (int r = threadIdx.x; r < nrows; r += blockDim.x) s.sval[r] = row_sum(s.sterm + r * S.tstride, S.nb);
    __syncthreads();
    probe.mark();  // 5: the row chains
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int jb = warp; jb < nrows / 64; jb += kWarps) {
        const float h = swiglu1(s.sval[jb * 64 + lane], s.sval[jb * 64 + 32 + lane], tab);
        const int j = row0 / 64 + jb;
        if (Hf) {  // FLAG_HADAMARD_DOWN: k_fwht_quant transforms and quantizes
            Hf[j * QK + lane] = h;
            continue;
        }
        float d;
        const int8_t q = quantize_lane(h, &d);
        HQ[j * QK + lane] = q;
        if (lane == 0) HD[j] = d;
    }
    probe.end();  // 6: SwiGLU + quantize
}

// ---------------------------------------------------------------- batched (prefill) elementwise kernels

// One CTA per token: rmsnorm + quantize (norm_w != null) or quantize only.
// DXT (optional): the block scales also in block-major order, DXT[b * ldt + t].
__global__ void __launch_bounds__(kThreads) k_norm_quant_rows(const float* __restrict__ X, const float* __restrict__ norm_w,
                                                              int dim, float eps, int8_t* __restrict__ XQ,
                                                              float* __restrict__ DX, float* __restrict__ DXT, int ldt) {
    __shared__ __align__(16) float sred[32 + 2048];
    NormW nw;
    if (norm_w) load_norm_w(norm_w, dim, nw);
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x;
    if (norm_w) norm_quant(X + size_t(t) * dim, nw, dim, eps, XQ + size_t(t) * dim, DX + size_t(t) * (dim / QK), nullptr, sred);
    else quant_only(X + size_t(t) * dim, dim, XQ + size_t(t) * dim, DX + size_t(t) * (dim / QK), nullptr);
    if (DXT) {
        __syncthreads();  // this CTA's scale stores are visible to it
        for (int b = threadIdx.x; b < dim / QK; b += blockDim.x) DXT[size_t(b) * ldt + t] = DX[size_t(t) * (dim / QK) + b];
    }
}

// R [n][fused rows] raw q|k|v -> bias + RoPE + store, token t at position pos0 + t.
__global__ void k_qkv_epilogue(QkvArgs a, const float* __restrict__ R, int n_tok, const int* __restrict__ pos_dev,
                               float* __restrict__ Q, TokMap tm) {
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.y;
    const int pairs = a.W.rows / 2;
    const int pos = tm.pos ? __ldcg(tm.pos + t) : __ldcg(pos_dev) + t;
    if (tm.pos) {  // this token's sequence cache
        const long long off = __ldcg(tm.off + t);
        a.kcache += off;
        a.vcache += off;
    }
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < pairs; p += gridDim.x * blockDim.x)
        qkv_pair_out(a, 2 * p, __ldcg(R + size_t(t) * a.W.rows + 2 * p), __ldcg(R + size_t(t) * a.W.rows + 2 * p + 1), pos,
                     Q + size_t(t) * a.n_heads * a.head_dim);
}

__global__ void k_residual(float* __restrict__ X, const float* __restrict__ R, long long n) {
    pdl_wait();
    pdl_launch_dependents();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        X[i] = fadd(__ldcg(X + i), __ldcg(R + i));
}

// R [n][2*ffn] raw interleaved gate|up -> SwiGLU -> quantize.  One warp per (token, ffn block).
// Hf (files with FLAG_HADAMARD_DOWN): the f32 SwiGLU output goes to Hf[t][ffn] for k_fwht_quant instead.
// One warp per (token, kSwiBlocks consecutive 32-blocks): the warp's gate and up loads are all issued before the
// first SwiGLU, so each warp keeps several L2 requests in flight (one block per warp left it latency-bound).
constexpr int kSwiBlocks = 4;
__global__ void k_swiglu_quant(const float* __restrict__ R, int n_tok, int ffn, int8_t* __restrict__ HQ,
                               float* __restrict__ HD, float* __restrict__ HDT, int ldt, ExpTab tab, float* __restrict__ Hf) {
    pdl_wait();
    pdl_launch_dependents();
    const long long w = blockIdx.x * (long long)(blockDim.x / 32) + (threadIdx.x >> 5);
    const int nbk = ffn / QK, ngr = (nbk + kSwiBlocks - 1) / kSwiBlocks;
    if (w >= (long long)n_tok * ngr) return;
    const int t = int(w / ngr), j0 = int(w - (long long)t * ngr) * kSwiBlocks, lane = threadIdx.x & 31;
    const float* r = R + size_t(t) * 2 * ffn;
    float gv[kSwiBlocks], uv[kSwiBlocks];
#pragma unroll
    for (int k = 0; k < kSwiBlocks; ++k) {
        const int j = j0 + k;
        gv[k] = j < nbk ? __ldcg(r + size_t(j) * 64 + lane) : 0.f;
        uv[k] = j < nbk ? __ldcg(r + size_t(j) * 64 + 32 + lane) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < kSwiBlocks; ++k) {
        const int j = j0 + k;  // uniform across the warp
        if (j >= nbk) break;
        const float h = swiglu1(gv[k], uv[k], tab);
        if (Hf) {
            Hf[size_t(t) * ffn + j * QK + lane] = h;
            continue;
        }
        float d;
        const int8_t q = quantize_lane(h, &d);
        HQ[size_t(t) * ffn + j * QK + lane] = q;
        if (lane == 0) {
            HD[size_t(t) * nbk + j] = d;
            if (HDT) HDT[size_t(j) * ldt + t] = d;
        }
    }
}

// fwht_blocks(h, ffn, 256) (engine/src/ops_ref.cpp:228-241, model.cpp:219,424) then quantize_q8 of the result for the
// down projection.  One warp per (token, 256-block); lane l holds elements [8 l, 8 l + 8).  Stage h pairs element j
// with j + h inside each 2h-block as (a + c, a - c): stages 1, 2, 4 stay inside a lane, stages 8 .. 128 pair lane l
// with lane l ^ (h / 8).  Every butterfly reads the previous stage's two values, so any order of the butterflies of a
// stage gives the reference's bits; the final scale 1 / sqrt(256) = 1/16 is exact.
__global__ void k_fwht_quant(const float* __restrict__ Hf, int n_tok, int ffn, int8_t* __restrict__ HQ,
                             float* __restrict__ HD, float* __restrict__ HDT, int ldt) {
    __shared__ __align__(16) float sv[kWarps][256];
    pdl_wait();
    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long w = blockIdx.x * (long long)kWarps + warp;
    const int nblk = ffn / 256;
    if (w >= (long long)n_tok * nblk) return;
    const int t = int(w / nblk), k = int(w - (long long)t * nblk);
    const float4* src = reinterpret_cast<const float4*>(Hf + size_t(t) * ffn + size_t(k) * 256) + 2 * lane;
    const float4 a0 = __ldcg(src), a1 = __ldcg(src + 1);
    float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
    for (int h = 1; h < 8; h *= 2) {
#pragma unroll
        for (int i = 0; i < 8; i += 2 * h) {
#pragma unroll
            for (int j = i; j < i + h; ++j) {
                const float a = v[j], c = v[j + h];
                v[j] = fadd(a, c);
                v[j + h] = fsub(a, c);
            }
        }
    }
#pragma unroll
    for (int m = 1; m < 32; m *= 2) {  // stage h = 8 m
        const bool upper = (lane & m) != 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float o = __shfl_xor_sync(0xffffffffu, v[j], m);
            v[j] = upper ? fsub(o, v[j]) : fadd(v[j], o);
        }
    }
    float* s = sv[warp];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[8 * lane + j] = fmul(v[j], 0.0625f);
    __syncwarp();
    const int nbk = ffn / QK;
#pragma unroll
    for (int b = 0; b < 8; ++b) {  // the eight 32-blocks of this 256-block
        float d;
        const int8_t q = quantize_lane(s[32 * b + lane], &d);
        const int jb = k * 8 + b;
        HQ[size_t(t) * ffn + jb * QK + lane] = q;
        if (lane == 0) {
            HD[size_t(t) * nbk + jb] = d;
            if (HDT) HDT[size_t(jb) * ldt + t] = d;
        }
    }
}

// ---------------------------------------------------------------- launchers

namespace {

int pick_u(int chunks) {
    const int per = (chunks + kThreads - 1) / kThreads;
    return per <= 1 ? 1 : per <= 2 ? 2 : per <= 4 ? 4 : per <= 8 ? 8 : 16;
}

}  // namespace

SlicePlan plan_rows(int dtype, int rows, int cols, int target_ctas, int row_multiple) {
    SlicePlan p;
    const int cpr = row_bytes_host(dtype, cols) / 16;
    // rows per CTA: the multiple of row_multiple nearest to rows / target_ctas (at least one multiple)
    int rpc = int((double(rows) / target_ctas) / row_multiple + 0.5) * row_multiple;
    if (rpc < row_multiple) rpc = row_multiple;
    while (rpc > row_multiple && rpc * cpr > kThreads * 16) rpc -= row_multiple;
    p.rows_per_cta = rpc;
    p.grid = (rows + rpc - 1) / rpc;
    p.u = pick_u(rpc * cpr);
    p.magic = div_magic(unsigned(cpr));
    p.smem = slice_smem_bytes(cols, rpc);
    return p;
}

#define QB_DISPATCH_U(U, ...)                   \
    switch (U) {                                \
        case 1: { constexpr int UU = 1; __VA_ARGS__; break; }  \
        case 2: { constexpr int UU = 2; __VA_ARGS__; break; }  \
        case 4: { constexpr int UU = 4; __VA_ARGS__; break; }  \
        case 8: { constexpr int UU = 8; __VA_ARGS__; break; }  \
        default: { constexpr int UU = 16; __VA_ARGS__; break; } \
    }

cudaError_t launch_embed(const DMat& E, const int* tokens, int n_tok, float* X, unsigned* status, cudaStream_t st, bool pdl) {
    return launch_pdl(k_embed, dim3(n_tok), dim3(kThreads), 0, st, pdl, E, tokens, n_tok, X, status);
}

cudaError_t launch_qkv_dec(const QkvArgs& a, const SlicePlan& p, const float* X, const float* norm_w, float eps,
                           const int* pos_dev, float* Q, cudaStream_t st, bool pdl) {
    cudaError_t e = cudaErrorInvalidValue;
    if (a.W.dtype == DT_Q8_0) {
        QB_DISPATCH_U(p.u, e = launch_pdl(k_qkv_dec<DT_Q8_0, UU>, dim3(p.grid), dim3(kThreads), p.smem, st, pdl, a, X, norm_w,
                                          eps, pos_dev, Q, p.rows_per_cta, p.magic));
    } else if (a.W.dtype == DT_Q4_0) {
        QB_DISPATCH_U(p.u, e = launch_pdl(k_qkv_dec<DT_Q4_0, UU>, dim3(p.grid), dim3(kThreads), p.smem, st, pdl, a, X, norm_w,
                                          eps, pos_dev, Q, p.rows_per_cta, p.magic));
    }
    return e;
}

cudaError_t launch_resid_dec(const DMat& W, const SlicePlan& p, const float* xin, const int8_t* qin, const float* din,
                             float* X, cudaStream_t st, bool pdl, const float* Xres) {
    cudaError_t e = cudaErrorInvalidValue;
    const bool pre = qin != nullptr;
    if (W.dtype == DT_Q8_0) {
        if (pre) { QB_DISPATCH_U(p.u, e = launch_pdl(k_resid_dec<DT_Q8_0, UU, 1>, dim3(p.grid), dim3(kThreads), p.smem, st, pdl, W, xin, qin, din, X, p.rows_per_cta, p.magic, Xres)); }
        else { QB_DISPATCH_U(p.u, e = launch_pdl(k_resid_dec<DT_Q8_0, UU, 0>, dim3(p.grid), dim3(kThreads), p.smem, st, pdl, W, xin, qin, din, X, p.rows_per_cta, p.magic, Xres)); }
    } else if (W.dtype == DT_Q4_0) {
        if (pre) { QB_DISPATCH_U(p.u, e = launch_pdl(k_resid_dec<DT_Q4_0, UU, 1>, dim3(p.grid), dim3(kThreads), p.smem, st, pdl, W, xin, qin, din, X, p.rows_per_cta, p.magic, Xres)); }
        else { QB_DISPATCH_U(p.u, e = launch_pdl(k_resid_dec<DT_Q4_0, UU, 0>, dim3(p.grid), dim3(kThreads), p.smem, st, pdl, W, xin, qin, din, X, p.rows_per_cta, p.magic, Xres)); }
    }
    return e;
}

namespace {
size_t rt_xn_off(const SlicePlan& p) { return (p.smem + 15) & ~size_t(15); }
}  // namespace

bool gateup_rt_supported(const DMat& W, const SlicePlan& p, int nbo) {
    const int dim = W.cols;
    return (W.dtype == DT_Q8_0 || W.dtype == DT_Q4_0) && p.grid % 8 == 0 && dim % QK == 0 && dim <= kMaxRounds * kThreads &&
           nbo > 0 && nbo % 4 == 0 && nbo <= kRtMaxNb && rt_xn_off(p) + size_t(dim) * 4 <= 227 * 1024;
}

cudaError_t launch_gateup_dec(const DMat& W, const SlicePlan& p, const float* X, const float* norm_w, float eps,
                              int8_t* HQ, float* HD, const ExpTab& tab, cudaStream_t st, bool pdl,
                              const float* T, int nbo, float* X2, float* Hf) {
    cudaError_t e = cudaErrorInvalidValue;
    const int bpc = p.rows_per_cta / 64;
    if (T) {  // residual-terms form: clusters of 8
        if (!gateup_rt_supported(W, p, nbo)) return cudaErrorNotSupported;
        const size_t smem = rt_xn_off(p) + size_t(W.cols) * 4;
        const int xo = int(rt_xn_off(p));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(unsigned(p.grid));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 8;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pdl ? 2 : 1;
        auto go = [&](auto kern) {
            cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
            if (r != cudaSuccess) return r;
            return cudaLaunchKernelEx(&cfg, kern, W, X, norm_w, eps, HQ, HD, bpc, p.magic, tab, T, nbo, X2, xo, Hf);
        };
        if (W.dtype == DT_Q8_0) { QB_DISPATCH_U(p.u, e = go(k_gateup_dec<DT_Q8_0, UU, true>)); }
        else { QB_DISPATCH_U(p.u, e = go(k_gateup_dec<DT_Q4_0, UU, true>)); }
        return e;
    }
    if (W.dtype == DT_Q8_0) {
        QB_DISPATCH_U(p.u, e = launch_pdl(k_gateup_dec<DT_Q8_0, UU, false>, dim3(p.grid), dim3(kThreads), p.smem, st, pdl, W, X,
                                          norm_w, eps, HQ, HD, bpc, p.magic, tab, static_cast<const float*>(nullptr), 0,
                                          static_cast<float*>(nullptr), 0, Hf));
    } else if (W.dtype == DT_Q4_0) {
        QB_DISPATCH_U(p.u, e = launch_pdl(k_gateup_dec<DT_Q4_0, UU, false>, dim3(p.grid), dim3(kThreads), p.smem, st, pdl, W, X,
                                          norm_w, eps, HQ, HD, bpc, p.magic, tab, static_cast<const float*>(nullptr), 0,
                                          static_cast<float*>(nullptr), 0, Hf));
    }
    return e;
}

QNT_PHASE_READER(qnt_phase_read_layers)

cudaError_t launch_norm_quant_rows(const float* X, const float* norm_w, int n_tok, int dim, float eps, int8_t* XQ, float* DX,
                                   float* DXT, int ldt, cudaStream_t st, bool pdl) {
    return launch_pdl(k_norm_quant_rows, dim3(n_tok), dim3(kThreads), 0, st, pdl, X, norm_w, dim, eps, XQ, DX, DXT, ldt);
}

cudaError_t launch_qkv_epilogue(const QkvArgs& a, const float* R, int n_tok, const int* pos_dev, float* Q, cudaStream_t st,
                                bool pdl, TokMap tm) {
    const int pairs = a.W.rows / 2;
    return launch_pdl(k_qkv_epilogue, dim3((pairs + kThreads - 1) / kThreads, n_tok), dim3(kThreads), 0, st, pdl, a, R, n_tok,
                      pos_dev, Q, tm);
}

cudaError_t launch_residual(float* X, const float* R, long long n, cudaStream_t st, bool pdl) {
    const int grid = int(std::min<long long>((n + kThreads - 1) / kThreads, 1184));
    return launch_pdl(k_residual, dim3(grid), dim3(kThreads), 0, st, pdl, X, R, n);
}

cudaError_t launch_swiglu_quant(const float* R, int n_tok, int ffn, int8_t* HQ, float* HD, float* HDT, int ldt, const ExpTab& tab,
                                cudaStream_t st, bool pdl, float* Hf) {
    const long long warps = (long long)n_tok * ((ffn / QK + kSwiBlocks - 1) / kSwiBlocks);
    return launch_pdl(k_swiglu_quant, dim3(unsigned((warps + kWarps - 1) / kWarps)), dim3(kThreads), 0, st, pdl, R, n_tok, ffn, HQ, HD,
                      HDT, ldt, tab, Hf);
}

cudaError_t launch_fwht_quant(const float* Hf, int n_tok, int ffn, int8_t* HQ, float* HD, float* HDT, int ldt, cudaStream_t st,
                              bool pdl) {
    if (ffn % 256 != 0) return cudaErrorInvalidValue;
    const long long warps = (long long)n_tok * (ffn / 256);
    return launch_pdl(k_fwht_quant, dim3(unsigned((warps + kWarps - 1) / kWarps)), dim3(kThreads), 0, st, pdl, Hf, n_tok, ffn, HQ, HD,
                      HDT, ldt);
}

}  // namespace qb
