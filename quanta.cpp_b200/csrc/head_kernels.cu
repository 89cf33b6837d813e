// Output head and sampling on the device.
//
// Full head (engine/src/model.cpp:230-238): the Q8 lm_head matvec over every vocab row.
// Exact Shortlist Head (engine/src/model.cpp:240-334), three kernels with the same semantics:
//   k_sl_coarse  4-bit score c_r of every row (same integer matvec on quanta.head_q4), the Cauchy-Schwarz bound
//                B_r = (sum_b err[r,b] * |x_b|) * 1.001 + 1e-5, upper_r = c_r + B_r, logits = -inf, and each CTA's
//                best k+8 coarse scores among valid non-`must` rows;
//   k_sl_seeds   merges those into the global k+8 seeds, rescores them exactly (Q8 rows) and takes tau = the k-th
//                best exact seed;
//   k_sl_cands   rescores exactly every valid row with upper >= tau that is not a seed or a must id, plus the must
//                ids, and clears the marks.
// Exact rows use the same block-sequential arithmetic as the full head, so their logits are bit-identical to it.
//
// Sampler (engine/src/sampler.cpp:22-85): repetition penalty on the history's unique ids, then greedy argmax
// (first max) or top-k (ties to the lower id) -> temperature softmax -> min-p -> top-p -> xorshift64* draw.
#include <climits>

#include "head_kernels.h"
#include "kernels.cuh"

namespace qb {

// ---------------------------------------------------------------- warp top-K lists (K <= 32)

struct Cand {
    float v;
    int id;
};

__device__ __forceinline__ bool better(float av, int aid, float bv, int bid) {
    return av > bv || (av == bv && aid < bid);
}

// Sorted list, lane i holds the i-th best (lanes >= K hold sentinels).
struct WarpTopK {
    float v;
    int id;
    __device__ void init() {
        v = -INFINITY;
        id = INT_MAX;
    }
    // Offer one candidate per lane (valid lanes only); K <= 32.
    __device__ void offer(float cv, int cid, bool valid, int K) {
        const int lane = threadIdx.x & 31;
        float tv = __shfl_sync(0xffffffffu, v, K - 1);
        int tid = __shfl_sync(0xffffffffu, id, K - 1);
        unsigned m = __ballot_sync(0xffffffffu, valid && better(cv, cid, tv, tid));
        while (m) {
            const int src = __ffs(m) - 1;
            m &= m - 1;
            const float xv = __shfl_sync(0xffffffffu, cv, src);
            const int xid = __shfl_sync(0xffffffffu, cid, src);
            if (!better(xv, xid, tv, tid)) continue;  // threshold moved up meanwhile
            const unsigned ahead = __ballot_sync(0xffffffffu, lane < K && better(v, id, xv, xid));
            const int p = __popc(ahead);
            const float uv = __shfl_up_sync(0xffffffffu, v, 1);
            const int uid = __shfl_up_sync(0xffffffffu, id, 1);
            if (lane > p && lane < K) {
                v = uv;
                id = uid;
            } else if (lane == p) {
                v = xv;
                id = xid;
            }
            tv = __shfl_sync(0xffffffffu, v, K - 1);
            tid = __shfl_sync(0xffffffffu, id, K - 1);
        }
    }
};

// Merges the CTA's per-warp lists into warp 0's list (written to slist[0..K)).
__device__ void cta_merge_lists(WarpTopK& L, int K, Cand* slist /* [kWarps][32] */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    slist[warp * 32 + lane] = Cand{L.v, L.id};
    __syncthreads();
    if (warp == 0) {
        for (int w = 1; w < nw; ++w) {
            const Cand c = slist[w * 32 + lane];
            L.offer(c.v, c.id, lane < K && c.id != INT_MAX, K);
        }
        slist[lane] = Cand{L.v, L.id};
    }
    __syncthreads();
}

// ---------------------------------------------------------------- head input

// rmsnorm(x, final_norm) + quantize (engine/src/model.cpp:225-226), plus the per-block |x_b| = d_b * sqrt(sum q^2)
// the shortlist bound needs (model.cpp:247-251; the int8 squares sum exactly in float).
__global__ void __launch_bounds__(kThreads) k_head_input(const float* __restrict__ X, const float* __restrict__ norm_w, int dim,
                                                         float eps, HeadIn hin, HeadState* hs, int full_rows) {
    __shared__ float sred[32];
    __shared__ int8_t sx[8192];
    __shared__ float sdx[256];
    __shared__ int ssum[256];
    pdl_launch_dependents();
    pdl_wait();
    norm_quant(X, norm_w, dim, eps, sx, sdx, ssum, sred);
    if (threadIdx.x == 0 && hs) {
        hs->rows_total += hs->calls ? hs->rows : 0;
        hs->calls += 1;
        hs->rows = full_rows;
    }
    for (int i = threadIdx.x; i < dim; i += blockDim.x) hin.xq[i] = sx[i];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int b = warp; b < dim / QK; b += kWarps) {
        const float q = float(sx[b * QK + lane]);
        // exact: integers below 2^24, any order
        float ss = fmul(q, q);
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) {
            hin.dx[b] = sdx[b];
            hin.xsum[b] = ssum[b];
            hin.xnorm[b] = fmul(sdx[b], __fsqrt_rn(ss));
        }
    }
}

// ---------------------------------------------------------------- full head

template <int DT, int U>
__global__ void __launch_bounds__(kThreads) k_head_rows(DMat W, HeadIn hin, int rows_per_cta, unsigned magic,
                                                        float* __restrict__ logits) {
    extern __shared__ __align__(16) unsigned char smem[];
    pdl_launch_dependents();
    const int cols = W.cols, nb = cols / QK;
    int8_t* sx = reinterpret_cast<int8_t*>(smem);
    float* sdx = reinterpret_cast<float*>(smem + cols);
    int* ssum = reinterpret_cast<int*>(sdx + nb);
    float* sterm = reinterpret_cast<float*>(ssum + nb);
    const int row0 = blockIdx.x * rows_per_cta, nrows = min(rows_per_cta, W.rows - row0);
    if (nrows <= 0) return;
    RowSlice S;
    const int rb = row_bytes(DT, cols);
    S.wq = W.q + size_t(row0) * rb;
    S.wd = W.d + size_t(row0) * nb;
    S.nrows = nrows;
    S.nb = nb;
    S.cpr = rb / 16;
    S.cpr_magic = magic;
    S.tstride = term_stride(nb);
    slice_terms<DT, U>(S, sx, sdx, ssum, sterm, [&] {
        pdl_wait();
        for (int i = threadIdx.x; i < cols / 16; i += blockDim.x)
            reinterpret_cast<int4*>(sx)[i] = reinterpret_cast<const int4*>(hin.xq)[i];
        for (int b = threadIdx.x; b < nb; b += blockDim.x) {
            sdx[b] = hin.dx[b];
            ssum[b] = hin.xsum[b];
        }
        __syncthreads();
    });
    __syncthreads();
    for (int r = threadIdx.x; r < nrows; r += blockDim.x) logits[row0 + r] = row_sum(sterm + r * S.tstride, nb);
}

// Exact Q8 logit of one row computed by one warp, same terms and order as k_head_rows.  wterm: nb floats per warp.
__device__ __forceinline__ float warp_exact_row(const DMat& W, int row, const int8_t* sx, const float* sdx, float* wterm) {
    const int lane = threadIdx.x & 31, cols = W.cols, nb = cols / QK, cpr = cols / 16;
    const uint4* src = reinterpret_cast<const uint4*>(W.q + size_t(row) * cols);
    for (int c0 = 0; c0 < cpr; c0 += 32) {
        const int c = c0 + lane;
        int s = 0;
        __half dw = __float2half(0.f);
        if (c < cpr) {
            s = chunk_dot<DT_Q8_0>(ld_stream(src + c), sx, c);
            dw = W.d[size_t(row) * nb + (c >> 1)];
        }
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        if (c < cpr && !(c & 1)) wterm[c >> 1] = block_term(s, __half2float(dw), sdx[c >> 1]);
    }
    __syncwarp();
    float acc = 0.f;
    if (lane == 0) acc = row_sum(wterm, nb);
    __syncwarp();
    return __shfl_sync(0xffffffffu, acc, 0);
}

// ---------------------------------------------------------------- shortlist head

// Marks the must ids: mark[id] = 1 for 0 <= id < n_valid (model.cpp:252-253).
__global__ void k_sl_mark(const int* __restrict__ must, const int* __restrict__ n_must_dev, int n_must_host, int window,
                          int n_valid, unsigned char* __restrict__ mark) {
    pdl_launch_dependents();
    pdl_wait();
    int n = n_must_dev ? *n_must_dev : n_must_host;
    int from = 0;
    if (window > 0 && n > window) from = n - window;
    for (int i = from + blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int id = must[i];
        if (id >= 0 && id < n_valid) mark[id] = 1;
    }
}

template <int U>
__global__ void __launch_bounds__(kThreads) k_sl_coarse(DMat W4, const __half* __restrict__ err, HeadIn hin, int rows_per_tile,
                                                        unsigned magic, int n_valid, int n_seed,
                                                        const unsigned char* __restrict__ mark, float* __restrict__ coarse,
                                                        float* __restrict__ upper, float* __restrict__ logits,
                                                        Cand* __restrict__ seed_buf) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ Cand slist[kWarps * 32];
    pdl_launch_dependents();
    const int cols = W4.cols, nb = cols / QK;
    int8_t* sx = reinterpret_cast<int8_t*>(smem);
    float* sdx = reinterpret_cast<float*>(smem + cols);
    int* ssum = reinterpret_cast<int*>(sdx + nb);
    float* sxn = reinterpret_cast<float*>(ssum + nb);
    float* sterm = sxn + nb;
    WarpTopK L;
    L.init();
    const int n_tiles = (W4.rows + rows_per_tile - 1) / rows_per_tile;
    bool first = true;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        const int row0 = tile * rows_per_tile, nrows = min(rows_per_tile, W4.rows - row0);
        RowSlice S;
        const int rb = cols / 2;
        S.wq = W4.q + size_t(row0) * rb;
        S.wd = W4.d + size_t(row0) * nb;
        S.nrows = nrows;
        S.nb = nb;
        S.cpr = rb / 16;
        S.cpr_magic = magic;
        S.tstride = term_stride(nb);
        __syncthreads();  // previous tile's terms consumed
        slice_terms<DT_Q4_0, U>(S, sx, sdx, ssum, sterm, [&] {
            if (!first) return;
            pdl_wait();
            for (int i = threadIdx.x; i < cols / 16; i += blockDim.x)
                reinterpret_cast<int4*>(sx)[i] = reinterpret_cast<const int4*>(hin.xq)[i];
            for (int b = threadIdx.x; b < nb; b += blockDim.x) {
                sdx[b] = hin.dx[b];
                ssum[b] = hin.xsum[b];
                sxn[b] = hin.xnorm[b];
            }
            __syncthreads();
        });
        first = false;
        __syncthreads();
        for (int base = 0; base < nrows; base += blockDim.x) {
            const int r = base + threadIdx.x;
            float cv = -INFINITY;
            int row = INT_MAX;
            bool ok = false;
            if (r < nrows) {
                row = row0 + r;
                cv = row_sum(sterm + r * S.tstride, nb);
                const __half* e = err + size_t(row) * nb;
                float bound = 0.f;
                for (int b = 0; b < nb; ++b) bound = fadd(bound, fmul(__half2float(e[b]), sxn[b]));
                bound = fadd(fmul(bound, 1.001f), 1e-5f);
                coarse[row] = cv;
                upper[row] = fadd(cv, bound);
                logits[row] = -INFINITY;
                ok = row < n_valid && mark[row] == 0;
            }
            L.offer(cv, row, ok, n_seed);
        }
    }
    if (first) pdl_wait();
    cta_merge_lists(L, n_seed, slist);
    if (threadIdx.x < n_seed) seed_buf[size_t(blockIdx.x) * n_seed + threadIdx.x] = slist[threadIdx.x];
}

// One CTA: global seeds, their exact logits, tau.
__global__ void __launch_bounds__(kThreads) k_sl_seeds(DMat W8, HeadIn hin, const Cand* __restrict__ seed_buf, int n_lists,
                                                       int n_seed, int k, unsigned char* __restrict__ mark,
                                                       float* __restrict__ logits, HeadState* __restrict__ hs) {
    __shared__ Cand slist[kWarps * 32];
    __shared__ __align__(16) int8_t sx[8192];
    __shared__ float sdx[256];
    __shared__ float wterm[kWarps][256];
    __shared__ Cand seeds[32];
    __shared__ float exact[32];
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cols = W8.cols, nb = cols / QK;
    for (int i = threadIdx.x; i < cols / 16; i += blockDim.x)
        reinterpret_cast<int4*>(sx)[i] = reinterpret_cast<const int4*>(hin.xq)[i];
    for (int b = threadIdx.x; b < nb; b += blockDim.x) sdx[b] = hin.dx[b];
    WarpTopK L;
    L.init();
    const int total = n_lists * n_seed;
    for (int base = warp * 32; base < total; base += blockDim.x) {
        const int i = base + lane;
        Cand c{-INFINITY, INT_MAX};
        if (i < total) c = seed_buf[i];
        L.offer(c.v, c.id, i < total && c.id != INT_MAX, n_seed);
    }
    cta_merge_lists(L, n_seed, slist);
    if (threadIdx.x < 32) seeds[threadIdx.x] = slist[threadIdx.x];
    __syncthreads();
    int ns = 0;
    while (ns < n_seed && seeds[ns].id != INT_MAX) ++ns;
    for (int s = warp; s < ns; s += kWarps) {
        const float v = warp_exact_row(W8, seeds[s].id, sx, sdx, wterm[warp]);
        if (lane == 0) {
            exact[s] = v;
            logits[seeds[s].id] = v;
            mark[seeds[s].id] = 2;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        // tau = k-th largest exact seed logit (model.cpp:308-313); insertion sort of <= 32 values, descending
        for (int i = 1; i < ns; ++i) {
            const float v = exact[i];
            int j = i - 1;
            while (j >= 0 && exact[j] < v) {
                exact[j + 1] = exact[j];
                --j;
            }
            exact[j + 1] = v;
        }
        const float tau = ns >= k ? exact[k - 1] : -INFINITY;
        hs->tau = tau;
        hs->rows = ns;
    }
}

// Candidate scan + exact rescoring of candidates and must ids; clears marks.  One warp per 32 rows at a time.
__global__ void __launch_bounds__(kThreads) k_sl_cands(DMat W8, HeadIn hin, int n_valid, unsigned char* __restrict__ mark,
                                                       const float* __restrict__ upper, float* __restrict__ logits,
                                                       HeadState* __restrict__ hs) {
    __shared__ __align__(16) int8_t sx[8192];
    __shared__ float sdx[256];
    __shared__ float wterm[kWarps][256];
    __shared__ int scount;
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cols = W8.cols, nb = cols / QK;
    for (int i = threadIdx.x; i < cols / 16; i += blockDim.x)
        reinterpret_cast<int4*>(sx)[i] = reinterpret_cast<const int4*>(hin.xq)[i];
    for (int b = threadIdx.x; b < nb; b += blockDim.x) sdx[b] = hin.dx[b];
    if (threadIdx.x == 0) scount = 0;
    __syncthreads();
    const float tau = hs->tau;
    int mine = 0;
    const int nwarps_total = gridDim.x * kWarps;
    for (int base = (blockIdx.x * kWarps + warp) * 32; base < W8.rows; base += nwarps_total * 32) {
        const int r = base + lane;
        bool want = false;
        if (r < W8.rows) {
            const unsigned char mk = mark[r];
            if (r < n_valid) want = mk == 1 || (mk == 0 && upper[r] >= tau);
            if (mk) mark[r] = 0;
        }
        unsigned m = __ballot_sync(0xffffffffu, want);
        mine += __popc(m);
        while (m) {
            const int src = __ffs(m) - 1;
            m &= m - 1;
            const int row = base + src;
            const float v = warp_exact_row(W8, row, sx, sdx, wterm[warp]);
            if (lane == 0) logits[row] = v;
        }
    }
    if (lane == 0) atomicAdd(&scount, mine);
    __syncthreads();
    if (threadIdx.x == 0 && scount) atomicAdd(&hs->rows, scount);
}

// ---------------------------------------------------------------- sampler

// Repetition penalty on the unique ids of history[from..n) (sampler.cpp:23-33); one CTA.  flag: V bytes, all zero.
__global__ void k_penalty(float* __restrict__ logits, int n_valid, const int* __restrict__ hist,
                          const int* __restrict__ n_hist_dev, int window, float penalty, unsigned* __restrict__ flag) {
    pdl_launch_dependents();
    pdl_wait();
    const int n = *n_hist_dev;
    const int from = (window > 0 && n > window) ? n - window : 0;
    for (int i = from + threadIdx.x; i < n; i += blockDim.x) {
        const int id = hist[i];
        if (id < 0 || id >= n_valid) continue;
        if (atomicExch(&flag[id], 1u) == 0u) {
            const float l = logits[id];
            logits[id] = l > 0.f ? fdiv(l, penalty) : fmul(l, penalty);
        }
    }
    __syncthreads();
    for (int i = from + threadIdx.x; i < n; i += blockDim.x) {
        const int id = hist[i];
        if (id >= 0 && id < n_valid) flag[id] = 0u;
    }
}

// Stage 1: each CTA's best K of logits[0, n_valid).
__global__ void __launch_bounds__(kThreads) k_topk_partial(const float* __restrict__ logits, int n_valid, int K,
                                                           Cand* __restrict__ out) {
    __shared__ Cand slist[kWarps * 32];
    pdl_launch_dependents();
    pdl_wait();
    WarpTopK L;
    L.init();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int per = (n_valid + gridDim.x - 1) / gridDim.x;
    const int r0 = blockIdx.x * per, r1 = min(n_valid, r0 + per);
    for (int base = r0 + warp * 32; base < r1; base += blockDim.x) {
        const int r = base + lane;
        const bool ok = r < r1;
        L.offer(ok ? logits[r] : -INFINITY, ok ? r : INT_MAX, ok, K);
    }
    cta_merge_lists(L, K, slist);
    if (threadIdx.x < K) out[size_t(blockIdx.x) * K + threadIdx.x] = slist[threadIdx.x];
}

__device__ __forceinline__ uint64_t xorshift64s(uint64_t& s) {
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    return s * 0x2545F4914F6CDD1DULL;
}

// Stage 2 (one CTA): merge, then greedy pick or softmax/min-p/top-p draw; appends the token to the history and
// advances the position.  Writes the chosen id to *token_out.
__global__ void __launch_bounds__(kThreads) k_sample_final(const Cand* __restrict__ parts, int n_lists, int K, SamplerArgs sa,
                                                           SamplerState* __restrict__ ss, int* __restrict__ hist,
                                                           int hist_cap) {
    __shared__ Cand slist[kWarps * 32];
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    WarpTopK L;
    L.init();
    const int total = n_lists * K;
    for (int base = warp * 32; base < total; base += blockDim.x) {
        const int i = base + lane;
        Cand c{-INFINITY, INT_MAX};
        if (i < total) c = parts[i];
        L.offer(c.v, c.id, i < total && c.id != INT_MAX, K);
    }
    cta_merge_lists(L, K, slist);
    if (threadIdx.x != 0) return;
    int n = 0;
    while (n < K && slist[n].id != INT_MAX) ++n;
    int pick = n > 0 ? slist[0].id : 0;
    if (sa.temperature > 0.f && n > 0) {
        float p[32];
        const float mx = slist[0].v;
        float sum = 0.f;
        for (int i = 0; i < n; ++i) {
            p[i] = expf(fdiv(fsub(slist[i].v, mx), sa.temperature));
            sum = fadd(sum, p[i]);
        }
        for (int i = 0; i < n; ++i) p[i] = fdiv(p[i], sum);
        int keep = n;
        if (sa.min_p > 0.f) {
            const float floor = fmul(p[0], sa.min_p);
            while (keep > 1 && p[keep - 1] < floor) --keep;
        }
        if (sa.top_p < 1.f) {
            float cum = 0.f;
            for (int i = 0; i < keep; ++i) {
                cum = fadd(cum, p[i]);
                if (cum >= sa.top_p) {
                    keep = i + 1;
                    break;
                }
            }
        }
        float total_p = 0.f;
        for (int i = 0; i < keep; ++i) total_p = fadd(total_p, p[i]);
        uint64_t st = ss->rng;
        const float u = fmul(float(xorshift64s(st) >> 40), 1.0f / 16777216.0f);
        ss->rng = st;
        float r = fmul(u, total_p);
        pick = slist[keep - 1].id;
        for (int i = 0; i < keep; ++i) {
            r = fsub(r, p[i]);
            if (r <= 0.f) {
                pick = slist[i].id;
                break;
            }
        }
    }
    ss->token = pick;
    if (sa.append) {
        const int nh = ss->n_hist;
        if (nh < hist_cap) {
            hist[nh] = pick;
            ss->n_hist = nh + 1;
            ss->pos = nh;  // the new token is fed at position len(history) - 1
        }
    }
}

// ---------------------------------------------------------------- launchers

namespace {

template <class... KArgs, class... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
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

}  // namespace

HeadPlan plan_head(int dtype, int rows, int cols) {
    HeadPlan p;
    const int cpr = row_bytes_host(dtype, cols) / 16;
    // ~1024 chunks (16 KB of weights) per CTA, U = 4
    int rpc = std::max(2, (kThreads * 4) / cpr) & ~1;
    p.rows_per_cta = rpc;
    p.grid = (rows + rpc - 1) / rpc;
    p.u = 4;
    p.magic = div_magic(unsigned(cpr));
    const int nb = cols / QK;
    p.smem = size_t(cols) + size_t(nb) * 12 + size_t(rpc) * (nb | 1) * 4;
    return p;
}

cudaError_t launch_head_input(const float* X, const float* norm_w, int dim, float eps, const HeadIn& hin, HeadState* hs,
                              int full_rows, cudaStream_t st, bool pdl) {
    if (dim > 8192) return cudaErrorInvalidValue;
    return launch_pdl(k_head_input, dim3(1), dim3(kThreads), 0, st, pdl, X, norm_w, dim, eps, hin, hs, full_rows);
}

cudaError_t launch_head_full(const DMat& W, const HeadPlan& p, const HeadIn& hin, float* logits, cudaStream_t st, bool pdl) {
    if (W.dtype == DT_Q8_0)
        return launch_pdl(k_head_rows<DT_Q8_0, 4>, dim3(p.grid), dim3(kThreads), p.smem, st, pdl, W, hin, p.rows_per_cta, p.magic,
                          logits);
    if (W.dtype == DT_Q4_0)
        return launch_pdl(k_head_rows<DT_Q4_0, 4>, dim3(p.grid), dim3(kThreads), p.smem, st, pdl, W, hin, p.rows_per_cta, p.magic,
                          logits);
    return cudaErrorInvalidValue;
}

cudaError_t launch_shortlist(const ShortlistArgs& a, const HeadIn& hin, cudaStream_t st, bool pdl) {
    const int n_seed = a.k + 8;
    if (a.k < 1 || n_seed > 32 || a.W8.cols > 8192) return cudaErrorInvalidValue;
    cudaError_t e = launch_pdl(k_sl_mark, dim3(4), dim3(kThreads), 0, st, pdl, a.must, a.n_must_dev, a.n_must_host, a.window,
                               a.n_valid, a.mark);
    if (e != cudaSuccess) return e;
    e = launch_pdl(k_sl_coarse<4>, dim3(a.coarse_ctas), dim3(kThreads), a.plan4.smem, st, pdl, a.W4, a.err, hin,
                   a.plan4.rows_per_cta, a.plan4.magic, a.n_valid, n_seed, (const unsigned char*)a.mark, a.coarse, a.upper,
                   a.logits, reinterpret_cast<Cand*>(a.seed_buf));
    if (e != cudaSuccess) return e;
    e = launch_pdl(k_sl_seeds, dim3(1), dim3(kThreads), 0, st, pdl, a.W8, hin, (const Cand*)reinterpret_cast<Cand*>(a.seed_buf),
                   a.coarse_ctas, n_seed, a.k, a.mark, a.logits, a.hs);
    if (e != cudaSuccess) return e;
    return launch_pdl(k_sl_cands, dim3(a.cand_ctas), dim3(kThreads), 0, st, pdl, a.W8, hin, a.n_valid, a.mark,
                      (const float*)a.upper, a.logits, a.hs);
}

cudaError_t launch_sampler(const SamplerLaunch& s, cudaStream_t st, bool pdl) {
    if (s.K < 1 || s.K > 32) return cudaErrorInvalidValue;
    cudaError_t e;
    if (s.args.repeat_penalty != 1.0f) {
        e = launch_pdl(k_penalty, dim3(1), dim3(1024), 0, st, pdl, s.logits, s.n_valid, (const int*)s.hist,
                       (const int*)s.n_hist_dev, s.window, s.args.repeat_penalty, s.flag);
        if (e != cudaSuccess) return e;
    }
    e = launch_pdl(k_topk_partial, dim3(s.parts), dim3(kThreads), 0, st, pdl, (const float*)s.logits, s.n_valid, s.K,
                   reinterpret_cast<Cand*>(s.part_buf));
    if (e != cudaSuccess) return e;
    return launch_pdl(k_sample_final, dim3(1), dim3(kThreads), 0, st, pdl, (const Cand*)reinterpret_cast<Cand*>(s.part_buf),
                      s.parts, s.K, s.args, s.state, s.hist, s.hist_cap);
}

}  // namespace qb
