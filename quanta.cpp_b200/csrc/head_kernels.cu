// Output head and sampling on the device.
//
// Full head (engine/src/model.cpp:230-238): the Q8 lm_head matvec over every vocab row.
// Exact Shortlist Head (engine/src/model.cpp:240-334):
//   k_sl_mark     mark[id] = 1 for the must ids (model.cpp:252-253)
//   k_head_stream coarse mode: the 4-bit score c_r of every row (same integer matvec on quanta.head_q4), the bound
//                 B_r = (sum_b err[r,b] * |x_b|) * 1.001 + 1e-5, upper_r = c_r + B_r, logits = -inf, and each
//                 CTA's best k+8 coarse scores among valid non-must rows (model.cpp:259-284)
//   k_sl_seeds    the global k+8 seeds, their exact Q8 logits, tau = the k-th best exact seed (model.cpp:293-313)
//   k_sl_cands    exact logits of every valid row with upper >= tau that is neither seed nor must, plus the must
//                 rows (model.cpp:315-332); clears the marks
// Exact rows use the same block-sequential arithmetic as the full head, so their logits are bit-identical to it.
//
// The big passes (full head: 145 MB of Q8 rows; coarse: 77 MB of Q4 rows + 8.5 MB of bounds) stream their rows
// through a shared-memory ring filled by cp.async (16-byte async copies, several tiles in flight per SM), one
// persistent CTA per SM.
//
// Sampler (engine/src/sampler.cpp:22-85).  Stage 1 -- each CTA's best K candidates after the repetition penalty
// (the unique history ids, marked in `mark`) -- is fused into whichever head kernel finishes the exact logits; stage 2
// (k_sample_final) merges the lists and draws: greedy = first max, else top-k (ties to the lower id) -> softmax(T) ->
// min-p -> top-p -> xorshift64*.
#include <climits>

#include "phase_stamps.cuh"
#include "head_kernels.h"
#include "kernels.cuh"

namespace qb {

constexpr int kHeadThreads = 512;
// Head passes: a tile of head_tile_rows rows per pipeline stage, kRowParts threads per row (a warp covers 8 rows).
constexpr int kRowParts = 4;
constexpr int kMaxBpp = 16;  // blocks per part: cols <= kRowParts * kMaxBpp * 32 (kernels instantiated for 8 and 16)
__host__ __device__ constexpr int head_tile_rows(int dtype) { return dtype == DT_Q4_0 ? 128 : 64; }
__host__ __device__ constexpr int head_threads(int dtype) { return head_tile_rows(dtype) * kRowParts; }
// The coarse Q4 pass may take tiles of 176 rows (22 warps): for the 0.5B vocabulary over 148 CTAs that is at most 6 tiles
// of 176 rows per CTA (1056 row slots) instead of 9 of 128 (1152), with more warps per SM to hide latency.
constexpr int kWideTileRows = 176;
constexpr int kHeadWarps = kHeadThreads / 32;

// ---------------------------------------------------------------- candidate lists (K <= 32), kept with bitonic networks

__device__ __forceinline__ bool better(float av, int aid, float bv, int bid) {
    return av > bv || (av == bv && aid < bid);
}

// ---- merging sorted candidate lists (K <= 32, best first, sentinels {-inf, INT_MAX} past the valid entries)

// Sorts a bitonic warp-wide sequence (one candidate per lane) best-first: five half-cleaner stages over shuffles.
__device__ __forceinline__ void warp_bitonic_to_sorted(float& v, int& id) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
        const float pv = __shfl_xor_sync(0xffffffffu, v, s);
        const int pid = __shfl_xor_sync(0xffffffffu, id, s);
        const bool keep_better = (lane & s) == 0;
        if (keep_better == better(pv, pid, v, id)) {
            v = pv;
            id = pid;
        }
    }
}

// (v, id) and (bv, bid) are warp-wide lists sorted best-first; leaves the best 32 of their union in (v, id), sorted.
// The lane-wise better of A and reversed B is bitonic and holds the top 32 of A u B.
__device__ __forceinline__ void warp_merge_top(float& v, int& id, float bv, int bid) {
    const int lane = threadIdx.x & 31;
    const float rv = __shfl_sync(0xffffffffu, bv, 31 - lane);
    const int rid = __shfl_sync(0xffffffffu, bid, 31 - lane);
    if (better(rv, rid, v, id)) {
        v = rv;
        id = rid;
    }
    warp_bitonic_to_sorted(v, id);
}

// Sorts one candidate per lane best-first (bitonic sorting network over shuffles).
__device__ __forceinline__ void warp_bitonic_sort(float& v, int& id) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const float pv = __shfl_xor_sync(0xffffffffu, v, j);
            const int pid = __shfl_xor_sync(0xffffffffu, id, j);
            const bool keep_better = ((lane & j) == 0) == ((lane & k) == 0);  // k-blocks alternate best-first / worst-first
            if (keep_better == better(pv, pid, v, id)) {
                v = pv;
                id = pid;
            }
        }
    }
}

// A warp's running list: lane i holds the i-th best candidate so far (sentinels {-inf, INT_MAX} past the filled part).
struct WarpTop32 {
    float v;
    int id;
    __device__ void init() {
        v = -INFINITY;
        id = INT_MAX;
    }
    // One candidate per lane (valid lanes only).  Candidates that do not beat the current K-th best cannot enter the
    // final best K; the others are sorted and merged in (the list keeps the best 32, a superset of the best K).
    __device__ void offer(float cv, int cid, bool valid, int K) {
        const float tv = __shfl_sync(0xffffffffu, v, K - 1);
        const int tid = __shfl_sync(0xffffffffu, id, K - 1);
        const bool beat = valid && better(cv, cid, tv, tid);
        if (__any_sync(0xffffffffu, beat)) {
            float nv = beat ? cv : -INFINITY;
            int nid = beat ? cid : INT_MAX;
            warp_bitonic_sort(nv, nid);
            warp_merge_top(v, id, nv, nid);
        }
    }
};

// Merges the CTA's warp lists into slist[0..32), best first, sentinels past K.  slist: (blockDim / 32) * 32 entries.
// Each level folds the upper half of the n live lists onto the lower (n odd: the middle list waits a level).
__device__ void cta_merge_lists(WarpTop32& L, int K, Cand* slist) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    slist[warp * 32 + lane] = Cand{L.v, L.id};
    __syncthreads();
    for (int n = int(blockDim.x >> 5); n > 1;) {
        const int half = (n + 1) >> 1;
        if (warp < n - half) {
            const Cand c = slist[(warp + half) * 32 + lane];
            warp_merge_top(L.v, L.id, c.v, c.id);
            slist[warp * 32 + lane] = Cand{L.v, L.id};
        }
        __syncthreads();
        n = half;
    }
    if (warp == 0 && lane >= K) slist[lane] = Cand{-INFINITY, INT_MAX};
    __syncthreads();
}

// Best K of n_lists sorted lists of K candidates each (global memory, written by other kernels) into slist[0..32),
// best first.  Each warp merges its share of the lists in registers, then a tree over the warps' results.
// slist: (blockDim / 32) * 32 entries; blockDim / 32 a power of two.
__device__ void cta_merge_sorted(const Cand* __restrict__ src, int n_lists, int K, Cand* slist) {
    constexpr int kBatch = 10;  // 16 warps x 10 lists cover the 148 lists of one stream pass in one round of loads
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float v = -INFINITY, v2 = -INFINITY;  // two independent merge chains (even / odd batch slots), merged at the end
    int id = INT_MAX, id2 = INT_MAX;
    for (int l0 = warp; l0 < n_lists; l0 += kBatch * nw) {
        float bv[kBatch];
        int bid[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {  // loads first: one list per batch slot
            const int l = l0 + u * nw;
            const bool ok = l < n_lists && lane < K;
            const float2 c = ok ? __ldcg(reinterpret_cast<const float2*>(src + size_t(l) * K + lane))
                                : make_float2(-INFINITY, __int_as_float(INT_MAX));  // (v, id) in one 8-byte load
            bv[u] = c.x;
            bid[u] = __float_as_int(c.y);
        }
#pragma unroll
        for (int u = 0; u < kBatch; u += 2) {
            if (l0 + u * nw < n_lists) warp_merge_top(v, id, bv[u], bid[u]);
            if (l0 + (u + 1) * nw < n_lists) warp_merge_top(v2, id2, bv[u + 1], bid[u + 1]);
        }
    }
    warp_merge_top(v, id, v2, id2);  // the top 32 of a union do not depend on the order of the merges
    slist[warp * 32 + lane] = Cand{v, id};
    __syncthreads();
    for (int half = nw / 2; half >= 1; half >>= 1) {
        if (warp < half) {
            const Cand c = slist[(warp + half) * 32 + lane];
            warp_merge_top(v, id, c.v, c.id);
            slist[warp * 32 + lane] = Cand{v, id};
        }
        __syncthreads();
    }
    if (lane >= K && warp == 0) slist[lane] = Cand{-INFINITY, INT_MAX};  // keep exactly the best K
    __syncthreads();
}

__device__ __forceinline__ float penalize(float l, float penalty) { return l > 0.f ? fdiv(l, penalty) : fmul(l, penalty); }

// ---------------------------------------------------------------- head input

// rmsnorm(x, final_norm) + quantize (engine/src/model.cpp:225-226), plus the per-block |x_b| = d_b * sqrt(sum q^2)
// the shortlist bound needs (model.cpp:247-251; the int8 squares sum exactly in float).
__global__ void __launch_bounds__(kThreads) k_head_input(const float* __restrict__ X, const float* __restrict__ norm_w, int dim,
                                                         float eps, HeadIn hin, HeadState* hs, int full_rows) {
    __shared__ __align__(16) float sred[32 + 2048];
    __shared__ __align__(16) int8_t sx[2048];
    __shared__ float sdx[64];
    __shared__ int ssum[64];
    PhaseProbe probe;
    probe.begin(6);
    NormW nw;
    load_norm_w(norm_w, dim, nw);
    pdl_wait();
    pdl_launch_dependents();
    probe.mark();
    norm_quant(X, nw, dim, eps, sx, sdx, ssum, sred);
    probe.mark();
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
        float ss = fmul(q, q), sa = fabsf(q);
        for (int o = 16; o > 0; o >>= 1) {
            ss += __shfl_xor_sync(0xffffffffu, ss, o);
            sa += __shfl_xor_sync(0xffffffffu, sa, o);
        }
        if (lane == 0) {
            hin.dx[b] = sdx[b];
            hin.xsum[b] = ssum[b];
            hin.xnorm[b] = fmul(sdx[b], __fsqrt_rn(ss));
            if (hin.xabs) hin.xabs[b] = sa;
        }
    }
    probe.end();
}

// Activation of the head in shared memory: sx [cols] int8, then sdx, ssum, sxn [cols/32] (sxn: coarse pass only).
struct HeadAct {
    int8_t* sx;
    float* sdx;
    int* ssum;
    float* sxn;
};

__device__ __forceinline__ HeadAct carve_act(unsigned char* smem, int cols, bool with_norm) {
    const int nb = cols / QK;
    HeadAct a;
    a.sx = reinterpret_cast<int8_t*>(smem);
    a.sdx = reinterpret_cast<float*>(smem + cols);
    a.ssum = reinterpret_cast<int*>(a.sdx + nb);
    a.sxn = with_norm ? reinterpret_cast<float*>(a.ssum + nb) : nullptr;
    return a;
}

// Every read of data another kernel wrote goes through L2 (__ldcg): a kernel started early by programmatic dependent
// launch may find stale lines of it in its SM's L1.
__device__ __forceinline__ void load_head_act(const HeadIn& hin, int cols, const HeadAct& a) {
    for (int i = threadIdx.x; i < cols / 16; i += blockDim.x)
        reinterpret_cast<int4*>(a.sx)[i] = __ldcg(reinterpret_cast<const int4*>(hin.xq) + i);
    for (int b = threadIdx.x; b < cols / QK; b += blockDim.x) {
        a.sdx[b] = __ldcg(hin.dx + b);
        a.ssum[b] = __ldcg(hin.xsum + b);
        if (a.sxn) a.sxn[b] = __ldcg(hin.xnorm + b);
    }
    __syncthreads();
}

// One block's term (float(s_b) * dw_b) * dx_b of a row whose quants (16-byte granules, wq) and fp16 scales (wd) sit in
// shared memory.
template <int DT>
__device__ __forceinline__ float smem_block_term(const uint4* wq, const __half* wd, const HeadAct& a, int b) {
    int s;
    if (DT == DT_Q4_0)
        s = chunk_dot<DT>(wq[b], a.sx, b) - 8 * a.ssum[b];
    else
        s = chunk_dot<DT>(wq[2 * b], a.sx, 2 * b) + chunk_dot<DT>(wq[2 * b + 1], a.sx, 2 * b + 1);
    return block_term(s, __half2float(wd[b]), a.sdx[b]);
}

// A row's value acc = ((0 + t_0) + t_1) + ... in block order (matvec_q_ref), and with BOUND the shortlist bound
// (sum_b err_b * |x_b| in block order) * 1.001 + 1e-5 (engine/src/model.cpp:271-277), computed by kRowParts lanes of
// one warp: lane l holds part l / 8 of the warp's row l % 8.  Each part forms its nb / kRowParts terms in registers;
// the chains then run part after part, each part continuing from the previous part's sum (shuffled up 8 lanes), so
// the order of the float adds is the reference's.  The results are valid in the last part's lanes.
template <int DT, bool BOUND, int MAXB>
__device__ __forceinline__ void row_value_parts(const uint4* wq, const __half* wd, const __half* we, const HeadAct& a,
                                                int nb, float& val, float& bnd) {
    const int part = (threadIdx.x & 31) >> 3;
    const int bpp = nb / kRowParts, b0 = part * bpp;
    float t[MAXB], u[MAXB];
#pragma unroll
    for (int k = 0; k < MAXB; ++k) {
        if (k < bpp) {
            t[k] = smem_block_term<DT>(wq, wd, a, b0 + k);
            if (BOUND) u[k] = fmul(__half2float(we[b0 + k]), a.sxn[b0 + k]);
        }
    }
    float acc = 0.f, bd = 0.f;
    if (part == 0) {
#pragma unroll
        for (int k = 0; k < MAXB; ++k) {
            if (k < bpp) {
                acc = fadd(acc, t[k]);
                if (BOUND) bd = fadd(bd, u[k]);
            }
        }
    }
#pragma unroll
    for (int q = 1; q < kRowParts; ++q) {
        const float pa = __shfl_up_sync(0xffffffffu, acc, 8);
        const float pb = BOUND ? __shfl_up_sync(0xffffffffu, bd, 8) : 0.f;
        if (part == q) {
            acc = pa;
            bd = pb;
#pragma unroll
            for (int k = 0; k < MAXB; ++k) {
                if (k < bpp) {
                    acc = fadd(acc, t[k]);
                    if (BOUND) bd = fadd(bd, u[k]);
                }
            }
        }
    }
    val = acc;
    bnd = BOUND ? fadd(fmul(bd, 1.001f), 1e-5f) : 0.f;
}

// The nibble-plane screen of one row (kScreenHi4), with the same part layout as row_value_parts.  wq holds the high
// nibbles hi = q >> 4 of the Q8 row as Q4_0 (hi + 8), wd the Q8 row's own scales.  With q = 16 hi + lo (0 <= lo <= 15)
// the block dot s = 16 sum(hi x) + 8 sum(x) + sum((lo - 8) x), so the screen takes s' = 16 sum(hi x) + 8 sum(x) and
// |s - s'| <= 8 sum|x|.  The row's exact logit E (block terms fl(fl(s dw) dx) chained in f32) and the screen value
// (the same chain over s') each differ from their real sums by at most (nb + 2) 2^-24 of the sum of their terms'
// magnitudes, so E <= value + (sum_b 8 |dw_b| dx_b sum|x_b| + (2 nb + 8) 2^-24 sum_b (|t'_b| + bound_b)) * 1.001 + 1e-6
// (the factor covers the bound's own f32 rounding).  Per block the bound is the smaller of 8 |dw| dx sum|x| and
// e_b |dw| dx ||x||_2, e_b = ||lo - 8||_2 of the row's block rounded up to f16 (k_hi_plane's table).
template <int MAXB>
__device__ __forceinline__ void row_screen_hi4(const uint4* wq, const __half* wd, const __half* we, const HeadAct& a,
                                               const float* sxa, int nb, float& val, float& bnd) {
    const int part = (threadIdx.x & 31) >> 3;
    const int bpp = nb / kRowParts, b0 = part * bpp;
    float t[MAXB];
    float bd = 0.f, mag = 0.f;  // order-free sums (bounds)
#pragma unroll
    for (int k = 0; k < MAXB; ++k) {
        if (k < bpp) {
            const int b = b0 + k;
            const int hx = chunk_dot<DT_Q4_0>(wq[b], a.sx, b) - 8 * a.ssum[b];  // sum(hi x)
            const float dw = __half2float(wd[b]);
            t[k] = block_term(16 * hx + 8 * a.ssum[b], dw, a.sdx[b]);
            // the smaller of the L1 bound 8 |dw| dx sum|x| and the L2 bound ||lo - 8||_2 |dw| dx ||x||_2
            const float u = fminf(fmul(fmul(8.0f * fabsf(dw), a.sdx[b]), sxa[b]),
                                  fmul(fmul(__half2float(we[b]), fabsf(dw)), a.sxn[b]));
            bd = fadd(bd, u);
            mag = fadd(mag, fadd(fabsf(t[k]), u));
        }
    }
    float acc = 0.f;
    if (part == 0) {
#pragma unroll
        for (int k = 0; k < MAXB; ++k)
            if (k < bpp) acc = fadd(acc, t[k]);
    }
#pragma unroll
    for (int q = 1; q < kRowParts; ++q) {
        const float pa = __shfl_up_sync(0xffffffffu, acc, 8);
        if (part == q) {
            acc = pa;
#pragma unroll
            for (int k = 0; k < MAXB; ++k)
                if (k < bpp) acc = fadd(acc, t[k]);
        }
    }
    // the parts' bound sums, gathered onto the last part's lanes
#pragma unroll
    for (int o = 8; o < 32; o <<= 1) {
        bd += __shfl_xor_sync(0xffffffffu, bd, o);
        mag += __shfl_xor_sync(0xffffffffu, mag, o);
    }
    const float gam = float(2 * nb + 8) * 5.9604644775390625e-8f;  // (2 nb + 8) 2^-24
    val = acc;
    bnd = fadd(fmul(fadd(bd, fmul(mag, gam)), 1.001f), 1e-6f);
}

__device__ __forceinline__ void cp_wait_upto(int n) {  // wait until at most n groups are pending (n in 0..3)
    if (n <= 0) cp_wait<0>();
    else if (n == 1) cp_wait<1>();
    else if (n == 2) cp_wait<2>();
    else cp_wait<3>();
}

// ---------------------------------------------------------------- streaming pass over all rows (full / coarse)

// One persistent CTA per SM streams its contiguous tiles of head_tile_rows rows through a cp.async ring; one thread
// owns one row of a tile and chains its blocks in order straight from shared memory (row stride padded by 16 bytes so
// the 16-byte loads of a warp hit distinct banks).
// mode 0 (full head): logits = exact rows of W (Q8_0 or Q4_0); with n_list > 0 each CTA also writes its best n_list
//   rows among [0, n_valid) after the repetition penalty of marked rows, and clears those marks.
// mode 1 (coarse): W = quanta.head_q4; coarse / upper / logits = -inf, and each CTA's best n_list coarse scores among
//   valid unmarked rows (the seeds).
// mode 2 (coarse, nibble-plane screen): W = the Q8 head's high nibble plane with the Q8 scales (row_screen_hi4); the
//   same outputs as mode 1, no bound table staged.
template <int DT, int MODE, int MAXB, int TR = head_tile_rows(DT)>
__global__ void __launch_bounds__(TR * kRowParts, 1) k_head_rows(DMat W, const __half* __restrict__ err, HeadIn hin,
                                                                     StreamPlan sp, int n_valid, int n_list, int penal,
                                                                     float penalty, unsigned char* __restrict__ mark,
                                                                     float* __restrict__ logits, float* __restrict__ coarse,
                                                                     float* __restrict__ upper, Cand* __restrict__ lists) {
    constexpr int NT = TR * kRowParts;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ Cand slist[NT];
    const int cols = W.cols, nb = cols / QK, rb = row_bytes(DT, cols), cpr = rb / 16, S = sp.stages;
    const HeadAct act = carve_act(smem, cols, MODE != 0);
    unsigned char* ring = smem + sp.ring_off;
    const int ta = int((long long)blockIdx.x * sp.n_tiles / gridDim.x);
    const int tb = int((long long)(blockIdx.x + 1) * sp.n_tiles / gridDim.x);

    auto issue = [&](int t) {
        if (t < tb) {
            unsigned char* st = ring + size_t((t - ta) % S) * sp.stage_bytes;
            const int row0 = t * TR, nrows = min(TR, W.rows - row0);
            const uint8_t* qsrc = W.q + size_t(row0) * rb;
            for (int c = threadIdx.x; c < nrows * cpr; c += NT) {
                const int rr = int(fast_div(unsigned(c), sp.cpr_magic));
                cp_async16(st + rr * sp.qstride + (c - rr * cpr) * 16, qsrc + size_t(c) * 16);
            }
            const uint8_t* dsrc = reinterpret_cast<const uint8_t*>(W.d) + size_t(row0) * nb * 2;
            const int dch = (nrows * nb * 2 + 15) / 16;  // may read up to 15 bytes of the allocation's tail padding
            for (int c = threadIdx.x; c < dch; c += NT) cp_async16(st + sp.d_off + c * 16, dsrc + size_t(c) * 16);
            if (MODE != 0) {
                const uint8_t* esrc = reinterpret_cast<const uint8_t*>(err) + size_t(row0) * nb * 2;
                for (int c = threadIdx.x; c < dch; c += NT) cp_async16(st + sp.e_off + c * 16, esrc + size_t(c) * 16);
            }
        }
        cp_commit();
    };

    PhaseProbe probe;
    probe.begin(7);
    for (int s = 0; s < S - 1; ++s) issue(ta + s);
    pdl_wait();
    pdl_launch_dependents();
    probe.mark();
    load_head_act(hin, cols, act);
    __shared__ float sxa[128];  // mode 2: sum|x| per block (nb <= 128)
    if (MODE == 2) {
        for (int b = threadIdx.x; b < nb; b += blockDim.x) sxa[b] = __ldcg(hin.xabs + b);
        __syncthreads();
    }

    WarpTop32 L;
    L.init();
    const int lane = threadIdx.x & 31;
    const int r = (threadIdx.x >> 5) * 8 + (lane & 7);  // this lane's row in the tile
    const bool last_part = (lane >> 3) == kRowParts - 1;
    for (int t = ta; t < tb; ++t) {
        // tile t landed (this thread's copies, then everyone's), and every thread is past tile t - 1, whose stage
        // the next tile's copies refill: one barrier per tile
        cp_wait_upto(S - 2);
        __syncthreads();
        issue(t + S - 1);
        const unsigned char* st = ring + size_t((t - ta) % S) * sp.stage_bytes;
        const int row0 = t * TR, nrows = min(TR, W.rows - row0);
        float v, bound;
        if constexpr (MODE == 2)
            row_screen_hi4<MAXB>(reinterpret_cast<const uint4*>(st + r * sp.qstride),
                                 reinterpret_cast<const __half*>(st + sp.d_off + r * nb * 2),
                                 reinterpret_cast<const __half*>(st + sp.e_off + r * nb * 2), act, sxa, nb, v, bound);
        else
            row_value_parts<DT, MODE == 1, MAXB>(reinterpret_cast<const uint4*>(st + r * sp.qstride),
                                                 reinterpret_cast<const __half*>(st + sp.d_off + r * nb * 2),
                                                 reinterpret_cast<const __half*>(st + sp.e_off + r * nb * 2), act, nb, v,
                                                 bound);
        float cv = -INFINITY;
        int row = INT_MAX;
        bool ok = false;
        if (last_part && r < nrows) {
            row = row0 + r;
            cv = v;
            if constexpr (MODE == 0) {
                logits[row] = v;
                if (n_list > 0) {
                    ok = row < n_valid;
                    if (penal) {
                        const unsigned char mk = __ldcg(mark + row);
                        if (mk) {
                            cv = penalize(v, penalty);
                            mark[row] = 0;
                        }
                    }
                }
            } else {
                coarse[row] = v;
                upper[row] = fadd(v, bound);
                logits[row] = -INFINITY;
                ok = row < n_valid && __ldcg(mark + row) == 0;
            }
        }
        if constexpr (MODE == 0) {
            if (n_list > 0) L.offer(cv, row, ok, n_list);
        } else if (last_part) {  // the seeds are selected once after the tiles, from every row's score kept here
            reinterpret_cast<Cand*>(smem + sp.cand_off)[(t - ta) * TR + r] = ok ? Cand{cv, row} : Cand{-INFINITY, INT_MAX};
        }
    }
    cp_wait<0>();
    probe.mark();
    if constexpr (MODE != 0) {
        __syncthreads();  // every row's candidate is in shared memory
        if (n_list > 0) {  // each warp offers 32 of the CTA's rows at a time
            const Cand* cb = reinterpret_cast<const Cand*>(smem + sp.cand_off);
            const int n_c = (tb - ta) * TR;
            for (int i0 = 0; i0 < n_c; i0 += NT) {
                const int i = i0 + int(threadIdx.x);
                const Cand c = i < n_c ? cb[i] : Cand{-INFINITY, INT_MAX};
                L.offer(c.v, c.id, c.id != INT_MAX, n_list);
            }
        }
    }
    if (n_list > 0) {
        cta_merge_lists(L, n_list, slist);
        if (threadIdx.x < n_list) lists[size_t(blockIdx.x) * n_list + threadIdx.x] = slist[threadIdx.x];
    }
    probe.end();
}

// ---------------------------------------------------------------- shortlist head

// Marks the must ids: mark[id] = 1 for 0 <= id < n_valid (model.cpp:252-253).
__global__ void k_sl_mark(const int* __restrict__ must, const int* __restrict__ n_must_dev, int n_must_host, int window,
                          int n_valid, unsigned char* __restrict__ mark) {
    PhaseProbe probe;
    probe.begin(5);
    pdl_wait();
    pdl_launch_dependents();
    probe.mark();
    int n = n_must_dev ? __ldcg(n_must_dev) : n_must_host;
    int from = 0;
    if (window > 0 && n > window) from = n - window;
    for (int i = from + blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int id = __ldcg(must + i);
        if (id >= 0 && id < n_valid) mark[id] = 1;
    }
    probe.end();
}

// Exact Q8 logit of one row by one warp, same terms and order as the streamed full head.  wterm: nb floats.
__device__ __forceinline__ float warp_exact_row(const DMat& W, int row, const int8_t* sx, const float* sdx, float* wterm) {
    const int lane = threadIdx.x & 31, cols = W.cols, nb = cols / QK, cpr = cols / 16;
    const uint4* src = reinterpret_cast<const uint4*>(W.q + size_t(row) * cols);
    uint4 w[8];
    __half dw[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {  // all of this lane's loads in flight together (cols <= 4096)
        const int c = k * 32 + lane;
        w[k] = c < cpr ? ld_stream(src + c) : make_uint4(0, 0, 0, 0);
        dw[k] = c < cpr ? W.d[size_t(row) * nb + (c >> 1)] : __float2half(0.f);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int c = k * 32 + lane;
        if (k * 32 >= cpr) break;
        int s = c < cpr ? chunk_dot<DT_Q8_0>(w[k], sx, c) : 0;
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        if (c < cpr && !(c & 1)) wterm[c >> 1] = block_term(s, __half2float(dw[k]), sdx[c >> 1]);
    }
    __syncwarp();
    float acc = 0.f;
    if (lane == 0) acc = row_sum(wterm, nb);
    __syncwarp();
    return __shfl_sync(0xffffffffu, acc, 0);
}

// Exact Q8 logits of rows ra and rb (< 0: none) by one warp for rows of at most 1024 columns: both rows' loads are in
// flight together and lane 0 runs the two block-order chains interleaved.  wterm: 2 * nb floats.
__device__ __forceinline__ void warp_exact_rows2(const DMat& W, int ra, int rb, const int8_t* sx, const float* sdx,
                                                 float* wterm, float& va, float& vb) {
    const int lane = threadIdx.x & 31, cols = W.cols, nb = cols / QK, cpr = cols / 16;
    const int rows[2] = {ra, rb};
    uint4 w[2][2];
    __half dw[2][2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int c = k * 32 + lane;
            const bool ok = rows[j] >= 0 && c < cpr;
            w[j][k] = ok ? ld_stream(reinterpret_cast<const uint4*>(W.q + size_t(rows[j]) * cols) + c) : make_uint4(0, 0, 0, 0);
            dw[j][k] = ok ? W.d[size_t(rows[j]) * nb + (c >> 1)] : __float2half(0.f);
        }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int c = k * 32 + lane;
            int s = c < cpr ? chunk_dot<DT_Q8_0>(w[j][k], sx, c) : 0;
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            if (c < cpr && !(c & 1)) wterm[j * nb + (c >> 1)] = block_term(s, __half2float(dw[j][k]), sdx[c >> 1]);
        }
    }
    __syncwarp();
    float a = 0.f, b = 0.f;
    if (lane == 0) {
        for (int i = 0; i < nb; ++i) {
            a = fadd(a, wterm[i]);
            b = fadd(b, wterm[nb + i]);
        }
    }
    __syncwarp();
    va = __shfl_sync(0xffffffffu, a, 0);
    vb = __shfl_sync(0xffffffffu, b, 0);
}

// One CTA: global seeds (the n_seed best coarse scores), their exact logits, tau.
__global__ void __launch_bounds__(kHeadThreads, 1) k_sl_seeds(DMat W8, HeadIn hin, const Cand* __restrict__ seed_lists,
                                                           int n_lists, int n_seed, int k, unsigned char* __restrict__ mark,
                                                           float* __restrict__ logits, HeadState* __restrict__ hs) {
    __shared__ Cand slist[kHeadWarps * 32];
    __shared__ __align__(16) int8_t sx[4096];
    __shared__ float sdx[128];
    __shared__ float wterm[kHeadWarps][128];
    __shared__ float exact[32];
    __shared__ int s_ns;
    PhaseProbe probe;
    probe.begin(8);
    pdl_wait();
    pdl_launch_dependents();
    probe.mark();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cols = W8.cols, nb = cols / QK;
    for (int i = threadIdx.x; i < cols / 16; i += blockDim.x)
        reinterpret_cast<int4*>(sx)[i] = __ldcg(reinterpret_cast<const int4*>(hin.xq) + i);
    for (int b = threadIdx.x; b < nb; b += blockDim.x) sdx[b] = __ldcg(hin.dx + b);
    cta_merge_sorted(seed_lists, n_lists, n_seed, slist);
    probe.mark();
    if (threadIdx.x == 0) {
        int n = 0;
        while (n < n_seed && slist[n].id != INT_MAX) ++n;
        s_ns = n;
    }
    __syncthreads();
    const int ns = s_ns;
    if (cols <= 1024) {  // two seeds per warp at once: every seed in one round of loads
        for (int s = warp; s < ns; s += 2 * kHeadWarps) {
            const int s2 = s + kHeadWarps;
            const int id = slist[s].id, id2 = s2 < ns ? slist[s2].id : -1;
            float v, v2;
            warp_exact_rows2(W8, id, id2, sx, sdx, wterm[warp], v, v2);
            if (lane == 0) {
                exact[s] = v;
                logits[id] = v;
                mark[id] = 2;
                if (id2 >= 0) {
                    exact[s2] = v2;
                    logits[id2] = v2;
                    mark[id2] = 2;
                }
            }
        }
    } else {
        for (int s = warp; s < ns; s += kHeadWarps) {
            const int id = slist[s].id;
            const float v = warp_exact_row(W8, id, sx, sdx, wterm[warp]);
            if (lane == 0) {
                exact[s] = v;
                logits[id] = v;
                mark[id] = 2;
            }
        }
    }
    __syncthreads();
    probe.mark();
    // tau = the k-th largest exact seed logit (model.cpp:308-313): the seed whose rank (ties by position) is k-1.
    if (threadIdx.x < 32) {
        const int i = threadIdx.x;
        bool is_kth = false;
        if (i < ns && ns >= k) {
            int rank = 0;
            for (int j = 0; j < ns; ++j) rank += exact[j] > exact[i] || (exact[j] == exact[i] && j < i);
            is_kth = rank == k - 1;
        }
        const unsigned m = __ballot_sync(0xffffffffu, is_kth);
        if (i == 0) {
            hs->tau = m ? exact[__ffs(m) - 1] : -INFINITY;
            hs->rows = ns;
        }
    }
    probe.end();
}

// Candidate pass over this CTA's contiguous rows.  One scan reads every mark / bound, clears the marks, and compacts
// two lists: rows that need an exact logit (must ids, mark 1, and rows with upper >= tau, mark 0) and the seeds (mark
// 2, exact already).  The exact logits of the first list are gathered through the cp.async ring (kRowParts threads per
// row); the sampler's stage 1 then looks at the two lists only.
template <int MAXB>
__global__ void __launch_bounds__(head_threads(DT_Q8_0), 1) k_sl_cands(DMat W8, HeadIn hin, StreamPlan sp, int n_valid,
                                                                       int n_list, int penal, float penalty,
                                                                       unsigned char* __restrict__ mark,
                                                                       const float* __restrict__ upper,
                                                                       float* __restrict__ logits,
                                                                       HeadState* __restrict__ hs, Cand* __restrict__ lists) {
    constexpr int TR = head_tile_rows(DT_Q8_0), NT = head_threads(DT_Q8_0);
    constexpr int kScanPer = 8;  // rows a thread scans per batch of loads
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ Cand slist[NT];
    __shared__ int s_count, s_seeds;
    const int cols = W8.cols, nb = cols / QK, cpr = cols / 16, S = sp.stages;
    const HeadAct act = carve_act(smem, cols, false);
    int* list = reinterpret_cast<int*>(smem + sp.list_off);  // exact rows from the front (bit 30: penalised), seeds from the back
    const int cap = sp.list_cap;
    unsigned char* ring = smem + sp.ring_off;
    const int V = W8.rows;
    const int r0 = int((long long)blockIdx.x * V / gridDim.x), r1 = int((long long)(blockIdx.x + 1) * V / gridDim.x);
    if (threadIdx.x == 0) {
        s_count = 0;
        s_seeds = 0;
    }
    PhaseProbe probe;
    probe.begin(9);
    pdl_wait();
    pdl_launch_dependents();
    probe.mark();
    load_head_act(hin, cols, act);
    const float tau = __ldcg(&hs->tau);
    const int lane = threadIdx.x & 31;
    for (int base = r0; base < r1; base += NT * kScanPer) {
        unsigned char mk[kScanPer];
        float up[kScanPer];
#pragma unroll
        for (int k = 0; k < kScanPer; ++k) {  // every load of the batch first
            const int r = base + k * NT + threadIdx.x;
            mk[k] = r < r1 ? __ldcg(mark + r) : 0;
            up[k] = r < r1 && r < n_valid ? __ldcg(upper + r) : -INFINITY;
        }
#pragma unroll
        for (int k = 0; k < kScanPer; ++k) {
            const int r = base + k * NT + threadIdx.x;
            const bool in = r < r1 && r < n_valid;
            const bool want = in && (mk[k] == 1 || (mk[k] == 0 && up[k] >= tau));
            const bool seed = in && mk[k] == 2;
            if (r < r1 && mk[k]) mark[r] = 0;
            const unsigned mw = __ballot_sync(0xffffffffu, want), ms = __ballot_sync(0xffffffffu, seed);
            int ow = 0, os = 0;
            if (lane == 0) {
                if (mw) ow = atomicAdd(&s_count, __popc(mw));
                if (ms) os = atomicAdd(&s_seeds, __popc(ms));
            }
            ow = __shfl_sync(0xffffffffu, ow, 0);
            os = __shfl_sync(0xffffffffu, os, 0);
            const unsigned below = (1u << lane) - 1;
            if (want) list[ow + __popc(mw & below)] = r | (mk[k] == 1 ? 1 << 30 : 0);
            if (seed) list[cap - 1 - (os + __popc(ms & below))] = r;
        }
    }
    __syncthreads();
    probe.mark();
    const int n = s_count, ns = s_seeds;
    const int n_tiles = (n + TR - 1) / TR;
    const int dpr = nb / 4;  // 8-byte scale groups per row (rows of scales are 8-byte aligned, not 16)
    auto issue = [&](int t) {
        if (t < n_tiles) {
            unsigned char* st = ring + size_t(t % S) * sp.stage_bytes;
            const int nrows = min(TR, n - t * TR);
            for (int c = threadIdx.x; c < nrows * cpr; c += NT) {
                const int rr = int(fast_div(unsigned(c), sp.cpr_magic)), cc = c - rr * cpr;
                const int row = list[t * TR + rr] & 0x3FFFFFFF;
                cp_async16(st + rr * sp.qstride + cc * 16, W8.q + size_t(row) * cols + size_t(cc) * 16);
            }
            for (int c = threadIdx.x; c < nrows * dpr; c += NT) {
                const int rr = c / dpr, cc = c - rr * dpr;
                const int row = list[t * TR + rr] & 0x3FFFFFFF;
                cp_async8(st + sp.d_off + (rr * nb + 4 * cc) * 2,
                          reinterpret_cast<const uint8_t*>(W8.d) + (size_t(row) * nb + 4 * cc) * 2);
            }
        }
        cp_commit();
    };
    for (int s = 0; s < S - 1; ++s) issue(s);
    const int r = (threadIdx.x >> 5) * 8 + (lane & 7);
    const bool last_part = (lane >> 3) == kRowParts - 1;
    WarpTop32 L;
    L.init();
    for (int t = 0; t < n_tiles; ++t) {
        cp_wait_upto(S - 2);  // as in k_head_rows: one barrier per tile
        __syncthreads();
        issue(t + S - 1);
        const unsigned char* st = ring + size_t(t % S) * sp.stage_bytes;
        const int nrows = min(TR, n - t * TR);
        float v, unused;
        row_value_parts<DT_Q8_0, false, MAXB>(reinterpret_cast<const uint4*>(st + r * sp.qstride),
                                        reinterpret_cast<const __half*>(st + sp.d_off + r * nb * 2), nullptr, act, nb, v,
                                        unused);
        bool ok = false;
        float cv = -INFINITY;
        int row = INT_MAX;
        if (last_part && r < nrows) {
            const int e = list[t * TR + r];
            row = e & 0x3FFFFFFF;
            logits[row] = v;
            ok = n_list > 0;
            cv = (penal && (e >> 30)) ? penalize(v, penalty) : v;
        }
        if (n_list > 0) L.offer(cv, ok ? row : INT_MAX, ok, n_list);
    }
    cp_wait<0>();
    probe.mark();
    if (n_list > 0) {
        // the seeds: exact logits from the seed pass, never penalised (a must id carries mark 1, not 2)
        for (int i0 = 0; i0 < ns; i0 += NT) {
            const int i = i0 + threadIdx.x;
            const bool ok = i < ns;
            const int row = ok ? list[cap - 1 - i] : INT_MAX;
            L.offer(ok ? __ldcg(logits + row) : -INFINITY, row, ok, n_list);
        }
        cta_merge_lists(L, n_list, slist);
        if (threadIdx.x < n_list) lists[size_t(blockIdx.x) * n_list + threadIdx.x] = slist[threadIdx.x];
    }
    if (threadIdx.x == 0 && n) atomicAdd(&hs->rows, n);
    probe.end();
}

// ---------------------------------------------------------------- sampler

// Sampler stage 1 straight from a logits array (after a prefill, and the standalone sampler): penalty on the unique
// marked ids (written back to wb[id] when wb is set, as Sampler::sample edits its logits in place), each CTA's best K
// of [0, n_valid); clears the marks it used.
__global__ void __launch_bounds__(kThreads) k_topk_partial(const float* logits, int n_valid, int K, int penal,
                                                           float penalty, unsigned char* __restrict__ mark,
                                                           Cand* __restrict__ out, float* wb) {
    __shared__ Cand slist[kWarps * 32];
    pdl_wait();
    pdl_launch_dependents();
    WarpTop32 L;
    L.init();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r0 = int((long long)blockIdx.x * n_valid / gridDim.x), r1 = int((long long)(blockIdx.x + 1) * n_valid / gridDim.x);
    for (int base = r0 + warp * 32; base < r1; base += blockDim.x) {
        const int r = base + lane;
        const bool ok = r < r1;
        float v = -INFINITY;
        if (ok) {
            v = __ldcg(logits + r);
            if (penal && __ldcg(mark + r)) {
                v = penalize(v, penalty);
                mark[r] = 0;
                if (wb) wb[r] = v;
            }
        }
        L.offer(v, ok ? r : INT_MAX, ok, K);
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

// Stage 2 (one CTA): merge, then greedy pick or softmax/min-p/top-p draw (sampler.cpp:35-84); appends the token to the
// history and advances the position.
__global__ void __launch_bounds__(kHeadThreads) k_sample_final(const Cand* __restrict__ parts, int n_lists, int K, SamplerArgs sa,
                                                               SamplerState* __restrict__ ss, int* __restrict__ hist,
                                                               int hist_cap, NextMarks nm) {
    __shared__ Cand slist[kHeadWarps * 32];
    PhaseProbe probe;
    probe.begin(10);
    pdl_wait();
    pdl_launch_dependents();
    probe.mark();
    // the history length and the generator state, read ahead of the merge (warp 0 updates them after its barriers)
    const int nh_before = __ldcg(&ss->n_hist);
    const unsigned long long rng0 = __ldcg(&ss->rng);
    cta_merge_sorted(parts, n_lists, K, slist);
    probe.mark();
    const bool appends = sa.append && nh_before < hist_cap;
    if (threadIdx.x >= 32) {
        // the next head's must ids already in the history (lane 0 marks the drawn id), while warp 0 draws
        if (nm.mark) {
            const int after = nh_before + (appends ? 1 : 0);
            const int first = nm.window > 0 && after > nm.window ? after - nm.window : 0;
            for (int i = first + int(threadIdx.x) - 32; i < nh_before; i += int(blockDim.x) - 32) {
                const int id = __ldcg(hist + i);
                if (id >= 0 && id < nm.n_valid) nm.mark[id] = 1;
            }
        }
        return;
    }
    const int lane = threadIdx.x;
    const int n = __popc(__ballot_sync(0xffffffffu, lane < K && slist[lane].id != INT_MAX));  // valid entries form a prefix
    const bool draw = sa.temperature > 0.f && n > 0;
    int pick_i = 0;
    if (draw) {
        // the n exps in parallel, one per lane; then every lane holds all of them in registers and runs the
        // reference's sequential sums and scans on them (the same operations in the same order on each lane)
        const float mx = slist[0].v;
        const float mine = lane < n ? exp_ref(fdiv(fsub(slist[lane].v, mx), sa.temperature), sa.exptab) : 0.f;
        float p[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) p[i] = __shfl_sync(0xffffffffu, mine, i);
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (i < n) sum = fadd(sum, p[i]);
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (i < n) p[i] = fdiv(p[i], sum);
        int keep = n;
        if (sa.min_p > 0.f) {  // while (keep > 1 && p[keep - 1] < floor) --keep
            const float floor = fmul(p[0], sa.min_p);
#pragma unroll
            for (int i = 31; i >= 1; --i)
                if (keep == i + 1 && p[i] < floor) keep = i;
        }
        if (sa.top_p < 1.f) {  // the first prefix whose cumulative sum reaches top_p
            float cum = 0.f;
            bool reached = false;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                if (!reached && i < keep) {
                    cum = fadd(cum, p[i]);
                    if (cum >= sa.top_p) {
                        keep = i + 1;
                        reached = true;
                    }
                }
            }
        }
        float total_p = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (i < keep) total_p = fadd(total_p, p[i]);
        uint64_t st = rng0;
        const float u = fmul(float(xorshift64s(st) >> 40), 1.0f / 16777216.0f);
        if (lane == 0) ss->rng = st;
        float r = fmul(u, total_p);
        pick_i = keep - 1;
        bool found = false;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            if (!found && i < keep) {
                r = fsub(r, p[i]);
                if (r <= 0.f) {
                    pick_i = i;
                    found = true;
                }
            }
        }
    }
    if (lane != 0) return;
    const int pick = n > 0 ? slist[pick_i].id : 0;
    probe.end();
    if (nm.mark && appends && pick >= 0 && pick < nm.n_valid) nm.mark[pick] = 1;
    ss->token = pick;
    if (appends) {
        hist[nh_before] = pick;
        ss->n_hist = nh_before + 1;
        ss->pos = nh_before;  // the new token is fed at position len(history) - 1
    }
}

// ---------------------------------------------------------------- the nibble plane of the Q8 head

// One thread per output byte: block b of row r holds 16 bytes, byte j = (q[j] >> 4) + 8 | ((q[j + 16] >> 4) + 8) << 4
// (q the block's int8 values; >> is the arithmetic shift, so hi in [-8, 7]).  The thread of byte 0 also writes
// err[b] = ||lo - 8||_2 over the block's 32 low nibbles lo = q & 15, rounded up to f16 (the sum of squares is an exact
// integer; the square root is rounded up, then the conversion).
__global__ void k_hi_plane(const int8_t* __restrict__ q, long long n_blocks, uint8_t* __restrict__ plane,
                           __half* __restrict__ err) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_blocks * 16; i += (long long)gridDim.x * blockDim.x) {
        const long long b = i >> 4;
        const int j = int(i & 15);
        const int lo = (q[b * QK + j] >> 4) + 8, hi = (q[b * QK + j + 16] >> 4) + 8;
        plane[i] = uint8_t(lo | (hi << 4));
        if (j == 0) {
            int ss = 0;
            for (int k = 0; k < QK; ++k) {
                const int e = (q[b * QK + k] & 15) - 8;
                ss += e * e;
            }
            err[b] = __float2half_ru(__fsqrt_ru(float(ss)));
        }
    }
}

QNT_PHASE_READER(qnt_phase_read_head)

// ---------------------------------------------------------------- launchers

namespace {

size_t align16(size_t n) { return (n + 15) & ~size_t(15); }

}  // namespace

namespace {
StreamPlan plan_stream_tr(int dtype, int rows, int cols, int grid, bool coarse, bool gather, int tr) {
    StreamPlan p;
    const int rb = row_bytes_host(dtype, cols), cpr = rb / 16, nb = cols / QK;
    p.tile_rows = tr;
    p.threads = tr * kRowParts;
    p.n_tiles = (rows + tr - 1) / tr;
    p.cpr_magic = div_magic(unsigned(cpr));
    p.qstride = rb + 16;
    p.d_off = int(align16(size_t(tr) * p.qstride));
    p.e_off = int(p.d_off + align16(size_t(tr) * nb * 2 + 16));
    p.stage_bytes = int(coarse ? p.e_off + align16(size_t(tr) * nb * 2 + 16) : p.e_off);
    const size_t act_bytes = align16(size_t(cols) + size_t(nb) * 12);
    p.list_cap = gather ? (rows + grid - 1) / grid + 64 : 0;  // every row of a CTA's range fits in one of the lists
    const size_t list_bytes = align16(size_t(p.list_cap) * 4);
    p.list_off = int(act_bytes);
    p.ring_off = int((act_bytes + list_bytes + 127) / 128 * 128);
    // minus the kernels' static shared memory: the CTA list, sxa of the nibble screen, a few counters
    const size_t budget = 227 * 1024 - size_t(p.threads) * sizeof(Cand) - 512 - 128;
    p.cand_cap = coarse && grid > 0 ? (p.n_tiles + grid - 1) / grid * tr : 0;
    const size_t cand_bytes = size_t(p.cand_cap) * sizeof(Cand), fixed = size_t(p.ring_off) + cand_bytes;
    const size_t fit = budget > fixed ? (budget - fixed) / size_t(p.stage_bytes) : 0;
    p.stages = int(std::min<size_t>(4, fit));
    if (p.stages < 2 || nb % 4 != 0 || nb % kRowParts != 0 || nb / kRowParts > kMaxBpp) p.stages = 0;
    p.cand_off = int(size_t(p.ring_off) + size_t(p.stages) * p.stage_bytes);
    p.smem = size_t(p.cand_off) + cand_bytes;
    p.grid = grid;
    return p;
}
}  // namespace

StreamPlan plan_stream(int dtype, int rows, int cols, int grid, bool coarse, bool gather) {
    StreamPlan p = plan_stream_tr(dtype, rows, cols, grid, coarse, gather, head_tile_rows(dtype));
    if (coarse && dtype == DT_Q4_0 && grid > 0) {  // the wide tile when it fits twice and leaves fewer padded rows per CTA
        const StreamPlan w = plan_stream_tr(dtype, rows, cols, grid, coarse, gather, kWideTileRows);
        const auto slots = [&](const StreamPlan& q) { return size_t((q.n_tiles + grid - 1) / grid) * size_t(q.tile_rows); };
        if (w.stages >= 2 && (p.stages == 0 || slots(w) <= slots(p))) p = w;
    }
    return p;
}

cudaError_t launch_hi_plane(const DMat& W8, uint8_t* plane, __half* err, cudaStream_t st) {
    if (W8.dtype != DT_Q8_0 || W8.cols % QK != 0) return cudaErrorInvalidValue;
    const long long nbk = (long long)W8.rows * (W8.cols / QK);
    k_hi_plane<<<unsigned(std::min<long long>((nbk * 16 + 255) / 256, 4096)), 256, 0, st>>>(
        reinterpret_cast<const int8_t*>(W8.q), nbk, plane, err);
    return cudaGetLastError();
}

cudaError_t launch_head_input(const float* X, const float* norm_w, int dim, float eps, const HeadIn& hin, HeadState* hs,
                              int full_rows, cudaStream_t st, bool pdl) {
    if (dim > 2048) return cudaErrorInvalidValue;
    return launch_pdl(k_head_input, dim3(1), dim3(kThreads), 0, st, pdl, X, norm_w, dim, eps, hin, hs, full_rows);
}

template <int DT, int MAXB>
cudaError_t launch_full_t(const HeadFullArgs& a, const HeadIn& hin, cudaStream_t st, bool pdl) {
    return launch_pdl(k_head_rows<DT, 0, MAXB>, dim3(a.plan.grid), dim3(a.plan.threads), a.plan.smem, st, pdl, a.W,
                      (const __half*)nullptr, hin, a.plan, a.n_valid, a.n_list, a.penal, a.penalty, a.mark, a.logits,
                      (float*)nullptr, (float*)nullptr, reinterpret_cast<Cand*>(a.lists));
}

cudaError_t launch_head_full(const HeadFullArgs& a, const HeadIn& hin, cudaStream_t st, bool pdl) {
    if (a.plan.stages == 0) return cudaErrorInvalidValue;
    const bool small = a.W.cols / QK / kRowParts <= 8;
    if (a.W.dtype == DT_Q8_0)
        return small ? launch_full_t<DT_Q8_0, 8>(a, hin, st, pdl) : launch_full_t<DT_Q8_0, kMaxBpp>(a, hin, st, pdl);
    if (a.W.dtype == DT_Q4_0)
        return small ? launch_full_t<DT_Q4_0, 8>(a, hin, st, pdl) : launch_full_t<DT_Q4_0, kMaxBpp>(a, hin, st, pdl);
    return cudaErrorInvalidValue;
}

cudaError_t launch_shortlist(const ShortlistArgs& a, const HeadIn& hin, cudaStream_t st, bool pdl, int* kernels) {
    const int n_seed = a.k + 8;
    if (a.k < 1 || n_seed > 32 || a.W8.cols > 4096 || a.n_list > 32 || a.plan4.stages == 0 || a.plan8g.stages == 0)
        return cudaErrorInvalidValue;
    cudaError_t e = cudaSuccess;
    if (!a.marked) {
        e = launch_pdl(k_sl_mark, dim3(4), dim3(kThreads), 0, st, pdl, a.must, a.n_must_dev, a.n_must_host, a.window,
                       a.n_valid, a.mark);
        if (e != cudaSuccess) return e;
    }
    const bool small = a.W8.cols / QK / kRowParts <= 8;
    const bool wide = a.plan4.tile_rows == kWideTileRows;
    constexpr int W = kWideTileRows;
    auto coarse_kernel =
        a.screen == kScreenHi4
            ? (wide ? (small ? k_head_rows<DT_Q4_0, 2, 8, W> : k_head_rows<DT_Q4_0, 2, kMaxBpp, W>)
                    : (small ? k_head_rows<DT_Q4_0, 2, 8> : k_head_rows<DT_Q4_0, 2, kMaxBpp>))
            : (wide ? (small ? k_head_rows<DT_Q4_0, 1, 8, W> : k_head_rows<DT_Q4_0, 1, kMaxBpp, W>)
                    : (small ? k_head_rows<DT_Q4_0, 1, 8> : k_head_rows<DT_Q4_0, 1, kMaxBpp>));
    e = launch_pdl(coarse_kernel, dim3(a.plan4.grid),
                   dim3(a.plan4.threads), a.plan4.smem, st, pdl, a.W4, a.err, hin, a.plan4, a.n_valid, n_seed, 0, 1.0f, a.mark,
                   a.logits, a.coarse, a.upper, reinterpret_cast<Cand*>(a.seed_buf));
    if (e != cudaSuccess) return e;
    e = launch_pdl(k_sl_seeds, dim3(1), dim3(kHeadThreads), 0, st, pdl, a.W8, hin, (const Cand*)a.seed_buf, a.plan4.grid,
                   n_seed, a.k, a.mark, a.logits, a.hs);
    if (e != cudaSuccess) return e;
    e = launch_pdl(small ? k_sl_cands<8> : k_sl_cands<kMaxBpp>, dim3(a.plan8g.grid), dim3(a.plan8g.threads), a.plan8g.smem, st, pdl, a.W8, hin, a.plan8g, a.n_valid,
                   a.n_list, a.penal, a.penalty, a.mark, (const float*)a.upper, a.logits, a.hs,
                   reinterpret_cast<Cand*>(a.lists));
    if (kernels) *kernels += a.marked ? 3 : 4;
    return e;
}

cudaError_t launch_mark(const int* must, const int* n_must_dev, int n_must_host, int window, int n_valid, unsigned char* mark,
                        cudaStream_t st, bool pdl) {
    return launch_pdl(k_sl_mark, dim3(4), dim3(kThreads), 0, st, pdl, must, n_must_dev, n_must_host, window, n_valid, mark);
}

cudaError_t launch_topk_partial(const float* logits, int n_valid, int K, int penal, float penalty, unsigned char* mark,
                                void* lists, int n_lists, cudaStream_t st, bool pdl, float* write_back) {
    if (K < 1 || K > 32) return cudaErrorInvalidValue;
    return launch_pdl(k_topk_partial, dim3(n_lists), dim3(kThreads), 0, st, pdl, logits, n_valid, K, penal, penalty, mark,
                      reinterpret_cast<Cand*>(lists), write_back);
}

cudaError_t launch_sample_final(const void* lists, int n_lists, int K, const SamplerArgs& sa, SamplerState* ss, int* hist,
                                int hist_cap, cudaStream_t st, bool pdl, const NextMarks* next) {
    if (K < 1 || K > 32) return cudaErrorInvalidValue;
    if (next && next->mark && !hist) return cudaErrorInvalidValue;
    return launch_pdl(k_sample_final, dim3(1), dim3(kHeadThreads), 0, st, pdl, reinterpret_cast<const Cand*>(lists), n_lists,
                      K, sa, ss, hist, hist_cap, next ? *next : NextMarks{});
}

}  // namespace qb
