// The device sampler for any top_k: Sampler::sample (engine/src/sampler.cpp:44-84) when top_k is 0 (disabled) or
// larger than the 32 candidates the fused head lists keep.
//
// The reference sorts the surviving candidates by logit (nth_element to top_k, then std::sort), exponentiates them,
// sums the exps in sorted order, divides, cuts by min-p and top-p, sums again and walks the cumulative draw.  Here:
//   1. a stable LSD radix sort of (logit, id) over ids < n_valid -- four 8-bit passes of histogram, scan and scatter,
//      keyed so that larger logits come first and equal logits keep ascending ids;
//   2. one CTA evaluates the reference's float sequence on the sorted prefix: the exps in parallel, then each
//      order-dependent sum as one chain in sorted order (every lane of a warp runs the same chain on values broadcast
//      by shuffles).  A chain stops as soon as every remaining term is below half an ulp of the running value: from
//      there on each rounded add or subtract returns its input unchanged, so the result has the same bits as the full
//      loop.  "Every remaining term" is a suffix maximum, computed once, so the stop is exact whatever the order of the
//      exps within ties of the sort.
#include "head_kernels.h"
#include "kernels.cuh"

namespace qb {

namespace {

constexpr int kSortThreads = 256;
constexpr int kSortItems = 8;
constexpr int kSortTile = kSortThreads * kSortItems;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kRadix = 256;
constexpr int kScanThreads = 1024;
constexpr int kFinalThreads = 1024;

// Order-preserving key: ascending keys = descending logits (the sign-magnitude float made unsigned, then inverted).
__device__ __forceinline__ unsigned desc_key(float v) {
    const unsigned u = __float_as_uint(v);
    return (u & 0x80000000u) ? u : ~(u | 0x80000000u);
}
__device__ __forceinline__ float key_value(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? k : ~k & 0x7fffffffu);
}

// Half the gap to the next float above s (s >= 0, finite): adding any t < this to s returns s.
__device__ __forceinline__ float half_gap_up(float s) {
    return fmul(fsub(__uint_as_float(__float_as_uint(s) + 1u), s), 0.5f);
}
// Half the gap to the next float below r (r > 0, finite): subtracting any t < this from r returns r.
__device__ __forceinline__ float half_gap_down(float r) {
    return fmul(fsub(r, __uint_as_float(__float_as_uint(r) - 1u)), 0.5f);
}

// Pass histogram: per tile, the count of each 8-bit digit.  keys == nullptr: the first pass, keys made from logits.
__global__ void __launch_bounds__(kSortThreads) k_sort_hist(const float* logits, const unsigned* keys, int n, int shift,
                                                            unsigned* __restrict__ hist) {
    __shared__ unsigned cnt[kRadix];
    pdl_wait();
    pdl_launch_dependents();
    for (int d = threadIdx.x; d < kRadix; d += kSortThreads) cnt[d] = 0;
    __syncthreads();
    const int base = blockIdx.x * kSortTile;
#pragma unroll
    for (int j = 0; j < kSortItems; ++j) {
        const int i = base + j * kSortThreads + threadIdx.x;
        if (i < n) {
            const unsigned k = keys ? __ldcg(keys + i) : desc_key(__ldcg(logits + i));
            atomicAdd(&cnt[(k >> shift) & (kRadix - 1)], 1u);
        }
    }
    __syncthreads();
    for (int d = threadIdx.x; d < kRadix; d += kSortThreads) hist[size_t(d) * gridDim.x + blockIdx.x] = cnt[d];
}

// Exclusive scan of the digit-major histogram [digit][tile] (one CTA): the output offset of every (digit, tile).
__global__ void __launch_bounds__(kScanThreads) k_sort_scan(unsigned* __restrict__ hist, int m) {
    __shared__ unsigned wsum[kScanThreads / 32];
    pdl_wait();
    pdl_launch_dependents();
    const int per = (m + kScanThreads - 1) / kScanThreads;
    const int i0 = threadIdx.x * per, i1 = min(m, i0 + per);
    unsigned s = 0;
    for (int i = i0; i < i1; ++i) s += __ldcg(hist + i);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned inc = s;  // inclusive scan of the thread sums within the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
    }
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    unsigned before = 0;
    for (int w = 0; w < warp; ++w) before += wsum[w];
    unsigned run = before + inc - s;  // exclusive prefix of this thread's first entry
    for (int i = i0; i < i1; ++i) {
        const unsigned v = __ldcg(hist + i);
        hist[i] = run;
        run += v;
    }
}

// Stable scatter of one tile: items are taken in index order, 256 per round (warp-major, lane-minor); an item's place is
// its digit's tile offset + the same-digit items of earlier rounds + of earlier warps + of lower lanes.
__global__ void __launch_bounds__(kSortThreads) k_sort_scatter(const float* logits, const unsigned* keys_in,
                                                               const int* ids_in, int n, int shift,
                                                               const unsigned* __restrict__ offs,
                                                               unsigned* __restrict__ keys_out, int* __restrict__ ids_out) {
    __shared__ unsigned wcount[kSortWarps][kRadix];
    __shared__ unsigned run[kRadix];
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int d = threadIdx.x; d < kRadix; d += kSortThreads) run[d] = __ldcg(offs + size_t(d) * gridDim.x + blockIdx.x);
    const int base = blockIdx.x * kSortTile;
    for (int j = 0; j < kSortItems; ++j) {
        for (int e = threadIdx.x; e < kSortWarps * kRadix; e += kSortThreads) (&wcount[0][0])[e] = 0;
        __syncthreads();
        const int i = base + j * kSortThreads + threadIdx.x;
        const bool ok = i < n;
        unsigned k = 0;
        int id = 0;
        if (ok) {
            k = keys_in ? __ldcg(keys_in + i) : desc_key(__ldcg(logits + i));
            id = ids_in ? __ldcg(ids_in + i) : i;
        }
        const unsigned d = ok ? (k >> shift) & (kRadix - 1) : unsigned(kRadix);  // past-the-end items match only each other
        const unsigned peers = __match_any_sync(0xffffffffu, d);
        const unsigned lower = peers & ((1u << lane) - 1u);
        if (ok && lower == 0) wcount[warp][d] = __popc(peers);
        __syncthreads();
        if (ok) {
            unsigned pos = run[d] + __popc(lower);
            for (int w = 0; w < warp; ++w) pos += wcount[w][d];
            keys_out[pos] = k;
            ids_out[pos] = id;
        }
        __syncthreads();
        for (int dd = threadIdx.x; dd < kRadix; dd += kSortThreads) {
            unsigned s = 0;
#pragma unroll
            for (int w = 0; w < kSortWarps; ++w) s += wcount[w][dd];
            run[dd] += s;
        }
        __syncthreads();
    }
}

// Runs one order-dependent chain over v[0..n) on a whole warp (every lane holds the same running value):
//   step(acc, t, index) -> bool done.  stop(acc, i0) -> true when no term from i0 on can change acc any more.
template <class Step, class Stop>
__device__ __forceinline__ void warp_chain(const float* v, int n, float& acc, Step step, Stop stop) {
    const int lane = threadIdx.x & 31;
    float nxt = lane < n ? __ldcg(v + lane) : 0.f;
    for (int i0 = 0; i0 < n; i0 += 32) {
        const float cur = nxt;
        if (i0 + 32 + lane < n) nxt = __ldcg(v + i0 + 32 + lane);
        if (stop(acc, i0)) return;
        const int m = min(32, n - i0);
        for (int k = 0; k < m; ++k) {
            const float t = __shfl_sync(0xffffffffu, cur, k);
            if (step(acc, t, i0 + k)) return;
        }
    }
}

__device__ __forceinline__ uint64_t xorshift64_star(uint64_t& s) {
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    return s * 0x2545F4914F6CDD1DULL;
}

// One CTA: softmax(T) over the n best sorted candidates, min-p, top-p and the draw (sampler.cpp:53-84).  c and smax are
// n-float scratch arrays: the exps (then the probabilities) and their suffix maxima.
__global__ void __launch_bounds__(kFinalThreads) k_sample_wide(const unsigned* __restrict__ keys, const int* __restrict__ ids,
                                                               int n, SamplerArgs sa, SamplerState* __restrict__ ss,
                                                               int* __restrict__ hist, int hist_cap, float* __restrict__ c,
                                                               float* __restrict__ smax) {
    __shared__ float s_part[kFinalThreads / 32];
    __shared__ int s_last[kFinalThreads / 32];
    __shared__ float s_val;
    __shared__ int s_keep, s_pick;
    pdl_wait();
    pdl_launch_dependents();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float mx = key_value(__ldcg(keys));
    // exps, each c = exp((v - mx) / T) as the reference writes it
    for (int i = tid; i < n; i += kFinalThreads) c[i] = exp_ref(fdiv(fsub(key_value(__ldcg(keys + i)), mx), sa.temperature), sa.exptab);
    __syncthreads();
    // suffix maxima of c: per-thread chunk, then across threads
    const int per = (n + kFinalThreads - 1) / kFinalThreads;
    const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
    float m = 0.f;
    for (int i = i0; i < i1; ++i) m = fmaxf(m, c[i]);
    float inc = m;  // inclusive suffix max within the warp (lanes above)
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float t = __shfl_down_sync(0xffffffffu, inc, o);
        if (lane + o < 32) inc = fmaxf(inc, t);
    }
    if (lane == 0) s_part[warp] = inc;
    __syncthreads();
    float after = 0.f;  // max of the chunks of later threads
    for (int w = warp + 1; w < kFinalThreads / 32; ++w) after = fmaxf(after, s_part[w]);
    const float later_lanes = __shfl_down_sync(0xffffffffu, inc, 1);
    if (lane < 31) after = fmaxf(after, later_lanes);
    for (int i = i1 - 1; i >= i0; --i) {
        after = fmaxf(after, c[i]);
        smax[i] = after;
    }
    __syncthreads();
    // sum of the exps in sorted order (sampler.cpp:55-58)
    if (warp == 0) {
        float sum = 0.f;
        warp_chain(c, n, sum, [](float& a, float t, int) { a = fadd(a, t); return false; },
                   [&](float a, int i) { return __ldcg(smax + i) < half_gap_up(a); });
        if (lane == 0) s_val = sum;
    }
    __syncthreads();
    const float sum = s_val;
    for (int i = tid; i < n; i += kFinalThreads) {
        c[i] = fdiv(c[i], sum);
        smax[i] = fdiv(smax[i], sum);  // division by the same positive sum keeps the maxima
    }
    if (tid == 0) s_keep = n;
    __syncthreads();
    // min-p (sampler.cpp:62-65): keep the prefix up to the last candidate with p >= p0 * min_p (at least one)
    if (sa.min_p > 0.f) {
        const float floor_p = fmul(c[0], sa.min_p);
        int last = 0;
        for (int i = 1 + tid; i < n; i += kFinalThreads)
            if (c[i] >= floor_p) last = i;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
        if (lane == 0) s_last[warp] = last;
        __syncthreads();
        if (tid == 0) {
            int l = 0;
            for (int w = 0; w < kFinalThreads / 32; ++w) l = max(l, s_last[w]);
            s_keep = l + 1;
        }
        __syncthreads();
    }
    if (warp == 0) {
        int keep = s_keep;
        // top-p (sampler.cpp:66-75): the first prefix whose running sum reaches top_p
        if (sa.top_p < 1.f) {
            float cum = 0.f;
            int cut = keep;
            warp_chain(c, keep, cum,
                       [&](float& a, float t, int i) {
                           a = fadd(a, t);
                           if (a >= sa.top_p) {
                               cut = i + 1;
                               return true;
                           }
                           return false;
                       },
                       [&](float a, int i) { return __ldcg(smax + i) < half_gap_up(a); });
            keep = cut;
        }
        // total of the kept probabilities, then the draw (sampler.cpp:77-84)
        float total = 0.f;
        warp_chain(c, keep, total, [](float& a, float t, int) { a = fadd(a, t); return false; },
                   [&](float a, int i) { return __ldcg(smax + i) < half_gap_up(a); });
        uint64_t st = __ldcg(&ss->rng);
        const float u = fmul(float(xorshift64_star(st) >> 40), 1.0f / 16777216.0f);
        float r = fmul(u, total);
        int pick = keep - 1;
        warp_chain(c, keep, r,
                   [&](float& a, float t, int i) {
                       a = fsub(a, t);
                       if (a <= 0.f) {
                           pick = i;
                           return true;
                       }
                       return false;
                   },
                   [&](float a, int i) { return a > 0.f && __ldcg(smax + i) < half_gap_down(a); });
        if (lane == 0) {
            ss->rng = st;
            s_pick = __ldcg(ids + pick);
        }
    }
    __syncthreads();
    if (tid == 0) {
        const int tok = s_pick;
        ss->token = tok;
        if (sa.append) {
            const int nh = __ldcg(&ss->n_hist);
            if (nh < hist_cap) {
                hist[nh] = tok;
                ss->n_hist = nh + 1;
                ss->pos = nh;  // the new token is fed at position len(history) - 1
            }
        }
    }
}

}  // namespace

int wide_sort_tiles(int n_valid) { return (n_valid + kSortTile - 1) / kSortTile; }

size_t wide_scratch_bytes(int n_valid) {
    const size_t n = size_t(n_valid);
    return 4 * (n * 4 + 256) + size_t(kRadix) * wide_sort_tiles(n_valid) * 4 + 256;
}

WideScratch wide_scratch_carve(void* base, int n_valid) {
    WideScratch w;
    auto* p = static_cast<unsigned char*>(base);
    const size_t arr = (size_t(n_valid) * 4 + 255) & ~size_t(255);
    w.keys[0] = reinterpret_cast<unsigned*>(p);
    w.keys[1] = reinterpret_cast<unsigned*>(p + arr);
    w.ids[0] = reinterpret_cast<int*>(p + 2 * arr);
    w.ids[1] = reinterpret_cast<int*>(p + 3 * arr);
    w.hist = reinterpret_cast<unsigned*>(p + 4 * arr);
    w.cap = n_valid;
    return w;
}

cudaError_t launch_sample_wide(const float* logits, int n_valid, int K, const SamplerArgs& sa, SamplerState* ss, int* hist,
                               int hist_cap, const WideScratch& ws, cudaStream_t st, bool pdl, int* kernels) {
    if (n_valid <= 0 || n_valid > ws.cap || !(sa.temperature > 0.f)) return cudaErrorInvalidValue;
    const int tiles = wide_sort_tiles(n_valid), m = kRadix * tiles;
    cudaError_t e = cudaSuccess;
    // four passes: logits -> [1] -> [0] -> [1] -> [0]
    for (int pass = 0; pass < 4 && e == cudaSuccess; ++pass) {
        const int src = pass & 1, dst = src ^ 1;  // pass 0 reads the logits and writes buffer 1
        const unsigned* kin = pass == 0 ? nullptr : ws.keys[src];
        const int* iin = pass == 0 ? nullptr : ws.ids[src];
        e = launch_pdl(k_sort_hist, dim3(tiles), dim3(kSortThreads), 0, st, pdl, logits, kin, n_valid, 8 * pass, ws.hist);
        if (e == cudaSuccess) e = launch_pdl(k_sort_scan, dim3(1), dim3(kScanThreads), 0, st, pdl, ws.hist, m);
        if (e == cudaSuccess)
            e = launch_pdl(k_sort_scatter, dim3(tiles), dim3(kSortThreads), 0, st, pdl, logits, kin, iin, n_valid, 8 * pass,
                           (const unsigned*)ws.hist, ws.keys[dst], ws.ids[dst]);
    }
    if (e != cudaSuccess) return e;
    const int n = (K > 0 && K < n_valid) ? K : n_valid;  // top_k <= 0 or >= n_valid keeps every candidate
    // the sorted order is in buffer 0; buffer 1 is free for the exps and their suffix maxima
    e = launch_pdl(k_sample_wide, dim3(1), dim3(kFinalThreads), 0, st, pdl, (const unsigned*)ws.keys[0], (const int*)ws.ids[0],
                   n, sa, ss, hist, hist_cap, reinterpret_cast<float*>(ws.keys[1]), reinterpret_cast<float*>(ws.ids[1]));
    if (kernels) *kernels += 13;
    return e;
}

}  // namespace qb
