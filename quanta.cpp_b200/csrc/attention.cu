// GQA attention over the f16 KV cache (engine/src/model.cpp:115-137), bit-identical to the reference.
//
// Query token t sits at position pos = pos0 + t and attends to [0, pos] in the reference's order:
//   score  s_j = (sum_i q_i * k_ji in dimension order) * scale
//   max    m = max_j s_j                                   (exact in any order)
//   weight e_j = exp(s_j - m); sum = e_0 + e_1 + ... in position order; a_j = e_j * (1 / sum)
//   output o_i = a_0 v_0i + a_1 v_1i + ... in position order
// The two sums are sequential chains (the reference's float order), so each query head gets its own SM resources:
// one thread-block cluster of CS CTAs per (query head, token), grid (CS * n_heads, n_tok), 256 threads per CTA,
// CS a power of two up to 8.
//   1. CTA r of the cluster scores the contiguous positions [r P, r P + P) (P = ceil((pos + 1) / CS)), one thread per
//      position (K tiles staged as f32 in shared memory), and posts its local maximum to the leader (rank 0) through
//      distributed shared memory.
//   2. cluster barrier; every CTA reads the CS maxima, exponentiates its own scores and stores the weights into the
//      weight row of every CTA of the cluster (distributed shared memory).
//   3. cluster barrier; every CTA sums the whole row in position order on one thread (the same sum, the same bits) and
//      owns 64 / CS output dimensions: its producer warps form the products a_j * v_jd (f32, the reference's separately
//      rounded multiply) of its dimensions for 512-row blocks into one of two buffers, and one lane per dimension adds
//      them in position order.  Splitting the dimensions spreads the f16 -> f32 conversions and the product traffic
//      over the cluster; each chain is still one load and one add per row.
//   4. with a quantized output requested, the CTAs post their outputs into the leader, which quantizes them.
// Decode can also take the layer's q|k|v rows into the same launch (k_attn<8, UW>, launch_qkv_attn): each CTA first
// computes 24 of its head's q / k / v rows (rmsnorm + quantize prologue, integer matvec, bias, RoPE) and the cluster
// exchanges them through distributed shared memory, so the q|k|v kernel and its launch gap disappear.  With o_proj
// folded in as well (k_attn<8, UW, UO>), every CTA then quantizes the head's outputs and writes the o_proj block terms
// of the head's two 32-blocks for an eighth of the rows; the gate|up kernel sums them onto the residual.
// K rows and each CTA's V columns below the launch's first position were written by earlier launches, so they are
// requested before the programmatic-launch wait (the first K tile into registers, the V columns by cp.async into
// shared memory) and land while the previous kernel finishes; only this launch's own rows and the query wait.
// The cluster barriers and named barriers are hardware barriers (no spin loops).
#include <cooperative_groups.h>

#include "kernels.cuh"
#include "layer_kernels.h"
#include "phase_stamps.cuh"

namespace qb {

namespace cg = cooperative_groups;

namespace {

constexpr int kPosChunk = 64;       // KV positions per chunk (the unit of max_chunks)
constexpr int kHd = 64;             // supported head_dim
constexpr int kTile = 128;          // positions scored per K tile (one thread each)
constexpr int kOutThreads = 64;     // warps 0-1: the chain lanes (one per owned dimension) and the quantizer
constexpr int kMaxCluster = 8;      // portable cluster size limit
constexpr int kKfStride = kHd + 1;  // f32 K tile row stride (conflict-free column walks)
constexpr int kPB = 512;            // rows per product block (fewer blocks: each hand-over costs a barrier round trip)

// Dynamic shared memory layout (byte offsets), the same for every CTA of a launch; dpc = 64 / CS dimensions per CTA.
constexpr int kOffQ = 0;                        // f32 [kHd] query
constexpr int kOffMax = kOffQ + kHd * 4;        // f32 [kMaxCluster] the cluster CTAs' local maxima (each CTA a copy)
constexpr int kOffOut = kOffMax + 256;          // f32 [kHd] the head's outputs, gathered in the leader
constexpr int kOffK = kOffOut + kHd * 4;        // f32 [kTile][kKfStride] K tile
constexpr int kKfBytes = kTile * kKfStride * 4;
constexpr int kOffProd = kOffK + kKfBytes;      // f32 [2][dpc][pb_rows + 4] products, dimension-major
static_assert(kOffK % 16 == 0 && kKfBytes % 16 == 0, "16-byte aligned regions");
static_assert(kThreads == 256 && kTile * 8 % kThreads == 0, "K tile loader");
constexpr int kProducers = kThreads - kOutThreads;
// named barriers (0 is __syncthreads): product buffer b full / free
constexpr int kBarFull = 2, kBarFree = 4;

__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }
template <int ID>
__device__ __forceinline__ void bar_sync(int count) { asm volatile("bar.sync %0, %1;" ::"n"(ID), "r"(count) : "memory"); }
template <int ID>
__device__ __forceinline__ void bar_arrive(int count) { asm volatile("bar.arrive %0, %1;" ::"n"(ID), "r"(count) : "memory"); }

__host__ __device__ inline int ls_len(int ctx, int cs) { return ((ctx + cs - 1) / cs + 3) & ~3; }
// then f16 [ctx][dpc] V columns, f32 [ls_len] own scores, f32 [ctx] weights
__host__ __device__ inline int pb_rows(int ctx) { return ctx < kPB ? ctx : kPB; }
// a dimension's products are contiguous (float4 loads by its chain lane); the +4 keeps the lanes' rows in distinct banks
__host__ __device__ inline int pb_stride(int ctx) { return pb_rows(ctx) + 4; }
__host__ __device__ inline int off_vs(int ctx, int cs) { return kOffProd + 2 * pb_stride(ctx) * (kHd / cs) * 4; }
__host__ __device__ inline int off_ls(int ctx, int cs) { return off_vs(ctx, cs) + ctx * (kHd / cs) * 2; }
inline size_t attn_smem_bytes(int ctx, int cs) { return size_t(off_ls(ctx, cs)) + size_t(ls_len(ctx, cs)) * 4 + size_t(ctx) * 4; }
// decode with the q|k|v rows fused in: after the weight row, sx [dim] int8, sdx [dim/32], the norm's scratch
// [32 + dim], terms [24][dim/32 | 1], the current token's k and v [64] each (f32 of the f16 values)
constexpr int kQkvRows = 24;  // 8 rows of each of the head's q, k and v units per CTA (cluster of 8)
inline size_t qkv_smem_bytes(int dim) {
    const int nb = dim / QK;
    return size_t(dim) + size_t(nb) * 4 + size_t(32 + dim) * 4 + size_t(kQkvRows) * (nb | 1) * 4 + 2 * kHd * 4;
}

// UW > 0: decode only (one token, CS = 8), with the layer's q|k|v matvec fused in front (UW weight chunks per
// thread): every CTA of the head's cluster computes 8 rows of each of the head's q, k and v units (the k and v units
// of the kv head are recomputed by each of its query heads' clusters, the same bits), applies bias and RoPE, and
// posts q and the f16-rounded k, v of the token into every CTA of the cluster; the first query head of each kv
// head also stores k, v into the cache.  This removes the q|k|v kernel, its launch gap and the attention's reads of
// q and of the token's own K/V row.  Bit-identical to k_qkv_dec followed by the unfused attention.
// UO > 0 (with UW > 0): o_proj folded in as well.  After the output chain every CTA holds the head's 64 outputs,
// quantizes them (the same bits as the leader's quantize for o_proj) and forms the o_proj block terms of the head's two
// 32-blocks for its eighth of the rows (UO weight chunks per thread, loaded before the wait) into oa.T.
template <int CS, int UW, int UO>
__global__ void __launch_bounds__(kThreads) k_attn(AttnArgs a, QkvArgs qa, OArgs oa, const float* __restrict__ X,
                                                   const float* __restrict__ norm_w, float eps, float* __restrict__ Qout,
                                                   const float* __restrict__ Q, const int* __restrict__ pos_dev, int n_tok,
                                                   float* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const int r = int(cluster.block_rank());  // CS = cluster.num_blocks(), fixed by the launch
    const int h = blockIdx.x / CS, t = blockIdx.y;
    const int group = a.n_heads / a.n_kv, g = h / group;
    const int ctx = a.max_chunks * kPosChunk;
    constexpr int dpc = kHd / CS;  // this CTA's output dimensions [d0, d0 + dpc)
    const int d0 = r * dpc;
    float* sq = reinterpret_cast<float*>(smem + kOffQ);
    float* smx = reinterpret_cast<float*>(smem + kOffMax);
    float* so = reinterpret_cast<float*>(smem + kOffOut);
    float* kf = reinterpret_cast<float*>(smem + kOffK);
    float* prod = reinterpret_cast<float*>(smem + kOffProd);
    __half* vs = reinterpret_cast<__half*>(smem + off_vs(ctx, CS));
    const int pbr = pb_rows(ctx), pbs = pb_stride(ctx);  // rows per product block, a dimension's stride
    float* LS = reinterpret_cast<float*>(smem + off_ls(ctx, CS));
    float* E = LS + ls_len(ctx, CS);
    __shared__ float sred[kWarps];
    __shared__ float s_m, s_inv;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    PhaseProbe probe;
    probe.begin(1);
    // every CTA of the cluster has started before any remote shared-memory access (the wait comes before the first)
    asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
    // The launch's first position was written by an earlier launch (the host or the step's first kernel); K / V rows
    // below it are final, rows from it on are this launch's (the previous kernel's) and wait for it.
    const int pos0 = __ldcg(pos_dev);
    const int n = pos0 + t + 1;
    const int P = (n + CS - 1) / CS, p0 = min(n, r * P), p1 = min(n, p0 + P);
    const bool producer = tid >= kOutThreads;
    const int nblk = (n + pb_rows(ctx) - 1) / pb_rows(ctx);
    const __half* V = a.vcache + g * kHd + d0;
    const __half* K = a.kcache + g * kHd;
    // this CTA's V columns of rows [j0, j1) into vs (16-byte granules, dpc / 8 per row), one cp.async group
    auto load_v = [&](int j0, int j1) {
        constexpr int gpr = dpc / 8;
        for (int i = tid; i < (j1 - j0) * gpr; i += kThreads) {
            const int row = j0 + i / gpr, c = i % gpr;
            cp_async16(vs + size_t(row) * dpc + c * 8, V + size_t(row) * a.kv_dim + c * 8);
        }
        cp_commit();
    };
    constexpr int U = kTile * 8 / kThreads;
    uint4 kv[U];
    // K rows [tile0, tile0 + tl) of the scored range, rows >= pos0 only when `late`
    auto load_k = [&](int tile0, int tl, bool late) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = u * kThreads + tid, row = i >> 3;
            if (row < tl && (tile0 + row < pos0) != late)
                kv[u] = __ldcg(reinterpret_cast<const uint4*>(K + size_t(tile0 + row) * a.kv_dim) + (i & 7));
            else if (!late)
                kv[u] = make_uint4(0, 0, 0, 0);
        }
    };
    // K tile rows -> f32 in shared memory: the rows below pos0 (early), from pos0 on (late), or all of them
    auto store_k = [&](int tile0, int which) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = u * kThreads + tid, row = i >> 3, c8 = (i & 7) * 8;
            if (which == 1 && tile0 + row >= pos0) continue;
            if (which == 2 && tile0 + row < pos0) continue;
            const __half2* h2 = reinterpret_cast<const __half2*>(&kv[u]);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = __half22float2(h2[k]);
                kf[row * kKfStride + c8 + 2 * k] = f.x;
                kf[row * kKfStride + c8 + 2 * k + 1] = f.y;
            }
        }
    };
    // fused q|k|v (UW > 0): virtual row vr of this CTA = unit vr / 8 (the head's q, its kv head's k, v), row 8 r + vr % 8
    const int qdim = qa.W.cols, qnb = qdim / QK, qcpr = qdim / 16, qts = qnb | 1, qtotal = kQkvRows * qcpr;
    auto qrow = [&](int vr) {
        const int u = vr >> 3;
        return (u == 0 ? h : u == 1 ? qa.n_heads + g : qa.n_heads + qa.n_kv + g) * kHd + 8 * r + (vr & 7);
    };
    constexpr int UWn = UW > 0 ? UW : 1;
    uint4 wv[UWn];
    __half wdv[UWn];
    // o_proj (UO > 0): chunk f of this CTA = row orow0 + f / 4, chunk f % 4 of the head's 64 columns (two per 32-block)
    constexpr int UOn = UO > 0 ? UO : 1;
    const int ocols = oa.W.cols, onb = ocols / QK, orpc = (oa.W.rows + CS - 1) / CS, orow0 = r * orpc;
    const int onr = UO > 0 ? min(orpc, oa.W.rows - orow0) : 0;
    uint4 wo[UOn];
    __half wdo[UOn];
    if constexpr (UO > 0) {
#pragma unroll
        for (int u = 0; u < UO; ++u) {
            const int f = u * kThreads + tid, orow = orow0 + (f >> 2), c = f & 3;
            if ((f >> 2) < onr) {
                wo[u] = ld_stream(reinterpret_cast<const uint4*>(oa.W.q + size_t(orow) * ocols + h * kHd) + c);
                wdo[u] = oa.W.d[size_t(orow) * onb + 2 * h + (c >> 1)];
            } else {
                wo[u] = make_uint4(0, 0, 0, 0);
                wdo[u] = __float2half(0.f);
            }
        }
    }
    NormW nw;
    float pba = 0.f, pbb = 0.f, pc = 1.f, ps = 0.f;  // pair lanes (tid < 12): bias of the two rows, RoPE cos / sin
    if constexpr (UW > 0) {  // the CTA's weight chunks, the norm weights and the pair constants before the wait
        load_norm_w(norm_w, qdim, nw);
        if (tid < kQkvRows / 2) {
            const int vr = 2 * tid, fr = qrow(vr), i = (8 * r + (vr & 7)) >> 1;
            pba = qa.bias[fr];
            pbb = qa.bias[fr + 1];
            if ((vr >> 3) < 2) {
                pc = qa.rope_cos[size_t(pos0) * (kHd / 2) + i];
                ps = qa.rope_sin[size_t(pos0) * (kHd / 2) + i];
            }
        }
#pragma unroll
        for (int u = 0; u < UW; ++u) {
            const int f = u * kThreads + tid;
            if (f < qtotal) {
                const int vr = f / qcpr, c = f - vr * qcpr, fr = qrow(vr);
                wv[u] = ld_stream(reinterpret_cast<const uint4*>(qa.W.q + size_t(fr) * qdim) + c);
                wdv[u] = qa.W.d[size_t(fr) * qnb + (c >> 1)];
            } else {
                wv[u] = make_uint4(0, 0, 0, 0);
                wdv[u] = __float2half(0.f);
            }
        }
    }
    // ---- before the wait: the first K tile's final rows (loaded and converted), this CTA's V columns of them
    load_k(p0, min(kTile, p1 - p0), false);
    store_k(p0, 1);
    load_v(0, min(pos0, n));
    pdl_wait();
    pdl_launch_dependents();
    probe.mark();  // 1: the previous kernel is done
    float* kc = nullptr;  // (fused) the token's k and v, f32 of their f16 values
    float* vc = nullptr;
    if constexpr (UW == 0) {
        load_v(min(pos0, n), n);  // this launch's own rows
        if (tid < kHd) sq[tid] = __ldcg(Q + (size_t(t) * a.n_heads + h) * kHd + tid);
        asm volatile("barrier.cluster.wait;" ::: "memory");
    } else {
        unsigned char* qs = smem + off_ls(ctx, CS) + (ls_len(ctx, CS) + ctx) * 4;
        int8_t* sx = reinterpret_cast<int8_t*>(qs);
        float* sdx = reinterpret_cast<float*>(qs + qdim);
        float* sredq = sdx + qnb;
        float* sterm = sredq + 32 + qdim;
        kc = sterm + kQkvRows * qts;
        vc = kc + kHd;
        norm_quant(X, nw, qdim, eps, sx, sdx, nullptr, sredq);
        probe.mark();  // 2: rmsnorm + quantize
#pragma unroll
        for (int u = 0; u < UW; ++u) {  // block terms (Q8_0: a block's two chunks sit in adjacent lanes)
            if (u * kThreads >= qtotal) break;
            const int f = u * kThreads + tid;
            const int vr = f / qcpr, c = f - vr * qcpr;
            int sdot = f < qtotal ? chunk_dot<DT_Q8_0>(wv[u], sx, c) : 0;
            sdot += __shfl_xor_sync(0xffffffffu, sdot, 1);
            if (f < qtotal && !(c & 1)) sterm[vr * qts + (c >> 1)] = block_term(sdot, __half2float(wdv[u]), sdx[c >> 1]);
        }
        __syncthreads();
        asm volatile("barrier.cluster.wait;" ::: "memory");
        // warp 0: lane l < 24 sums row l; lane p < 12 then takes rows 2 p, 2 p + 1 (dimensions i, i + 32 of its unit)
        if (warp == 0) {
            const float rs = lane < kQkvRows ? row_sum(sterm + lane * qts, qnb) : 0.f;
            const float ra = __shfl_sync(0xffffffffu, rs, (2 * lane) & 31);
            const float rb = __shfl_sync(0xffffffffu, rs, (2 * lane + 1) & 31);
            if (lane < kQkvRows / 2) {
                const int vr = 2 * lane, u = vr >> 3, i = (8 * r + (vr & 7)) >> 1;
                float va = fadd(ra, pba), vb = fadd(rb, pbb);
                if (u < 2) rope_pair(va, vb, pc, ps);
                if (u == 0) {
                    for (int q = 0; q < CS; ++q) {
                        float* dst = cluster.map_shared_rank(sq, q);
                        dst[i] = va;
                        dst[i + kHd / 2] = vb;
                    }
                    Qout[h * kHd + i] = va;
                    Qout[h * kHd + i + kHd / 2] = vb;
                } else {
                    const __half ha = __float2half_rn(va), hb = __float2half_rn(vb);
                    for (int q = 0; q < CS; ++q) {
                        float* dst = cluster.map_shared_rank(u == 1 ? kc : vc, q);
                        dst[i] = __half2float(ha);
                        dst[i + kHd / 2] = __half2float(hb);
                    }
                    if (h == g * group) {  // one cluster per kv head writes the cache
                        __half* C = (u == 1 ? qa.kcache : qa.vcache) + size_t(pos0) * qa.kv_dim + g * kHd;
                        C[i] = ha;
                        C[i + kHd / 2] = hb;
                    }
                }
            }
        }
        cluster_arrive();  // q, k and v of the token are in every CTA
        cluster_wait();
        probe.mark();  // 3: q|k|v rows, bias, RoPE, exchange
        if (tid < dpc) vs[size_t(pos0) * dpc + tid] = __float2half_rn(vc[d0 + tid]);  // exact: vc holds f16 values
    }

    // ---- 1. scores of [p0, p1), one position per thread
    for (int tile0 = p0; tile0 < p1; tile0 += kTile) {
        const int tl = min(kTile, p1 - tile0);
        if (tile0 == p0) {  // the first tile's final rows came (and were converted) before the wait
            if constexpr (UW == 0) {
                load_k(tile0, tl, true);
                store_k(tile0, 2);
            }
        } else {
            load_k(tile0, tl, false);
            if constexpr (UW == 0) load_k(tile0, tl, true);
            __syncthreads();  // the previous tile's readers are done
            store_k(tile0, UW == 0 ? 0 : 1);
        }
        if constexpr (UW > 0) {  // the token's own row (position pos0) from the posted k
            if (pos0 >= tile0 && pos0 < tile0 + tl && tid < kHd) kf[(pos0 - tile0) * kKfStride + tid] = kc[tid];
        }
        __syncthreads();  // the tile (and the query) are visible
        if (tid < tl) {
            const float* kj = kf + tid * kKfStride;
            float s = 0.f;
#pragma unroll 16
            for (int i = 0; i < kHd; ++i) s = fadd(s, fmul(sq[i], kj[i]));
            LS[tile0 - p0 + tid] = fmul(s, a.scale);
        }
    }
    __syncthreads();
    float lm = -INFINITY;
    for (int j = tid; j < p1 - p0; j += kThreads) lm = fmaxf(lm, LS[j]);
    lm = warp_max(lm);
    if (lane == 0) sred[warp] = lm;
    __syncthreads();
    if (tid < CS) {  // this CTA's maximum into slot r of every CTA's table
        float m = sred[0];
        for (int k = 1; k < kWarps; ++k) m = fmaxf(m, sred[k]);
        cluster.map_shared_rank(smx, tid)[r] = m;
    }
    cluster.sync();
    probe.mark();  // 4: scores and the maxima exchange

    // ---- 2. weights of [p0, p1) into every CTA's row
    if (warp == 0) {
        float m = lane < CS ? smx[lane] : -INFINITY;
        m = warp_max(m);
        if (lane == 0) s_m = m;
    }
    __syncthreads();
    for (int j = tid; j < p1 - p0; j += kThreads) {
        const float e = exp_ref(fsub(LS[j], s_m), a.exptab);
        for (int q = 0; q < CS; ++q) cluster.map_shared_rank(E, q)[p0 + j] = e;
    }
    cp_wait<0>();  // this thread's V copies (the barriers below publish them)
    cluster_arrive();
    cluster_wait();
    probe.mark();  // 5: the exps and their exchange

    // ---- 3. every CTA: the ordered sum, then the products and chains of its dimensions
    if (tid == 0) s_inv = __frcp_rn(ordered_sum(E, n));  // = 1.0f / sum (IEEE round to nearest)
    __syncthreads();
    probe.mark();  // 6: the softmax sum
    const float inv = s_inv;
    float o = 0.f;
    if (producer) {
        // block b: products of rows [128 b, ..) and dims [d0, d0 + dpc) into buffer b % 2, once the chains are done
        // with block b - 2
        const int ptid = tid - kOutThreads;
        constexpr int hp = dpc / 2;
        for (int b = 0; b < nblk; ++b) {
            if (b >= 2) {
                if (b & 1) bar_sync<kBarFree + 1>(kThreads);
                else bar_sync<kBarFree>(kThreads);
            }
            const int r0 = b * pbr, rows = min(pbr, n - r0);
            const __half2* v2 = reinterpret_cast<const __half2*>(vs + size_t(r0) * dpc);
            float* pbuf = prod + (b & 1) * dpc * pbs;
            for (int i = ptid; i < rows * hp; i += kProducers) {
                const int j = i / hp, q = i - j * hp;
                const float aj = fmul(E[r0 + j], inv);
                const float2 v = __half22float2(v2[i]);
                pbuf[(2 * q) * pbs + j] = fmul(aj, v.x);
                pbuf[(2 * q + 1) * pbs + j] = fmul(aj, v.y);
            }
            if (b & 1) bar_arrive<kBarFull + 1>(kThreads);
            else bar_arrive<kBarFull>(kThreads);
        }
    } else {
        // chain lanes tid < dpc: dimension d0 + tid, o = ((0 + p_0) + p_1) + ... in position order, 16 rows ahead
        for (int b = 0; b < nblk; ++b) {
            if (b & 1) bar_sync<kBarFull + 1>(kThreads);
            else bar_sync<kBarFull>(kThreads);
            const int rows = min(pbr, n - b * pbr);
            if (tid < dpc) o = ordered_sum(prod + ((b & 1) * dpc + tid) * pbs, rows, o);  // float4 loads ahead of the adds
            if (b + 2 < nblk) {  // the producers of block b + 2 wait for it
                if (b & 1) bar_arrive<kBarFree + 1>(kThreads);
                else bar_arrive<kBarFree>(kThreads);
            }
        }
        if (tid < dpc) out[(size_t(t) * a.n_heads + h) * kHd + d0 + tid] = o;
        probe.mark();  // 7: the output chains
    }
    if constexpr (UO > 0) {  // every CTA: the head's outputs, their quantization, this CTA's o_proj terms
        __shared__ __align__(16) int8_t sxo[kHd];
        __shared__ float sdo[kHd / QK];
        if (tid < dpc) {
#pragma unroll
            for (int q = 0; q < CS; ++q) cluster.map_shared_rank(so, q)[d0 + tid] = o;
        }
        cluster_arrive();
        cluster_wait();
        if (tid < kHd) {  // warp w quantizes block 2 h + w
            float d;
            sxo[tid] = quantize_lane(so[tid], &d);
            if (lane == 0) sdo[warp] = d;
        }
        __syncthreads();
#pragma unroll
        for (int u = 0; u < UO; ++u) {  // a block's two chunks sit in adjacent lanes
            const int f = u * kThreads + tid, c = f & 3;
            const bool ok = (f >> 2) < onr;
            int sdot = ok ? chunk_dot<DT_Q8_0>(wo[u], sxo, c) : 0;
            sdot += __shfl_xor_sync(0xffffffffu, sdot, 1);
            if (ok && !(c & 1))
                oa.T[size_t(orow0 + (f >> 2)) * onb + 2 * h + (c >> 1)] = block_term(sdot, __half2float(wdo[u]), sdo[c >> 1]);
        }
    } else if (a.xq && n_tok == 1) {  // quantize_q8 of the head's 64 outputs in the leader: warp w holds block 2 h + w
        if (tid < dpc) cluster.map_shared_rank(so, 0)[d0 + tid] = o;
        cluster_arrive();
        cluster_wait();
        if (r == 0 && tid < kHd) {
            float d;
            a.xq[h * kHd + tid] = quantize_lane(so[tid], &d);
            if (lane == 0) a.dx[h * (kHd / QK) + warp] = d;
        }
    }
    probe.end();  // 8: o_proj terms (or the output's quantization)
}


// ---------------------------------------------------------------- multi-token (prefill) attention

// One CTA per (kv head, token), 256 threads: warp h owns query head g * group + h.  K and V stream through one shared
// tile (f32, converted once for all the group's heads); each warp keeps its head's scores / weights in shared memory
// and runs its own ordered sums: lane 0 the softmax sum, every lane two output dimensions (lane, lane + 32).
constexpr int kGmax = kWarps;                   // query heads per kv head: one warp each
constexpr int kPfTile = 128;                    // positions per K / V tile
constexpr int kPfStride = kHd + 1;              // f32 K tile row stride (conflict-free column walks)
constexpr int kPfStrideV = kHd + 2;             // f32 V tile row stride (8-byte aligned dimension pairs)
constexpr int kPfTileBytes = kPfTile * kPfStrideV * 4;

// Scores of the first NG 32-position groups of a K tile for one query head (lane l: positions l, l + 32, ...): each
// the dimension-order sum of the rounded products q_i * k_i.
template <int NG>
__device__ __forceinline__ void pf_scores(const float* qh, const float* tile, int lane, float (&sc)[4]) {
#pragma unroll 8
    for (int i = 0; i < kHd; ++i) {
        const float qi = qh[i];
#pragma unroll
        for (int u = 0; u < NG; ++u) sc[u] = fadd(sc[u], fmul(qi, tile[(lane + 32 * u) * kPfStride + i]));
    }
}

__global__ void __launch_bounds__(kThreads) k_attn_prefill(AttnArgs a, const float* __restrict__ Q,
                                                           const int* __restrict__ pos_dev, int n_cap,
                                                           float* __restrict__ out, TokMap tm, QuantOut qo) {
    extern __shared__ __align__(16) unsigned char smem[];
    float* sq = reinterpret_cast<float*>(smem);                    // [kGmax][kHd]
    float* tile = sq + kGmax * kHd;                                // [kPfTile][kPfStride] K, [kPfTile][kPfStrideV] V
    float* E = tile + kPfTile * kPfStrideV;                        // [group][ecap]
    pdl_wait();
    pdl_launch_dependents();
    // the last tokens attend to the most positions: they take the lowest block indices, so the longest CTAs start
    // first and the short ones fill in behind them
    const int g = blockIdx.x, t = int(gridDim.y) - 1 - int(blockIdx.y);
    const int group = a.n_heads / a.n_kv;
    const int n = (tm.pos ? __ldcg(tm.pos + t) : __ldcg(pos_dev) + t) + 1;
    if (tm.pos) {  // this token's sequence cache
        const long long off = __ldcg(tm.off + t);
        a.kcache += off;
        a.vcache += off;
    }
    const int ecap = (n_cap + 3) & ~3;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool head = warp < group;
    float* Eh = E + warp * ecap;
    for (int i = tid; i < group * kHd; i += kThreads) sq[i] = __ldcg(Q + (size_t(t) * a.n_heads + size_t(g) * group) * kHd + i);
    // loads the rows [p, p + kPfTile) of C (this kv head) as f32 into the tile; 4 granules of 16 bytes per thread
    constexpr int U = kPfTile * 8 / kThreads;
    uint4 buf[U];
    auto fetch = [&](const __half* C, int p) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = u * kThreads + tid, row = i >> 3;
            buf[u] = p + row < n ? __ldcg(reinterpret_cast<const uint4*>(C + size_t(p + row) * a.kv_dim + g * kHd) + (i & 7))
                                 : make_uint4(0, 0, 0, 0);
        }
    };
    auto store = [&](int stride) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = u * kThreads + tid, row = i >> 3, c8 = (i & 7) * 8;
            const __half2* h2 = reinterpret_cast<const __half2*>(&buf[u]);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = __half22float2(h2[k]);
                tile[row * stride + c8 + 2 * k] = f.x;
                tile[row * stride + c8 + 2 * k + 1] = f.y;
            }
        }
    };
    // ---- scores, four positions per lane per tile
    float lmax = -INFINITY;
    fetch(a.kcache, 0);
    for (int p = 0; p < n; p += kPfTile) {
        __syncthreads();  // the previous tile's readers are done (and the queries are visible)
        store(kPfStride);
        __syncthreads();
        if (p + kPfTile < n) fetch(a.kcache, p + kPfTile);  // next tile in flight during this one's dots
        if (head) {
            const float* qh = sq + warp * kHd;
            float sc[4] = {0.f, 0.f, 0.f, 0.f};
            const int groups = (min(kPfTile, n - p) + 31) >> 5;  // 32-position groups of the tile inside [0, n)
            if (groups == 4) pf_scores<4>(qh, tile, lane, sc);
            else if (groups == 3) pf_scores<3>(qh, tile, lane, sc);
            else if (groups == 2) pf_scores<2>(qh, tile, lane, sc);
            else pf_scores<1>(qh, tile, lane, sc);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int j = p + lane + 32 * u;
                if (j < n) {
                    const float v = fmul(sc[u], a.scale);
                    Eh[j] = v;
                    lmax = fmaxf(lmax, v);
                }
            }
        }
    }
    // ---- softmax of this warp's head: exps in parallel, the sum in position order on lane 0
    float inv = 0.f;
    if (head) {
        const float m = warp_max(lmax);
        for (int j = lane; j < n; j += 32) Eh[j] = exp_ref(fsub(Eh[j], m), a.exptab);
        __syncwarp();
        if (lane == 0) inv = __frcp_rn(ordered_sum(Eh, n));  // = 1.0f / sum (IEEE round to nearest)
        inv = __shfl_sync(0xffffffffu, inv, 0);
        for (int j = lane; j < n; j += 32) Eh[j] = fmul(Eh[j], inv);
        __syncwarp();
    }
    // ---- outputs in position order, dimensions (2 lane, 2 lane + 1) per lane as one f32x2 pair: the product
    // a_j * v_jd as fma(v, a, -0.0) (exactly fmul's rounding; a mul feeding the add would be contracted), then the add
    float2 o2 = make_float2(0.f, 0.f);
    const float2 nz2 = make_float2(a.neg_zero, a.neg_zero);
    fetch(a.vcache, 0);
    for (int p = 0; p < n; p += kPfTile) {
        __syncthreads();
        store(kPfStrideV);
        __syncthreads();
        if (p + kPfTile < n) fetch(a.vcache, p + kPfTile);
        if (head) {
            const int rows = min(kPfTile, n - p);
            const float* e = Eh + p;
            const float2* v2 = reinterpret_cast<const float2*>(tile) + lane;
            int j = 0;
            for (; j + 8 <= rows; j += 8) {
                float av[8];
                float2 vv[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    av[k] = e[j + k];
                    vv[k] = v2[(j + k) * (kPfStrideV / 2)];
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) o2 = __fadd2_rn(o2, __ffma2_rn(vv[k], make_float2(av[k], av[k]), nz2));
            }
            for (; j < rows; ++j) o2 = __fadd2_rn(o2, __ffma2_rn(v2[j * (kPfStrideV / 2)], make_float2(e[j], e[j]), nz2));
        }
    }
    if (head) {
        const int hh = g * group + warp;
        if (qo.xq) {  // quantize_q8 of the head's two 32-blocks: lanes 0-15 hold block 2 hh, lanes 16-31 block 2 hh + 1
            float amax = fmaxf(fabsf(o2.x), fabsf(o2.y));
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const float d = div127(amax);
            const float inv = d > 0.f ? __frcp_rn(d) : 0.0f;
            const int dim = a.n_heads * kHd, b = 2 * hh + (lane >> 4);
            char2 qv;
            qv.x = (signed char)round_away(fmul(o2.x, inv));
            qv.y = (signed char)round_away(fmul(o2.y, inv));
            reinterpret_cast<char2*>(qo.xq + size_t(t) * dim + hh * kHd)[lane] = qv;
            if ((lane & 15) == 0) {
                qo.dx[size_t(t) * (dim / QK) + b] = d;
                if (qo.dxt) qo.dxt[size_t(b) * qo.ldt + t] = d;
            }
        } else {
            float2* o = reinterpret_cast<float2*>(out + (size_t(t) * a.n_heads + hh) * kHd);
            o[lane] = o2;
        }
    }
}

inline size_t prefill_smem_bytes(int group, int n_cap) {
    return size_t(kGmax) * kHd * 4 + size_t(kPfTileBytes) + size_t(group) * ((n_cap + 3) & ~3) * 4;
}

}  // namespace

QNT_PHASE_READER(qnt_phase_read_attn)

cudaError_t launch_attn_prefill(const AttnArgs& a, const float* Q, const int* pos_dev, int n_tok, int pos_bound, float* out,
                                cudaStream_t st, bool pdl, TokMap tm, const QuantOut* qo) {
    const int group = a.n_kv > 0 ? a.n_heads / a.n_kv : 0;
    if (a.head_dim != kHd || group < 1 || group > kGmax || group * a.n_kv != a.n_heads || pos_bound < (tm.pos ? 1 : n_tok))
        return cudaErrorInvalidValue;
    const size_t smem = prefill_smem_bytes(group, pos_bound);
    if (smem > 227 * 1024) {  // very long contexts (single sequence only)
        if (tm.pos) return cudaErrorInvalidValue;
        cudaError_t e = launch_attn(a, Q, pos_dev, n_tok, out, st, pdl);
        if (e == cudaSuccess && qo)
            e = launch_norm_quant_rows(out, nullptr, n_tok, a.n_heads * kHd, 0.f, qo->xq, qo->dx, qo->dxt, qo->ldt, st, pdl);
        return e;
    }
    return launch_pdl(k_attn_prefill, dim3(a.n_kv, n_tok), dim3(kThreads), smem, st, pdl, a, Q, pos_dev, pos_bound, out, tm,
                      qo ? *qo : QuantOut{});
}

cudaError_t launch_attn(const AttnArgs& a, const float* Q, const int* pos_dev, int n_tok, float* out, cudaStream_t st, bool pdl) {
    const int group = a.n_kv > 0 ? a.n_heads / a.n_kv : 0;
    if (a.head_dim != kHd || group < 1 || group * a.n_kv != a.n_heads || a.max_chunks < 1) return cudaErrorInvalidValue;
    const int ctx = a.max_chunks * kPosChunk;
    // a cluster of cs CTAs per (head, token): the largest power of two up to 8 and the chunk count
    int cs = 1;
    while (cs * 2 <= std::min(kMaxCluster, a.max_chunks)) cs *= 2;
    auto kern = cs == 8 ? k_attn<8, 0, 0> : cs == 4 ? k_attn<4, 0, 0> : cs == 2 ? k_attn<2, 0, 0> : k_attn<1, 0, 0>;
    const size_t smem = attn_smem_bytes(ctx, cs);
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(cs * a.n_heads), unsigned(n_tok));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(cs);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, a, QkvArgs{}, OArgs{}, static_cast<const float*>(nullptr), static_cast<const float*>(nullptr),
                              0.f, static_cast<float*>(nullptr), Q, pos_dev, n_tok, out);
}

namespace {
// weight chunks per thread of the fused forms: q|k|v (24 rows per CTA), o_proj (an eighth of the rows, 4 chunks each)
int qkv_uw(int dim) { return (kQkvRows * (dim / 16) + kThreads - 1) / kThreads; }
int o_uo(const DMat& o) { return ((o.rows + kMaxCluster - 1) / kMaxCluster * 4 + kThreads - 1) / kThreads; }
}  // namespace

bool qkv_attn_supported(const QkvArgs& qa, const AttnArgs& a, const DMat* o) {
    const int group = a.n_kv > 0 ? a.n_heads / a.n_kv : 0;
    const int dim = qa.W.cols;
    if (a.head_dim != kHd || group < 1 || group * a.n_kv != a.n_heads || a.max_chunks < kMaxCluster ||
        qa.W.dtype != DT_Q8_0 || qa.head_dim != kHd || dim % QK != 0 || dim > kMaxRounds * kThreads ||
        qa.W.rows != (a.n_heads + 2 * a.n_kv) * kHd || qkv_uw(dim) > 12)
        return false;
    if (o && (o->dtype != DT_Q8_0 || o->cols != a.n_heads * kHd || o_uo(*o) > 4 || o->rows < kMaxCluster)) return false;
    const size_t smem = attn_smem_bytes(a.max_chunks * kPosChunk, kMaxCluster) + qkv_smem_bytes(dim);
    return smem <= 227 * 1024;
}

cudaError_t launch_qkv_attn(const QkvArgs& qa, const AttnArgs& a, const float* X, const float* norm_w, float eps,
                            const int* pos_dev, float* Qout, float* out, cudaStream_t st, bool pdl, const OArgs* o) {
    // the fused form covers the decode shapes it was built for; anything else takes the separate kernels
    if (!qkv_attn_supported(qa, a, o ? &o->W : nullptr)) return cudaErrorNotSupported;
    const int dim = qa.W.cols;
    const size_t smem = attn_smem_bytes(a.max_chunks * kPosChunk, kMaxCluster) + qkv_smem_bytes(dim);
    const bool u6 = qkv_uw(dim) <= 6;
    const int uo = o ? (o_uo(o->W) <= 2 ? 2 : 4) : 0;
    auto kern = uo == 0 ? (u6 ? k_attn<kMaxCluster, 6, 0> : k_attn<kMaxCluster, 12, 0>)
              : uo == 2 ? (u6 ? k_attn<kMaxCluster, 6, 2> : k_attn<kMaxCluster, 12, 2>)
                        : (u6 ? k_attn<kMaxCluster, 6, 4> : k_attn<kMaxCluster, 12, 4>);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(kMaxCluster * a.n_heads), 1u);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(kMaxCluster);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, a, qa, o ? *o : OArgs{}, X, norm_w, eps, Qout, static_cast<const float*>(nullptr),
                              pos_dev, 1, out);
}

}  // namespace qb
