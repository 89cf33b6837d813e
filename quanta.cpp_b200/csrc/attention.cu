// GQA attention over the f16 KV cache (engine/src/model.cpp:115-137), bit-identical to the reference.
//
// Query token t sits at position pos = pos0 + t and attends to [0, pos] in the reference's order:
//   score  s_j = (sum_i q_i * k_ji in dimension order) * scale
//   max    m = max_j s_j                                   (exact in any order)
//   weight e_j = exp(s_j - m); sum = e_0 + e_1 + ... in position order; a_j = e_j * (1 / sum)
//   output o_i = a_0 v_0i + a_1 v_1i + ... in position order
// The two sums are sequential chains (the reference's float order), so each query head gets its own SM resources:
// one thread-block cluster of CS CTAs per (query head, token), grid (CS * n_heads, n_tok), 256 threads per CTA.
//   1. CTA r of the cluster scores the contiguous positions [r P, r P + P) (P = ceil((pos + 1) / CS)), one thread per
//      position (K tiles staged as f32 in shared memory), and posts its local maximum to the leader (rank 0) through
//      distributed shared memory.
//   2. cluster barrier; every CTA reads the CS maxima, exponentiates its own scores and stores the weights straight
//      into the leader's weight row (distributed shared memory).
//   3. cluster barrier; the other CTAs exit.  The leader sums the row in position order on one thread, normalises it,
//      and two warps chain the outputs (one lane per dimension) over V rows that stream through a cp.async ring the
//      leader filled from its first instruction on.
// Decode launches CS = min(8, chunks); multi-token (prefill) launches use CS = 1, one CTA per (head, token), which
// keeps the SMs busy with many tokens at once.  The cluster barriers are hardware barriers (no spin loops).
#include <cooperative_groups.h>

#include "kernels.cuh"
#include "layer_kernels.h"

namespace qb {

namespace cg = cooperative_groups;

namespace {

constexpr int kPosChunk = 64;       // KV positions per chunk (the unit of max_chunks)
constexpr int kHd = 64;             // supported head_dim
constexpr int kTile = 128;          // positions scored per K tile (one thread each)
constexpr int kVBlk = 64;           // V rows per ring slot
constexpr int kRing = 4;            // V ring slots
constexpr int kOutThreads = 64;     // output threads of the leader (one per dimension)
constexpr int kMaxCluster = 8;      // portable cluster size limit
constexpr int kKfStride = kHd + 1;  // f32 K tile row stride (conflict-free column walks)

// Dynamic shared memory layout (byte offsets): the same for every CTA of a launch.
constexpr int kOffQ = 0;                                       // f32 [kHd] query
constexpr int kOffMax = kOffQ + kHd * 4;                       // f32 [kMaxCluster] local maxima (leader's copy used)
constexpr int kOffKf = kOffMax + 256;                          // f32 [kTile][kKfStride] K tile
constexpr int kOffRing = kOffKf + kTile * kKfStride * 4;       // f16 [kRing][kVBlk][kHd] V ring (leader)
constexpr int kOffLs = kOffRing + kRing * kVBlk * kHd * 2;     // f32 [lsmax] own scores, then f32 [ctx] weights
static_assert(kOffKf % 16 == 0 && kOffRing % 16 == 0 && kOffLs % 16 == 0, "16-byte aligned regions");
static_assert(kThreads == 256 && kTile * 8 % kThreads == 0, "K tile loader");

__host__ __device__ inline int ls_len(int ctx, int cs) { return ((ctx + cs - 1) / cs + 3) & ~3; }
inline size_t attn_smem_bytes(int ctx, int cs) { return size_t(kOffLs) + size_t(ls_len(ctx, cs)) * 4 + size_t(ctx) * 4; }

__device__ __forceinline__ void bar_out() { asm volatile("bar.sync 1, %0;" ::"n"(kOutThreads) : "memory"); }

__global__ void __launch_bounds__(kThreads) k_attn(AttnArgs a, const float* __restrict__ Q, const int* __restrict__ pos_dev,
                                                   int n_tok, float* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const int CS = int(cluster.num_blocks()), r = int(cluster.block_rank());
    const int h = blockIdx.x / CS, t = blockIdx.y;
    const int group = a.n_heads / a.n_kv, g = h / group;
    const int ctx = a.max_chunks * kPosChunk;
    float* sq = reinterpret_cast<float*>(smem + kOffQ);
    float* smx = reinterpret_cast<float*>(smem + kOffMax);
    float* kf = reinterpret_cast<float*>(smem + kOffKf);
    __half* ring = reinterpret_cast<__half*>(smem + kOffRing);
    float* LS = reinterpret_cast<float*>(smem + kOffLs);
    float* E = LS + ls_len(ctx, CS);
    __shared__ float sred[kWarps];
    __shared__ float s_m, s_inv;
    pdl_launch_dependents();
    pdl_wait();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n = __ldcg(pos_dev) + t + 1;
    const int P = (n + CS - 1) / CS, p0 = min(n, r * P), p1 = min(n, p0 + P);
    const bool leader = r == 0, out_thread = tid < kOutThreads;
    const int nblk = (n + kVBlk - 1) / kVBlk;
    const __half* V = a.vcache + g * kHd;
    auto issue_v = [&](int b) {  // V rows [64 b, min(64 b + 64, n)) into slot b % kRing; an empty group past the end
        if (b < nblk) {
            const int r0 = b * kVBlk, rows = min(kVBlk, n - r0);
            __half* dst = ring + (b % kRing) * kVBlk * kHd;
            for (int i = tid; i < rows * 8; i += kOutThreads)
                cp_async16(dst + (i >> 3) * kHd + (i & 7) * 8, V + size_t(r0 + (i >> 3)) * a.kv_dim + (i & 7) * 8);
        }
        cp_commit();
    };
    if (leader && out_thread)
        for (int b = 0; b < kRing - 1; ++b) issue_v(b);
    if (tid < kHd) sq[tid] = __ldcg(Q + (size_t(t) * a.n_heads + h) * kHd + tid);

    // ---- 1. scores of [p0, p1), one position per thread
    const __half* K = a.kcache + g * kHd;
    for (int tile0 = p0; tile0 < p1; tile0 += kTile) {
        const int tl = min(kTile, p1 - tile0);
        constexpr int U = kTile * 8 / kThreads;
        uint4 kv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = u * kThreads + tid, row = i >> 3;
            kv[u] = row < tl ? __ldcg(reinterpret_cast<const uint4*>(K + size_t(tile0 + row) * a.kv_dim) + (i & 7))
                             : make_uint4(0, 0, 0, 0);
        }
        __syncthreads();  // the previous tile's readers are done (and the query is visible)
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = u * kThreads + tid, row = i >> 3, c8 = (i & 7) * 8;
            const __half2* h2 = reinterpret_cast<const __half2*>(&kv[u]);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = __half22float2(h2[k]);
                kf[row * kKfStride + c8 + 2 * k] = f.x;
                kf[row * kKfStride + c8 + 2 * k + 1] = f.y;
            }
        }
        __syncthreads();
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
    float* lead_max = cluster.map_shared_rank(smx, 0);
    if (tid == 0) {
        float m = sred[0];
        for (int k = 1; k < kWarps; ++k) m = fmaxf(m, sred[k]);
        lead_max[r] = m;
    }
    cluster.sync();

    // ---- 2. weights of [p0, p1) into the leader's row
    if (warp == 0) {
        float m = lane < CS ? lead_max[lane] : -INFINITY;
        m = warp_max(m);
        if (lane == 0) s_m = m;
    }
    __syncthreads();
    {
        float* lead_E = cluster.map_shared_rank(E, 0);
        const float m = s_m;
        for (int j = tid; j < p1 - p0; j += kThreads) lead_E[p0 + j] = exp_ref(fsub(LS[j], m), a.exptab);
    }
    cluster.sync();
    if (!leader) return;

    // ---- 3. leader: ordered sum, normalise, output chains
    if (tid == 0) {
        float sum = 0.f;
        int j = 0;
        for (; j + 8 <= n; j += 8) {
            const float4 v0 = *reinterpret_cast<const float4*>(E + j);
            const float4 v1 = *reinterpret_cast<const float4*>(E + j + 4);
            sum = fadd(sum, v0.x);
            sum = fadd(sum, v0.y);
            sum = fadd(sum, v0.z);
            sum = fadd(sum, v0.w);
            sum = fadd(sum, v1.x);
            sum = fadd(sum, v1.y);
            sum = fadd(sum, v1.z);
            sum = fadd(sum, v1.w);
        }
        for (; j < n; ++j) sum = fadd(sum, E[j]);
        s_inv = fdiv(1.0f, sum);
    }
    __syncthreads();
    {
        const float iv = s_inv;
        for (int j = tid; j < n; j += kThreads) E[j] = fmul(E[j], iv);
    }
    __syncthreads();
    if (!out_thread) return;
    float o = 0.f;
    for (int b = 0; b < nblk; ++b) {
        issue_v(b + kRing - 1);
        cp_wait<kRing - 1>();
        bar_out();
        const int rows = min(kVBlk, n - b * kVBlk);
        const float* e = E + b * kVBlk;
        const __half* v = ring + (b % kRing) * kVBlk * kHd + tid;
        int j = 0;
        for (; j + 8 <= rows; j += 8) {
            float av[8], vv[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                av[k] = e[j + k];
                vv[k] = __half2float(v[(j + k) * kHd]);
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) o = fadd(o, fmul(av[k], vv[k]));
        }
        for (; j < rows; ++j) o = fadd(o, fmul(e[j], __half2float(v[j * kHd])));
        bar_out();  // slot b % kRing is free again
    }
    cp_wait<0>();
    out[(size_t(t) * a.n_heads + h) * kHd + tid] = o;
}

}  // namespace

cudaError_t launch_attn(const AttnArgs& a, const float* Q, const int* pos_dev, int n_tok, float* out, cudaStream_t st, bool pdl) {
    const int group = a.n_kv > 0 ? a.n_heads / a.n_kv : 0;
    if (a.head_dim != kHd || group < 1 || group * a.n_kv != a.n_heads || a.max_chunks < 1) return cudaErrorInvalidValue;
    const int ctx = a.max_chunks * kPosChunk;
    const int cs = n_tok == 1 ? std::min(kMaxCluster, a.max_chunks) : 1;
    const size_t smem = attn_smem_bytes(ctx, cs);
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(k_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
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
    return cudaLaunchKernelEx(&cfg, k_attn, a, Q, pos_dev, n_tok, out);
}

}  // namespace qb
