// Tensor-core (tcgen05) int8 matmul for prefill chunks and batched decode: out[t * ldo + r] for weight rows r in
// [r0, r1) and tokens t in [0, n), bit-identical to the CUDA-core matmul and to matvec_q_ref
// (engine/src/ops_ref.cpp:122-160): per (row, token) acc = acc + (float(s_b) * dw_b) * dx_b over the 32-blocks b in
// order, s_b the exact int32 block dot.
//
// The per-block scales rule out accumulating across blocks in the tensor core: every block's int32 dot has to leave
// the MMA on its own.  A tcgen05.mma.kind::i8 step is K = 32 deep, exactly one quant block, so each block gets one
// MMA (M = 128 weight rows, N = 32 tokens) into 32 TMEM columns of its own; a TMEM slot of 128 columns holds the four
// blocks of a pipeline stage.  Tiles of 128 weight rows x 32 tokens; persistent CTAs (one per SM) walk their tiles
// with the pipeline running across tile boundaries.
// Weights are int8 rows: Q8_0 as stored, Q4_0 through an int8 copy of q - 8 made once (tc_prepare_weights).
// A TMA instruction costs the SM about the same whatever its size (about 0.12 us of its TMA unit), so each one moves
// two K-steps: a stage is 2 x (128 weight rows x 128 B) and 2 x (32 tokens x 128 B), 128B-swizzled, through 3-D
// tensor maps, and the stage's block scales (weights: 4 f16 per row and K-step, from a stage-major copy; activations:
// f32 [block][token], from a block-major copy) come in two more loads into a deeper ring that the epilogue frees.
//   warp 0      TMA producers, one lane per kind of load (weights, activations, weight scales, activation scales)
//               and parity of the stage (a thread's bulk loads complete one after another)
//   warp 1      allocates TMEM; one lane issues each K-step's four MMAs into one of four TMEM slots; the stage is
//               free again when its last MMA completes
//   warps 4-19  epilogue: warp w reads TMEM lanes 32 (w % 4) .. +32 (its 32 weight rows) and, for each block, the
//               columns of tokens 8 ((w - 4) / 4) .. +8, and folds the four blocks into 8 f32 accumulators per
//               thread in block order, two tokens per instruction (f32x2: every lane rounds as the scalar op)
// Every wait is bounded: a wait that gives up sets ERR_WAIT_TIMEOUT in the status word and an abort flag that ends
// every other wait, so the kernel always returns (and frees its TMEM once its issued MMAs have completed).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <vector>
#include <mutex>

#include <climits>

#include "gemm_tc.h"
#include "head_kernels.h"
#include "kernels.cuh"
#include "qkv_pair.cuh"

namespace qb {

namespace {

constexpr int kEpiWarps = 16;
constexpr int kTcThreads = 128 + 32 * kEpiWarps;
constexpr int kTileRows = 128;
constexpr int kStageBlocks = 4;                    // quant blocks per K-step (128 bytes of K)
constexpr int kSlots = 4;                          // TMEM accumulator slots (one K-step each)
constexpr int kASw = kTileRows * 128;              // swizzled int8 weight tile of a K-step
constexpr int kKPS = 2;                            // K-steps per stage (per TMA instruction)
constexpr int kStages = 4;
constexpr int kDWRows = kTileRows + 2;             // weight-scale rows per load (from an even row: 16-byte start)
constexpr int kEpiDW = 2176;                       // weight scales of a stage: [K-step][kDWRows] x 4 f16 (padded)
constexpr int kEpiRing = 8;                        // >= stages + slots / kKPS: the scales never hold the producer back

// Token tiles of TOK = 32 tokens, or 16 where a matrix has too few 32-token tiles to fill the SMs (twice the tiles,
// each with half the epilogue work).
template <int TOK>
struct Tc {
    static constexpr int cols = TOK * kStageBlocks;         // TMEM columns of a K-step: block b of token t in column TOK b + t
    static constexpr int tpt = TOK / 4;                     // tokens per epilogue thread
    static constexpr int tmem_cols = kSlots * cols;         // 512 / 256 (a power of two, as tcgen05.alloc requires)
    static constexpr int b = TOK * 128;                     // activation tile of a K-step
    static constexpr int stage_bytes = kKPS * (kASw + b);   // kKPS weight tiles, then kKPS activation tiles
    static constexpr int epi_dx = kKPS * kStageBlocks * TOK * 4;  // activation scales of a stage: [block][token] f32
    static constexpr int epi = epi_dx + kEpiDW;             // epilogue ring entry (TMA destinations 128-byte aligned)
    static constexpr int swi_bytes = 2 * 8 * 32 * tpt * 4;  // EPI 3: silu(gate) of each gate warp, per tile parity
    // instruction descriptor: int32 accumulator, signed int8 A and B, both K-major, M = 128, N = TOK
    static constexpr uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(TOK >> 3) << 17) | (uint32_t(kTileRows >> 4) << 24);
    static_assert(epi % 128 == 0 && (tmem_cols & (tmem_cols - 1)) == 0, "ring entries and TMEM allocation");
};
constexpr unsigned kWaitLimit = 1u << 22;
constexpr unsigned kSuspendHintNs = 20000;  // a waiting thread sleeps (up to this long) instead of spinning

__device__ __forceinline__ unsigned smem_u32(const void* p) { return static_cast<unsigned>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    return ok != 0;
}
// Bounded wait: false when it gave up after `limit` tries or another role aborted (then the caller unwinds).
__device__ __forceinline__ bool mbar_wait(uint64_t* b, unsigned parity, volatile int* abort_flag, unsigned* status,
                                          unsigned limit = kWaitLimit) {
    for (unsigned i = 0; i < limit; ++i) {
        if (mbar_try(b, parity)) return true;
        if (*abort_flag) return false;
    }
    *abort_flag = 1;
    set_error(status, ERR_WAIT_TIMEOUT);
    return false;
}

// The same bounded wait run by a whole warp: every lane polls and a vote makes the outcome warp-uniform (a lane that
// saw the phase complete polls again until all have; a completed phase keeps reading as complete until the barrier
// moves on, which needs this warp's own arrival).
__device__ __forceinline__ bool warp_wait(uint64_t* b, unsigned parity, volatile int* abort_flag, unsigned* status) {
    for (unsigned i = 0; i < kWaitLimit; ++i) {
        if (__all_sync(0xffffffffu, mbar_try(b, parity))) return true;
        if (__any_sync(0xffffffffu, *abort_flag != 0)) return false;
    }
    *abort_flag = 1;
    set_error(status, ERR_WAIT_TIMEOUT);
    return false;
}

// The timeout path of the waits above, on its own: one thread waits on an mbarrier that nothing arrives on, with the
// given limit, so the wait runs out, sets ERR_WAIT_TIMEOUT and the kernel returns (no copies or MMAs in flight).
__global__ void k_wait_probe(unsigned limit, unsigned* status) {
    __shared__ uint64_t never;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&never, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        mbar_wait(&never, 0, &abort_flag, status, limit);
    }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms 1024 bytes apart (tcgen05 format).
__device__ __forceinline__ uint64_t sw128_desc(const void* p) {
    const uint64_t addr = smem_u32(p);
    uint64_t d = (addr >> 4) & 0x3FFF;      // start address
    d |= uint64_t(1) << 16;                 // leading byte offset (unused for swizzled K-major)
    d |= uint64_t(1024 >> 4) << 32;         // stride byte offset: next 8-row atom
    d |= uint64_t(1) << 46;                 // descriptor version (sm_100)
    d |= uint64_t(2) << 61;                 // layout: 128B swizzle
    return d;
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate ? 1 : 0), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// registers -> TMEM: this warp's 32 lanes, NC columns at each of taddr + 4 NC b (b = 0..3), all set to x.
template <int NC>
__device__ __forceinline__ void tmem_fill(uint32_t taddr, unsigned x) {
    if constexpr (NC == 8) {
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%4,%4,%4,%4,%4,%4,%4,%4};\n\t"
            "tcgen05.st.sync.aligned.32x32b.x8.b32 [%1], {%4,%4,%4,%4,%4,%4,%4,%4};\n\t"
            "tcgen05.st.sync.aligned.32x32b.x8.b32 [%2], {%4,%4,%4,%4,%4,%4,%4,%4};\n\t"
            "tcgen05.st.sync.aligned.32x32b.x8.b32 [%3], {%4,%4,%4,%4,%4,%4,%4,%4};\n\t"
            "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
            "r"(taddr + 32u), "r"(taddr + 64u), "r"(taddr + 96u), "r"(x)
            : "memory");
    } else {
        static_assert(NC == 4, "4 or 8 columns per block");
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%4,%4,%4,%4};\n\t"
            "tcgen05.st.sync.aligned.32x32b.x4.b32 [%1], {%4,%4,%4,%4};\n\t"
            "tcgen05.st.sync.aligned.32x32b.x4.b32 [%2], {%4,%4,%4,%4};\n\t"
            "tcgen05.st.sync.aligned.32x32b.x4.b32 [%3], {%4,%4,%4,%4};\n\t"
            "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
            "r"(taddr + 16u), "r"(taddr + 32u), "r"(taddr + 48u), "r"(x)
            : "memory");
    }
}

// TMEM -> registers: this warp's 32 lanes, NC consecutive 32-bit columns at each of taddr + 4 NC b (b = 0..3):
// v[NC b + i] = column 4 NC b + i.  One load and its wait per block.
template <int NC>
__device__ __forceinline__ void tmem_ld_blocks(uint32_t taddr, int* v) {
    if constexpr (NC == 4) {  // the four blocks' loads in flight together, one wait
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%16];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%4,%5,%6,%7}, [%17];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%8,%9,%10,%11}, [%18];\n\t"
            "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%12,%13,%14,%15}, [%19];\n\t"
            "tcgen05.wait::ld.sync.aligned;"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
              "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
            : "r"(taddr), "r"(taddr + 16u), "r"(taddr + 32u), "r"(taddr + 48u)
            : "memory");
    } else {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const uint32_t ta = taddr + uint32_t(4 * NC * b);
            int* w = v + NC * b;
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n\t"
                "tcgen05.wait::ld.sync.aligned;"
                : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
                : "r"(ta)
                : "memory");
        }
    }
}

// The accumulators start at the bits of 2^23 + 2^22 (kMagic): the MMA then leaves 12582912 + s, whose float value
// carries the exact block dot s (|s| < 2^22), and fma(f, dw, -12582912 * dw) rounds s * dw once, exactly like
// fmul(float(s), dw): 12582912 * dw is exact in f32 for an fp16 dw.
constexpr unsigned kMagic = 0x4B400000u;
constexpr float kMagicF = 12582912.0f;




__device__ __forceinline__ bool cand_better(float av, int aid, float bv, int bid) {
    return av > bv || (av == bv && aid < bid);
}

// EPI 0: store the rows; EPI 1: per 32-row group and token, the best (value, id) into g.cand; EPI 2: add the rows onto
// out (the residual stream: out = out + row, the reference's separate residual add, one rounding); EPI 3: gate|up rows
// interleaved per 32-row block (gate block j = rows 64 j .., up block j = rows 64 j + 32 ..): the SwiGLU
// h = silu(gate) * up and its quantize_q8 per block go to g.hq / g.hd / g.hdt (the gate rows' quadrant passes
// silu(gate) to the up rows' quadrant through shared memory; one warp then holds a whole 32-block of h per token);
// EPI 4: fused q|k|v rows (pair-interleaved: rows 2 i, 2 i + 1 sit in adjacent lanes), the even lane of each pair
// applies bias and RoPE and stores q (f32) or the f16 K / V cache entry of each token.
// Programmatic dependent launch: the weight loads (and the set-up) need nothing from the previous kernel on the stream,
// so only the threads that read its outputs (the activation producers) or write this kernel's (the epilogue) wait.
template <int EPI, int TOK>
__global__ void __launch_bounds__(kTcThreads, 1) k_gemm_tc(const __grid_constant__ CUtensorMap tmA,
                                                           const __grid_constant__ CUtensorMap tmB,
                                                           const __grid_constant__ CUtensorMap tmDW,
                                                           const __grid_constant__ CUtensorMap tmDX, GemmTcArgs g) {
    using C = Tc<TOK>;
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte aligned (the 128-byte swizzle's period), as an offset from smem_raw so that loads stay shared-window
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    unsigned char* epi_ring = smem + kStages * C::stage_bytes;
    float* swi = reinterpret_cast<float*>(epi_ring + kEpiRing * C::epi);
    __shared__ uint64_t full[kStages], empty[kStages], mma_done[kSlots], slot_free[kSlots];
    __shared__ uint64_t epi_full[kEpiRing], epi_empty[kEpiRing], fin;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nks = g.nb / kStageBlocks, nst = (nks + kKPS - 1) / kKPS;  // K-steps and stages per tile
    const int n_tt = (g.n + TOK - 1) / TOK, n_tiles = ((g.r1 - g.r0 + kTileRows - 1) / kTileRows) * n_tt;
    // tile -> (first weight row, first token); tiles blockIdx.x, blockIdx.x + gridDim.x, ...
    auto tile_m0 = [&](int tile) { return g.r0 + (tile / n_tt) * kTileRows; };
    auto tile_t0 = [&](int tile) { return (tile % n_tt) * TOK; };
    const int my_tiles = (n_tiles - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x);
    pdl_launch_dependents();  // the next kernel waits for this grid's completion before it reads anything

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 2);   // the weight and activation producers (one arrive.expect_tx each)
            mbar_init(&empty[s], 1);  // the MMA commit
        }
        for (int j = 0; j < kSlots; ++j) {
            mbar_init(&mma_done[j], 1);
            mbar_init(&slot_free[j], kEpiWarps);
        }
        for (int d = 0; d < kEpiRing; ++d) {
            mbar_init(&epi_full[d], 2);  // the two scale producers
            mbar_init(&epi_empty[d], kEpiWarps);
        }
        mbar_init(&fin, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                     "r"(C::tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    volatile int* ab = &abort_flag;

    if (warp == 0) {
        if (lane < 8) {  // TMA producers: kind = lane / 2 (weights, activations, their scales), parity of the stage
            const int kind = lane >> 1, ph = lane & 1;
            if (kind & 1) pdl_wait();  // the activations and their scales come from the previous kernel
            int u = 0;
            bool go = true;
            for (int tile = blockIdx.x; tile < n_tiles && go; tile += gridDim.x) {
                const int m0 = tile_m0(tile), t0 = tile_t0(tile);
                for (int j = 0; j < nst; ++j, ++u) {
                    if ((u & 1) != ph) continue;
                    // full boxes: TMA zero-fills rows, tokens, K-chunks and blocks past the tensor
                    if (kind < 2) {
                        const int s = u % kStages, round = u / kStages;
                        if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1, ab, g.status)) {
                            go = false;
                            break;
                        }
                        unsigned char* st = smem + s * C::stage_bytes;
                        if (kind == 0) {
                            mbar_expect_tx(&full[s], kKPS * kASw);
                            tma_load_3d(st, &tmA, 0, m0, j * kKPS, &full[s]);
                        } else {
                            mbar_expect_tx(&full[s], kKPS * C::b);
                            tma_load_3d(st + kKPS * kASw, &tmB, 0, t0, j * kKPS, &full[s]);
                        }
                    } else {
                        const int d = u % kEpiRing, dround = u / kEpiRing;
                        if (dround > 0 && !mbar_wait(&epi_empty[d], (dround - 1) & 1, ab, g.status)) {
                            go = false;
                            break;
                        }
                        unsigned char* e = epi_ring + d * C::epi;
                        if (kind == 2) {  // x even: a TMA start must be 16-byte aligned
                            mbar_expect_tx(&epi_full[d], kKPS * kDWRows * 8);
                            tma_load_2d(e + C::epi_dx, &tmDW, m0 & ~1, j * kKPS, &epi_full[d]);
                        } else {
                            mbar_expect_tx(&epi_full[d], C::epi_dx);
                            tma_load_2d(e, &tmDX, t0, j * kKPS * kStageBlocks, &epi_full[d]);
                        }
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer: one K = 32 MMA per block, into the block's columns of the K-step's slot
            int step = 0;
            bool go = true;
            for (int u = 0; u < my_tiles * nst && go; ++u) {
                const int s = u % kStages, round = u / kStages;
                if (!mbar_wait(&full[s], round & 1, ab, g.status)) break;
                const int j = u % nst, kk = min(kKPS, nks - j * kKPS);  // K-steps of this stage in its tile
                unsigned char* st = smem + s * C::stage_bytes;
                for (int h = 0; h < kk; ++h, ++step) {
                    const int slot = step % kSlots, use = step / kSlots;
                    // phase `use` of slot_free: the epilogue refilled the slot with the magic (phase 0: the initial fill)
                    if (!mbar_wait(&slot_free[slot], use & 1, ab, g.status)) {
                        go = false;
                        break;
                    }
                    tc_fence_after();
                    const unsigned char* a = st + h * kASw;
                    const unsigned char* b = st + kKPS * kASw + h * C::b;
#pragma unroll
                    for (int k = 0; k < kStageBlocks; ++k)  // accumulate onto the magic-filled columns
                        mma_i8(tmem + uint32_t(slot * C::cols + k * TOK), sw128_desc(a + 32 * k), sw128_desc(b + 32 * k),
                               C::idesc, true);
                    mma_commit(&mma_done[slot]);
                }
                if (go) mma_commit(&empty[s]);
            }
            mma_commit(&fin);  // arrives once every MMA issued above has completed
        }
    } else if (warp >= 4) {  // epilogue
        pdl_wait();
        const int q = warp & 3, cg = (warp - 4) >> 2;
        const uint32_t my_cols = tmem + (uint32_t(q * 32) << 16) + uint32_t(cg * C::tpt);
        for (int j = 0; j < kSlots; ++j) tmem_fill<C::tpt>(my_cols + uint32_t(j * C::cols), kMagic);
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
            for (int j = 0; j < kSlots; ++j) mbar_arrive(&slot_free[j]);
        const float2 nz2 = make_float2(__int_as_float(int(g.nzero)), __int_as_float(int(g.nzero)));
        int step = 0, u = 0, par = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, par ^= 1) {
            const int m0 = tile_m0(tile), t0 = tile_t0(tile);
            const int row = m0 + q * 32 + lane;
            const bool row_ok = row < g.r1;
            float xo[EPI == 2 ? C::tpt : 1];  // EPI 2: the residual rows, loaded while the K loop runs
            if constexpr (EPI == 2) {
#pragma unroll
                for (int i = 0; i < C::tpt; ++i) {
                    const int t = t0 + cg * C::tpt + i;
                    xo[i] = row_ok && t < g.n ? __ldcg(g.out + size_t(t) * g.ldo + row) : 0.f;
                }
            }
            float2 acc[C::tpt / 2];  // tokens (2 j, 2 j + 1) of this thread's tpt
#pragma unroll
            for (int j = 0; j < C::tpt / 2; ++j) acc[j] = make_float2(0.f, 0.f);
            for (int j = 0; j < nst && ok; ++j, ++u) {
                const int d = u % kEpiRing, dround = u / kEpiRing, kk = min(kKPS, nks - j * kKPS);
                const unsigned char* e = epi_ring + d * C::epi;
                if (!warp_wait(&epi_full[d], dround & 1, ab, g.status)) {
                    ok = false;
                    break;
                }
                for (int h = 0; h < kk; ++h, ++step) {
                    const int slot = step % kSlots, use = step / kSlots;
                    if (!warp_wait(&mma_done[slot], use & 1, ab, g.status)) {  // warp-uniform before the .sync.aligned TMEM load
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    int v[4 * C::tpt];  // v[tpt b + i]: kMagic + block b's dot of token cg * tpt + i
                    tmem_ld_blocks<C::tpt>(my_cols + uint32_t(slot * C::cols), v);
                    tmem_fill<C::tpt>(my_cols + uint32_t(slot * C::cols), kMagic);  // ready for the slot's next use
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&slot_free[slot]);
                    const uint2 dq =
                        *reinterpret_cast<const uint2*>(e + C::epi_dx + (h * kDWRows + (m0 & 1) + q * 32 + lane) * 8);
                    const float2 d01 = __half22float2(*reinterpret_cast<const __half2*>(&dq.x));
                    const float2 d23 = __half22float2(*reinterpret_cast<const __half2*>(&dq.y));
                    const float dw[4] = {d01.x, d01.y, d23.x, d23.y};
#pragma unroll
                    for (int b = 0; b < 4; ++b) {  // acc = acc + (float(s) * dw) * dx, each rounded as in the reference
                        const float2 dw2 = make_float2(dw[b], dw[b]);
                        const float nm = -fmul(kMagicF, dw[b]);
                        const float2 nm2 = make_float2(nm, nm);
                        const float4* sdx = reinterpret_cast<const float4*>(e + ((h * kStageBlocks + b) * TOK + cg * C::tpt) * 4);
                        float2 dx2[C::tpt / 2];
#pragma unroll
                        for (int k = 0; k < C::tpt / 4; ++k) {
                            const float4 x = sdx[k];
                            dx2[2 * k] = make_float2(x.x, x.y);
                            dx2[2 * k + 1] = make_float2(x.z, x.w);
                        }
#pragma unroll
                        for (int i = 0; i < C::tpt / 2; ++i) {
                            const float2 f = make_float2(__int_as_float(v[C::tpt * b + 2 * i]), __int_as_float(v[C::tpt * b + 2 * i + 1]));
                            acc[i] = __fadd2_rn(acc[i], __ffma2_rn(__ffma2_rn(f, dw2, nm2), dx2[i], nz2));
                        }
                    }
                }
                __syncwarp();  // the ring entry is read before it is freed
                if (lane == 0 && ok) mbar_arrive(&epi_empty[d]);
            }
            if (!ok) break;
            float res[C::tpt];
#pragma unroll
            for (int i = 0; i < C::tpt / 2; ++i) {
                const float2 p = acc[i];
                res[2 * i] = p.x;
                res[2 * i + 1] = p.y;
            }
            if (EPI == 0) {
                if (row_ok) {
#pragma unroll
                    for (int i = 0; i < C::tpt; ++i) {
                        const int t = t0 + cg * C::tpt + i;
                        if (t < g.n) g.out[size_t(t) * g.ldo + row] = res[i];
                    }
                }
            } else if (EPI == 3) {
                float* xg = swi + ((par * 8 + (q >> 1) * 4 + cg) * C::tpt) * 32;  // [token i][lane]
                if (!(q & 1)) {
#pragma unroll
                    for (int i = 0; i < C::tpt; ++i) xg[i * 32 + lane] = fdiv(res[i], fadd(1.0f, exp_ref(-res[i], g.tab)));
                }
                asm volatile("bar.sync %0, 64;" ::"r"(1 + (q >> 1) * 4 + cg) : "memory");  // the gate/up warp pair
                if (q & 1) {
                    const int j = (m0 - g.r0 + 32 * (q - 1)) >> 6, ffn = (g.r1 - g.r0) >> 1, nbk = ffn / QK;
#pragma unroll
                    for (int i = 0; i < C::tpt; ++i) {
                        const int t = t0 + cg * C::tpt + i;
                        float d;
                        const int8_t qv = quantize_lane(fmul(xg[i * 32 + lane], res[i]), &d);  // the whole warp
                        if (t < g.n) {
                            g.hq[size_t(t) * ffn + j * QK + lane] = qv;
                            if (lane == 0) {
                                g.hd[size_t(t) * nbk + j] = d;
                                if (g.hdt) g.hdt[size_t(j) * g.ldt + t] = d;
                            }
                        }
                    }
                }
            } else if (EPI == 4) {
                PairIn p;
                pair_bias(g.qa, row & ~1, p);
                const int pos_base = g.tm.pos ? 0 : __ldcg(g.pos_dev);
#pragma unroll
                for (int i = 0; i < C::tpt; ++i) {
                    const float vb = __shfl_down_sync(0xffffffffu, res[i], 1);  // row + 1 of the pair
                    const int t = t0 + cg * C::tpt + i;
                    if (!(lane & 1) && t < g.n) {
                        QkvArgs a = g.qa;
                        int pos = pos_base + t;
                        if (g.tm.pos) {  // this token's sequence cache
                            pos = __ldcg(g.tm.pos + t);
                            const long long off = __ldcg(g.tm.off + t);
                            a.kcache += off;
                            a.vcache += off;
                        }
                        pair_rope(a, row, pos, p);
                        qkv_pair_store(a, row, res[i], vb, pos, p, g.qout + size_t(t) * a.n_heads * a.head_dim);
                    }
                }
            } else if (EPI == 2) {
                if (row_ok) {
#pragma unroll
                    for (int i = 0; i < C::tpt; ++i) {
                        const int t = t0 + cg * C::tpt + i;
                        if (t < g.n) g.out[size_t(t) * g.ldo + row] = fadd(xo[EPI == 2 ? i : 0], res[i]);
                    }
                }
            } else {
                const int mt = tile / n_tt;
#pragma unroll
                for (int i = 0; i < C::tpt; ++i) {
                    float v = row_ok && row < g.n_valid ? res[i] : -INFINITY;
                    int id = row_ok && row < g.n_valid ? row : INT_MAX;
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const float pv = __shfl_xor_sync(0xffffffffu, v, o);
                        const int pid = __shfl_xor_sync(0xffffffffu, id, o);
                        if (cand_better(pv, pid, v, id)) {
                            v = pv;
                            id = pid;
                        }
                    }
                    const int t = t0 + cg * C::tpt + i;
                    if (lane == 0 && t < g.n) static_cast<Cand*>(g.cand)[(size_t(mt) * 4 + q) * g.n + t] = Cand{v, id};
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        if (lane == 0) {  // the issued MMAs must be done before their TMEM goes (bounded: they depend on nothing)
            for (unsigned i = 0; i < kWaitLimit && !mbar_try(&fin, 0); ++i) {
            }
        }
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::tmem_cols) : "memory");
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 3-D view of a [rows][cols] int8 matrix as (128-byte K-chunk x rows x chunks): a box of 128 x box_rows x kKPS lands
// as kKPS consecutive 128B-swizzled [box_rows][128 B] tiles, one per K-step.
bool encode_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer, uint64_t pitch,
               uint32_t box_in, uint32_t box_out, CUtensorMapSwizzle sw) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {pitch};
    const cuuint32_t box[2] = {box_in, box_out};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_kchunks(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn || cols % 128 != 0) return false;
    const cuuint64_t dims[3] = {128, rows, cols / 128};
    const cuuint64_t strides[2] = {cols, 128};
    const cuuint32_t box[3] = {128, box_rows, kKPS};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool gemm_tc_supported(const DMat& W) {
    return (W.dtype == DT_Q8_0 || W.dtype == DT_Q4_0) && W.cols % (kStageBlocks * QK) == 0 && encode_fn() != nullptr;
}

namespace {

// Unpacks a packed Q4 word (4 low nibbles = elements j..j+3 or 4 high nibbles = j+16..j+19) into 4 int8 (q - 8).
__device__ __forceinline__ unsigned q4_bytes(unsigned nib) { return ((nib | 0x80808080u) - 0x08080808u) ^ 0x80808080u; }

// One thread per 32-element block: its 16 packed bytes (byte j = element j | element j + 16 << 4) -> 32 int8 q - 8.
__global__ void __launch_bounds__(256) k_unpack_q4_i8(const uint4* __restrict__ q, uint4* __restrict__ out, size_t n_blocks) {
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n_blocks; i += size_t(gridDim.x) * blockDim.x) {
        const uint4 w = __ldg(q + i);
        out[2 * i] = make_uint4(q4_bytes(w.x & 0x0F0F0F0Fu), q4_bytes(w.y & 0x0F0F0F0Fu), q4_bytes(w.z & 0x0F0F0F0Fu),
                                q4_bytes(w.w & 0x0F0F0F0Fu));
        out[2 * i + 1] = make_uint4(q4_bytes((w.x >> 4) & 0x0F0F0F0Fu), q4_bytes((w.y >> 4) & 0x0F0F0F0Fu),
                                    q4_bytes((w.z >> 4) & 0x0F0F0F0Fu), q4_bytes((w.w >> 4) & 0x0F0F0F0Fu));
    }
}

// out[g * ldr + r] = the 4 scales of row r, K-step g (blocks 4 g .. 4 g + 3).
__global__ void __launch_bounds__(256) k_scale_copy(const uint2* __restrict__ d, int rows, int ng, uint2* __restrict__ out, int ldr) {
    const size_t n = size_t(rows) * ng;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
        const int g = int(i / rows), r = int(i - size_t(g) * rows);
        out[size_t(g) * ldr + r] = __ldg(d + size_t(r) * ng + g);
    }
}

int rows_pad(int rows) { return (rows + 1) & ~1; }  // scale-copy pitch: a multiple of 16 bytes

__global__ void __launch_bounds__(256) k_transpose_scales(const float* __restrict__ dx, int n, int nb, float* __restrict__ dxt,
                                                          int ldt) {
    const size_t total = size_t(n) * nb;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        const int t = int(i / nb), b = int(i - size_t(t) * nb);
        dxt[size_t(b) * ldt + t] = dx[i];
    }
}

unsigned grid_for(size_t n) { return unsigned(std::max<size_t>(1, std::min<size_t>((n + 255) / 256, 148 * 16))); }

}  // namespace

size_t tc_weight_bytes(const DMat& W) {
    const size_t sc = (size_t(W.cols / (kStageBlocks * QK)) * size_t(rows_pad(W.rows)) * 8 + 255) / 256 * 256;
    return sc + (W.dtype == DT_Q4_0 ? size_t(W.rows) * size_t(W.cols) : 0);
}

cudaError_t tc_prepare_weights(const DMat& W, void* buf, TcMap* out, cudaStream_t st) {
    if (!gemm_tc_supported(W) || !buf || reinterpret_cast<uintptr_t>(buf) % 256 != 0 || reinterpret_cast<uintptr_t>(W.q) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(W.d) % 8 != 0)
        return cudaErrorInvalidValue;
    const int ng = W.cols / (kStageBlocks * QK), ldr = rows_pad(W.rows);
    unsigned char* sc = static_cast<unsigned char*>(buf);
    const size_t sc_bytes = (size_t(ng) * ldr * 8 + 255) / 256 * 256;
    k_scale_copy<<<grid_for(size_t(W.rows) * ng), 256, 0, st>>>(reinterpret_cast<const uint2*>(W.d), W.rows, ng,
                                                                reinterpret_cast<uint2*>(sc), ldr);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const void* rows8 = W.q;
    if (W.dtype == DT_Q4_0) {
        void* i8 = sc + sc_bytes;
        const size_t n_blocks = size_t(W.rows) * size_t(W.cols / QK);
        k_unpack_q4_i8<<<grid_for(n_blocks), 256, 0, st>>>(reinterpret_cast<const uint4*>(W.q), static_cast<uint4*>(i8),
                                                          n_blocks);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        rows8 = i8;
    }
    // weight scales: kDWRows rows from an even row (the tile's first row is m0 or m0 - 1 in the box), kKPS K-steps
    return encode_kchunks(&out->m, rows8, uint64_t(W.rows), uint64_t(W.cols), kTileRows) &&
                   encode_2d(&out->s, CU_TENSOR_MAP_DATA_TYPE_UINT64, sc, uint64_t(ldr), uint64_t(ng), uint64_t(ldr) * 8, kDWRows,
                             kKPS, CU_TENSOR_MAP_SWIZZLE_NONE)
               ? cudaSuccess
               : cudaErrorInvalidValue;
}

bool make_act_maps(const int8_t* qx, const float* dxt, int rows, int ldt, int cols, TcAct* out) {
    if (cols % (kStageBlocks * QK) != 0 || rows <= 0 || ldt % 32 != 0 || ldt < rows || reinterpret_cast<uintptr_t>(dxt) % 16 != 0)
        return false;
    const int nb = cols / QK;
    auto maps = [&](int tok, TcActMap* q, TcActMap* d) {  // boxes of one token tile
        return encode_kchunks(&q->m, qx, uint64_t(rows), uint64_t(cols), uint32_t(tok)) &&
               encode_2d(&d->m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, dxt, uint64_t(rows), uint64_t(nb), uint64_t(ldt) * 4,
                         uint32_t(tok), kKPS * kStageBlocks, CU_TENSOR_MAP_SWIZZLE_NONE);
    };
    return maps(32, &out->q, &out->d) && maps(16, &out->q16, &out->d16);
}

cudaError_t launch_transpose_scales(const float* dx, int n, int nb, float* dxt, int ldt, cudaStream_t st) {
    if (n <= 0 || nb <= 0) return cudaSuccess;
    k_transpose_scales<<<grid_for(size_t(n) * nb), 256, 0, st>>>(dx, n, nb, dxt, ldt);
    return cudaGetLastError();
}

namespace {

template <int TOK>
size_t gemm_tc_smem() {
    using C = Tc<TOK>;
    return size_t(kStages) * C::stage_bytes + size_t(kEpiRing) * C::epi + C::swi_bytes + 1024;
}

int sm_count() {
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return sms;
}

// TOK: 32-token tiles, or 16 (TOK = 0: 16 when even the 16-token tiles fit on the SMs at once, i.e. the 32-token tiles
// would leave half of them idle, and the tokens fill more than one 16-token tile).  Measured at 256 tokens (the
// batched decode step) the small matrices gain from 16; at 512 they lose (weight tiles loaded twice as often).
template <int EPI, int TOK = 0>
cudaError_t launch_tc_any(const DMat& W, const TcMap& wmap, const TcAct& act, GemmTcArgs g, cudaStream_t st, bool pdl) {
    g.nzero = 0x80000000u;
    const int sms = sm_count(), row_tiles = (g.r1 - g.r0 + kTileRows - 1) / kTileRows;
    if constexpr (TOK == 0) {
        if (2 * row_tiles * ((g.n + 31) / 32) <= sms && g.n > 16) return launch_tc_any<EPI, 16>(W, wmap, act, g, st, pdl);
        return launch_tc_any<EPI, 32>(W, wmap, act, g, st, pdl);
    } else {
        const int tiles = row_tiles * ((g.n + TOK - 1) / TOK);
        const dim3 grid(unsigned(std::min(tiles, sms)));  // persistent: one CTA per SM at most
        if (W.dtype != DT_Q8_0 && W.dtype != DT_Q4_0) return cudaErrorInvalidValue;
        const TcActMap& q = TOK == 16 ? act.q16 : act.q;
        const TcActMap& d = TOK == 16 ? act.d16 : act.d;
        return launch_pdl(k_gemm_tc<EPI, TOK>, grid, dim3(kTcThreads), gemm_tc_smem<TOK>(), st, pdl, wmap.m, q.m, wmap.s, d.m, g);
    }
}

// Peak probe: back-to-back tcgen05.mma.kind::i8 (M = 128, N = 256, K = 32, the largest single-CTA shape) on operands
// that stay in shared memory, accumulating into one 256-column TMEM accumulator, four K offsets in turn as a real
// K-step would.  One lane issues; the commit's mbarrier wait is bounded.  elapsed[blockIdx.x] = globaltimer ns from
// the first issue to the last MMA's completion.
constexpr int kPeakN = 256;
constexpr uint32_t kPeakIdesc =
    (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(kPeakN >> 3) << 17) | (uint32_t(kTileRows >> 4) << 24);
// 120 KB of shared memory keeps it to one CTA per SM (two would not fit), so each SM's time is its own tensor pipe's
constexpr size_t kPeakSmem = 120 * 1024;
static_assert(kPeakSmem >= size_t(kTileRows) * 128 + size_t(kPeakN) * 128 + 1024, "operand tiles fit");

__global__ void __launch_bounds__(128, 1) k_mma_i8_peak(int iters, unsigned long long* elapsed, unsigned* status) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t done;
    __shared__ uint32_t tmem_base;
    const int warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < (kTileRows + kPeakN) * 128 / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(smem)[i] = make_uint4(0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic-proxy writes visible to the MMA
    if (threadIdx.x == 0) {
        mbar_init(&done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                     "r"(kPeakN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    if (threadIdx.x == 0) {
        unsigned long long t0, t1;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
        const unsigned char* a = smem;
        const unsigned char* b = smem + kTileRows * 128;
        for (int it = 0; it < iters; ++it) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                asm volatile(
                    "{\n\t.reg .pred p;\n\t"
                    "setp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
                    ::"r"(tmem), "l"(sw128_desc(a + 32 * k)), "l"(sw128_desc(b + 32 * k)), "r"(kPeakIdesc),
                    "r"((it | k) ? 1 : 0)
                    : "memory");
            }
        }
        mma_commit(&done);
        bool ok = false;
        for (unsigned i = 0; i < kWaitLimit && !(ok = mbar_try(&done, 0)); ++i) {
        }
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
        elapsed[blockIdx.x] = t1 - t0;
        if (!ok) set_error(status, ERR_WAIT_TIMEOUT);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPeakN) : "memory");
    }
}

// One CTA per token: the best (value desc, id asc) of its n_parts candidates.
__global__ void __launch_bounds__(256) k_argmax_reduce(const Cand* __restrict__ cand, int n_parts, int n, int* __restrict__ ids,
                                                       float* __restrict__ vals) {
    __shared__ float sv[8];
    __shared__ int si[8];
    const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float v = -INFINITY;
    int id = INT_MAX;
    for (int p = threadIdx.x; p < n_parts; p += blockDim.x) {
        const Cand c = cand[size_t(p) * n + t];
        if (cand_better(c.v, c.id, v, id)) {
            v = c.v;
            id = c.id;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float pv = __shfl_xor_sync(0xffffffffu, v, o);
        const int pid = __shfl_xor_sync(0xffffffffu, id, o);
        if (cand_better(pv, pid, v, id)) {
            v = pv;
            id = pid;
        }
    }
    if (lane == 0) {
        sv[warp] = v;
        si[warp] = id;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < int(blockDim.x >> 5); ++w)
            if (cand_better(sv[w], si[w], v, id)) {
                v = sv[w];
                id = si[w];
            }
        ids[t] = id == INT_MAX ? 0 : id;
        if (vals) vals[t] = v;
    }
}

}  // namespace

cudaError_t launch_matmul_tc(const DMat& W, const TcMap& wmap, const TcAct& act, int n, int r0, int r1, float* out, int ldo,
                             unsigned* status, cudaStream_t st, bool pdl, bool residual) {
    if (r1 <= r0 || n <= 0) return cudaSuccess;
    if (W.cols % (kStageBlocks * QK) != 0) return cudaErrorInvalidValue;
    GemmTcArgs g{};
    g.r0 = r0;
    g.r1 = r1;
    g.nb = W.cols / QK;
    g.n = n;
    g.out = out;
    g.ldo = ldo;
    g.status = status;
    return residual ? launch_tc_any<2>(W, wmap, act, g, st, pdl) : launch_tc_any<0>(W, wmap, act, g, st, pdl);
}

cudaError_t launch_matmul_tc_swiglu(const DMat& W, const TcMap& wmap, const TcAct& act, int n, int8_t* hq, float* hd,
                                    float* hdt, int ldt, const ExpTab& tab, unsigned* status, cudaStream_t st, bool pdl) {
    if (n <= 0) return cudaSuccess;
    if (W.cols % (kStageBlocks * QK) != 0 || W.rows % kTileRows != 0 || !hq || !hd) return cudaErrorInvalidValue;
    GemmTcArgs g{};
    g.r0 = 0;
    g.r1 = W.rows;
    g.nb = W.cols / QK;
    g.n = n;
    g.status = status;
    g.hq = hq;
    g.hd = hd;
    g.hdt = hdt;
    g.ldt = ldt;
    g.tab = tab;
    return launch_tc_any<3, 32>(W, wmap, act, g, st, pdl);
}

cudaError_t launch_matmul_tc_qkv(const DMat& W, const TcMap& wmap, const TcAct& act, int n, const QkvArgs& qa,
                                 const int* pos_dev, TokMap tm, float* qout, unsigned* status, cudaStream_t st, bool pdl) {
    if (n <= 0) return cudaSuccess;
    if (W.cols % (kStageBlocks * QK) != 0 || W.rows % kTileRows != 0 || !qout || (!tm.pos && !pos_dev))
        return cudaErrorInvalidValue;
    GemmTcArgs g{};
    g.r0 = 0;
    g.r1 = W.rows;
    g.nb = W.cols / QK;
    g.n = n;
    g.status = status;
    g.qa = qa;
    g.tm = tm;
    g.pos_dev = pos_dev;
    g.qout = qout;
    return launch_tc_any<4, 32>(W, wmap, act, g, st, pdl);
}

int argmax_parts(int rows) { return ((rows + kTileRows - 1) / kTileRows) * 4; }

cudaError_t launch_wait_probe(unsigned limit, unsigned* status, cudaStream_t st) {
    k_wait_probe<<<1, 32, 0, st>>>(limit, status);
    return cudaGetLastError();
}

cudaError_t bench_mma_i8(int iters, double* tops, unsigned* status_host) {
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    unsigned long long* el = nullptr;
    unsigned* status = nullptr;
    e = cudaMalloc(&el, sizeof(unsigned long long) * sms);
    if (e == cudaSuccess) e = cudaMalloc(&status, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(status, 0, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k_mma_i8_peak, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kPeakSmem));
    std::vector<unsigned long long> h(size_t(sms > 0 ? sms : 1), 0);
    unsigned st = 0;
    if (e == cudaSuccess) {
        k_mma_i8_peak<<<sms, 128, kPeakSmem>>>(iters / 8, el, status);  // warm-up
        k_mma_i8_peak<<<sms, 128, kPeakSmem>>>(iters, el, status);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(h.data(), el, sizeof(unsigned long long) * sms, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(&st, status, sizeof st, cudaMemcpyDeviceToHost);
    cudaFree(el);
    cudaFree(status);
    if (e != cudaSuccess) return e;
    const unsigned long long worst = *std::max_element(h.begin(), h.end());
    const double ops = 2.0 * kTileRows * kPeakN * 32 * 4 * double(iters) * sms;
    if (tops) *tops = worst ? ops / (double(worst) * 1e-9) / 1e12 : 0.0;
    if (status_host) *status_host = st;
    return cudaSuccess;
}

cudaError_t launch_matmul_tc_argmax(const DMat& W, const TcMap& wmap, const TcAct& act, int n, int n_valid, void* cand,
                                    unsigned* status, cudaStream_t st, bool pdl) {
    if (n <= 0) return cudaSuccess;
    if (W.cols % (kStageBlocks * QK) != 0) return cudaErrorInvalidValue;
    GemmTcArgs g{};
    g.r0 = 0;
    g.r1 = W.rows;
    g.nb = W.cols / QK;
    g.n = n;
    g.status = status;
    g.n_valid = n_valid;
    g.cand = cand;
    return launch_tc_any<1, 32>(W, wmap, act, g, st, pdl);
}

cudaError_t launch_argmax_reduce(const void* cand, int n_parts, int n, int* ids, float* vals, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    k_argmax_reduce<<<n, 256, 0, st>>>(static_cast<const Cand*>(cand), n_parts, n, ids, vals);
    return cudaGetLastError();
}

}  // namespace qb
