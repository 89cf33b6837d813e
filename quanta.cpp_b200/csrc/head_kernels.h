// Launchers for the output head, the Exact Shortlist Head and the device sampler (head_kernels.cu).
#pragma once

#include <algorithm>

#include "common.cuh"
#include "exp_table.h"
#include "ops.h"

namespace qb {

struct Cand {
    float v;
    int id;
};

// Quantized final hidden state the head reads (written by k_head_input).
struct HeadIn {
    int8_t* xq;     // [dim]
    float* dx;      // [dim/32] block scales
    int* xsum;      // [dim/32] sum of q per block (Q4 offset)
    float* xnorm;   // [dim/32] d_b * ||q_b||_2 (shortlist bound)
    float* xabs;    // [dim/32] sum of |q| per block (the nibble-plane screen's bound; null: not computed)
};

struct HeadState {
    float tau;             // cut-off of the last shortlist pass
    int rows;              // 8-bit head rows read by the last head pass
    long long rows_total;  // rows of the earlier passes since the last reset
    int calls;             // head passes since the last reset
    int pad;
};

// Tiling of a streamed head pass: rows in tiles of tile_rows (one thread per row), tiles split over `grid` persistent
// CTAs, each tile staged in one of `stages` shared-memory ring slots of stage_bytes: quants at 0 with a row stride of
// qstride bytes (the row padded by 16 bytes), fp16 scales at d_off, bound errors at e_off (coarse pass).
struct StreamPlan {
    int tile_rows = 0, n_tiles = 0, threads = 0;
    unsigned cpr_magic = 0;
    int qstride = 0, d_off = 0, e_off = 0, stage_bytes = 0, stages = 0;
    int list_off = 0, list_cap = 0, ring_off = 0;
    int cand_off = 0, cand_cap = 0;  // coarse pass: every row's (score, id) of the CTA, selected from after the tiles
    size_t smem = 0;
    int grid = 0;
};
// coarse: stage the bounds too; gather: room for the CTA's compacted row list.  stages == 0 when it cannot fit.
StreamPlan plan_stream(int dtype, int rows, int cols, int grid, bool coarse, bool gather);
// The high nibble plane of a Q8_0 matrix as Q4_0 nibbles: per 32-block, byte j = (q[j] >> 4) + 8 | ((q[j + 16] >> 4) + 8) << 4
// (plane: rows * cols / 2 bytes), and err[row][block] = ||(q & 15) - 8||_2 rounded up to f16 (rows * cols / 32 halves).
cudaError_t launch_hi_plane(const DMat& W8, uint8_t* plane, __half* err, cudaStream_t st);

struct HeadFullArgs {
    DMat W;
    StreamPlan plan;
    int n_valid;
    int n_list;         // sampler stage-1 list length per CTA (0: logits only)
    int penal;          // apply the repetition penalty to marked rows (and clear the marks)
    float penalty;
    unsigned char* mark;
    float* logits;
    void* lists;        // plan.grid * n_list candidates
};

// The shortlist's screen.  kScreenQ4: the file's quanta.head_q4 with the bound of quanta.head_err (the reference's).
// kScreenHi4: the high nibble plane of the Q8 head itself (W4 = the plane as Q4_0 nibbles q8 >> 4 offset by 8, with
// the Q8 head's own scales; err = ||lo - 8||_2 per row and block, f16 rounded up): screen s' = 16 sum(hi q) + 8 sum(q)
// per block, bound min(8 sum|q_b|, err_b ||q_b||_2) |d_b| dx_b plus the f32 rounding of both sums (head_kernels.cu).  Exact rows, tau and the sampled ids are the same either way.
constexpr int kScreenQ4 = 0, kScreenHi4 = 1;

struct ShortlistArgs {
    DMat W8;                // lm_head (Q8_0)
    DMat W4;                // quanta.head_q4, or the Q8 head's high nibble plane (kScreenHi4)
    const __half* err;      // [V][dim/32]: quanta.head_err (kScreenQ4), or the low nibbles' norms (kScreenHi4)
    int screen = kScreenQ4;
    StreamPlan plan4;       // streamed coarse pass over W4
    StreamPlan plan8g;      // candidate gather over W8
    int k, n_valid;
    const int* must;        // must ids (device)
    const int* n_must_dev;  // device count (or null: n_must_host)
    int n_must_host;
    int window;             // only the last `window` must ids (0 = all)
    unsigned char* mark;    // [V] zero between passes
    float* coarse;          // [V]
    float* upper;           // [V]
    float* logits;          // [V]
    void* seed_buf;         // plan4.grid * (k + 8) candidates
    HeadState* hs;
    int n_list;             // sampler stage-1 list length (0: none)
    int penal;
    float penalty;
    void* lists;            // plan8g.grid * n_list candidates
    bool marked = false;    // the must ids are marked already (k_sample_final's NextMarks): no mark kernel
};

struct SamplerArgs {
    float temperature, top_p, min_p, repeat_penalty;
    int append;  // 1: append the pick to the history and advance the position
    ExpTab exptab;
};

struct SamplerState {
    unsigned long long rng;  // xorshift64* state
    int token;               // last pick
    int n_hist;              // history length
    int pos;                 // position of the next token to feed
    int pad;
};

// full_rows: rows the coming head pass reads when it is the full head (V), 0 for the shortlist (which counts itself).
cudaError_t launch_head_input(const float* X, const float* norm_w, int dim, float eps, const HeadIn& hin, HeadState* hs,
                              int full_rows, cudaStream_t st, bool pdl);
cudaError_t launch_head_full(const HeadFullArgs& a, const HeadIn& hin, cudaStream_t st, bool pdl);
// Launches 4 kernels (mark, coarse, seeds, candidates; 3 without the mark kernel when a.marked); adds them to *kernels.
cudaError_t launch_shortlist(const ShortlistArgs& a, const HeadIn& hin, cudaStream_t st, bool pdl, int* kernels);
cudaError_t launch_mark(const int* must, const int* n_must_dev, int n_must_host, int window, int n_valid, unsigned char* mark,
                        cudaStream_t st, bool pdl);
// write_back: where the penalised logits go (the logits array itself for an in-place edit), or null.
cudaError_t launch_topk_partial(const float* logits, int n_valid, int K, int penal, float penalty, unsigned char* mark,
                                void* lists, int n_lists, cudaStream_t st, bool pdl, float* write_back = nullptr);
// The next head pass's must ids, marked by k_sample_final while it draws (a decode step's sampler, whose head follows
// in the same step): mark[id] = 1 for the ids in [0, n_valid) among the last `window` ids of the history after this
// draw's append (0: the whole history), the same marks the mark kernel would set before that head.
struct NextMarks {
    unsigned char* mark = nullptr;  // null: none
    int window = 0, n_valid = 0;
};
cudaError_t launch_sample_final(const void* lists, int n_lists, int K, const SamplerArgs& sa, SamplerState* ss, int* hist,
                                int hist_cap, cudaStream_t st, bool pdl, const NextMarks* next = nullptr);

// nll.cu: *acc += -log softmax(logits[0..n_valid))[target] (the perplexity's term), f64 accumulation.
cudaError_t launch_token_nll(const float* logits, int n_valid, int target, double* acc, cudaStream_t st, bool pdl);

// The sampler for any top_k (sampler_wide.cu): top_k <= 0 (every candidate) or top_k > 32.  A stable radix sort of
// (logit, id) over ids < n_valid, then the softmax / min-p / top-p / draw of the n best on one CTA.  Temperature > 0
// only (greedy takes the argmax path).  Scratch: 4 arrays of n_valid words and a digit histogram.
struct WideScratch {
    unsigned* keys[2];
    int* ids[2];
    unsigned* hist;
    int cap;  // largest n_valid the scratch holds
};
int wide_sort_tiles(int n_valid);
size_t wide_scratch_bytes(int n_valid);
WideScratch wide_scratch_carve(void* base, int n_valid);  // base: wide_scratch_bytes(n_valid) bytes, 256-byte aligned
// Launches 13 kernels (adds 13 to *kernels).  logits: already penalised.
cudaError_t launch_sample_wide(const float* logits, int n_valid, int K, const SamplerArgs& sa, SamplerState* ss, int* hist,
                               int hist_cap, const WideScratch& ws, cudaStream_t st, bool pdl, int* kernels);

}  // namespace qb
