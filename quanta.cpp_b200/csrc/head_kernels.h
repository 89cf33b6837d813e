// Launchers for the output head, the Exact Shortlist Head and the device sampler (head_kernels.cu).
#pragma once

#include <algorithm>

#include "common.cuh"
#include "ops.h"

namespace qb {

// Quantized final hidden state the head reads (written by k_head_input).
struct HeadIn {
    int8_t* xq;     // [dim]
    float* dx;      // [dim/32] block scales
    int* xsum;      // [dim/32] sum of q per block (Q4 offset)
    float* xnorm;   // [dim/32] d_b * ||q_b||_2 (shortlist bound)
};

struct HeadState {
    float tau;             // cut-off of the last shortlist pass
    int rows;              // 8-bit head rows read by the last head pass
    long long rows_total;  // rows of the earlier passes since the last reset
    int calls;             // head passes since the last reset
    int pad;
};

struct HeadPlan {
    int rows_per_cta = 0, grid = 0, u = 0;
    unsigned magic = 0;
    size_t smem = 0;
};
HeadPlan plan_head(int dtype, int rows, int cols);

struct ShortlistArgs {
    DMat W8;                // lm_head (Q8_0)
    DMat W4;                // quanta.head_q4
    const __half* err;      // quanta.head_err [V][dim/32]
    HeadPlan plan4;         // tiles of W4
    int coarse_ctas;        // persistent CTAs of the coarse pass (lists merged by the seed kernel)
    int cand_ctas;
    int k, n_valid;
    const int* must;        // must ids (device)
    const int* n_must_dev;  // device count (or null: n_must_host)
    int n_must_host;
    int window;             // only the last `window` must ids (0 = all)
    unsigned char* mark;    // [V] zero between passes
    float* coarse;          // [V]
    float* upper;           // [V]
    float* logits;          // [V]
    void* seed_buf;         // coarse_ctas * (k + 8) candidates
    HeadState* hs;
};

struct SamplerArgs {
    float temperature, top_p, min_p, repeat_penalty;
    int append;  // 1: append the pick to the history and advance the position
};

struct SamplerState {
    unsigned long long rng;  // xorshift64* state
    int token;               // last pick
    int n_hist;              // history length
    int pos;                 // position of the next token to feed
    int pad;
};

struct SamplerLaunch {
    float* logits;
    int n_valid;
    int K;             // 1 = greedy
    int parts;         // stage-1 CTAs
    void* part_buf;    // parts * K candidates
    SamplerArgs args;
    SamplerState* state;
    int* hist;
    const int* n_hist_dev;
    int hist_cap;
    int window;
    unsigned* flag;    // [V] zero between calls
};

// full_rows: rows the coming head pass reads when it is the full head (V), 0 for the shortlist (which counts itself).
cudaError_t launch_head_input(const float* X, const float* norm_w, int dim, float eps, const HeadIn& hin, HeadState* hs,
                              int full_rows, cudaStream_t st, bool pdl);
cudaError_t launch_head_full(const DMat& W, const HeadPlan& p, const HeadIn& hin, float* logits, cudaStream_t st, bool pdl);
cudaError_t launch_shortlist(const ShortlistArgs& a, const HeadIn& hin, cudaStream_t st, bool pdl);
cudaError_t launch_sampler(const SamplerLaunch& s, cudaStream_t st, bool pdl);

}  // namespace qb
