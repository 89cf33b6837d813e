// extern "C" shim over the reference engine (Quanta.cpp engine/src), compiled together with the
// reference's own sources by oracle/Makefile into oracle/_ref/libquanta_ref.so.
//
// TEST INFRASTRUCTURE ONLY.  The tests and bench.py's reference/CPU-baseline arm load this library through
// ctypes as the checker and as the timed CPU path; the product (quanta.cpp_b200) never links it.
//
// Every function here forwards to the reference's public interface:
//   Model::load / forward / forward_batch / head / last_head_rows / head_coarse / head_upper
//       (engine/src/model.h:35-51)
//   quantize_q8, matvec_q_ref, matmul_q_ref (engine/src/ops.h:52-70)
//   Sampler::sample (engine/src/sampler.h:26), Session::feed / generate / head_fraction (engine/src/session.h:27-35)
//   kernel_selftest, check_batch, check_head (engine/src/checks.h:20-27)
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "checks.h"
#include "model.h"
#include "ops.h"
#include "sampler.h"
#include "session.h"
#include "tokenizer.h"

using namespace quanta;

namespace {

struct RefModel {
    Model model;
    std::unique_ptr<Tokenizer> tok;
};

HeadQuery make_hq(int top_k, int n_valid, const int* must, int n_must) {
    HeadQuery hq;
    hq.top_k = top_k;
    hq.n_valid = n_valid;
    hq.must = must;
    hq.n_must = n_must;
    return hq;
}

Tensor make_tensor(int dtype, int rows, int cols, const uint8_t* data) {
    Tensor W;
    W.dtype = DType(dtype);
    W.rows = rows;
    W.cols = cols;
    W.data = data;
    return W;
}

QuantVec make_qv(const int8_t* q, const float* d, int n) {
    QuantVec v;
    v.n = n;
    v.q.assign(q, q + n);
    v.d.assign(d, d + n / QK);
    return v;
}

}  // namespace

extern "C" {

void* ref_model_open(const char* path, int ctx, int n_threads, int kv_f16, char* err, int errlen) {
    auto* m = new RefModel;
    std::string e;
    if (!m->model.load(path, ctx, &e, n_threads, kv_f16 != 0)) {
        if (err && errlen > 0) std::snprintf(err, size_t(errlen), "%s", e.c_str());
        delete m;
        return nullptr;
    }
    try {
        m->tok = std::make_unique<Tokenizer>(m->model.file().tokenizer());
    } catch (const std::exception& ex) {
        if (err && errlen > 0) std::snprintf(err, size_t(errlen), "%s", ex.what());
        delete m;
        return nullptr;
    }
    return m;
}

void ref_model_close(void* h) { delete static_cast<RefModel*>(h); }

int ref_vocab(void* h) { return static_cast<RefModel*>(h)->model.hparams().vocab_size; }
int ref_n_tokens(void* h) { return static_cast<RefModel*>(h)->tok->n_tokens(); }
int ref_ctx_len(void* h) { return static_cast<RefModel*>(h)->model.ctx_len(); }
int ref_n_threads(void* h) { return static_cast<RefModel*>(h)->model.n_threads(); }
int ref_has_shortlist(void* h) { return static_cast<RefModel*>(h)->model.has_shortlist_head() ? 1 : 0; }
int ref_last_head_rows(void* h) { return static_cast<RefModel*>(h)->model.last_head_rows(); }

// Returns 0 on success, -1 on a reference exception (bad position etc.).  out may be null.
int ref_forward(void* h, int token, int pos, int top_k, int n_valid, const int* must, int n_must, float* out) {
    auto* m = static_cast<RefModel*>(h);
    try {
        HeadQuery hq = make_hq(top_k, n_valid, must, n_must);
        const float* lg = m->model.forward(token, pos, top_k > 0 ? &hq : nullptr);
        if (out) std::memcpy(out, lg, sizeof(float) * size_t(m->model.hparams().vocab_size));
    } catch (const std::exception&) {
        return -1;
    }
    return 0;
}

int ref_forward_batch(void* h, const int* tokens, int n, int pos0, int top_k, int n_valid, const int* must,
                      int n_must, float* out) {
    auto* m = static_cast<RefModel*>(h);
    try {
        HeadQuery hq = make_hq(top_k, n_valid, must, n_must);
        const float* lg = m->model.forward_batch(tokens, n, pos0, top_k > 0 ? &hq : nullptr);
        if (out) std::memcpy(out, lg, sizeof(float) * size_t(m->model.hparams().vocab_size));
    } catch (const std::exception&) {
        return -1;
    }
    return 0;
}

// Re-runs the head for the last forward() token.  coarse/upper (may be null) receive the shortlist pass's
// 4-bit scores and upper bounds when top_k > 0 and the file has a shortlist head.
int ref_head(void* h, int top_k, int n_valid, const int* must, int n_must, float* out, float* coarse, float* upper) {
    auto* m = static_cast<RefModel*>(h);
    HeadQuery hq = make_hq(top_k, n_valid, must, n_must);
    const float* lg = m->model.head(top_k > 0 ? &hq : nullptr);
    const size_t V = size_t(m->model.hparams().vocab_size);
    if (out) std::memcpy(out, lg, sizeof(float) * V);
    if (top_k > 0 && m->model.has_shortlist_head()) {
        if (coarse) std::memcpy(coarse, m->model.head_coarse(), sizeof(float) * V);
        if (upper) std::memcpy(upper, m->model.head_upper(), sizeof(float) * V);
    }
    return m->model.last_head_rows();
}

// ---- ops level (engine/src/ops.h)

void ref_quantize_q8(const float* x, int n, int8_t* q, float* d) {
    QuantVec v;
    quantize_q8(x, n, v);
    std::memcpy(q, v.q.data(), size_t(n));
    std::memcpy(d, v.d.data(), sizeof(float) * size_t(n / QK));
}

void ref_matvec_q(int dtype, int rows, int cols, const uint8_t* data, const int8_t* q, const float* d, int r0, int r1,
                  float* out) {
    const Tensor W = make_tensor(dtype, rows, cols, data);
    const QuantVec x = make_qv(q, d, cols);
    matvec_q_ref(out, W, x, r0, r1);
}

// x: n activations, q [n][cols], d [n][cols/32]; out[t * ldo + r].
void ref_matmul_q(int dtype, int rows, int cols, const uint8_t* data, const int8_t* q, const float* d, int n, int r0,
                  int r1, float* out, int ldo) {
    const Tensor W = make_tensor(dtype, rows, cols, data);
    std::vector<QuantVec> xs;
    xs.reserve(size_t(n));
    for (int t = 0; t < n; ++t) xs.push_back(make_qv(q + size_t(t) * cols, d + size_t(t) * (cols / QK), cols));
    matmul_q_ref(out, ldo, W, xs.data(), n, r0, r1);
}

// Float-math matvec (engine/src/ops_ref.cpp matvec_ref) for f32/f16/q8/q4 weights.
void ref_matvec_f(int dtype, int rows, int cols, const uint8_t* data, const float* x, int r0, int r1, float* out) {
    const Tensor W = make_tensor(dtype, rows, cols, data);
    matvec_ref(out, W, x, r0, r1);
}

void ref_get_row(int dtype, int rows, int cols, const uint8_t* data, int row, float* out) {
    const Tensor W = make_tensor(dtype, rows, cols, data);
    get_row(out, W, row);
}

void ref_rmsnorm(float* out, const float* x, const float* w, int n, float eps) { rmsnorm(out, x, w, n, eps); }
void ref_rope(float* v, int n_heads, int head_dim, int pos, float theta) { rope(v, n_heads, head_dim, pos, theta); }
void ref_softmax(float* x, int n) { softmax(x, n); }
void ref_swiglu(float* out, const float* g, const float* u, int n) { swiglu(out, g, u, n); }

// ---- sampler (engine/src/sampler.h)

void* ref_sampler_new(float temp, int top_k, float top_p, float min_p, float repeat_penalty, int repeat_window,
                      unsigned long long seed) {
    SamplerParams p;
    p.temperature = temp;
    p.top_k = top_k;
    p.top_p = top_p;
    p.min_p = min_p;
    p.repeat_penalty = repeat_penalty;
    p.repeat_window = repeat_window;
    p.seed = seed;
    return new Sampler(p);
}

void ref_sampler_free(void* s) { delete static_cast<Sampler*>(s); }

int ref_sample(void* s, float* logits, int n_valid, const int* history, int n_hist) {
    std::vector<int> hist(history, history + n_hist);
    return static_cast<Sampler*>(s)->sample(logits, n_valid, hist);
}

// ---- session level: feed a prompt and generate (engine/src/session.cpp:13-52).  This is what the CPU baseline
// times.  use_shortlist=1 passes the sampler params to the session (HeadQuery from session.cpp:63-79).
// Returns the number of generated tokens; out_ids receives them.
int ref_generate(void* h, const int* ids, int n_ids, int batch_prefill, int use_shortlist, float temp, int top_k,
                 float top_p, float min_p, float repeat_penalty, unsigned long long seed, int n_gen, int* out_ids,
                 double* t_prefill, double* t_decode, double* head_fraction) {
    auto* m = static_cast<RefModel*>(h);
    SamplerParams sp;
    sp.temperature = temp;
    sp.top_k = top_k;
    sp.top_p = top_p;
    sp.min_p = min_p;
    sp.repeat_penalty = repeat_penalty;
    sp.seed = seed;
    Sampler sampler(sp);
    Session s(m->model, *m->tok);
    s.set_batch_prefill(batch_prefill != 0);
    if (use_shortlist) s.set_sampler(&sp);
    std::vector<int> prompt(ids, ids + n_ids);
    double tp = 0, td = 0;
    if (!s.feed(prompt, &tp)) return -1;
    int k = 0;
    const int n = s.generate(sampler, n_gen, {}, [&](int id) { out_ids[k++] = id; return true; }, &td);
    if (t_prefill) *t_prefill = tp;
    if (t_decode) *t_decode = td;
    if (head_fraction) *head_fraction = s.head_fraction();
    return n;
}

// ---- tokenizer (engine/src/tokenizer.h): encode returns the id count and writes at most max of them
int ref_tokenize(void* h, const char* text, int len, int* out, int max) {
    const std::vector<int> ids = static_cast<RefModel*>(h)->tok->encode(std::string(text, size_t(len)));
    std::memcpy(out, ids.data(), sizeof(int) * std::min(ids.size(), size_t(max)));
    return int(ids.size());
}

int ref_token_id(void* h, const char* literal) { return static_cast<RefModel*>(h)->tok->token_id(literal); }

// ---- the reference's own self-checks (engine/src/checks.h)

static void print_line(const std::string& s) { std::printf("%s\n", s.c_str()); std::fflush(stdout); }

int ref_kernel_selftest(void) { return kernel_selftest(print_line) ? 1 : 0; }

int ref_check_batch(void* h, const int* ids, int n, int quick) {
    auto* m = static_cast<RefModel*>(h);
    return check_batch(m->model, std::vector<int>(ids, ids + n), print_line, quick != 0) ? 1 : 0;
}

int ref_check_head(void* h, const int* ids, int n) {
    auto* m = static_cast<RefModel*>(h);
    return check_head(m->model, *m->tok, std::vector<int>(ids, ids + n), print_line) ? 1 : 0;
}

}  // extern "C"
