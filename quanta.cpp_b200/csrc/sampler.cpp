// The standalone device sampler of include/quanta_b200.h: Sampler::sample (engine/src/sampler.cpp:22-85) over
// device-resident logits.  The kernels are the ones the decode loop uses (head_kernels.cu): k_sl_mark marks the unique
// penalised history ids, k_topk_partial applies the penalty (in place) and keeps each CTA's best K, k_sample_final
// merges the lists and draws.
#include <cuda_runtime.h>

#include <algorithm>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "quanta_b200.h"
#include "capi_util.h"
#include "head_kernels.h"

namespace {

// The host libm's expf exceptions on each device (constant data shared by every sampler of the process).
qb::ExpTab device_exp_table(int dev, std::string* err) {
    static std::mutex mu;
    static std::vector<qb::ExpTab> tabs;
    std::lock_guard<std::mutex> lock(mu);
    if (int(tabs.size()) <= dev) tabs.resize(size_t(dev) + 1);
    if (!tabs[size_t(dev)].slots) {
        const std::vector<uint64_t>& slots = qb::expf_exception_slots(nullptr);
        void* p = nullptr;
        cudaError_t e = cudaMalloc(&p, slots.size() * 8);
        if (e == cudaSuccess) e = cudaMemcpy(p, slots.data(), slots.size() * 8, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            if (p) cudaFree(p);
            *err = std::string("exp table upload: ") + cudaGetErrorString(e);
            return qb::ExpTab{};
        }
        tabs[size_t(dev)].slots = static_cast<const unsigned long long*>(p);
        tabs[size_t(dev)].mask = unsigned(slots.size() - 1);
    }
    return tabs[size_t(dev)];
}

}  // namespace

struct qnt_sampler {
    qnt_sampler_params p{};
    int device = 0;
    int n_lists = 0;
    qb::ExpTab tab{};
    qb::SamplerState* ss = nullptr;  // rng state + last pick
    qb::Cand* lists = nullptr;       // n_lists * 32 stage-1 candidates
    unsigned char* mark = nullptr;   // [mark_cap] penalised-id marks, all zero between calls
    int mark_cap = 0;
    int* hist = nullptr;             // device copy of the history
    int hist_cap = 0;
    void* wide_buf = nullptr;        // the sorting sampler's scratch (top_k 0 or > 32), grown to n_valid
    qb::WideScratch wide{};

    ~qnt_sampler() {
        cudaFree(ss);
        cudaFree(lists);
        cudaFree(mark);
        cudaFree(hist);
        cudaFree(wide_buf);
    }
};

extern "C" {

int qnt_sampler_create(const qnt_sampler_params* sp, qnt_sampler** out) {
    using namespace qnt_capi;
    if (!sp || !out) return set_err(QNT_ERR_INVALID, "qnt_sampler_create: null argument");
    *out = nullptr;
    auto s = std::make_unique<qnt_sampler>();
    s->p = *sp;
    cudaError_t e = cudaGetDevice(&s->device);
    if (e != cudaSuccess) return cuda_err(e, "cudaGetDevice");
    e = cudaDeviceGetAttribute(&s->n_lists, cudaDevAttrMultiProcessorCount, s->device);
    if (e != cudaSuccess) return cuda_err(e, "cudaDeviceGetAttribute");
    std::string err;
    s->tab = device_exp_table(s->device, &err);
    if (!s->tab.slots) return set_err(QNT_ERR_CUDA, err);
    e = cudaMalloc(&s->ss, sizeof(qb::SamplerState));
    if (e == cudaSuccess) e = cudaMalloc(&s->lists, size_t(s->n_lists) * 32 * sizeof(qb::Cand));
    if (e != cudaSuccess) return cuda_err(e, "cudaMalloc");
    qb::SamplerState st{};
    st.rng = (sp->seed ? sp->seed : 0x9E3779B97F4A7C15ULL) | 1ULL;  // Sampler::Sampler (sampler.cpp:10-13)
    e = cudaMemcpy(s->ss, &st, sizeof st, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_err(e, "cudaMemcpy");
    *out = s.release();
    return QNT_OK;
}

int qnt_sampler_sample(qnt_sampler* s, float* logits, int n_valid, const int* history, int n_history, int* token,
                       void* stream) {
    using namespace qnt_capi;
    if (!s || !logits || !token || n_valid <= 0 || n_history < 0 || (n_history > 0 && !history))
        return set_err(QNT_ERR_INVALID, "qnt_sampler_sample: bad argument");
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != s->device) return set_err(QNT_ERR_INVALID, "qnt_sampler_sample: the sampler lives on another device");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const qnt_sampler_params& p = s->p;
    const bool greedy = p.temperature <= 0.f;
    // top_k <= 0 keeps every id, as does top_k >= n_valid (sampler.cpp:45-50); beyond 32 the sorting sampler runs
    const bool wide = !greedy && (p.top_k <= 0 || p.top_k > 32);
    const int K = greedy ? 1 : wide ? 1 : std::min(p.top_k, n_valid);
    const bool penal = p.repeat_penalty != 1.0f && n_history > 0;
    cudaError_t e = cudaSuccess;
    if (wide && s->wide.cap < n_valid) {
        cudaFree(s->wide_buf);
        s->wide_buf = nullptr;
        s->wide.cap = 0;
        e = cudaMalloc(&s->wide_buf, qb::wide_scratch_bytes(n_valid));
        if (e != cudaSuccess) return cuda_err(e, "sampler sort scratch");
        s->wide = qb::wide_scratch_carve(s->wide_buf, n_valid);
    }
    if (penal) {
        if (s->mark_cap < n_valid) {
            cudaFree(s->mark);
            s->mark = nullptr;
            s->mark_cap = 0;
            e = cudaMalloc(&s->mark, size_t(n_valid));
            if (e == cudaSuccess) e = cudaMemset(s->mark, 0, size_t(n_valid));
            if (e != cudaSuccess) return cuda_err(e, "sampler marks");
            s->mark_cap = n_valid;
        }
        if (s->hist_cap < n_history) {
            cudaFree(s->hist);
            s->hist = nullptr;
            s->hist_cap = 0;
            e = cudaMalloc(&s->hist, size_t(n_history) * 4);
            if (e != cudaSuccess) return cuda_err(e, "sampler history");
            s->hist_cap = n_history;
        }
        e = cudaMemcpyAsync(s->hist, history, size_t(n_history) * 4, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = qb::launch_mark(s->hist, nullptr, n_history, p.repeat_window, n_valid, s->mark, st, false);
        if (e != cudaSuccess) return cuda_err(e, "sampler penalty marks");
    }
    // stage 1: the penalty written back into the logits (and, for the list sampler, each CTA's best K)
    if (!wide || penal) {
        e = qb::launch_topk_partial(logits, n_valid, K, penal ? 1 : 0, p.repeat_penalty, s->mark, s->lists, s->n_lists, st,
                                    false, logits);
        if (e != cudaSuccess) return cuda_err(e, "sampler stage 1");
    }
    const qb::SamplerArgs sa{p.temperature, p.top_p, p.min_p, p.repeat_penalty, 0, s->tab};
    e = wide ? qb::launch_sample_wide(logits, n_valid, p.top_k, sa, s->ss, nullptr, 0, s->wide, st, false, nullptr)
             : qb::launch_sample_final(s->lists, s->n_lists, K, sa, s->ss, nullptr, 0, st, false);
    if (e != cudaSuccess) return cuda_err(e, "sampler stage 2");
    int tok = -1;
    e = cudaMemcpyAsync(&tok, &s->ss->token, 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_err(e, "sampler result");
    *token = tok;
    return QNT_OK;
}

void qnt_sampler_free(qnt_sampler* s) { delete s; }

}  // extern "C"
