// qnt_sampler_sample_noalloc: the standalone device sampler (sampler.cpp here, Sampler::sample of
// engine/src/sampler.cpp:22-85) without a sampler object and without allocating memory.  Its scratch -- the sampler
// state, the stage-1 candidate lists, the history copy and the penalty marks -- lives in one file-scope device array
// of fixed size, and the host libm exp table in a second one; both are resolved once per device.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "quanta_b200.h"
#include "capi_util.h"
#include "head_kernels.h"

namespace {

constexpr int kMaxVocab = 262144;    // n_valid limit: one mark byte per id
constexpr int kMaxHistory = 32768;   // history ids copied per call
constexpr int kMaxLists = 256;       // stage-1 lists (one per SM, capped)
constexpr int kListLen = 32;         // top_k limit
constexpr size_t kOffLists = 256;    // the SamplerState sits at offset 0
constexpr size_t kOffHist = kOffLists + size_t(kMaxLists) * kListLen * sizeof(qb::Cand);
constexpr size_t kOffMark = kOffHist + size_t(kMaxHistory) * 4;
constexpr size_t kScratchBytes = kOffMark + size_t(kMaxVocab);  // 459,008 bytes
constexpr int kExpSlots = 1 << 19;   // capacity of the static exp table (4 MiB)
static_assert(sizeof(qb::SamplerState) <= kOffLists && kOffHist % 256 == 0 && kOffMark % 256 == 0, "scratch layout");

// The marks region must be all zero when a call starts: static device memory starts zeroed and every call clears the
// marks it sets (k_topk_partial), so it stays zero between calls.
static __device__ __align__(256) unsigned char g_sampler_scratch[kScratchBytes];
static __device__ __align__(256) unsigned long long g_sampler_exptab[kExpSlots];

struct DeviceSetup {
    bool ready = false;
    unsigned char* scratch = nullptr;
    unsigned long long* tab = nullptr;
    unsigned mask = 0;
    int n_lists = 0;
};

constexpr int kMaxDevices = 64;
DeviceSetup g_setup[kMaxDevices];
std::mutex g_setup_mu;

// Once per device, with that device current: the scratch address, the exp table copied in, the SM count.
int device_setup(int dev, DeviceSetup* out) {
    using namespace qnt_capi;
    std::lock_guard<std::mutex> lock(g_setup_mu);
    DeviceSetup& s = g_setup[dev];
    if (!s.ready) {
        void* scratch = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&scratch, g_sampler_scratch);
        if (e != cudaSuccess) return cuda_err(e, "cudaGetSymbolAddress(g_sampler_scratch)");
        void* tab = nullptr;
        e = cudaGetSymbolAddress(&tab, g_sampler_exptab);
        if (e != cudaSuccess) return cuda_err(e, "cudaGetSymbolAddress(g_sampler_exptab)");
        const std::vector<uint64_t>& slots = qb::expf_exception_slots(nullptr);
        if (slots.empty() || slots.size() > size_t(kExpSlots))
            return set_err(QNT_ERR_UNSUPPORTED, "host exp table does not fit the static table of " +
                                                    std::to_string(kExpSlots) + " slots");
        e = cudaMemcpy(tab, slots.data(), slots.size() * 8, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return cuda_err(e, "exp table copy");
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_err(e, "cudaDeviceGetAttribute");
        s.scratch = static_cast<unsigned char*>(scratch);
        s.tab = static_cast<unsigned long long*>(tab);
        s.mask = unsigned(slots.size() - 1);
        s.n_lists = std::min(sms, kMaxLists);
        s.ready = true;
    }
    *out = s;
    return QNT_OK;
}

}  // namespace

extern "C" int qnt_sampler_sample_noalloc(const qnt_sampler_params* sp, uint64_t* rng_state, float* logits, int n_valid,
                                          const int* history, int n_history, int* token, void* stream) {
    using namespace qnt_capi;
    if (!sp || !rng_state || !logits || !token || n_valid <= 0 || n_history < 0 || (n_history > 0 && !history))
        return set_err(QNT_ERR_INVALID, "qnt_sampler_sample_noalloc: bad argument");
    if (n_valid > kMaxVocab)
        return set_err(QNT_ERR_INVALID, "qnt_sampler_sample_noalloc: n_valid " + std::to_string(n_valid) +
                                            " exceeds the no-alloc maximum of " + std::to_string(kMaxVocab));
    if (n_history > kMaxHistory)
        return set_err(QNT_ERR_INVALID, "qnt_sampler_sample_noalloc: n_history " + std::to_string(n_history) +
                                            " exceeds the no-alloc maximum of " + std::to_string(kMaxHistory));
    if (sp->temperature > 0.f && (sp->top_k < 1 || sp->top_k > kListLen))
        return set_err(QNT_ERR_UNSUPPORTED, "the no-alloc sampler supports 1 <= top_k <= 32 when temperature > 0 (qnt_sampler_sample takes any top_k)");
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_err(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return set_err(QNT_ERR_INVALID, "qnt_sampler_sample_noalloc: device id out of range");
    DeviceSetup s;
    if (int r = device_setup(dev, &s)) return r;
    qb::SamplerState* ss = reinterpret_cast<qb::SamplerState*>(s.scratch);
    qb::Cand* lists = reinterpret_cast<qb::Cand*>(s.scratch + kOffLists);
    int* hist = reinterpret_cast<int*>(s.scratch + kOffHist);
    unsigned char* mark = s.scratch + kOffMark;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool greedy = sp->temperature <= 0.f;
    const int K = greedy ? 1 : std::min(sp->top_k, n_valid);
    const bool penal = sp->repeat_penalty != 1.0f && n_history > 0;
    qb::SamplerState in{};
    in.rng = *rng_state;
    e = cudaMemcpyAsync(ss, &in, sizeof in, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_err(e, "sampler state in");
    // Once marks may have been set, a failure must not leave them behind for the next call: clear the ids this call
    // could have marked (stream-ordered memset, no allocation) before reporting it.
    auto fail_marked = [&](cudaError_t err, const char* what) {
        cudaMemsetAsync(mark, 0, size_t(n_valid), st);
        return cuda_err(err, what);
    };
    if (penal) {
        e = cudaMemcpyAsync(hist, history, size_t(n_history) * 4, cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) return cuda_err(e, "sampler history copy");
        e = qb::launch_mark(hist, nullptr, n_history, sp->repeat_window, n_valid, mark, st, false);
        if (e != cudaSuccess) return fail_marked(e, "sampler penalty marks");
    }
    e = qb::launch_topk_partial(logits, n_valid, K, penal ? 1 : 0, sp->repeat_penalty, mark, lists, s.n_lists, st, false,
                                logits);
    if (e != cudaSuccess) return penal ? fail_marked(e, "sampler stage 1") : cuda_err(e, "sampler stage 1");
    const qb::SamplerArgs sa{sp->temperature, sp->top_p, sp->min_p, sp->repeat_penalty, 0, qb::ExpTab{s.tab, s.mask}};
    e = qb::launch_sample_final(lists, s.n_lists, K, sa, ss, nullptr, 0, st, false);
    if (e != cudaSuccess) return cuda_err(e, "sampler stage 2");
    qb::SamplerState outst{};
    e = cudaMemcpyAsync(&outst, ss, sizeof outst, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_err(e, "sampler result");
    *rng_state = outst.rng;
    *token = outst.token;
    return QNT_OK;
}
