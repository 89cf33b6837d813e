// The reference's kernel registry (the interface of engine/src/ops_dispatch.cpp:53-77 -- matvec_q, matmul_q,
// matvec_q_kernel_name, available_matvec_q_kernels, available_matmul_q_kernels) with the B200 kernels added as two
// more families, reached through the C ABI of include/quanta_b200.h:
//   cuda      qnt_matvec_host, and qnt_matmul_host on the CUDA cores
//   cuda_tc   the same matvec, and qnt_matmul_host on the tensor cores (tcgen05)
// oracle/Makefile links this file in place of the reference's ops_dispatch.cpp, with the reference's other engine
// sources and its CLI, into oracle/_ref/cuda/quanta: the reference's own `quanta selftest` (engine/src/checks.cpp:64-146)
// then checks every family against matvec_q_ref and each family's matmul against its matvec, bit for bit.
// QUANTA_KERNEL=cuda or cuda_tc makes that family the one Model::linear uses.
//
// TEST INFRASTRUCTURE (the drop-in's worked example); the product never links it.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "ops.h"
#include "quanta_b200.h"

namespace quanta {

namespace {

// The function-pointer interface has no error channel, so a device failure ends the process with the reason.
[[noreturn]] void device_failure(const char* what) {
    std::fprintf(stderr, "cuda kernel family: %s failed: %s\n", what, qnt_last_error());
    std::abort();
}

// A cheap fingerprint of a weight matrix's bytes (both ends of the quants and of the scales), so that a caller reusing
// one buffer for other weights gets a fresh upload.
uint64_t fingerprint(const Tensor& W) {
    const size_t qbytes = W.quant_bytes(), sbytes = size_t(W.rows) * W.cols / QK * 2;
    uint64_t h = 0xcbf29ce484222325ULL ^ (uint64_t(W.rows) << 32 | uint32_t(W.cols)) ^ uint64_t(W.dtype);
    auto mix = [&h](const uint8_t* p, size_t n) {
        for (size_t i = 0; i < n; ++i) h = (h ^ p[i]) * 0x100000001b3ULL;
    };
    const size_t k = 256;
    mix(W.data, std::min(k, qbytes));
    mix(W.data + qbytes - std::min(k, qbytes), std::min(k, qbytes));
    mix(W.data + qbytes, std::min(k, sbytes));
    mix(W.data + qbytes + sbytes - std::min(k, sbytes), std::min(k, sbytes));
    return h;
}

// One device copy per weight matrix, uploaded on its first use (the .qnt bytes as they are mapped).
qnt_dtensor* device_copy(const Tensor& W) {
    struct Entry {
        uint64_t sig;
        qnt_dtensor* t;
    };
    static std::mutex mu;
    static std::unordered_map<const void*, Entry> cache;
    const uint64_t sig = fingerprint(W);
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(W.data);
    if (it != cache.end() && it->second.sig == sig) return it->second.t;
    if (it != cache.end()) qnt_tensor_free(it->second.t);
    qnt_dtensor* t = nullptr;
    if (qnt_tensor_upload(int(W.dtype), W.rows, W.cols, W.data, &t) != QNT_OK) device_failure("qnt_tensor_upload");
    cache[W.data] = Entry{sig, t};
    return t;
}

void matvec_q_cuda(float* out, const Tensor& W, const QuantVec& x, int r0, int r1) {
    if (qnt_matvec_host(device_copy(W), x.q.data(), x.d.data(), r0, r1, out) != QNT_OK) device_failure("qnt_matvec_host");
}

// n QuantVecs as the contiguous [n][cols] / [n][cols/32] arrays the C ABI takes
void matmul_q_cuda_impl(float* out, int ldo, const Tensor& W, const QuantVec* x, int n, int r0, int r1, int impl) {
    thread_local std::vector<int8_t> q;
    thread_local std::vector<float> d;
    const int cols = W.cols, nb = cols / QK;
    q.resize(size_t(n) * cols);
    d.resize(size_t(n) * nb);
    for (int t = 0; t < n; ++t) {
        std::memcpy(q.data() + size_t(t) * cols, x[t].q.data(), size_t(cols));
        std::memcpy(d.data() + size_t(t) * nb, x[t].d.data(), size_t(nb) * 4);
    }
    if (qnt_matmul_host(device_copy(W), q.data(), d.data(), n, r0, r1, out, ldo, impl) != QNT_OK)
        device_failure("qnt_matmul_host");
}
void matmul_q_cuda(float* out, int ldo, const Tensor& W, const QuantVec* x, int n, int r0, int r1) {
    matmul_q_cuda_impl(out, ldo, W, x, n, r0, r1, 1);
}
void matmul_q_cuda_tc(float* out, int ldo, const Tensor& W, const QuantVec* x, int n, int r0, int r1) {
    matmul_q_cuda_impl(out, ldo, W, x, n, r0, r1, 2);
}

struct Family {
    const char* name;
    MatvecQFn mv;
    MatmulQFn mm;
};

// The families this process can run: the scalar reference always, the device ones when a GPU is present.
const std::vector<Family>& families() {
    static const std::vector<Family> fs = [] {
        std::vector<Family> v = {{"ref", matvec_q_ref, matmul_q_ref}};
        if (qnt_device_count() > 0) {
            v.push_back({"cuda", matvec_q_cuda, matmul_q_cuda});
            v.push_back({"cuda_tc", matvec_q_cuda, matmul_q_cuda_tc});
        }
        return v;
    }();
    return fs;
}

// QUANTA_KERNEL names the family; the default stays the reference's choice on this CPU (ref).
const Family& active() {
    static const Family& f = [] () -> const Family& {
        const char* want = std::getenv("QUANTA_KERNEL");
        for (const Family& c : families())
            if (want && std::strcmp(want, c.name) == 0) return c;
        return families().front();
    }();
    return f;
}

}  // namespace

void matvec_q(float* out, const Tensor& W, const QuantVec& x, int r0, int r1) { active().mv(out, W, x, r0, r1); }

void matmul_q(float* out, int ldo, const Tensor& W, const QuantVec* x, int n, int r0, int r1) {
    active().mm(out, ldo, W, x, n, r0, r1);
}

const char* matvec_q_kernel_name() { return active().name; }

std::vector<std::pair<const char*, MatvecQFn>> available_matvec_q_kernels() {
    std::vector<std::pair<const char*, MatvecQFn>> v;
    for (const Family& f : families()) v.emplace_back(f.name, f.mv);
    return v;
}

std::vector<std::pair<const char*, MatmulQFn>> available_matmul_q_kernels() {
    std::vector<std::pair<const char*, MatmulQFn>> v;
    for (const Family& f : families()) v.emplace_back(f.name, f.mm);
    return v;
}

}  // namespace quanta
