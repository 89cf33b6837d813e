// The host's expf, measured: every float x whose expf(x) differs from the double-precision exp rounded once to float.
//
// The reference evaluates e^x with the host libm's expf (std::exp on float: engine/src/ops_ref.cpp:221, :247;
// sampler.cpp:58).  glibc's expf is within 0.502 ulp of e^x, so it returns the correctly rounded value except for
// inputs whose e^x lies within ~0.002 ulp of a rounding midpoint, where it may pick the other neighbour.  The device
// computes the correctly rounded value (double exp) and, only in that near-midpoint case, looks x up in this table
// to return the libm's choice -- so softmax, SwiGLU and the sampler see the reference's bits.
//
// The table is built by scanning all floats in (-104, 89) (outside, expf is 0 / inf or its argument never occurs),
// on all host threads, and cached in a file keyed by a fingerprint of the libm.
#include "exp_table.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace qb {

namespace {

uint32_t f2u(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}
float u2f(uint32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

void scan_range(uint32_t b0, uint32_t b1, std::vector<uint64_t>* out, long* far) {
    for (uint32_t b = b0; b < b1; ++b) {
        const float x = u2f(b);
        if (!(x > -104.f && x < 89.f)) continue;
        const float a = std::exp(x);  // float overload: the libm's expf, like the reference
        const double y = std::exp(double(x));
        const float f = float(y);
        if (f2u(a) != f2u(f)) {
            out->push_back((uint64_t(b) << 32) | f2u(a));
            // the device only looks up near-midpoint inputs: count any exception outside that band
            const double df = double(f), e = y - df;
            const float nb = e >= 0 ? std::nextafter(f, INFINITY) : std::nextafter(f, -INFINITY);
            const double half = std::fabs(double(nb) - df) * 0.5;
            if (!(half - std::fabs(e) < half * kExpNearMidpoint)) ++*far;
        }
    }
}

uint64_t fingerprint() {
    uint64_t h = 1469598103934665603ULL;
    for (float x : {0.1f, -1.5f, 3.14159f, -20.25f, 0.000123f, 80.5f, -90.0f, 0.0078125f}) {
        h = (h ^ f2u(std::exp(x))) * 1099511628211ULL;
    }
    return h;
}

std::vector<uint64_t> build_entries(std::string* note) {
    const uint64_t fp = fingerprint();
    const char* dir = std::getenv("QNT_CACHE_DIR");
    const std::string path = std::string(dir ? dir : "/tmp") + "/qnt_b200_expf_" + std::to_string(fp) + ".bin";
    if (FILE* f = std::fopen(path.c_str(), "rb")) {
        uint64_t n = 0;
        std::vector<uint64_t> v;
        if (std::fread(&n, 8, 1, f) == 1 && n < (1u << 24)) {
            v.resize(size_t(n));
            if (std::fread(v.data(), 8, size_t(n), f) != size_t(n)) v.clear();
        }
        std::fclose(f);
        // spot-check the cache against the live libm
        bool ok = !v.empty();
        for (size_t i = 0; ok && i < v.size(); i += 997)
            ok = f2u(std::exp(u2f(uint32_t(v[i] >> 32)))) == uint32_t(v[i]);
        if (ok) {
            if (note) *note = "cached " + path;
            return v;
        }
    }
    unsigned nt = std::thread::hardware_concurrency();
    if (nt == 0) nt = 4;
    std::vector<std::vector<uint64_t>> parts(nt);
    std::vector<long> far(nt, 0);
    std::vector<std::thread> ts;
    const uint64_t total = 0x100000000ULL;
    for (unsigned t = 0; t < nt; ++t)
        ts.emplace_back([&, t] {
            scan_range(uint32_t(total * t / nt), uint32_t(std::min<uint64_t>(total * (t + 1) / nt, 0xFFFFFFFFu)), &parts[t],
                       &far[t]);
        });
    for (auto& th : ts) th.join();
    std::vector<uint64_t> v;
    long nfar = 0;
    for (unsigned t = 0; t < nt; ++t) {
        v.insert(v.end(), parts[t].begin(), parts[t].end());
        nfar += far[t];
    }
    if (note) *note = "scanned (" + std::to_string(v.size()) + " exceptions, " + std::to_string(nfar) + " outside the band)";
    if (FILE* f = std::fopen((path + ".tmp").c_str(), "wb")) {
        const uint64_t n = v.size();
        std::fwrite(&n, 8, 1, f);
        std::fwrite(v.data(), 8, v.size(), f);
        std::fclose(f);
        std::rename((path + ".tmp").c_str(), path.c_str());
    }
    return v;
}

std::mutex g_mu;
std::vector<uint64_t>* g_slots = nullptr;  // host copy of the hash table (built once per process)
std::string g_note;

}  // namespace

const std::vector<uint64_t>& expf_exception_slots(std::string* note) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_slots) {
        const std::vector<uint64_t> entries = build_entries(&g_note);
        size_t cap = 1;
        while (cap < entries.size() * 3) cap <<= 1;
        g_slots = new std::vector<uint64_t>(cap, ~0ULL);
        const uint32_t mask = uint32_t(cap - 1);
        for (uint64_t e : entries) {
            uint32_t h = exp_hash(uint32_t(e >> 32)) & mask;
            while ((*g_slots)[h] != ~0ULL) h = (h + 1) & mask;
            (*g_slots)[h] = e;
        }
    }
    if (note) *note = g_note;
    return *g_slots;
}

}  // namespace qb
