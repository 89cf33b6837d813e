// quanta_b200: the command-line driver of the reference (tools/cli/main.cpp:55-75, 168-303) over the C ABI of
// include/quanta_b200.h.  Commands that need the tokenizer (run, chat, tokenize, ppl) take token ids instead and say so;
// the checks print the reference's result lines (engine/src/checks.cpp:109-110, 140-176, 178-239).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "quanta_b200.h"

namespace {

using Clock = std::chrono::steady_clock;
double seconds_since(Clock::time_point t) { return std::chrono::duration<double>(Clock::now() - t).count(); }

struct Args {
    std::string cmd, model, out, ids;
    int n_gen = 64;
    int ctx = 4096;
    bool batch = true, full_head = false;
    qnt_sampler_params sp{0.7f, 20, 0.8f, 0.0f, 1.1f, 0, 0};
};

[[noreturn]] void usage() {
    std::fprintf(stderr,
                 "usage:\n"
                 "  quanta_b200 gen        -m model.qnt --ids 1,2,3 [-n 64]     greedy ids after the prompt\n"
                 "  quanta_b200 logits     -m model.qnt --ids 1,2,3 -o out.bin  logits of every position (f32)\n"
                 "  quanta_b200 checkbatch -m model.qnt --ids ...              batched prefill must equal token-by-token\n"
                 "  quanta_b200 checkhead  -m model.qnt --ids ...              shortlist head must equal the full head\n"
                 "  quanta_b200 bench      -m model.qnt [--ids ...] [-n 256]   prefill / decode throughput\n"
                 "  quanta_b200 selftest                                        check + time the matvec / matmul kernels\n"
                 "  (run, chat, tokenize, ppl need the tokenizer: pass token ids with --ids)\n"
                 "common: --ctx 4096  --no-batch (prefill token by token)  --full-head (skip the shortlist head)\n"
                 "sampling: --temp 0.7 --top-k 20 --top-p 0.8 --min-p 0 --repeat-penalty 1.1 --seed N --greedy\n");
    std::exit(2);
}

std::vector<int> parse_ids(const std::string& s) {
    std::vector<int> v;
    const char* p = s.c_str();
    while (*p) {
        char* e = nullptr;
        const long x = std::strtol(p, &e, 10);
        if (e == p) break;
        v.push_back(int(x));
        p = *e == ',' ? e + 1 : e;
    }
    return v;
}

Args parse(int argc, char** argv) {
    if (argc < 2) usage();
    Args a;
    a.cmd = argv[1];
    for (int i = 2; i < argc; ++i) {
        const std::string k = argv[i];
        auto next = [&]() -> std::string {
            if (i + 1 >= argc) usage();
            return argv[++i];
        };
        if (k == "-m") a.model = next();
        else if (k == "-o") a.out = next();
        else if (k == "--ids") a.ids = next();
        else if (k == "-n") a.n_gen = std::atoi(next().c_str());
        else if (k == "--ctx") a.ctx = std::atoi(next().c_str());
        else if (k == "--no-batch") a.batch = false;
        else if (k == "--full-head") a.full_head = true;
        else if (k == "--temp") a.sp.temperature = float(std::atof(next().c_str()));
        else if (k == "--top-k") a.sp.top_k = std::atoi(next().c_str());
        else if (k == "--top-p") a.sp.top_p = float(std::atof(next().c_str()));
        else if (k == "--min-p") a.sp.min_p = float(std::atof(next().c_str()));
        else if (k == "--repeat-penalty") a.sp.repeat_penalty = float(std::atof(next().c_str()));
        else if (k == "--seed") a.sp.seed = std::strtoull(next().c_str(), nullptr, 10);
        else if (k == "--greedy") {
            a.sp.temperature = 0.f;
            a.sp.repeat_penalty = 1.f;
        } else usage();
    }
    return a;
}

bool ok_or_report(int rc, const char* what) {
    if (rc >= 0) return true;
    std::fprintf(stderr, "%s failed (%d): %s\n", what, rc, qnt_last_error());
    return false;
}

// ---- selftest: engine/src/checks.cpp:64-143 on the device

uint64_t g_rng = 0x9E3779B97F4A7C15ULL;
uint64_t next_u64() {
    g_rng ^= g_rng << 13;
    g_rng ^= g_rng >> 7;
    g_rng ^= g_rng << 17;
    return g_rng;
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = uint32_t(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {  // subnormal: renormalise
            int ee = -1;
            uint32_t mm = m;
            do {
                ++ee;
                mm <<= 1;
            } while (!(mm & 0x400u));
            bits = sign | uint32_t(127 - 15 - ee) << 23 | (mm & 0x3FFu) << 13;
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | m << 13;
    } else {
        bits = sign | (e + 112) << 23 | m << 13;
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// The definition of the integer matvec (matvec_q_ref): per row, acc = acc + (float(s_b) * dw_b) * dx_b in block order.
void host_matvec(int dt, int rows, int cols, const uint8_t* buf, const int8_t* q, const float* d, float* out) {
    const int nb = cols / 32;
    const size_t qbytes = dt == QNT_Q8_0 ? size_t(rows) * cols : size_t(rows) * cols / 2;
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(buf + qbytes);
    for (int r = 0; r < rows; ++r) {
        volatile float acc = 0.f;  // one rounding per operation, in order
        for (int b = 0; b < nb; ++b) {
            int s = 0;
            for (int i = 0; i < 32; ++i) {
                int w;
                if (dt == QNT_Q8_0) {
                    w = int8_t(buf[size_t(r) * cols + size_t(b) * 32 + i]);
                } else {
                    const uint8_t byte = buf[size_t(r) * cols / 2 + size_t(b) * 16 + (i & 15)];
                    w = int(i < 16 ? (byte & 15) : (byte >> 4)) - 8;
                }
                s += w * q[b * 32 + i];
            }
            volatile float t = float(s);
            t = t * f16_to_f32(sc[size_t(r) * nb + b]);
            t = t * d[b];
            acc = acc + t;
        }
        out[r] = acc;
    }
}

int selftest() {
    bool ok = true;
    const int rows = 4864, cols = 896;  // one Qwen2.5-0.5B MLP matrix
    for (int dt : {QNT_Q8_0, QNT_Q4_0}) {
        const size_t qbytes = dt == QNT_Q8_0 ? size_t(rows) * cols : size_t(rows) * cols / 2;
        std::vector<uint8_t> buf(qbytes + size_t(rows) * cols / 32 * 2);
        for (size_t i = 0; i < qbytes; ++i) buf[i] = uint8_t(next_u64());
        uint16_t* scales = reinterpret_cast<uint16_t*>(buf.data() + qbytes);
        for (int i = 0; i < rows * cols / 32; ++i) scales[i] = uint16_t(0x2000 + next_u64() % 0x800);
        std::vector<float> x(cols);
        for (float& v : x) v = float(int(next_u64() % 2001) - 1000) / 1000.f;
        std::vector<int8_t> q(cols);
        std::vector<float> d(cols / 32);
        if (!ok_or_report(qnt_quantize_q8_host(x.data(), cols, q.data(), d.data()), "quantize_q8")) return 1;
        qnt_dtensor* W = nullptr;
        if (!ok_or_report(qnt_tensor_upload(dt, rows, cols, buf.data(), &W), "tensor upload")) return 1;
        std::vector<float> want(rows), got(rows);
        host_matvec(dt, rows, cols, buf.data(), q.data(), d.data(), want.data());
        if (!ok_or_report(qnt_matvec_host(W, q.data(), d.data(), 0, rows, got.data()), "matvec")) return 1;
        double max_abs = 0, scale = 0;
        for (int r = 0; r < rows; ++r) {
            max_abs = std::max(max_abs, std::fabs(double(got[r]) - want[r]));
            scale = std::max(scale, std::fabs(double(want[r])));
        }
        const bool exact = std::equal(got.begin(), got.end(), want.begin());
        ok &= exact;
        const int iters = 50;
        auto t = Clock::now();
        for (int i = 0; i < iters; ++i) qnt_matvec_host(W, q.data(), d.data(), 0, rows, got.data());
        const double sec = seconds_since(t) / iters;
        std::printf("%-5s cuda      matvec max err %.2e (of output scale) %s  %7.1f us  (host buffers in and out)\n",
                    dt == QNT_Q8_0 ? "Q8_0" : "Q4_0", max_abs / scale, exact ? "PASS" : "FAIL", sec * 1e6);
        // matmul: n tokens at once must equal the matvec per token, bit for bit (CUDA cores and tensor cores)
        const int n = 32;
        std::vector<int8_t> qs(size_t(n) * cols);
        std::vector<float> ds(size_t(n) * (cols / 32)), want_mm(size_t(n) * rows), got_mm(size_t(n) * rows);
        for (int tk = 0; tk < n; ++tk) {
            for (float& v : x) v = float(int(next_u64() % 2001) - 1000) / 1000.f;
            qnt_quantize_q8_host(x.data(), cols, qs.data() + size_t(tk) * cols, ds.data() + size_t(tk) * (cols / 32));
            qnt_matvec_host(W, qs.data() + size_t(tk) * cols, ds.data() + size_t(tk) * (cols / 32), 0, rows,
                            want_mm.data() + size_t(tk) * rows);
        }
        for (int impl : {1, 2}) {
            bool exact_mm = true;
            for (int n_try : {n, 7}) {
                std::fill(got_mm.begin(), got_mm.end(), 0.f);
                if (!ok_or_report(qnt_matmul_host(W, qs.data(), ds.data(), n_try, 0, rows, got_mm.data(), rows, impl), "matmul"))
                    return 1;
                exact_mm &= std::equal(got_mm.begin(), got_mm.begin() + size_t(n_try) * rows, want_mm.begin());
            }
            ok &= exact_mm;
            std::printf("%-5s %-9s matmul x%d: bit-exact %s\n", dt == QNT_Q8_0 ? "Q8_0" : "Q4_0",
                        impl == 1 ? "cuda" : "tcgen05", n, exact_mm ? "PASS" : "FAIL");
        }
        qnt_tensor_free(W);
    }
    std::printf("selftest %s\n", ok ? "PASS" : "FAIL");
    return ok ? 0 : 1;
}

// ---- model commands

struct Model {
    qnt_model* m = nullptr;
    qnt_hparams hp{};
    ~Model() {
        if (m) qnt_model_close(m);
    }
};

bool open_model(const Args& a, Model& md) {
    if (a.model.empty()) usage();
    auto t0 = Clock::now();
    if (!ok_or_report(qnt_model_open(a.model.c_str(), a.ctx, 0, &md.m), "load")) return false;
    qnt_model_hparams(md.m, &md.hp);
    std::fprintf(stderr, "quanta_b200: loaded %s in %.2fs (dim=%d layers=%d heads=%d/%d vocab=%d ctx=%d)\n", a.model.c_str(),
                 seconds_since(t0), md.hp.dim, md.hp.n_layers, md.hp.n_heads, md.hp.n_kv_heads, md.hp.vocab_size,
                 md.hp.ctx_len);
    return true;
}

int check_batch(Model& md, const std::vector<int>& ids) {  // engine/src/checks.cpp:148-176
    const int V = md.hp.vocab_size;
    std::vector<float> want(static_cast<size_t>(V)), got(static_cast<size_t>(V));
    bool ok = true;
    auto check = [&](int pos0, int n) {
        if (pos0 + n > int(ids.size()) || pos0 + n > md.hp.ctx_len) return;
        for (int p = 0; p < pos0 + n; ++p) qnt_model_forward(md.m, ids[size_t(p)], p, nullptr, want.data());
        if (pos0 > 0) qnt_model_forward_batch(md.m, ids.data(), pos0, 0, nullptr, nullptr);
        qnt_model_forward_batch(md.m, ids.data() + pos0, n, pos0, nullptr, got.data());
        float maxd = 0.f;
        for (int i = 0; i < V; ++i) maxd = std::max(maxd, std::fabs(got[size_t(i)] - want[size_t(i)]));
        std::printf("batch pos0=%4d n=%4d  max |diff| %.3g  %s\n", pos0, n, maxd, maxd == 0.f ? "PASS" : "FAIL");
        ok &= maxd == 0.f;
    };
    for (int n : {1, 31, 32, 33, 100}) check(0, n);
    check(40, 45);
    if (ids.size() > 100) check(0, int(ids.size()));
    return ok ? 0 : 1;
}

int check_head(Model& md, const std::vector<int>& ids) {  // engine/src/checks.cpp:178-239
    if (!md.hp.has_shortlist) {
        std::printf("this file has no shortlist head (export with --shortlist)\n");
        return 1;
    }
    const int V = md.hp.vocab_size, nv = std::min(md.hp.n_tokens, V);
    const int n = std::min(int(ids.size()), md.hp.ctx_len);
    std::vector<float> full(static_cast<size_t>(V)), sl(static_cast<size_t>(V)), coarse(static_cast<size_t>(V)), upper(static_cast<size_t>(V));
    std::vector<int> order(static_cast<size_t>(nv));
    long bad = 0, violations = 0;
    for (int k : {1, 20}) {
        double t_full = 0, t_sl = 0, rows = 0, sum_bound = 0, sum_diff = 0;
        std::vector<int> row_counts;
        for (int p = 0; p < n; ++p) {
            qnt_model_forward(md.m, ids[size_t(p)], p, nullptr, nullptr);
            auto t = Clock::now();
            qnt_model_head(md.m, nullptr, full.data(), nullptr, nullptr);
            t_full += seconds_since(t);
            std::vector<int> must(ids.begin() + std::max(0, p - 63), ids.begin() + p + 1);
            qnt_head_query hq{k, nv, must.data(), int(must.size())};
            t = Clock::now();
            if (!ok_or_report(qnt_model_head(md.m, &hq, sl.data(), coarse.data(), upper.data()), "shortlist head")) return 1;
            t_sl += seconds_since(t);
            const int r = qnt_model_last_head_rows(md.m);
            row_counts.push_back(r);
            rows += r;
            for (int v = 0; v < V; ++v) {
                const float bnd = upper[size_t(v)] - coarse[size_t(v)];
                const float dif = std::fabs(full[size_t(v)] - coarse[size_t(v)]);
                if (dif > bnd) ++violations;
                sum_bound += bnd;
                sum_diff += dif;
            }
            for (int v = 0; v < nv; ++v) order[size_t(v)] = v;
            std::partial_sort(order.begin(), order.begin() + k, order.end(),
                              [&](int x, int y) { return full[size_t(x)] > full[size_t(y)]; });
            for (int v = 0; v < nv; ++v)
                if (sl[size_t(v)] != -INFINITY && sl[size_t(v)] != full[size_t(v)]) ++bad;
            for (int i = 0; i < k; ++i)
                if (sl[size_t(order[size_t(i)])] != full[size_t(order[size_t(i)])]) ++bad;
            for (int id : must)
                if (id < nv && sl[size_t(id)] != full[size_t(id)]) ++bad;
        }
        std::sort(row_counts.begin(), row_counts.end());
        std::printf("head top_k=%2d over %d tokens: exact rows mean %.0f median %d p99 %d of %d (%.2f%%) | "
                    "head time full %.2f ms, shortlist %.2f ms\n",
                    k, n, rows / n, row_counts[size_t(n / 2)], row_counts[size_t(std::min(n - 1, n * 99 / 100))], V,
                    100.0 * rows / n / V, 1e3 * t_full / n, 1e3 * t_sl / n);
        std::printf("  mean bound %.3f vs mean actual |exact - coarse| %.3f\n", sum_bound / n / V, sum_diff / n / V);
    }
    std::printf("head bound violations: %ld   mismatches: %ld   %s\n", violations, bad,
                violations == 0 && bad == 0 ? "PASS" : "FAIL");
    return violations == 0 && bad == 0 ? 0 : 1;
}

int gen(Model& md, const Args& a, const std::vector<int>& ids, bool greedy) {
    qnt_sampler_params sp = a.sp;
    if (greedy) {
        sp.temperature = 0.f;
        sp.repeat_penalty = 1.f;
    }
    std::vector<int> out(static_cast<size_t>(std::max(a.n_gen, 1)));
    qnt_gen_stats st{};
    const int flags = (a.full_head ? 0 : QNT_GEN_SHORTLIST) | (a.batch ? QNT_GEN_BATCH_PREFILL : 0);
    const int n = qnt_generate(md.m, ids.data(), int(ids.size()), &sp, flags, a.n_gen, out.data(), &st);
    if (!ok_or_report(n, "generate")) return 1;
    for (int i = 0; i < n; ++i) std::printf(i ? ",%d" : "%d", out[size_t(i)]);
    std::printf("\n");
    std::fprintf(stderr, "prefill: %zu tok %.2f tok/s | decode: %d tok %.2f tok/s\n", ids.size(),
                 ids.size() / (st.prefill_ms / 1e3), n, n / (st.decode_ms / 1e3));
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc >= 2 && std::strcmp(argv[1], "selftest") == 0) return selftest();
    Args a = parse(argc, argv);
    if (a.cmd == "run" || a.cmd == "chat" || a.cmd == "tokenize" || a.cmd == "ppl") {
        std::fprintf(stderr, "%s needs the tokenizer, which this build does not carry: give token ids to gen --ids\n",
                     a.cmd.c_str());
        return 2;
    }
    Model md;
    if (!open_model(a, md)) return 1;
    const std::vector<int> ids = parse_ids(a.ids);
    if (ids.empty() && a.cmd != "bench") {
        std::fprintf(stderr, "no input: pass --ids\n");
        return 1;
    }
    if (a.cmd == "gen") return gen(md, a, ids, true);
    if (a.cmd == "logits") {
        FILE* f = std::fopen(a.out.c_str(), "wb");
        if (!f) {
            std::fprintf(stderr, "cannot write %s\n", a.out.c_str());
            return 1;
        }
        std::vector<float> lg(static_cast<size_t>(md.hp.vocab_size));
        for (size_t p = 0; p < ids.size(); ++p) {
            if (!ok_or_report(qnt_model_forward(md.m, ids[p], int(p), nullptr, lg.data()), "forward")) return 1;
            std::fwrite(lg.data(), sizeof(float), lg.size(), f);
        }
        std::fclose(f);
        return 0;
    }
    if (a.cmd == "checkbatch") return check_batch(md, ids);
    if (a.cmd == "checkhead") return check_head(md, ids);
    if (a.cmd == "bench") {
        std::vector<int> prompt = ids;
        uint64_t s = 42;
        while (prompt.size() < 512) {
            s = s * 6364136223846793005ULL + 1442695040888963407ULL;
            prompt.push_back(int((s >> 33) % uint64_t(md.hp.n_tokens)));
        }
        Args b = a;
        b.n_gen = a.n_gen > 0 ? a.n_gen : 256;
        std::printf("bench: %zu-token prompt, %d decode tokens, T=%.2f top-k %d top-p %.2f repeat %.2f, %s head\n",
                    prompt.size(), b.n_gen, b.sp.temperature, b.sp.top_k, b.sp.top_p, b.sp.repeat_penalty,
                    b.full_head ? "full" : "shortlist");
        return gen(md, b, prompt, false);
    }
    usage();
}
