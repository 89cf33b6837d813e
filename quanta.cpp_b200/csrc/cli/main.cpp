// quanta_b200: the command-line driver of the reference (tools/cli/main.cpp:55-75, 168-328) over the C ABI of
// include/quanta_b200.h, with the same commands, flags and result lines (engine/src/checks.cpp:109-110, 140-176,
// 178-239, 241-263, 299-301, 307-423).  Text goes through the host tokenizer (qnt_tokenize); the model runs on the GPU.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <functional>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

#include "quanta_b200.h"

namespace {

using Clock = std::chrono::steady_clock;
double seconds_since(Clock::time_point t) { return std::chrono::duration<double>(Clock::now() - t).count(); }

// The chat template's default system message (the Qwen2.5 convention, the reference CLI's default).
const char* kDefaultSystem = "You are Qwen, created by Alibaba Cloud. You are a helpful assistant.";

struct Args {
    std::string cmd, model, out, ids, prompt, file, system = kDefaultSystem;
    int n_gen = 256;
    int ctx = 4096;
    int threads = 0;  // accepted for the reference's flag set; the device does not use host threads
    bool batch = true, full_head = false, kv_f32 = false, nibble_head = false;
    qnt_sampler_params sp{0.7f, 20, 0.8f, 0.0f, 1.1f, 0, 0};
};

[[noreturn]] void usage() {
    std::fprintf(stderr,
                 "usage:\n"
                 "  quanta_b200 chat     -m model.qnt [--system TEXT] [sampling flags]\n"
                 "  quanta_b200 run      -m model.qnt (-p TEXT | -f FILE) [-n 256] [sampling flags]\n"
                 "  quanta_b200 tokenize -m model.qnt (-p TEXT | -f FILE)\n"
                 "  quanta_b200 logits   -m model.qnt --ids 1,2,3 -o out.bin\n"
                 "  quanta_b200 gen      -m model.qnt --ids 1,2,3 [-n 64]\n"
                 "  quanta_b200 ppl      -m model.qnt -f FILE [-n 1024]         perplexity of the first n tokens\n"
                 "  quanta_b200 checkbatch -m model.qnt (-p TEXT | -f FILE)     batched prefill must equal token-by-token\n"
                 "  quanta_b200 checkhead  -m model.qnt (-p TEXT | -f FILE)     shortlist head must equal the full head\n"
                 "  quanta_b200 batchcurve -m model.qnt                         cost of a pass of 1..32 tokens vs one decode step\n"
                 "  quanta_b200 compare   -m model.qnt                          engine-comparison protocol (RESULT lines)\n"
                 "  quanta_b200 prompt                                          print the comparison prompt\n"
                 "  quanta_b200 bench     -m model.qnt                          full report (checks + speed)\n"
                 "  quanta_b200 selftest                                        check + time kernels (no model needed)\n"
                 "  quanta_b200 export-layout IN.qnt OUT.qnt                    copy with the device's fused tensors pre-packed\n"
                 "common: --ctx 4096  -t THREADS (ignored: the GPU runs the model)  --no-batch (prefill token by token)\n"
                 "        --full-head (skip the shortlist head)  (--kv-f32 is not available: the device KV cache is f16)\n"
                 "        --nibble-head (screen the shortlist head with the Q8 head's high nibble plane; no head_q4 needed)\n"
                 "        --ids 1,2,3 (token ids instead of -p / -f text, any command that takes text)\n"
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
        else if (k == "-p") a.prompt = next();
        else if (k == "-f") a.file = next();
        else if (k == "--system") a.system = next();
        else if (k == "-n") a.n_gen = std::atoi(next().c_str());
        else if (k == "--ctx") a.ctx = std::atoi(next().c_str());
        else if (k == "-t") a.threads = std::atoi(next().c_str());
        else if (k == "--kv-f32") a.kv_f32 = true;
        else if (k == "--no-batch") a.batch = false;
        else if (k == "--full-head") a.full_head = true;
        else if (k == "--nibble-head") a.nibble_head = true;
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
    if (a.model.empty()) usage();
    return a;
}

std::string read_file(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) {
        std::fprintf(stderr, "cannot read %s\n", path.c_str());
        std::exit(1);
    }
    std::ostringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

void print_piece(const std::string& s) {
    std::fwrite(s.data(), 1, s.size(), stdout);
    std::fflush(stdout);
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
        std::printf("%-5s cuda      matvec max err %.2e (of output scale) %s  %7.1f us  %6.2f GB/s (host buffers in and out)\n",
                    dt == QNT_Q8_0 ? "q8_0" : "q4_0", max_abs / scale, exact ? "PASS" : "FAIL", sec * 1e6,
                    double(buf.size()) / sec / 1e9);
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
            std::printf("%-5s %-9s matmul x%d: bit-exact %s\n", dt == QNT_Q8_0 ? "q8_0" : "q4_0",
                        impl == 1 ? "cuda" : "cuda_tc", n, exact_mm ? "PASS" : "FAIL");
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
    if (a.kv_f32) {
        std::fprintf(stderr, "--kv-f32: the device keeps the KV cache in f16 only\n");
        return false;
    }
    auto t0 = Clock::now();
    if (!ok_or_report(qnt_model_open(a.model.c_str(), a.ctx, a.nibble_head ? QNT_OPEN_NIBBLE_SCREEN : 0, &md.m), "load"))
        return false;
    qnt_model_hparams(md.m, &md.hp);
    std::fprintf(stderr, "quanta_b200: loaded %s in %.2fs (dim=%d layers=%d heads=%d/%d vocab=%d ctx=%d)\n", a.model.c_str(),
                 seconds_since(t0), md.hp.dim, md.hp.n_layers, md.hp.n_heads, md.hp.n_kv_heads, md.hp.vocab_size,
                 md.hp.ctx_len);
    return true;
}

// The model file's tokenizer on the host.
struct Text {
    qnt_tokenizer* t = nullptr;
    ~Text() {
        if (t) qnt_tokenizer_free(t);
    }
    bool open(const std::string& path) { return ok_or_report(qnt_tokenizer_open(path.c_str(), &t), "tokenizer"); }
    std::vector<int> encode(const std::string& s) const {
        const int n = qnt_tokenize(t, s.data(), s.size(), nullptr, 0);
        std::vector<int> ids(size_t(std::max(n, 0)));
        if (n > 0) qnt_tokenize(t, s.data(), s.size(), ids.data(), n);
        return ids;
    }
    std::string piece(int id) const {
        const int n = qnt_token_piece(t, id, nullptr, 0);
        std::string p(size_t(std::max(n, 0)), '\0');
        if (n > 0) qnt_token_piece(t, id, &p[0], n);
        return p;
    }
    int id(const char* literal) const { return qnt_token_id(t, literal); }
};

// Plain prose for the speed report, the batch curve and the comparison prompt (a few hundred tokens).
const char* sample_text() {
    return "The ferry left the east bank every morning at six, whatever the weather. Its pilot had learned the river "
           "from her grandfather, who could tell the depth of the channel from the colour of the water and the way the "
           "reeds leaned in the current. In spring the snowmelt turned the river brown and fast, and she kept the engine "
           "low so the hull would not be pushed sideways onto the gravel bars. In late summer the water dropped so far "
           "that she had to mark a new route with painted poles, moving them a little every week. Farmers crossed with "
           "crates of apples and sacks of flour, children crossed to reach the school in town, and once a travelling "
           "orchestra crossed with a piano tied to the deck under a blue tarpaulin. She wrote each crossing in a ledger: "
           "the time, the passengers, the height of the water against the old stone pier. When the county finally "
           "built a bridge two miles downstream, people asked whether she would miss the work. She said the river "
           "would still be there, and that somebody ought to keep counting how high it rose each year. The ledger is "
           "now kept in the town library, where anyone can read how many mornings the boat went out, and how few it "
           "did not.";
}

std::string compare_prompt() { return std::string(sample_text()) + "\n\n" + sample_text() + "\n\nContinue the story:"; }

int check_batch(Model& md, const std::vector<int>& ids, bool quick) {  // engine/src/checks.cpp:148-176
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
    if (!quick && ids.size() > 100) check(0, int(ids.size()));
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

// Session (engine/src/session.h) on the device session API: Session::feed, and Session::generate's loop
// (session.cpp:33-52) one step at a time, so that stop ids end the reply and pieces stream out as they are sampled.
struct DeviceSession {
    Model& md;
    qnt_sampler_params sp;
    int flags;
    int len = 0;       // Session::pos()
    bool used = false;  // a session ran on this model before (its sampler state carries over a reset)
    long long head_rows = 0, head_calls = 0;

    DeviceSession(Model& m, const qnt_sampler_params& p, bool shortlist, bool batch)
        : md(m), sp(p), flags((shortlist ? QNT_GEN_SHORTLIST : 0) | (batch ? QNT_GEN_BATCH_PREFILL : 0)) {}

    bool feed(const std::vector<int>& ids, double* seconds) {
        if (len + int(ids.size()) >= md.hp.ctx_len) return false;  // Session::feed (session.cpp:14)
        const auto t0 = Clock::now();
        const int rc = len == 0 ? qnt_session_begin(md.m, ids.data(), int(ids.size()), &sp, flags | (used ? QNT_GEN_KEEP_RNG : 0))
                                : qnt_session_feed(md.m, ids.data(), int(ids.size()));
        if (!ok_or_report(rc, "feed")) return false;
        qnt_session_last(md.m, nullptr, &len);
        used = true;
        if (seconds) *seconds = seconds_since(t0);
        return true;
    }
    void reset() { len = 0; }
    int generate(int max_tokens, const std::vector<int>& stops, const std::function<bool(int)>& on_token, double* seconds) {
        const auto t0 = Clock::now();
        int n = 0;
        while (n < max_tokens && len < md.hp.ctx_len - 1) {
            if (!ok_or_report(qnt_session_step(md.m, 1), "decode step")) break;
            int id = -1;
            qnt_session_last(md.m, &id, &len);
            ++n;
            if (std::find(stops.begin(), stops.end(), id) != stops.end()) {  // never appended by the reference
                qnt_session_rewind(md.m, 1);
                --len;
                break;
            }
            if (!on_token(id)) break;
        }
        qnt_gen_stats st{};
        if (qnt_session_read(md.m, nullptr, 0, &st) >= 0) {
            head_rows = st.head_rows;
            head_calls = st.head_calls;
        }
        if (seconds) *seconds = seconds_since(t0);
        return n;
    }
    double head_fraction() const {
        return head_calls ? double(head_rows) / (double(head_calls) * md.hp.vocab_size) : 1.0;
    }
};

// Chat::reply (engine/src/session.cpp:94-118): ChatML turns on one growing session.
struct Chat {
    Text& tok;
    std::string system;
    DeviceSession s;
    std::vector<int> stops;
    bool open_turn = false;  // the last reply's <|im_end|> is not in the cache yet
    struct Stats {
        int prompt_tokens = 0, reply_tokens = 0, ctx_used = 0;
        double prefill_seconds = 0, decode_seconds = 0;
    };

    Chat(Model& m, Text& t, std::string sys, const qnt_sampler_params& sp, bool batch, bool shortlist)
        : tok(t), system(std::move(sys)), s(m, sp, shortlist, batch) {
        stops = {tok.id("<|im_end|>"), tok.id("<|endoftext|>")};
    }
    void reset() {
        s.reset();
        open_turn = false;
    }
    bool reply(const std::string& user, int max_tokens, const std::function<bool(const std::string&)>& on_piece, Stats* st) {
        std::string turn;
        if (s.len == 0) turn = "<|im_start|>system\n" + system + "<|im_end|>\n";
        if (open_turn) turn += "<|im_end|>\n";
        turn += "<|im_start|>user\n" + user + "<|im_end|>\n<|im_start|>assistant\n";
        std::vector<int> ids = tok.encode(turn);
        Stats out;
        if (!s.feed(ids, &out.prefill_seconds)) {  // context full: start over with just this message
            reset();
            ids = tok.encode("<|im_start|>system\n" + system + "<|im_end|>\n<|im_start|>user\n" + user +
                             "<|im_end|>\n<|im_start|>assistant\n");
            if (!s.feed(ids, &out.prefill_seconds)) {
                reset();
                return false;
            }
        }
        out.prompt_tokens = int(ids.size());
        out.reply_tokens = s.generate(max_tokens, stops, [&](int id) { return on_piece(tok.piece(id)); }, &out.decode_seconds);
        open_turn = true;
        out.ctx_used = s.len;
        if (st) *st = out;
        return true;
    }
};

int run_text(Model& md, Text& tok, const Args& a, const std::string& text) {  // tools/cli/main.cpp:286-303
    if (text.empty()) usage();
    DeviceSession s(md, a.sp, !a.full_head, a.batch);
    double t_prefill = 0, t_decode = 0;
    const std::vector<int> ids = tok.encode(text);
    if (!s.feed(ids, &t_prefill)) {
        std::fprintf(stderr, "prompt too long for context\n");
        return 1;
    }
    print_piece(text);
    const std::vector<int> stops = {tok.id("<|im_end|>"), tok.id("<|endoftext|>")};
    const int n = s.generate(a.n_gen, stops, [&](int id) { print_piece(tok.piece(id)); return true; }, &t_decode);
    std::fprintf(stderr, "\n[prefill %zu tok @ %.1f tok/s | decode %d tok @ %.1f tok/s | 8-bit head read %.1f%%]\n",
                 ids.size(), ids.size() / t_prefill, n, n / t_decode, 100 * s.head_fraction());
    return 0;
}

int chat_loop(Model& md, Text& tok, const Args& a) {  // tools/cli/main.cpp:305-328
    Chat chat(md, tok, a.system, a.sp, a.batch, !a.full_head);
    std::fprintf(stderr, "Quanta chat. Commands: /reset, /exit\n");
    std::string line;
    while (true) {
        std::fprintf(stderr, "\n> ");
        if (!std::getline(std::cin, line) || line == "/exit") break;
        if (!line.empty() && line.back() == '\r') line.pop_back();
        if (line.empty()) continue;
        if (line == "/reset") {
            chat.reset();
            std::fprintf(stderr, "(conversation cleared)\n");
            continue;
        }
        Chat::Stats st;
        if (!chat.reply(line, a.n_gen, [](const std::string& piece) { print_piece(piece); return true; }, &st)) {
            std::fprintf(stderr, "(message too long)\n");
            continue;
        }
        std::fprintf(stderr, "\n[prefill %d tok @ %.1f tok/s | %d tok @ %.1f tok/s | ctx %d/%d]\n", st.prompt_tokens,
                     st.prompt_tokens / st.prefill_seconds, st.reply_tokens, st.reply_tokens / st.decode_seconds,
                     st.ctx_used, md.hp.ctx_len);
    }
    return 0;
}

int perplexity(Model& md, const Args& a, std::vector<int> ids) {  // tools/cli/main.cpp:261-282
    if (int(ids.size()) > a.n_gen) ids.resize(size_t(a.n_gen));
    if (int(ids.size()) >= md.hp.ctx_len) ids.resize(size_t(md.hp.ctx_len - 1));
    if (ids.size() < 2) {
        std::fprintf(stderr, "ppl needs at least two tokens\n");
        return 1;
    }
    double nll = 0;
    const auto t0 = Clock::now();
    if (!ok_or_report(qnt_model_nll(md.m, ids.data(), int(ids.size()), &nll), "ppl")) return 1;
    const double n = double(ids.size() - 1);
    std::printf("ppl %.4f over %d tokens (%.1f tok/s)\n", std::exp(nll / n), int(n), n / seconds_since(t0));
    return 0;
}

// Cost of one batched pass of n = 1..32 tokens at context pos0 against one decode step (engine/src/checks.cpp:241-263).
void batch_curve(Model& md, const std::vector<int>& ids, int pos0) {
    std::vector<int> toks;
    while (int(toks.size()) < pos0 + 32) toks.insert(toks.end(), ids.begin(), ids.end());
    qnt_model_forward_batch(md.m, toks.data(), pos0, 0, nullptr, nullptr);
    auto time_ms = [&](const std::function<void()>& pass) {
        pass();
        double best = 1e30;
        for (int rep = 0; rep < 5; ++rep) {
            const auto t = Clock::now();
            pass();
            best = std::min(best, seconds_since(t) * 1e3);
        }
        return best;
    };
    const double one = time_ms([&] { qnt_model_forward(md.m, toks[size_t(pos0)], pos0, nullptr, nullptr); });
    std::printf("context %d, 1 GPU; decode step (forward) %.2f ms\n", pos0, one);
    std::printf("   n    ms/pass   cost vs decode   tok/s\n");
    for (int n : {1, 2, 4, 8, 16, 32}) {
        const double ms = time_ms([&] { qnt_model_forward_batch(md.m, toks.data() + pos0, n, pos0, nullptr, nullptr); });
        std::printf("  %2d  %9.2f   %10.2fx   %8.1f\n", n, ms, ms / one, n * 1e3 / ms);
    }
}

// Session::feed + n_gen steps queued at once, for the speed sections: (ids, prefill s, decode s, head fraction).
struct Timed {
    std::vector<int> ids;
    double prefill_s = 0, decode_s = 0, head_fraction = 1;
};
Timed timed_generate(Model& md, const std::vector<int>& prompt, const qnt_sampler_params& sp, bool shortlist, bool batch,
                     int n_gen) {
    Timed t;
    const int flags = (shortlist ? QNT_GEN_SHORTLIST : 0) | (batch ? QNT_GEN_BATCH_PREFILL : 0);
    auto t0 = Clock::now();
    if (!ok_or_report(qnt_session_begin(md.m, prompt.data(), int(prompt.size()), &sp, flags), "feed")) return t;
    qnt_session_last(md.m, nullptr, nullptr);
    t.prefill_s = seconds_since(t0);
    t0 = Clock::now();
    qnt_session_step(md.m, n_gen);
    t.ids.resize(size_t(n_gen));
    qnt_gen_stats st{};
    const int n = qnt_session_read(md.m, t.ids.data(), n_gen, &st);
    t.decode_s = seconds_since(t0);
    t.ids.resize(size_t(std::max(n, 0)));
    t.head_fraction = st.head_calls ? double(st.head_rows) / (double(st.head_calls) * md.hp.vocab_size) : 1.0;
    return t;
}

int compare(Model& md, Text& tok, const Args& a) {  // engine/src/checks.cpp:269-305: RESULT lines
    std::vector<int> ids = tok.encode(compare_prompt());
    if (int(ids.size()) > md.hp.ctx_len - 65) ids.resize(size_t(std::max(md.hp.ctx_len - 65, 32)));  // small contexts
    qnt_sampler_params greedy = a.sp;
    greedy.temperature = 0.f;
    greedy.repeat_penalty = 1.f;
    const int gen_n = 64, reps = 2;
    for (int sl = 0; sl < (md.hp.has_shortlist ? 2 : 1); ++sl) {
        double pre = 0, dec = 0;
        for (int rep = -1; rep < reps; ++rep) {  // -1: untimed warm-up
            const std::vector<int> feed = rep < 0 ? std::vector<int>(ids.begin(), ids.begin() + std::min<size_t>(32, ids.size())) : ids;
            const Timed t = timed_generate(md, feed, greedy, sl != 0, true, rep < 0 ? 8 : gen_n);
            if (rep < 0) continue;
            pre += feed.size() / t.prefill_s / reps;
            dec += t.ids.size() / t.decode_s / reps;
        }
        std::printf("RESULT engine=quanta_b200 model=%s%s threads=0 prefill_tok=%zu prefill_tps=%.2f decode_tok=%d "
                    "decode_tps=%.2f\n",
                    a.model.c_str(), sl ? "+shortlist" : "", ids.size(), pre, gen_n, dec);
    }
    return 0;
}

int bench_report(Model& md, Text& tok, const Args& a) {  // engine/src/checks.cpp:307-423
    const auto t_start = Clock::now();
    bool ok = true;
    std::printf("== quanta_b200 benchmark\n");
    std::printf("gpus: %d\n", qnt_device_count());
    std::printf("== kernels\n");
    ok &= selftest() == 0;
    std::printf("== load\n");
    std::printf("loaded %s, shortlist head: %s\n", a.model.c_str(), md.hp.has_shortlist ? "yes" : "no");
    const std::vector<int> ids = tok.encode(sample_text());
    std::vector<int> long_ids;
    while (long_ids.size() < 500) long_ids.insert(long_ids.end(), ids.begin(), ids.end());
    long_ids.resize(500);
    const std::vector<int> pids = tok.encode(
        "<|im_start|>system\nYou are a helpful assistant.<|im_end|>\n<|im_start|>user\n"
        "Write a short story about a river ferry.<|im_end|>\n<|im_start|>assistant\n");

    std::printf("== prefill speed\n");
    {
        qnt_sampler_params greedy = a.sp;
        greedy.temperature = 0.f;
        const Timed b = timed_generate(md, long_ids, greedy, false, true, 0);
        std::printf("prefill batched        %3zu tok: %6.1f tok/s\n", long_ids.size(), long_ids.size() / b.prefill_s);
        const std::vector<int> short_ids(long_ids.begin(), long_ids.begin() + 64);
        const Timed t = timed_generate(md, short_ids, greedy, false, false, 0);
        std::printf("prefill token-by-token  %2zu tok: %6.1f tok/s\n", short_ids.size(), short_ids.size() / t.prefill_s);
    }
    std::printf("== decode speed (device)\n");
    {
        // Qwen chat defaults with a fixed seed: the full head and the shortlist head must give the same ids; runs are
        // ordered A-B-B-A
        qnt_sampler_params sp{0.7f, 20, 0.8f, 0.0f, 1.1f, 0, 1234};
        const bool has_sl = md.hp.has_shortlist;
        const std::vector<int> order = has_sl ? std::vector<int>{0, 1, 1, 0} : std::vector<int>{0};
        double tok_s[2] = {0, 0}, head[2] = {1, 1};
        int runs[2] = {0, 0};
        std::vector<int> outs[2];
        for (int sl : order) {
            const Timed t = timed_generate(md, pids, sp, sl != 0, true, 64);
            tok_s[sl] += t.ids.size() / t.decode_s;
            head[sl] = t.head_fraction;
            ++runs[sl];
            if (outs[sl].empty()) outs[sl] = t.ids;
            else ok &= outs[sl] == t.ids;
        }
        std::printf("decode full head:      %6.2f tok/s\n", tok_s[0] / runs[0]);
        if (has_sl) {
            std::printf("decode shortlist head: %6.2f tok/s  (8-bit head read %.1f%%)  -> %.2fx\n", tok_s[1] / runs[1],
                        100 * head[1], (tok_s[1] / runs[1]) / (tok_s[0] / runs[0]));
            const bool same = outs[0] == outs[1];
            ok &= same;
            std::printf("decode output identical (full vs shortlist): %s\n", same ? "PASS" : "FAIL");
        }
        std::string sample;
        for (int id : outs[0]) sample += tok.piece(id);
        std::printf("sample output: %.300s\n", sample.c_str());
    }
    std::printf("== batch cost curve\n");
    batch_curve(md, ids, 256);
    std::printf("== exactness: batched prefill\n");
    ok &= check_batch(md, std::vector<int>(ids.begin(), ids.begin() + std::min<size_t>(ids.size(), 100)), true) == 0;
    if (md.hp.has_shortlist) {
        std::printf("== exactness: shortlist head\n");
        ok &= check_head(md, std::vector<int>(ids.begin(), ids.begin() + std::min<size_t>(ids.size(), 24))) == 0;
    }
    std::printf("== done in %.1f s: %s\n", seconds_since(t_start), ok ? "ALL PASS" : "SOME CHECKS FAILED");
    return ok ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc >= 2 && std::strcmp(argv[1], "selftest") == 0) return selftest();
    if (argc >= 2 && std::strcmp(argv[1], "export-layout") == 0) {
        if (argc != 4) usage();
        if (qnt_export_device_layout(argv[2], argv[3]) != QNT_OK) {
            std::fprintf(stderr, "export-layout: %s\n", qnt_last_error());
            return 1;
        }
        std::printf("wrote %s\n", argv[3]);
        return 0;
    }
    if (argc >= 2 && std::strcmp(argv[1], "prompt") == 0) {
        std::fputs(compare_prompt().c_str(), stdout);
        return 0;
    }
    Args a = parse(argc, argv);
    Text tok;
    if (!tok.open(a.model)) return 1;
    const std::string text = a.file.empty() ? a.prompt : read_file(a.file);
    // token ids: --ids, else the text through the tokenizer
    const std::vector<int> ids = !a.ids.empty() ? parse_ids(a.ids) : tok.encode(text);
    if (a.cmd == "tokenize") {
        for (size_t i = 0; i < ids.size(); ++i) std::printf(i ? ",%d" : "%d", ids[i]);
        std::printf("\n");
        return 0;
    }
    Model md;
    if (!open_model(a, md)) return 1;
    if (a.cmd == "run") return run_text(md, tok, a, text);
    if (a.cmd == "chat") return chat_loop(md, tok, a);
    if (a.cmd == "compare") return compare(md, tok, a);
    if (a.cmd == "bench") return bench_report(md, tok, a);
    if (a.cmd == "batchcurve") {
        batch_curve(md, tok.encode(sample_text()), 256);
        return 0;
    }
    if (ids.empty()) {
        std::fprintf(stderr, "no input\n");
        return 1;
    }
    if (a.cmd == "gen") return gen(md, a, ids, true);
    if (a.cmd == "ppl") return perplexity(md, a, ids);
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
    if (a.cmd == "checkbatch") return check_batch(md, ids, false);
    if (a.cmd == "checkhead") return check_head(md, ids);
    usage();
}
