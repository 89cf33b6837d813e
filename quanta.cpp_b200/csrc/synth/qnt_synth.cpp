// Seeded random-init .qnt writer: the synthetic stand-in for scripts/export.py when there is no checkpoint.
//
// File layout follows the .qnt v2 spec (scripts/export.py:1-13, writer at :290-315; reader
// engine/src/model_file.cpp:149-211): magic "QNT1", version, hparams, length-prefixed tokenizer section,
// tensor table (name, dtype, ndim, dims, u64 offset), then 64-byte aligned tensor data.  Quantized tensors
// store quants first and fp16 block scales after them (engine/src/model_file.h:26).
//
// Quantizers restate the exporter's:
//   Q8_0  export.py:84-90   d = amax/127 (f32), inv = 1/d, q = clip(round_half_even(x*inv), +-127), fp16(d)
//   GPTQ-sym Q4_0 codes     export.py:104-108 packing, byte j = q[j] | q[j+16] << 4, value (q-8)*d; codes are
//                           drawn uniform in [-8, 7] with one scale per 128 columns replicated over four
//                           32-blocks (the g128 groups that the 32-block format expresses)
//   shortlist head          export.py:119-148: a 4-bit copy of the dequantized Q8 head picked by a 13x2 scale
//                           search, plus per-block ||w8 - w4||_2 rounded UP to fp16 (the bound the engine uses)
// Weights are N(0, w_std) from a counter-based generator keyed by (seed, tensor name, row), so a file is the
// same bytes whatever the thread count.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "qnt_synth.h"

namespace {

constexpr int QK = 32;
enum : uint32_t { DT_F32 = 0, DT_F16 = 1, DT_Q8_0 = 2, DT_Q4_0 = 3 };

uint64_t splitmix64(uint64_t& s) {
    uint64_t z = (s += 0x9E3779B97F4A7C15ULL);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

uint64_t hash_name(const std::string& s) {
    uint64_t h = 1469598103934665603ULL;  // FNV-1a
    for (unsigned char c : s) h = (h ^ c) * 1099511628211ULL;
    return h;
}

struct RowRng {
    uint64_t s;
    RowRng(uint64_t seed, uint64_t name, uint64_t row) : s(seed ^ (name * 0x9E3779B97F4A7C15ULL) ^ (row * 0xD1B54A32D192ED03ULL)) {
        splitmix64(s);
    }
    uint64_t u64() { return splitmix64(s); }
    double uniform() { return double(u64() >> 11) * (1.0 / 9007199254740992.0); }  // [0, 1)
    // Box-Muller pairs; cached second value.
    bool have = false;
    double spare = 0;
    double normal() {
        if (have) {
            have = false;
            return spare;
        }
        double u1 = uniform(), u2 = uniform();
        if (u1 < 1e-300) u1 = 1e-300;
        const double r = std::sqrt(-2.0 * std::log(u1)), a = 6.283185307179586 * u2;
        spare = r * std::sin(a);
        have = true;
        return r * std::cos(a);
    }
};

uint16_t f32_to_f16_bits(float f) {
    _Float16 h = static_cast<_Float16>(f);  // round to nearest even
    uint16_t b;
    std::memcpy(&b, &h, 2);
    return b;
}
float f16_bits_to_f32(uint16_t b) {
    _Float16 h;
    std::memcpy(&h, &b, 2);
    return static_cast<float>(h);
}

template <class F>
void parallel_rows(int rows, int n_threads, F&& fn) {
    n_threads = std::max(1, std::min(n_threads, rows));
    std::vector<std::thread> ts;
    for (int t = 0; t < n_threads; ++t)
        ts.emplace_back([&, t] {
            const int r0 = int(int64_t(rows) * t / n_threads), r1 = int(int64_t(rows) * (t + 1) / n_threads);
            for (int r = r0; r < r1; ++r) fn(r);
        });
    for (auto& th : ts) th.join();
}

struct Encoded {
    std::string name;
    uint32_t dtype;
    std::vector<uint32_t> shape;
    std::vector<uint8_t> data;
};

// One row of N(0, std) floats.
void normal_row(float* out, int cols, uint64_t seed, uint64_t name, int row, float stdv) {
    RowRng g(seed, name, uint64_t(row));
    for (int i = 0; i < cols; ++i) out[i] = float(g.normal() * stdv);
}

// Q8_0 quantization of one row into q (cols int8) and d (cols/32 fp16 bits).  export.py:84-90.
void quantize_row_q8(const float* x, int cols, int8_t* q, uint16_t* d) {
    for (int b = 0; b < cols / QK; ++b) {
        const float* xb = x + b * QK;
        float amax = 0.f;
        for (int i = 0; i < QK; ++i) amax = std::max(amax, std::fabs(xb[i]));
        const float dd = amax / 127.0f;
        const float inv = dd > 0 ? 1.0f / dd : 0.0f;
        for (int i = 0; i < QK; ++i) {
            float v = std::nearbyint(xb[i] * inv);  // default rounding mode: half to even, like np.round
            v = std::min(127.f, std::max(-127.f, v));
            q[b * QK + i] = int8_t(v);
        }
        d[b] = f32_to_f16_bits(dd);
    }
}

Encoded make_f32(const std::string& name, int n, float value_or_nan, uint64_t seed, float stdv) {
    Encoded e{name, DT_F32, {uint32_t(n)}, std::vector<uint8_t>(size_t(n) * 4)};
    std::vector<float> v(static_cast<size_t>(n));
    if (std::isnan(value_or_nan)) normal_row(v.data(), n, seed, hash_name(name), 0, stdv);
    else std::fill(v.begin(), v.end(), value_or_nan);
    std::memcpy(e.data.data(), v.data(), e.data.size());
    return e;
}

Encoded make_q8(const std::string& name, int rows, int cols, uint64_t seed, float stdv, int n_threads) {
    const size_t n = size_t(rows) * cols;
    Encoded e{name, DT_Q8_0, {uint32_t(rows), uint32_t(cols)}, std::vector<uint8_t>(n + n / QK * 2)};
    int8_t* q = reinterpret_cast<int8_t*>(e.data.data());
    uint16_t* d = reinterpret_cast<uint16_t*>(e.data.data() + n);
    const uint64_t h = hash_name(name);
    parallel_rows(rows, n_threads, [&](int r) {
        std::vector<float> x(static_cast<size_t>(cols));
        normal_row(x.data(), cols, seed, h, r, stdv);
        quantize_row_q8(x.data(), cols, q + size_t(r) * cols, d + size_t(r) * (cols / QK));
    });
    return e;
}

// GPTQ-symmetric int4 codes: code uniform in [-8, 7] (stored q = code + 8), one fp16 scale per `group` columns
// replicated over its 32-blocks.  Scale = w_std / sqrt(255/12) * U(0.75, 1.25), so dequantized weights have
// std ~ w_std.
Encoded make_q4_gptq(const std::string& name, int rows, int cols, int group, uint64_t seed, float stdv, int n_threads) {
    const size_t n = size_t(rows) * cols;
    Encoded e{name, DT_Q4_0, {uint32_t(rows), uint32_t(cols)}, std::vector<uint8_t>(n / 2 + n / QK * 2)};
    uint8_t* p = e.data.data();
    uint16_t* d = reinterpret_cast<uint16_t*>(e.data.data() + n / 2);
    const uint64_t h = hash_name(name);
    const double base = stdv / std::sqrt(255.0 / 12.0);
    parallel_rows(rows, n_threads, [&](int r) {
        RowRng g(seed, h, uint64_t(r));
        std::vector<uint8_t> qi(static_cast<size_t>(cols));
        for (int i = 0; i < cols; ++i) qi[i] = uint8_t(g.u64() % 16);  // code + 8 in [0, 15]
        for (int b = 0; b < cols / QK; ++b) {
            uint8_t* dst = p + (size_t(r) * cols + size_t(b) * QK) / 2;
            for (int j = 0; j < QK / 2; ++j) dst[j] = uint8_t((qi[b * QK + j] & 0xF) | (qi[b * QK + j + 16] << 4));
        }
        const int nb = cols / QK, per = std::max(1, group / QK);
        for (int b = 0; b < nb; b += per) {
            const uint16_t s = f32_to_f16_bits(float(base * (0.75 + 0.5 * g.uniform())));
            for (int k = b; k < std::min(nb, b + per); ++k) d[size_t(r) * nb + k] = s;
        }
    });
    return e;
}

// Exact Shortlist Head tensors from the Q8 head (export.py:111-148): w8 = q8 * fp16(d) (float32); per 32-block
// a 4-bit copy chosen by a scale search over f in linspace(0.8, 1.1, 13) x sign(+-8) minimizing the squared
// error, and err = ||(q4-8)*d4 - w8||_2 (float64) rounded up to fp16.
void make_shortlist(const Encoded& head, Encoded& q4, Encoded& err, int n_threads) {
    const int rows = int(head.shape[0]), cols = int(head.shape[1]), nb = cols / QK;
    const size_t n = size_t(rows) * cols;
    const int8_t* hq = reinterpret_cast<const int8_t*>(head.data.data());
    const uint16_t* hd = reinterpret_cast<const uint16_t*>(head.data.data() + n);
    q4 = Encoded{"quanta.head_q4", DT_Q4_0, {uint32_t(rows), uint32_t(cols)}, std::vector<uint8_t>(n / 2 + n / QK * 2)};
    err = Encoded{"quanta.head_err", DT_F16, {uint32_t(rows), uint32_t(nb)}, std::vector<uint8_t>(size_t(rows) * nb * 2)};
    uint8_t* pq = q4.data.data();
    uint16_t* pd = reinterpret_cast<uint16_t*>(q4.data.data() + n / 2);
    uint16_t* pe = reinterpret_cast<uint16_t*>(err.data.data());
    parallel_rows(rows, n_threads, [&](int r) {
        float w[QK];
        for (int b = 0; b < nb; ++b) {
            const size_t blk = size_t(r) * nb + b;
            const float s8 = f16_bits_to_f32(hd[blk]);
            int arg = 0;
            for (int i = 0; i < QK; ++i) {
                w[i] = float(hq[blk * QK + i]) * s8;
                if (std::fabs(w[i]) > std::fabs(w[arg])) arg = i;
            }
            const float mx = w[arg];
            double best_e = INFINITY;
            float best_d = 0.f;
            uint8_t best_q[QK] = {0};
            for (int fi = 0; fi < 13; ++fi) {
                const double f = 0.8 + 0.3 * fi / 12.0;
                for (double sgn : {-8.0, 8.0}) {
                    const float dd = f16_bits_to_f32(f32_to_f16_bits(float(double(mx) / sgn * f)));
                    const float inv = dd != 0.f ? 1.0f / dd : 0.0f;
                    uint8_t qq[QK];
                    double e = 0;
                    for (int i = 0; i < QK; ++i) {
                        float v = std::nearbyint(w[i] * inv + 8.0f);
                        v = std::min(15.f, std::max(0.f, v));
                        qq[i] = uint8_t(v);
                        const double diff = (double(v) - 8.0) * dd - w[i];
                        e += diff * diff;
                    }
                    if (e < best_e) {
                        best_e = e;
                        best_d = dd;
                        std::memcpy(best_q, qq, QK);
                    }
                }
            }
            double ss = 0;
            for (int i = 0; i < QK; ++i) {
                const double diff = (double(best_q[i]) - 8.0) * double(best_d) - double(w[i]);
                ss += diff * diff;
            }
            const double e = std::sqrt(ss);
            uint16_t eb = f32_to_f16_bits(float(e));
            if (double(f16_bits_to_f32(eb)) < e) eb = uint16_t(eb + 1);  // positive finite: next fp16 up
            pe[blk] = eb;
            uint8_t* dst = pq + blk * (QK / 2);
            for (int j = 0; j < QK / 2; ++j) dst[j] = uint8_t((best_q[j] & 0xF) | (best_q[j + 16] << 4));
            pd[blk] = f32_to_f16_bits(best_d);
        }
    });
}

void put_u32(std::vector<uint8_t>& o, uint32_t v) {
    uint8_t b[4];
    std::memcpy(b, &v, 4);
    o.insert(o.end(), b, b + 4);
}
void put_f32(std::vector<uint8_t>& o, float v) {
    uint32_t u;
    std::memcpy(&u, &v, 4);
    put_u32(o, u);
}
void put_blob(std::vector<uint8_t>& o, const std::string& s) {
    put_u32(o, uint32_t(s.size()));
    o.insert(o.end(), s.begin(), s.end());
}

// Synthetic byte-level vocabulary: ids 0..255 are the single bytes (the reference tokenizer requires all of them,
// engine/src/tokenizer.cpp:59-61), then unique placeholder strings, then the ChatML specials.
std::vector<uint8_t> tokenizer_section(int n_tokens) {
    std::vector<uint8_t> o;
    const char* specials[] = {"<|endoftext|>", "<|im_start|>", "<|im_end|>"};
    const int n_special = 3;
    const int first_special = std::max(256, n_tokens - n_special);
    put_u32(o, uint32_t(n_tokens));
    for (int i = 0; i < n_tokens; ++i) {
        if (i < 256) put_blob(o, std::string(1, char(i)));
        else if (i >= first_special) put_blob(o, specials[i - first_special]);
        else put_blob(o, "<t" + std::to_string(i) + ">");
    }
    put_u32(o, 0);  // no merges: text encodes to byte tokens
    put_u32(o, uint32_t(std::min(n_special, n_tokens - first_special)));
    for (int i = first_special; i < n_tokens; ++i) {
        put_u32(o, uint32_t(i));
        put_blob(o, specials[i - first_special]);
    }
    const uint32_t letters[][2] = {{0x41, 0x5A}, {0x61, 0x7A}, {0xC0, 0x24F}};
    const uint32_t numbers[][2] = {{0x30, 0x39}};
    const uint32_t spaces[][2] = {{0x09, 0x0D}, {0x20, 0x20}};
    put_u32(o, 3);
    for (auto& r : letters) put_u32(o, r[0]), put_u32(o, r[1]);
    put_u32(o, 1);
    for (auto& r : numbers) put_u32(o, r[0]), put_u32(o, r[1]);
    put_u32(o, 2);
    for (auto& r : spaces) put_u32(o, r[0]), put_u32(o, r[1]);
    return o;
}

thread_local std::string g_err;

}  // namespace

extern "C" {

const char* qnt_synth_last_error(void) { return g_err.c_str(); }

int qnt_synth_write(const char* path, const qnt_synth_cfg* c) {
    try {
        if (c->dim % QK || c->ffn_dim % QK || c->n_heads * c->head_dim != c->dim || c->n_kv_heads <= 0 ||
            c->n_heads % c->n_kv_heads) {
            g_err = "bad shape";
            return -1;
        }
        const int nt = c->n_threads > 0 ? c->n_threads : int(std::max(1u, std::thread::hardware_concurrency()));
        const uint64_t seed = c->seed;
        const float sd = c->w_std > 0 ? c->w_std : 0.02f;
        const int kv_dim = c->n_kv_heads * c->head_dim;
        std::vector<Encoded> ts;
        ts.push_back(make_q8("model.embed_tokens.weight", c->vocab_size, c->dim, seed, sd, nt));
        ts.push_back(make_f32("model.norm.weight", c->dim, 1.0f, seed, sd));
        for (int l = 0; l < c->n_layers; ++l) {
            const std::string p = "model.layers." + std::to_string(l) + ".";
            ts.push_back(make_f32(p + "input_layernorm.weight", c->dim, 1.0f, seed, sd));
            ts.push_back(make_f32(p + "post_attention_layernorm.weight", c->dim, 1.0f, seed, sd));
            ts.push_back(make_q8(p + "self_attn.q_proj.weight", c->dim, c->dim, seed, sd, nt));
            ts.push_back(make_q8(p + "self_attn.k_proj.weight", kv_dim, c->dim, seed, sd, nt));
            ts.push_back(make_q8(p + "self_attn.v_proj.weight", kv_dim, c->dim, seed, sd, nt));
            ts.push_back(make_q8(p + "self_attn.o_proj.weight", c->dim, c->dim, seed, sd, nt));
            ts.push_back(make_f32(p + "self_attn.q_proj.bias", c->dim, NAN, seed, sd));
            ts.push_back(make_f32(p + "self_attn.k_proj.bias", kv_dim, NAN, seed, sd));
            ts.push_back(make_f32(p + "self_attn.v_proj.bias", kv_dim, NAN, seed, sd));
            if (c->mlp_q4) {
                ts.push_back(make_q4_gptq(p + "mlp.gate_proj.weight", c->ffn_dim, c->dim, c->q4_group, seed, sd, nt));
                ts.push_back(make_q4_gptq(p + "mlp.up_proj.weight", c->ffn_dim, c->dim, c->q4_group, seed, sd, nt));
                ts.push_back(make_q4_gptq(p + "mlp.down_proj.weight", c->dim, c->ffn_dim, c->q4_group, seed, sd, nt));
            } else {
                ts.push_back(make_q8(p + "mlp.gate_proj.weight", c->ffn_dim, c->dim, seed, sd, nt));
                ts.push_back(make_q8(p + "mlp.up_proj.weight", c->ffn_dim, c->dim, seed, sd, nt));
                ts.push_back(make_q8(p + "mlp.down_proj.weight", c->dim, c->ffn_dim, seed, sd, nt));
            }
        }
        if (c->shortlist) {
            Encoded q4, err;
            make_shortlist(ts[0], q4, err, nt);
            ts.push_back(std::move(q4));
            ts.push_back(std::move(err));
        }
        std::sort(ts.begin(), ts.end(), [](const Encoded& a, const Encoded& b) { return a.name < b.name; });

        std::vector<uint8_t> head;
        head.insert(head.end(), {'Q', 'N', 'T', '1'});
        put_u32(head, 2);
        for (int v : {c->vocab_size, c->dim, c->n_layers, c->n_heads, c->n_kv_heads, c->head_dim, c->ffn_dim, c->max_seq})
            put_u32(head, uint32_t(v));
        put_f32(head, c->rope_theta);
        put_f32(head, c->norm_eps);
        put_u32(head, 1);  // tied embeddings
        put_u32(head, 1);  // qkv bias
        put_u32(head, c->flags);
        const std::vector<uint8_t> tok = c->tok_blob && c->tok_len
                                             ? std::vector<uint8_t>(c->tok_blob, c->tok_blob + c->tok_len)
                                             : tokenizer_section(c->n_tokens > 0 ? c->n_tokens : c->vocab_size);
        put_u32(head, uint32_t(tok.size()));
        head.insert(head.end(), tok.begin(), tok.end());

        auto table = [&](const std::vector<uint64_t>& off) {
            std::vector<uint8_t> t;
            put_u32(t, uint32_t(ts.size()));
            for (size_t i = 0; i < ts.size(); ++i) {
                put_blob(t, ts[i].name);
                put_u32(t, ts[i].dtype);
                put_u32(t, uint32_t(ts[i].shape.size()));
                for (uint32_t s : ts[i].shape) put_u32(t, s);
                uint64_t o = off.empty() ? 0 : off[i];
                uint8_t b[8];
                std::memcpy(b, &o, 8);
                t.insert(t.end(), b, b + 8);
            }
            return t;
        };
        uint64_t pos = head.size() + table({}).size();
        std::vector<uint64_t> off(ts.size());
        for (size_t i = 0; i < ts.size(); ++i) {
            pos = (pos + 63) / 64 * 64;
            off[i] = pos;
            pos += ts[i].data.size();
        }
        FILE* f = std::fopen(path, "wb");
        if (!f) {
            g_err = std::string("cannot write ") + path;
            return -1;
        }
        const std::vector<uint8_t> tb = table(off);
        std::fwrite(head.data(), 1, head.size(), f);
        std::fwrite(tb.data(), 1, tb.size(), f);
        uint64_t at = head.size() + tb.size();
        static const uint8_t zeros[64] = {0};
        for (size_t i = 0; i < ts.size(); ++i) {
            std::fwrite(zeros, 1, size_t(off[i] - at), f);
            std::fwrite(ts[i].data.data(), 1, ts[i].data.size(), f);
            at = off[i] + ts[i].data.size();
        }
        std::fclose(f);
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

}  // extern "C"
