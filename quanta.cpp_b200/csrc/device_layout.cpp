// The device's fused row order on the host, and the pre-packed .qnt writer (device_layout.h).
#include "device_layout.h"

#include <sys/stat.h>

#include <cstdio>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <utility>

namespace qb {

namespace {

constexpr int kBlock = 32;
constexpr uint64_t kDataAlign = 64;  // the format's tensor data alignment

size_t row_quant_bytes(const HostTensor& t) { return t.rows ? t.quant_bytes() / size_t(t.rows) : 0; }

// (source tensor, source row) for every fused row
std::vector<std::pair<const HostTensor*, int>> fused_order(const std::vector<const HostTensor*>& parts, int mode, int head_dim) {
    std::vector<std::pair<const HostTensor*, int>> order;
    if (mode == 0) {
        const int half = head_dim / 2;
        for (const HostTensor* p : parts)
            for (int u = 0; u < p->rows / head_dim; ++u)
                for (int i = 0; i < half; ++i) {
                    order.emplace_back(p, u * head_dim + i);
                    order.emplace_back(p, u * head_dim + i + half);
                }
    } else {
        const HostTensor *g = parts[0], *up = parts[1];
        for (int j = 0; j < g->rows / kBlock; ++j) {
            for (int i = 0; i < kBlock; ++i) order.emplace_back(g, j * kBlock + i);
            for (int i = 0; i < kBlock; ++i) order.emplace_back(up, j * kBlock + i);
        }
    }
    return order;
}

}  // namespace

FusedHost fuse_rows(const std::vector<const HostTensor*>& parts, int mode, int head_dim) {
    FusedHost f;
    f.dtype = parts[0]->dtype;
    f.cols = parts[0]->cols;
    for (const HostTensor* p : parts) {
        if (p->dtype != f.dtype || p->cols != f.cols) throw std::runtime_error("fused matrices need one dtype and width");
        if (p->dtype != 2 && p->dtype != 3) throw std::runtime_error("weight matrices must be q8_0 or q4_0");
        f.rows += p->rows;
    }
    if (mode == 1 && (parts.size() != 2 || parts[0]->rows != parts[1]->rows || parts[0]->rows % kBlock != 0))
        throw std::runtime_error("gate and up need equal row counts in whole 32-row blocks");
    if (mode == 0)
        for (const HostTensor* p : parts)
            if (head_dim <= 0 || p->rows % head_dim != 0) throw std::runtime_error("q/k/v rows are not whole heads");
    const size_t rb = row_quant_bytes(*parts[0]), nb = size_t(f.cols / kBlock);
    f.q.resize(size_t(f.rows) * rb);
    f.d.resize(size_t(f.rows) * nb);
    const auto order = fused_order(parts, mode, head_dim);
    for (size_t r = 0; r < order.size(); ++r) {
        const HostTensor* src = order[r].first;
        const size_t sr = size_t(order[r].second);
        std::memcpy(f.q.data() + r * rb, src->data + sr * rb, rb);
        std::memcpy(f.d.data() + r * nb, src->scales() + sr * nb, nb * 2);
    }
    return f;
}

bool packed_rows_match(const HostTensor& packed, const std::vector<const HostTensor*>& parts, int mode, int head_dim) {
    int rows = 0;
    for (const HostTensor* p : parts) {
        if (p->dtype != packed.dtype || p->cols != packed.cols) return false;
        rows += p->rows;
    }
    if (packed.rows != rows || rows == 0 || (packed.dtype != 2 && packed.dtype != 3)) return false;
    if (mode == 0 && head_dim <= 0) return false;
    if (mode == 1 && (parts.size() != 2 || parts[0]->rows != parts[1]->rows || parts[0]->rows % kBlock != 0)) return false;
    const auto order = fused_order(parts, mode, head_dim);
    if (int(order.size()) != rows) return false;
    const size_t rb = row_quant_bytes(packed), nb = size_t(packed.cols / kBlock);
    constexpr int kSamples = 64;
    for (int k = 0; k <= kSamples; ++k) {
        const size_t r = size_t((long long)k * (rows - 1) / kSamples);
        const HostTensor* src = order[r].first;
        const size_t sr = size_t(order[r].second);
        if (std::memcmp(packed.data + r * rb, src->data + sr * rb, rb) != 0 ||
            std::memcmp(packed.scales() + r * nb, src->scales() + sr * nb, nb * 2) != 0)
            return false;
    }
    return true;
}

std::vector<float> fuse_qkv_bias(const std::vector<const HostTensor*>& biases, int head_dim) {
    std::vector<float> b;
    const int half = head_dim / 2;
    for (const HostTensor* t : biases) {
        if (t->dtype != 0) throw std::runtime_error("qkv biases must be f32");
        const float* v = reinterpret_cast<const float*>(t->data);
        for (int u = 0; u < t->cols / head_dim; ++u)
            for (int i = 0; i < half; ++i) {
                b.push_back(v[u * head_dim + i]);
                b.push_back(v[u * head_dim + i + half]);
            }
    }
    return b;
}

namespace {

struct OutTensor {
    std::string name;
    int dtype = 0, rank = 2, rows = 0, cols = 0;
    std::vector<std::pair<const uint8_t*, size_t>> pieces;  // the tensor's bytes, in order
    size_t bytes() const {
        size_t n = 0;
        for (const auto& p : pieces) n += p.second;
        return n;
    }
};

void put_u32(std::vector<uint8_t>* b, uint32_t v) {
    for (int i = 0; i < 4; ++i) b->push_back(uint8_t(v >> (8 * i)));
}
void put_u64(std::vector<uint8_t>* b, uint64_t v) {
    for (int i = 0; i < 8; ++i) b->push_back(uint8_t(v >> (8 * i)));
}

}  // namespace

bool export_device_layout(const std::string& in_path, const std::string& out_path, std::string* err) {
    auto bad = [&](const std::string& m) {
        if (err) *err = m;
        return false;
    };
    QntFile in;
    std::string e;
    if (!in.open(in_path, &e)) return bad(e);
    // the input stays mapped while the output is written: the output must not be the same file under another name
    struct stat si, so;
    if (in_path == out_path ||
        (::stat(in_path.c_str(), &si) == 0 && ::stat(out_path.c_str(), &so) == 0 && si.st_dev == so.st_dev && si.st_ino == so.st_ino))
        return bad("export_device_layout: the output must be another file");
    const HParams& hp = in.hparams();
    std::vector<OutTensor> outs;
    for (const std::string& name : in.tensor_names()) {
        if (name.rfind("b200.", 0) == 0) continue;  // an earlier export's pre-packed tensors are rebuilt
        const HostTensor* t = in.find(name);
        OutTensor o;
        o.name = name;
        o.dtype = t->dtype;
        o.rank = t->rank;
        o.rows = t->rows;
        o.cols = t->cols;
        o.pieces.emplace_back(t->data, t->total_bytes());
        outs.push_back(std::move(o));
    }
    static const float kVersion = float(kDeviceLayoutVersion);
    {
        OutTensor o;
        o.name = "b200.layout";
        o.dtype = 0;
        o.rank = 1;
        o.rows = 1;
        o.cols = 1;
        o.pieces.emplace_back(reinterpret_cast<const uint8_t*>(&kVersion), 4);
        outs.push_back(std::move(o));
    }
    std::vector<std::unique_ptr<FusedHost>> keep;
    std::vector<std::unique_ptr<std::vector<float>>> keep_b;
    try {
        for (int l = 0; l < hp.n_layers; ++l) {
            const std::string p = "model.layers." + std::to_string(l) + ".", q = "b200.layers." + std::to_string(l) + ".";
            const struct {
                const char* name;
                std::vector<const HostTensor*> parts;
                int mode;
            } groups[2] = {{"qkv",
                            {&in.require(p + "self_attn.q_proj.weight"), &in.require(p + "self_attn.k_proj.weight"),
                             &in.require(p + "self_attn.v_proj.weight")},
                            0},
                           {"gate_up", {&in.require(p + "mlp.gate_proj.weight"), &in.require(p + "mlp.up_proj.weight")}, 1}};
            for (const auto& g : groups) {
                keep.push_back(std::make_unique<FusedHost>(fuse_rows(g.parts, g.mode, hp.head_dim)));
                const FusedHost& f = *keep.back();
                OutTensor o;
                o.name = q + g.name;
                o.dtype = f.dtype;
                o.rows = f.rows;
                o.cols = f.cols;
                o.pieces.emplace_back(f.q.data(), f.q.size());
                o.pieces.emplace_back(reinterpret_cast<const uint8_t*>(f.d.data()), f.d.size() * 2);
                outs.push_back(std::move(o));
            }
            if (hp.qkv_bias) {
                keep_b.push_back(std::make_unique<std::vector<float>>(
                    fuse_qkv_bias({&in.require(p + "self_attn.q_proj.bias"), &in.require(p + "self_attn.k_proj.bias"),
                                   &in.require(p + "self_attn.v_proj.bias")},
                                  hp.head_dim)));
                const std::vector<float>& b = *keep_b.back();
                OutTensor o;
                o.name = q + "qkv_bias";
                o.dtype = 0;
                o.rank = 1;
                o.rows = 1;
                o.cols = int(b.size());
                o.pieces.emplace_back(reinterpret_cast<const uint8_t*>(b.data()), b.size() * 4);
                outs.push_back(std::move(o));
            }
        }
    } catch (const std::exception& x) {
        return bad(std::string("export_device_layout: ") + x.what());
    }
    // the directory, then the data at 64-byte aligned offsets after it
    std::vector<uint8_t> dir;
    auto entry_bytes = [&](const OutTensor& o) { return 4 + o.name.size() + 4 + 4 + 4 * size_t(o.rank) + 8; };
    size_t dir_bytes = 4;
    for (const OutTensor& o : outs) dir_bytes += entry_bytes(o);
    uint64_t pos = uint64_t(in.directory_offset() + dir_bytes);
    std::vector<uint64_t> offs;
    for (const OutTensor& o : outs) {
        pos = (pos + kDataAlign - 1) / kDataAlign * kDataAlign;
        offs.push_back(pos);
        pos += o.bytes();
    }
    put_u32(&dir, uint32_t(outs.size()));
    for (size_t i = 0; i < outs.size(); ++i) {
        const OutTensor& o = outs[i];
        put_u32(&dir, uint32_t(o.name.size()));
        dir.insert(dir.end(), o.name.begin(), o.name.end());
        put_u32(&dir, uint32_t(o.dtype));
        put_u32(&dir, uint32_t(o.rank));
        if (o.rank == 2) put_u32(&dir, uint32_t(o.rows));
        put_u32(&dir, uint32_t(o.cols));
        put_u64(&dir, offs[i]);
    }
    std::unique_ptr<FILE, int (*)(FILE*)> f(std::fopen(out_path.c_str(), "wb"), &std::fclose);
    if (!f) return bad("export_device_layout: cannot write '" + out_path + "'");
    bool ok = std::fwrite(in.bytes(), 1, in.directory_offset(), f.get()) == in.directory_offset() &&
              std::fwrite(dir.data(), 1, dir.size(), f.get()) == dir.size();
    uint64_t at = uint64_t(in.directory_offset() + dir.size());
    static const uint8_t zeros[kDataAlign] = {};
    for (size_t i = 0; ok && i < outs.size(); ++i) {
        ok = std::fwrite(zeros, 1, size_t(offs[i] - at), f.get()) == size_t(offs[i] - at);
        at = offs[i];
        for (const auto& piece : outs[i].pieces) {
            ok = ok && std::fwrite(piece.first, 1, piece.second, f.get()) == piece.second;
            at += piece.second;
        }
    }
    ok = ok && std::fflush(f.get()) == 0;
    ok = std::fclose(f.release()) == 0 && ok;
    if (!ok) {
        std::remove(out_path.c_str());  // no partial file is left behind
        return bad("export_device_layout: writing '" + out_path + "' failed");
    }
    return true;
}

}  // namespace qb
