// Host reader for the .qnt model format: mmap + header / tokenizer / tensor-table parse, zero-copy tensor views.
// Mirrors the reference loader's checks (engine/src/model_file.cpp:149-211): magic "QNT1", version 1..2,
// truncation and out-of-bounds tensors are errors, ndim must be 1 or 2.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace qb {

struct HostTensor {
    int dtype = 0;  // 0 f32, 1 f16, 2 q8_0, 3 q4_0 (engine/src/model_file.h:16)
    int rows = 0, cols = 0;
    const uint8_t* data = nullptr;  // quants, then fp16 scales for quantized types
    size_t quant_bytes() const;
    size_t total_bytes() const;
    const uint16_t* scales() const { return reinterpret_cast<const uint16_t*>(data + quant_bytes()); }
};

struct HParams {
    int vocab_size = 0, dim = 0, n_layers = 0, n_heads = 0, n_kv_heads = 0, head_dim = 0, ffn_dim = 0, max_seq = 0;
    float rope_theta = 0, norm_eps = 0;
    bool tied_embeddings = false, qkv_bias = false;
    uint32_t flags = 0;
};

struct TokenizerInfo {
    int n_tokens = 0;
    std::vector<std::string> tokens;                         // raw bytes per id
    std::vector<std::pair<int, std::string>> specials;       // (id, text)
};

class QntFile {
public:
    QntFile() = default;
    ~QntFile();
    QntFile(const QntFile&) = delete;
    QntFile& operator=(const QntFile&) = delete;

    bool open(const std::string& path, std::string* err);
    const HParams& hparams() const { return hp_; }
    const TokenizerInfo& tokenizer() const { return tok_; }
    const HostTensor* find(const std::string& name) const;
    const HostTensor& get(const std::string& name) const;  // throws std::runtime_error if missing
    size_t size_bytes() const { return size_; }
    int special_id(const std::string& text) const;         // -1 if absent

private:
    void unmap();
    HParams hp_;
    TokenizerInfo tok_;
    std::unordered_map<std::string, HostTensor> tensors_;
    const uint8_t* base_ = nullptr;
    size_t size_ = 0;
};

}  // namespace qb
