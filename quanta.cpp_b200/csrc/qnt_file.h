// Host side of the .qnt model format: the file is mapped read-only, its header, tokenizer section and tensor
// directory are decoded and validated in one pass, and every tensor becomes a zero-copy view into the mapping that
// the engine uploads to HBM once.
//
// Format (writer: scripts/export.py:1-13,290-315 of Quanta.cpp; the reference reader is engine/src/model_file.cpp):
//   "QNT1" | u32 version (1 or 2) | hyper-parameters (u32/f32, `flags` from version 2 on)
//   | u32 length + tokenizer section (tokens, merges, specials, three code-point range lists)
//   | u32 tensor count + directory entries (name, dtype, rank, dims, u64 byte offset)
//   tensor data: quants row-major, then one fp16 scale per 32 values for the block-quantized dtypes.
// The checks are the format's own invariants: a known signature and version, every field inside the file, rank 1
// or 2, a known dtype, quantized rows made of whole 32-value blocks, every tensor's bytes inside the file.  Each
// failed check is reported as a QntFault with a message naming the field or tensor.
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace qb {

// Which invariant of the file failed (None: the file opened).
enum class QntFault {
    None = 0,
    Open,       // the path cannot be opened, sized or mapped
    Signature,  // the first four bytes are not "QNT1"
    Version,    // format version outside 1..2
    Header,     // the hyper-parameter block is cut short or holds a non-positive size
    Tokenizer,  // the tokenizer section is cut short or inconsistent
    Directory,  // a tensor directory entry is cut short, or a name repeats
    Rank,       // a tensor of rank other than 1 or 2
    DType,      // an unknown dtype code
    BlockCols,  // a block-quantized tensor whose rows are not whole 32-value blocks
    Extent,     // a tensor's bytes reach past the end of the file
    Missing,    // a tensor the engine needs is not in the file
};
const char* qnt_fault_name(QntFault f);

struct HostTensor {
    int dtype = 0;  // 0 f32, 1 f16, 2 q8_0, 3 q4_0 (engine/src/model_file.h:16)
    int rank = 2;   // as stored in the directory (rank 1: rows == 1)
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

// The tokenizer section, decoded (its meaning: engine/src/tokenizer.h:15-39).
struct TokenizerInfo {
    int n_tokens = 0;
    std::vector<std::string> tokens;                       // raw bytes per id
    std::vector<std::array<uint32_t, 3>> merges;           // (left id, right id, merged id), highest priority first
    std::vector<std::pair<int, std::string>> specials;     // (id, text)
    std::vector<std::pair<uint32_t, uint32_t>> letters, numbers, spaces;  // inclusive code-point ranges
};

// Thrown by QntFile::require for a tensor the file does not hold.
struct QntMissingTensor : std::runtime_error {
    explicit QntMissingTensor(const std::string& name);
};

class QntFile {
public:
    QntFile() = default;
    ~QntFile();
    QntFile(const QntFile&) = delete;
    QntFile& operator=(const QntFile&) = delete;

    // Maps and validates the file.  On failure returns false, fault() names the check and *err the details.
    bool open(const std::string& path, std::string* err);
    QntFault fault() const { return fault_; }

    const HParams& hparams() const { return hp_; }
    const TokenizerInfo& tokenizer() const { return tok_; }
    const HostTensor* find(const std::string& name) const;
    const HostTensor& require(const std::string& name) const;  // throws QntMissingTensor
    size_t size_bytes() const { return size_; }
    size_t tensor_count() const { return tensors_.size(); }
    int special_id(const std::string& text) const;         // -1 if absent
    // The raw file: its bytes, the offset of the tensor directory (everything before it is the header and the
    // tokenizer section), and the tensor names in directory order.
    const uint8_t* bytes() const { return map_; }
    size_t directory_offset() const { return dir_offset_; }
    const std::vector<std::string>& tensor_names() const { return order_; }

private:
    void release();
    HParams hp_;
    TokenizerInfo tok_;
    std::unordered_map<std::string, HostTensor> tensors_;
    const uint8_t* map_ = nullptr;
    size_t size_ = 0;
    size_t dir_offset_ = 0;
    std::vector<std::string> order_;
    QntFault fault_ = QntFault::None;
};

}  // namespace qb
