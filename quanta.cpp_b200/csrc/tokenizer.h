// Byte-level BPE text <-> ids for the .qnt vocabulary, on the host (the interface of engine/src/tokenizer.h:15-39:
// encode with the special tokens written literally in the text, decode of one id to its raw bytes, special-token
// lookup).  Text is UTF-8 and expected to be NFC-normalised already, as the reference expects.
//
// encode = special-token split -> pre-tokenizer -> BPE per piece:
//   * specials: at every byte, the longest special literal that starts there is taken as its id;
//   * pre-tokenizer: the Qwen2 split pattern
//       (?i:'s|'t|'re|'ve|'m|'ll|'d) | [^\r\n\p{L}\p{N}]?\p{L}+ | \p{N} | ?[^\s\p{L}\p{N}]+[\r\n]* | \s*[\r\n]+ |
//       \s+(?!\S) | \s+
//     evaluated by a matcher per alternative over code points classified as letter / number / space / other (ASCII
//     directly, the rest from the file's code-point range lists; an invalid UTF-8 byte is one U+FFFD);
//   * BPE: a piece starts as its byte tokens and the pair of lowest merge rank is merged until none is left (the
//     leftmost one among equal ranks); here with a min-heap of (rank, position) over a linked list of symbols.
#pragma once

#include <cstdint>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "qnt_file.h"

namespace qb {

class BpeTokenizer {
public:
    // Throws std::runtime_error when the vocabulary lacks a single-byte token for some byte value (below the first
    // special id), which byte-level BPE needs to encode any input.
    explicit BpeTokenizer(const TokenizerInfo& info);

    std::vector<int> encode(const std::string& text) const;
    const std::string& piece(int id) const;  // raw bytes (may end inside a UTF-8 sequence); empty for a bad id
    int special_id(const std::string& literal) const;  // -1 if absent
    int n_tokens() const { return int(pieces_.size()); }

private:
    enum Cls : uint8_t { kOther = 0, kLetter = 1, kNumber = 2, kSpace = 3 };
    struct Sym {
        uint32_t cp;
        uint32_t at;  // byte offset in the text
        Cls cls;
    };
    Cls classify(uint32_t cp) const;
    void split(const std::string& text, size_t b, size_t e, std::vector<std::pair<size_t, size_t>>* pieces) const;
    void merge_piece(const std::string& text, size_t b, size_t e, std::vector<int>* out) const;

    std::vector<std::string> pieces_;
    std::unordered_map<uint64_t, std::pair<uint32_t, int>> rank_of_;  // (left << 32 | right) -> (rank, merged id)
    int byte_id_[256];
    std::unordered_map<std::string, int> special_;
    std::vector<std::vector<std::pair<std::string, int>>> special_by_byte_;  // first byte -> specials, longest first
    std::vector<std::pair<uint32_t, uint32_t>> letters_, numbers_, spaces_;
    std::string empty_;
};

}  // namespace qb
