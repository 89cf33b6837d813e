#include "tokenizer.h"

#include <algorithm>
#include <queue>
#include <stdexcept>
#include <tuple>

namespace qb {

namespace {

// One code point from UTF-8 at text[i]: the lead byte gives the length, every continuation byte must be 10xxxxxx and
// the bytes must be there; otherwise the single byte stands for U+FFFD.  Returns the byte length.
int next_code_point(const std::string& text, size_t i, uint32_t* cp) {
    const unsigned char lead = static_cast<unsigned char>(text[i]);
    int len;
    uint32_t v;
    if (lead < 0x80) {
        *cp = lead;
        return 1;
    } else if ((lead & 0xE0) == 0xC0) {
        len = 2, v = lead & 0x1F;
    } else if ((lead & 0xF0) == 0xE0) {
        len = 3, v = lead & 0x0F;
    } else if ((lead & 0xF8) == 0xF0) {
        len = 4, v = lead & 0x07;
    } else {
        *cp = 0xFFFD;
        return 1;
    }
    if (i + size_t(len) > text.size()) {
        *cp = 0xFFFD;
        return 1;
    }
    for (int k = 1; k < len; ++k) {
        const unsigned char c = static_cast<unsigned char>(text[i + k]);
        if ((c & 0xC0) != 0x80) {
            *cp = 0xFFFD;
            return 1;
        }
        v = (v << 6) | (c & 0x3F);
    }
    *cp = v;
    return len;
}

bool in_table(const std::vector<std::pair<uint32_t, uint32_t>>& t, uint32_t cp) {
    // ranges sorted by start: the last range starting at or below cp decides
    auto it = std::upper_bound(t.begin(), t.end(), cp,
                               [](uint32_t v, const std::pair<uint32_t, uint32_t>& r) { return v < r.first; });
    return it != t.begin() && cp <= (it - 1)->second;
}

uint64_t pair_key(int left, int right) { return (uint64_t(uint32_t(left)) << 32) | uint32_t(right); }

bool is_newline(uint32_t cp) { return cp == '\r' || cp == '\n'; }

uint32_t ascii_fold(uint32_t cp) { return cp < 0x80 ? (cp | 0x20u) : 0u; }

}  // namespace

BpeTokenizer::BpeTokenizer(const TokenizerInfo& info)
    : pieces_(info.tokens), letters_(info.letters), numbers_(info.numbers), spaces_(info.spaces) {
    for (auto* t : {&letters_, &numbers_, &spaces_}) std::sort(t->begin(), t->end());
    rank_of_.reserve(info.merges.size() * 2);
    for (size_t r = 0; r < info.merges.size(); ++r) {
        const auto& m = info.merges[r];
        rank_of_.emplace(pair_key(int(m[0]), int(m[1])), std::make_pair(uint32_t(r), int(m[2])));  // first rank kept
    }
    int first_special = int(pieces_.size());
    special_by_byte_.assign(256, {});
    for (const auto& sp : info.specials) {
        special_[sp.second] = sp.first;
        first_special = std::min(first_special, sp.first);
        if (!sp.second.empty())
            special_by_byte_[static_cast<unsigned char>(sp.second[0])].emplace_back(sp.second, sp.first);
    }
    for (auto& list : special_by_byte_)
        std::stable_sort(list.begin(), list.end(), [](const auto& a, const auto& b) { return a.first.size() > b.first.size(); });
    std::fill(std::begin(byte_id_), std::end(byte_id_), -1);
    for (int id = 0; id < first_special && id < int(pieces_.size()); ++id)
        if (pieces_[size_t(id)].size() == 1) byte_id_[static_cast<unsigned char>(pieces_[size_t(id)][0])] = id;
    for (int b = 0; b < 256; ++b)
        if (byte_id_[b] < 0)
            throw std::runtime_error("tokenizer: no single-byte token for byte " + std::to_string(b) +
                                     " below the special ids; byte-level BPE needs all 256");
}

BpeTokenizer::Cls BpeTokenizer::classify(uint32_t cp) const {
    if (cp < 0x80) {
        if ((cp >= 'a' && cp <= 'z') || (cp >= 'A' && cp <= 'Z')) return kLetter;
        if (cp >= '0' && cp <= '9') return kNumber;
        if (cp == ' ' || (cp >= 0x09 && cp <= 0x0D)) return kSpace;
        return kOther;
    }
    if (in_table(letters_, cp)) return kLetter;
    if (in_table(numbers_, cp)) return kNumber;
    if (in_table(spaces_, cp)) return kSpace;
    return kOther;
}

// The split pattern's alternatives, tried in order at each position; each returns the end of its match (in code
// points) or 0 when it does not match there.
void BpeTokenizer::split(const std::string& text, size_t b, size_t e, std::vector<std::pair<size_t, size_t>>* pieces) const {
    std::vector<Sym> s;
    s.reserve(e - b);
    for (size_t i = b; i < e;) {
        uint32_t cp;
        const int len = next_code_point(text, i, &cp);
        s.push_back(Sym{cp, uint32_t(i), classify(cp)});
        i += size_t(len);
    }
    const size_t n = s.size();
    auto cls = [&](size_t k) { return k < n ? s[k].cls : kOther; };
    auto has = [&](size_t k, Cls c) { return k < n && s[k].cls == c; };
    auto newline = [&](size_t k) { return k < n && is_newline(s[k].cp); };

    auto contraction = [&](size_t i) -> size_t {  // (?i:'s|'t|'re|'ve|'m|'ll|'d), ASCII case folding
        if (s[i].cp != '\'') return 0;
        const uint32_t a = i + 1 < n ? ascii_fold(s[i + 1].cp) : 0, c = i + 2 < n ? ascii_fold(s[i + 2].cp) : 0;
        if (a == 's' || a == 't' || a == 'm' || a == 'd') return i + 2;
        if ((a == 'r' && c == 'e') || (a == 'v' && c == 'e') || (a == 'l' && c == 'l')) return i + 3;
        return 0;
    };
    auto word = [&](size_t i) -> size_t {  // [^\r\n\p{L}\p{N}]?\p{L}+
        size_t k;
        if (has(i, kLetter)) k = i;
        else if (!newline(i) && cls(i) != kNumber && has(i + 1, kLetter)) k = i + 1;
        else return 0;
        while (has(k, kLetter)) ++k;
        return k;
    };
    auto number = [&](size_t i) -> size_t { return has(i, kNumber) ? i + 1 : 0; };  // \p{N}
    auto symbols = [&](size_t i) -> size_t {  //  ?[^\s\p{L}\p{N}]+[\r\n]*
        size_t k;
        if (s[i].cp == ' ' && has(i + 1, kOther)) k = i + 1;
        else if (has(i, kOther)) k = i;
        else return 0;
        while (has(k, kOther)) ++k;
        while (newline(k)) ++k;
        return k;
    };
    auto blanks = [&](size_t i) -> size_t {  // \s*[\r\n]+ | \s+(?!\S) | \s+
        if (!has(i, kSpace)) return 0;
        size_t end = i, after_newline = 0;
        for (; has(end, kSpace); ++end)
            if (is_newline(s[end].cp)) after_newline = end + 1;
        if (after_newline) return after_newline;     // the run up to its last line break
        if (end == n || end - i == 1) return end;    // the whole run (end of text, or a single blank)
        return end - 1;                              // leave one blank to lead the next piece
    };

    for (size_t i = 0; i < n;) {
        size_t j = contraction(i);
        if (!j) j = word(i);
        if (!j) j = number(i);
        if (!j) j = symbols(i);
        if (!j) j = blanks(i);
        if (!j) j = i + 1;
        pieces->emplace_back(s[i].at, j < n ? s[j].at : e);
        i = j;
    }
}

void BpeTokenizer::merge_piece(const std::string& text, size_t b, size_t e, std::vector<int>* out) const {
    const int n = int(e - b);
    if (n <= 0) return;
    std::vector<int> id(static_cast<size_t>(n)), nxt(static_cast<size_t>(n)), prv(static_cast<size_t>(n));
    for (int k = 0; k < n; ++k) {
        id[size_t(k)] = byte_id_[static_cast<unsigned char>(text[b + size_t(k)])];
        nxt[size_t(k)] = k + 1 < n ? k + 1 : -1;
        prv[size_t(k)] = k - 1;
    }
    // candidate merges (rank, left position, left id, right id); stale entries are skipped when popped
    using Cand = std::tuple<uint32_t, int, int, int>;
    std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> heap;
    auto offer = [&](int left) {
        if (left < 0 || nxt[size_t(left)] < 0) return;
        const int a = id[size_t(left)], c = id[size_t(nxt[size_t(left)])];
        const auto it = rank_of_.find(pair_key(a, c));
        if (it != rank_of_.end()) heap.emplace(it->second.first, left, a, c);
    };
    for (int k = 0; k + 1 < n; ++k) offer(k);
    while (!heap.empty()) {
        const auto [rank, left, a, c] = heap.top();
        heap.pop();
        const int right = nxt[size_t(left)];
        if (right < 0 || id[size_t(left)] != a || id[size_t(right)] != c || id[size_t(left)] < 0) continue;
        id[size_t(left)] = rank_of_.find(pair_key(a, c))->second.second;
        id[size_t(right)] = -1;  // gone
        nxt[size_t(left)] = nxt[size_t(right)];
        if (nxt[size_t(right)] >= 0) prv[size_t(nxt[size_t(right)])] = left;
        offer(prv[size_t(left)]);
        offer(left);
        (void)rank;
    }
    for (int k = 0; k >= 0; k = nxt[size_t(k)]) out->push_back(id[size_t(k)]);
}

std::vector<int> BpeTokenizer::encode(const std::string& text) const {
    std::vector<int> out;
    std::vector<std::pair<size_t, size_t>> pieces;
    auto plain = [&](size_t b, size_t e) {
        if (b >= e) return;
        pieces.clear();
        split(text, b, e, &pieces);
        for (const auto& p : pieces) merge_piece(text, p.first, p.second, &out);
    };
    size_t start = 0;
    for (size_t i = 0; i < text.size();) {
        const std::pair<std::string, int>* hit = nullptr;
        for (const auto& sp : special_by_byte_[static_cast<unsigned char>(text[i])])
            if (text.compare(i, sp.first.size(), sp.first) == 0) {
                hit = &sp;
                break;
            }
        if (!hit) {
            ++i;
            continue;
        }
        plain(start, i);
        out.push_back(hit->second);
        i += hit->first.size();
        start = i;
    }
    plain(start, text.size());
    return out;
}

const std::string& BpeTokenizer::piece(int id) const {
    return id >= 0 && id < int(pieces_.size()) ? pieces_[size_t(id)] : empty_;
}

int BpeTokenizer::special_id(const std::string& literal) const {
    const auto it = special_.find(literal);
    return it == special_.end() ? -1 : it->second;
}

}  // namespace qb
