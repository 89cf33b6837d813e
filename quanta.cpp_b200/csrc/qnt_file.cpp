// .qnt reader: one read-only mapping, then a single validating pass over three regions -- the fixed header (decoded
// from a field table), the length-prefixed tokenizer section and the tensor directory -- into zero-copy views.
#include "qnt_file.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <climits>
#include <cstddef>
#include <cstring>

namespace qb {

const char* qnt_fault_name(QntFault f) {
    switch (f) {
        case QntFault::None: return "none";
        case QntFault::Open: return "open";
        case QntFault::Signature: return "signature";
        case QntFault::Version: return "version";
        case QntFault::Header: return "header";
        case QntFault::Tokenizer: return "tokenizer";
        case QntFault::Directory: return "directory";
        case QntFault::Rank: return "rank";
        case QntFault::DType: return "dtype";
        case QntFault::BlockCols: return "block-cols";
        case QntFault::Extent: return "extent";
        case QntFault::Missing: return "missing";
    }
    return "?";
}

QntMissingTensor::QntMissingTensor(const std::string& name)
    : std::runtime_error("the model file has no tensor named '" + name + "'") {}

size_t HostTensor::quant_bytes() const {
    const size_t n = size_t(rows) * size_t(cols);
    switch (dtype) {
        case 0: return n * 4;
        case 1: return n * 2;
        case 2: return n;
        case 3: return n / 2;
    }
    return 0;
}

size_t HostTensor::total_bytes() const {
    const bool blocked = dtype == 2 || dtype == 3;
    return quant_bytes() + (blocked ? size_t(rows) * size_t(cols) / 32 * 2 : 0);
}

namespace {

constexpr char kSignature[4] = {'Q', 'N', 'T', '1'};
constexpr uint32_t kOldestVersion = 1, kNewestVersion = 2;

// A failed check: which invariant, and a message for the caller.
struct Failure {
    QntFault fault = QntFault::None;
    std::string what;
};

// Little-endian fields read from a byte window [at, end) of the mapping.  Every read first checks that the window
// still holds the bytes; a short window records `region` in the failure and leaves the cursor alone.
class Window {
public:
    Window(const uint8_t* at, const uint8_t* end, QntFault region, const char* region_name)
        : at_(at), end_(end), region_(region), region_name_(region_name) {}

    size_t left() const { return size_t(end_ - at_); }
    const uint8_t* at() const { return at_; }

    bool bytes(size_t n, const uint8_t** out, const char* field, Failure* f) {
        if (left() < n) {
            f->fault = region_;
            f->what = std::string(region_name_) + ": field '" + field + "' needs " + std::to_string(n) +
                      " byte(s) but only " + std::to_string(left()) + " remain";
            return false;
        }
        *out = at_;
        at_ += n;
        return true;
    }
    template <typename T>
    bool scalar(T* v, const char* field, Failure* f) {
        const uint8_t* p;
        if (!bytes(sizeof(T), &p, field, f)) return false;
        std::memcpy(v, p, sizeof(T));
        return true;
    }
    bool text(std::string* s, const char* field, Failure* f) {
        uint32_t n;
        const uint8_t* p;
        if (!scalar(&n, field, f) || !bytes(n, &p, field, f)) return false;
        s->assign(reinterpret_cast<const char*>(p), n);
        return true;
    }
    // a u32 count, then `count` records of `rec_bytes` each: checks the whole array fits before reading any of it
    bool counted(uint32_t* count, size_t rec_bytes, const char* field, Failure* f) {
        if (!scalar(count, field, f)) return false;
        if (left() / rec_bytes < *count) {
            f->fault = region_;
            f->what = std::string(region_name_) + ": '" + field + "' lists " + std::to_string(*count) + " record(s) of " +
                      std::to_string(rec_bytes) + " bytes, more than the " + std::to_string(left()) + " bytes left";
            return false;
        }
        return true;
    }

private:
    const uint8_t* at_;
    const uint8_t* end_;
    QntFault region_;
    const char* region_name_;
};

// The fixed header after the version word, in file order.  kind: 'n' positive count, 'f' f32, 'b' u32 flag,
// 'u' raw u32.  `since`: the first version that stores the field (older files leave the default).
struct HeaderField {
    const char* name;
    char kind;
    size_t offset;
    uint32_t since;
};
constexpr HeaderField kHeaderFields[] = {
    {"vocab_size", 'n', offsetof(HParams, vocab_size), 1}, {"dim", 'n', offsetof(HParams, dim), 1},
    {"n_layers", 'n', offsetof(HParams, n_layers), 1},     {"n_heads", 'n', offsetof(HParams, n_heads), 1},
    {"n_kv_heads", 'n', offsetof(HParams, n_kv_heads), 1}, {"head_dim", 'n', offsetof(HParams, head_dim), 1},
    {"ffn_dim", 'n', offsetof(HParams, ffn_dim), 1},       {"max_seq", 'n', offsetof(HParams, max_seq), 1},
    {"rope_theta", 'f', offsetof(HParams, rope_theta), 1}, {"norm_eps", 'f', offsetof(HParams, norm_eps), 1},
    {"tied_embeddings", 'b', offsetof(HParams, tied_embeddings), 1},
    {"qkv_bias", 'b', offsetof(HParams, qkv_bias), 1},     {"flags", 'u', offsetof(HParams, flags), 2},
};

bool decode_header(Window& w, uint32_t version, HParams* hp, Failure* f) {
    unsigned char* base = reinterpret_cast<unsigned char*>(hp);
    for (const HeaderField& fd : kHeaderFields) {
        if (version < fd.since) continue;
        uint32_t raw;
        if (!w.scalar(&raw, fd.name, f)) return false;
        switch (fd.kind) {
            case 'n':
                if (raw == 0 || raw > uint32_t(INT_MAX)) {
                    f->fault = QntFault::Header;
                    f->what = "header: '" + std::string(fd.name) + "' = " + std::to_string(raw) + " is not a positive size";
                    return false;
                }
                *reinterpret_cast<int*>(base + fd.offset) = int(raw);
                break;
            case 'f': std::memcpy(base + fd.offset, &raw, 4); break;
            case 'b': *reinterpret_cast<bool*>(base + fd.offset) = raw != 0; break;
            default: *reinterpret_cast<uint32_t*>(base + fd.offset) = raw; break;
        }
    }
    return true;
}

bool decode_ranges(Window& w, const char* field, std::vector<std::pair<uint32_t, uint32_t>>* out, Failure* f) {
    uint32_t n;
    if (!w.counted(&n, 8, field, f)) return false;
    out->resize(n);
    for (auto& r : *out) {
        w.scalar(&r.first, field, f);
        w.scalar(&r.second, field, f);
    }
    return true;
}

bool decode_tokenizer(Window& w, TokenizerInfo* tok, Failure* f) {
    uint32_t n_tokens;
    if (!w.counted(&n_tokens, 4, "token count", f)) return false;  // each token costs at least its length word
    tok->n_tokens = int(n_tokens);
    tok->tokens.resize(n_tokens);
    for (auto& s : tok->tokens)
        if (!w.text(&s, "token bytes", f)) return false;
    uint32_t n_merges;
    if (!w.counted(&n_merges, 12, "merges", f)) return false;
    tok->merges.resize(n_merges);
    for (auto& m : tok->merges)
        for (uint32_t& x : m) w.scalar(&x, "merges", f);
    uint32_t n_special;
    if (!w.counted(&n_special, 8, "specials", f)) return false;
    tok->specials.resize(n_special);
    for (auto& s : tok->specials) {
        uint32_t id;
        if (!w.scalar(&id, "special id", f) || !w.text(&s.second, "special text", f)) return false;
        s.first = int(id);
    }
    return decode_ranges(w, "letter ranges", &tok->letters, f) && decode_ranges(w, "number ranges", &tok->numbers, f) &&
           decode_ranges(w, "space ranges", &tok->spaces, f);
}

const char* dtype_label(int dt) {
    static const char* names[] = {"f32", "f16", "q8_0", "q4_0"};
    return dt >= 0 && dt < 4 ? names[dt] : "?";
}

// One directory entry, decoded and checked against the file's size.
bool decode_entry(Window& w, uint32_t index, const uint8_t* map, size_t file_size, std::string* name, HostTensor* t,
                  Failure* f) {
    uint32_t dtype, rank;
    if (!w.text(name, "tensor name", f) || !w.scalar(&dtype, "tensor dtype", f) || !w.scalar(&rank, "tensor rank", f))
        return false;
    const std::string who = "tensor '" + *name + "' (directory entry " + std::to_string(index) + ")";
    if (rank != 1 && rank != 2) {
        f->fault = QntFault::Rank;
        f->what = who + " has rank " + std::to_string(rank) + "; the format stores 1-D and 2-D tensors only";
        return false;
    }
    uint32_t dims[2] = {1, 0};
    for (uint32_t i = 2 - rank; i < 2; ++i)
        if (!w.scalar(&dims[i], "tensor shape", f)) return false;
    uint64_t offset;
    if (!w.scalar(&offset, "tensor offset", f)) return false;
    if (dtype > 3) {
        f->fault = QntFault::DType;
        f->what = who + " has dtype code " + std::to_string(dtype) + " (known: 0 f32, 1 f16, 2 q8_0, 3 q4_0)";
        return false;
    }
    if (dims[0] > uint32_t(INT_MAX) || dims[1] > uint32_t(INT_MAX)) {
        f->fault = QntFault::Extent;
        f->what = who + " has a dimension above 2^31 - 1";
        return false;
    }
    t->dtype = int(dtype);
    t->rank = int(rank);
    t->rows = int(dims[0]);
    t->cols = int(dims[1]);
    if ((dtype == 2 || dtype == 3) && t->cols % 32 != 0) {
        f->fault = QntFault::BlockCols;
        f->what = who + " is " + dtype_label(t->dtype) + " with rows of " + std::to_string(t->cols) +
                  " values, not whole 32-value blocks";
        return false;
    }
    const uint64_t bytes = t->total_bytes();
    if (offset > file_size || bytes > file_size - offset) {
        f->fault = QntFault::Extent;
        f->what = who + " occupies bytes [" + std::to_string(offset) + ", " + std::to_string(offset + bytes) +
                  ") but the file ends at byte " + std::to_string(file_size);
        return false;
    }
    t->data = map + offset;
    return true;
}

}  // namespace

QntFile::~QntFile() { release(); }

void QntFile::release() {
    if (map_) munmap(const_cast<uint8_t*>(map_), size_);
    map_ = nullptr;
    size_ = 0;
    tensors_.clear();
    tok_ = TokenizerInfo{};
    hp_ = HParams{};
}

bool QntFile::open(const std::string& path, std::string* err) {
    release();
    Failure f;
    auto fail = [&]() {
        fault_ = f.fault;
        if (err) *err = f.what;
        release();
        return false;
    };
    const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    struct stat st {};
    if (fd < 0 || fstat(fd, &st) != 0 || st.st_size <= 0) {
        const int code = errno;
        if (fd >= 0) ::close(fd);
        f = {QntFault::Open, "cannot read model file '" + path + "': " +
                                 (fd >= 0 && st.st_size <= 0 ? std::string("empty file") : std::string(std::strerror(code)))};
        return fail();
    }
    void* m = mmap(nullptr, size_t(st.st_size), PROT_READ, MAP_SHARED, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) {
        f = {QntFault::Open, "cannot map model file '" + path + "': " + std::strerror(errno)};
        return fail();
    }
    map_ = static_cast<const uint8_t*>(m);
    size_ = size_t(st.st_size);

    // region 1: signature, version, hyper-parameters
    if (size_ < sizeof kSignature || std::memcmp(map_, kSignature, sizeof kSignature) != 0) {
        f = {QntFault::Signature, "'" + path + "' is not a quanta model file: it does not start with \"QNT1\""};
        return fail();
    }
    Window head(map_ + sizeof kSignature, map_ + size_, QntFault::Header, "header");
    uint32_t version;
    if (!head.scalar(&version, "version", &f)) return fail();
    if (version < kOldestVersion || version > kNewestVersion) {
        f = {QntFault::Version, "model format version " + std::to_string(version) + " is not supported (this reader handles " +
                                    std::to_string(kOldestVersion) + " to " + std::to_string(kNewestVersion) + ")"};
        return fail();
    }
    if (!decode_header(head, version, &hp_, &f)) return fail();

    // region 2: the tokenizer section, decoded inside its own length
    uint32_t tok_bytes;
    const uint8_t* tok_at;
    if (!head.scalar(&tok_bytes, "tokenizer length", &f) || !head.bytes(tok_bytes, &tok_at, "tokenizer section", &f))
        return fail();
    Window tok(tok_at, tok_at + tok_bytes, QntFault::Tokenizer, "tokenizer section");
    if (!decode_tokenizer(tok, &tok_, &f)) return fail();

    // region 3: the tensor directory
    dir_offset_ = size_t(head.at() - map_);
    order_.clear();
    Window dir(head.at(), map_ + size_, QntFault::Directory, "tensor directory");
    uint32_t n_tensors;
    if (!dir.scalar(&n_tensors, "tensor count", &f)) return fail();
    tensors_.reserve(n_tensors);
    for (uint32_t i = 0; i < n_tensors; ++i) {
        std::string name;
        HostTensor t;
        if (!decode_entry(dir, i, map_, size_, &name, &t, &f)) return fail();
        if (!tensors_.emplace(name, t).second) {
            f = {QntFault::Directory, "tensor '" + name + "' appears twice in the directory"};
            return fail();
        }
        order_.push_back(name);
    }
    fault_ = QntFault::None;
    return true;
}

const HostTensor* QntFile::find(const std::string& name) const {
    const auto it = tensors_.find(name);
    return it != tensors_.end() ? &it->second : nullptr;
}

const HostTensor& QntFile::require(const std::string& name) const {
    if (const HostTensor* t = find(name)) return *t;
    throw QntMissingTensor(name);
}

int QntFile::special_id(const std::string& text) const {
    for (const auto& s : tok_.specials)
        if (s.second == text) return s.first;
    return -1;
}

}  // namespace qb
