#include "qnt_file.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <stdexcept>

namespace qb {

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
    size_t t = quant_bytes();
    if (dtype == 2 || dtype == 3) t += size_t(rows) * size_t(cols) / 32 * 2;
    return t;
}

namespace {

// Bounds-checked little-endian reader.
struct Reader {
    const uint8_t* p;
    const uint8_t* end;
    void need(size_t n) const {
        if (size_t(end - p) < n) throw std::runtime_error("model file truncated");
    }
    uint32_t u32() {
        need(4);
        uint32_t v;
        std::memcpy(&v, p, 4);
        p += 4;
        return v;
    }
    uint64_t u64() {
        need(8);
        uint64_t v;
        std::memcpy(&v, p, 8);
        p += 8;
        return v;
    }
    float f32() {
        const uint32_t u = u32();
        float f;
        std::memcpy(&f, &u, 4);
        return f;
    }
    std::string str() {
        const uint32_t n = u32();
        need(n);
        std::string s(reinterpret_cast<const char*>(p), n);
        p += n;
        return s;
    }
    void skip_ranges() {
        const uint32_t n = u32();
        need(size_t(n) * 8);
        p += size_t(n) * 8;
    }
};

}  // namespace

QntFile::~QntFile() { unmap(); }

void QntFile::unmap() {
    if (base_) munmap(const_cast<uint8_t*>(base_), size_);
    base_ = nullptr;
    size_ = 0;
    tensors_.clear();
}

bool QntFile::open(const std::string& path, std::string* err) {
    unmap();
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        if (err) *err = "cannot open " + path;
        return false;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) {
        ::close(fd);
        if (err) *err = "cannot stat " + path;
        return false;
    }
    size_ = size_t(st.st_size);
    void* m = mmap(nullptr, size_, PROT_READ, MAP_SHARED, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) {
        size_ = 0;
        if (err) *err = "mmap failed";
        return false;
    }
    base_ = static_cast<const uint8_t*>(m);
    try {
        Reader r{base_, base_ + size_};
        r.need(4);
        if (std::memcmp(r.p, "QNT1", 4) != 0) throw std::runtime_error("bad magic (not a .qnt file)");
        r.p += 4;
        const uint32_t version = r.u32();
        if (version < 1 || version > 2) throw std::runtime_error("unsupported version " + std::to_string(version));
        hp_.vocab_size = int(r.u32());
        hp_.dim = int(r.u32());
        hp_.n_layers = int(r.u32());
        hp_.n_heads = int(r.u32());
        hp_.n_kv_heads = int(r.u32());
        hp_.head_dim = int(r.u32());
        hp_.ffn_dim = int(r.u32());
        hp_.max_seq = int(r.u32());
        hp_.rope_theta = r.f32();
        hp_.norm_eps = r.f32();
        hp_.tied_embeddings = r.u32() != 0;
        hp_.qkv_bias = r.u32() != 0;
        hp_.flags = version >= 2 ? r.u32() : 0;

        const uint32_t tok_len = r.u32();
        r.need(tok_len);
        Reader t{r.p, r.p + tok_len};
        r.p += tok_len;
        tok_.n_tokens = int(t.u32());
        tok_.tokens.resize(size_t(tok_.n_tokens));
        for (auto& s : tok_.tokens) s = t.str();
        const uint32_t n_merges = t.u32();
        t.need(size_t(n_merges) * 12);
        t.p += size_t(n_merges) * 12;
        const uint32_t n_special = t.u32();
        for (uint32_t i = 0; i < n_special; ++i) {
            const int id = int(t.u32());
            tok_.specials.emplace_back(id, t.str());
        }
        t.skip_ranges();
        t.skip_ranges();
        t.skip_ranges();

        const uint32_t n_tensors = r.u32();
        for (uint32_t i = 0; i < n_tensors; ++i) {
            std::string name = r.str();
            HostTensor ht;
            ht.dtype = int(r.u32());
            if (ht.dtype < 0 || ht.dtype > 3) throw std::runtime_error("bad dtype for " + name);
            const uint32_t ndim = r.u32();
            if (ndim == 1) {
                ht.rows = 1;
                ht.cols = int(r.u32());
            } else if (ndim == 2) {
                ht.rows = int(r.u32());
                ht.cols = int(r.u32());
            } else {
                throw std::runtime_error("unsupported ndim for " + name);
            }
            if ((ht.dtype == 2 || ht.dtype == 3) && ht.cols % 32 != 0)
                throw std::runtime_error("quantized tensor cols not a multiple of 32: " + name);
            const uint64_t off = r.u64();
            if (off > size_) throw std::runtime_error("bad offset for " + name);
            ht.data = base_ + off;
            if (off + ht.total_bytes() > size_) throw std::runtime_error("tensor out of bounds: " + name);
            tensors_.emplace(std::move(name), ht);
        }
    } catch (const std::exception& e) {
        if (err) *err = e.what();
        unmap();
        return false;
    }
    return true;
}

const HostTensor* QntFile::find(const std::string& name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
}

const HostTensor& QntFile::get(const std::string& name) const {
    if (const HostTensor* t = find(name)) return *t;
    throw std::runtime_error("missing tensor: " + name);
}

int QntFile::special_id(const std::string& text) const {
    for (const auto& s : tok_.specials)
        if (s.second == text) return s.first;
    return -1;
}

}  // namespace qb
