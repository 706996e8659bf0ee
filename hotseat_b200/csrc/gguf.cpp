// GGUF reader. Field order, value types, alignment and tensor byte lengths
// follow the format as hotseat's gguf.rs:154-284 reads it.
#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "common.h"

namespace hs {
namespace {

class Reader {
  public:
    Reader(const uint8_t* b, uint64_t n) : b_(b), n_(n) {}
    uint64_t pos() const { return p_; }
    bool take(uint64_t k, const uint8_t** out) {
        if (k > n_ || p_ > n_ - k) {
            set_error("file truncated: needed " + std::to_string(p_ + k) + " bytes, have " + std::to_string(n_));
            return false;
        }
        *out = b_ + p_;
        p_ += k;
        return true;
    }
    template <typename T>
    bool scalar(T* v) {
        const uint8_t* q;
        if (!take(sizeof(T), &q)) return false;
        std::memcpy(v, q, sizeof(T));
        return true;
    }
    bool str(std::string* s) {
        uint64_t k;
        const uint8_t* q;
        if (!scalar(&k) || !take(k, &q)) return false;
        s->assign(reinterpret_cast<const char*>(q), k);
        return true;
    }

  private:
    const uint8_t* b_;
    uint64_t n_, p_ = 0;
};

bool value_width(uint32_t t, uint64_t* w) {
    switch (t) {
        case 0: case 1: case 7: *w = 1; return true;
        case 2: case 3: *w = 2; return true;
        case 4: case 5: case 6: *w = 4; return true;
        case 10: case 11: case 12: *w = 8; return true;
        default: set_error("unknown metadata value type " + std::to_string(t)); return false;
    }
}

bool read_value(Reader& r, uint32_t t, GgufValue* v) {
    v->type = t;
    switch (t) {
        case 0: { uint8_t x; if (!r.scalar(&x)) return false; v->u = x; return true; }
        case 1: { int8_t x; if (!r.scalar(&x)) return false; v->u = (uint64_t)(int64_t)x; return true; }
        case 2: { uint16_t x; if (!r.scalar(&x)) return false; v->u = x; return true; }
        case 3: { int16_t x; if (!r.scalar(&x)) return false; v->u = (uint64_t)(int64_t)x; return true; }
        case 4: { uint32_t x; if (!r.scalar(&x)) return false; v->u = x; return true; }
        case 5: { int32_t x; if (!r.scalar(&x)) return false; v->u = (uint64_t)(uint32_t)x; return true; }
        case 6: { float x; if (!r.scalar(&x)) return false; v->f = x; return true; }
        case 7: { uint8_t x; if (!r.scalar(&x)) return false; v->u = x != 0; return true; }
        case 8: return r.str(&v->s);
        case 9: {
            if (!r.scalar(&v->arr_type) || !r.scalar(&v->arr_len)) return false;
            const uint8_t* q;
            if (v->arr_type == 8) {
                for (uint64_t i = 0; i < v->arr_len; i++) {
                    uint64_t k;
                    if (!r.scalar(&k) || !r.take(k, &q)) return false;
                }
                return true;
            }
            uint64_t w;
            if (!value_width(v->arr_type, &w)) return false;
            if (v->arr_len > (UINT64_MAX / w)) {
                set_error("metadata array too long");
                return false;
            }
            return r.take(v->arr_len * w, &q);
        }
        case 10: return r.scalar(&v->u);
        case 11: { int64_t x; if (!r.scalar(&x)) return false; v->u = (uint64_t)x; return true; }
        case 12: return r.scalar(&v->f);
        default: set_error("unknown metadata value type " + std::to_string(t)); return false;
    }
}

}  // namespace

Gguf::~Gguf() {
    if (base_) munmap(const_cast<uint8_t*>(base_), size_ ? size_ : 1);
}

int Gguf::open(const char* path) {
    int fd = ::open(path, O_RDONLY);
    if (fd < 0) return fail(HS_E_IO, std::string("io: cannot open ") + path);
    struct stat st;
    if (fstat(fd, &st) != 0) {
        ::close(fd);
        return fail(HS_E_IO, std::string("io: cannot stat ") + path);
    }
    size_ = (uint64_t)st.st_size;
    void* p = mmap(nullptr, size_ ? size_ : 1, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (p == MAP_FAILED) return fail(HS_E_IO, "io: mmap failed");
    base_ = static_cast<const uint8_t*>(p);

    Reader r(base_, size_);
    uint32_t magic = 0, version = 0;
    if (!r.scalar(&magic)) return HS_E_IO;
    if (magic != 0x46554747u) {
        char buf[64];
        snprintf(buf, sizeof buf, "not a GGUF file (magic %#010x)", magic);
        return fail(HS_E_IO, buf);
    }
    if (!r.scalar(&version)) return HS_E_IO;
    if (version != 2 && version != 3) return fail(HS_E_IO, "unsupported GGUF version " + std::to_string(version));
    uint64_t n_tensors = 0, n_kv = 0;
    if (!r.scalar(&n_tensors) || !r.scalar(&n_kv)) return HS_E_IO;
    for (uint64_t i = 0; i < n_kv; i++) {
        std::string key;
        uint32_t t;
        GgufValue v;
        if (!r.str(&key) || !r.scalar(&t) || !read_value(r, t, &v)) return HS_E_IO;
        meta_[key] = v;
    }
    std::vector<GgufTensor> raw;
    for (uint64_t i = 0; i < n_tensors; i++) {
        GgufTensor t;
        uint32_t nd;
        if (!r.str(&t.name) || !r.scalar(&nd)) return HS_E_IO;
        t.dims.resize(nd);
        for (uint32_t d = 0; d < nd; d++)
            if (!r.scalar(&t.dims[d])) return HS_E_IO;
        if (!r.scalar(&t.type) || !r.scalar(&t.off)) return HS_E_IO;
        uint64_t be, bb;
        if (!ggml_block(t.type, &be, &bb)) return fail(HS_E_IO, "unknown tensor type " + std::to_string(t.type));
        raw.push_back(t);
    }
    uint64_t align = 32;
    auto it = meta_.find("general.alignment");
    if (it != meta_.end() && it->second.type == 4 && it->second.u) align = it->second.u;
    uint64_t data_start = (r.pos() + align - 1) / align * align;
    for (auto& t : raw) {
        uint64_t be, bb;
        ggml_block(t.type, &be, &bb);
        t.len = (t.elems() / be) * bb;
        t.off += data_start;
        if (t.off > size_ || t.len > size_ - t.off)
            return fail(HS_E_IO, "tensor \"" + t.name + "\" runs past end of file");
        order_.push_back(t.name);
        tensors_[t.name] = t;
    }
    return HS_OK;
}

const GgufTensor* Gguf::tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
}

int Gguf::get_u32(const std::string& key, uint32_t* v) const {
    auto it = meta_.find(key);
    if (it == meta_.end()) return fail(HS_E_IO, "missing metadata key \"" + key + "\"");
    uint32_t t = it->second.type;
    if (t == 4 || t == 5 || t == 10) {  // gguf.rs:298-306 accepts U32, I32, U64
        *v = (uint32_t)it->second.u;
        return HS_OK;
    }
    return fail(HS_E_IO, "key \"" + key + "\" is not an integer");
}

int Gguf::get_f32(const std::string& key, float* v) const {
    auto it = meta_.find(key);
    if (it == meta_.end()) return fail(HS_E_IO, "missing metadata key \"" + key + "\"");
    if (it->second.type == 6 || it->second.type == 12) {
        *v = (float)it->second.f;
        return HS_OK;
    }
    return fail(HS_E_IO, "key \"" + key + "\" is not a float");
}

int Gguf::get_str(const std::string& key, std::string* v) const {
    auto it = meta_.find(key);
    if (it == meta_.end()) return fail(HS_E_IO, "missing metadata key \"" + key + "\"");
    if (it->second.type != 8) return fail(HS_E_IO, "key \"" + key + "\" is not a string");
    *v = it->second.s;
    return HS_OK;
}

int Gguf::get_str_array_len(const std::string& key, uint64_t* n) const {
    auto it = meta_.find(key);
    if (it == meta_.end()) return fail(HS_E_IO, "missing metadata key \"" + key + "\"");
    if (it->second.type != 9 || it->second.arr_type != 8)
        return fail(HS_E_IO, "key \"" + key + "\" is not a string array");
    *n = it->second.arr_len;
    return HS_OK;
}

}  // namespace hs
