// GGUF v2/v3 reader over a read-only mapping (the format hotseat's
// hs-engine gguf.rs:225-350 reads). Only the pieces the token loop needs:
// metadata scalars, string-array lengths, and the tensor table.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace hs {

struct GgufTensor {
    std::string name;
    std::vector<uint64_t> dims;  // ne0 first: dims[0] is the row length
    uint32_t type = 0;           // ggml type id
    uint64_t off = 0;            // absolute file offset
    uint64_t len = 0;            // bytes: (elems / block_elems) * block_bytes (gguf.rs:272-274)
    uint64_t elems() const {
        uint64_t e = 1;
        for (uint64_t d : dims) e *= d;
        return e;
    }
};

struct GgufValue {
    uint32_t type = 0;  // GGUF value type
    uint64_t u = 0;     // integer payloads (and bool)
    double f = 0.0;     // f32 / f64 payloads
    std::string s;      // string payload
    uint32_t arr_type = 0;
    uint64_t arr_len = 0;
};

class Gguf {
  public:
    ~Gguf();
    // Returns HS_OK or HS_E_IO with the message set.
    int open(const char* path);
    const uint8_t* data() const { return base_; }
    uint64_t size() const { return size_; }
    const GgufTensor* tensor(const std::string& name) const;
    const std::vector<std::string>& order() const { return order_; }
    // Typed metadata getters; on failure set the error and return HS_E_IO.
    int get_u32(const std::string& key, uint32_t* v) const;
    int get_f32(const std::string& key, float* v) const;
    int get_str(const std::string& key, std::string* v) const;
    int get_str_array_len(const std::string& key, uint64_t* n) const;
    bool has(const std::string& key) const { return meta_.count(key) != 0; }

  private:
    const uint8_t* base_ = nullptr;
    uint64_t size_ = 0;
    std::map<std::string, GgufValue> meta_;
    std::map<std::string, GgufTensor> tensors_;
    std::vector<std::string> order_;
};

}  // namespace hs
