// Shared internals of libhotseat: status handling and small host helpers.
#pragma once

#include <cstdint>
#include <cstring>
#include <string>

#include "../../include/hotseat.h"

namespace hs {

// Thread-local message behind hs_last_error().
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);

inline uint32_t f2u(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
inline float u2f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

// IEEE binary16 -> binary32, exact (the same function as f16.rs:10-31).
inline float h2f_host(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = ((uint32_t)h >> 10) & 0x1f;
    uint32_t man = (uint32_t)h & 0x3ff;
    if (exp == 0) {
        if (man == 0) return u2f(sign);
        uint32_t shift = (uint32_t)__builtin_clz(man) - 22;
        return u2f(sign | ((127 - 15 - shift) << 23) | (((man << (shift + 1)) & 0x3ff) << 13));
    }
    if (exp == 0x1f) return u2f(sign | 0x7f800000u | (man << 13));
    return u2f(sign | ((exp + 112) << 23) | (man << 13));
}

// ggml type -> (elements per block, bytes per block); false for types the
// reference does not load (gguf.rs:70-95).
inline bool ggml_block(uint32_t ty, uint64_t* be, uint64_t* bb) {
    switch (ty) {
        case 0: *be = 1; *bb = 4; return true;
        case 1: *be = 1; *bb = 2; return true;
        case 6: *be = 32; *bb = 22; return true;
        case 8: *be = 32; *bb = 34; return true;
        case 12: *be = 256; *bb = 144; return true;
        case 13: *be = 256; *bb = 176; return true;
        case 14: *be = 256; *bb = 210; return true;
        default: return false;
    }
}

}  // namespace hs

#define HS_CUDA_TRY(expr)                                                                      \
    do {                                                                                       \
        cudaError_t e_ = (expr);                                                               \
        if (e_ != cudaSuccess)                                                                 \
            return hs::fail(HS_E_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_));   \
    } while (0)
