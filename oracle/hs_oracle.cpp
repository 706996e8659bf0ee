// hs_oracle.cpp — CPU restatement of hotseat's hs-engine token loop.
//
// TEST INFRASTRUCTURE ONLY (the checker). Used by tests/, __graft_entry__.smoke()
// and bench.py's CPU baseline; the product never links it.
//
// Every function follows the reference file:line it cites (paths are inside the
// hotseat repository, crates/hs-engine/src unless stated). Build flags matter:
// -O3 -ffp-contract=off, no -ffast-math, so float expressions evaluate exactly as
// written, one IEEE f32 operation at a time, like the Rust original.

#include "hs_oracle.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <functional>
#include <map>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <thread>
#include <unistd.h>
#include <vector>

namespace {

thread_local std::string g_err;

inline uint32_t f2u(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
inline float u2f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

// ---------------------------------------------------------------- f16.rs:10-31
float f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = ((uint32_t)h >> 10) & 0x1f;
    uint32_t man = (uint32_t)h & 0x3ff;
    if (exp == 0) {
        if (man == 0) return u2f(sign);
        uint32_t shift = (uint32_t)__builtin_clz(man) - 22;  // leading zeros in the 10-bit field
        uint32_t e = 127 - 15 - shift;
        uint32_t m = (man << (shift + 1)) & 0x3ff;
        return u2f(sign | (e << 23) | (m << 13));
    }
    if (exp == 0x1f) return u2f(sign | 0x7f800000u | (man << 13));
    return u2f(sign | ((exp + (127 - 15)) << 23) | (man << 13));
}

// ---------------------------------------------------------------- f16.rs:35-69
uint16_t f32_to_f16(float f) {
    uint32_t x = f2u(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000);
    int32_t exp = (int32_t)((x >> 23) & 0xff);
    uint32_t man = x & 0x7fffff;
    if (exp == 0xff) {
        uint16_t m = (uint16_t)(man >> 13);
        return (uint16_t)(sign | 0x7c00 | ((man != 0 && m == 0) ? 1 : m));
    }
    exp -= 127 - 15;
    if (exp >= 0x1f) return (uint16_t)(sign | 0x7c00);
    if (exp <= 0) {
        if (exp < -10) return sign;
        uint32_t m = man | 0x800000u;
        uint32_t shift = (uint32_t)(14 - exp);
        uint32_t half = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1);
        uint32_t tie = 1u << (shift - 1);
        uint32_t round = (rem > tie || (rem == tie && (half & 1) == 1)) ? 1u : 0u;
        return (uint16_t)(sign | (uint16_t)(half + round));
    }
    uint32_t half = ((uint32_t)exp << 10) | (man >> 13);
    uint32_t rem = man & 0x1fff;
    uint32_t round = (rem > 0x1000 || (rem == 0x1000 && ((man >> 13) & 1) == 1)) ? 1u : 0u;
    return (uint16_t)((uint16_t)(half + round) | sign);
}

// --------------------------------------------------------------- math.rs:27-30
const float LOG2_E = 1.44269504f;
const float LN2_HI = 0.693359375f;
const float LN2_LO = -2.1219444e-4f;

// --------------------------------------------------------------- math.rs:65-75
float pow2i(int32_t k) {
    int32_t e = k + 127;
    if (e <= 0) {
        if (e <= -23) return 0.0f;
        return u2f(1u << (22 + e));
    }
    return u2f((uint32_t)e << 23);
}

// --------------------------------------------------------------- math.rs:39-61
float exp_f32(float x) {
    if (std::isnan(x)) return x;
    if (x >= 89.0f) return INFINITY;
    if (x <= -104.0f) return 0.0f;
    float kf = roundf(x * LOG2_E);  // Rust round(): half away from zero, as C roundf
    float r = x - kf * LN2_HI - kf * LN2_LO;
    float p = 1.0f +
              r * (1.0f +
                   r * (0.5f + r * (0.16666667f +
                                    r * (0.04166667f + r * (0.00833333f + r * 0.001388889f)))));
    int32_t k = (int32_t)kf;
    int32_t k1 = k >> 1;
    int32_t k2 = k - k1;
    return p * pow2i(k1) * pow2i(k2);
}

// --------------------------------------------------------------- math.rs:79-81
float silu(float x) { return x / (1.0f + exp_f32(-x)); }

// --------------------------------------------------------------- math.rs:89-93
constexpr size_t LANES = 8;
inline float fold(const float a[LANES]) {
    float l = (a[0] + a[1]) + (a[2] + a[3]);
    float r = (a[4] + a[5]) + (a[6] + a[7]);
    return l + r;
}

// ------------------------------------------------------------- math.rs:117-128
// The x86 path of dot_f16 (math.rs:101-112 picks the scalar form off aarch64).
float dot_f16(const uint16_t* w, const float* x, size_t n) {
    float acc[LANES] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (size_t i = 0; i < n; i += LANES)
        for (size_t l = 0; l < LANES; l++) acc[l] += f16_to_f32(w[i + l]) * x[i + l];
    return fold(acc);
}

// ------------------------------------------------------------- math.rs:160-181
float dot_f32(const float* a, const float* b, size_t n) {
    float acc[LANES] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t full = n / LANES * LANES;
    size_t i = 0;
    while (i < full) {
        for (size_t l = 0; l < LANES; l++) acc[l] += a[i + l] * b[i + l];
        i += LANES;
    }
    float s = fold(acc);
    while (i < n) {
        s += a[i] * b[i];
        i++;
    }
    return s;
}

// ------------------------------------------------------------- math.rs:185-190
inline void axpy(float* y, const float* v, float s, size_t n) {
    for (size_t i = 0; i < n; i++) y[i] += s * v[i];
}

// ------------------------------------------------------------- math.rs:200-207
void rmsnorm(float* out, const float* x, const float* g, size_t n, float eps) {
    float ss = dot_f32(x, x, n);
    float scale = 1.0f / sqrtf(ss / (float)n + eps);
    for (size_t i = 0; i < n; i++) out[i] = x[i] * scale * g[i];
}

// ------------------------------------------------------------- math.rs:210-226
void softmax(float* x, size_t n) {
    float m = -INFINITY;
    for (size_t i = 0; i < n; i++)
        if (x[i] > m) m = x[i];
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) {
        x[i] = exp_f32(x[i] - m);
        sum += x[i];
    }
    float inv = 1.0f / sum;
    for (size_t i = 0; i < n; i++) x[i] *= inv;
}

// ------------------------------------------------------------- math.rs:250-264
float ln_f32(float x) {
    uint32_t bits = f2u(x);
    int32_t e = (int32_t)((bits >> 23) & 0xff) - 127;
    float m = u2f((bits & 0x007fffff) | (127u << 23));
    if (m > 1.4142136f) {
        m *= 0.5f;
        e += 1;
    }
    float s = (m - 1.0f) / (m + 1.0f);
    float s2 = s * s;
    float p = s * (2.0f + s2 * (0.6666667f + s2 * (0.4f + s2 * (0.2857143f + s2 * 0.2222222f))));
    return p + (float)e * (LN2_HI + LN2_LO);
}

// ------------------------------------------------------------- math.rs:285-294
float sin_poly(float r) {
    float r2 = r * r;
    return r * (1.0f + r2 * (-0.16666667f + r2 * (0.00833333f + r2 * (-1.984127e-4f + r2 * 2.755732e-6f))));
}
float cos_poly(float r) {
    float r2 = r * r;
    return 1.0f + r2 * (-0.5f + r2 * (0.04166667f + r2 * (-0.001388889f + r2 * 2.480159e-5f)));
}

// ------------------------------------------------------------- math.rs:272-282
// q uses the f32 constant pi/2 widened to f64; r uses the f64 constant.
void sincos_f32(float x, float* so, float* co) {
    const float PI_2 = 1.57079632679489661923f;
    const double FRAC_PI_2_F64 = 1.57079632679489661923;
    double q = std::round((double)x / (double)PI_2);
    float r = (float)((double)x - q * FRAC_PI_2_F64);
    float s = sin_poly(r), c = cos_poly(r);
    int64_t qi = (int64_t)q;
    int64_t k = ((qi % 4) + 4) % 4;  // rem_euclid(4)
    switch (k) {
        case 0: *so = s; *co = c; break;
        case 1: *so = c; *co = -s; break;
        case 2: *so = -s; *co = -c; break;
        default: *so = -c; *co = s; break;
    }
}

// ------------------------------------------------------------ quant.rs:59-62
inline float half_at(const uint8_t* b, size_t at) {
    return f16_to_f32((uint16_t)(b[at] | ((uint16_t)b[at + 1] << 8)));
}

// ------------------------------------------------------------ quant.rs:64-74
void dequant_q8_0(const uint8_t* src, size_t n, uint16_t* dst) {
    const size_t QK = 32, BS = 34;
    for (size_t bi = 0; bi < n / QK; bi++) {
        const uint8_t* blk = src + bi * BS;
        float d = half_at(blk, 0);
        for (size_t l = 0; l < QK; l++) {
            float q = (float)(int8_t)blk[2 + l];
            dst[bi * QK + l] = f32_to_f16(d * q);
        }
    }
}

// ------------------------------------------------------------ quant.rs:79-96
void dequant_q5_0(const uint8_t* src, size_t n, uint16_t* dst) {
    const size_t QK = 32, BS = 22;
    for (size_t bi = 0; bi < n / QK; bi++) {
        const uint8_t* blk = src + bi * BS;
        float d = half_at(blk, 0);
        uint32_t qh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) | ((uint32_t)blk[4] << 16) |
                      ((uint32_t)blk[5] << 24);
        const uint8_t* qs = blk + 6;
        size_t base = bi * QK;
        for (size_t j = 0; j < QK / 2; j++) {
            uint8_t h0 = (uint8_t)((qh >> j) << 4) & 0x10;
            uint8_t h1 = (uint8_t)(qh >> (j + 12)) & 0x10;
            int32_t x0 = (int32_t)((qs[j] & 0x0F) | h0) - 16;
            int32_t x1 = (int32_t)((qs[j] >> 4) | h1) - 16;
            dst[base + j] = f32_to_f16(d * (float)x0);
            dst[base + j + QK / 2] = f32_to_f16(d * (float)x1);
        }
    }
}

// ----------------------------------------------------------- quant.rs:101-107
inline void scale_min_k4(size_t j, const uint8_t* q, uint8_t* sc, uint8_t* m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

// ----------------------------------------------------------- quant.rs:109-139
void dequant_q4_k(const uint8_t* src, size_t n, uint16_t* dst) {
    const size_t QK = 256, BS = 144;
    for (size_t bi = 0; bi < n / QK; bi++) {
        const uint8_t* blk = src + bi * BS;
        float d = half_at(blk, 0);
        float dmin = half_at(blk, 2);
        const uint8_t* scales = blk + 4;
        const uint8_t* qs = blk + 16;
        size_t base = bi * QK, o = 0, is = 0;
        for (size_t g = 0; g < 4; g++) {
            const uint8_t* q = qs + g * 32;
            uint8_t sc1, m1, sc2, m2;
            scale_min_k4(is, scales, &sc1, &m1);
            scale_min_k4(is + 1, scales, &sc2, &m2);
            float d1 = d * (float)sc1, mm1 = dmin * (float)m1;
            float d2 = d * (float)sc2, mm2 = dmin * (float)m2;
            for (size_t l = 0; l < 32; l++) dst[base + o + l] = f32_to_f16(d1 * (float)(q[l] & 0x0F) - mm1);
            for (size_t l = 0; l < 32; l++) dst[base + o + 32 + l] = f32_to_f16(d2 * (float)(q[l] >> 4) - mm2);
            o += 64;
            is += 2;
        }
    }
}

// ----------------------------------------------------------- quant.rs:143-176
void dequant_q5_k(const uint8_t* src, size_t n, uint16_t* dst) {
    const size_t QK = 256, BS = 176;
    for (size_t bi = 0; bi < n / QK; bi++) {
        const uint8_t* blk = src + bi * BS;
        float d = half_at(blk, 0);
        float dmin = half_at(blk, 2);
        const uint8_t* scales = blk + 4;
        const uint8_t* qh = blk + 16;
        const uint8_t* ql = blk + 48;
        size_t base = bi * QK, o = 0, is = 0;
        uint8_t u1 = 1, u2 = 2;
        for (size_t g = 0; g < 4; g++) {
            const uint8_t* q = ql + g * 32;
            uint8_t sc1, m1, sc2, m2;
            scale_min_k4(is, scales, &sc1, &m1);
            scale_min_k4(is + 1, scales, &sc2, &m2);
            float d1 = d * (float)sc1, mm1 = dmin * (float)m1;
            float d2 = d * (float)sc2, mm2 = dmin * (float)m2;
            for (size_t l = 0; l < 32; l++) {
                uint32_t hi = (qh[l] & u1) ? 16 : 0;
                dst[base + o + l] = f32_to_f16(d1 * (float)((q[l] & 0x0F) + hi) - mm1);
            }
            for (size_t l = 0; l < 32; l++) {
                uint32_t hi = (qh[l] & u2) ? 16 : 0;
                dst[base + o + 32 + l] = f32_to_f16(d2 * (float)((q[l] >> 4) + hi) - mm2);
            }
            o += 64;
            is += 2;
            u1 = (uint8_t)(u1 << 2);
            u2 = (uint8_t)(u2 << 2);
        }
    }
}

// ----------------------------------------------------------- quant.rs:178-206
void dequant_q6_k(const uint8_t* src, size_t n, uint16_t* dst) {
    const size_t QK = 256, BS = 210;
    for (size_t bi = 0; bi < n / QK; bi++) {
        const uint8_t* blk = src + bi * BS;
        float d = half_at(blk, 208);
        size_t base = bi * QK;
        for (size_t h = 0; h < 2; h++) {
            const uint8_t* ql = blk + h * 64;
            const uint8_t* qh = blk + 128 + h * 32;
            const uint8_t* sc = blk + 192 + h * 8;
            size_t out = base + h * 128;
            for (size_t l = 0; l < 32; l++) {
                size_t is = l / 16;
                int32_t q1 = (int32_t)((ql[l] & 0x0F) | (((qh[l] >> 0) & 3) << 4)) - 32;
                int32_t q2 = (int32_t)((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int32_t q3 = (int32_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int32_t q4 = (int32_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                dst[out + l] = f32_to_f16(d * (float)(int8_t)sc[is] * (float)q1);
                dst[out + l + 32] = f32_to_f16(d * (float)(int8_t)sc[is + 2] * (float)q2);
                dst[out + l + 64] = f32_to_f16(d * (float)(int8_t)sc[is + 4] * (float)q3);
                dst[out + l + 96] = f32_to_f16(d * (float)(int8_t)sc[is + 6] * (float)q4);
            }
        }
    }
}

// ------------------------------------------------------------- quant.rs:18-38
int dequant_to_f16(uint32_t ty, const uint8_t* src, size_t n, uint16_t* dst) {
    switch (ty) {
        case 1:
            for (size_t i = 0; i < n; i++) dst[i] = (uint16_t)(src[i * 2] | (src[i * 2 + 1] << 8));
            return 0;
        case 0:
            for (size_t i = 0; i < n; i++) {
                float f;
                std::memcpy(&f, src + i * 4, 4);
                dst[i] = f32_to_f16(f);
            }
            return 0;
        case 6: dequant_q5_0(src, n, dst); return 0;
        case 8: dequant_q8_0(src, n, dst); return 0;
        case 12: dequant_q4_k(src, n, dst); return 0;
        case 13: dequant_q5_k(src, n, dst); return 0;
        case 14: dequant_q6_k(src, n, dst); return 0;
        default: return -1;
    }
}

// -------------------------------------------------------------- gguf.rs:84-95
bool block_of(uint32_t ty, size_t* be, size_t* bb) {
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

// `t.ty as u32` in model.rs:152 is the Rust enum's declaration index
// (gguf.rs:60-68: F32, F16, Q5_0, Q8_0, Q4K, Q5K, Q6K), not the ggml id.
uint32_t enum_index(uint32_t ty) {
    switch (ty) {
        case 0: return 0;
        case 1: return 1;
        case 6: return 2;
        case 8: return 3;
        case 12: return 4;
        case 13: return 5;
        case 14: return 6;
        default: return 0xffffffffu;
    }
}

// ---------------------------------------------------------------- hash.rs:9-58
const uint64_t FNV_OFFSET = 0xcbf29ce484222325ull;
const uint64_t FNV_PRIME = 0x00000100000001b3ull;
struct Fnv {
    uint64_t h = FNV_OFFSET;
    void write(const uint8_t* p, size_t n) {
        for (size_t i = 0; i < n; i++) {
            h ^= p[i];
            h *= FNV_PRIME;
        }
    }
    void write_u64(uint64_t v) { uint8_t b[8]; std::memcpy(b, &v, 8); write(b, 8); }
    void write_u32(uint32_t v) { uint8_t b[4]; std::memcpy(b, &v, 4); write(b, 4); }
};

// ------------------------------------------------------------- hash.rs:63-126
inline uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }
struct Wide {
    uint64_t l[4] = {0x243f6a8885a308d3ull, 0x13198a2e03707344ull, 0xa4093822299f31d0ull,
                     0x082efa98ec4e6c89ull};
    uint64_t len = 0;
    void write(const uint8_t* b, size_t n) {
        len += n;
        size_t full = n / 32 * 32;
        for (size_t c = 0; c < full; c += 32)
            for (int k = 0; k < 4; k++) {
                uint64_t w;
                std::memcpy(&w, b + c + k * 8, 8);
                l[k] = (l[k] ^ w) * FNV_PRIME;
                l[k] ^= l[k] >> 29;
            }
        for (size_t i = 0; i < n - full; i++) {
            int k = (int)(i % 4);
            l[k] = (l[k] ^ (uint64_t)b[full + i]) * FNV_PRIME;
        }
    }
    uint64_t finish() const {
        uint64_t h = l[0] ^ rotl(l[1], 17) ^ rotl(l[2], 34) ^ rotl(l[3], 51);
        h += len;
        h ^= h >> 33;
        h *= 0xff51afd7ed558ccdull;
        h ^= h >> 33;
        return h;
    }
};

// ------------------------------------------------------------- sampler.rs:47-80
void rng_seed(uint64_t seed, hso_rng* r) {
    uint64_t z = seed;
    for (int i = 0; i < 4; i++) {
        z += 0x9E3779B97F4A7C15ull;
        uint64_t x = z;
        x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
        x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
        r->s[i] = x ^ (x >> 31);
    }
    r->draws = 0;
}
uint64_t rng_next_u64(hso_rng* r) {
    uint64_t* s = r->s;
    uint64_t result = rotl(s[1] * 5, 7) * 9;
    uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl(s[3], 45);
    r->draws += 1;
    return result;
}
float rng_next_f32(hso_rng* r) { return (float)(rng_next_u64(r) >> 40) * (1.0f / 16777216.0f); }

// f32::total_cmp key: flip the magnitude bits of negatives so signed integer
// order equals the IEEE total order (-NaN < -inf < ... < -0 < +0 < ... < +NaN).
inline int32_t total_key(float f) {
    int32_t b = (int32_t)f2u(f);
    b ^= (int32_t)(((uint32_t)(b >> 31)) >> 1);
    return b;
}

// ----------------------------------------------------------- sampler.rs:170-175
// cmp_desc: larger value first (total order), then lower id first.
inline bool desc_less(const std::pair<float, uint32_t>& a, const std::pair<float, uint32_t>& b) {
    int32_t ka = total_key(a.first), kb = total_key(b.first);
    if (ka != kb) return ka > kb;
    return a.second < b.second;
}

// ----------------------------------------------------------- sampler.rs:177-187
uint32_t argmax(const float* l, size_t n) {
    uint32_t best = 0;
    float bv = -INFINITY;
    for (size_t i = 0; i < n; i++)
        if (l[i] > bv) {
            bv = l[i];
            best = (uint32_t)i;
        }
    return best;
}

// ----------------------------------------------------------- sampler.rs:103-111
void apply_penalty(const hso_sampler_cfg* cfg, float* logits, const uint32_t* hist, size_t n_hist) {
    if (cfg->repeat_penalty != 1.0f && cfg->repeat_last_n > 0) {
        size_t n = std::min((size_t)cfg->repeat_last_n, n_hist);
        for (size_t i = n_hist - n; i < n_hist; i++) {
            float* l = &logits[hist[i]];
            *l = (*l > 0.0f) ? *l / cfg->repeat_penalty : *l * cfg->repeat_penalty;
        }
    }
}

// ----------------------------------------------------------- sampler.rs:100-167
uint32_t sample(const hso_sampler_cfg* cfg, hso_rng* rng, float* logits, size_t n, const uint32_t* hist,
                size_t n_hist) {
    apply_penalty(cfg, logits, hist, n_hist);
    if (cfg->temperature <= 0.0f) return argmax(logits, n);
    size_t k = cfg->top_k == 0 ? n : std::min((size_t)cfg->top_k, n);
    std::vector<std::pair<float, uint32_t>> cand(n);
    for (size_t i = 0; i < n; i++) cand[i] = {logits[i], (uint32_t)i};
    // select_nth_unstable + truncate + sort under a strict total order: the
    // result is exactly the k smallest under desc_less, in order.
    if (k < cand.size()) {
        std::nth_element(cand.begin(), cand.begin() + (k - 1), cand.end(), desc_less);
        cand.resize(k);
    }
    std::sort(cand.begin(), cand.end(), desc_less);
    float inv_t = 1.0f / cfg->temperature;
    float mx = cand[0].first;
    float sum = 0.0f;
    for (auto& c : cand) {
        c.first = exp_f32((c.first - mx) * inv_t);
        sum += c.first;
    }
    size_t cut = cand.size();
    if (cfg->top_p < 1.0f) {
        float target = cfg->top_p * sum;
        float acc = 0.0f;
        for (size_t i = 0; i < cand.size(); i++) {
            acc += cand[i].first;
            if (acc >= target) {
                cut = i + 1;
                break;
            }
        }
        // Iterator::sum over f32 folds left to right; the values are >= 0, so
        // the neutral element's sign cannot matter.
        sum = 0.0f;
        for (size_t i = 0; i < cut; i++) sum += cand[i].first;
    }
    float r = rng_next_f32(rng) * sum;
    float acc = 0.0f;
    for (size_t i = 0; i < cut; i++) {
        acc += cand[i].first;
        if (r < acc) return cand[i].second;
    }
    return cand[cut - 1].second;
}

// ------------------------------------------------------------- pool.rs:139-145
inline void split(size_t rows, size_t n, size_t tid, size_t* a, size_t* b) {
    size_t per = rows / n, rem = rows % n;
    size_t start = tid * per + std::min(tid, rem);
    size_t len = per + (tid < rem ? 1 : 0);
    *a = start;
    *b = start + len;
}

// Fixed-range worker pool with a spin barrier (pool.rs:104-128). Work is split
// by `split`, so which thread runs a row never changes a result.
class Pool {
  public:
    explicit Pool(size_t n) : n_(n ? n : 1) {
        for (size_t t = 1; t < n_; t++) th_.emplace_back([this, t] { worker(t); });
    }
    ~Pool() {
        stop_.store(true, std::memory_order_release);
        for (auto& t : th_) t.join();
    }
    size_t threads() const { return n_; }
    void broadcast(const std::function<void(size_t)>& f) {
        if (n_ == 1) {
            f(0);
            return;
        }
        job_ = &f;
        done_.store(0, std::memory_order_relaxed);
        seq_.fetch_add(1, std::memory_order_release);
        f(0);
        size_t spins = 0;
        while (done_.load(std::memory_order_acquire) != n_ - 1)
            if (++spins > 20000) std::this_thread::yield();
    }
    void range(size_t rows, size_t tid, size_t* a, size_t* b) const { split(rows, n_, tid, a, b); }

  private:
    void worker(size_t tid) {
        uint64_t last = 0;
        for (;;) {
            size_t spins = 0;
            while (!stop_.load(std::memory_order_acquire) && seq_.load(std::memory_order_acquire) == last)
                if (++spins > 20000) std::this_thread::yield();
            if (stop_.load(std::memory_order_acquire)) return;
            last = seq_.load(std::memory_order_acquire);
            (*job_)(tid);
            done_.fetch_add(1, std::memory_order_release);
        }
    }
    size_t n_;
    std::vector<std::thread> th_;
    std::atomic<uint64_t> seq_{0};
    std::atomic<size_t> done_{0};
    std::atomic<bool> stop_{false};
    const std::function<void(size_t)>* job_ = nullptr;
};

// ---------------------------------------------------------------- kv.rs:75-104
struct KvSpec {
    uint64_t n_layers, n_kv_heads, head_dim, max_ctx;
    uint32_t layout;
    uint64_t plane() const { return max_ctx * n_kv_heads * head_dim; }
    uint64_t layer_stride() const { return 2 * plane(); }
    uint64_t floats() const { return n_layers * layer_stride(); }
    uint64_t row_off(uint64_t layer, bool is_v, uint64_t pos, uint64_t head) const {
        uint64_t p = layer * layer_stride() + (is_v ? plane() : 0);
        uint64_t within = layout == 0 ? (pos * n_kv_heads + head) * head_dim
                                      : (head * max_ctx + pos) * head_dim;
        return p + within;
    }
};
KvSpec spec_of(const hso_kv_spec* s) {
    return KvSpec{s->n_layers, s->n_kv_heads, s->head_dim, s->max_ctx, s->layout};
}

// ------------------------------------------------------------- kv.rs:150-175
std::vector<std::pair<uint64_t, uint64_t>> live_ranges_between(const KvSpec& s, uint64_t from, uint64_t to) {
    std::vector<std::pair<uint64_t, uint64_t>> out;
    if (to <= from) return out;
    uint64_t n = to - from;
    for (uint64_t layer = 0; layer < s.n_layers; layer++)
        for (int is_v = 0; is_v < 2; is_v++) {
            uint64_t plane_off = (layer * s.layer_stride() + (is_v ? s.plane() : 0)) * 4;
            if (s.layout == 0) {
                uint64_t w = s.n_kv_heads * s.head_dim * 4;
                out.push_back({plane_off + from * w, n * w});
            } else {
                uint64_t w = s.head_dim * 4;
                for (uint64_t h = 0; h < s.n_kv_heads; h++)
                    out.push_back({plane_off + (h * s.max_ctx + from) * w, n * w});
            }
        }
    return out;
}

size_t emit(const std::vector<std::pair<uint64_t, uint64_t>>& v, uint64_t* out, size_t cap) {
    for (size_t i = 0; i < v.size() && i < cap; i++) {
        out[2 * i] = v[i].first;
        out[2 * i + 1] = v[i].second;
    }
    return v.size();
}

// -------------------------------------------------- hs-track pageset.rs:79-113
std::vector<std::pair<uint64_t, uint64_t>> pageset_runs(const uint64_t* words, size_t n_pages) {
    std::vector<std::pair<uint64_t, uint64_t>> out;
    bool have = false;
    uint64_t start = 0;
    size_t n_words = (n_pages + 63) / 64;
    for (size_t i = 0; i < n_words; i++) {
        uint64_t w = words[i];
        if (w == 0) {
            if (have) {
                out.push_back({start, i * 64 - start});
                have = false;
            }
            continue;
        }
        for (size_t b = 0; b < 64; b++) {
            size_t page = i * 64 + b;
            if (page >= n_pages) break;
            bool set = (w & 1) == 1;
            w >>= 1;
            if (set && !have) {
                start = page;
                have = true;
            } else if (!set && have) {
                out.push_back({start, page - start});
                have = false;
            }
        }
    }
    if (have) out.push_back({start, n_pages - start});
    return out;
}

// ---------------------------------------------------- hs-wire lib.rs:418-446
void push_merged(std::vector<std::pair<uint64_t, uint64_t>>& v, uint64_t off, uint64_t len) {
    if (!v.empty()) {
        auto& last = v.back();
        if (last.first + last.second >= off) {
            uint64_t end = std::max(last.first + last.second, off + len);
            last.second = end - last.first;
            return;
        }
    }
    v.push_back({off, len});
}

// --------------------------------------------------------------- GGUF reader
// gguf.rs:154-284, reading the whole file through a read-only mapping.
struct TensorInfo {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t ty;
    size_t off, len;
    size_t elems() const {
        uint64_t e = 1;
        for (auto d : dims) e *= d;
        return (size_t)e;
    }
};

struct Value {
    uint32_t ty = 0;
    uint64_t u = 0;
    double f = 0;
    std::string s;
    uint32_t arr_ty = 0;
    size_t arr_len = 0, arr_off = 0;
};

struct Gguf {
    const uint8_t* b = nullptr;
    size_t n = 0;
    std::map<std::string, Value> meta;
    std::map<std::string, TensorInfo> tensors;
    std::vector<std::string> order;
    ~Gguf() {
        if (b) munmap((void*)b, n);
    }
};

struct Cur {
    const uint8_t* b;
    size_t n, p;
    bool take(size_t k, const uint8_t** out) {
        if (p + k > n) {
            g_err = "file truncated: needed " + std::to_string(p + k) + " bytes, have " + std::to_string(n);
            return false;
        }
        *out = b + p;
        p += k;
        return true;
    }
    bool u32(uint32_t* v) {
        const uint8_t* q;
        if (!take(4, &q)) return false;
        std::memcpy(v, q, 4);
        return true;
    }
    bool u64(uint64_t* v) {
        const uint8_t* q;
        if (!take(8, &q)) return false;
        std::memcpy(v, q, 8);
        return true;
    }
    bool str(std::string* s) {
        uint64_t k;
        const uint8_t* q;
        if (!u64(&k) || !take((size_t)k, &q)) return false;
        s->assign((const char*)q, (size_t)k);
        return true;
    }
};

bool scalar_width(uint32_t ty, size_t* w) {
    switch (ty) {
        case 0: case 1: case 7: *w = 1; return true;
        case 2: case 3: *w = 2; return true;
        case 4: case 5: case 6: *w = 4; return true;
        case 10: case 11: case 12: *w = 8; return true;
        default: g_err = "unknown metadata value type " + std::to_string(ty); return false;
    }
}

bool read_value(Cur& c, uint32_t ty, Value* v) {
    v->ty = ty;
    const uint8_t* q;
    switch (ty) {
        case 0: case 1: case 7:
            if (!c.take(1, &q)) return false;
            v->u = ty == 1 ? (uint64_t)(int64_t)(int8_t)q[0] : q[0];
            return true;
        case 2: case 3:
            if (!c.take(2, &q)) return false;
            v->u = (uint64_t)(q[0] | (q[1] << 8));
            return true;
        case 4: case 5: {
            uint32_t x;
            if (!c.u32(&x)) return false;
            v->u = x;
            return true;
        }
        case 6: {
            uint32_t x;
            if (!c.u32(&x)) return false;
            v->f = (double)u2f(x);
            return true;
        }
        case 8: return c.str(&v->s);
        case 9: {
            uint32_t ety;
            uint64_t len;
            if (!c.u32(&ety) || !c.u64(&len)) return false;
            v->arr_ty = ety;
            v->arr_len = (size_t)len;
            v->arr_off = c.p;
            if (ety == 8) {
                for (uint64_t i = 0; i < len; i++) {
                    uint64_t k;
                    if (!c.u64(&k) || !c.take((size_t)k, &q)) return false;
                }
            } else {
                size_t w;
                if (!scalar_width(ety, &w) || !c.take((size_t)len * w, &q)) return false;
            }
            return true;
        }
        case 10: case 11: return c.u64(&v->u);
        case 12: {
            uint64_t x;
            if (!c.u64(&x)) return false;
            std::memcpy(&v->f, &x, 8);
            return true;
        }
        default: g_err = "unknown metadata value type " + std::to_string(ty); return false;
    }
}

bool gguf_open(const char* path, Gguf* g) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) {
        g_err = std::string("io: cannot open ") + path;
        return false;
    }
    struct stat st;
    fstat(fd, &st);
    g->n = (size_t)st.st_size;
    void* p = mmap(nullptr, g->n ? g->n : 1, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) {
        g_err = "io: mmap failed";
        return false;
    }
    g->b = (const uint8_t*)p;
    Cur c{g->b, g->n, 0};
    uint32_t magic, version;
    if (!c.u32(&magic)) return false;
    if (magic != 0x46554747u) {
        char buf[64];
        snprintf(buf, sizeof buf, "not a GGUF file (magic %#010x)", magic);
        g_err = buf;
        return false;
    }
    if (!c.u32(&version)) return false;
    if (version != 2 && version != 3) {
        g_err = "unsupported GGUF version " + std::to_string(version);
        return false;
    }
    uint64_t n_tensors, n_kv;
    if (!c.u64(&n_tensors) || !c.u64(&n_kv)) return false;
    for (uint64_t i = 0; i < n_kv; i++) {
        std::string key;
        uint32_t ty;
        Value v;
        if (!c.str(&key) || !c.u32(&ty) || !read_value(c, ty, &v)) return false;
        g->meta[key] = v;
    }
    struct Raw { std::string name; std::vector<uint64_t> dims; uint32_t ty; uint64_t off; };
    std::vector<Raw> raw;
    for (uint64_t i = 0; i < n_tensors; i++) {
        Raw r;
        uint32_t nd;
        if (!c.str(&r.name) || !c.u32(&nd)) return false;
        for (uint32_t d = 0; d < nd; d++) {
            uint64_t x;
            if (!c.u64(&x)) return false;
            r.dims.push_back(x);
        }
        if (!c.u32(&r.ty) || !c.u64(&r.off)) return false;
        size_t be, bb;
        if (!block_of(r.ty, &be, &bb)) {
            g_err = "unknown tensor type " + std::to_string(r.ty);
            return false;
        }
        raw.push_back(r);
    }
    size_t align = 32;
    auto it = g->meta.find("general.alignment");
    if (it != g->meta.end() && it->second.ty == 4) align = (size_t)it->second.u;
    size_t data_start = (c.p + align - 1) / align * align;
    for (auto& r : raw) {
        TensorInfo t;
        t.name = r.name;
        t.dims = r.dims;
        t.ty = r.ty;
        size_t be, bb;
        block_of(r.ty, &be, &bb);
        t.len = (t.elems() / be) * bb;
        t.off = data_start + (size_t)r.off;
        if (t.off + t.len > g->n) {
            g_err = "tensor \"" + r.name + "\" runs past end of file";
            return false;
        }
        g->order.push_back(r.name);
        g->tensors[r.name] = t;
    }
    return true;
}

// gguf.rs:298-323
bool get_u32(const Gguf& g, const std::string& k, uint32_t* v) {
    auto it = g.meta.find(k);
    if (it == g.meta.end()) {
        g_err = "missing metadata key \"" + k + "\"";
        return false;
    }
    uint32_t t = it->second.ty;
    if (t == 4 || t == 5 || t == 10) {
        *v = (uint32_t)it->second.u;
        return true;
    }
    g_err = "key \"" + k + "\" is not an integer";
    return false;
}
bool get_f32(const Gguf& g, const std::string& k, float* v) {
    auto it = g.meta.find(k);
    if (it == g.meta.end()) {
        g_err = "missing metadata key \"" + k + "\"";
        return false;
    }
    if (it->second.ty == 6 || it->second.ty == 12) {
        *v = (float)it->second.f;
        return true;
    }
    g_err = "key \"" + k + "\" is not a float";
    return false;
}
bool get_str_array_len(const Gguf& g, const std::string& k, size_t* len) {
    auto it = g.meta.find(k);
    if (it == g.meta.end()) {
        g_err = "missing metadata key \"" + k + "\"";
        return false;
    }
    if (it->second.ty != 9 || it->second.arr_ty != 8) {
        g_err = "key \"" + k + "\" is not a string array";
        return false;
    }
    *len = it->second.arr_len;
    return true;
}

}  // namespace

// -------------------------------------------------------------------- model
struct Layer {
    std::vector<float> attn_norm, bq, bk, bv, ffn_norm;
    std::vector<uint16_t> wq, wk, wv, wo, w_gate, w_up, w_down;
};

struct hso_model {
    hso_config cfg;
    std::vector<uint16_t> embd;
    std::vector<float> out_norm;
    std::vector<uint16_t> out_w;
    bool has_out_w = false;
    std::vector<Layer> layers;
    std::vector<float> rope_cos, rope_sin;
    std::map<std::string, const std::vector<uint16_t>*> f16_by_name;
    std::map<std::string, const std::vector<float>*> f32_by_name;
    Pool* pool = nullptr;
    // model.rs:330-342 Scratch
    std::vector<float> x, xb, xb2, q, k, v, att, scores, hb, hb2, logits;
    ~hso_model() { delete pool; }
};

namespace {

// model.rs:375-396
bool load_f16(const Gguf& g, const std::string& name, Pool& pool, std::vector<uint16_t>* out) {
    auto it = g.tensors.find(name);
    if (it == g.tensors.end()) {
        g_err = "missing tensor \"" + name + "\"";
        return false;
    }
    const TensorInfo& t = it->second;
    size_t n = t.elems();
    out->assign(n, 0);
    size_t be, bb;
    block_of(t.ty, &be, &bb);
    size_t n_blocks = n / be;
    const uint8_t* src = g.b + t.off;
    uint16_t* dst = out->data();
    uint32_t ty = t.ty;
    pool.broadcast([&](size_t tid) {
        size_t b0, b1;
        pool.range(n_blocks, tid, &b0, &b1);
        if (b0 == b1) return;
        dequant_to_f16(ty, src + b0 * bb, (b1 - b0) * be, dst + b0 * be);
    });
    return true;
}

// model.rs:398-413
bool load_f32(const Gguf& g, const std::string& name, std::vector<float>* out) {
    auto it = g.tensors.find(name);
    if (it == g.tensors.end()) {
        g_err = "missing tensor \"" + name + "\"";
        return false;
    }
    const TensorInfo& t = it->second;
    size_t n = t.elems();
    out->assign(n, 0.0f);
    if (t.ty == 0) {
        std::memcpy(out->data(), g.b + t.off, n * 4);
    } else {
        std::vector<uint16_t> h(n);
        dequant_to_f16(t.ty, g.b + t.off, n, h.data());
        for (size_t i = 0; i < n; i++) (*out)[i] = f16_to_f32(h[i]);
    }
    return true;
}

// model.rs:345-361
void matvec(Pool& pool, const uint16_t* w, const float* x, size_t n_in, const float* bias, float* y,
            size_t rows) {
    pool.broadcast([&](size_t tid) {
        size_t a, b;
        pool.range(rows, tid, &a, &b);
        for (size_t r = a; r < b; r++) {
            float v = dot_f16(w + r * n_in, x, n_in);
            if (bias) v += bias[r];
            y[r] = v;
        }
    });
}

// model.rs:365-373
inline void rope_apply(float* v, size_t hd, const float* cos, const float* sin) {
    size_t half = hd / 2;
    for (size_t i = 0; i < half; i++) {
        float c = cos[i], s = sin[i];
        float a = v[i], b = v[i + half];
        v[i] = a * c - b * s;
        v[i + half] = a * s + b * c;
    }
}

// seq.rs:321-330
uint32_t penalised_argmax(const hso_sampler_cfg* cfg, float* logits, size_t n, const uint32_t* hist,
                          size_t n_hist) {
    apply_penalty(cfg, logits, hist, n_hist);
    return argmax(logits, n);
}

}  // namespace

extern "C" {

float hso_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
uint16_t hso_f32_to_f16(float f) { return f32_to_f16(f); }
float hso_exp_f32(float x) { return exp_f32(x); }
float hso_ln_f32(float x) { return ln_f32(x); }
void hso_sincos_f32(float x, float* s, float* c) { sincos_f32(x, s, c); }
float hso_silu(float x) { return silu(x); }
float hso_dot_f16(const uint16_t* w, const float* x, size_t n) { return dot_f16(w, x, n); }
float hso_dot_f32(const float* a, const float* b, size_t n) { return dot_f32(a, b, n); }
void hso_rmsnorm(float* out, const float* x, const float* g, size_t n, float eps) { rmsnorm(out, x, g, n, eps); }
void hso_softmax(float* x, size_t n) { softmax(x, n); }
// examples/ppl.rs:35-43: the negative log-likelihood of `next` under the
// logits, max-shifted: max by f32::max from -inf, then the exponentials
// (exp_f32 of the f32 difference) summed in f64 in order, natural log in f64.
double hso_nll(const float* logits, size_t n, uint32_t next) {
    float mx = -INFINITY;
    for (size_t i = 0; i < n; i++) mx = std::fmax(mx, logits[i]);
    double sum = 0.0;
    for (size_t i = 0; i < n; i++) sum += (double)exp_f32(logits[i] - mx);
    return -((double)(logits[next] - mx) - std::log(sum));
}
int hso_dequant_f16(uint32_t ty, const uint8_t* src, size_t n, uint16_t* dst) {
    return dequant_to_f16(ty, src, n, dst);
}
uint32_t hso_scale_min_k4(uint32_t j, const uint8_t* q12) {
    uint8_t sc, m;
    scale_min_k4(j, q12, &sc, &m);
    return ((uint32_t)sc << 8) | m;
}
uint64_t hso_fnv1a(const uint8_t* p, size_t n) {
    Fnv f;
    f.write(p, n);
    return f.h;
}
uint64_t hso_wide(const uint8_t* p, size_t n) {
    Wide w;
    w.write(p, n);
    return w.finish();
}

// sampler.rs:22-33
void hso_sampler_cfg_default(hso_sampler_cfg* c) {
    c->temperature = 0.8f;
    c->top_p = 0.95f;
    c->top_k = 40;
    c->repeat_penalty = 1.1f;
    c->repeat_last_n = 64;
    c->seed = 0xC0FFEE0012345678ull;
}
void hso_rng_seed(uint64_t seed, hso_rng* r) { rng_seed(seed, r); }
uint64_t hso_rng_next_u64(hso_rng* r) { return rng_next_u64(r); }
float hso_rng_next_f32(hso_rng* r) { return rng_next_f32(r); }
uint32_t hso_sample(const hso_sampler_cfg* cfg, hso_rng* rng, float* logits, size_t n, const uint32_t* hist,
                    size_t n_hist) {
    return sample(cfg, rng, logits, n, hist, n_hist);
}
uint32_t hso_argmax(const float* l, size_t n) { return argmax(l, n); }
uint32_t hso_penalised_argmax(const hso_sampler_cfg* cfg, float* logits, size_t n, const uint32_t* hist,
                              size_t n_hist) {
    return penalised_argmax(cfg, logits, n, hist, n_hist);
}
void hso_split(size_t rows, size_t n, size_t tid, size_t* a, size_t* b) { split(rows, n, tid, a, b); }

uint64_t hso_kv_row_off(const hso_kv_spec* s, uint64_t layer, int is_v, uint64_t pos, uint64_t head) {
    return spec_of(s).row_off(layer, is_v != 0, pos, head);
}

// kv.rs:110-131
size_t hso_kv_written_ranges(const hso_kv_spec* s, uint64_t pos, uint64_t* out, size_t cap) {
    KvSpec k = spec_of(s);
    std::vector<std::pair<uint64_t, uint64_t>> v;
    for (uint64_t layer = 0; layer < k.n_layers; layer++)
        for (int is_v = 0; is_v < 2; is_v++) {
            if (k.layout == 0) {
                v.push_back({k.row_off(layer, is_v, pos, 0) * 4, k.n_kv_heads * k.head_dim * 4});
            } else {
                for (uint64_t h = 0; h < k.n_kv_heads; h++)
                    v.push_back({k.row_off(layer, is_v, pos, h) * 4, k.head_dim * 4});
            }
        }
    return emit(v, out, cap);
}
size_t hso_kv_live_ranges_between(const hso_kv_spec* s, uint64_t from, uint64_t to, uint64_t* out, size_t cap) {
    return emit(live_ranges_between(spec_of(s), from, to), out, cap);
}
// kv.rs:267-274
uint64_t hso_kv_hash(const hso_kv_spec* s, const void* base, uint64_t n_pos) {
    Wide h;
    for (auto& r : live_ranges_between(spec_of(s), 0, n_pos)) h.write((const uint8_t*)base + r.first, r.second);
    return h.finish();
}
size_t hso_pageset_runs(const uint64_t* words, size_t n_pages, uint64_t* out, size_t cap) {
    return emit(pageset_runs(words, n_pages), out, cap);
}
// hs-wire lib.rs:418-435
size_t hso_runs_to_byte_runs(const uint64_t* words, size_t n_pages, uint64_t page_size, const uint64_t* live,
                             size_t n_live, uint64_t* out, size_t cap) {
    std::vector<std::pair<uint64_t, uint64_t>> acc;
    for (auto& run : pageset_runs(words, n_pages)) {
        uint64_t a = run.first * page_size, b = (run.first + run.second) * page_size;
        for (size_t i = 0; i < n_live; i++) {
            uint64_t lo = live[2 * i], llen = live[2 * i + 1];
            uint64_t c = std::max(a, lo), d = std::min(b, lo + llen);
            if (c < d) push_merged(acc, c, d - c);
        }
    }
    std::stable_sort(acc.begin(), acc.end(),
                     [](const std::pair<uint64_t, uint64_t>& x, const std::pair<uint64_t, uint64_t>& y) {
                         return x.first < y.first;
                     });
    std::vector<std::pair<uint64_t, uint64_t>> merged;
    for (auto& r : acc) push_merged(merged, r.first, r.second);
    return emit(merged, out, cap);
}

const char* hso_last_error(void) { return g_err.c_str(); }

// model.rs:110-215
int hso_model_load(const char* path, uint64_t max_ctx, uint32_t threads, hso_model** out) {
    Gguf g;
    if (!gguf_open(path, &g)) return -1;
    auto ait = g.meta.find("general.architecture");
    if (ait == g.meta.end()) {
        g_err = "missing metadata key \"general.architecture\"";
        return -1;
    }
    if (ait->second.ty != 8) {
        g_err = "key \"general.architecture\" is not a string";
        return -1;
    }
    std::string arch = ait->second.s;
    if (arch != "qwen2") {
        g_err = "general.architecture = \"" + arch + "\"; only qwen2 is implemented";
        return -1;
    }
    auto k = [&](const char* s) { return arch + "." + s; };
    uint32_t n_layers, d_model, d_ff, n_heads, n_kv_heads, train_ctx;
    float eps, rope_base;
    if (!get_u32(g, k("block_count"), &n_layers) || !get_u32(g, k("embedding_length"), &d_model) ||
        !get_u32(g, k("feed_forward_length"), &d_ff) || !get_u32(g, k("attention.head_count"), &n_heads) ||
        !get_u32(g, k("attention.head_count_kv"), &n_kv_heads) ||
        !get_f32(g, k("attention.layer_norm_rms_epsilon"), &eps))
        return -1;
    if (!get_f32(g, k("rope.freq_base"), &rope_base)) rope_base = 10000.0f;
    if (!get_u32(g, k("context_length"), &train_ctx)) return -1;
    // tok.rs:54-82: tokens and merges must be string arrays; eos must exist.
    size_t vocab, n_merges;
    uint32_t eos;
    if (!get_str_array_len(g, "tokenizer.ggml.tokens", &vocab)) return -1;
    if (!get_str_array_len(g, "tokenizer.ggml.merges", &n_merges)) return -1;
    if (!get_u32(g, "tokenizer.ggml.eos_token_id", &eos)) return -1;

    hso_model* m = new hso_model();
    m->pool = new Pool(threads ? threads : 1);
    hso_config& c = m->cfg;
    c.n_layers = n_layers;
    c.n_heads = n_heads;
    c.n_kv_heads = n_kv_heads;
    c.head_dim = d_model / n_heads;
    c.d_model = d_model;
    c.d_ff = d_ff;
    c.vocab = vocab;
    c.eps = eps;
    c.rope_base = rope_base;
    c.train_ctx = train_ctx;
    c.eos = eos;
    c.max_ctx = max_ctx;

    // model.rs:147-156
    Fnv fp;
    fp.write_u64((uint64_t)g.n);
    for (auto& name : g.order) {
        const TensorInfo& t = g.tensors[name];
        fp.write((const uint8_t*)name.data(), name.size());
        fp.write_u32(enum_index(t.ty));
        fp.write_u64((uint64_t)t.off);
        fp.write_u64((uint64_t)t.len);
    }
    c.fingerprint = fp.h;

    Pool& pool = *m->pool;
    bool ok = load_f16(g, "token_embd.weight", pool, &m->embd) && load_f32(g, "output_norm.weight", &m->out_norm);
    if (ok && g.tensors.count("output.weight")) {
        m->has_out_w = true;
        ok = load_f16(g, "output.weight", pool, &m->out_w);
    }
    m->layers.resize(n_layers);
    for (uint32_t i = 0; ok && i < n_layers; i++) {
        auto b = [&](const char* s) { return "blk." + std::to_string(i) + "." + s; };
        Layer& L = m->layers[i];
        ok = load_f32(g, b("attn_norm.weight"), &L.attn_norm) && load_f16(g, b("attn_q.weight"), pool, &L.wq) &&
             load_f32(g, b("attn_q.bias"), &L.bq) && load_f16(g, b("attn_k.weight"), pool, &L.wk) &&
             load_f32(g, b("attn_k.bias"), &L.bk) && load_f16(g, b("attn_v.weight"), pool, &L.wv) &&
             load_f32(g, b("attn_v.bias"), &L.bv) && load_f16(g, b("attn_output.weight"), pool, &L.wo) &&
             load_f32(g, b("ffn_norm.weight"), &L.ffn_norm) && load_f16(g, b("ffn_gate.weight"), pool, &L.w_gate) &&
             load_f16(g, b("ffn_up.weight"), pool, &L.w_up) && load_f16(g, b("ffn_down.weight"), pool, &L.w_down);
        if (ok) {
            std::string p = "blk." + std::to_string(i) + ".";
            m->f16_by_name[p + "attn_q.weight"] = &L.wq;
            m->f16_by_name[p + "attn_k.weight"] = &L.wk;
            m->f16_by_name[p + "attn_v.weight"] = &L.wv;
            m->f16_by_name[p + "attn_output.weight"] = &L.wo;
            m->f16_by_name[p + "ffn_gate.weight"] = &L.w_gate;
            m->f16_by_name[p + "ffn_up.weight"] = &L.w_up;
            m->f16_by_name[p + "ffn_down.weight"] = &L.w_down;
            m->f32_by_name[p + "attn_norm.weight"] = &L.attn_norm;
            m->f32_by_name[p + "attn_q.bias"] = &L.bq;
            m->f32_by_name[p + "attn_k.bias"] = &L.bk;
            m->f32_by_name[p + "attn_v.bias"] = &L.bv;
            m->f32_by_name[p + "ffn_norm.weight"] = &L.ffn_norm;
        }
    }
    if (!ok) {
        delete m;
        return -1;
    }
    m->f16_by_name["token_embd.weight"] = &m->embd;
    if (m->has_out_w) m->f16_by_name["output.weight"] = &m->out_w;
    m->f32_by_name["output_norm.weight"] = &m->out_norm;

    // model.rs:190-201
    size_t hd = c.head_dim, half = hd / 2;
    m->rope_cos.assign(max_ctx * half, 0.0f);
    m->rope_sin.assign(max_ctx * half, 0.0f);
    float ln_base = ln_f32(rope_base);
    for (size_t i = 0; i < half; i++) {
        float inv_freq = exp_f32(-(2.0f * (float)i / (float)hd) * ln_base);
        for (size_t p = 0; p < max_ctx; p++) {
            float s, co;
            sincos_f32((float)p * inv_freq, &s, &co);
            m->rope_cos[p * half + i] = co;
            m->rope_sin[p * half + i] = s;
        }
    }
    // model.rs:221-236
    m->x.assign(d_model, 0);
    m->xb.assign(d_model, 0);
    m->xb2.assign(d_model, 0);
    m->q.assign(n_heads * hd, 0);
    m->k.assign(n_kv_heads * hd, 0);
    m->v.assign(n_kv_heads * hd, 0);
    m->att.assign(n_heads * hd, 0);
    m->scores.assign(n_heads * max_ctx, 0);
    m->hb.assign(d_ff, 0);
    m->hb2.assign(d_ff, 0);
    m->logits.assign(vocab, 0);
    *out = m;
    return 0;
}

void hso_model_free(hso_model* m) { delete m; }
void hso_model_config(const hso_model* m, hso_config* out) { *out = m->cfg; }
const uint16_t* hso_model_tensor_f16(const hso_model* m, const char* name, size_t* n) {
    auto it = m->f16_by_name.find(name);
    if (it == m->f16_by_name.end()) return nullptr;
    *n = it->second->size();
    return it->second->data();
}
const float* hso_model_tensor_f32(const hso_model* m, const char* name, size_t* n) {
    auto it = m->f32_by_name.find(name);
    if (it == m->f32_by_name.end()) return nullptr;
    *n = it->second->size();
    return it->second->data();
}
const float* hso_model_rope_cos(const hso_model* m) { return m->rope_cos.data(); }
const float* hso_model_rope_sin(const hso_model* m) { return m->rope_sin.data(); }

// model.rs:240-327
int hso_forward(hso_model* m, float* kvp, uint32_t layout, uint32_t token, uint64_t pos, float* logits,
                float* trace) {
    const hso_config& c = m->cfg;
    if (pos >= c.max_ctx) {
        g_err = "position " + std::to_string(pos) + " past max_ctx " + std::to_string(c.max_ctx);
        return -2;
    }
    if (token >= c.vocab) {
        g_err = "token " + std::to_string(token) + " out of range";
        return -2;
    }
    Pool& pool = *m->pool;
    KvSpec ks{c.n_layers, c.n_kv_heads, c.head_dim, c.max_ctx, layout};
    size_t hd = c.head_dim, half = hd / 2, d = c.d_model;
    size_t row = (size_t)token * d;
    for (size_t i = 0; i < d; i++) m->x[i] = f16_to_f32(m->embd[row + i]);

    for (size_t l = 0; l < c.n_layers; l++) {
        const Layer& L = m->layers[l];
        rmsnorm(m->xb.data(), m->x.data(), L.attn_norm.data(), d, c.eps);
        matvec(pool, L.wq.data(), m->xb.data(), d, L.bq.data(), m->q.data(), c.n_heads * hd);
        matvec(pool, L.wk.data(), m->xb.data(), d, L.bk.data(), m->k.data(), c.n_kv_heads * hd);
        matvec(pool, L.wv.data(), m->xb.data(), d, L.bv.data(), m->v.data(), c.n_kv_heads * hd);
        const float* cs = m->rope_cos.data() + pos * half;
        const float* sn = m->rope_sin.data() + pos * half;
        for (size_t h = 0; h < c.n_heads; h++) rope_apply(m->q.data() + h * hd, hd, cs, sn);
        for (size_t h = 0; h < c.n_kv_heads; h++) rope_apply(m->k.data() + h * hd, hd, cs, sn);
        for (size_t h = 0; h < c.n_kv_heads; h++) {
            std::memcpy(kvp + ks.row_off(l, false, pos, h), m->k.data() + h * hd, hd * 4);
            std::memcpy(kvp + ks.row_off(l, true, pos, h), m->v.data() + h * hd, hd * 4);
        }
        float scale = 1.0f / sqrtf((float)hd);
        size_t groups = c.n_heads / c.n_kv_heads;
        size_t max_ctx = c.max_ctx;
        pool.broadcast([&](size_t tid) {
            size_t h0, h1;
            pool.range(c.n_heads, tid, &h0, &h1);
            for (size_t h = h0; h < h1; h++) {
                size_t kvh = h / groups;
                const float* q = m->q.data() + h * hd;
                float* sc = m->scores.data() + h * max_ctx;
                float* out = m->att.data() + h * hd;
                for (size_t p = 0; p <= pos; p++) sc[p] = dot_f32(q, kvp + ks.row_off(l, false, p, kvh), hd) * scale;
                softmax(sc, pos + 1);
                for (size_t i = 0; i < hd; i++) out[i] = 0.0f;
                for (size_t p = 0; p <= pos; p++) axpy(out, kvp + ks.row_off(l, true, p, kvh), sc[p], hd);
            }
        });
        matvec(pool, L.wo.data(), m->att.data(), c.n_heads * hd, nullptr, m->xb2.data(), d);
        for (size_t i = 0; i < d; i++) m->x[i] += m->xb2[i];
        rmsnorm(m->xb.data(), m->x.data(), L.ffn_norm.data(), d, c.eps);
        matvec(pool, L.w_gate.data(), m->xb.data(), d, nullptr, m->hb.data(), c.d_ff);
        matvec(pool, L.w_up.data(), m->xb.data(), d, nullptr, m->hb2.data(), c.d_ff);
        for (size_t i = 0; i < c.d_ff; i++) m->hb[i] = silu(m->hb[i]) * m->hb2[i];
        matvec(pool, L.w_down.data(), m->hb.data(), c.d_ff, nullptr, m->xb2.data(), d);
        for (size_t i = 0; i < d; i++) m->x[i] += m->xb2[i];
        if (trace) std::memcpy(trace + l * d, m->x.data(), d * 4);
    }
    rmsnorm(m->xb.data(), m->x.data(), m->out_norm.data(), d, c.eps);
    const uint16_t* head = m->has_out_w ? m->out_w.data() : m->embd.data();
    matvec(pool, head, m->xb.data(), d, nullptr, m->logits.data(), c.vocab);
    if (logits) std::memcpy(logits, m->logits.data(), c.vocab * 4);
    return 0;
}

// seq.rs:230-318 (one sequence, no pause/migration plumbing: a caller that wants
// to hand the sequence over stops at `stop_at_filled` and resumes elsewhere).
int hso_seq_run(hso_model* m, float* kv, uint32_t layout, uint32_t* tokens, uint64_t* n_tokens, uint64_t cap,
                hso_seq_state* st, const hso_sampler_cfg* cfg, hso_rng* rng, uint64_t stop_at_filled) {
    const hso_config& c = m->cfg;
    while (!st->done) {
        if (stop_at_filled && st->filled >= stop_at_filled) return 0;
        if (st->filled >= *n_tokens) {
            g_err = "internal: nothing to feed at the token boundary";
            return -3;
        }
        int rc = hso_forward(m, kv, layout, tokens[st->filled], st->filled, nullptr, nullptr);
        if (rc) return rc;
        st->filled += 1;
        if (st->filled == *n_tokens) {
            std::vector<float> l(m->logits);
            uint32_t next;
            if (cfg->temperature <= 0.0f)
                next = penalised_argmax(cfg, l.data(), c.vocab, tokens, *n_tokens);
            else
                next = sample(cfg, rng, l.data(), c.vocab, tokens, *n_tokens);
            uint64_t generated = *n_tokens - st->prompt_len;
            if (next == c.eos) {
                st->done = 1;
                st->done_reason = 1;
            } else if (generated >= st->max_tokens) {
                st->done = 1;
                st->done_reason = 2;
            } else if (*n_tokens + 1 >= c.max_ctx) {
                st->done = 1;
                st->done_reason = 3;
            } else {
                if (*n_tokens >= cap) {
                    g_err = "token buffer full";
                    return -4;
                }
                tokens[(*n_tokens)++] = next;
            }
        }
    }
    return 0;
}

}  // extern "C"
