// Host-side RoPE tables, computed once at load exactly as hotseat's
// Model::load does (model.rs:187-201), with the reference's own libm-free
// exp/ln/sincos (math.rs:39-61, 250-294). This file must be compiled with
// -ffp-contract=off: every operation is a separately rounded IEEE f32 (or
// f64, for the sincos argument reduction) operation, as in the Rust source.
#include <cmath>
#include <cstdint>
#include <vector>

#include "common.h"

namespace hs {
namespace {

// math.rs:27-30
const float kLog2E = 1.44269504f;
const float kLn2Hi = 0.693359375f;
const float kLn2Lo = -2.1219444e-4f;

// 2^k from the exponent field (math.rs:65-75).
float exp2i(int32_t k) {
    int32_t e = k + 127;
    if (e <= 0) return e <= -23 ? 0.0f : u2f(1u << (22 + e));
    return u2f((uint32_t)e << 23);
}

}  // namespace

// math.rs:39-61
float ref_exp(float x) {
    if (std::isnan(x)) return x;
    if (x >= 89.0f) return INFINITY;
    if (x <= -104.0f) return 0.0f;
    float kf = std::round(x * kLog2E);
    float r = x - kf * kLn2Hi - kf * kLn2Lo;
    float p = 1.0f + r * (1.0f + r * (0.5f + r * (0.16666667f + r * (0.04166667f + r * (0.00833333f + r * 0.001388889f)))));
    int32_t k = (int32_t)kf;
    int32_t k1 = k >> 1;
    return p * exp2i(k1) * exp2i(k - k1);
}

// math.rs:250-264
float ref_ln(float x) {
    uint32_t bits = f2u(x);
    int32_t e = (int32_t)((bits >> 23) & 0xff) - 127;
    float m = u2f((bits & 0x007fffffu) | (127u << 23));
    if (m > 1.4142136f) {
        m *= 0.5f;
        e += 1;
    }
    float s = (m - 1.0f) / (m + 1.0f);
    float s2 = s * s;
    float p = s * (2.0f + s2 * (0.6666667f + s2 * (0.4f + s2 * (0.2857143f + s2 * 0.2222222f))));
    return p + (float)e * (kLn2Hi + kLn2Lo);
}

// math.rs:272-294: quadrant from the f32 constant pi/2 widened to f64,
// remainder against the f64 constant, polynomials in f32.
void ref_sincos(float x, float* sn, float* cs) {
    const float kHalfPiF = 1.57079632679489661923f;
    const double kHalfPiD = 1.57079632679489661923;
    double q = std::round((double)x / (double)kHalfPiF);
    float r = (float)((double)x - q * kHalfPiD);
    float r2 = r * r;
    float s = r * (1.0f + r2 * (-0.16666667f + r2 * (0.00833333f + r2 * (-1.984127e-4f + r2 * 2.755732e-6f))));
    float c = 1.0f + r2 * (-0.5f + r2 * (0.04166667f + r2 * (-0.001388889f + r2 * 2.480159e-5f)));
    int64_t quad = (((int64_t)q % 4) + 4) % 4;
    switch (quad) {
        case 0: *sn = s; *cs = c; break;
        case 1: *sn = c; *cs = -s; break;
        case 2: *sn = -s; *cs = -c; break;
        default: *sn = -c; *cs = s; break;
    }
}

// model.rs:190-201: cos/sin[p * half + i] for p < max_ctx, i < head_dim/2.
void rope_tables(uint32_t head_dim, uint32_t max_ctx, float rope_base, std::vector<float>* cos_t,
                 std::vector<float>* sin_t) {
    uint32_t half = head_dim / 2;
    cos_t->assign((size_t)max_ctx * half, 0.0f);
    sin_t->assign((size_t)max_ctx * half, 0.0f);
    float ln_base = ref_ln(rope_base);
    for (uint32_t i = 0; i < half; i++) {
        float inv_freq = ref_exp(-(2.0f * (float)i / (float)head_dim) * ln_base);
        for (uint32_t p = 0; p < max_ctx; p++) {
            float s, c;
            ref_sincos((float)p * inv_freq, &s, &c);
            (*cos_t)[(size_t)p * half + i] = c;
            (*sin_t)[(size_t)p * half + i] = s;
        }
    }
}

}  // namespace hs
