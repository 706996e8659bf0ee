// Seeded synthetic Qwen2 GGUF writer (test fixture generator; not part of
// the product library).
//
// Writes a GGUF v3 file with the metadata keys, tokenizer keys and tensor
// names hotseat's Model::load reads (model.rs:110-185, tok.rs:54-82), with
// weights drawn N(0, weight_std), biases N(0, bias_std) and norm gains 1.0.
// 2-D weights are quantised as flat streams of blocks that may straddle rows,
// which is how the reference dequantises them (model.rs:375-396) — 896-wide
// rows are 3.5 Q4_K blocks. Any valid encoding is acceptable: the contract
// between the CPU reference and the GPU is defined on the dequantised values.
//
// Every random value is a pure function of (seed, tensor name, element
// index), so the file is identical for any thread count.
//
// Built by tests/golden/synth.py into tests/golden/_build/libhs_synth.so; the
// tests, the benchmark and the microbenchmarks write their model files with
// it, so a process that only times the CPU restatement maps no product code.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

extern "C" {
typedef struct {
    uint32_t n_layers, d_model, n_heads, n_kv_heads, d_ff, vocab, context_length, eos;
    float eps, rope_base, weight_std, bias_std;
    uint32_t embd_type;   /* ggml type of token_embd.weight (14 = Q6_K) */
    uint32_t weight_type; /* ggml type of the other 2-D weights (12 = Q4_K) */
    uint32_t tied;        /* 1: no output.weight (tied LM head) */
    uint32_t threads;
    uint64_t seed;
} hs_synth_spec;
}

// Status codes: the same values as the library's HS_OK / HS_E_*.
#define SYN_OK 0
#define SYN_E_ARG (-1)
#define SYN_E_IO (-2)
#define SYN_E_UNSUPPORTED (-6)

namespace synth {
namespace {

thread_local std::string g_err;
int fail(int code, const std::string& msg) {
    g_err = msg;
    return code;
}

uint32_t f2u(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
float u2f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

// IEEE binary16 -> binary32, exact.
float h2f_host(uint16_t h) {
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

// ggml type -> (elements per block, bytes per block) for the encodable types.
bool ggml_block(uint32_t ty, uint64_t* be, uint64_t* bb) {
    switch (ty) {
        case 0: *be = 1; *bb = 4; return true;
        case 1: *be = 1; *bb = 2; return true;
        case 8: *be = 32; *bb = 34; return true;
        case 12: *be = 256; *bb = 144; return true;
        case 14: *be = 256; *bb = 210; return true;
        default: return false;
    }
}

uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t name_seed(uint64_t seed, const std::string& name) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (unsigned char c : name) h = (h ^ c) * 0x100000001b3ull;
    return mix64(seed ^ h);
}

// Element i of a tensor's N(0, std) stream (Box-Muller on a pair of
// counter-based uniforms; element 2k and 2k+1 share a pair).
float normal_at(uint64_t tseed, uint64_t i, float stdv) {
    uint64_t k = i >> 1;
    double u1 = ((double)(mix64(tseed + 2 * k) >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    double u2 = (double)(mix64(tseed + 2 * k + 1) >> 11) * (1.0 / 9007199254740992.0);
    double r = std::sqrt(-2.0 * std::log(u1));
    double t = 6.283185307179586 * u2;
    return (float)((i & 1) ? r * std::sin(t) : r * std::cos(t)) * stdv;
}

// binary32 -> binary16, round to nearest even (normals, subnormals, overflow).
uint16_t f2h(float f) {
    uint32_t x = f2u(f);
    uint32_t sign = (x >> 16) & 0x8000;
    int32_t e = (int32_t)((x >> 23) & 0xff) - 112;
    uint32_t m = x & 0x7fffff;
    if (((x >> 23) & 0xff) == 0xff) return (uint16_t)(sign | 0x7c00 | (m ? 0x200 : 0));
    if (e >= 31) return (uint16_t)(sign | 0x7c00);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        m |= 0x800000;
        uint32_t sh = (uint32_t)(14 - e);
        uint32_t h = m >> sh, rem = m & ((1u << sh) - 1), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (h & 1))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (m >> 13), rem = m & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
    return (uint16_t)(sign | h);
}

void put16(uint8_t* p, uint16_t v) {
    p[0] = (uint8_t)v;
    p[1] = (uint8_t)(v >> 8);
}

int iround(float v) { return (int)std::lround(v); }
int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// One Q4_K super-block: 8 sub-blocks of 32, x ~ d*sc*q - dmin*m (the form
// quant.rs:109-139 decodes), scales/mins packed as scale_min_k4 unpacks them.
void quant_q4_k(const float* x, uint8_t* out) {
    float scale[8], mins[8];
    for (int j = 0; j < 8; j++) {
        float lo = 0.0f, hi = -INFINITY;
        for (int l = 0; l < 32; l++) {
            lo = std::min(lo, x[32 * j + l]);
            hi = std::max(hi, x[32 * j + l]);
        }
        scale[j] = (hi - lo) / 15.0f;
        mins[j] = -lo;
    }
    float ms = *std::max_element(scale, scale + 8), mm = *std::max_element(mins, mins + 8);
    uint16_t dh = f2h(ms / 63.0f), mh = f2h(mm / 63.0f);
    float d = h2f_host(dh), dmin = h2f_host(mh);
    int sc[8], mn[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = d > 0 ? clampi(iround(scale[j] / d), 0, 63) : 0;
        mn[j] = dmin > 0 ? clampi(iround(mins[j] / dmin), 0, 63) : 0;
    }
    put16(out, dh);
    put16(out + 2, mh);
    uint8_t* s = out + 4;
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
    }
    uint8_t q[256];
    for (int j = 0; j < 8; j++) {
        float D = d * (float)sc[j], M = dmin * (float)mn[j];
        for (int l = 0; l < 32; l++) q[32 * j + l] = (uint8_t)(D > 0 ? clampi(iround((x[32 * j + l] + M) / D), 0, 15) : 0);
    }
    uint8_t* qs = out + 16;
    for (int g = 0; g < 4; g++)
        for (int l = 0; l < 32; l++) qs[32 * g + l] = (uint8_t)(q[64 * g + l] | (q[64 * g + 32 + l] << 4));
}

// One Q6_K super-block: 16 sub-blocks of 16, x ~ d*sc*(q-32) with int8
// scales (the form quant.rs:178-206 decodes).
void quant_q6_k(const float* x, uint8_t* out) {
    float scale[16];
    for (int s = 0; s < 16; s++) {
        float a = 0.0f;
        for (int l = 0; l < 16; l++) a = std::max(a, std::fabs(x[16 * s + l]));
        scale[s] = a / 31.0f;
    }
    uint16_t dh = f2h(*std::max_element(scale, scale + 16) / 127.0f);
    float d = h2f_host(dh);
    int sc[16];
    for (int s = 0; s < 16; s++) sc[s] = d > 0 ? clampi(iround(scale[s] / d), 0, 127) : 0;
    std::memset(out, 0, 210);
    uint8_t *ql = out, *qh = out + 128;
    for (int e = 0; e < 256; e++) {
        int s = e / 16;
        float D = d * (float)sc[s];
        int q = D > 0 ? clampi(iround(x[e] / D) + 32, 0, 63) : 32;
        int h = e / 128, c = (e % 128) / 32, l = e % 32;
        uint8_t* lo = ql + h * 64 + l + 32 * (c & 1);
        *lo |= (uint8_t)((q & 15) << (4 * (c >> 1)));
        qh[h * 32 + l] |= (uint8_t)(((q >> 4) & 3) << (2 * c));
    }
    for (int s = 0; s < 16; s++) out[192 + s] = (uint8_t)(int8_t)sc[s];
    put16(out + 208, dh);
}

// One Q8_0 block of 32 (quant.rs:64-74 decodes d*q).
void quant_q8_0(const float* x, uint8_t* out) {
    float a = 0.0f;
    for (int l = 0; l < 32; l++) a = std::max(a, std::fabs(x[l]));
    uint16_t dh = f2h(a / 127.0f);
    float d = h2f_host(dh);
    put16(out, dh);
    for (int l = 0; l < 32; l++) out[2 + l] = (uint8_t)(int8_t)(d > 0 ? clampi(iround(x[l] / d), -127, 127) : 0);
}

struct Tensor {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type;
    int kind;  // 0 = weight, 1 = bias, 2 = norm gain
    uint64_t rel_off = 0, bytes = 0;
};

uint64_t elems_of(const Tensor& t) {
    uint64_t e = 1;
    for (auto d : t.dims) e *= d;
    return e;
}

// Encode one tensor into `out` using `threads` workers over whole blocks.
void encode(const hs_synth_spec& sp, const Tensor& t, std::vector<uint8_t>& out) {
    uint64_t n = elems_of(t), be, bb;
    ggml_block(t.type, &be, &bb);
    uint64_t nb = n / be;
    out.assign(nb * bb, 0);
    uint64_t tseed = name_seed(sp.seed, t.name);
    float stdv = t.kind == 0 ? sp.weight_std : sp.bias_std;
    unsigned nt = std::max(1u, sp.threads);
    std::vector<std::thread> th;
    for (unsigned w = 0; w < nt; w++) {
        th.emplace_back([&, w] {
            std::vector<float> buf(be);
            for (uint64_t b = w; b < nb; b += nt) {
                for (uint64_t i = 0; i < be; i++)
                    buf[i] = t.kind == 2 ? 1.0f : normal_at(tseed, b * be + i, stdv);
                uint8_t* o = out.data() + b * bb;
                switch (t.type) {
                    case 0: std::memcpy(o, buf.data(), 4); break;
                    case 1: put16(o, f2h(buf[0])); break;
                    case 8: quant_q8_0(buf.data(), o); break;
                    case 12: quant_q4_k(buf.data(), o); break;
                    case 14: quant_q6_k(buf.data(), o); break;
                }
            }
        });
    }
    for (auto& x : th) x.join();
}

class Out {
  public:
    explicit Out(FILE* f) : f_(f) {}
    void bytes(const void* p, size_t n) { ok_ = ok_ && fwrite(p, 1, n, f_) == n; n_ += n; }
    void u32(uint32_t v) { bytes(&v, 4); }
    void u64(uint64_t v) { bytes(&v, 8); }
    void f32(float v) { bytes(&v, 4); }
    void str(const std::string& s) { u64(s.size()); bytes(s.data(), s.size()); }
    void kv_u32(const std::string& k, uint32_t v) { str(k); u32(4); u32(v); }
    void kv_f32(const std::string& k, float v) { str(k); u32(6); f32(v); }
    void kv_str(const std::string& k, const std::string& v) { str(k); u32(8); str(v); }
    void pad(uint64_t align) {
        static const uint8_t z[64] = {0};
        while (n_ % align) bytes(z, std::min<uint64_t>(align - n_ % align, 64));
    }
    bool ok() const { return ok_; }

  private:
    FILE* f_;
    uint64_t n_ = 0;
    bool ok_ = true;
};

}  // namespace
}  // namespace synth

extern "C" const char* hs_synth_last_error() { return synth::g_err.c_str(); }

extern "C" int hs_synth_write(const char* path, const hs_synth_spec* spec) {
    using namespace synth;
    if (!path || !spec) return fail(SYN_E_ARG, "null argument");
    const hs_synth_spec& sp = *spec;
    uint64_t be, bb;
    for (uint32_t ty : {sp.embd_type, sp.weight_type})
        if (!(ty == 0 || ty == 1 || ty == 8 || ty == 12 || ty == 14))
            return fail(SYN_E_UNSUPPORTED, "synthetic writer encodes F32, F16, Q8_0, Q4_K, Q6_K only");
    if (!sp.n_layers || !sp.d_model || !sp.n_heads || !sp.n_kv_heads || !sp.d_ff || !sp.vocab ||
        sp.d_model % sp.n_heads || sp.n_heads % sp.n_kv_heads)
        return fail(SYN_E_ARG, "inconsistent model shape");
    uint32_t hd = sp.d_model / sp.n_heads;
    std::vector<Tensor> ts;
    auto w2 = [&](const std::string& n, uint64_t cols, uint64_t rows, uint32_t ty) {
        ts.push_back(Tensor{n, {cols, rows}, ty, 0});
    };
    auto v1 = [&](const std::string& n, uint64_t len, int kind) { ts.push_back(Tensor{n, {len}, 0u, kind}); };
    w2("token_embd.weight", sp.d_model, sp.vocab, sp.embd_type);
    v1("output_norm.weight", sp.d_model, 2);
    if (!sp.tied) w2("output.weight", sp.d_model, sp.vocab, sp.weight_type);
    for (uint32_t i = 0; i < sp.n_layers; i++) {
        std::string p = "blk." + std::to_string(i) + ".";
        v1(p + "attn_norm.weight", sp.d_model, 2);
        w2(p + "attn_q.weight", sp.d_model, (uint64_t)sp.n_heads * hd, sp.weight_type);
        v1(p + "attn_q.bias", (uint64_t)sp.n_heads * hd, 1);
        w2(p + "attn_k.weight", sp.d_model, (uint64_t)sp.n_kv_heads * hd, sp.weight_type);
        v1(p + "attn_k.bias", (uint64_t)sp.n_kv_heads * hd, 1);
        w2(p + "attn_v.weight", sp.d_model, (uint64_t)sp.n_kv_heads * hd, sp.weight_type);
        v1(p + "attn_v.bias", (uint64_t)sp.n_kv_heads * hd, 1);
        w2(p + "attn_output.weight", (uint64_t)sp.n_heads * hd, sp.d_model, sp.weight_type);
        v1(p + "ffn_norm.weight", sp.d_model, 2);
        w2(p + "ffn_gate.weight", sp.d_model, sp.d_ff, sp.weight_type);
        w2(p + "ffn_up.weight", sp.d_model, sp.d_ff, sp.weight_type);
        w2(p + "ffn_down.weight", sp.d_ff, sp.d_model, sp.weight_type);
    }
    uint64_t off = 0;
    for (auto& t : ts) {
        ggml_block(t.type, &be, &bb);
        if (elems_of(t) % be) return fail(SYN_E_ARG, "tensor " + t.name + " is not a whole number of blocks");
        t.rel_off = off;
        t.bytes = elems_of(t) / be * bb;
        off = (off + t.bytes + 31) / 32 * 32;
    }
    FILE* f = fopen(path, "wb");
    if (!f) return fail(SYN_E_IO, std::string("io: cannot create ") + path);
    Out o(f);
    o.u32(0x46554747u);
    o.u32(3);
    o.u64(ts.size());
    o.u64(15);
    o.kv_str("general.architecture", "qwen2");
    o.kv_u32("general.alignment", 32);
    o.kv_u32("qwen2.block_count", sp.n_layers);
    o.kv_u32("qwen2.context_length", sp.context_length);
    o.kv_u32("qwen2.embedding_length", sp.d_model);
    o.kv_u32("qwen2.feed_forward_length", sp.d_ff);
    o.kv_u32("qwen2.attention.head_count", sp.n_heads);
    o.kv_u32("qwen2.attention.head_count_kv", sp.n_kv_heads);
    o.kv_f32("qwen2.rope.freq_base", sp.rope_base);
    o.kv_f32("qwen2.attention.layer_norm_rms_epsilon", sp.eps);
    o.kv_str("tokenizer.ggml.model", "gpt2");
    o.str("tokenizer.ggml.tokens");
    o.u32(9);
    o.u32(8);
    o.u64(sp.vocab);
    for (uint32_t i = 0; i < sp.vocab; i++) o.str("<t" + std::to_string(i) + ">");
    o.str("tokenizer.ggml.merges");
    o.u32(9);
    o.u32(8);
    o.u64(0);
    o.kv_u32("tokenizer.ggml.eos_token_id", sp.eos);
    o.kv_u32("tokenizer.ggml.bos_token_id", sp.eos);
    for (auto& t : ts) {
        o.str(t.name);
        o.u32((uint32_t)t.dims.size());
        for (auto d : t.dims) o.u64(d);
        o.u32(t.type);
        o.u64(t.rel_off);
    }
    o.pad(32);
    std::vector<uint8_t> buf;
    uint64_t at = 0;
    for (auto& t : ts) {
        static const uint8_t z[32] = {0};
        o.bytes(z, t.rel_off - at);
        encode(sp, t, buf);
        o.bytes(buf.data(), buf.size());
        at = t.rel_off + t.bytes;
    }
    bool ok = o.ok();
    ok = (fclose(f) == 0) && ok;
    if (!ok) return fail(SYN_E_IO, std::string("io: write failed for ") + path);
    return SYN_OK;
}
