// Launch-side descriptions of the token-loop kernels (defined in decode.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "device.cuh"

namespace hs {

// GEMV input modes.
enum GemvIn : int { IN_PLAIN = 0, IN_NORM = 1, IN_EMBED_NORM = 2 };
// GEMV epilogues: y = W x (+b); x_resid += W x; hb = silu(Wg x) * (Wu x).
enum GemvOut : int { OUT_STORE = 0, OUT_RESID = 1, OUT_SILU = 2 };

struct GemvArgs {
    const float* src;       // activation input (n floats); residual stream for IN_NORM
    const uint16_t* embd;   // IN_EMBED_NORM: embedding table [vocab][n]
    const float* norm_g;    // rmsnorm gain (IN_NORM / IN_EMBED_NORM)
    float eps;
    const float* bias;      // OUT_STORE: optional bias [rows]
    float* dst;             // OUT_STORE: y; OUT_RESID: residual x; OUT_SILU: hb
    float* x_out;           // IN_EMBED_NORM: CTA 0 stores the embedded row here
    DevCtl* ctl;
    uint32_t n;             // row length (multiple of 64)
    uint32_t rows;          // output rows
    uint32_t rt;            // rows per tile (TMA box height)
    uint32_t nst;           // pipeline stages
    uint32_t slab_stride;   // bytes between 64-column slabs of one tile (multiple of 1024)
    uint32_t lanes;         // dot lanes per thread (1, 2, 4, 8)
    uint64_t* trace;        // optional per-launch timestamps (see KTrace)
    uint32_t trace_slot;
};

// One planned GEMV launch (shapes fixed at load).
struct GemvPlan {
    int in_mode = IN_PLAIN, out_mode = OUT_STORE;
    bool fast = false;      // GPU-native order (decode_fast.cu); `lanes` then holds threads per row
    uint32_t cmax = 0;      // fast: 16-byte chunks per thread (template width)
    uint32_t n = 0, rows = 0, rt = 0, nst = 1, slab_stride = 0, lanes = 1, grid = 0, threads = 256;
    size_t smem = 0;
    CUtensorMap tm0{}, tm1{};
};

struct AttnArgs {
    const float* qkv;        // [nh*hd q | nkv*hd k | nkv*hd v], bias included, before RoPE
    float* kv;               // KV region (reference byte layout)
    uint64_t* dirty;         // page bitmap words
    const uint32_t* tracking;
    const float* rope_cos;   // [max_ctx][hd/2]
    const float* rope_sin;
    float* att;              // [nh*hd]
    DevCtl* ctl;
    uint32_t layer, nh, nkv, max_ctx, layout, page_shift;
    uint64_t* trace;
    uint32_t trace_slot;
};

struct SampleArgs {
    const float* logits;
    const uint32_t* tokens;  // history (device)
    uint32_t* tokens_w;      // same buffer, written by the commit
    uint64_t* cand;          // per-CTA top-k keys
    uint64_t* argbuf;        // per-CTA (value bits, index) for greedy
    DevCtl* ctl;
    uint32_t vocab, n_cta, kmax;
    uint64_t* trace;
    uint32_t trace_slot;
};

int launch_dequant(uint32_t ty, const void* src, uint64_t n, void* dst, cudaStream_t st, int n_sm);

// Launchers (PDL attribute set; may be captured in a graph).
cudaError_t launch_gemv(const GemvPlan& p, const GemvArgs& a, cudaStream_t st);
cudaError_t launch_attention(uint32_t head_dim, uint32_t nh, size_t smem, const AttnArgs& a, cudaStream_t st);
size_t attention_smem(uint32_t head_dim, uint32_t max_ctx);
cudaError_t launch_sample(const SampleArgs& a, cudaStream_t st);
size_t sample_final_smem(uint32_t n_cta, uint32_t kmax);
cudaError_t gemv_set_smem_limits(int optin);

// GPU-native numeric order (decode_fast.cu).
uint32_t fast_cmax_for(uint32_t chunks_per_thread);
cudaError_t fast_set_smem_limits(int optin);
cudaError_t launch_gemv_fast(const GemvPlan& p, const GemvArgs& a, cudaStream_t st);
size_t attention_fast_smem(uint32_t head_dim, uint32_t max_ctx);
cudaError_t launch_attention_fast(uint32_t head_dim, uint32_t nh, size_t smem, const AttnArgs& a, cudaStream_t st);

constexpr uint32_t kSampleSlice = 1024;  // logits per CTA of the candidate kernel
constexpr uint32_t kMaxTopK = 64;        // top_k supported by the device sampler

}  // namespace hs
