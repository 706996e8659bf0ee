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
    float* sc_global;        // non-null: attention scores [nh][max_ctx] here instead of shared memory
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
    // Batched launch (gridDim.y = slots; 0 or 1 = the single-slot layout):
    // slot s uses logits + s*logits_stride, cand + s*cand_stride,
    // argbuf + s*n_cta, ctl + s, and history buffer tok_tab[s] when set.
    uint32_t slots;
    uint64_t logits_stride, cand_stride;
    uint32_t* const* tok_tab;
    // Logits per candidate CTA: 0 = kSampleSlice; else a multiple of 256 up
    // to kMaxSlice (kmax <= kMaxTopK, or sort mode).
    uint32_t slice;
    // Sort mode (several candidate CTAs and kmax > kMaxTopK; kmax = the
    // slice): every candidate CTA writes its whole slice in key order
    // (cand_stride = n_cta x slice per slot), a rank kernel scatters the
    // global top-k keys of each slot to wkeys + s*wide_stride in order, and
    // the final kernel keeps its weights' running sums in wps + s*wide_stride.
    uint64_t* wkeys;
    float* wps;
    uint64_t wide_stride;
};

int launch_dequant(uint32_t ty, const void* src, uint64_t n, void* dst, cudaStream_t st, int n_sm);

// KV byte-run transfers (kv_xfer.cu): `n` runs of at most kXferPiece bytes,
// src + src_off -> dst + dst_off; dst may be another GPU's peer-mapped memory.
struct XferRun {
    uint64_t src_off, dst_off, len;
};
constexpr uint64_t kXferPiece = 64 * 1024;
cudaError_t launch_copy_runs(const uint8_t* src, uint8_t* dst, const XferRun* runs, uint32_t n, int n_sm,
                             cudaStream_t st);

// Perplexity score (nll.cu): out[r] = NLL of next[r] under logits row r.
cudaError_t launch_logits_nll(const float* logits, uint64_t stride, const uint32_t* next, uint32_t rows,
                              uint32_t vocab, double* out, cudaStream_t st);

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

// Tensor-core path (batch_tc.cu).
enum TcEpi : int { TC_STORE = 0, TC_PART = 1, TC_SILU = 2 };

struct TcGemmArgs {
    uint32_t K;              // reduction length (multiple of 64)
    uint32_t rows;           // weight rows = output features
    uint32_t n_tile;         // weight rows per tile (multiple of 8; SiLU: gate + up rows <= 256)
    uint32_t n_tiles;        // ceil(rows / n_tile)
    uint32_t splits;         // K splits per tile (TC_PART: partial sums per split)
    uint32_t slots;          // live activation rows (groups of 64 along gridDim.y)
    uint32_t nst;            // shared-memory pipeline stages (activations only when wres)
    uint32_t wres;           // 1: the CTA's one unit keeps all its weight boxes in shared memory,
                             //    loaded before the dependency wait; only activations stream
    uint32_t ld;             // row stride (elements) of the outputs
    uint32_t m_loop;         // 1: one grid row; a CTA walks (unit, 64-slot group) items
    uint64_t part_stride;    // TC_PART: elements between splits
    float* out;              // TC_STORE: out = D; TC_PART: out[split] = partial D
    uint16_t* out_hi;        // TC_SILU: f16 pair of silu(gate) * up
    uint16_t* out_lo;
    uint32_t* err;           // error bits (ERR_TIMEOUT)
    uint64_t* trace;
    uint32_t trace_slot;
};

struct TcGemmPlan {
    int epi = TC_STORE;
    uint32_t K = 0, rows = 0, n_tile = 0, n_tiles = 0, splits = 1, nst = 0, grid = 0, m_tiles = 1;
    bool wres = false;       // weights resident (see TcGemmArgs::wres)
    bool m_loop = false;     // CTAs walk the 64-slot groups (see TcGemmArgs::m_loop); grid set per launch
    size_t smem = 0;
    CUtensorMap tm0{}, tm1{};  // weight boxes {64 columns, n_tile rows}
};

size_t tc_gemm_smem(uint32_t n_tile, uint32_t nst, bool silu);
// Weights-resident layout: nst activation stages + kw k-blocks of weight boxes.
size_t tc_gemm_smem_wres(uint32_t n_tile, uint32_t nst, bool silu, uint32_t kw);
bool tc_tile_ok(uint32_t n_tile, bool silu);
cudaError_t tc_set_smem_limits(int optin);
cudaError_t launch_tc_gemm(const TcGemmPlan& p, const CUtensorMap& ahi, const CUtensorMap& alo, const TcGemmArgs& a,
                           cudaStream_t st);

struct TcNormArgs {
    float* x;                // [slots][d] residual stream (updated when embd or n_part)
    const float* part;       // split-K partials [n_part][slots][d] added before the norm
    uint32_t n_part;
    uint64_t part_stride;    // elements between splits
    const uint16_t* embd;    // non-null: x = embedding row of the slot's token (layer 0)
    const float* g;          // RMSNorm gain [d]
    uint16_t* out_hi;        // [slots][d] f16 pair of the normed row
    uint16_t* out_lo;
    DevCtl* ctl;             // per-slot control blocks
    uint32_t d, vocab;
    float eps;
    uint64_t* trace;
    uint32_t trace_slot;
};

// Split-KV decode attention (attn_split.cu), GPU-native paths.
struct SplitAttnArgs {
    const float* qkv;        // QKV product: sum of n_part partials (part_stride apart), then + bias
    uint32_t n_part;
    uint64_t part_stride;
    const float* bias;       // [qkv_rows] or null (already added)
    uint32_t qkv_rows;       // elements between sequences' QKV rows
    float* const* kv;        // per-sequence KV regions, dirty bitmaps, tracking flags
    uint64_t* const* dirty;
    const uint32_t* const* tracking;
    const float* rope_cos;
    const float* rope_sin;
    float* out_f32;          // non-null: f32 output; else the f16 hi/lo pair
    uint16_t* out_hi;
    uint16_t* out_lo;
    uint32_t out_stride;     // elements between sequences' outputs
    float* partials;         // [sequences][nkv][max_splits][attn_record(groups, hd)]
    uint32_t* counters;      // [sequences][nkv], zero between launches
    DevCtl* ctl;             // per-sequence control blocks
    uint32_t layer, nh, nkv, max_ctx, layout, page_shift, max_splits;
    uint32_t mode;           // ATTN_* below
    uint32_t head_split;     // items per (split, KV head): the group's query heads in this many parts (0 = 1)
    uint32_t nbuf;           // K/V chunk buffers per item, 2..4 (0 = by head_dim)
    uint32_t tensor_cores;   // chunk products on the tensor cores (split tf32), else fp32 on the CUDA cores
    uint32_t unstaged_combine;  // the last CTA's combine reads the splits through L2 per element (always at <= 8 splits)
    uint32_t ws_from;        // from this many positions on, the warp-split item form (0: never)
    uint32_t tcw;            // tensor-core path: the tensor-core warp-split item form
    uint32_t min_split;      // target positions per split (0: spread over max_splits)
    uint64_t* trace;
    uint32_t trace_slot;
};
enum AttnMode : uint32_t { ATTN_FULL = 0, ATTN_APPEND_ONLY = 1, ATTN_ATTEND_ONLY = 2 };
// Query-head parts per (split, KV head), at most the group size.
__host__ __device__ inline uint32_t attn_head_split(const SplitAttnArgs& a) {
    const uint32_t g = a.nh / a.nkv, h = a.head_split ? a.head_split : 1;
    return h < g ? h : g;
}
// Positions per split for n cached positions: a multiple of 64, so that at
// most max_splits splits cover n.
// The item form for n positions: warp-split blocks from ws_from positions
// on (0: never), the chunked form below.
__host__ __device__ inline bool attn_use_ws(uint32_t n, uint32_t ws_from) { return ws_from && n >= ws_from; }
// Positions per split: a multiple of 64 covering n in at most max_splits
// splits; at least 512 where the warp-split form runs (fewer, longer items
// whose warps each take several blocks). With a target length (the
// tensor-core path: the length max_splits was sized for) n is cut into
// ceil(n / target) splits (at most max_splits) of equal length, so a short
// context under a long max_ctx is not cut into 64-position items.
__host__ __device__ inline uint32_t attn_split_len(uint32_t n, uint32_t max_splits, uint32_t ws_from,
                                                   uint32_t target = 0) {
    const uint32_t chunks = (n + 63) / 64;
    uint32_t splits = max_splits;
    if (target) {
        const uint32_t want = (n + target - 1) / target;
        if (want < splits) splits = want;
    }
    const uint32_t L = (chunks + splits - 1) / splits * 64;
    const uint32_t min_len = attn_use_ws(n, ws_from) ? 512 : 64;
    return L > min_len ? L : min_len;
}
// Floats per published split of one (sequence, KV head): the group's
// unnormalised outputs [G][hd], maxima [G], sums [G], padded to 16 bytes.
__host__ __device__ inline uint32_t attn_record(uint32_t groups, uint32_t hd) {
    return (groups * hd + 2 * groups + 3) / 4 * 4;
}
size_t attn_split_smem(uint32_t head_dim, uint32_t nbufs = 0);
uint32_t attn_max_splits(uint32_t max_ctx);
// The warp-split attend fits an item with `nbufs` chunk buffers at head_dim hd.
bool attn_ws_fits(uint32_t hd, uint32_t nbufs);
cudaError_t attn_split_set_smem_limits(int optin);
cudaError_t launch_attn_split(uint32_t head_dim, const SplitAttnArgs& a, uint32_t slots, cudaStream_t st);

// Prompt prefill attention by query blocks (attn_prefill.cu): the ATTEND_ONLY
// half of a prefill pass (every slot one token of the same sequence, whose
// k, v rows are appended), over segments of attn_prefill_seg(max_ctx)
// positions with their records in a.partials [slots][nkv][a.max_splits]
// [attn_record] (a.max_splits >= attn_prefill_segs(max_ctx)), then their
// merge: two launches, trace slots trace_slot and trace_slot + 1.
constexpr uint32_t kPrefillMaxSegs = 32;
uint32_t attn_prefill_seg(uint32_t max_ctx);
uint32_t attn_prefill_segs(uint32_t max_ctx);
bool attn_prefill_supported(uint32_t head_dim, uint32_t nh, uint32_t nkv);
cudaError_t attn_prefill_set_smem_limits(int optin);
// tensor_cores: the products on mma.sync with f16 hi/lo operands (128-row
// blocks), else fp32 FMA chains on the CUDA cores (64-row blocks).
cudaError_t launch_attn_prefill(uint32_t head_dim, const SplitAttnArgs& a, uint32_t slots, uint32_t seg,
                                cudaStream_t st, uint32_t trace_slot, bool tensor_cores);
size_t attn_prefill_smem(uint32_t head_dim, bool tensor_cores);
// The append half of a prefill pass (every slot's k, v rows written and their
// pages marked), the same rows as ATTN_APPEND_ONLY's items: one launch.
cudaError_t launch_prefill_append(uint32_t head_dim, const SplitAttnArgs& a, uint32_t slots, cudaStream_t st);

cudaError_t launch_tc_norm(const TcNormArgs& a, uint32_t slots, cudaStream_t st);

// One decode token of the fast path as one persistent kernel (token_fast.cu).
struct TokLayer {
    const float *attn_norm, *ffn_norm, *bqkv;
    const uint16_t *wqkv, *wo, *wgate, *wup, *wdown;
};
struct TokenArgs {
    const TokLayer* layers;  // device [n_layers]
    uint32_t n_layers, d, ff, nh, nkv, hd, vocab;
    float eps;
    const uint16_t* embd;    // [vocab][d]
    const float* out_norm;
    const uint16_t* head_w;  // [vocab][d]
    // activations as tagged entries (value, tag of the phase that wrote it)
    uint64_t *tx, *tqkv, *tatt, *thb;  // [d], [qkv rows], [nh*hd], [ff]
    uint64_t* trec;          // attention split records [nkv][max_splits][attn_record]
    float* logits;
    SplitAttnArgs attn;      // attention items (KV tables, partials, counters)
    DevCtl* ctl;
    uint32_t* seq;           // launch counter (the tags' high part), advanced by every launch
    uint32_t slot_bytes;     // weight ring: slot size (multiple of 1024) and count
    uint32_t nslot;
    uint64_t* trace;
    uint32_t trace_slot;
    uint64_t* phase_ts;      // trace mode: CTA 0's timeline per phase interval
    // Polling rounds before a reader of tagged entries gives up and the
    // launch reports ERR_TIMEOUT (the weight ring's waits are not affected).
    uint32_t poll_limit;
};
struct TokenPlan {
    uint32_t grid = 0, slot_bytes = 0, nslot = 0;
    int shape = -1;          // compiled shape class
    size_t smem = 0;
};
// Plans the launch for the given shapes within `smem_cap` (ring slots of
// `slot_only` bytes when non-zero); false if they do not fit (the per-kernel
// path is then used).
bool token_fast_plan(TokenPlan* p, uint32_t n_layers, uint32_t d, uint32_t ff, uint32_t nh, uint32_t nkv,
                     uint32_t hd, uint32_t vocab, int n_sm, size_t smem_cap, uint32_t slot_only);
cudaError_t token_fast_set_smem_limits(int optin);
// One CTA of the planned size fits on an SM (so the cooperative grid of one
// CTA per SM is resident).
bool token_fast_resident(const TokenPlan& p);
cudaError_t launch_token_fast(const TokenPlan& p, const TokenArgs& a, cudaStream_t st);

constexpr uint32_t kSampleSlice = 1024;  // logits per CTA of the candidate kernel
constexpr uint32_t kMaxSlice = 4096;     // largest slice a candidate CTA takes
constexpr uint32_t kMaxTopK = 64;        // keys kept per candidate CTA in list mode

// True when a sampler launch runs in sort mode (three kernels: slice sort,
// rank, final), which serves any top_k, instead of per-slice top-kmax lists.
__host__ __device__ inline bool sample_sort_mode(uint32_t n_cta, uint32_t kmax) { return n_cta > 1 && kmax > kMaxTopK; }

}  // namespace hs
