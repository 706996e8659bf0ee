// Host side of libhotseat: model load, KV regions, the per-thread scratch with
// its captured CUDA graphs, and the C ABI declared in include/hotseat.h.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "common.h"
#include "gguf.h"
#include "kernels.h"

namespace hs {

void rope_tables(uint32_t head_dim, uint32_t max_ctx, float rope_base, std::vector<float>* cos_t,
                 std::vector<float>* sin_t);

namespace {
thread_local std::string g_err;
}
void set_error(const std::string& msg) { g_err = msg; }
int fail(int code, const std::string& msg) {
    g_err = msg;
    return code;
}

namespace {

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library loads on hosts without a CUDA driver (it then fails at first use).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int make_weight_map(CUtensorMap* map, const uint16_t* w, uint32_t n, uint32_t rows, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(HS_E_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {n, rows};
    cuuint64_t strides[1] = {(cuuint64_t)n * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(w), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(HS_E_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return HS_OK;
}

uint32_t round_up(uint32_t v, uint32_t m) { return (v + m - 1) / m * m; }

// Choose tile height, stages and lanes for one GEMV so the CTA's working set
// fits in shared memory; prefer keeping a CTA's whole row range resident
// (one stage, loaded before the PDL wait), else stream tiles through 2-3 stages.
int plan_gemv(GemvPlan* p, int in_mode, int out_mode, uint32_t rows, uint32_t n, const uint16_t* w0,
              const uint16_t* w1, int n_sm, size_t smem_cap) {
    if (n % 64) return fail(HS_E_UNSUPPORTED, "row length must be a multiple of 64, got " + std::to_string(n));
    const uint32_t nmat = out_mode == OUT_SILU ? 2 : 1, kslabs = n / 64;
    p->in_mode = in_mode;
    p->out_mode = out_mode;
    p->n = n;
    p->rows = rows;
    p->grid = std::min<uint32_t>(rows, (uint32_t)n_sm);
    const uint32_t per = (rows + p->grid - 1) / p->grid;
    // Mirrors the kernel's shared-memory carve-up (decode.cu k_gemv).
    auto need = [&](uint32_t rt, uint32_t nst) -> size_t {
        size_t slab = round_up(rt * 128, 1024);
        return 1024 + (size_t)nst * nmat * kslabs * slab + (size_t)n * 10 + 3 * rt * 4 + 4 + 128 + (nst + 1) * 8;
    };
    uint32_t rt = 0, nst = 0;
    if (per * nmat <= 256 && need(per, 1) <= smem_cap) {
        rt = per;
        nst = 1;
    } else {
        for (uint32_t s : {3u, 2u}) {
            for (uint32_t r = std::min<uint32_t>(per, 256 / nmat); r >= 1; r--) {
                if (r < per && r > 8 && r % 8) continue;  // whole swizzle atoms when streaming
                if (need(r, s) <= smem_cap) {
                    rt = r;
                    break;
                }
            }
            if (rt) {
                nst = s;
                break;
            }
        }
    }
    if (!rt) return fail(HS_E_UNSUPPORTED, "GEMV tile does not fit in shared memory");
    p->rt = rt;
    p->nst = nst;
    p->slab_stride = round_up(rt * 128, 1024);
    // Lanes per thread: the fewest per-SMSP instructions for one tile pass,
    // counting ~7/9/10/19 instructions per step at 1/2/4/8 lanes and the
    // warps an SMSP must issue in turn.
    const uint32_t vrows = rt * nmat;
    const uint32_t instr[4] = {7, 7, 10, 19};
    uint64_t best = ~0ull;
    for (uint32_t li = 0; li < 4; li++) {
        const uint32_t L = 1u << li, threads = vrows * (8 / L);
        if (threads > 512) continue;
        const uint32_t warps = (threads + 31) / 32;
        const uint64_t cost = (uint64_t)((warps + 3) / 4) * instr[li];
        if (cost < best) {
            best = cost;
            p->lanes = L;
            p->threads = std::max<uint32_t>(128, (threads + 31) / 32 * 32);
        }
    }
    p->smem = need(rt, nst);
    int rc = make_weight_map(&p->tm0, w0, n, rows, rt);
    if (rc == HS_OK && w1) rc = make_weight_map(&p->tm1, w1, n, rows, rt);
    return rc;
}

// Fast path: threads per row T from the row length alone (a power of two
// with at most 6 chunks of 8 elements per thread), 256 threads per CTA.
int plan_gemv_fast(GemvPlan* p, int in_mode, int out_mode, uint32_t rows, uint32_t n, const uint16_t* w0,
                   const uint16_t* w1, int n_sm, size_t smem_cap) {
    if (n % 64) return fail(HS_E_UNSUPPORTED, "row length must be a multiple of 64, got " + std::to_string(n));
    const uint32_t nmat = out_mode == OUT_SILU ? 2 : 1, kslabs = n / 64, nchunks = n / 8;
    uint32_t T = 32;
    while (T < 256 && (nchunks + T - 1) / T > 6) T *= 2;
    const uint32_t cmax = fast_cmax_for((nchunks + T - 1) / T);
    if (!cmax) return fail(HS_E_UNSUPPORTED, "row too long for the fast GEMV");
    p->fast = true;
    p->cmax = cmax;
    p->lanes = T;
    p->threads = 256;
    p->in_mode = in_mode;
    p->out_mode = out_mode;
    p->n = n;
    p->rows = rows;
    p->grid = std::min<uint32_t>(rows, (uint32_t)n_sm);
    const uint32_t per = (rows + p->grid - 1) / p->grid;
    // Mirrors the kernel's shared-memory carve-up (decode_fast.cu k_gemv_fast).
    auto need = [&](uint32_t rt, uint32_t nst) -> size_t {
        size_t slab = round_up(rt * 128, 1024);
        return 1024 + (size_t)nst * nmat * kslabs * slab + (size_t)n * 10 + 2 * rt * 8 * 4 + rt * 4 + 4 + 128 +
               (nst + 1) * 8;
    };
    uint32_t rt = 0, nst = 0;
    if (per <= 256 / nmat && need(per, 1) <= smem_cap) {
        rt = per;
        nst = 1;
    } else {
        for (uint32_t s : {3u, 2u}) {
            for (uint32_t r = std::min<uint32_t>(per, 256 / nmat); r >= 1; r--) {
                if (r < per && r > 8 && r % 8) continue;
                if (need(r, s) <= smem_cap) {
                    rt = r;
                    break;
                }
            }
            if (rt) {
                nst = s;
                break;
            }
        }
    }
    if (!rt) return fail(HS_E_UNSUPPORTED, "GEMV tile does not fit in shared memory");
    p->rt = rt;
    p->nst = nst;
    p->slab_stride = round_up(rt * 128, 1024);
    p->smem = need(rt, nst);
    int rc = make_weight_map(&p->tm0, w0, n, rows, rt);
    if (rc == HS_OK && w1) rc = make_weight_map(&p->tm1, w1, n, rows, rt);
    return rc;
}

cudaError_t launch_plan(const GemvPlan& p, const GemvArgs& a, cudaStream_t st) {
    return p.fast ? launch_gemv_fast(p, a, st) : launch_gemv(p, a, st);
}

struct TensorRef {
    void* ptr;
    uint64_t count;
    uint32_t dtype;  // 1 = f16, 0 = f32
};

}  // namespace
}  // namespace hs

using namespace hs;

struct LayerDev {
    float *attn_norm = nullptr, *ffn_norm = nullptr, *bqkv = nullptr;
    uint16_t *wqkv = nullptr, *wo = nullptr, *wgate = nullptr, *wup = nullptr, *wdown = nullptr;
    GemvPlan qkv, o, gu, down;
    TcGemmPlan tq, to, tgu, tdown;  // tensor-core path (decode: split-K over a few M tiles)
    TcGemmPlan pq, po, pgu, pdown;  // tensor-core prefill (many M tiles, no split)
};

struct hs_model {
    hs_config cfg{};
    int device = 0, n_sm = 0;
    size_t smem_cap = 0;
    uint16_t *embd = nullptr, *out_w = nullptr;
    float *out_norm = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
    std::vector<LayerDev> layers;
    GemvPlan head;
    size_t attn_smem = 0;
    bool attn_global = false;     // attention scores in a global buffer (long max_ctx)
    bool attn_split = false;      // split-KV attention (GPU-native paths)
    uint32_t max_splits = 0;
    uint32_t attn_head_split = 1;  // query-head parts per split-KV attention item
    uint32_t attn_nbuf = 0;        // K/V chunk buffers per item (0 = by head_dim)
    uint32_t attn_unstaged = 0;    // HS_ATTN_UNSTAGED_COMBINE=1: the per-element combine (same bits; measurement)
    uint32_t attn_ws_from = 0;     // warp-split item form from this many positions on (0: never)
    uint32_t attn_tcw = 0;         // tensor-core path: the tensor-core warp-split item form
    uint32_t attn_min_split = 0;   // tensor-core path: target positions per split
    bool pf_qblock = false;        // prefill attends by query blocks (attn_prefill.cu)
    bool pf_tc = false;            // ... with the products on the tensor cores
    uint32_t pf_seg = 0, pf_nseg = 0;  // its segment length and segments per token at most
    uint32_t numeric = HS_NUMERIC_REFERENCE;
    TcGemmPlan thead;             // tensor-core LM head
    bool tok = false;             // fast path: one persistent kernel per token (token_fast.cu)
    TokenPlan tokp;
    TokLayer* tok_layers = nullptr;  // device copy of the layers' weight pointers
    uint64_t tc_part_per_slot = 0;  // max over split-K GEMMs of splits * rows
    const uint16_t* head_w = nullptr;
    std::map<std::string, TensorRef> tensors;
    std::vector<void*> allocs;
    ~hs_model() {
        if (!allocs.empty()) cudaSetDevice(device);
        for (void* p : allocs) cudaFree(p);
    }
};

struct hs_kv {
    hs_kv_spec spec{};
    int device = 0;
    uint64_t bytes = 0, n_pages = 0, n_words = 0;
    uint32_t page_size = 0, page_shift = 0;
    float* base = nullptr;
    uint64_t* dirty = nullptr;
    uint64_t* harvest_buf = nullptr;
    uint32_t* tracking = nullptr;
    uint64_t fingerprint = 0;
    cudaStream_t st = nullptr;
    int n_sm = 148;
    // byte-run transfers: packed staging (grown on demand), the run table
    // (pinned upload buffer and device copy) and the event after its last use
    uint8_t* stage = nullptr;
    uint64_t stage_cap = 0;
    hs::XferRun *tab_h = nullptr, *tab_dev = nullptr;
    uint64_t tab_cap = 0;
    cudaEvent_t tab_ev = nullptr;
    bool ipc_view = false;  // `base` maps another process's region (hs_kv_open_ipc)
    ~hs_kv() {
        cudaSetDevice(device);
        if (tab_ev) cudaEventSynchronize(tab_ev);
        if (st) cudaStreamDestroy(st);
        if (tab_ev) cudaEventDestroy(tab_ev);
        cudaFreeHost(tab_h);
        cudaFree(tab_dev);
        cudaFree(stage);
        if (ipc_view)
            cudaIpcCloseMemHandle(base);
        else
            cudaFree(base);
        cudaFree(dirty);
        cudaFree(harvest_buf);
        cudaFree(tracking);
    }
};

struct hs_scratch {
    const hs_model* m = nullptr;
    cudaStream_t st = nullptr;
    DevCtl* ctl = nullptr;       // device
    DevCtl* ctl_h = nullptr;     // pinned host mirror
    float *x = nullptr, *qkv = nullptr, *att = nullptr, *hb = nullptr, *logits = nullptr;
    uint32_t* tokens = nullptr;
    uint64_t cap = 0;
    uint64_t *cand = nullptr, *argbuf = nullptr;
    uint32_t n_cta = 0, kmax = 0, slice = 0;  // sampler: candidate CTAs, keys kept per CTA, logits per CTA
    // sampler sort mode (any top_k), allocated at its first use: every
    // slice's keys in order, the top-k keys in order, their running sums
    uint64_t *sort_cand = nullptr, *wkeys = nullptr;
    float* wps = nullptr;
    double* nll = nullptr;          // perplexity score of the last forward (hs_scratch_nll)
    uint32_t* nll_next = nullptr;
    cudaGraphExec_t g_fwd = nullptr, g_step = nullptr;
    const hs_kv* graph_kv = nullptr;
    uint32_t graph_kmax = 0;
    uint32_t launches_fwd = 0;
    float* sc_global = nullptr;     // attention scores [nh][max_ctx] for long contexts
    float* att_part = nullptr;      // split-KV attention partials and counters
    uint32_t* att_cnt = nullptr;
    void** kv_tab = nullptr;        // one-entry KV / dirty / tracking tables for split attention
    // persistent token kernel: its launch counter (16 bytes), then its
    // tagged activations x, qkv, att, hb and attention records
    uint8_t* tok_mem = nullptr;
    uint64_t tok_launches = 0;      // token-kernel launches (tag refresh)
    // token kernel: polling rounds before a reader of tagged entries gives up
    // (HS_POLL_LIMIT at creation, a test knob; default 2^22)
    uint32_t poll_limit = 1u << 22;
    uint64_t* trace = nullptr;      // device, 4 u64 per launch slot (trace mode only)
    uint64_t* trace_init = nullptr; // pinned host template: start=~0, rest 0
    uint32_t trace_slots = 0;
    ~hs_scratch() {
        cudaSetDevice(m->device);
        if (g_fwd) cudaGraphExecDestroy(g_fwd);
        if (g_step) cudaGraphExecDestroy(g_step);
        if (st) cudaStreamDestroy(st);
        cudaFree(ctl);
        cudaFreeHost(ctl_h);
        cudaFree(trace);
        cudaFreeHost(trace_init);
        for (void* p : {(void*)x, (void*)qkv, (void*)att, (void*)hb, (void*)logits, (void*)tokens, (void*)cand,
                        (void*)argbuf, (void*)sc_global, (void*)att_part, (void*)att_cnt, (void*)kv_tab,
                        (void*)tok_mem, (void*)sort_cand, (void*)wkeys, (void*)wps, (void*)nll, (void*)nll_next})
            cudaFree(p);
    }
};

namespace hs {
namespace {

template <typename T>
int dev_alloc(hs_model* m, T** p, uint64_t count) {
    void* q = nullptr;
    cudaError_t e = cudaMalloc(&q, std::max<uint64_t>(count, 1) * sizeof(T));
    if (e != cudaSuccess) return fail(HS_E_NOMEM, std::string("cudaMalloc: ") + cudaGetErrorString(e));
    m->allocs.push_back(q);
    *p = static_cast<T*>(q);
    return HS_OK;
}

// Dequantise one GGUF tensor to f16 on the device at `dst` (model.rs:375-396).
int load_f16(hs_model* m, const Gguf& g, const std::string& name, uint16_t* dst, uint64_t expect, uint8_t* staging,
             cudaStream_t st) {
    const GgufTensor* t = g.tensor(name);
    if (!t) return fail(HS_E_IO, "missing tensor \"" + name + "\"");
    if (t->elems() != expect)
        return fail(HS_E_IO, "tensor \"" + name + "\" has " + std::to_string(t->elems()) + " elements, expected " +
                                 std::to_string(expect));
    HS_CUDA_TRY(cudaMemcpyAsync(staging, g.data() + t->off, t->len, cudaMemcpyHostToDevice, st));
    int rc = launch_dequant(t->type, staging, t->elems(), dst, st, m->n_sm);
    if (rc) return rc;
    HS_CUDA_TRY(cudaStreamSynchronize(st));
    m->tensors[name] = TensorRef{dst, expect, 1};
    return HS_OK;
}

// model.rs:398-413: F32 tensors as stored, anything else through f16.
int load_f32(hs_model* m, const Gguf& g, const std::string& name, float* dst, uint64_t expect) {
    const GgufTensor* t = g.tensor(name);
    if (!t) return fail(HS_E_IO, "missing tensor \"" + name + "\"");
    if (t->elems() != expect)
        return fail(HS_E_IO, "tensor \"" + name + "\" has " + std::to_string(t->elems()) + " elements, expected " +
                                 std::to_string(expect));
    std::vector<float> host(expect);
    if (t->type == 0) {
        std::memcpy(host.data(), g.data() + t->off, expect * 4);
    } else {
        // Rare (norms and biases are F32 in practice): dequantise on the device.
        uint8_t* raw = nullptr;
        uint16_t* h16 = nullptr;
        HS_CUDA_TRY(cudaMalloc(&raw, t->len));
        HS_CUDA_TRY(cudaMalloc(&h16, expect * 2));
        cudaMemcpy(raw, g.data() + t->off, t->len, cudaMemcpyHostToDevice);
        int rc = launch_dequant(t->type, raw, expect, h16, nullptr, m->n_sm);
        std::vector<uint16_t> hh(expect);
        if (rc == HS_OK) cudaMemcpy(hh.data(), h16, expect * 2, cudaMemcpyDeviceToHost);
        cudaFree(raw);
        cudaFree(h16);
        if (rc) return rc;
        for (uint64_t i = 0; i < expect; i++) host[i] = h2f_host(hh[i]);
    }
    HS_CUDA_TRY(cudaMemcpy(dst, host.data(), expect * 4, cudaMemcpyHostToDevice));
    m->tensors[name] = TensorRef{dst, expect, 0};
    return HS_OK;
}

// Kernel-side FNV-1a of the tensor table (model.rs:145-156). `t.ty as u32`
// there is the Rust enum's declaration index, not the ggml id.
uint64_t fingerprint_of(const Gguf& g) {
    auto enum_index = [](uint32_t ty) -> uint32_t {
        switch (ty) {
            case 0: return 0;
            case 1: return 1;
            case 6: return 2;
            case 8: return 3;
            case 12: return 4;
            case 13: return 5;
            case 14: return 6;
        }
        return 0xffffffffu;
    };
    uint64_t h = 0xcbf29ce484222325ull;
    auto put = [&](const void* p, size_t n) {
        const uint8_t* b = static_cast<const uint8_t*>(p);
        for (size_t i = 0; i < n; i++) h = (h ^ b[i]) * 0x100000001b3ull;
    };
    uint64_t len = g.size();
    put(&len, 8);
    for (const auto& name : g.order()) {
        const GgufTensor* t = g.tensor(name);
        put(name.data(), name.size());
        uint32_t e = enum_index(t->type);
        put(&e, 4);
        uint64_t off = t->off, l = t->len;
        put(&off, 8);
        put(&l, 8);
    }
    return h;
}

int check_kv(const hs_model* m, const hs_kv* kv) {
    const hs_config& c = m->cfg;
    if (kv->spec.n_layers != c.n_layers || kv->spec.n_kv_heads != c.n_kv_heads || kv->spec.head_dim != c.head_dim ||
        kv->spec.max_ctx != c.max_ctx)
        return fail(HS_E_ARG, "KV cache shape does not match the model");
    if (kv->device != m->device) return fail(HS_E_ARG, "KV cache lives on another device than the model");
    return HS_OK;
}

uint32_t env_u32(const char* name, uint32_t dflt) {
    const char* v = std::getenv(name);
    return v && *v ? (uint32_t)std::strtoul(v, nullptr, 10) : dflt;
}

// Tensor-core GEMM plan: weight-row tile, K splits and pipeline depth so
// that about one work unit lands on each SM.
//   TC_SILU : gate+up rows of one tile per CTA, no split (the SiLU needs
//             whole sums);
//   TC_STORE: tiles of up to 256 rows, CTAs loop over tiles (LM head);
//   TC_PART : 64/128-row tiles, K split so tiles x splits ~ SM count; the
//             consumer adds the split partials in split order.
int plan_tc(TcGemmPlan* p, int epi, uint32_t rows, uint32_t K, const uint16_t* w0, const uint16_t* w1, int n_sm,
            size_t smem_cap, bool prefill = false) {
    if (K % 64) return fail(HS_E_UNSUPPORTED, "GEMM reduction length must be a multiple of 64");
    const bool silu = epi == TC_SILU;
    const uint32_t kt_n = K / 64, sm = (uint32_t)n_sm;
    p->epi = epi;
    p->K = K;
    p->rows = rows;
    p->splits = 1;
    if (prefill) {
        // Prompt passes bring many 64-token groups. These GEMMs are bound by
        // the latency of each k-block's loads, not by bandwidth (measured: L2
        // and tensor pipes both under a quarter busy), so the widest weight
        // tiles (N = 256: twice the MMA work per k-block of 128) and CTAs
        // that walk (tile, group) items; the partial-sum GEMMs add a K split
        // fixed per model, the one with the fewest k-blocks on the busiest
        // CTA over a 1024-token pass (a token's bits then depend on the
        // model only, never on the pass).
        uint32_t nt = silu ? env_u32("HS_TC_PREFILL_SILU_TILE", 128) : env_u32("HS_TC_PREFILL_TILE", 256);
        while (nt > 16 && nt / 2 >= rows) nt /= 2;
        p->n_tile = nt;
        p->m_loop = env_u32("HS_TC_PREFILL_MLOOP", 1) != 0;
        if (epi == TC_PART && p->m_loop) {
            const uint32_t tiles = (rows + nt - 1) / nt, groups = 1024 / 64;
            const uint32_t max_s = std::min<uint32_t>(env_u32("HS_TC_PREFILL_MAX_SPLITS", 8), std::max<uint32_t>(1, kt_n / 4));
            uint64_t best = ~0ull;
            for (uint32_t S = 1; S <= max_s; S++) {
                const uint64_t items = (uint64_t)tiles * groups * S, rounds = (items + sm - 1) / sm;
                const uint64_t cost = rounds * ((kt_n + S - 1) / S);
                if (cost < best) {
                    best = cost;
                    p->splits = S;
                }
            }
        }
    } else if (silu) {
        uint32_t nt = 8;
        while (nt < 128 && (rows + nt - 1) / nt > sm) nt += 8;
        p->n_tile = nt;
    } else if (epi == TC_STORE) {
        uint64_t best = ~0ull;
        for (uint32_t nt = 16; nt <= 256; nt += 16) {
            const uint64_t tiles = (rows + nt - 1) / nt, per = (tiles + sm - 1) / sm;
            const uint64_t cost = per * nt;
            if (cost < best || (cost == best && nt > p->n_tile)) {
                best = cost;
                p->n_tile = nt;
            }
        }
    } else if (!prefill) {
        // The most CTAs in one wave with at most HS_TC_MAX_SPLITS (32) partials for the
        // consumer to add, then the wider tile (fewer activation re-reads).
        const uint32_t max_splits = env_u32("HS_TC_MAX_SPLITS", 32);
        uint32_t best = 0;
        for (uint32_t nt : {128u, 64u, 32u, 16u}) {
            const uint32_t tiles = (rows + nt - 1) / nt;
            if (tiles > sm) continue;
            const uint32_t S = std::max<uint32_t>(1, std::min<uint32_t>({kt_n, max_splits, sm / tiles}));
            if (tiles * S > best) {
                best = tiles * S;
                p->n_tile = nt;
                p->splits = S;
            }
        }
        if (!best) return fail(HS_E_UNSUPPORTED, "no split-K plan fits");
    }
    p->n_tiles = (rows + p->n_tile - 1) / p->n_tile;
    const uint32_t units = p->n_tiles * p->splits;
    p->grid = std::min<uint32_t>(units, sm);
    p->m_tiles = 1;
    const uint32_t per_cta = (p->m_loop ? 16 : (units + p->grid - 1) / p->grid) * ((kt_n + p->splits - 1) / p->splits);
    uint32_t nst = std::min<uint32_t>(16, per_cta);
    // A smaller budget lets the next kernel's CTA share the SM and start its
    // weight prefetch (programmatic dependent launch) while this one drains.
    smem_cap = std::min<size_t>(smem_cap, (size_t)env_u32("HS_TC_SMEM_KB", 1024) * 1024);
    while (nst > 1 && tc_gemm_smem(p->n_tile, nst, silu) > smem_cap) nst--;
    p->nst = nst;
    p->smem = tc_gemm_smem(p->n_tile, nst, silu);
    // One unit per CTA: keep all its weight boxes in shared memory, loaded
    // before the dependency wait, and stream only the activations after it
    // (HS_TC_WRES=0 keeps weights and activations in the same stages).
    if (units <= p->grid && !p->m_loop && env_u32("HS_TC_WRES", 1) != 0) {
        const uint32_t kw = (kt_n + p->splits - 1) / p->splits;
        uint32_t na = std::min<uint32_t>(16, kw);
        while (na > 1 && tc_gemm_smem_wres(p->n_tile, na, silu, kw) > smem_cap) na--;
        if (tc_gemm_smem_wres(p->n_tile, na, silu, kw) <= smem_cap && (na >= 2 || kw == 1)) {
            p->wres = true;
            p->nst = na;
            p->smem = tc_gemm_smem_wres(p->n_tile, na, silu, kw);
        }
    }
    if (p->smem > smem_cap || !tc_tile_ok(p->n_tile, silu)) return fail(HS_E_UNSUPPORTED, "tensor-core GEMM tile does not fit");
    int rc = make_weight_map(&p->tm0, w0, K, rows, p->n_tile);
    if (rc == HS_OK) rc = make_weight_map(&p->tm1, w1 ? w1 : w0, K, rows, p->n_tile);
    return rc;
}

// Split-KV attention over the scratch's one sequence (layer set by the caller).
SplitAttnArgs scratch_attn_args(const hs_scratch* s, const hs_kv* kv) {
    const hs_model* m = s->m;
    const hs_config& c = m->cfg;
    SplitAttnArgs sa{};
    sa.qkv = s->qkv;
    sa.n_part = 1;
    sa.kv = reinterpret_cast<float* const*>(s->kv_tab);
    sa.dirty = reinterpret_cast<uint64_t* const*>(s->kv_tab + 1);
    sa.tracking = reinterpret_cast<const uint32_t* const*>(s->kv_tab + 2);
    sa.rope_cos = m->rope_cos;
    sa.rope_sin = m->rope_sin;
    sa.out_f32 = s->att;
    sa.partials = s->att_part;
    sa.counters = s->att_cnt;
    sa.ctl = s->ctl;
    sa.nh = c.n_heads;
    sa.nkv = c.n_kv_heads;
    sa.max_ctx = c.max_ctx;
    sa.layout = kv->spec.layout;
    sa.page_shift = kv->page_shift;
    sa.max_splits = m->max_splits;
    sa.head_split = m->attn_head_split;
    sa.nbuf = m->attn_nbuf;
    sa.tensor_cores = m->numeric == HS_NUMERIC_TC ? 1u : 0u;
    sa.unstaged_combine = m->attn_unstaged;
    sa.ws_from = m->attn_ws_from;
    sa.trace = s->trace;
    return sa;
}

// Tagged entries of the persistent token kernel's buffers, after its
// 16-byte launch counter: x, qkv, att, hb, attention records.
struct TokBufs {
    size_t x, qkv, att, hb, rec, total;  // offsets and total in entries
};
TokBufs tok_bufs(const hs_model* m) {
    const hs_config& c = m->cfg;
    TokBufs t{};
    t.x = 0;
    t.qkv = t.x + c.d_model;
    t.att = t.qkv + (size_t)(c.n_heads + 2 * c.n_kv_heads) * c.head_dim;
    t.hb = t.att + (size_t)c.n_heads * c.head_dim;
    t.rec = t.hb + c.d_ff;
    t.total = t.rec + (size_t)c.n_kv_heads * m->max_splits * attn_record(c.n_heads / c.n_kv_heads, c.head_dim);
    return t;
}

// Before a launch of the graph holding the token kernel: the kernel's tags
// are the launch counter x 1024 + (layer, phase), which repeat every 2^22
// launches; entries not rewritten by every launch (the attention output when
// the readers combine split records) could then carry a current-looking tag.
// Clearing the tagged entries every 2^21 launches keeps every entry younger
// than that.
int refresh_tags(hs_scratch* s) {
    if (!s->tok_mem) return HS_OK;
    if (++s->tok_launches % (1ull << 21) == 0)
        HS_CUDA_TRY(cudaMemsetAsync(s->tok_mem + 16, 0, tok_bufs(s->m).total * 8, s->st));
    return HS_OK;
}

// The fast path's whole token as one persistent kernel.
int enqueue_token_kernel(hs_scratch* s, const hs_kv* kv) {
    const hs_model* m = s->m;
    const hs_config& c = m->cfg;
    TokenArgs a{};
    a.layers = m->tok_layers;
    a.n_layers = c.n_layers;
    a.d = c.d_model;
    a.ff = c.d_ff;
    a.nh = c.n_heads;
    a.nkv = c.n_kv_heads;
    a.hd = c.head_dim;
    a.vocab = c.vocab;
    a.eps = c.eps;
    a.embd = m->embd;
    a.out_norm = m->out_norm;
    a.head_w = m->head_w;
    const TokBufs tb = tok_bufs(m);
    uint64_t* ent = reinterpret_cast<uint64_t*>(s->tok_mem + 16);
    a.tx = ent + tb.x;
    a.tqkv = ent + tb.qkv;
    a.tatt = ent + tb.att;
    a.thb = ent + tb.hb;
    a.trec = ent + tb.rec;
    a.logits = s->logits;
    a.attn = scratch_attn_args(s, kv);
    a.attn.trace = nullptr;
    a.ctl = s->ctl;
    a.seq = reinterpret_cast<uint32_t*>(s->tok_mem);
    a.slot_bytes = m->tokp.slot_bytes;
    a.nslot = m->tokp.nslot;
    a.trace = s->trace;
    a.trace_slot = 0;
    // trace slots 0-2: this kernel and the two sampler kernels; then the
    // timeline, 20 words per phase interval (5 per layer, then the head)
    a.phase_ts = s->trace ? s->trace + 3 * 8 : nullptr;
    a.poll_limit = s->poll_limit;
    HS_CUDA_TRY(launch_token_fast(m->tokp, a, s->st));
    return HS_OK;
}

// Enqueue one forward pass (the 5 kernels per layer + final norm/LM head, or
// the fast path's single persistent kernel).
int enqueue_forward(hs_scratch* s, const hs_kv* kv) {
    const hs_model* m = s->m;
    const hs_config& c = m->cfg;
    if (m->tok) return enqueue_token_kernel(s, kv);
    cudaStream_t st = s->st;
    uint32_t slot = 0;
    for (uint32_t l = 0; l < c.n_layers; l++) {
        const LayerDev& L = m->layers[l];
        GemvArgs a{};
        a.ctl = s->ctl;
        a.eps = c.eps;
        // rmsnorm + fused QKV (+bias); layer 0 also reads the embedding row.
        a.src = s->x;
        a.embd = m->embd;
        a.x_out = s->x;
        a.norm_g = L.attn_norm;
        a.bias = L.bqkv;
        a.dst = s->qkv;
        a.n = L.qkv.n;
        a.rows = L.qkv.rows;
        a.rt = L.qkv.rt;
        a.nst = L.qkv.nst;
        a.slab_stride = L.qkv.slab_stride;
        a.lanes = L.qkv.lanes;
        GemvPlan pq = L.qkv;
        pq.in_mode = l == 0 ? IN_EMBED_NORM : IN_NORM;
        a.trace = s->trace;
        a.trace_slot = slot++;
        HS_CUDA_TRY(launch_plan(pq, a, st));
        AttnArgs at{};
        at.qkv = s->qkv;
        at.kv = kv->base;
        at.dirty = kv->dirty;
        at.tracking = kv->tracking;
        at.rope_cos = m->rope_cos;
        at.rope_sin = m->rope_sin;
        at.att = s->att;
        at.ctl = s->ctl;
        at.layer = l;
        at.nh = c.n_heads;
        at.nkv = c.n_kv_heads;
        at.max_ctx = c.max_ctx;
        at.layout = kv->spec.layout;
        at.page_shift = kv->page_shift;
        at.trace = s->trace;
        at.trace_slot = slot++;
        at.sc_global = s->sc_global;
        if (m->attn_split) {
            SplitAttnArgs sa = scratch_attn_args(s, kv);
            sa.layer = l;
            sa.trace_slot = at.trace_slot;
            HS_CUDA_TRY(launch_attn_split(c.head_dim, sa, 1, st));
        } else
            HS_CUDA_TRY(launch_attention(c.head_dim, c.n_heads, m->attn_smem, at, st));
        GemvArgs o{};
        o.ctl = s->ctl;
        o.src = s->att;
        o.dst = s->x;
        o.n = L.o.n;
        o.rows = L.o.rows;
        o.rt = L.o.rt;
        o.nst = L.o.nst;
        o.slab_stride = L.o.slab_stride;
        o.lanes = L.o.lanes;
        o.trace = s->trace;
        o.trace_slot = slot++;
        HS_CUDA_TRY(launch_plan(L.o, o, st));
        GemvArgs gu{};
        gu.ctl = s->ctl;
        gu.eps = c.eps;
        gu.src = s->x;
        gu.norm_g = L.ffn_norm;
        gu.dst = s->hb;
        gu.n = L.gu.n;
        gu.rows = L.gu.rows;
        gu.rt = L.gu.rt;
        gu.nst = L.gu.nst;
        gu.slab_stride = L.gu.slab_stride;
        gu.lanes = L.gu.lanes;
        gu.trace = s->trace;
        gu.trace_slot = slot++;
        HS_CUDA_TRY(launch_plan(L.gu, gu, st));
        GemvArgs dn{};
        dn.ctl = s->ctl;
        dn.src = s->hb;
        dn.dst = s->x;
        dn.n = L.down.n;
        dn.rows = L.down.rows;
        dn.rt = L.down.rt;
        dn.nst = L.down.nst;
        dn.slab_stride = L.down.slab_stride;
        dn.lanes = L.down.lanes;
        dn.trace = s->trace;
        dn.trace_slot = slot++;
        HS_CUDA_TRY(launch_plan(L.down, dn, st));
    }
    GemvArgs h{};
    h.ctl = s->ctl;
    h.eps = c.eps;
    h.src = s->x;
    h.norm_g = m->out_norm;
    h.dst = s->logits;
    h.n = m->head.n;
    h.rows = m->head.rows;
    h.rt = m->head.rt;
    h.nst = m->head.nst;
    h.slab_stride = m->head.slab_stride;
    h.lanes = m->head.lanes;
    h.trace = s->trace;
    h.trace_slot = slot++;
    HS_CUDA_TRY(launch_plan(m->head, h, st));
    return HS_OK;
}

SampleArgs sample_args(hs_scratch* s) {
    SampleArgs a{};
    a.logits = s->logits;
    a.tokens = s->tokens;
    a.tokens_w = s->tokens;
    a.cand = s->cand;
    a.argbuf = s->argbuf;
    a.ctl = s->ctl;
    a.vocab = s->m->cfg.vocab;
    a.n_cta = s->n_cta;
    a.kmax = s->kmax;
    a.slice = s->slice;
    if (sample_sort_mode(s->n_cta, s->kmax)) {
        a.cand = s->sort_cand;
        a.cand_stride = (uint64_t)s->n_cta * s->slice;
        a.wkeys = s->wkeys;
        a.wps = s->wps;
        a.wide_stride = s->m->cfg.vocab;
    }
    a.trace = s->trace;
    a.trace_slot = s->launches_fwd;  // and launches_fwd + 1 for the second kernel
    return a;
}

int capture(hs_scratch* s, const hs_kv* kv, bool with_sampler, cudaGraphExec_t* out) {
    cudaGraph_t g = nullptr;
    HS_CUDA_TRY(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_forward(s, kv);
    if (rc == HS_OK && with_sampler) {
        cudaError_t e = launch_sample(sample_args(s), s->st);
        if (e != cudaSuccess) rc = fail(HS_E_CUDA, std::string("sampler launch: ") + cudaGetErrorString(e));
    }
    cudaError_t e = cudaStreamEndCapture(s->st, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return fail(HS_E_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail(HS_E_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
    return HS_OK;
}

// (Re)build the graphs for this KV region and sampler width.
int ensure_graphs(hs_scratch* s, const hs_kv* kv, uint32_t kmax) {
    if (s->graph_kv == kv && s->graph_kmax == kmax && s->g_fwd && s->g_step) return HS_OK;
    if (s->g_fwd) cudaGraphExecDestroy(s->g_fwd);
    if (s->g_step) cudaGraphExecDestroy(s->g_step);
    s->g_fwd = s->g_step = nullptr;
    s->kmax = kmax;
    if (s->kv_tab) {
        void* t[3] = {kv->base, kv->dirty, kv->tracking};
        HS_CUDA_TRY(cudaMemcpy(s->kv_tab, t, sizeof(t), cudaMemcpyHostToDevice));
    }
    int rc = capture(s, kv, false, &s->g_fwd);
    if (rc == HS_OK) rc = capture(s, kv, true, &s->g_step);
    if (rc) return rc;
    s->graph_kv = kv;
    s->graph_kmax = kmax;
    return HS_OK;
}

int ctl_err(uint32_t err) {
    if (!err) return HS_OK;
    std::string why;
    if (err & ERR_TIMEOUT) why += " bounded-wait-timeout";
    if (err & ERR_TOKEN) why += " token-out-of-range";
    if (err & ERR_POS) why += " position-past-max_ctx";
    if (err & ERR_CAP) why += " token-buffer-full";
    if (err & ERR_INVARIANT) why += " nothing-to-feed-at-token-boundary";
    int code = (err & (ERR_INVARIANT | ERR_CAP)) ? HS_E_STATE : (err & ERR_TIMEOUT) ? HS_E_CUDA : HS_E_ARG;
    return fail(code, "device reported:" + why);
}

// After a bounded wait ran out, split-attention items may have left their
// last-CTA counters short; reset them so the next launch starts clean.
int check_ctl_err(hs_scratch* s) {
    const uint32_t err = s->ctl_h->err;
    if ((err & ERR_TIMEOUT) && s->att_cnt) {
        HS_CUDA_TRY(cudaMemsetAsync(s->att_cnt, 0, s->m->cfg.n_kv_heads * 4, s->st));
        HS_CUDA_TRY(cudaStreamSynchronize(s->st));
    }
    return ctl_err(err);
}

int sync_ctl(hs_scratch* s) {
    HS_CUDA_TRY(cudaMemcpyAsync(s->ctl_h, s->ctl, sizeof(DevCtl), cudaMemcpyDeviceToHost, s->st));
    HS_CUDA_TRY(cudaStreamSynchronize(s->st));
    return HS_OK;
}

// Sampler width for a configuration: one candidate CTA sorts the whole
// vocabulary (vocab <= 1024, any top_k); with several, top_k <= 64 keeps 64
// keys per slice (list mode) and a larger top_k (or 0 = all) runs sort mode,
// whose buffers are allocated here at its first use.
int validate_cfg(hs_scratch* s, const hs_sampler_cfg* cfg, uint32_t* kmax) {
    const uint32_t vocab = s->m->cfg.vocab;
    const uint32_t k = cfg->top_k == 0 ? vocab : std::min(cfg->top_k, vocab);
    *kmax = s->n_cta > 1 ? kMaxTopK : kSampleSlice;
    if (*kmax > vocab) *kmax = std::min<uint32_t>(kSampleSlice, vocab);
    if (cfg->temperature > 0.0f && s->n_cta > 1 && k > kMaxTopK) {
        *kmax = s->slice;
        if (!s->sort_cand) {
            HS_CUDA_TRY(cudaSetDevice(s->m->device));
            HS_CUDA_TRY(cudaMalloc(&s->sort_cand, (size_t)s->n_cta * s->slice * 8));
            HS_CUDA_TRY(cudaMalloc(&s->wkeys, (size_t)vocab * 8));
            HS_CUDA_TRY(cudaMalloc(&s->wps, (size_t)vocab * 4));
        }
    }
    return HS_OK;
}

}  // namespace
}  // namespace hs

extern "C" {

const char* hs_last_error(void) { return g_err.c_str(); }

int hs_model_load(const char* path, uint32_t max_ctx, int device, hs_model** out) {
    return hs_model_load_ex(path, max_ctx, device, HS_NUMERIC_REFERENCE, out);
}

int hs_model_load_ex(const char* path, uint32_t max_ctx, int device, uint32_t numeric, hs_model** out) {
    if (!path || !out) return fail(HS_E_ARG, "null argument");
    if (numeric > HS_NUMERIC_TC) return fail(HS_E_ARG, "unknown numeric path");
    if (max_ctx == 0) return fail(HS_E_ARG, "max_ctx must be positive");
    *out = nullptr;
    Gguf g;
    int rc = g.open(path);
    if (rc) return rc;
    std::string arch;
    if ((rc = g.get_str("general.architecture", &arch))) return rc;
    if (arch != "qwen2") return fail(HS_E_IO, "general.architecture = \"" + arch + "\"; only qwen2 is implemented");
    auto k = [&](const char* s) { return arch + "." + s; };
    uint32_t n_layers, d_model, d_ff, n_heads, n_kv, train_ctx, eos;
    float eps, rope_base;
    if ((rc = g.get_u32(k("block_count"), &n_layers)) || (rc = g.get_u32(k("embedding_length"), &d_model)) ||
        (rc = g.get_u32(k("feed_forward_length"), &d_ff)) || (rc = g.get_u32(k("attention.head_count"), &n_heads)) ||
        (rc = g.get_u32(k("attention.head_count_kv"), &n_kv)) ||
        (rc = g.get_f32(k("attention.layer_norm_rms_epsilon"), &eps)))
        return rc;
    if (g.get_f32(k("rope.freq_base"), &rope_base) != HS_OK) rope_base = 10000.0f;  // model.rs:127
    if ((rc = g.get_u32(k("context_length"), &train_ctx))) return rc;
    uint64_t vocab = 0, n_merges = 0;
    if ((rc = g.get_str_array_len("tokenizer.ggml.tokens", &vocab)) ||
        (rc = g.get_str_array_len("tokenizer.ggml.merges", &n_merges)) ||
        (rc = g.get_u32("tokenizer.ggml.eos_token_id", &eos)))
        return rc;
    if (!n_heads || !n_kv || d_model % n_heads || n_heads % n_kv)
        return fail(HS_E_IO, "inconsistent attention shape");
    const uint32_t hd = d_model / n_heads;
    if (hd != 64 && hd != 128) return fail(HS_E_UNSUPPORTED, "head_dim must be 64 or 128");
    if (d_model % 64 || d_ff % 64) return fail(HS_E_UNSUPPORTED, "d_model and d_ff must be multiples of 64");

    auto m = std::make_unique<hs_model>();
    m->device = device;
    HS_CUDA_TRY(cudaSetDevice(device));
    HS_CUDA_TRY(cudaDeviceGetAttribute(&m->n_sm, cudaDevAttrMultiProcessorCount, device));
    int optin = 0;
    HS_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    m->smem_cap = (size_t)optin;
    HS_CUDA_TRY(gemv_set_smem_limits(optin));
    HS_CUDA_TRY(fast_set_smem_limits(optin));
    HS_CUDA_TRY(tc_set_smem_limits(optin));
    m->numeric = numeric;
    const bool fast = numeric == HS_NUMERIC_FAST, tc = numeric == HS_NUMERIC_TC;
    hs_config& c = m->cfg;
    c.n_layers = n_layers;
    c.n_heads = n_heads;
    c.n_kv_heads = n_kv;
    c.head_dim = hd;
    c.d_model = d_model;
    c.d_ff = d_ff;
    c.vocab = (uint32_t)vocab;
    c.eps = eps;
    c.rope_base = rope_base;
    c.train_ctx = train_ctx;
    c.max_ctx = max_ctx;
    c.eos = eos;
    c.fingerprint = fingerprint_of(g);
    c.numeric = numeric;
    if (fast || tc) {
        // Mix the path into the fingerprint: workers on different numeric
        // paths must not hand sequences to each other.
        const char* tag = fast ? "hotseat-b200 numeric=fast" : "hotseat-b200 numeric=tc";
        for (const char* q = tag; *q; q++) c.fingerprint = (c.fingerprint ^ (uint8_t)*q) * 0x100000001b3ull;
    }
    if (tc && n_heads / n_kv > 8) return fail(HS_E_UNSUPPORTED, "tensor-core path supports up to 8 query heads per KV head");
    if (tc && d_model > 2048) return fail(HS_E_UNSUPPORTED, "tensor-core path supports d_model up to 2048");
    // Attention: the GPU-native paths split the cached positions over CTAs
    // (split-KV with an online softmax); the exact path keeps one CTA per
    // query head in the reference's order.
    m->attn_split = tc || fast;
    if (m->attn_split) {
        // Batch 1 spreads a sequence's positions over many CTAs (64 per
        // split); a batch already has a (sequence, KV head) item per SM or
        // more, so the tensor-core path splits only past 1024 positions per
        // split: no combine at short contexts. Both depend on max_ctx only,
        // never on the batch.
        // At head_dim 128 an item holds most of an SM's shared memory (one CTA
        // per SM), so its splits are shorter: measured on the 1.5B shape at
        // batch 16 and 2-2.5k positions (4 splits, one wave of 128 items),
        // attention 35.4 µs per layer at 704 positions against 41.6 at 1024
        // and 45.6 at 640 (two waves).
        const uint32_t tc_split =
            (std::max<uint32_t>(64, env_u32("HS_TC_SPLIT_POSITIONS", hd == 128 ? 704 : 1024)) + 63) / 64 * 64;
        // ... and n cut into ceil(n / tc_split) equal splits: a 1k context
        // under a 32k max_ctx is 2 items, not 17 of 64 positions
        // (HS_TC_MIN_SPLIT=0: spread over max_splits)
        m->attn_min_split = tc && env_u32("HS_TC_MIN_SPLIT", 1) != 0 ? tc_split : 0u;
        m->max_splits = tc ? std::min<uint32_t>(128, std::max<uint32_t>(1, (max_ctx + tc_split - 1) / tc_split))
                           : attn_max_splits(max_ctx);
        m->attn_head_split = std::max<uint32_t>(1, env_u32("HS_ATTN_HEAD_SPLIT", 1));
        m->attn_nbuf = env_u32("HS_ATTN_NBUF", 0);
        m->attn_unstaged = env_u32("HS_ATTN_UNSTAGED_COMBINE", 0);
        // The GPU-native path's persistent token kernel runs its items with one
        // chunk buffer, and its per-kernel form must run the same arithmetic:
        // warp-split only where the one-buffer item holds it.
        // Measured: the warp-split form is faster at batch 1 from about 8k
        // positions (512-position items, several blocks per warp) and slower
        // below and on the batched path, where the chunked form stays.
        // HS_ATTN_WS_FROM overrides (positions; 0 = never).
        m->attn_ws_from = env_u32("HS_ATTN_WS_FROM", tc ? 0u : 8192u);
        // Tensor-core path at head_dim 64 with four chunk buffers: the items'
        // products on mma.sync with f16 hi/lo operands, positions split over
        // the 8 warps (HS_ATTN_TCW=0 keeps the chunked tf32 form).
        // The form stages its own blocks, so the chunk-buffer knob does not
        // apply to it: its launches always take the default item space (four
        // buffers at head_dim 64, three at 128), which fixes its warp count.
        m->attn_tcw = tc && (hd == 64 || hd == 128) && env_u32("HS_ATTN_TCW", 1) != 0 ? 1u : 0u;
        if (!tc && !attn_ws_fits(hd, 1)) m->attn_ws_from = 0;
        HS_CUDA_TRY(attn_split_set_smem_limits(optin));
        // Prefill attends by query blocks (128 rows share each K/V chunk,
        // products on the tensor cores); HS_PREFILL_ATTN=1 runs 64-row blocks
        // on the CUDA cores, 0 the per-token split items (measurement).
        const uint32_t pf_mode = env_u32("HS_PREFILL_ATTN", 2);
        if (tc && attn_prefill_supported(hd, n_heads, n_kv) && pf_mode != 0 &&
            attn_prefill_smem(hd, pf_mode >= 2) <= (size_t)optin) {
            m->pf_qblock = true;
            m->pf_tc = pf_mode >= 2;
            m->pf_seg = attn_prefill_seg(max_ctx);
            // HS_PREFILL_SEG (a multiple of 64 giving at most 32 segments):
            // another segment length, for measurement
            const uint32_t want = env_u32("HS_PREFILL_SEG", 0);
            if (want >= 64 && want % 64 == 0 && (max_ctx + want - 1) / want <= kPrefillMaxSegs) m->pf_seg = want;
            m->pf_nseg = (max_ctx + m->pf_seg - 1) / m->pf_seg;
            HS_CUDA_TRY(attn_prefill_set_smem_limits(optin));
        }
    }
    m->attn_smem = m->attn_split ? attn_split_smem(hd, m->attn_nbuf) : attention_smem(hd, max_ctx);
    if (!m->attn_split && m->attn_smem > m->smem_cap) {
        // Long contexts: the scores move to a global buffer (L2-resident per head).
        m->attn_global = true;
        m->attn_smem = attention_smem(hd, 0);
    }
    // Fast path: the whole token as one persistent kernel when the shapes
    // fit (HS_TOKEN_KERNEL=0 keeps the per-kernel launches; same bits).
    if (fast && env_u32("HS_TOKEN_KERNEL", 1) != 0 &&
        token_fast_plan(&m->tokp, n_layers, d_model, d_ff, n_heads, n_kv, hd, (uint32_t)vocab, m->n_sm,
                        std::min<size_t>(m->smem_cap, (size_t)env_u32("HS_TOKEN_SMEM_KB", 1024) * 1024),
                        env_u32("HS_TOKEN_SLOT_KB", 0) * 1024)) {
        HS_CUDA_TRY(token_fast_set_smem_limits(optin));
        m->tok = token_fast_resident(m->tokp);
    }
    if (m->attn_smem > m->smem_cap) return fail(HS_E_UNSUPPORTED, "attention staging does not fit in shared memory");

    // Staging buffer for the largest quantised tensor.
    uint64_t max_raw = 0;
    for (const auto& name : g.order()) max_raw = std::max(max_raw, g.tensor(name)->len);
    uint8_t* staging = nullptr;
    HS_CUDA_TRY(cudaMalloc(&staging, max_raw + 16));
    cudaStream_t st = nullptr;
    HS_CUDA_TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    struct Cleanup {
        uint8_t* p;
        cudaStream_t s;
        ~Cleanup() {
            cudaFree(p);
            cudaStreamDestroy(s);
        }
    } cleanup{staging, st};

    const uint64_t qrows = (uint64_t)(n_heads + 2 * n_kv) * hd;
    if ((rc = dev_alloc(m.get(), &m->embd, (uint64_t)vocab * d_model)) ||
        (rc = load_f16(m.get(), g, "token_embd.weight", m->embd, (uint64_t)vocab * d_model, staging, st)) ||
        (rc = dev_alloc(m.get(), &m->out_norm, d_model)) ||
        (rc = load_f32(m.get(), g, "output_norm.weight", m->out_norm, d_model)))
        return rc;
    const uint16_t* head_w = m->embd;  // tied to the embedding unless output.weight exists (model.rs:163-166)
    if (g.tensor("output.weight")) {
        if ((rc = dev_alloc(m.get(), &m->out_w, (uint64_t)vocab * d_model)) ||
            (rc = load_f16(m.get(), g, "output.weight", m->out_w, (uint64_t)vocab * d_model, staging, st)))
            return rc;
        head_w = m->out_w;
    }
    m->layers.resize(n_layers);
    for (uint32_t i = 0; i < n_layers; i++) {
        LayerDev& L = m->layers[i];
        std::string p = "blk." + std::to_string(i) + ".";
        const uint64_t dq = (uint64_t)n_heads * hd * d_model, dk = (uint64_t)n_kv * hd * d_model;
        if ((rc = dev_alloc(m.get(), &L.attn_norm, d_model)) || (rc = dev_alloc(m.get(), &L.ffn_norm, d_model)) ||
            (rc = dev_alloc(m.get(), &L.bqkv, qrows)) || (rc = dev_alloc(m.get(), &L.wqkv, qrows * d_model)) ||
            (rc = dev_alloc(m.get(), &L.wo, (uint64_t)d_model * n_heads * hd)) ||
            (rc = dev_alloc(m.get(), &L.wgate, (uint64_t)d_ff * d_model)) ||
            (rc = dev_alloc(m.get(), &L.wup, (uint64_t)d_ff * d_model)) ||
            (rc = dev_alloc(m.get(), &L.wdown, (uint64_t)d_model * d_ff)))
            return rc;
        // Wq, Wk, Wv stacked row-wise into one matrix, biases likewise.
        if ((rc = load_f32(m.get(), g, p + "attn_norm.weight", L.attn_norm, d_model)) ||
            (rc = load_f16(m.get(), g, p + "attn_q.weight", L.wqkv, dq, staging, st)) ||
            (rc = load_f32(m.get(), g, p + "attn_q.bias", L.bqkv, (uint64_t)n_heads * hd)) ||
            (rc = load_f16(m.get(), g, p + "attn_k.weight", L.wqkv + dq, dk, staging, st)) ||
            (rc = load_f32(m.get(), g, p + "attn_k.bias", L.bqkv + n_heads * hd, (uint64_t)n_kv * hd)) ||
            (rc = load_f16(m.get(), g, p + "attn_v.weight", L.wqkv + dq + dk, dk, staging, st)) ||
            (rc = load_f32(m.get(), g, p + "attn_v.bias", L.bqkv + (n_heads + n_kv) * hd, (uint64_t)n_kv * hd)) ||
            (rc = load_f16(m.get(), g, p + "attn_output.weight", L.wo, (uint64_t)d_model * n_heads * hd, staging, st)) ||
            (rc = load_f32(m.get(), g, p + "ffn_norm.weight", L.ffn_norm, d_model)) ||
            (rc = load_f16(m.get(), g, p + "ffn_gate.weight", L.wgate, (uint64_t)d_ff * d_model, staging, st)) ||
            (rc = load_f16(m.get(), g, p + "ffn_up.weight", L.wup, (uint64_t)d_ff * d_model, staging, st)) ||
            (rc = load_f16(m.get(), g, p + "ffn_down.weight", L.wdown, (uint64_t)d_model * d_ff, staging, st)))
            return rc;
        if (tc) {
            if ((rc = plan_tc(&L.tq, TC_PART, (uint32_t)qrows, d_model, L.wqkv, nullptr, m->n_sm, m->smem_cap)) ||
                (rc = plan_tc(&L.to, TC_PART, d_model, n_heads * hd, L.wo, nullptr, m->n_sm, m->smem_cap)) ||
                (rc = plan_tc(&L.tgu, TC_SILU, d_ff, d_model, L.wgate, L.wup, m->n_sm, m->smem_cap)) ||
                (rc = plan_tc(&L.tdown, TC_PART, d_model, d_ff, L.wdown, nullptr, m->n_sm, m->smem_cap)))
                return rc;
            if ((rc = plan_tc(&L.pq, TC_PART, (uint32_t)qrows, d_model, L.wqkv, nullptr, m->n_sm, m->smem_cap, true)) ||
                (rc = plan_tc(&L.po, TC_PART, d_model, n_heads * hd, L.wo, nullptr, m->n_sm, m->smem_cap, true)) ||
                (rc = plan_tc(&L.pgu, TC_SILU, d_ff, d_model, L.wgate, L.wup, m->n_sm, m->smem_cap, true)) ||
                (rc = plan_tc(&L.pdown, TC_PART, d_model, d_ff, L.wdown, nullptr, m->n_sm, m->smem_cap, true)))
                return rc;
            for (const TcGemmPlan* q : {&L.tq, &L.to, &L.tdown, &L.pq, &L.po, &L.pdown})
                m->tc_part_per_slot = std::max<uint64_t>(m->tc_part_per_slot, (uint64_t)q->splits * q->rows);
            continue;
        }
        auto plan = fast ? plan_gemv_fast : plan_gemv;
        if ((rc = plan(&L.qkv, IN_NORM, OUT_STORE, (uint32_t)qrows, d_model, L.wqkv, nullptr, m->n_sm, m->smem_cap)) ||
            (rc = plan(&L.o, IN_PLAIN, OUT_RESID, d_model, n_heads * hd, L.wo, nullptr, m->n_sm, m->smem_cap)) ||
            (rc = plan(&L.gu, IN_NORM, OUT_SILU, d_ff, d_model, L.wgate, L.wup, m->n_sm, m->smem_cap)) ||
            (rc = plan(&L.down, IN_PLAIN, OUT_RESID, d_model, d_ff, L.wdown, nullptr, m->n_sm, m->smem_cap)))
            return rc;
    }
    m->head_w = head_w;
    if (m->tok) {
        std::vector<TokLayer> tl(n_layers);
        for (uint32_t l = 0; l < n_layers; l++) {
            const LayerDev& L = m->layers[l];
            tl[l] = TokLayer{L.attn_norm, L.ffn_norm, L.bqkv, L.wqkv, L.wo, L.wgate, L.wup, L.wdown};
        }
        if ((rc = dev_alloc(m.get(), &m->tok_layers, n_layers))) return rc;
        HS_CUDA_TRY(cudaMemcpy(m->tok_layers, tl.data(), n_layers * sizeof(TokLayer), cudaMemcpyHostToDevice));
    }
    if (tc) {
        if ((rc = plan_tc(&m->thead, TC_STORE, (uint32_t)vocab, d_model, head_w, nullptr, m->n_sm, m->smem_cap)))
            return rc;
    } else if ((rc = (fast ? plan_gemv_fast : plan_gemv)(&m->head, IN_NORM, OUT_STORE, (uint32_t)vocab, d_model, head_w,
                                                          nullptr, m->n_sm, m->smem_cap))) {
        return rc;
    }
    std::vector<float> cs, sn;
    rope_tables(hd, max_ctx, rope_base, &cs, &sn);
    if ((rc = dev_alloc(m.get(), &m->rope_cos, cs.size())) || (rc = dev_alloc(m.get(), &m->rope_sin, sn.size())))
        return rc;
    HS_CUDA_TRY(cudaMemcpy(m->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    HS_CUDA_TRY(cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    *out = m.release();
    return HS_OK;
}

int hs_model_config(const hs_model* m, hs_config* out) {
    if (!m || !out) return fail(HS_E_ARG, "null argument");
    *out = m->cfg;
    return HS_OK;
}

void hs_model_free(hs_model* m) { delete m; }

int hs_model_tensor(const hs_model* m, const char* name, void* host, uint64_t bytes, uint32_t* dtype_out) {
    if (!m || !name) return fail(HS_E_ARG, "null argument");
    auto it = m->tensors.find(name);
    if (it == m->tensors.end()) return fail(HS_E_ARG, std::string("no tensor \"") + name + "\"");
    const TensorRef& t = it->second;
    uint64_t need = t.count * (t.dtype == 1 ? 2 : 4);
    if (dtype_out) *dtype_out = t.dtype;
    if (!host) return bytes == 0 ? (int)HS_OK : fail(HS_E_ARG, "null buffer");
    if (bytes < need) return fail(HS_E_ARG, "buffer too small: need " + std::to_string(need) + " bytes");
    HS_CUDA_TRY(cudaSetDevice(m->device));
    HS_CUDA_TRY(cudaMemcpy(host, t.ptr, need, cudaMemcpyDeviceToHost));
    return HS_OK;
}

// ---------------------------------------------------------------- KV cache

int hs_kv_alloc(const hs_model* m, uint32_t layout, uint32_t page_size, hs_kv** out) {
    if (!m || !out) return fail(HS_E_ARG, "null argument");
    if (layout > 1) return fail(HS_E_ARG, "unknown KV layout");
    if (page_size < 256 || (page_size & (page_size - 1))) return fail(HS_E_ARG, "page_size must be a power of two >= 256");
    HS_CUDA_TRY(cudaSetDevice(m->device));
    auto kv = std::make_unique<hs_kv>();
    kv->device = m->device;
    kv->spec = hs_kv_spec{m->cfg.n_layers, m->cfg.n_kv_heads, m->cfg.head_dim, m->cfg.max_ctx, layout};
    kv->bytes = (uint64_t)kv->spec.n_layers * 2 * kv->spec.max_ctx * kv->spec.n_kv_heads * kv->spec.head_dim * 4;
    kv->page_size = page_size;
    kv->page_shift = (uint32_t)__builtin_ctz(page_size);
    kv->n_pages = (kv->bytes + page_size - 1) / page_size;
    kv->n_words = (kv->n_pages + 63) / 64;
    kv->fingerprint = m->cfg.fingerprint;
    HS_CUDA_TRY(cudaStreamCreateWithFlags(&kv->st, cudaStreamNonBlocking));
    HS_CUDA_TRY(cudaMalloc(&kv->base, kv->bytes));
    HS_CUDA_TRY(cudaMemset(kv->base, 0, kv->bytes));
    HS_CUDA_TRY(cudaMalloc(&kv->dirty, kv->n_words * 8));
    HS_CUDA_TRY(cudaMemset(kv->dirty, 0, kv->n_words * 8));
    HS_CUDA_TRY(cudaMalloc(&kv->harvest_buf, kv->n_words * 8));
    HS_CUDA_TRY(cudaMalloc(&kv->tracking, 4));
    HS_CUDA_TRY(cudaMemset(kv->tracking, 0, 4));
    HS_CUDA_TRY(cudaEventCreateWithFlags(&kv->tab_ev, cudaEventDisableTiming));
    kv->n_sm = m->n_sm;
    *out = kv.release();
    return HS_OK;
}

int hs_kv_ipc_handle(hs_kv* kv, void* out, uint64_t out_bytes) {
    if (!kv || !out) return fail(HS_E_ARG, "null argument");
    if (out_bytes < sizeof(cudaIpcMemHandle_t)) return fail(HS_E_ARG, "handle buffer smaller than HS_IPC_HANDLE_BYTES");
    if (kv->ipc_view) return fail(HS_E_ARG, "the region belongs to another process");
    HS_CUDA_TRY(cudaSetDevice(kv->device));
    cudaIpcMemHandle_t h;
    HS_CUDA_TRY(cudaIpcGetMemHandle(&h, kv->base));
    std::memcpy(out, &h, sizeof h);
    return HS_OK;
}

int hs_kv_open_ipc(const hs_model* m, const void* handle, uint32_t layout, uint32_t page_size, hs_kv** out) {
    if (!m || !handle || !out) return fail(HS_E_ARG, "null argument");
    if (layout > 1) return fail(HS_E_ARG, "unknown KV layout");
    if (page_size < 256 || (page_size & (page_size - 1))) return fail(HS_E_ARG, "page_size must be a power of two >= 256");
    HS_CUDA_TRY(cudaSetDevice(m->device));
    auto kv = std::make_unique<hs_kv>();
    kv->device = m->device;
    kv->spec = hs_kv_spec{m->cfg.n_layers, m->cfg.n_kv_heads, m->cfg.head_dim, m->cfg.max_ctx, layout};
    kv->bytes = (uint64_t)kv->spec.n_layers * 2 * kv->spec.max_ctx * kv->spec.n_kv_heads * kv->spec.head_dim * 4;
    kv->page_size = page_size;
    kv->page_shift = (uint32_t)__builtin_ctz(page_size);
    kv->n_pages = (kv->bytes + page_size - 1) / page_size;
    kv->n_words = (kv->n_pages + 63) / 64;
    kv->fingerprint = m->cfg.fingerprint;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof h);
    void* p = nullptr;
    HS_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    kv->base = static_cast<float*>(p);
    kv->ipc_view = true;
    HS_CUDA_TRY(cudaStreamCreateWithFlags(&kv->st, cudaStreamNonBlocking));
    // the view is written and read, never decoded into: its own page bits
    // exist only so that every region has them
    HS_CUDA_TRY(cudaMalloc(&kv->dirty, kv->n_words * 8));
    HS_CUDA_TRY(cudaMemset(kv->dirty, 0, kv->n_words * 8));
    HS_CUDA_TRY(cudaMalloc(&kv->harvest_buf, kv->n_words * 8));
    HS_CUDA_TRY(cudaMalloc(&kv->tracking, 4));
    HS_CUDA_TRY(cudaMemset(kv->tracking, 0, 4));
    HS_CUDA_TRY(cudaEventCreateWithFlags(&kv->tab_ev, cudaEventDisableTiming));
    kv->n_sm = m->n_sm;
    *out = kv.release();
    return HS_OK;
}

int hs_kv_fingerprint(const hs_kv* kv, uint64_t* out) {
    if (!kv || !out) return fail(HS_E_ARG, "null argument");
    *out = kv->fingerprint;
    return HS_OK;
}

int hs_kv_info(const hs_kv* kv, hs_kv_spec* spec, uint64_t* bytes, uint32_t* page_size, uint64_t* n_pages) {
    if (!kv) return fail(HS_E_ARG, "null argument");
    if (spec) *spec = kv->spec;
    if (bytes) *bytes = kv->bytes;
    if (page_size) *page_size = kv->page_size;
    if (n_pages) *n_pages = kv->n_pages;
    return HS_OK;
}

void hs_kv_free(hs_kv* kv) { delete kv; }

int hs_kv_read(hs_kv* kv, uint64_t off, uint64_t len, void* host) {
    if (!kv || (!host && len)) return fail(HS_E_ARG, "null argument");
    if (off > kv->bytes || len > kv->bytes - off) return fail(HS_E_ARG, "range outside the KV region");
    HS_CUDA_TRY(cudaSetDevice(kv->device));
    HS_CUDA_TRY(cudaMemcpy(host, reinterpret_cast<uint8_t*>(kv->base) + off, len, cudaMemcpyDeviceToHost));
    return HS_OK;
}

int hs_kv_write(hs_kv* kv, uint64_t off, uint64_t len, const void* host) {
    if (!kv || (!host && len)) return fail(HS_E_ARG, "null argument");
    if (off > kv->bytes || len > kv->bytes - off) return fail(HS_E_ARG, "range outside the KV region");
    HS_CUDA_TRY(cudaSetDevice(kv->device));
    HS_CUDA_TRY(cudaMemcpy(reinterpret_cast<uint8_t*>(kv->base) + off, host, len, cudaMemcpyHostToDevice));
    return HS_OK;
}

uint64_t hs_kv_live_ranges_between(const hs_kv_spec* s, uint32_t from, uint32_t to, uint64_t* out, uint64_t cap) {
    // kv.rs:150-175
    if (!s || to <= from) return 0;
    const uint64_t plane = (uint64_t)s->max_ctx * s->n_kv_heads * s->head_dim, n = to - from;
    uint64_t count = 0;
    auto push = [&](uint64_t off, uint64_t len) {
        if (out && count < cap) {
            out[2 * count] = off;
            out[2 * count + 1] = len;
        }
        count++;
    };
    for (uint64_t layer = 0; layer < s->n_layers; layer++)
        for (int is_v = 0; is_v < 2; is_v++) {
            const uint64_t plane_off = (layer * 2 * plane + (is_v ? plane : 0)) * 4;
            if (s->layout == 0) {
                const uint64_t w = (uint64_t)s->n_kv_heads * s->head_dim * 4;
                push(plane_off + from * w, n * w);
            } else {
                const uint64_t w = (uint64_t)s->head_dim * 4;
                for (uint64_t h = 0; h < s->n_kv_heads; h++) push(plane_off + (h * s->max_ctx + from) * w, n * w);
            }
        }
    return count;
}

int hs_kv_hash(hs_kv* kv, uint32_t n_pos, uint64_t* out) {
    // kv.rs:267-274 with hash::Wide (hash.rs:63-126), over bytes staged to the host.
    if (!kv || !out) return fail(HS_E_ARG, "null argument");
    if (n_pos > kv->spec.max_ctx) return fail(HS_E_ARG, "n_pos past max_ctx");
    const uint64_t nr = hs_kv_live_ranges_between(&kv->spec, 0, n_pos, nullptr, 0);
    std::vector<uint64_t> r(2 * nr);
    hs_kv_live_ranges_between(&kv->spec, 0, n_pos, r.data(), nr);
    uint64_t lanes[4] = {0x243f6a8885a308d3ull, 0x13198a2e03707344ull, 0xa4093822299f31d0ull, 0x082efa98ec4e6c89ull};
    uint64_t total = 0;
    const uint64_t P = 0x00000100000001b3ull;
    std::vector<uint8_t> buf;
    HS_CUDA_TRY(cudaSetDevice(kv->device));
    for (uint64_t i = 0; i < nr; i++) {
        const uint64_t off = r[2 * i], len = r[2 * i + 1];
        buf.resize(len);
        HS_CUDA_TRY(cudaMemcpy(buf.data(), reinterpret_cast<uint8_t*>(kv->base) + off, len, cudaMemcpyDeviceToHost));
        total += len;
        const uint64_t full = len / 32 * 32;
        for (uint64_t c = 0; c < full; c += 32)
            for (int k = 0; k < 4; k++) {
                uint64_t w;
                std::memcpy(&w, buf.data() + c + 8 * k, 8);
                lanes[k] = (lanes[k] ^ w) * P;
                lanes[k] ^= lanes[k] >> 29;
            }
        for (uint64_t j = 0; j < len - full; j++) lanes[j % 4] = (lanes[j % 4] ^ buf[full + j]) * P;
    }
    auto rotl = [](uint64_t x, int k) { return (x << k) | (x >> (64 - k)); };
    uint64_t h = lanes[0] ^ rotl(lanes[1], 17) ^ rotl(lanes[2], 34) ^ rotl(lanes[3], 51);
    h += total;
    h ^= h >> 33;
    h *= 0xff51afd7ed558ccdull;
    h ^= h >> 33;
    *out = h;
    return HS_OK;
}

uint64_t hs_runs_to_byte_runs(const uint64_t* words, uint64_t n_pages, uint64_t page_size, const uint64_t* live,
                              uint64_t n_live, uint64_t* out, uint64_t cap) {
    // hs-track pageset.rs:79-113 (runs of set bits) clipped to the live byte
    // ranges and merged (hs-wire lib.rs:418-446).
    std::vector<std::pair<uint64_t, uint64_t>> acc;
    auto merge = [](std::vector<std::pair<uint64_t, uint64_t>>& v, uint64_t off, uint64_t len) {
        if (!v.empty() && v.back().first + v.back().second >= off) {
            uint64_t end = std::max(v.back().first + v.back().second, off + len);
            v.back().second = end - v.back().first;
            return;
        }
        v.push_back({off, len});
    };
    uint64_t p = 0;
    while (p < n_pages) {
        if (!((words[p >> 6] >> (p & 63)) & 1)) {
            p++;
            continue;
        }
        uint64_t q = p;
        while (q < n_pages && ((words[q >> 6] >> (q & 63)) & 1)) q++;
        const uint64_t a = p * page_size, b = q * page_size;
        for (uint64_t i = 0; i < n_live; i++) {
            const uint64_t lo = live[2 * i], hi = lo + live[2 * i + 1];
            const uint64_t c = std::max(a, lo), d = std::min(b, hi);
            if (c < d) merge(acc, c, d - c);
        }
        p = q;
    }
    std::stable_sort(acc.begin(), acc.end(), [](const auto& x, const auto& y) { return x.first < y.first; });
    std::vector<std::pair<uint64_t, uint64_t>> merged;
    for (auto& r : acc) merge(merged, r.first, r.second);
    for (uint64_t i = 0; i < merged.size() && i < cap && out; i++) {
        out[2 * i] = merged[i].first;
        out[2 * i + 1] = merged[i].second;
    }
    return merged.size();
}

}  // extern "C"

namespace hs {
namespace {

// Runs (off, len pairs) inside a region of `bytes` bytes; their total.
int check_runs(const uint64_t* runs, uint64_t n_runs, uint64_t bytes, uint64_t* total) {
    if (!runs && n_runs) return fail(HS_E_ARG, "null run list");
    uint64_t t = 0;
    for (uint64_t i = 0; i < n_runs; i++) {
        if (runs[2 * i] > bytes || runs[2 * i + 1] > bytes - runs[2 * i])
            return fail(HS_E_ARG, "run " + std::to_string(i) + " outside the KV region");
        t += runs[2 * i + 1];
    }
    *total = t;
    return HS_OK;
}

// The transfer table of `runs`, split into pieces of at most kXferPiece
// bytes: mode 0 region -> packed, 1 packed -> region, 2 region -> region.
std::vector<XferRun> xfer_table(const uint64_t* runs, uint64_t n_runs, int mode) {
    std::vector<XferRun> t;
    uint64_t packed = 0;
    for (uint64_t i = 0; i < n_runs; i++) {
        const uint64_t off = runs[2 * i], len = runs[2 * i + 1];
        for (uint64_t p = 0; p < len; p += kXferPiece) {
            const uint64_t n = std::min<uint64_t>(kXferPiece, len - p);
            const uint64_t r = off + p, k = packed + p;
            t.push_back(mode == 0 ? XferRun{r, k, n} : mode == 1 ? XferRun{k, r, n} : XferRun{r, r, n});
        }
        packed += len;
    }
    return t;
}

// Upload `t` into kv's device table on `st` and launch the copy there; the
// table buffers are reused only after the event that follows this kernel.
int launch_table(hs_kv* kv, const std::vector<XferRun>& t, const uint8_t* src, uint8_t* dst, cudaStream_t st) {
    if (t.empty()) return HS_OK;
    HS_CUDA_TRY(cudaEventSynchronize(kv->tab_ev));
    if (t.size() > kv->tab_cap) {
        cudaFreeHost(kv->tab_h);
        cudaFree(kv->tab_dev);
        kv->tab_h = nullptr;
        kv->tab_dev = nullptr;
        kv->tab_cap = 0;
        const uint64_t cap = std::max<uint64_t>(t.size(), 256);
        HS_CUDA_TRY(cudaMallocHost(&kv->tab_h, cap * sizeof(XferRun)));
        HS_CUDA_TRY(cudaMalloc(&kv->tab_dev, cap * sizeof(XferRun)));
        kv->tab_cap = cap;
    }
    std::memcpy(kv->tab_h, t.data(), t.size() * sizeof(XferRun));
    HS_CUDA_TRY(cudaMemcpyAsync(kv->tab_dev, kv->tab_h, t.size() * sizeof(XferRun), cudaMemcpyHostToDevice, st));
    HS_CUDA_TRY(launch_copy_runs(src, dst, kv->tab_dev, (uint32_t)t.size(), kv->n_sm, st));
    HS_CUDA_TRY(cudaEventRecord(kv->tab_ev, st));
    return HS_OK;
}

int ensure_stage(hs_kv* kv, uint64_t bytes) {
    if (bytes <= kv->stage_cap) return HS_OK;
    HS_CUDA_TRY(cudaStreamSynchronize(kv->st));
    cudaFree(kv->stage);
    kv->stage = nullptr;
    kv->stage_cap = 0;
    HS_CUDA_TRY(cudaMalloc(&kv->stage, bytes));
    kv->stage_cap = bytes;
    return HS_OK;
}

}  // namespace
}  // namespace hs

extern "C" {

int hs_kv_read_runs(hs_kv* kv, const uint64_t* runs, uint64_t n_runs, void* host, uint64_t host_bytes) {
    if (!kv) return fail(HS_E_ARG, "null KV region");
    uint64_t total;
    int rc = check_runs(runs, n_runs, kv->bytes, &total);
    if (rc) return rc;
    if (total && !host) return fail(HS_E_ARG, "null host buffer");
    if (host_bytes < total) return fail(HS_E_ARG, "host buffer smaller than the runs' bytes");
    if (!total) return HS_OK;
    HS_CUDA_TRY(cudaSetDevice(kv->device));
    if ((rc = ensure_stage(kv, total))) return rc;
    if ((rc = launch_table(kv, xfer_table(runs, n_runs, 0), reinterpret_cast<const uint8_t*>(kv->base), kv->stage,
                           kv->st)))
        return rc;
    HS_CUDA_TRY(cudaMemcpyAsync(host, kv->stage, total, cudaMemcpyDeviceToHost, kv->st));
    HS_CUDA_TRY(cudaStreamSynchronize(kv->st));
    return HS_OK;
}

int hs_kv_write_runs(hs_kv* kv, const uint64_t* runs, uint64_t n_runs, const void* host, uint64_t host_bytes) {
    if (!kv) return fail(HS_E_ARG, "null KV region");
    uint64_t total;
    int rc = check_runs(runs, n_runs, kv->bytes, &total);
    if (rc) return rc;
    if (total && !host) return fail(HS_E_ARG, "null host buffer");
    if (host_bytes < total) return fail(HS_E_ARG, "host buffer smaller than the runs' bytes");
    if (!total) return HS_OK;
    HS_CUDA_TRY(cudaSetDevice(kv->device));
    if ((rc = ensure_stage(kv, total))) return rc;
    HS_CUDA_TRY(cudaMemcpyAsync(kv->stage, host, total, cudaMemcpyHostToDevice, kv->st));
    if ((rc = launch_table(kv, xfer_table(runs, n_runs, 1), kv->stage, reinterpret_cast<uint8_t*>(kv->base),
                           kv->st)))
        return rc;
    HS_CUDA_TRY(cudaStreamSynchronize(kv->st));
    return HS_OK;
}

int hs_kv_peer_copy(hs_kv* src, hs_kv* dst, const uint64_t* runs, uint64_t n_runs, void* stream) {
    if (!src || !dst) return fail(HS_E_ARG, "null KV region");
    if (std::memcmp(&src->spec, &dst->spec, sizeof(hs_kv_spec)) != 0)
        return fail(HS_E_ARG, "KV specs differ between source and destination");
    uint64_t total;
    int rc = check_runs(runs, n_runs, src->bytes, &total);
    if (rc || !total) return rc;
    cudaStream_t st = stream ? reinterpret_cast<cudaStream_t>(stream) : src->st;
    HS_CUDA_TRY(cudaSetDevice(src->device));
    bool direct = src->device == dst->device;
    if (!direct) {
        int can = 0;
        HS_CUDA_TRY(cudaDeviceCanAccessPeer(&can, src->device, dst->device));
        if (can) {
            cudaError_t e = cudaDeviceEnablePeerAccess(dst->device, 0);
            if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled)
                return fail(HS_E_CUDA, std::string("enable peer access: ") + cudaGetErrorString(e));
            cudaGetLastError();
            direct = true;
        }
    }
    if (direct)  // one kernel: local reads, stores into the destination (over NVLink across GPUs)
        return launch_table(src, xfer_table(runs, n_runs, 2), reinterpret_cast<const uint8_t*>(src->base),
                            reinterpret_cast<uint8_t*>(dst->base), st);
    for (uint64_t i = 0; i < n_runs; i++)  // no peer mapping: the driver's peer copies
        HS_CUDA_TRY(cudaMemcpyPeerAsync(reinterpret_cast<uint8_t*>(dst->base) + runs[2 * i], dst->device,
                                        reinterpret_cast<const uint8_t*>(src->base) + runs[2 * i], src->device,
                                        runs[2 * i + 1], st));
    return HS_OK;
}

int hs_kv_copy_runs(hs_kv* src, hs_kv* dst, const uint64_t* runs, uint64_t n_runs) {
    int rc = hs_kv_peer_copy(src, dst, runs, n_runs, nullptr);
    if (rc) return rc;
    HS_CUDA_TRY(cudaSetDevice(src->device));
    HS_CUDA_TRY(cudaStreamSynchronize(src->st));
    return HS_OK;
}

// ---------------------------------------------------------------- scratch

int hs_scratch_new(const hs_model* m, hs_scratch** out) {
    if (!m || !out) return fail(HS_E_ARG, "null argument");
    if (m->numeric == HS_NUMERIC_TC)
        return fail(HS_E_UNSUPPORTED, "a tensor-core model decodes through hs_batch_* (a batch of one is fine)");
    HS_CUDA_TRY(cudaSetDevice(m->device));
    auto s = std::make_unique<hs_scratch>();
    s->m = m;
    const hs_config& c = m->cfg;
    HS_CUDA_TRY(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
    HS_CUDA_TRY(cudaMalloc(&s->ctl, sizeof(DevCtl)));
    HS_CUDA_TRY(cudaMemset(s->ctl, 0, sizeof(DevCtl)));
    HS_CUDA_TRY(cudaMallocHost(&s->ctl_h, sizeof(DevCtl)));
    std::memset(s->ctl_h, 0, sizeof(DevCtl));
    if (m->attn_global) HS_CUDA_TRY(cudaMalloc(&s->sc_global, (size_t)c.n_heads * c.max_ctx * 4));
    if (m->attn_split) {
        const uint32_t G = c.n_heads / c.n_kv_heads;
        HS_CUDA_TRY(cudaMalloc(&s->att_part, (size_t)c.n_kv_heads * m->max_splits * attn_record(G, c.head_dim) * 4));
        HS_CUDA_TRY(cudaMalloc(&s->att_cnt, c.n_kv_heads * 4));
        HS_CUDA_TRY(cudaMemset(s->att_cnt, 0, c.n_kv_heads * 4));
        HS_CUDA_TRY(cudaMalloc(&s->kv_tab, 3 * sizeof(void*)));
    }
    HS_CUDA_TRY(cudaMalloc(&s->x, c.d_model * 4));
    HS_CUDA_TRY(cudaMalloc(&s->qkv, (size_t)(c.n_heads + 2 * c.n_kv_heads) * c.head_dim * 4));
    HS_CUDA_TRY(cudaMalloc(&s->att, (size_t)c.n_heads * c.head_dim * 4));
    HS_CUDA_TRY(cudaMalloc(&s->hb, (size_t)c.d_ff * 4));
    HS_CUDA_TRY(cudaMalloc(&s->logits, (size_t)c.vocab * 4));
    s->cap = (uint64_t)c.max_ctx + 1;
    HS_CUDA_TRY(cudaMalloc(&s->tokens, s->cap * 4));
    // Large vocabularies: 4096-logit slices per candidate CTA (exact radix
    // select of the best 64); the kept candidates are the same exact top-k.
    s->slice = c.vocab > kMaxSlice ? kMaxSlice : kSampleSlice;
    s->n_cta = (c.vocab + s->slice - 1) / s->slice;
    if (s->n_cta > 256) return fail(HS_E_UNSUPPORTED, "vocab too large for the device sampler");
    HS_CUDA_TRY(cudaMalloc(&s->cand, (size_t)s->n_cta * kSampleSlice * 8));
    HS_CUDA_TRY(cudaMalloc(&s->argbuf, (size_t)s->n_cta * 8));
    if (m->tok) {
        const size_t bytes = 16 + tok_bufs(m).total * 8;
        HS_CUDA_TRY(cudaMalloc(&s->tok_mem, bytes));
        HS_CUDA_TRY(cudaMemset(s->tok_mem, 0, bytes));  // counter 0, tags 0 (no launch writes tag 0)
    }
    s->launches_fwd = m->tok ? 1 : c.n_layers * 5 + 1;
    const char* penv = getenv("HS_POLL_LIMIT");
    if (penv && *penv) s->poll_limit = (uint32_t)std::strtoul(penv, nullptr, 10);
    const char* tenv = getenv("HS_TRACE");
    if (tenv && tenv[0] == '1') {
        s->trace_slots = s->launches_fwd + 2 + (m->tok ? (20 * (5 * c.n_layers + 1) + 7) / 8 : 0);
        HS_CUDA_TRY(cudaMalloc(&s->trace, (size_t)s->trace_slots * 8 * 8));
        HS_CUDA_TRY(cudaMallocHost(&s->trace_init, (size_t)s->trace_slots * 8 * 8));
        for (uint32_t i = 0; i < s->trace_slots; i++) {
            // launch slots start at ~0 (the entry is a minimum); the token
            // kernel's timeline words after them start at 0
            s->trace_init[8 * i] = i < s->launches_fwd + 2 ? ~0ull : 0;
            for (int j = 1; j < 8; j++) s->trace_init[8 * i + j] = 0;
        }
    }
    *out = s.release();
    return HS_OK;
}

void hs_scratch_free(hs_scratch* s) { delete s; }

void* hs_scratch_stream(hs_scratch* s) { return s ? (void*)s->st : nullptr; }

int hs_scratch_trace(hs_scratch* s, uint64_t* out, uint64_t n_slots, uint64_t* used) {
    if (!s || !used) return fail(HS_E_ARG, "null argument");
    *used = s->trace_slots;
    if (!s->trace) return fail(HS_E_STATE, "tracing is off (set HS_TRACE=1 before creating the scratch)");
    if (!out) return HS_OK;
    HS_CUDA_TRY(cudaSetDevice(s->m->device));
    HS_CUDA_TRY(cudaStreamSynchronize(s->st));
    HS_CUDA_TRY(cudaMemcpy(out, s->trace, std::min<uint64_t>(n_slots, s->trace_slots) * 64, cudaMemcpyDeviceToHost));
    return HS_OK;
}

int hs_seq_launches_per_step(hs_scratch* s, uint32_t* out) {
    if (!s || !out) return fail(HS_E_ARG, "null argument");
    *out = s->launches_fwd + (sample_sort_mode(s->n_cta, s->kmax) ? 3 : 2);
    return HS_OK;
}

int hs_forward(const hs_model* m, hs_kv* kv, uint32_t token, uint32_t pos, hs_scratch* s) {
    if (!m || !kv || !s || s->m != m) return fail(HS_E_ARG, "null or mismatched argument");
    int rc = check_kv(m, kv);
    if (rc) return rc;
    if (pos >= m->cfg.max_ctx)
        return fail(HS_E_ARG, "position " + std::to_string(pos) + " past max_ctx " + std::to_string(m->cfg.max_ctx));
    if (token >= m->cfg.vocab) return fail(HS_E_ARG, "token " + std::to_string(token) + " out of range");
    HS_CUDA_TRY(cudaSetDevice(m->device));
    if ((rc = ensure_graphs(s, kv, s->kmax ? s->kmax : kMaxTopK))) return rc;
    DevCtl& h = *s->ctl_h;
    std::memset(&h, 0, sizeof(DevCtl));
    h.token = token;
    h.pos = pos;
    h.active = 1;
    h.mode = 0;
    h.vocab = m->cfg.vocab;
    h.max_ctx = m->cfg.max_ctx;
    HS_CUDA_TRY(cudaMemcpyAsync(s->ctl, &h, sizeof(DevCtl), cudaMemcpyHostToDevice, s->st));
    if ((rc = refresh_tags(s))) return rc;
    HS_CUDA_TRY(cudaGraphLaunch(s->g_fwd, s->st));
    if ((rc = sync_ctl(s))) return rc;
    return check_ctl_err(s);
}

int hs_scratch_logits(hs_scratch* s, float* host, uint64_t n) {
    if (!s || !host) return fail(HS_E_ARG, "null argument");
    if (n > s->m->cfg.vocab) return fail(HS_E_ARG, "more logits requested than the vocabulary has");
    HS_CUDA_TRY(cudaSetDevice(s->m->device));
    HS_CUDA_TRY(cudaMemcpyAsync(host, s->logits, n * 4, cudaMemcpyDeviceToHost, s->st));
    HS_CUDA_TRY(cudaStreamSynchronize(s->st));
    return HS_OK;
}

int hs_scratch_nll(hs_scratch* s, uint32_t next, double* out) {
    if (!s || !out) return fail(HS_E_ARG, "null argument");
    if (next >= s->m->cfg.vocab) return fail(HS_E_ARG, "token out of range");
    HS_CUDA_TRY(cudaSetDevice(s->m->device));
    if (!s->nll) {
        HS_CUDA_TRY(cudaMalloc(&s->nll, 8));
        HS_CUDA_TRY(cudaMalloc(&s->nll_next, 4));
    }
    HS_CUDA_TRY(cudaMemcpyAsync(s->nll_next, &next, 4, cudaMemcpyHostToDevice, s->st));
    HS_CUDA_TRY(launch_logits_nll(s->logits, s->m->cfg.vocab, s->nll_next, 1, s->m->cfg.vocab, s->nll, s->st));
    HS_CUDA_TRY(cudaMemcpyAsync(out, s->nll, 8, cudaMemcpyDeviceToHost, s->st));
    HS_CUDA_TRY(cudaStreamSynchronize(s->st));
    return HS_OK;
}

int hs_scratch_set_logits(hs_scratch* s, const float* host, uint64_t n) {
    if (!s || !host) return fail(HS_E_ARG, "null argument");
    if (n != s->m->cfg.vocab) return fail(HS_E_ARG, "expected exactly vocab logits");
    HS_CUDA_TRY(cudaSetDevice(s->m->device));
    HS_CUDA_TRY(cudaMemcpyAsync(s->logits, host, n * 4, cudaMemcpyHostToDevice, s->st));
    HS_CUDA_TRY(cudaStreamSynchronize(s->st));
    return HS_OK;
}

void hs_sampler_cfg_default(hs_sampler_cfg* c) {
    if (!c) return;
    c->temperature = 0.8f;
    c->top_p = 0.95f;
    c->top_k = 40;
    c->repeat_penalty = 1.1f;
    c->repeat_last_n = 64;
    c->seed = 0xC0FFEE0012345678ull;
}

void hs_rng_seed(uint64_t seed, hs_rng* r) {
    // sampler.rs:47-58
    if (!r) return;
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

static void fill_cfg(DevCtl& h, const hs_sampler_cfg* cfg, const hs_rng* rng) {
    h.temperature = cfg->temperature;
    h.top_p = cfg->top_p;
    h.top_k = cfg->top_k;
    h.repeat_penalty = cfg->repeat_penalty;
    h.repeat_last_n = cfg->repeat_last_n;
    for (int i = 0; i < 4; i++) h.rng[i] = rng->s[i];
    h.draws = rng->draws;
}

int hs_sample(hs_scratch* s, const hs_sampler_cfg* cfg, hs_rng* rng, const uint32_t* hist, uint64_t n_hist,
              uint32_t* out) {
    if (!s || !cfg || !rng || !out || (!hist && n_hist)) return fail(HS_E_ARG, "null argument");
    uint32_t kmax;
    int rc = validate_cfg(s, cfg, &kmax);
    if (rc) return rc;
    const hs_model* m = s->m;
    // Only the tail the penalty reads matters (sampler.rs:103-111).
    const uint64_t win = (cfg->repeat_penalty != 1.0f && cfg->repeat_last_n > 0)
                             ? std::min<uint64_t>(cfg->repeat_last_n, n_hist)
                             : 0;
    if (win > s->cap) return fail(HS_E_UNSUPPORTED, "repeat_last_n longer than max_ctx");
    hist += n_hist - win;
    n_hist = win;
    for (uint64_t i = 0; i < n_hist; i++)
        if (hist[i] >= m->cfg.vocab) return fail(HS_E_ARG, "history token out of range");
    HS_CUDA_TRY(cudaSetDevice(m->device));
    s->kmax = kmax;
    DevCtl& h = *s->ctl_h;
    std::memset(&h, 0, sizeof(DevCtl));
    h.mode = 1;
    h.n_tokens = n_hist;
    h.vocab = m->cfg.vocab;
    h.max_ctx = m->cfg.max_ctx;
    fill_cfg(h, cfg, rng);
    if (n_hist) HS_CUDA_TRY(cudaMemcpyAsync(s->tokens, hist, n_hist * 4, cudaMemcpyHostToDevice, s->st));
    HS_CUDA_TRY(cudaMemcpyAsync(s->ctl, &h, sizeof(DevCtl), cudaMemcpyHostToDevice, s->st));
    cudaError_t e = launch_sample(sample_args(s), s->st);
    if (e != cudaSuccess) return fail(HS_E_CUDA, std::string("sampler launch: ") + cudaGetErrorString(e));
    if ((rc = sync_ctl(s))) return rc;
    if ((rc = check_ctl_err(s))) return rc;
    *out = s->ctl_h->out_token;
    for (int i = 0; i < 4; i++) rng->s[i] = s->ctl_h->rng[i];
    rng->draws = s->ctl_h->draws;
    return HS_OK;
}

int hs_argmax(hs_scratch* s, uint32_t* out) {
    hs_sampler_cfg cfg{};
    cfg.temperature = 0.0f;
    cfg.top_p = 1.0f;
    cfg.top_k = 1;
    cfg.repeat_penalty = 1.0f;
    hs_rng r{};
    return hs_sample(s, &cfg, &r, nullptr, 0, out);
}

// ---------------------------------------------------------------- the loop

int hs_seq_begin(hs_scratch* s, hs_kv* kv, const uint32_t* tokens, uint64_t n_tokens, uint64_t cap,
                 const hs_seq_state* st, const hs_sampler_cfg* cfg, const hs_rng* rng, uint64_t stop_at_filled) {
    if (!s || !kv || !tokens || !st || !cfg || !rng) return fail(HS_E_ARG, "null argument");
    const hs_model* m = s->m;
    int rc = check_kv(m, kv);
    if (rc) return rc;
    if (n_tokens == 0 || st->filled > n_tokens || st->prompt_len > n_tokens)
        return fail(HS_E_ARG, "inconsistent sequence state");
    if (n_tokens > s->cap) return fail(HS_E_ARG, "history longer than max_ctx");
    for (uint64_t i = 0; i < n_tokens; i++)
        if (tokens[i] >= m->cfg.vocab) return fail(HS_E_ARG, "token " + std::to_string(tokens[i]) + " out of range");
    uint32_t kmax;
    if ((rc = validate_cfg(s, cfg, &kmax))) return rc;
    HS_CUDA_TRY(cudaSetDevice(m->device));
    if ((rc = ensure_graphs(s, kv, kmax))) return rc;
    DevCtl& h = *s->ctl_h;
    std::memset(&h, 0, sizeof(DevCtl));
    h.mode = 0;
    h.n_tokens = n_tokens;
    h.filled = st->filled;
    h.prompt_len = st->prompt_len;
    h.max_tokens = st->max_tokens;
    h.cap = std::min<uint64_t>(cap, s->cap);
    h.stop_at = stop_at_filled;
    h.done = st->done;
    h.done_reason = st->done_reason;
    h.eos = m->cfg.eos;
    h.max_ctx = m->cfg.max_ctx;
    h.vocab = m->cfg.vocab;
    fill_cfg(h, cfg, rng);
    const bool runnable = !st->done && st->filled < n_tokens && !(stop_at_filled && st->filled >= stop_at_filled);
    if (!st->done && st->filled >= n_tokens) return fail(HS_E_STATE, "internal: nothing to feed at the token boundary");
    if (runnable && st->filled >= m->cfg.max_ctx) return fail(HS_E_ARG, "position past max_ctx");
    h.active = runnable ? 1 : 0;
    h.token = runnable ? tokens[st->filled] : 0;
    h.pos = (uint32_t)st->filled;
    HS_CUDA_TRY(cudaMemcpyAsync(s->tokens, tokens, n_tokens * 4, cudaMemcpyHostToDevice, s->st));
    HS_CUDA_TRY(cudaMemcpyAsync(s->ctl, &h, sizeof(DevCtl), cudaMemcpyHostToDevice, s->st));
    return HS_OK;
}

int hs_seq_step(hs_scratch* s, uint32_t n_steps) {
    if (!s || !s->g_step) return fail(HS_E_ARG, "hs_seq_begin has not been called");
    HS_CUDA_TRY(cudaSetDevice(s->m->device));
    for (uint32_t i = 0; i < n_steps; i++) {
        if (s->trace)
            HS_CUDA_TRY(cudaMemcpyAsync(s->trace, s->trace_init, (size_t)s->trace_slots * 64, cudaMemcpyHostToDevice,
                                        s->st));
        const int rc = refresh_tags(s);
        if (rc) return rc;
        HS_CUDA_TRY(cudaGraphLaunch(s->g_step, s->st));
    }
    return HS_OK;
}

int hs_seq_end(hs_scratch* s, uint32_t* tokens, uint64_t* n_tokens, uint64_t cap, hs_seq_state* st, hs_rng* rng) {
    if (!s) return fail(HS_E_ARG, "null argument");
    HS_CUDA_TRY(cudaSetDevice(s->m->device));
    int rc = sync_ctl(s);
    if (rc) return rc;
    const DevCtl& h = *s->ctl_h;
    if (tokens && n_tokens) {
        if (h.n_tokens > cap) return fail(HS_E_ARG, "token buffer too small");
        HS_CUDA_TRY(cudaMemcpy(tokens, s->tokens, h.n_tokens * 4, cudaMemcpyDeviceToHost));
        *n_tokens = h.n_tokens;
    }
    if (st) {
        st->filled = h.filled;
        st->done = h.done;
        st->done_reason = h.done_reason;
    }
    if (rng) {
        for (int i = 0; i < 4; i++) rng->s[i] = h.rng[i];
        rng->draws = h.draws;
    }
    return check_ctl_err(s);
}

int hs_seq_run(const hs_model* m, hs_kv* kv, hs_scratch* s, uint32_t* tokens, uint64_t* n_tokens, uint64_t cap,
               hs_seq_state* st, const hs_sampler_cfg* cfg, hs_rng* rng, uint64_t stop_at_filled) {
    if (!m || !s || s->m != m || !n_tokens) return fail(HS_E_ARG, "null or mismatched argument");
    int rc = hs_seq_begin(s, kv, tokens, *n_tokens, cap, st, cfg, rng, stop_at_filled);
    if (rc) return rc;
    // Every chunk advances `filled` by at least one unless the sequence
    // stopped, so max_ctx chunks is a hard upper bound.
    for (uint32_t guard = 0;; guard++) {
        const DevCtl& h = *s->ctl_h;
        if (h.done || !h.active) break;
        if (guard > m->cfg.max_ctx) return fail(HS_E_STATE, "decode loop made no progress");
        // Forwards still possible before the sequence must stop on its own:
        // the rest of the prompt, then one per token still allowed.
        const uint64_t pre = h.n_tokens - h.filled;
        const uint64_t gen = h.n_tokens - h.prompt_len;
        uint64_t bound = pre + (h.max_tokens > gen ? h.max_tokens - gen : 0);
        if (h.stop_at && h.stop_at > h.filled) bound = std::min<uint64_t>(bound, h.stop_at - h.filled);
        bound = std::max<uint64_t>(1, std::min<uint64_t>(bound, 256));
        if ((rc = hs_seq_step(s, (uint32_t)bound))) return rc;
        if ((rc = sync_ctl(s))) return rc;
        if ((rc = check_ctl_err(s))) return rc;
    }
    return hs_seq_end(s, tokens, n_tokens, cap, st, rng);
}

int hs_dequant_f16(uint32_t ggml_type, const void* src, uint64_t n, void* dst, void* stream) {
    if ((!src || !dst) && n) return fail(HS_E_ARG, "null argument");
    int dev = 0, n_sm = 0;
    HS_CUDA_TRY(cudaGetDevice(&dev));
    HS_CUDA_TRY(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
    return launch_dequant(ggml_type, src, n, dst, static_cast<cudaStream_t>(stream), n_sm);
}

}  // extern "C"

namespace hs {
namespace {
// Take-and-clear of the dirty bitmap: a concurrent atomicOr from the
// KV-append kernel lands either in this harvest or in the next one
// (the swap of PageSet::drain_into, hs-track pageset.rs:64-72).
__global__ void k_harvest(unsigned long long* words, unsigned long long* out, uint64_t n) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = atomicExch(&words[i], 0ull);
}
}  // namespace
}  // namespace hs

extern "C" {

int hs_kv_harvest(hs_kv* kv, uint64_t* words, uint64_t n_words) {
    if (!kv || !words) return fail(HS_E_ARG, "null argument");
    if (n_words < kv->n_words) return fail(HS_E_ARG, "need " + std::to_string(kv->n_words) + " words");
    HS_CUDA_TRY(cudaSetDevice(kv->device));
    const unsigned grid = (unsigned)std::min<uint64_t>((kv->n_words + 255) / 256, 1024);
    hs::k_harvest<<<grid, 256, 0, kv->st>>>(reinterpret_cast<unsigned long long*>(kv->dirty),
                                            reinterpret_cast<unsigned long long*>(kv->harvest_buf), kv->n_words);
    HS_CUDA_TRY(cudaGetLastError());
    HS_CUDA_TRY(cudaMemcpyAsync(words, kv->harvest_buf, kv->n_words * 8, cudaMemcpyDeviceToHost, kv->st));
    HS_CUDA_TRY(cudaStreamSynchronize(kv->st));
    for (uint64_t i = kv->n_words; i < n_words; i++) words[i] = 0;
    return HS_OK;
}

// Arm and disarm run on the region's own stream and are waited for; a
// decode step may be in flight on another stream meanwhile (its appends are
// marked once the flag is set).
int hs_kv_arm(hs_kv* kv) {
    if (!kv) return fail(HS_E_ARG, "null argument");
    HS_CUDA_TRY(cudaSetDevice(kv->device));
    HS_CUDA_TRY(cudaMemsetAsync(kv->dirty, 0, kv->n_words * 8, kv->st));
    HS_CUDA_TRY(cudaMemsetAsync(kv->tracking, 0, 4, kv->st));
    HS_CUDA_TRY(cudaMemsetAsync(kv->tracking, 1, 1, kv->st));  // tracking = 1 (little-endian u32)
    HS_CUDA_TRY(cudaStreamSynchronize(kv->st));
    return HS_OK;
}

int hs_kv_disarm(hs_kv* kv) {
    if (!kv) return fail(HS_E_ARG, "null argument");
    HS_CUDA_TRY(cudaSetDevice(kv->device));
    HS_CUDA_TRY(cudaMemsetAsync(kv->tracking, 0, 4, kv->st));
    HS_CUDA_TRY(cudaMemsetAsync(kv->dirty, 0, kv->n_words * 8, kv->st));
    HS_CUDA_TRY(cudaStreamSynchronize(kv->st));
    return HS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- batched decode

struct hs_batch {
    const hs_model* m = nullptr;
    uint32_t cap_slots = 0;       // slot capacity, a multiple of 64
    cudaStream_t st = nullptr;
    float *x = nullptr, *part = nullptr, *logits = nullptr;
    uint16_t *xn_hi = nullptr, *xn_lo = nullptr, *att_hi = nullptr, *att_lo = nullptr, *hb_hi = nullptr,
             *hb_lo = nullptr;
    DevCtl* ctl = nullptr;        // device [cap_slots]
    DevCtl* ctl_h = nullptr;      // pinned host mirror
    uint32_t* tokens = nullptr;   // device [cap_slots][tok_cap] histories
    uint64_t tok_cap = 0;
    uint32_t** tok_tab = nullptr;  // device [cap_slots] -> tokens rows
    float** kv_tab = nullptr;      // device per-slot KV regions, dirty bitmaps, tracking flags
    uint64_t** dirty_tab = nullptr;
    uint32_t** track_tab = nullptr;
    void** tab_h = nullptr;        // pinned staging for the three tables
    uint64_t *cand = nullptr, *argbuf = nullptr;
    uint32_t n_cta = 0, kmax_alloc = 0, slice = 0;
    // sampler sort mode (any top_k), allocated at its first use, per slot:
    // every slice's keys in order, the top-k keys in order, their running sums
    uint64_t *sort_cand = nullptr, *wkeys = nullptr;
    float* wps = nullptr;
    double* nll = nullptr;         // perplexity scores of the last forward (hs_batch_nll) [cap_slots]
    uint32_t* nll_next = nullptr;
    uint32_t* err = nullptr;       // GEMM error word (device)
    uint32_t err_h = 0;
    float* sc_global = nullptr;    // attention scores for long contexts [cap_slots][nh][max_ctx]
    float* att_part = nullptr;     // split-KV attention partials [cap_slots][nkv][max_splits][record]
    uint32_t* att_cnt = nullptr;   // [cap_slots][nkv]
    float* pf_part = nullptr;      // prefill segment records [cap_slots][nkv][pf_nseg][record], at first prefill
    uint64_t* trace = nullptr;     // launch timeline (HS_TRACE=1 at creation): 8 u64 per launch
    uint64_t* trace_init = nullptr;
    uint32_t trace_slots = 0;
    uint32_t layout = 0, page_shift = 0;
    // Graphs by (slots, sampler width, KV layout, page shift); forward-only
    // graphs use sampler width 0. Value: the graph and its kernel count.
    std::map<uint64_t, std::pair<cudaGraphExec_t, uint32_t>> graphs;
    cudaGraphExec_t g_step = nullptr;
    uint32_t step_n = 0, launches = 0;
    ~hs_batch() {
        cudaSetDevice(m->device);
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second.first);
        if (st) cudaStreamDestroy(st);
        cudaFreeHost(ctl_h);
        cudaFreeHost(tab_h);
        cudaFreeHost(trace_init);
        cudaFree(trace);
        for (void* p : {(void*)x, (void*)part, (void*)logits, (void*)xn_hi, (void*)xn_lo, (void*)att_hi, (void*)att_lo,
                        (void*)hb_hi, (void*)hb_lo, (void*)ctl, (void*)tokens, (void*)tok_tab, (void*)kv_tab,
                        (void*)dirty_tab, (void*)track_tab, (void*)cand, (void*)argbuf, (void*)err,
                        (void*)sc_global, (void*)att_part, (void*)att_cnt, (void*)sort_cand, (void*)wkeys,
                        (void*)wps, (void*)nll, (void*)nll_next, (void*)pf_part})
            cudaFree(p);
    }
};

namespace hs {
namespace {

// Activation operand map: rows = the live slots (rows past them read as
// zeros), box 64 columns x 64 slots.
int act_map(CUtensorMap* mp, const uint16_t* base, uint32_t cols, uint32_t slots) {
    return make_weight_map(mp, base, cols, slots, 64);
}

int batch_gemm(hs_batch* b, const TcGemmPlan& p, const uint16_t* a_hi, const uint16_t* a_lo, uint32_t n, float* out,
               uint16_t* out_hi, uint16_t* out_lo, uint32_t ld, uint32_t* launches) {
    CUtensorMap mh, ml;
    int rc = act_map(&mh, a_hi, p.K, n);
    if (rc == HS_OK) rc = act_map(&ml, a_lo, p.K, n);
    if (rc) return rc;
    TcGemmPlan q = p;
    q.m_tiles = (n + 63) / 64;
    if (p.m_loop) {  // one grid row of at most one CTA per SM walking all (unit, group) items
        q.grid = std::min<uint32_t>(p.n_tiles * p.splits * q.m_tiles, (uint32_t)b->m->n_sm);
        q.m_tiles = 1;
    }
    TcGemmArgs a{};
    a.K = p.K;
    a.rows = p.rows;
    a.n_tile = p.n_tile;
    a.n_tiles = p.n_tiles;
    a.splits = p.splits;
    a.slots = n;
    a.nst = p.nst;
    a.wres = p.wres ? 1u : 0u;
    a.m_loop = p.m_loop ? 1u : 0u;
    a.ld = ld;
    a.part_stride = (uint64_t)b->cap_slots * p.rows;
    a.out = out;
    a.out_hi = out_hi;
    a.out_lo = out_lo;
    a.err = b->err;
    a.trace = b->trace;
    a.trace_slot = *launches;
    cudaError_t e = launch_tc_gemm(q, mh, ml, a, b->st);
    if (e != cudaSuccess) return fail(HS_E_CUDA, std::string("tensor-core GEMM launch: ") + cudaGetErrorString(e));
    (*launches)++;
    return HS_OK;
}

// One batched forward for slots [0, n): 7 launches per layer + final norm + LM head.
int batch_enqueue_forward(hs_batch* b, uint32_t n, uint32_t* launches, bool prefill) {
    const hs_model* m = b->m;
    const hs_config& c = m->cfg;
    const uint32_t d = c.d_model, hd = c.head_dim, qrows = (c.n_heads + 2 * c.n_kv_heads) * hd;
    int rc;
    const TcGemmPlan* prev_down = nullptr;
    auto norm = [&](const float* g, const TcGemmPlan* part_of, bool embed) -> int {
        TcNormArgs a{};
        a.x = b->x;
        a.part = part_of ? b->part : nullptr;
        a.n_part = part_of ? part_of->splits : 0;
        a.part_stride = part_of ? (uint64_t)b->cap_slots * part_of->rows : 0;
        a.embd = embed ? m->embd : nullptr;
        a.g = g;
        a.out_hi = b->xn_hi;
        a.out_lo = b->xn_lo;
        a.ctl = b->ctl;
        a.d = d;
        a.vocab = c.vocab;
        a.eps = c.eps;
        a.trace = b->trace;
        a.trace_slot = *launches;
        cudaError_t e = launch_tc_norm(a, n, b->st);
        if (e != cudaSuccess) return fail(HS_E_CUDA, std::string("norm launch: ") + cudaGetErrorString(e));
        (*launches)++;
        return HS_OK;
    };
    for (uint32_t l = 0; l < c.n_layers; l++) {
        const LayerDev& L = m->layers[l];
        const TcGemmPlan& Pq = prefill ? L.pq : L.tq;
        const TcGemmPlan& Po = prefill ? L.po : L.to;
        const TcGemmPlan& Pgu = prefill ? L.pgu : L.tgu;
        const TcGemmPlan& Pdown = prefill ? L.pdown : L.tdown;
        if ((rc = norm(L.attn_norm, prev_down, l == 0))) return rc;
        if ((rc = batch_gemm(b, Pq, b->xn_hi, b->xn_lo, n, b->part, nullptr, nullptr, qrows, launches))) return rc;
        cudaError_t e;
        if (m->attn_split) {
            SplitAttnArgs sa{};
            sa.qkv = b->part;
            sa.n_part = Pq.splits;
            sa.part_stride = (uint64_t)b->cap_slots * Pq.rows;
            sa.bias = L.bqkv;
            sa.qkv_rows = qrows;
            sa.kv = b->kv_tab;
            sa.dirty = b->dirty_tab;
            sa.tracking = b->track_tab;
            sa.rope_cos = m->rope_cos;
            sa.rope_sin = m->rope_sin;
            sa.out_hi = b->att_hi;
            sa.out_lo = b->att_lo;
            sa.out_stride = c.n_heads * hd;
            sa.partials = b->att_part;
            sa.counters = b->att_cnt;
            sa.ctl = b->ctl;
            sa.layer = l;
            sa.nh = c.n_heads;
            sa.nkv = c.n_kv_heads;
            sa.max_ctx = c.max_ctx;
            sa.layout = b->layout;
            sa.page_shift = b->page_shift;
            sa.max_splits = m->max_splits;
            sa.head_split = m->attn_head_split;
            sa.nbuf = m->attn_tcw ? (hd == 64 ? 4u : 3u) : m->attn_nbuf;
            sa.unstaged_combine = m->attn_unstaged;
            sa.ws_from = m->attn_ws_from;
            sa.tcw = m->attn_tcw;
            sa.min_split = m->attn_min_split;
            sa.tensor_cores = m->numeric == HS_NUMERIC_TC ? 1u : 0u;
            sa.trace = b->trace;
            sa.trace_slot = *launches;
            if (prefill) {
                // tokens of one sequence: every k, v appended before any attends
                sa.mode = ATTN_APPEND_ONLY;
                e = m->pf_qblock ? launch_prefill_append(hd, sa, n, b->st) : launch_attn_split(hd, sa, n, b->st);
                if (e != cudaSuccess) return fail(HS_E_CUDA, std::string("attention launch: ") + cudaGetErrorString(e));
                (*launches)++;
                sa.mode = ATTN_ATTEND_ONLY;
                sa.trace_slot = *launches;
            }
            if (prefill && m->pf_qblock) {
                // query blocks over fixed segments, then the segments' merge
                sa.partials = b->pf_part;
                sa.max_splits = m->pf_nseg;
                e = launch_attn_prefill(hd, sa, n, m->pf_seg, b->st, *launches, m->pf_tc);
                if (e == cudaSuccess) (*launches)++;
            } else {
                e = launch_attn_split(hd, sa, n, b->st);
            }
        } else {
            return fail(HS_E_STATE, "internal: tensor-core model without split attention");
        }
        if (e != cudaSuccess) return fail(HS_E_CUDA, std::string("attention launch: ") + cudaGetErrorString(e));
        (*launches)++;
        if ((rc = batch_gemm(b, Po, b->att_hi, b->att_lo, n, b->part, nullptr, nullptr, d, launches))) return rc;
        if ((rc = norm(L.ffn_norm, &Po, false))) return rc;
        if ((rc = batch_gemm(b, Pgu, b->xn_hi, b->xn_lo, n, nullptr, b->hb_hi, b->hb_lo, c.d_ff, launches))) return rc;
        if ((rc = batch_gemm(b, Pdown, b->hb_hi, b->hb_lo, n, b->part, nullptr, nullptr, d, launches))) return rc;
        prev_down = &Pdown;
    }
    if (prefill) return HS_OK;  // prompt positions: no logits (x past the last layer is not read)
    if ((rc = norm(m->out_norm, prev_down, false))) return rc;
    return batch_gemm(b, m->thead, b->xn_hi, b->xn_lo, n, b->logits, nullptr, nullptr, c.vocab, launches);
}

SampleArgs batch_sample_args(hs_batch* b, uint32_t n, uint32_t kmax) {
    SampleArgs a{};
    a.logits = b->logits;
    a.tokens = b->tokens;
    a.tokens_w = b->tokens;
    a.cand = b->cand;
    a.argbuf = b->argbuf;
    a.ctl = b->ctl;
    a.vocab = b->m->cfg.vocab;
    a.n_cta = b->n_cta;
    a.kmax = kmax;
    a.slots = n;
    a.logits_stride = b->m->cfg.vocab;
    a.cand_stride = (uint64_t)b->n_cta * kmax;
    a.tok_tab = b->tok_tab;
    a.slice = b->slice;
    if (sample_sort_mode(b->n_cta, kmax)) {
        a.cand = b->sort_cand;
        a.wkeys = b->wkeys;
        a.wps = b->wps;
        a.wide_stride = b->m->cfg.vocab;
    }
    return a;
}

int batch_graph(hs_batch* b, uint32_t n, uint32_t kmax, cudaGraphExec_t* out, uint32_t* launches,
                bool prefill = false) {
    const uint64_t key = (uint64_t)n | (uint64_t)kmax << 16 | (uint64_t)b->layout << 32 | (uint64_t)b->page_shift << 40 |
                         (uint64_t)prefill << 48;
    auto it = b->graphs.find(key);
    if (it != b->graphs.end()) {
        *out = it->second.first;
        *launches = it->second.second;
        return HS_OK;
    }
    *launches = 0;
    cudaGraph_t g = nullptr;
    HS_CUDA_TRY(cudaStreamBeginCapture(b->st, cudaStreamCaptureModeThreadLocal));
    int rc = batch_enqueue_forward(b, n, launches, prefill);
    if (rc == HS_OK && kmax) {
        SampleArgs sa = batch_sample_args(b, n, kmax);
        sa.trace = b->trace;
        sa.trace_slot = *launches;  // and the next slot for the second kernel
        cudaError_t e = launch_sample(sa, b->st);
        if (e != cudaSuccess) rc = fail(HS_E_CUDA, std::string("sampler launch: ") + cudaGetErrorString(e));
        *launches += sample_sort_mode(b->n_cta, kmax) ? 3 : 2;
    }
    cudaError_t e = cudaStreamEndCapture(b->st, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return fail(HS_E_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
    cudaGraphExec_t ex = nullptr;
    e = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail(HS_E_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
    b->graphs[key] = std::make_pair(ex, *launches);
    *out = ex;
    return HS_OK;
}

// Per-slot KV tables (all regions must share layout and page size).
int batch_kv_tables(hs_batch* b, hs_kv* const* kvs, uint32_t n, bool same_sequence = false) {
    const hs_model* m = b->m;
    for (uint32_t i = 0; i < n; i++) {
        if (!kvs[i]) return fail(HS_E_ARG, "null KV region");
        int rc = check_kv(m, kvs[i]);
        if (rc) return rc;
        if (kvs[i]->spec.layout != kvs[0]->spec.layout || kvs[i]->page_shift != kvs[0]->page_shift)
            return fail(HS_E_ARG, "KV regions of one batch must share layout and page size");
        for (uint32_t j = 0; j < i && !same_sequence; j++)
            if (kvs[j] == kvs[i]) return fail(HS_E_ARG, "a KV region appears twice in one batch");
    }
    b->layout = kvs[0]->spec.layout;
    b->page_shift = kvs[0]->page_shift;
    void** h = b->tab_h;
    const uint32_t C = b->cap_slots;
    for (uint32_t i = 0; i < n; i++) {
        h[i] = kvs[i]->base;
        h[C + i] = kvs[i]->dirty;
        h[2 * C + i] = kvs[i]->tracking;
    }
    HS_CUDA_TRY(cudaMemcpyAsync(b->kv_tab, h, n * sizeof(void*), cudaMemcpyHostToDevice, b->st));
    HS_CUDA_TRY(cudaMemcpyAsync(b->dirty_tab, h + C, n * sizeof(void*), cudaMemcpyHostToDevice, b->st));
    HS_CUDA_TRY(cudaMemcpyAsync(b->track_tab, h + 2 * C, n * sizeof(void*), cudaMemcpyHostToDevice, b->st));
    return HS_OK;
}

int batch_sync(hs_batch* b, uint32_t n) {
    HS_CUDA_TRY(cudaMemcpyAsync(b->ctl_h, b->ctl, (size_t)n * sizeof(DevCtl), cudaMemcpyDeviceToHost, b->st));
    HS_CUDA_TRY(cudaMemcpyAsync(&b->err_h, b->err, 4, cudaMemcpyDeviceToHost, b->st));
    HS_CUDA_TRY(cudaStreamSynchronize(b->st));
    if (b->err_h) return fail(HS_E_CUDA, "tensor-core GEMM reported a bounded-wait timeout");
    for (uint32_t i = 0; i < n; i++) {
        int rc = ctl_err(b->ctl_h[i].err);
        if (rc) return fail(rc, "sequence " + std::to_string(i) + ": " + hs_last_error());
    }
    return HS_OK;
}

}  // namespace
}  // namespace hs

extern "C" {

int hs_batch_new(const hs_model* m, uint32_t max_seqs, hs_batch** out) {
    if (!m || !out) return fail(HS_E_ARG, "null argument");
    if (m->numeric != HS_NUMERIC_TC) return fail(HS_E_UNSUPPORTED, "hs_batch needs a model loaded with HS_NUMERIC_TC");
    if (max_seqs == 0 || max_seqs > 4096) return fail(HS_E_ARG, "max_seqs must be 1..4096");
    HS_CUDA_TRY(cudaSetDevice(m->device));
    auto b = std::make_unique<hs_batch>();
    b->m = m;
    const hs_config& c = m->cfg;
    const uint32_t C = (max_seqs + 63) / 64 * 64;
    b->cap_slots = C;
    const uint32_t qrows = (c.n_heads + 2 * c.n_kv_heads) * c.head_dim;
    HS_CUDA_TRY(cudaStreamCreateWithFlags(&b->st, cudaStreamNonBlocking));
    auto alloc = [&](auto** p, uint64_t count) -> int {
        using T = std::remove_reference_t<decltype(**p)>;
        cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), std::max<uint64_t>(count, 1) * sizeof(T));
        if (e != cudaSuccess) return fail(HS_E_NOMEM, std::string("cudaMalloc: ") + cudaGetErrorString(e));
        e = cudaMemset(*p, 0, std::max<uint64_t>(count, 1) * sizeof(T));
        return e == cudaSuccess ? (int)HS_OK : fail(HS_E_CUDA, cudaGetErrorString(e));
    };
    b->tok_cap = (uint64_t)c.max_ctx + 1;
    // Large vocabularies take 4096 logits per candidate CTA (fewer, longer
    // CTAs for many sequences at once); the selection is exact either way.
    b->slice = c.vocab > kMaxSlice ? kMaxSlice : kSampleSlice;
    b->n_cta = (c.vocab + b->slice - 1) / b->slice;
    if (b->n_cta > 256) return fail(HS_E_UNSUPPORTED, "vocab too large for the device sampler");
    b->kmax_alloc = b->n_cta > 1 ? kMaxTopK : kSampleSlice;
    int rc;
    if ((rc = alloc(&b->x, (uint64_t)C * c.d_model)) ||
        (rc = alloc(&b->part, (uint64_t)C * std::max<uint64_t>(m->tc_part_per_slot, qrows))) ||
        (rc = alloc(&b->logits, (uint64_t)C * c.vocab)) || (rc = alloc(&b->xn_hi, (uint64_t)C * c.d_model)) ||
        (rc = alloc(&b->xn_lo, (uint64_t)C * c.d_model)) ||
        (rc = alloc(&b->att_hi, (uint64_t)C * c.n_heads * c.head_dim)) ||
        (rc = alloc(&b->att_lo, (uint64_t)C * c.n_heads * c.head_dim)) ||
        (rc = alloc(&b->hb_hi, (uint64_t)C * c.d_ff)) || (rc = alloc(&b->hb_lo, (uint64_t)C * c.d_ff)) ||
        (rc = alloc(&b->ctl, C)) || (rc = alloc(&b->tokens, (uint64_t)C * b->tok_cap)) ||
        (rc = alloc(&b->tok_tab, C)) || (rc = alloc(&b->kv_tab, C)) || (rc = alloc(&b->dirty_tab, C)) ||
        (rc = alloc(&b->track_tab, C)) || (rc = alloc(&b->cand, (uint64_t)C * b->n_cta * b->kmax_alloc)) ||
        (rc = alloc(&b->argbuf, (uint64_t)C * b->n_cta)) || (rc = alloc(&b->err, 1)) ||
        (m->attn_global && (rc = alloc(&b->sc_global, (uint64_t)C * c.n_heads * c.max_ctx))) ||
        (m->attn_split &&
         ((rc = alloc(&b->att_part, (uint64_t)C * c.n_kv_heads * m->max_splits *
                                        attn_record(c.n_heads / c.n_kv_heads, c.head_dim))) ||
          (rc = alloc(&b->att_cnt, (uint64_t)C * c.n_kv_heads)))))
        return rc;
    HS_CUDA_TRY(cudaMallocHost(&b->ctl_h, (size_t)C * sizeof(DevCtl)));
    std::memset(b->ctl_h, 0, (size_t)C * sizeof(DevCtl));
    HS_CUDA_TRY(cudaMallocHost(&b->tab_h, (size_t)3 * C * sizeof(void*)));
    const char* tenv = getenv("HS_TRACE");
    if (tenv && tenv[0] == '1') {
        b->trace_slots = c.n_layers * 9 + 5;  // prefill: 9 launches a layer; decode: 7 + norm, head, sampler
        HS_CUDA_TRY(cudaMalloc(&b->trace, (size_t)b->trace_slots * 64));
        HS_CUDA_TRY(cudaMallocHost(&b->trace_init, (size_t)b->trace_slots * 64));
        for (uint32_t i = 0; i < b->trace_slots; i++) {
            b->trace_init[8 * i] = ~0ull;
            for (int j = 1; j < 8; j++) b->trace_init[8 * i + j] = 0;
        }
    }
    std::vector<uint32_t*> rows(C);
    for (uint32_t i = 0; i < C; i++) rows[i] = b->tokens + (uint64_t)i * b->tok_cap;
    HS_CUDA_TRY(cudaMemcpy(b->tok_tab, rows.data(), C * sizeof(uint32_t*), cudaMemcpyHostToDevice));
    *out = b.release();
    return HS_OK;
}

void hs_batch_free(hs_batch* b) { delete b; }

void* hs_batch_stream(hs_batch* b) { return b ? (void*)b->st : nullptr; }

int hs_batch_launches_per_step(hs_batch* b, uint32_t* out) {
    if (!b || !out) return fail(HS_E_ARG, "null argument");
    if (!b->g_step) return fail(HS_E_ARG, "hs_batch_seq_begin has not been called");
    *out = b->launches;
    return HS_OK;
}

int hs_forward_batch(const hs_model* m, hs_kv* const* kvs, const uint32_t* tokens, const uint32_t* pos, uint32_t n,
                     hs_batch* b) {
    if (!m || !b || b->m != m || !kvs || !tokens || !pos) return fail(HS_E_ARG, "null or mismatched argument");
    if (n == 0 || n > b->cap_slots) return fail(HS_E_ARG, "sequence count outside the batch capacity");
    for (uint32_t i = 0; i < n; i++) {
        if (pos[i] >= m->cfg.max_ctx) return fail(HS_E_ARG, "position past max_ctx");
        if (tokens[i] >= m->cfg.vocab) return fail(HS_E_ARG, "token " + std::to_string(tokens[i]) + " out of range");
    }
    HS_CUDA_TRY(cudaSetDevice(m->device));
    int rc = batch_kv_tables(b, kvs, n);
    if (rc) return rc;
    for (uint32_t i = 0; i < n; i++) {
        DevCtl& h = b->ctl_h[i];
        std::memset(&h, 0, sizeof(DevCtl));
        h.token = tokens[i];
        h.pos = pos[i];
        h.active = 1;
        h.mode = 1;
        h.vocab = m->cfg.vocab;
        h.max_ctx = m->cfg.max_ctx;
    }
    HS_CUDA_TRY(cudaMemcpyAsync(b->ctl, b->ctl_h, (size_t)n * sizeof(DevCtl), cudaMemcpyHostToDevice, b->st));
    cudaGraphExec_t g = nullptr;
    uint32_t launches = 0;
    if ((rc = batch_graph(b, n, 0, &g, &launches))) return rc;
    if (b->trace)
        HS_CUDA_TRY(cudaMemcpyAsync(b->trace, b->trace_init, (size_t)b->trace_slots * 64, cudaMemcpyHostToDevice, b->st));
    HS_CUDA_TRY(cudaGraphLaunch(g, b->st));
    return batch_sync(b, n);
}

int hs_prefill(const hs_model* m, hs_kv* kv, const uint32_t* tokens, uint32_t n, uint32_t pos0, hs_batch* b) {
    if (!m || !b || b->m != m || !kv || (!tokens && n)) return fail(HS_E_ARG, "null or mismatched argument");
    int rc = check_kv(m, kv);
    if (rc) return rc;
    if ((uint64_t)pos0 + n > m->cfg.max_ctx) return fail(HS_E_ARG, "prompt runs past max_ctx");
    for (uint32_t i = 0; i < n; i++)
        if (tokens[i] >= m->cfg.vocab) return fail(HS_E_ARG, "token " + std::to_string(tokens[i]) + " out of range");
    HS_CUDA_TRY(cudaSetDevice(m->device));
    const uint32_t C = b->cap_slots;
    if (m->pf_qblock && !b->pf_part)
        HS_CUDA_TRY(cudaMalloc(&b->pf_part, (size_t)C * m->cfg.n_kv_heads * m->pf_nseg *
                                                attn_record(m->cfg.n_heads / m->cfg.n_kv_heads, m->cfg.head_dim) * 4));
    std::vector<hs_kv*> same(std::min(C, std::max(n, 1u)), kv);
    for (uint32_t off = 0; off < n; off += C) {
        const uint32_t cnt = std::min(C, n - off);
        if ((rc = batch_kv_tables(b, same.data(), cnt, true))) return rc;
        for (uint32_t i = 0; i < cnt; i++) {
            DevCtl& h = b->ctl_h[i];
            std::memset(&h, 0, sizeof(DevCtl));
            h.token = tokens[off + i];
            h.pos = pos0 + off + i;
            h.active = 1;
            h.mode = 1;
            h.vocab = m->cfg.vocab;
            h.max_ctx = m->cfg.max_ctx;
        }
        HS_CUDA_TRY(cudaMemcpyAsync(b->ctl, b->ctl_h, (size_t)cnt * sizeof(DevCtl), cudaMemcpyHostToDevice, b->st));
        cudaGraphExec_t g = nullptr;
        uint32_t launches = 0;
        if ((rc = batch_graph(b, cnt, 0, &g, &launches, true))) return rc;
        if (b->trace)
            HS_CUDA_TRY(cudaMemcpyAsync(b->trace, b->trace_init, (size_t)b->trace_slots * 64, cudaMemcpyHostToDevice,
                                        b->st));
        HS_CUDA_TRY(cudaGraphLaunch(g, b->st));
        if ((rc = batch_sync(b, cnt))) return rc;
    }
    return HS_OK;
}

int hs_batch_nll(hs_batch* b, const uint32_t* next, uint32_t n, double* out) {
    if (!b || (!next && n) || (!out && n)) return fail(HS_E_ARG, "null argument");
    if (n > b->cap_slots) return fail(HS_E_ARG, "more rows than the batch holds");
    const uint32_t vocab = b->m->cfg.vocab;
    for (uint32_t i = 0; i < n; i++)
        if (next[i] >= vocab) return fail(HS_E_ARG, "token out of range");
    if (!n) return HS_OK;
    HS_CUDA_TRY(cudaSetDevice(b->m->device));
    if (!b->nll) {
        HS_CUDA_TRY(cudaMalloc(&b->nll, (size_t)b->cap_slots * 8));
        HS_CUDA_TRY(cudaMalloc(&b->nll_next, (size_t)b->cap_slots * 4));
    }
    HS_CUDA_TRY(cudaMemcpyAsync(b->nll_next, next, (size_t)n * 4, cudaMemcpyHostToDevice, b->st));
    HS_CUDA_TRY(launch_logits_nll(b->logits, vocab, b->nll_next, n, vocab, b->nll, b->st));
    HS_CUDA_TRY(cudaMemcpyAsync(out, b->nll, (size_t)n * 8, cudaMemcpyDeviceToHost, b->st));
    HS_CUDA_TRY(cudaStreamSynchronize(b->st));
    return HS_OK;
}

int hs_batch_logits(hs_batch* b, uint32_t slot, float* host, uint64_t n) {
    if (!b || !host) return fail(HS_E_ARG, "null argument");
    if (slot >= b->cap_slots) return fail(HS_E_ARG, "slot outside the batch capacity");
    if (n > b->m->cfg.vocab) return fail(HS_E_ARG, "more logits than the vocabulary");
    HS_CUDA_TRY(cudaSetDevice(b->m->device));
    HS_CUDA_TRY(cudaMemcpy(host, b->logits + (uint64_t)slot * b->m->cfg.vocab, n * 4, cudaMemcpyDeviceToHost));
    return HS_OK;
}

int hs_batch_seq_begin(hs_batch* b, hs_kv* const* kvs, uint32_t n, uint32_t* const* tokens, const uint64_t* n_tokens,
                       uint64_t cap, const hs_seq_state* st, const hs_sampler_cfg* cfg, const hs_rng* rng,
                       uint64_t stop_at_filled) {
    if (!b || !kvs || !tokens || !n_tokens || !st || !cfg || !rng) return fail(HS_E_ARG, "null argument");
    if (n == 0 || n > b->cap_slots) return fail(HS_E_ARG, "sequence count outside the batch capacity");
    const hs_model* m = b->m;
    const uint32_t vocab = m->cfg.vocab;
    uint32_t kmax = b->n_cta > 1 ? kMaxTopK : std::min<uint32_t>(kSampleSlice, vocab);
    for (uint32_t i = 0; i < n; i++) {
        const std::string who = "sequence " + std::to_string(i) + ": ";
        if (!tokens[i]) return fail(HS_E_ARG, who + "null token buffer");
        if (n_tokens[i] == 0 || st[i].filled > n_tokens[i] || st[i].prompt_len > n_tokens[i])
            return fail(HS_E_ARG, who + "inconsistent sequence state");
        if (n_tokens[i] > b->tok_cap) return fail(HS_E_ARG, who + "history longer than max_ctx");
        for (uint64_t j = 0; j < n_tokens[i]; j++)
            if (tokens[i][j] >= vocab) return fail(HS_E_ARG, who + "token out of range");
        const uint32_t k = cfg[i].top_k == 0 ? vocab : std::min(cfg[i].top_k, vocab);
        if (cfg[i].temperature > 0.0f && b->n_cta > 1 && k > kMaxTopK) kmax = b->slice;  // sort mode
        if (!st[i].done && st[i].filled >= n_tokens[i])
            return fail(HS_E_STATE, who + "nothing to feed at the token boundary");
    }
    HS_CUDA_TRY(cudaSetDevice(m->device));
    if (sample_sort_mode(b->n_cta, kmax) && !b->sort_cand) {
        const uint64_t C = b->cap_slots;
        HS_CUDA_TRY(cudaMalloc(&b->sort_cand, C * b->n_cta * b->slice * 8));
        HS_CUDA_TRY(cudaMalloc(&b->wkeys, C * vocab * 8));
        HS_CUDA_TRY(cudaMalloc(&b->wps, C * vocab * 4));
    }
    int rc = batch_kv_tables(b, kvs, n);
    if (rc) return rc;
    for (uint32_t i = 0; i < n; i++) {
        DevCtl& h = b->ctl_h[i];
        std::memset(&h, 0, sizeof(DevCtl));
        h.mode = 0;
        h.n_tokens = n_tokens[i];
        h.filled = st[i].filled;
        h.prompt_len = st[i].prompt_len;
        h.max_tokens = st[i].max_tokens;
        h.cap = std::min<uint64_t>(cap, b->tok_cap);
        h.stop_at = stop_at_filled;
        h.done = st[i].done;
        h.done_reason = st[i].done_reason;
        h.eos = m->cfg.eos;
        h.max_ctx = m->cfg.max_ctx;
        h.vocab = vocab;
        fill_cfg(h, &cfg[i], &rng[i]);
        const bool runnable =
            !st[i].done && st[i].filled < n_tokens[i] && !(stop_at_filled && st[i].filled >= stop_at_filled);
        if (runnable && st[i].filled >= m->cfg.max_ctx) return fail(HS_E_ARG, "position past max_ctx");
        h.active = runnable ? 1 : 0;
        h.token = runnable ? tokens[i][st[i].filled] : 0;
        h.pos = (uint32_t)st[i].filled;
        HS_CUDA_TRY(cudaMemcpyAsync(b->tokens + (uint64_t)i * b->tok_cap, tokens[i], n_tokens[i] * 4,
                                    cudaMemcpyHostToDevice, b->st));
    }
    HS_CUDA_TRY(cudaMemcpyAsync(b->ctl, b->ctl_h, (size_t)n * sizeof(DevCtl), cudaMemcpyHostToDevice, b->st));
    if ((rc = batch_graph(b, n, kmax, &b->g_step, &b->launches))) return rc;
    b->step_n = n;
    return HS_OK;
}

int hs_batch_seq_step(hs_batch* b, uint32_t n_steps) {
    if (!b || !b->g_step) return fail(HS_E_ARG, "hs_batch_seq_begin has not been called");
    HS_CUDA_TRY(cudaSetDevice(b->m->device));
    for (uint32_t i = 0; i < n_steps; i++) {
        if (b->trace)
            HS_CUDA_TRY(cudaMemcpyAsync(b->trace, b->trace_init, (size_t)b->trace_slots * 64, cudaMemcpyHostToDevice,
                                        b->st));
        HS_CUDA_TRY(cudaGraphLaunch(b->g_step, b->st));
    }
    return HS_OK;
}

int hs_batch_trace(hs_batch* b, uint64_t* out, uint64_t n_slots, uint64_t* used) {
    if (!b || !used) return fail(HS_E_ARG, "null argument");
    *used = b->trace_slots;
    if (!b->trace) return fail(HS_E_STATE, "tracing is off (set HS_TRACE=1 before creating the batch)");
    if (!out) return HS_OK;
    HS_CUDA_TRY(cudaSetDevice(b->m->device));
    HS_CUDA_TRY(cudaStreamSynchronize(b->st));
    HS_CUDA_TRY(cudaMemcpy(out, b->trace, std::min<uint64_t>(n_slots, b->trace_slots) * 64, cudaMemcpyDeviceToHost));
    return HS_OK;
}

int hs_batch_seq_end(hs_batch* b, uint32_t* const* tokens, uint64_t* n_tokens, uint64_t cap, hs_seq_state* st,
                     hs_rng* rng) {
    if (!b || !b->g_step) return fail(HS_E_ARG, "hs_batch_seq_begin has not been called");
    HS_CUDA_TRY(cudaSetDevice(b->m->device));
    const uint32_t n = b->step_n;
    int rc = batch_sync(b, n);
    if (rc) return rc;
    for (uint32_t i = 0; i < n; i++) {
        const DevCtl& h = b->ctl_h[i];
        if (tokens && n_tokens && tokens[i]) {
            if (h.n_tokens > cap) return fail(HS_E_ARG, "token buffer too small");
            HS_CUDA_TRY(cudaMemcpy(tokens[i], b->tokens + (uint64_t)i * b->tok_cap, h.n_tokens * 4,
                                   cudaMemcpyDeviceToHost));
            n_tokens[i] = h.n_tokens;
        }
        if (st) {
            st[i].filled = h.filled;
            st[i].done = h.done;
            st[i].done_reason = h.done_reason;
        }
        if (rng) {
            for (int k = 0; k < 4; k++) rng[i].s[k] = h.rng[k];
            rng[i].draws = h.draws;
        }
    }
    return HS_OK;
}

int hs_batch_seq_run(const hs_model* m, hs_kv* const* kvs, hs_batch* b, uint32_t n, uint32_t* const* tokens,
                     uint64_t* n_tokens, uint64_t cap, hs_seq_state* st, const hs_sampler_cfg* cfg, hs_rng* rng,
                     uint64_t stop_at_filled) {
    if (!m || !b || b->m != m || !n_tokens) return fail(HS_E_ARG, "null or mismatched argument");
    int rc = hs_batch_seq_begin(b, kvs, n, tokens, n_tokens, cap, st, cfg, rng, stop_at_filled);
    if (rc) return rc;
    // Each chunk advances every running sequence; max_ctx chunks bound the loop.
    for (uint32_t guard = 0;; guard++) {
        uint64_t bound = 0;
        for (uint32_t i = 0; i < n; i++) {
            const DevCtl& h = b->ctl_h[i];
            if (h.done || !h.active) continue;
            const uint64_t pre = h.n_tokens - h.filled, gen = h.n_tokens - h.prompt_len;
            uint64_t bi = pre + (h.max_tokens > gen ? h.max_tokens - gen : 0);
            if (h.stop_at && h.stop_at > h.filled) bi = std::min<uint64_t>(bi, h.stop_at - h.filled);
            bound = std::max<uint64_t>(bound, std::max<uint64_t>(1, bi));
        }
        if (bound == 0) break;
        if (guard > m->cfg.max_ctx) return fail(HS_E_STATE, "decode loop made no progress");
        if ((rc = hs_batch_seq_step(b, (uint32_t)std::min<uint64_t>(bound, 256)))) return rc;
        if ((rc = batch_sync(b, n))) return rc;
    }
    return hs_batch_seq_end(b, tokens, n_tokens, cap, st, rng);
}

}  // extern "C"
