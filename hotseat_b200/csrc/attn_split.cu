// Split-KV GQA decode attention for the GPU-native paths (HS_NUMERIC_FAST
// batch-1 and HS_NUMERIC_TC batched): model.rs:259-305 computed with an
// online softmax over chunks of 64 cached positions, the positions of one
// (sequence, KV head) spread over several CTAs.
//
// Grid (max_splits * head parts, n_kv_heads, sequences). A sequence at `pos`
// has n = pos+1 positions; split_len(n) positions per split (a multiple of
// 64, so that at most max_splits splits are needed) and S = ceil(n /
// split_len) splits; CTA s >= S exits at once. Every CTA rebuilds q (its
// part of the group's query heads: one part unless head_split asks for more)
// and the new k, v from the QKV product (split-K partials added in split
// order, then the bias), applies RoPE (model.rs:365-373); split 0 appends k,
// v at `pos` to the sequence's KV region and marks the dirty pages
// (model.rs:268-275); the split holding `pos` uses its own copy of that row.
// The first chunks' cached rows are loaded before the wait for the QKV
// product.
//
// Per chunk: scores for the group's heads, chunk maximum, rescale of the
// running sum and output, P.V: on mma.sync tiles with split tf32 operands
// (tensor-core path) or in fp32 FMA chains (fast path, the same item the
// persistent token kernel runs). A single split writes the normalised
// output; otherwise each split writes (max, sum, unnormalised output) and
// the CTA that arrives last at the (sequence, KV head) counter combines the
// splits in split order and resets the counter. Every choice depends on n
// and max_ctx only, never on the batch, so a sequence's bits are the same in
// any batch.
#include "attn_body.cuh"
#include "common.h"
#include "kernels.h"

namespace hs {
namespace {

// K/V chunk buffers by default: three chunks load while one computes (two at
// head_dim 128, for shared memory). Fewer buffers let more CTAs share an SM.
__host__ __device__ constexpr int nbuf(int hd) { return hd == 64 ? 4 : 3; }
uint32_t buffers(uint32_t hd, uint32_t want) { return want >= 2 && want <= 4 ? want : nbuf((int)hd); }

// Two CTAs per SM where the item's space allows it (head_dim 64); at 128 the
// item takes most of an SM's shared memory, so one CTA may use every register.
template <int HD, int NB, bool TC>
__global__ void __launch_bounds__(attn::kThreads, HD == 64 ? 2 : 1) k_attn_split(const SplitAttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    const uint32_t hsplit = attn_head_split(a);
    const uint32_t s = blockIdx.x / hsplit, hpart = blockIdx.x % hsplit, kvh = blockIdx.y, slot = blockIdx.z;
    const KTrace tr(a.trace, a.trace_slot);
    tr.enter();
    DevCtl* ctl = a.ctl + slot;
    const bool active = attn::ldv(&ctl->active) != 0;
    const uint32_t pos = attn::ldv(&ctl->pos);
    pdl_launch_dependents();
    // The cached rows (all but pos) and the RoPE row do not depend on the
    // kernels this launch overlaps: with a whole item (append and attend),
    // start loading the first chunks before waiting for the QKV product.
    const uint32_t n = pos + 1, L = attn_split_len(n, a.max_splits, a.ws_from, a.min_split), S = (n + L - 1) / L;
    uint32_t npre = 0;
    if (a.mode == ATTN_FULL && active && pos < a.max_ctx && s < S) {
        bool tcw = false;  // the same choice as attn::item's
        if constexpr (TC && attn::TcwGeom<HD, NB>::OK) tcw = a.tcw != 0;
        if (tcw) {
            if constexpr (TC && attn::TcwGeom<HD, NB>::OK)
                npre = attn::tcw_prefetch<HD, NB>(a, a.layer, s, kvh, slot, pos, sm);
        } else {
            npre = attn_use_ws(n, a.ws_from) ? attn::ws_prefetch<HD, NB>(a, a.layer, s, kvh, slot, pos, sm)
                                : attn::prefetch<HD, NB>(a, a.layer, s, kvh, slot, pos, sm, NB - 1 > 0 ? NB - 1 : 1);
        }
    }
    pdl_wait();
    if (!active) return;
    if (pos >= a.max_ctx) {
        if (threadIdx.x == 0 && s == 0 && kvh == 0) atomicOr(&ctl->err, ERR_POS);
        return;
    }
    if (s >= (a.mode != ATTN_APPEND_ONLY ? S : 1u)) return;
    if (a.mode == ATTN_APPEND_ONLY && hpart != 0) return;
    // with a trace: the item's checkpoints (SM clock), reported as the
    // maximum over CTAs of the cycles from the item's start to RoPE done,
    // first chunk ready, last chunk done and the end (trace words 4..7)
    __shared__ uint64_t probe[8];
    attn::item<HD, NB, TC>(a, a.layer, s, kvh, hpart, slot, pos, sm, npre, false, a.trace ? probe : nullptr);
    if (a.trace && threadIdx.x == 0) {
        const uint64_t t = clock64();
        unsigned long long* q = reinterpret_cast<unsigned long long*>(a.trace + 8 * a.trace_slot);
        atomicMax(q + 4, (unsigned long long)(probe[2] - probe[0]));
        atomicMax(q + 5, (unsigned long long)(probe[3] - probe[0]));
        atomicMax(q + 6, (unsigned long long)(probe[6] - probe[0]));
        atomicMax(q + 7, (unsigned long long)(t - probe[0]));
    }
    tr.exit();
}

}  // namespace

size_t attn_split_smem(uint32_t head_dim, uint32_t nbufs) {
    return attn::item_smem(head_dim, buffers(head_dim, nbufs));
}

bool attn_ws_fits(uint32_t hd, uint32_t nbufs) {
    switch (hd * 8 + nbufs) {
        case 64 * 8 + 1: return attn::WsGeom<64, 1>::OK;
        case 64 * 8 + 2: return attn::WsGeom<64, 2>::OK;
        case 64 * 8 + 3: return attn::WsGeom<64, 3>::OK;
        case 64 * 8 + 4: return attn::WsGeom<64, 4>::OK;
        case 128 * 8 + 1: return attn::WsGeom<128, 1>::OK;
        case 128 * 8 + 2: return attn::WsGeom<128, 2>::OK;
        case 128 * 8 + 3: return attn::WsGeom<128, 3>::OK;
        case 128 * 8 + 4: return attn::WsGeom<128, 4>::OK;
        default: return false;
    }
}

uint32_t attn_max_splits(uint32_t max_ctx) {
    const uint32_t chunks = (max_ctx + attn::kCh - 1) / attn::kCh;
    return chunks < 128 ? chunks : 128;
}

cudaError_t attn_split_set_smem_limits(int optin) {
    const void* fns[] = {
        (const void*)k_attn_split<64, 2, false>,  (const void*)k_attn_split<64, 3, false>,
        (const void*)k_attn_split<64, 4, false>,  (const void*)k_attn_split<128, 2, false>,
        (const void*)k_attn_split<128, 3, false>, (const void*)k_attn_split<128, 4, false>,
        (const void*)k_attn_split<64, 2, true>,   (const void*)k_attn_split<64, 3, true>,
        (const void*)k_attn_split<64, 4, true>,   (const void*)k_attn_split<128, 2, true>,
        (const void*)k_attn_split<128, 3, true>,  (const void*)k_attn_split<128, 4, true>};
    for (int i = 0; i < 12; i++) {
        const size_t need = attn::item_smem(i % 6 < 3 ? 64 : 128, 2 + i % 3);
        if (need > (size_t)optin) continue;  // not launchable on this device (the model load refuses it)
        const cudaError_t e = cudaFuncSetAttribute(fns[i], cudaFuncAttributeMaxDynamicSharedMemorySize, (int)need);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

namespace {
template <bool TC>
cudaError_t launch_variant(cudaLaunchConfig_t& cfg, uint32_t head_dim, uint32_t nb, const SplitAttnArgs& a) {
    if (head_dim == 64)
        return nb == 2 ? cudaLaunchKernelEx(&cfg, k_attn_split<64, 2, TC>, a)
                       : nb == 3 ? cudaLaunchKernelEx(&cfg, k_attn_split<64, 3, TC>, a)
                                 : cudaLaunchKernelEx(&cfg, k_attn_split<64, 4, TC>, a);
    if (head_dim == 128)
        return nb == 2 ? cudaLaunchKernelEx(&cfg, k_attn_split<128, 2, TC>, a)
                       : nb == 3 ? cudaLaunchKernelEx(&cfg, k_attn_split<128, 3, TC>, a)
                                 : cudaLaunchKernelEx(&cfg, k_attn_split<128, 4, TC>, a);
    return cudaErrorInvalidValue;
}
}  // namespace

cudaError_t launch_attn_split(uint32_t head_dim, const SplitAttnArgs& a, uint32_t slots, cudaStream_t st) {
    if (a.nkv == 0 || a.nh % a.nkv || a.nh / a.nkv > 8 || a.max_splits == 0 || (!a.out_f32 && !a.out_hi))
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(a.mode == ATTN_APPEND_ONLY ? 1 : a.max_splits * attn_head_split(a), a.nkv, slots);
    cfg.blockDim = dim3(attn::kThreads);
    const uint32_t nb = buffers(head_dim, a.nbuf);
    cfg.dynamicSmemBytes = attn_split_smem(head_dim, nb);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return a.tensor_cores ? launch_variant<true>(cfg, head_dim, nb, a) : launch_variant<false>(cfg, head_dim, nb, a);
}

}  // namespace hs
