// Split-KV GQA decode attention for the GPU-native paths (HS_NUMERIC_FAST
// batch-1 and HS_NUMERIC_TC batched): model.rs:259-305 computed with an
// online softmax over chunks of 64 cached positions, the positions of one
// (sequence, KV head) spread over several CTAs.
//
// Grid (max_splits, n_kv_heads, sequences). A sequence at `pos` has n = pos+1
// positions; split_len(n) positions per split (a multiple of 64, so that at
// most max_splits splits are needed) and S = ceil(n / split_len) splits; CTA
// s >= S exits at once. Every CTA rebuilds q (the group's query heads) and
// the new k, v from the QKV product (split-K partials added in split order,
// then the bias), applies RoPE (model.rs:365-373); split 0 appends k, v at
// `pos` to the sequence's KV region and marks the dirty pages
// (model.rs:268-275); the split holding `pos` uses its own copy of that row.
//
// Per chunk: scores for the group's heads, chunk maximum, rescale of the
// running sum and output, P.V. A single split writes the normalised output;
// otherwise each split writes (max, sum, unnormalised output) and the CTA
// that arrives last at the (sequence, KV head) counter combines the splits in
// split order and resets the counter. Every choice depends on n and max_ctx
// only, never on the batch, so a sequence's bits are the same in any batch.
#include "attn_body.cuh"
#include "common.h"
#include "kernels.h"

namespace hs {
namespace {

// K/V chunk buffers: three chunks load while one computes (two at
// head_dim 128, for shared memory).
__host__ __device__ constexpr int nbuf(int hd) { return hd == 64 ? 4 : 3; }

template <int HD>
__global__ void __launch_bounds__(attn::kThreads) k_attn_split(const SplitAttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    const uint32_t s = blockIdx.x, kvh = blockIdx.y, slot = blockIdx.z;
    const KTrace tr(a.trace, a.trace_slot);
    tr.enter();
    DevCtl* ctl = a.ctl + slot;
    const bool active = attn::ldv(&ctl->active) != 0;
    const uint32_t pos = attn::ldv(&ctl->pos);
    pdl_launch_dependents();
    pdl_wait();
    if (!active) return;
    if (pos >= a.max_ctx) {
        if (threadIdx.x == 0 && s == 0 && kvh == 0) atomicOr(&ctl->err, ERR_POS);
        return;
    }
    const uint32_t n = pos + 1, L = attn_split_len(n, a.max_splits), S = (n + L - 1) / L;
    if (s >= (a.mode != ATTN_APPEND_ONLY ? S : 1u)) return;
    attn::item<HD, nbuf(HD)>(a, a.layer, s, kvh, slot, pos, sm);
    tr.exit();
}

}  // namespace

size_t attn_split_smem(uint32_t head_dim) { return attn::item_smem(head_dim, nbuf((int)head_dim)); }

uint32_t attn_max_splits(uint32_t max_ctx) {
    const uint32_t chunks = (max_ctx + attn::kCh - 1) / attn::kCh;
    return chunks < 128 ? chunks : 128;
}

cudaError_t attn_split_set_smem_limits(int optin) {
    cudaError_t e = cudaFuncSetAttribute(k_attn_split<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_attn_split<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
}

cudaError_t launch_attn_split(uint32_t head_dim, const SplitAttnArgs& a, uint32_t slots, cudaStream_t st) {
    if (a.nkv == 0 || a.nh % a.nkv || a.nh / a.nkv > 8 || a.max_splits == 0 || (!a.out_f32 && !a.out_hi))
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(a.mode == ATTN_APPEND_ONLY ? 1 : a.max_splits, a.nkv, slots);
    cfg.blockDim = dim3(attn::kThreads);
    cfg.dynamicSmemBytes = attn_split_smem(head_dim);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (head_dim == 64) return cudaLaunchKernelEx(&cfg, k_attn_split<64>, a);
    if (head_dim == 128) return cudaLaunchKernelEx(&cfg, k_attn_split<128>, a);
    return cudaErrorInvalidValue;
}

}  // namespace hs
