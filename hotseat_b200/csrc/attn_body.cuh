// One (split, KV head, sequence) item of the split-KV GQA decode attention
// (model.rs:259-305 with an online softmax over chunks of 64 cached
// positions), shared by the split-attention kernel (attn_split.cu) and the
// persistent token kernel (token_fast.cu).
//
// A sequence at `pos` has n = pos+1 positions; split_len(n) positions per
// split (a multiple of 64, at most max_splits splits) and S = ceil(n /
// split_len) splits. The item rebuilds q (the group's query heads) and the new
// k, v from the QKV product (split-K partials added in split order, then the
// bias), applies RoPE (model.rs:365-373); split 0 appends k, v at `pos` to the
// sequence's KV region and marks the dirty pages (model.rs:268-275); the split
// holding `pos` uses its own copy of that row.
//
// Per chunk: scores for the group's heads, chunk maximum, rescale of the
// running sum and output, P.V. A single split writes the normalised output;
// otherwise each split writes (max, sum, unnormalised output) and the item
// that arrives last at the (sequence, KV head) counter combines the splits in
// split order and resets the counter. Every choice depends on n and max_ctx
// only, never on the batch or the grid, so a sequence's bits are the same in
// any batch and in either kernel. NBUF (1-4) is the number of K/V chunk
// buffers (NBUF - 1 chunks load while one computes): it changes how loads
// overlap compute, not the arithmetic.
//
// Runs on threads 0..255 of the CTA and synchronises them with named barrier
// 1, so a CTA may keep other warps (a producer) outside it.
#pragma once

#include <cfloat>

#include "kernels.h"

namespace hs {
namespace attn {

constexpr uint32_t kThreads = 256;
constexpr uint32_t kCh = 64;  // positions per chunk

__device__ __forceinline__ uint32_t ldv(const uint32_t* p) { return *(const volatile uint32_t*)p; }
__device__ __forceinline__ void sync256() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Tagged entries: a value and the tag of the write that produced it in one
// 8-byte word (value bits low, tag high), stored and loaded as single-copy
// atomic 8-byte accesses, so a reader that sees the tag it waits for sees
// that write's value: the data is its own completion flag (no barrier, no
// separate flag, no fence).
constexpr uint32_t kPollLimit = 1u << 22;  // polling rounds before a reader gives up
__device__ __forceinline__ void st_tagged(uint64_t* p, float v, uint32_t tag) {
    const uint64_t e = ((uint64_t)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(e) : "memory");
}
__device__ __forceinline__ void ld_tagged2(const uint64_t* p, uint64_t& e0, uint64_t& e1) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(e0), "=l"(e1) : "l"(p) : "memory");
}
__device__ __forceinline__ float tagged_value(uint64_t e) { return __uint_as_float((uint32_t)e); }

// The 256 consumer threads copy n_pairs pairs of tagged entries into shared
// memory once both entries of a pair carry `want`: map(i, &src, &dst) gives
// pair i's source (16-byte aligned) and destination. Each thread takes pairs
// tid, tid + 256, ..., B at a time, every round's loads in flight together.
// Returns false (values left unset) after `limit` rounds.
template <uint32_t B, typename Map>
__device__ bool poll_copy(uint32_t n_pairs, uint32_t want, uint32_t limit, Map map) {
    bool ok = true;
    for (uint32_t base = threadIdx.x; base < n_pairs; base += B * kThreads) {
        uint32_t pend = 0;
#pragma unroll
        for (uint32_t j = 0; j < B; j++)
            if (base + j * kThreads < n_pairs) pend |= 1u << j;
        uint32_t rounds = 0;
        while (pend) {
            uint64_t e[B][2];
#pragma unroll
            for (uint32_t j = 0; j < B; j++)
                if (pend >> j & 1) {
                    const uint64_t* src;
                    float* dst;
                    map(base + j * kThreads, &src, &dst);
                    ld_tagged2(src, e[j][0], e[j][1]);
                }
#pragma unroll
            for (uint32_t j = 0; j < B; j++)
                if ((pend >> j & 1) && (uint32_t)(e[j][0] >> 32) == want && (uint32_t)(e[j][1] >> 32) == want) {
                    const uint64_t* src;
                    float* dst;
                    map(base + j * kThreads, &src, &dst);
                    dst[0] = tagged_value(e[j][0]);
                    dst[1] = tagged_value(e[j][1]);
                    pend &= ~(1u << j);
                }
            if (pend && ++rounds > limit) {
                ok = false;
                break;
            }
        }
    }
    return ok;
}

// Tagged inputs and outputs of an item inside the persistent token kernel:
// q/k/v rows awaited with tag `want`, outputs (or, with reader_combines,
// the split records) written with tag `tag`.
struct TagIO {
    const uint64_t* qkv;  // [qkv rows]
    uint64_t* out;        // [n_heads * head_dim]
    uint64_t* rec;        // [n_kv][max_splits][attn_record]
    uint32_t want, tag;
    uint32_t poll_limit;  // polling rounds before the item gives up (ERR_TIMEOUT)
};

__device__ __forceinline__ void split_f16(float x, uint16_t* hi, uint16_t* lo) {
    const __half h = __float2half_rn(x);
    *hi = __half_as_ushort(h);
    *lo = __half_as_ushort(__float2half_rn(__fsub_rn(x, __half2float(h))));
}
__device__ __forceinline__ float4 f4add(float4 a, float4 b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

// Row strides (floats) of the K and V chunk buffers and of the score rows,
// chosen so that the tensor-core operand reads of a warp hit 32 distinct
// banks (K: 4 (row) + column; V: 8 (row) + column; scores: 4 (head) + position).
__host__ __device__ constexpr uint32_t k_stride(uint32_t hd) { return hd + 4; }
__host__ __device__ constexpr uint32_t v_stride(uint32_t hd) { return hd + 8; }
constexpr uint32_t SPS = kCh + 4;

// Shared memory of one item (floats): q [8][HD], k, v [HD], K chunks
// [NBUF][kCh][HD+4], V chunks [NBUF][kCh][HD+8], scores [2][8][SPS] (the two
// halves of the dimensions; probabilities in the first), per-head
// max/rescale/sum [3][8], a flag word (4 floats), q as tf32 operand fragments
// [2 halves][HD/16 k-steps][32 lanes][4] (hi, hi, lo, lo), the RoPE row of
// `pos` [HD/2 cos, HD/2 sin].
__host__ __device__ constexpr uint32_t item_rope_off(uint32_t hd, uint32_t nbuf) {
    return 8 * hd + 2 * hd + nbuf * kCh * (k_stride(hd) + v_stride(hd)) + 2 * 8 * SPS + 3 * 8 + 4 + 16 * hd;
}
__host__ __device__ constexpr size_t item_smem(uint32_t hd, uint32_t nbuf) {
    return (item_rope_off(hd, nbuf) + hd) * sizeof(float);
}

// x as a tf32 pair: hi = x rounded to tf32, lo = the rest rounded to tf32.
__device__ __forceinline__ void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hi) : "f"(x));
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(lo) : "f"(__fsub_rn(x, __uint_as_float(hi))));
}
// c += a . b, one m16n8k8 tile (a row-major 16x8, b column-major 8x8).
__device__ __forceinline__ void mma_tf32(float (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Split-order combine of the S published splits of one (sequence, KV head)
// for output element idx (head idx / HD of the group, dimension idx % HD):
// the maximum of the split maxima, then the rescaled sums and outputs in
// split order. GLOBAL: the partials are read through L2 (written by other
// CTAs); else from a shared-memory copy.
template <bool GLOBAL>
__device__ __forceinline__ float combine(const float* part, uint32_t S, uint32_t G, uint32_t hd, uint32_t idx) {
    const uint32_t rec = attn_record(G, hd), h = idx / hd;
    auto ld = [&](size_t i) { return GLOBAL ? __ldcg(part + i) : part[i]; };
    float M = -FLT_MAX;
    for (uint32_t q = 0; q < S; q++) M = fmaxf(M, ld((size_t)q * rec + G * hd + h));
    float num = 0.0f, den = 0.0f;
    for (uint32_t q = 0; q < S; q++) {
        const float w = __expf(__fsub_rn(ld((size_t)q * rec + G * hd + h), M));
        num = __fadd_rn(num, __fmul_rn(w, ld((size_t)q * rec + idx)));
        den = __fadd_rn(den, __fmul_rn(w, ld((size_t)q * rec + G * hd + G + h)));
    }
    return __fdiv_rn(num, den);
}

// combine<true> for every output element of the group at once, by the
// CTA's 256 threads, with the same operations in the same split order (the
// same bits): the S splits' maxima and sums are staged into shared memory
// `st` (the item's space, free by now) with parallel loads, the weights
// exp(m_q - M) computed once per (split, head), then the outputs kCombTile
// splits at a time, each element accumulating its splits one after another.
// Needs (3 * S * G + 19 + kCombTile * G * hd) floats of `st` (16-byte
// aligned), S <= 128, G <= 8.
constexpr uint32_t kCombTile = 16;
template <typename Store>
__device__ void combine_staged(const float* part, uint32_t S, uint32_t G, uint32_t hd, float* st, Store store) {
    const uint32_t rec = attn_record(G, hd), gh = G * hd, tid = threadIdx.x;
    float* ms = st;            // [S][G] maxima
    float* ls = ms + S * G;    // [S][G] sums
    float* ws = ls + S * G;    // [S][G] weights
    float* mx = ws + S * G;    // [8]
    float* den = mx + 8;       // [8]
    float* tile = st + ((3 * S * G + 16 + 3) & ~3u);  // [kCombTile][gh], 16-byte aligned for the float4 stores
    for (uint32_t i = tid; i < S * G; i += kThreads) {
        const uint32_t q = i / G, h = i % G;
        ms[i] = __ldcg(part + (size_t)q * rec + gh + h);
        ls[i] = __ldcg(part + (size_t)q * rec + gh + G + h);
    }
    sync256();
    if (tid < G) {
        float M = -FLT_MAX;
        for (uint32_t q = 0; q < S; q++) M = fmaxf(M, ms[q * G + tid]);
        mx[tid] = M;
    }
    sync256();
    for (uint32_t i = tid; i < S * G; i += kThreads) ws[i] = __expf(__fsub_rn(ms[i], mx[i % G]));
    sync256();
    if (tid < G) {
        float d = 0.0f;
        for (uint32_t q = 0; q < S; q++) d = __fadd_rn(d, __fmul_rn(ws[q * G + tid], ls[q * G + tid]));
        den[tid] = d;
    }
    constexpr uint32_t NPT = 4;  // outputs per thread: gh <= 8 * 128
    float num[NPT] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (uint32_t q0 = 0; q0 < S; q0 += kCombTile) {
        const uint32_t cnt = S - q0 < kCombTile ? S - q0 : kCombTile;
        sync256();  // the previous tile is consumed (and den is written)
        for (uint32_t i = tid; i < cnt * (gh / 4); i += kThreads) {
            const uint32_t t = i / (gh / 4), c4 = i % (gh / 4);
            reinterpret_cast<float4*>(tile + t * gh)[c4] =
                __ldcg(reinterpret_cast<const float4*>(part + (size_t)(q0 + t) * rec) + c4);
        }
        sync256();
#pragma unroll
        for (uint32_t j = 0; j < NPT; j++) {
            const uint32_t idx = tid + j * kThreads;
            if (idx < gh) {
                const uint32_t h = idx / hd;
                for (uint32_t t = 0; t < cnt; t++)
                    num[j] = __fadd_rn(num[j], __fmul_rn(ws[(q0 + t) * G + h], tile[t * gh + idx]));
            }
        }
    }
#pragma unroll
    for (uint32_t j = 0; j < NPT; j++) {
        const uint32_t idx = tid + j * kThreads;
        if (idx < gh) store(idx, __fdiv_rn(num[j], den[idx / hd]));
    }
}

__device__ __forceinline__ uint64_t kv_row_off(const SplitAttnArgs& a, uint32_t layer, uint32_t kvh, uint32_t hd,
                                               uint32_t p, uint32_t is_v) {
    const uint64_t plane = (uint64_t)a.max_ctx * a.nkv * hd;
    const uint64_t within = a.layout == 0 ? ((uint64_t)p * a.nkv + kvh) * hd : ((uint64_t)kvh * a.max_ctx + p) * hd;
    return (uint64_t)layer * 2 * plane + (is_v ? plane : 0) + within;
}

// Warp-split attend (SplitAttnArgs::ws_from): each of the 8 warps takes
// the blocks of WB positions b = w, w + 8, ... of the item's range and keeps
// WBUF of its blocks in flight in its own part of the chunk buffers.
template <int HD, int NBUF>
struct WsGeom {
    static constexpr uint32_t WB = 8, RW = HD + 4;
    static constexpr uint32_t AREA = NBUF * kCh * (k_stride(HD) + v_stride(HD)) + 2 * 8 * SPS;  // floats from kb on
    static constexpr uint32_t WONE = 2 * WB * RW;                                                 // one block's K and V rows
    static constexpr uint32_t QP = 8 * RW;  // q rows padded to RW (the head pairs' rows in distinct banks)
    static constexpr uint32_t FIT = AREA > QP ? ((AREA - QP) / 8 - 8 * WB - 8) / WONE : 0;
    static constexpr uint32_t WBUF = FIT > 4 ? 4 : (FIT < 1 ? 1 : FIT);
    static constexpr uint32_t WS = WBUF * WONE + 8 * WB + 8;                                      // floats of a warp's area
    static constexpr bool OK = 8 * WS + QP <= AREA && 8 * 8 * HD + 3 * 64 <= AREA;  // fits this item's buffers
};

// Stages block b of warp `warp` (local block index b / 8 picks the buffer)
// of the range [p0, p1) into its area: every cached row with 16-byte
// asynchronous copies, the row at `pos` from kn / vn when `fill_pos` (the
// item appends it and it is not in memory yet) or left out when `skip_pos`
// (a prefetch before kn / vn exist). One commit group per call, empty past
// the range's end.
template <int HD, int NBUF>
__device__ __forceinline__ void ws_stage(const SplitAttnArgs& a, const float* kv, uint32_t layer, uint32_t kvh,
                                         float* kb, uint32_t warp, uint32_t lane, uint32_t b, uint32_t p0,
                                         uint32_t p1, uint32_t pos, bool fill_pos, bool skip_pos, const float* kn,
                                         const float* vn) {
    using W = WsGeom<HD, NBUF>;
    const uint32_t nb = (p1 - p0 + W::WB - 1) / W::WB;
    if (b < nb) {
        const uint32_t pb = p0 + b * W::WB, cnt = p1 - pb < W::WB ? p1 - pb : W::WB;
        float* wk = kb + warp * W::WS + ((b / 8) % W::WBUF) * W::WONE;
        float* wv = wk + W::WB * W::RW;
        for (uint32_t i = lane; i < cnt * (HD / 4); i += 32) {
            const uint32_t rr = i / (HD / 4), c4 = i % (HD / 4);
            if (pb + rr == pos && (fill_pos || skip_pos)) {
                if (fill_pos) {
                    *reinterpret_cast<float4*>(wk + rr * W::RW + 4 * c4) = *reinterpret_cast<const float4*>(kn + 4 * c4);
                    *reinterpret_cast<float4*>(wv + rr * W::RW + 4 * c4) = *reinterpret_cast<const float4*>(vn + 4 * c4);
                }
            } else {
                cp_async16(wk + rr * W::RW + 4 * c4, kv + kv_row_off(a, layer, kvh, HD, pb + rr, 0) + 4 * c4);
                cp_async16(wv + rr * W::RW + 4 * c4, kv + kv_row_off(a, layer, kvh, HD, pb + rr, 1) + 4 * c4);
            }
        }
    }
    cp_commit();
}

// The warp-split counterpart of prefetch(): the RoPE row of `pos` and each
// warp's first WBUF blocks (all but the row at `pos`), WBUF commit groups
// per thread (the first with the RoPE row). Returns WBUF.
template <int HD, int NBUF>
__device__ uint32_t ws_prefetch(const SplitAttnArgs& a, uint32_t layer, uint32_t s, uint32_t kvh, uint32_t slot,
                                uint32_t pos, float* sm) {
    using W = WsGeom<HD, NBUF>;
    static_assert(W::OK, "warp-split staging must fit the item's chunk buffers");
    const uint32_t n = pos + 1, L = attn_split_len(n, a.max_splits, a.ws_from, a.min_split);
    const uint32_t p0 = s * L, p1 = p0 + L < n ? p0 + L : n;
    float* rope = sm + item_rope_off(HD, NBUF);
    if (threadIdx.x < HD / 4) {
        const uint32_t i = threadIdx.x % (HD / 8), half = threadIdx.x / (HD / 8);
        const float* src = (half ? a.rope_sin : a.rope_cos) + (size_t)pos * (HD / 2) + 4 * i;
        cp_async16(rope + half * (HD / 2) + 4 * i, src);
    }
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (uint32_t i = 0; i < W::WBUF; i++)
        ws_stage<HD, NBUF>(a, a.kv[slot], layer, kvh, sm + 10 * HD, warp, lane, warp + 8 * i, p0, p1, pos, false, true,
                           nullptr, nullptr);
    return W::WBUF;
}

// Issues the asynchronous loads of the RoPE row and of the cached rows of
// an item's first `nch` chunks (at most NBUF), all but `pos`, into its
// buffers, one commit group per chunk (the RoPE row with the first): those
// rows do not depend on this token, so a caller may start them before the
// QKV product exists and then run item(..., npre = the chunks issued).
// Returns the chunks issued (fewer when the split has fewer).
template <int HD, int NBUF>
__device__ uint32_t prefetch(const SplitAttnArgs& a, uint32_t layer, uint32_t s, uint32_t kvh, uint32_t slot,
                             uint32_t pos, float* sm, uint32_t nch = 1) {
    constexpr uint32_t RSK = k_stride(HD), RSV = v_stride(HD);
    float* kb = sm + 10 * HD;
    float* vb = kb + NBUF * kCh * RSK;
    const uint32_t n = pos + 1, L = attn_split_len(n, a.max_splits, a.ws_from, a.min_split);
    const uint32_t p0 = s * L, p1 = p0 + L < n ? p0 + L : n, have = (p1 - p0 + kCh - 1) / kCh;
    if (nch > have) nch = have;
    const float* kv = a.kv[slot];
    float* rope = sm + item_rope_off(HD, NBUF);
    if (threadIdx.x < HD / 4) {  // HD/8 16-byte pieces of each of the cos and sin halves
        const uint32_t i = threadIdx.x % (HD / 8), half = threadIdx.x / (HD / 8);
        const float* src = (half ? a.rope_sin : a.rope_cos) + (size_t)pos * (HD / 2) + 4 * i;
        cp_async16(rope + half * (HD / 2) + 4 * i, src);
    }
    for (uint32_t c = 0; c < nch; c++) {
        const uint32_t c0 = p0 + c * kCh, cnt = p1 - c0 < kCh ? p1 - c0 : kCh;
        for (uint32_t idx = threadIdx.x; idx < cnt * (HD / 4); idx += kThreads) {
            const uint32_t r = idx / (HD / 4), c4 = idx % (HD / 4);
            if (c0 + r == pos) continue;
            cp_async16(kb + (c * kCh + r) * RSK + 4 * c4, kv + kv_row_off(a, layer, kvh, HD, c0 + r, 0) + 4 * c4);
            cp_async16(vb + (c * kCh + r) * RSV + 4 * c4, kv + kv_row_off(a, layer, kvh, HD, c0 + r, 1) + 4 * c4);
        }
        cp_commit();
    }
    if (nch == 0) cp_commit();  // the RoPE row alone
    return nch > 0 ? nch : 1;
}

// Tensor-core warp-split attend (SplitAttnArgs::tcw; tensor-core path):
// warp w < NW takes the blocks of 16 positions b = w, w + NW, ... of the
// item's range, staged by cp.async into its own WB = 2 buffers, one block
// ahead (K rows padded by 8 floats, V rows by 4: the fragment loads of a
// warp hit distinct banks); NW = 8 warps at head_dim 64, 6 at 128 (the
// buffers that fit the item's space; the other warps take no block; 4 warps
// x 3 buffers at 128 measured slower, 34.5 vs 31.2 µs per layer at batch
// 16, 2k positions: the warps' compute matters more than the extra block in
// flight), and runs scores and P.V on
// mma.sync m16n8k16 with every
// operand an f16 pair hi = f16(x), lo = f16(x - hi) and every product
// lo*hi + hi*lo + hi*hi into the same f32 accumulator; rows are the group's
// query heads (16-row tile, rows past the group zero), each warp keeps its
// own online softmax, and the warps merge in warp order at the end.
template <int HD_, int NBUF>
struct TcwGeom {
    static constexpr uint32_t HD = HD_, PB = 16, KS = HD + 8, VS = HD + 4;
    static constexpr uint32_t BUF = PB * KS + PB * VS;  // floats of one block buffer (K then V)
    static constexpr uint32_t WB = 2;                   // buffers per warp
    static constexpr uint32_t WS = WB * BUF;            // floats of a warp's area
    static constexpr uint32_t AREA = NBUF * kCh * (k_stride(HD) + v_stride(HD)) + 2 * 8 * SPS;
    static constexpr uint32_t FIT = AREA / WS;
    static constexpr uint32_t NW = FIT > 8 ? 8 : FIT;  // warps that take blocks
    static constexpr bool OK = (HD == 64 || HD == 128) && NW >= 4 && 3 * 64 + 8 * 8 * HD <= AREA;
};

__device__ __forceinline__ void h2split(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(__fsub_rn(x0, hf.x), __fsub_rn(x1, hf.y));
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Stages block b of warp `warp` (local block b / NW picks buffer (b / NW) % WB)
// of the range [p0, p1): every cached row with 16-byte cp.async copies, the
// row at `pos` from kn / vn when `fill_pos` or left out when `skip_pos` (a
// prefetch before kn / vn exist); V rows past the range's end zero (their
// probabilities are 0, and 0 times a stale non-finite value would not be).
// One commit group per call, empty past the range's end.
template <int HD, int NBUF>
__device__ __forceinline__ void tcw_stage(const SplitAttnArgs& a, const float* kv, uint32_t layer, uint32_t kvh,
                                          float* area, uint32_t warp, uint32_t lane, uint32_t b, uint32_t p0,
                                          uint32_t p1, uint32_t pos, bool fill_pos, bool skip_pos, const float* kn,
                                          const float* vn) {
    using T = TcwGeom<HD, NBUF>;
    const uint32_t nb = (p1 - p0 + T::PB - 1) / T::PB;
    if (warp < T::NW && b < nb) {
        const uint32_t pb = p0 + b * T::PB, cnt = p1 - pb < T::PB ? p1 - pb : T::PB;
        float* kd = area + warp * T::WS + ((b / T::NW) % T::WB) * T::BUF;
        float* vd = kd + T::PB * T::KS;
        for (uint32_t i = lane; i < T::PB * (T::HD / 4); i += 32) {
            const uint32_t rr = i / (T::HD / 4), c4 = i % (T::HD / 4);
            if (rr >= cnt) {
                *reinterpret_cast<float4*>(vd + rr * T::VS + 4 * c4) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            } else if (pb + rr == pos && (fill_pos || skip_pos)) {
                if (fill_pos) {
                    *reinterpret_cast<float4*>(kd + rr * T::KS + 4 * c4) = *reinterpret_cast<const float4*>(kn + 4 * c4);
                    *reinterpret_cast<float4*>(vd + rr * T::VS + 4 * c4) = *reinterpret_cast<const float4*>(vn + 4 * c4);
                }
            } else {
                cp_async16(kd + rr * T::KS + 4 * c4, kv + kv_row_off(a, layer, kvh, T::HD, pb + rr, 0) + 4 * c4);
                cp_async16(vd + rr * T::VS + 4 * c4, kv + kv_row_off(a, layer, kvh, T::HD, pb + rr, 1) + 4 * c4);
            }
        }
    }
    cp_commit();
}

// The tensor-core warp-split counterpart of prefetch(): the RoPE row of
// `pos` and each warp's first block (all but the row at `pos`), one commit
// group per thread. Returns 1.
template <int HD, int NBUF>
__device__ uint32_t tcw_prefetch(const SplitAttnArgs& a, uint32_t layer, uint32_t s, uint32_t kvh, uint32_t slot,
                                 uint32_t pos, float* sm) {
    using T = TcwGeom<HD, NBUF>;
    static_assert(T::OK, "tensor-core warp-split staging must fit the item's chunk buffers");
    const uint32_t n = pos + 1, L = attn_split_len(n, a.max_splits, a.ws_from, a.min_split);
    const uint32_t p0 = s * L, p1 = p0 + L < n ? p0 + L : n;
    float* rope = sm + item_rope_off(T::HD, NBUF);
    if (threadIdx.x < T::HD / 4) {
        const uint32_t i = threadIdx.x % (T::HD / 8), half = threadIdx.x / (T::HD / 8);
        const float* src = (half ? a.rope_sin : a.rope_cos) + (size_t)pos * (T::HD / 2) + 4 * i;
        cp_async16(rope + half * (T::HD / 2) + 4 * i, src);
    }
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    tcw_stage<HD, NBUF>(a, a.kv[slot], layer, kvh, sm + 10 * T::HD, warp, lane, warp, p0, p1, pos, false, true,
                        nullptr, nullptr);
    return 1;
}

// Waits until at most n (0..3) commit groups are pending.
__device__ __forceinline__ void cp_wait_pending(uint32_t n) {
    switch (n) {
        case 0: cp_wait<0>(); break;
        case 1: cp_wait<1>(); break;
        case 2: cp_wait<2>(); break;
        default: cp_wait<3>(); break;
    }
}

// One item: split s of KV head kvh, query-head part hpart, for sequence
// slot `slot` at `pos`. Preconditions (checked by the caller): the sequence
// is active, pos < max_ctx, s < S (attend) or s == 0 (append only); `npre` >
// 0 only in ATTN_FULL mode, as prefetch()'s return for the same item (whose
// first group also loaded the RoPE row), with no commit group issued since.
// `layer` selects the KV planes (a.layer is not read). TC: the chunk
// products on the tensor cores, else on the CUDA cores. With
// `reader_combines`, several splits only publish their partials: the reader
// of the output combines them once all are published (the persistent token
// kernel's O phase, polling the tagged records).
template <int HD, int NBUF, bool TC>
__device__ void item(const SplitAttnArgs& a, uint32_t layer, uint32_t s, uint32_t kvh, uint32_t hpart, uint32_t slot,
                     uint32_t pos, float* sm, uint32_t npre = 0, bool reader_combines = false,
                     uint64_t* probe = nullptr, const TagIO* tio = nullptr) {
    // probe (timing): thread 0 stores clock64() at the item's checkpoints
    auto at = [&](int k) {
        if (probe && threadIdx.x == 0) probe[k] = clock64();
    };
    at(0);
    static_assert(NBUF >= 1 && NBUF <= 4, "one to four chunk buffers");
    constexpr uint32_t RSK = k_stride(HD), RSV = v_stride(HD), HALF = HD / 2;
    constexpr uint32_t HSETS = kThreads / HD, HPT = (8 + HSETS - 1) / HSETS;
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // this item's query heads: part hpart of the group's Gf heads
    const uint32_t Gf = a.nh / a.nkv, hsplit = attn_head_split(a);
    const uint32_t hlo = hpart * Gf / hsplit, G = (hpart + 1) * Gf / hsplit - hlo;
    float* qs = sm;                        // [8][HD]
    float* kn = qs + 8 * HD;               // [HD]
    float* vn = kn + HD;                   // [HD]
    float* kb = vn + HD;                   // [NBUF][kCh][RSK]
    float* vb = kb + NBUF * kCh * RSK;     // [NBUF][kCh][RSV]
    float* sp = vb + NBUF * kCh * RSV;     // [2][8][SPS] scores, then probabilities
    float* hs_m = sp + 2 * 8 * SPS;        // [8] running maximum per head
    float* hs_f = hs_m + 8;                // [8] rescale of the running sums this chunk
    float* hs_l = hs_f + 8;                // [8] running sums
    uint32_t* flag = reinterpret_cast<uint32_t*>(hs_l + 8);
    uint4* qfrag = reinterpret_cast<uint4*>(hs_l + 12);  // [2][HD/16][32]
    const float* rope = sm + item_rope_off(HD, NBUF);
    const uint32_t n = pos + 1, L = attn_split_len(n, a.max_splits, a.ws_from, a.min_split), S = (n + L - 1) / L;
    // Prefill runs append (every token's k, v) and attend (reading all rows
    // from memory) as two launches, so tokens of one sequence in one batch
    // see each other's rows.
    const bool append = a.mode != ATTN_ATTEND_ONLY, attend = a.mode != ATTN_APPEND_ONLY;
    const uint32_t p0 = s * L, p1 = p0 + L < n ? p0 + L : n;
    float* kv = a.kv[slot];
    auto row_off = [&](uint32_t p, uint32_t is_v) -> uint64_t { return kv_row_off(a, layer, kvh, HD, p, is_v); };
    // split 0's first head part appends the new row; read the tracking flag
    // now, mark later
    const bool appender = s == 0 && hpart == 0 && append;
    const bool track = appender && tid < 2 && ldv(a.tracking[slot]) != 0;

    // q, k, v of this group; split-K partials in split order, then the bias
    // (or, tagged, the finished rows once they carry the awaited tag).
    const uint32_t qrow0 = (kvh * Gf + hlo) * HD, krow0 = a.nh * HD + kvh * HD, vrow0 = (a.nh + a.nkv) * HD + kvh * HD;
    if (tio) {
        const bool got = poll_copy<2>((G + 2) * HD / 2, tio->want, tio->poll_limit,
                                      [&](uint32_t i, const uint64_t** src, float** dst) {
            const uint32_t idx = 2 * i;
            *src = tio->qkv + (idx < G * HD ? qrow0 + idx
                                            : (idx < (G + 1) * HD ? krow0 + idx - G * HD : vrow0 + idx - (G + 1) * HD));
            *dst = idx < G * HD ? qs + idx : (idx < (G + 1) * HD ? kn + idx - G * HD : vn + idx - (G + 1) * HD);
        });
        if (!got) atomicOr(&a.ctl[slot].err, ERR_TIMEOUT);
    }
    for (uint32_t c = tid; !tio && c < (G + 2) * HD / 4; c += kThreads) {
        const uint32_t idx = 4 * c;
        const uint32_t row = idx < G * HD ? qrow0 + idx : (idx < (G + 1) * HD ? krow0 + idx - G * HD : vrow0 + idx - (G + 1) * HD);
        const float* src = a.qkv + (size_t)slot * a.qkv_rows + row;
        float4 p = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (uint32_t q0 = 0; q0 < a.n_part; q0 += 8) {
            float4 v[8];
#pragma unroll
            for (uint32_t j = 0; j < 8; j++)
                if (q0 + j < a.n_part) v[j] = __ldcg(reinterpret_cast<const float4*>(src + (q0 + j) * a.part_stride));
#pragma unroll
            for (uint32_t j = 0; j < 8; j++)
                if (q0 + j < a.n_part) p = f4add(p, v[j]);
        }
        if (a.bias) p = f4add(p, *reinterpret_cast<const float4*>(a.bias + row));
        float* dst = idx < G * HD ? qs + idx : (idx < (G + 1) * HD ? kn + idx - G * HD : vn + idx - (G + 1) * HD);
        *reinterpret_cast<float4*>(dst) = p;
    }
    const bool prefetched = npre > 0;
    if (prefetched) cp_wait_pending(npre - 1);  // the RoPE row and the first chunk
    sync256();
    at(1);
    for (uint32_t idx = tid; idx < (G + 1) * HALF; idx += kThreads) {
        const uint32_t h = idx / HALF, i = idx % HALF;
        float* r = h < G ? qs + h * HD : kn;
        const float c = prefetched ? rope[i] : a.rope_cos[(size_t)pos * HALF + i];
        const float sn = prefetched ? rope[HALF + i] : a.rope_sin[(size_t)pos * HALF + i];
        const float x0 = r[i], x1 = r[i + HALF];
        r[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
        r[i + HALF] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
    if (tid < 8) {
        hs_m[tid] = -FLT_MAX;
        hs_l[tid] = 0.0f;
    }
    sync256();
    at(2);
    if (appender && tid < HD) {
        kv[row_off(pos, 0) + tid] = kn[tid];
        kv[row_off(pos, 1) + tid] = vn[tid];
    }
    // Dirty-page bits of the appended row, set after the row is visible (a
    // harvest may run concurrently); called after a block barrier that
    // follows the row's stores.
    auto mark_dirty = [&]() {
        if (track) {
            __threadfence();
            const uint64_t off = row_off(pos, tid) * 4, last = off + HD * 4 - 1;
            uint64_t* dirty = a.dirty[slot];
            for (uint64_t pg = off >> a.page_shift; pg <= (last >> a.page_shift); pg++)
                atomicOr(reinterpret_cast<unsigned long long*>(&dirty[pg >> 6]), 1ull << (pg & 63));
        }
    };
    if (!attend) {
        sync256();
        mark_dirty();
        return;
    }

    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
    const uint32_t dd = tid % HD, hs0 = tid / HD;
    float o[HPT];  // dimension dd of heads hs0 + j HSETS (both paths end here)
#pragma unroll
    for (uint32_t j = 0; j < HPT; j++) o[j] = 0.0f;
    // (the warp-split form exists only where its staging fits this item's buffers)
    bool use_ws = false, use_tcw = false;
    if constexpr (TC && TcwGeom<HD, NBUF>::OK) use_tcw = a.tcw != 0;
    if constexpr (WsGeom<HD, NBUF>::OK) use_ws = !use_tcw && attn_use_ws(n, a.ws_from);
    if (use_tcw) {
      if constexpr (TC && TcwGeom<HD, NBUF>::OK) {
        using T = TcwGeom<HD, NBUF>;
        constexpr uint32_t PB = T::PB, KS = T::KS, VS = T::VS, NW = T::NW, WB = T::WB, KK = HD / 16, ND = HD / 8;
        const uint32_t g = lane >> 2, t4 = lane & 3;
        const uint32_t nb = (p1 - p0 + PB - 1) / PB;
        float* area = kb;
        // q as A fragments: row g = query head g of the part (zero past G),
        // rows 8-15 zero; split into f16 pairs once
        uint32_t qh[KK][2], ql[KK][2];
        const bool live = g < G;
#pragma unroll
        for (uint32_t kk = 0; kk < KK; kk++) {
            const float* qr = qs + g * HD + 16 * kk + 2 * t4;
            h2split(live ? qr[0] : 0.0f, live ? qr[1] : 0.0f, qh[kk][0], ql[kk][0]);
            h2split(live ? qr[8] : 0.0f, live ? qr[9] : 0.0f, qh[kk][1], ql[kk][1]);
        }
        // block 0 of every block-taking warp was staged by tcw_prefetch()
        // without the row at pos: the warp that holds it fills it now
        if (npre > 0 && pos >= p0 && pos < p1 && (pos - p0) / PB == warp && warp < NW) {
            float* kd = area + warp * T::WS;
            float* vd = kd + PB * KS;
            const uint32_t rr = (pos - p0) % PB;
            for (uint32_t c4 = lane; c4 < HD / 4; c4 += 32) {
                *reinterpret_cast<float4*>(kd + rr * KS + 4 * c4) = *reinterpret_cast<const float4*>(kn + 4 * c4);
                *reinterpret_cast<float4*>(vd + rr * VS + 4 * c4) = *reinterpret_cast<const float4*>(vn + 4 * c4);
            }
        }
        auto stage = [&](uint32_t i) {  // this warp's local block i
            tcw_stage<HD, NBUF>(a, kv, layer, kvh, area, warp, lane, warp + NW * i, p0, p1, pos, append, false, kn,
                                vn);
        };
        // local blocks 0 .. WB-2 in flight before the loop (block 0 from
        // tcw_prefetch() when it ran); each iteration issues block i + WB - 1
        // (an empty group past the end) and waits for block i
        for (uint32_t i = npre > 0 ? 1u : 0u; i + 1 < WB; i++) stage(i);
        float rm = -FLT_MAX, rl = 0.0f;  // running max / sum of row g
        float O[ND][2];                  // row g's output, dimensions 8 d + 2 t4 (+1)
#pragma unroll
        for (uint32_t d = 0; d < ND; d++) O[d][0] = O[d][1] = 0.0f;
        const uint32_t nloc = warp < NW && nb > warp ? (nb - warp + NW - 1) / NW : 0;
        for (uint32_t i = 0; i < nloc; i++) {
            stage(i + WB - 1);
            cp_wait<WB - 1>();  // block i landed
            __syncwarp();
            if (i == 0 && warp == 0) at(3);
            const uint32_t pb = p0 + (warp + NW * i) * PB, cnt = p1 - pb < PB ? p1 - pb : PB;
            const float* kd = area + warp * T::WS + (i % WB) * T::BUF;
            const float* vd = kd + PB * KS;
            float S[2][4];
#pragma unroll
            for (uint32_t j = 0; j < 2; j++) S[j][0] = S[j][1] = S[j][2] = S[j][3] = 0.0f;
#pragma unroll
            for (uint32_t kk = 0; kk < KK; kk++) {
                const uint32_t ah[4] = {qh[kk][0], 0u, qh[kk][1], 0u}, al[4] = {ql[kk][0], 0u, ql[kk][1], 0u};
#pragma unroll
                for (uint32_t j = 0; j < 2; j++) {
                    const float* kr = kd + (8 * j + g) * KS + 16 * kk + 2 * t4;
                    const float2 x0 = *reinterpret_cast<const float2*>(kr);
                    const float2 x1 = *reinterpret_cast<const float2*>(kr + 8);
                    uint32_t bh0, bl0, bh1, bl1;
                    h2split(x0.x, x0.y, bh0, bl0);
                    h2split(x1.x, x1.y, bh1, bl1);
                    mma16816(S[j], al, bh0, bh1);
                    mma16816(S[j], ah, bl0, bl1);
                    mma16816(S[j], ah, bh0, bh1);
                }
            }
            // online softmax of row g over the block's positions 8 j + 2 t4 + e;
            // selects, not branches: every lane takes every shuffle
            float sv[4] = {S[0][0], S[0][1], S[1][0], S[1][1]};
            float mx = -FLT_MAX;
#pragma unroll
            for (uint32_t e = 0; e < 4; e++) {
                const uint32_t col = (e >> 1) * 8 + 2 * t4 + (e & 1);
                sv[e] = live && col < cnt ? __fmul_rn(sv[e], scale) : -FLT_MAX;
                mx = fmaxf(mx, sv[e]);
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const bool none = mx == -FLT_MAX;
            const float mn = none ? rm : fmaxf(rm, mx);
            float sum = 0.0f;
#pragma unroll
            for (uint32_t e = 0; e < 4; e++) {
                sv[e] = sv[e] == -FLT_MAX ? 0.0f : __expf(__fsub_rn(sv[e], mn));
                sum = __fadd_rn(sum, sv[e]);
            }
            sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 1));
            sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 2));
            const float f = none ? 1.0f : (rm == -FLT_MAX ? 0.0f : __expf(__fsub_rn(rm, mn)));
            rl = none ? rl : __fadd_rn(__fmul_rn(rl, f), sum);
            rm = mn;
            uint32_t ph[4], pl[4];
            h2split(sv[0], sv[1], ph[0], pl[0]);
            h2split(sv[2], sv[3], ph[2], pl[2]);
            ph[1] = pl[1] = ph[3] = pl[3] = 0u;
#pragma unroll
            for (uint32_t d = 0; d < ND; d++) {
                // rows 8-15 of P are zero, so their outputs stay zero: fresh
                // zeros stand in for them
                float acc[4] = {__fmul_rn(O[d][0], f), __fmul_rn(O[d][1], f), 0.0f, 0.0f};
                const float* vr = vd + 2 * t4 * VS + 8 * d + g;
                uint32_t bh0, bl0, bh1, bl1;
                h2split(vr[0], vr[VS], bh0, bl0);
                h2split(vr[8 * VS], vr[9 * VS], bh1, bl1);
                mma16816(acc, pl, bh0, bh1);
                mma16816(acc, ph, bl0, bl1);
                mma16816(acc, ph, bh0, bh1);
                O[d][0] = acc[0];
                O[d][1] = acc[1];
            }
            __syncwarp();  // this buffer is restaged WB blocks on
        }
        cp_wait0();
        sync256();  // every warp is done with its area: the merge reuses it
        // merge: warp w's maxima, sums and outputs of rows 0-7 (warps past NW:
        // no block, weight 0), then per head the weights exp(m_w - M) and the
        // sums in warp order
        float* mm = kb;          // [8 warps][8 heads]
        float* ll = mm + 64;     // [8][8]
        float* wt = ll + 64;     // [8][8] weights
        float* ao = wt + 64;     // [8 warps][8 heads][HD]
        if (t4 == 0) {
            mm[warp * 8 + g] = rm;
            ll[warp * 8 + g] = rl;
        }
#pragma unroll
        for (uint32_t d = 0; d < ND; d++)
            *reinterpret_cast<float2*>(ao + (warp * 8 + g) * HD + 8 * d + 2 * t4) = make_float2(O[d][0], O[d][1]);
        sync256();
        if (tid < G) {
            float M = -FLT_MAX;
            for (uint32_t w = 0; w < 8; w++) M = fmaxf(M, mm[w * 8 + tid]);
            float l = 0.0f;
            for (uint32_t w = 0; w < 8; w++) {
                const float m_w = mm[w * 8 + tid];
                const float x = m_w == -FLT_MAX ? 0.0f : __expf(__fsub_rn(m_w, M));
                wt[w * 8 + tid] = x;
                l = __fadd_rn(l, __fmul_rn(x, ll[w * 8 + tid]));
            }
            hs_m[tid] = M;
            hs_l[tid] = l;
        }
        sync256();
#pragma unroll
        for (uint32_t j = 0; j < HPT; j++) {
            const uint32_t h = hs0 + j * HSETS;
            if (h < G) {
                float v = 0.0f;
                for (uint32_t w = 0; w < 8; w++) v = __fadd_rn(v, __fmul_rn(wt[w * 8 + h], ao[(w * 8 + h) * HD + dd]));
                o[j] = v;
            }
        }
      }
    } else if (use_ws) {
      if constexpr (WsGeom<HD, NBUF>::OK) {
        // Warp-split attend: warp w takes the blocks of WB positions b = w,
        // w + 8, w + 16, ... of [p0, p1) and keeps its own online softmax per
        // head, with no block barrier inside the loop (each warp stages its
        // blocks' K and V rows itself, WBUF blocks in flight); the warps'
        // states merge in warp order at the end. Scores on the CUDA cores in
        // fp32 (lane: position b*WB + lane % WB, heads 2 (lane / WB) and +1),
        // P.V on the CUDA cores (lane: dimensions DPL lane .. +DPL-1).
        using W = WsGeom<HD, NBUF>;
        constexpr uint32_t WB = W::WB, DPL = HD / 32, RW = W::RW, WBUF = W::WBUF, WS = W::WS, WONE = W::WONE;
        float* wa = kb + warp * WS;
        float* wp = wa + WBUF * WONE;  // [WB][8 heads] probabilities of the block
        float* wf = wp + 8 * WB;       // [8] rescale of the running sums
        float* qp = kb + 8 * WS;       // [8][RW] q rows, padded
        for (uint32_t i = tid; i < G * (HD / 4); i += kThreads)
            reinterpret_cast<float4*>(qp + (i / (HD / 4)) * RW)[i % (HD / 4)] = reinterpret_cast<const float4*>(qs)[i];
        sync256();
        const uint32_t nr = p1 - p0, nb = (nr + WB - 1) / WB;
        const uint32_t r = lane % WB, hq = lane / WB, h0 = 2 * hq, h1 = 2 * hq + 1;
        // blocks of this warp staged so far: WBUF when ws_prefetch() ran
        // (the row at pos left out: filled here once kn / vn exist)
        uint32_t issued = npre > 0 ? WBUF : 0;
        if (npre > 0 && append && pos >= p0 && pos < p1) {
            const uint32_t bp = (pos - p0) / WB;
            if (bp % 8 == warp && bp / 8 < WBUF) {
                float* wk = wa + ((bp / 8) % WBUF) * WONE;
                const uint32_t rr = (pos - p0) % WB;
                for (uint32_t c4 = lane; c4 < HD / 4; c4 += 32) {
                    reinterpret_cast<float4*>(wk + rr * RW)[c4] = reinterpret_cast<const float4*>(kn)[c4];
                    reinterpret_cast<float4*>(wk + WB * RW + rr * RW)[c4] = reinterpret_cast<const float4*>(vn)[c4];
                }
            }
        }
        auto stage = [&](uint32_t i) {  // this warp's local block i
            ws_stage<HD, NBUF>(a, kv, layer, kvh, kb, warp, lane, warp + 8 * i, p0, p1, pos, append, false, kn, vn);
        };
        float rm0 = -FLT_MAX, rm1 = -FLT_MAX, rl0 = 0.0f, rl1 = 0.0f;  // running max / sum of heads h0, h1
        float acc[8][DPL];
#pragma unroll
        for (uint32_t h = 0; h < 8; h++)
#pragma unroll
            for (uint32_t k = 0; k < DPL; k++) acc[h][k] = 0.0f;
        for (; issued + 1 < WBUF; issued++) stage(issued);
        for (uint32_t b = warp; b < nb; b += 8) {
            for (; issued < b / 8 + WBUF; issued++) stage(issued);
            cp_wait<WBUF - 1>();  // this block's group: exactly WBUF - 1 younger ones are committed
            __syncwarp();
            if (b == warp) at(3);  // warp 0's first block ready
            const uint32_t pb = p0 + b * WB, cnt = p1 - pb < WB ? p1 - pb : WB;
            const float* wk = wa + ((b / 8) % WBUF) * WONE;
            const float* wv = wk + WB * RW;
            float s0 = -FLT_MAX, s1 = -FLT_MAX;
            if (r < cnt) {
                float a0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, a1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                const float4* k4 = reinterpret_cast<const float4*>(wk + r * RW);
                const float4* q0 = reinterpret_cast<const float4*>(qp + (h0 < G ? h0 : 0) * RW);
                const float4* q1 = reinterpret_cast<const float4*>(qp + (h1 < G ? h1 : 0) * RW);
#pragma unroll 8
                for (uint32_t d4 = 0; d4 < HD / 4; d4++) {
                    const float4 kk = k4[d4], x = q0[d4], y = q1[d4];
                    a0[0] = __fmaf_rn(x.x, kk.x, a0[0]);
                    a0[1] = __fmaf_rn(x.y, kk.y, a0[1]);
                    a0[2] = __fmaf_rn(x.z, kk.z, a0[2]);
                    a0[3] = __fmaf_rn(x.w, kk.w, a0[3]);
                    a1[0] = __fmaf_rn(y.x, kk.x, a1[0]);
                    a1[1] = __fmaf_rn(y.y, kk.y, a1[1]);
                    a1[2] = __fmaf_rn(y.z, kk.z, a1[2]);
                    a1[3] = __fmaf_rn(y.w, kk.w, a1[3]);
                }
                if (h0 < G) s0 = __fmul_rn(__fadd_rn(__fadd_rn(a0[0], a0[1]), __fadd_rn(a0[2], a0[3])), scale);
                if (h1 < G) s1 = __fmul_rn(__fadd_rn(__fadd_rn(a1[0], a1[1]), __fadd_rn(a1[2], a1[3])), scale);
            }
            // the block's maximum and sum per head over the WB lanes of the group
            float mx0 = s0, mx1 = s1;
#pragma unroll
            for (uint32_t off = 1; off < WB; off <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
            }
            const float n0 = fmaxf(rm0, mx0), n1 = fmaxf(rm1, mx1);
            const float e0 = r < cnt && h0 < G ? __expf(__fsub_rn(s0, n0)) : 0.0f;
            const float e1 = r < cnt && h1 < G ? __expf(__fsub_rn(s1, n1)) : 0.0f;
            float sm0 = e0, sm1 = e1;
#pragma unroll
            for (uint32_t off = 1; off < WB; off <<= 1) {
                sm0 = __fadd_rn(sm0, __shfl_xor_sync(0xffffffffu, sm0, off));
                sm1 = __fadd_rn(sm1, __shfl_xor_sync(0xffffffffu, sm1, off));
            }
            const float f0 = rm0 == -FLT_MAX ? 0.0f : __expf(__fsub_rn(rm0, n0));
            const float f1 = rm1 == -FLT_MAX ? 0.0f : __expf(__fsub_rn(rm1, n1));
            rl0 = __fadd_rn(__fmul_rn(rl0, f0), sm0);
            rl1 = __fadd_rn(__fmul_rn(rl1, f1), sm1);
            rm0 = n0;
            rm1 = n1;
            wp[r * 8 + h0] = e0;
            wp[r * 8 + h1] = e1;
            if (r == 0) {
                wf[h0] = f0;
                wf[h1] = f1;
            }
            __syncwarp();
            // each position's V slice and all heads' probabilities read once
            float pv[8][DPL];
#pragma unroll
            for (uint32_t h = 0; h < 8; h++)
#pragma unroll
                for (uint32_t k = 0; k < DPL; k++) pv[h][k] = 0.0f;
            for (uint32_t rr = 0; rr < cnt; rr++) {
                const float4 pa = *reinterpret_cast<const float4*>(wp + rr * 8);
                const float4 pb = *reinterpret_cast<const float4*>(wp + rr * 8 + 4);
                const float pr[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
                float vv[DPL];
                if constexpr (DPL == 2) {
                    const float2 t = *reinterpret_cast<const float2*>(wv + rr * RW + 2 * lane);
                    vv[0] = t.x;
                    vv[1] = t.y;
                } else {
                    const float4 t = *reinterpret_cast<const float4*>(wv + rr * RW + 4 * lane);
                    vv[0] = t.x;
                    vv[1] = t.y;
                    vv[2] = t.z;
                    vv[3] = t.w;
                }
#pragma unroll
                for (uint32_t h = 0; h < 8; h++)
                    if (h < G)
#pragma unroll
                        for (uint32_t k = 0; k < DPL; k++) pv[h][k] = __fmaf_rn(pr[h], vv[k], pv[h][k]);
            }
#pragma unroll
            for (uint32_t h = 0; h < 8; h++) {
                if (h < G) {
                    const float f = wf[h];
#pragma unroll
                    for (uint32_t k = 0; k < DPL; k++) acc[h][k] = __fadd_rn(__fmul_rn(acc[h][k], f), pv[h][k]);
                }
            }
            __syncwarp();  // the block's buffers and probabilities are reused
        }
        cp_wait0();
        sync256();
        // merge: warp w's maxima, sums and outputs, then per head the weights
        // exp(m_w - M) and the sums in warp order
        float* mm = kb;               // [8 warps][8 heads]
        float* ll = mm + 64;          // [8][8]
        float* wt = ll + 64;          // [8][8] weights
        float* ao = wt + 64;          // [8 warps][8 heads][HD]
        if (r == 0) {
            mm[warp * 8 + h0] = rm0;
            mm[warp * 8 + h1] = rm1;
            ll[warp * 8 + h0] = rl0;
            ll[warp * 8 + h1] = rl1;
        }
#pragma unroll
        for (uint32_t h = 0; h < 8; h++)
            if (h < G)
#pragma unroll
                for (uint32_t k = 0; k < DPL; k++) ao[(warp * 8 + h) * HD + DPL * lane + k] = acc[h][k];
        sync256();
        if (tid < G) {
            float M = -FLT_MAX;
            for (uint32_t w = 0; w < 8; w++) M = fmaxf(M, mm[w * 8 + tid]);
            float l = 0.0f;
            for (uint32_t w = 0; w < 8; w++) {
                const float m_w = mm[w * 8 + tid];
                const float x = m_w == -FLT_MAX ? 0.0f : __expf(__fsub_rn(m_w, M));
                wt[w * 8 + tid] = x;
                l = __fadd_rn(l, __fmul_rn(x, ll[w * 8 + tid]));
            }
            hs_m[tid] = M;
            hs_l[tid] = l;
        }
        sync256();
#pragma unroll
        for (uint32_t j = 0; j < HPT; j++) {
            const uint32_t h = hs0 + j * HSETS;
            if (h < G) {
                float v = 0.0f;
                for (uint32_t w = 0; w < 8; w++) v = __fadd_rn(v, __fmul_rn(wt[w * 8 + h], ao[(w * 8 + h) * HD + dd]));
                o[j] = v;
            }
        }
      }
    } else {
    const uint32_t nch = (p1 - p0 + kCh - 1) / kCh;
    auto issue = [&](uint32_t c) {
        if (c < nch) {
            const uint32_t c0 = p0 + c * kCh, cnt = p1 - c0 < kCh ? p1 - c0 : kCh;
            float* kd = kb + (c % NBUF) * kCh * RSK;
            float* vd = vb + (c % NBUF) * kCh * RSV;
            for (uint32_t idx = tid; idx < cnt * (HD / 4); idx += kThreads) {
                const uint32_t r = idx / (HD / 4), c4 = idx % (HD / 4);
                if (c0 + r == pos && append) {
                    *reinterpret_cast<float4*>(kd + r * RSK + 4 * c4) = *reinterpret_cast<const float4*>(kn + 4 * c4);
                    *reinterpret_cast<float4*>(vd + r * RSV + 4 * c4) = *reinterpret_cast<const float4*>(vn + 4 * c4);
                } else if (c >= npre) {
                    cp_async16(kd + r * RSK + 4 * c4, kv + row_off(c0 + r, 0) + 4 * c4);
                    cp_async16(vd + r * RSV + 4 * c4, kv + row_off(c0 + r, 1) + 4 * c4);
                }
            }
            // TC: V rows past the split's end are zero (the tiles span the
            // whole chunk; their probabilities are 0, and 0 times a stale
            // non-finite value would not be)
            if constexpr (TC)
                for (uint32_t idx = cnt * (HD / 4) + tid; idx < kCh * (HD / 4); idx += kThreads)
                    *reinterpret_cast<float4*>(vd + (idx / (HD / 4)) * RSV + 4 * (idx % (HD / 4))) =
                        make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        if (c >= npre) cp_commit();  // a prefetched chunk's group is committed already
    };
    // TC: both products of a chunk on the tensor cores (mma.sync m16n8k8,
    // tf32 operands split hi + lo so that lo*hi + hi*lo + hi*hi keeps about
    // 22 significant bits: the split-precision method of Ootomo & Yokota,
    // "Recovering single precision accuracy from Tensor Cores", 2022).
    //   scores^T [64 positions][8 heads] = K [64][HD] . q^T [HD][8]: warp w
    //     takes positions 16 (w % 4) .. +15 and half w / 4 of the dimensions;
    //     the two halves are added in the softmax;
    //   out^T [HD][8 heads] += V^T [HD][64] . P^T [64][8]: warp w takes
    //     dimensions 16 (w % MTV) .. +15 and positions part w / MTV of the
    //     chunk; the parts' accumulators are added after the last chunk.
    // Otherwise fp32 FMA chains on the CUDA cores (fewer registers: the
    // persistent token kernel inlines this item among its GEMV phases).
    constexpr uint32_t KSQ = HD / 16;                 // k-steps of 8 dimensions per half
    constexpr uint32_t MTV = HD / 16, WPV = 8 / MTV;  // m-tiles of out^T, warps per m-tile
    constexpr uint32_t KSV = 8 / WPV;                 // k-steps of 8 positions per warp
    const uint32_t g = lane >> 2, t4 = lane & 3;
    const uint32_t mq = warp & 3, kq = warp >> 2, mv = warp % MTV, kvp = warp / MTV;
    const uint4* qf = qfrag + kq * KSQ * 32 + lane;
    if constexpr (TC) {
        // q^T operand fragments, split once per item (read by the first
        // iteration after its barrier)
        for (uint32_t e = tid; e < 2 * KSQ * 32; e += kThreads) {
            const uint32_t ln = e % 32, gg = ln >> 2, d = (e / 32) * 8 + (ln & 3);
            uint4 f;
            tf32_split(gg < G ? qs[gg * HD + d] : 0.0f, f.x, f.z);
            tf32_split(gg < G ? qs[gg * HD + d + 4] : 0.0f, f.y, f.w);
            qfrag[e] = f;
        }
    }
    float oa[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // TC: out^T (16 mv + g, 2 t4), (.., 2 t4 + 1), (+8, ..), (+8, ..)
    // chunks 0 .. NBUF-2 in flight before the loop; each iteration issues
    // chunk c + NBUF - 1 (an empty group past the end) and waits for chunk c
#pragma unroll
    for (uint32_t c = 0; c + 1 < NBUF; c++) issue(c);
    for (uint32_t c = 0; c < nch; c++) {
        issue(c + NBUF - 1);
        cp_wait<NBUF - 1>();
        sync256();
        if (c == 0) at(3);
        const uint32_t c0 = p0 + c * kCh, cnt = p1 - c0 < kCh ? p1 - c0 : kCh;
        const float* kc = kb + (c % NBUF) * kCh * RSK;
        const float* vc = vb + (c % NBUF) * kCh * RSV;
        if constexpr (TC) {
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            const float* kr = kc + (16 * mq + g) * RSK + kq * (HD / 2) + t4;
#pragma unroll
            for (uint32_t j = 0; j < KSQ; j++) {
                uint32_t ah[4], al[4];
                tf32_split(kr[8 * j], ah[0], al[0]);
                tf32_split(kr[8 * RSK + 8 * j], ah[1], al[1]);
                tf32_split(kr[8 * j + 4], ah[2], al[2]);
                tf32_split(kr[8 * RSK + 8 * j + 4], ah[3], al[3]);
                const uint4 f = qf[j * 32];
                const uint32_t bh[2] = {f.x, f.y}, bl[2] = {f.z, f.w};
                mma_tf32(acc, al, bh);
                mma_tf32(acc, ah, bl);
                mma_tf32(acc, ah, bh);
            }
            float* sk = sp + kq * 8 * SPS;
            const uint32_t r = 16 * mq + g;
            sk[(2 * t4) * SPS + r] = acc[0];
            sk[(2 * t4 + 1) * SPS + r] = acc[1];
            sk[(2 * t4) * SPS + r + 8] = acc[2];
            sk[(2 * t4 + 1) * SPS + r + 8] = acc[3];
        } else {
            // thread t takes position t % 64 and heads t/64, t/64 + 4 (each
            // K row read once for both heads); scaled scores, masked past cnt
            constexpr uint32_t HSETS_S = kThreads / kCh, HPT_S = (8 + HSETS_S - 1) / HSETS_S;
            const uint32_t r = tid % kCh, h0 = tid / kCh;
            float sc[HPT_S][4];
#pragma unroll
            for (uint32_t j = 0; j < HPT_S; j++) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
            if (r < cnt) {
                const float4* k4 = reinterpret_cast<const float4*>(kc + r * RSK);
#pragma unroll
                for (uint32_t d4 = 0; d4 < HD / 4; d4++) {
                    const float4 kk = k4[d4];
#pragma unroll
                    for (uint32_t j = 0; j < HPT_S; j++) {
                        const uint32_t h = h0 + j * HSETS_S;
                        if (h < G) {
                            const float4 qq = reinterpret_cast<const float4*>(qs + h * HD)[d4];
                            sc[j][0] = __fmaf_rn(qq.x, kk.x, sc[j][0]);
                            sc[j][1] = __fmaf_rn(qq.y, kk.y, sc[j][1]);
                            sc[j][2] = __fmaf_rn(qq.z, kk.z, sc[j][2]);
                            sc[j][3] = __fmaf_rn(qq.w, kk.w, sc[j][3]);
                        }
                    }
                }
            }
#pragma unroll
            for (uint32_t j = 0; j < HPT_S; j++) {
                const uint32_t h = h0 + j * HSETS_S;
                if (h < G)
                    sp[h * SPS + r] = r < cnt ? __fmul_rn(__fadd_rn(__fadd_rn(sc[j][0], sc[j][1]),
                                                                    __fadd_rn(sc[j][2], sc[j][3])),
                                                          scale)
                                              : -FLT_MAX;
            }
        }
        sync256();
        if (c == 0) at(4);
        // online softmax: warp h owns head h; probabilities in the first
        // score half
        if (warp < G) {
            float* sh = sp + warp * SPS;
            float a0, a1;
            if constexpr (TC) {
                const float* sh2 = sh + 8 * SPS;
                a0 = lane < cnt ? __fmul_rn(__fadd_rn(sh[lane], sh2[lane]), scale) : -FLT_MAX;
                a1 = lane + 32 < cnt ? __fmul_rn(__fadd_rn(sh[lane + 32], sh2[lane + 32]), scale) : -FLT_MAX;
            } else {
                a0 = sh[lane];
                a1 = sh[lane + 32];
            }
            float mx = fmaxf(a0, a1);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_old = hs_m[warp], m_new = fmaxf(m_old, mx);
            const float e0 = lane < cnt ? __expf(__fsub_rn(a0, m_new)) : 0.0f;
            const float e1 = lane + 32 < cnt ? __expf(__fsub_rn(a1, m_new)) : 0.0f;
            sh[lane] = e0;
            sh[lane + 32] = e1;
            float sum = __fadd_rn(e0, e1);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, off));
            if (lane == 0) {
                const float f = m_old == -FLT_MAX ? 0.0f : __expf(__fsub_rn(m_old, m_new));
                hs_f[warp] = f;
                hs_m[warp] = m_new;
                hs_l[warp] = __fadd_rn(__fmul_rn(hs_l[warp], f), sum);
            }
        } else if (TC && lane == 0) {
            hs_f[warp] = 1.0f;  // heads past the group (their columns are discarded)
        }
        sync256();
        if (c == 0) at(5);
        if constexpr (TC) {
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            const float* vr = vc + (kvp * KSV * 8 + t4) * RSV + 16 * mv + g;
            const float* pr = sp + g * SPS + kvp * KSV * 8 + t4;
#pragma unroll
            for (uint32_t j = 0; j < KSV; j++) {
                uint32_t ah[4], al[4], bh[2], bl[2];
                tf32_split(vr[8 * j * RSV], ah[0], al[0]);
                tf32_split(vr[8 * j * RSV + 8], ah[1], al[1]);
                tf32_split(vr[(8 * j + 4) * RSV], ah[2], al[2]);
                tf32_split(vr[(8 * j + 4) * RSV + 8], ah[3], al[3]);
                tf32_split(pr[8 * j], bh[0], bl[0]);
                tf32_split(pr[8 * j + 4], bh[1], bl[1]);
                mma_tf32(acc, al, bh);
                mma_tf32(acc, ah, bl);
                mma_tf32(acc, ah, bh);
            }
            const float f0 = hs_f[2 * t4], f1 = hs_f[2 * t4 + 1];
            oa[0] = __fadd_rn(__fmul_rn(oa[0], f0), acc[0]);
            oa[1] = __fadd_rn(__fmul_rn(oa[1], f1), acc[1]);
            oa[2] = __fadd_rn(__fmul_rn(oa[2], f0), acc[2]);
            oa[3] = __fadd_rn(__fmul_rn(oa[3], f1), acc[3]);
        } else {
            // thread t owns dimension t % HD of heads t/HD, t/HD + HSETS, ...:
            // one chain per head over the positions in order, each V element
            // read once for all of them
            float pv[HPT];
#pragma unroll
            for (uint32_t j = 0; j < HPT; j++) pv[j] = 0.0f;
            // four positions at a time: their probabilities as one 16-byte read
            uint32_t r = 0;
            for (; r + 4 <= cnt; r += 4) {
                const float v0 = vc[r * RSV + dd], v1 = vc[(r + 1) * RSV + dd], v2 = vc[(r + 2) * RSV + dd],
                            v3 = vc[(r + 3) * RSV + dd];
#pragma unroll
                for (uint32_t j = 0; j < HPT; j++) {
                    const uint32_t h = hs0 + j * HSETS;
                    if (h < G) {
                        const float4 p4 = *reinterpret_cast<const float4*>(sp + h * SPS + r);
                        pv[j] = __fmaf_rn(p4.x, v0, pv[j]);
                        pv[j] = __fmaf_rn(p4.y, v1, pv[j]);
                        pv[j] = __fmaf_rn(p4.z, v2, pv[j]);
                        pv[j] = __fmaf_rn(p4.w, v3, pv[j]);
                    }
                }
            }
            for (; r < cnt; r++) {
                const float vv = vc[r * RSV + dd];
#pragma unroll
                for (uint32_t j = 0; j < HPT; j++) {
                    const uint32_t h = hs0 + j * HSETS;
                    if (h < G) pv[j] = __fmaf_rn(sp[h * SPS + r], vv, pv[j]);
                }
            }
#pragma unroll
            for (uint32_t j = 0; j < HPT; j++) {
                const uint32_t h = hs0 + j * HSETS;
                if (h < G) o[j] = __fadd_rn(__fmul_rn(o[j], hs_f[h]), pv[j]);
            }
        }
        sync256();
    }
    cp_wait0();
    if constexpr (TC) {
        // out^T parts through shared memory (the K buffers are free): [WPV][8][HD]
        float* ot = kb + kvp * 8 * HD;
        const uint32_t d = 16 * mv + g;
        ot[(2 * t4) * HD + d] = oa[0];
        ot[(2 * t4 + 1) * HD + d] = oa[1];
        ot[(2 * t4) * HD + d + 8] = oa[2];
        ot[(2 * t4 + 1) * HD + d + 8] = oa[3];
        sync256();
#pragma unroll
        for (uint32_t j = 0; j < HPT; j++) {
            const uint32_t h = hs0 + j * HSETS;
            if (h < 8) {
                o[j] = kb[h * HD + dd];
#pragma unroll
                for (uint32_t q = 1; q < WPV; q++) o[j] = __fadd_rn(o[j], kb[(q * 8 + h) * HD + dd]);
            }
        }
    }
    }  // chunked attend
    at(6);
    mark_dirty();

    auto store = [&](size_t at, float v) {
        if (tio) {
            st_tagged(tio->out + at, v, tio->tag);
        } else if (a.out_f32) {
            a.out_f32[at] = v;
        } else {
            uint16_t hi, lo;
            split_f16(v, &hi, &lo);
            a.out_hi[at] = hi;
            a.out_lo[at] = lo;
        }
    };
    if (S == 1) {
#pragma unroll
        for (uint32_t j = 0; j < HPT; j++) {
            const uint32_t h = hs0 + j * HSETS;
            if (h < G) store((size_t)slot * a.out_stride + (size_t)(kvh * Gf + hlo + h) * HD + dd, __fdiv_rn(o[j], hs_l[h]));
        }
        return;
    }
    // Several splits: publish (unnormalised output, max, sum); the last item
    // to arrive combines all splits in split order.
    const uint32_t rec = attn_record(Gf, HD);
    const size_t rec0 = (size_t)(slot * a.nkv + kvh) * a.max_splits * rec + (size_t)s * rec;
    if (tio && reader_combines) {
        // tagged records: the readers poll them
#pragma unroll
        for (uint32_t j = 0; j < HPT; j++) {
            const uint32_t h = hs0 + j * HSETS;
            if (h < G) st_tagged(tio->rec + rec0 + (hlo + h) * HD + dd, o[j], tio->tag);
        }
        if (tid < G) {
            st_tagged(tio->rec + rec0 + Gf * HD + hlo + tid, hs_m[tid], tio->tag);
            st_tagged(tio->rec + rec0 + Gf * HD + Gf + hlo + tid, hs_l[tid], tio->tag);
        }
        at(7);
        return;
    }
    float* part = a.partials + rec0 - (size_t)s * rec;
#pragma unroll
    for (uint32_t j = 0; j < HPT; j++) {
        const uint32_t h = hs0 + j * HSETS;
        if (h < G) part[(size_t)s * rec + (hlo + h) * HD + dd] = o[j];
    }
    if (tid < G) {
        part[(size_t)s * rec + Gf * HD + hlo + tid] = hs_m[tid];
        part[(size_t)s * rec + Gf * HD + Gf + hlo + tid] = hs_l[tid];
    }
    if (reader_combines) {
        at(7);
        return;
    }
    __threadfence();
    sync256();
    uint32_t* counter = a.counters + slot * a.nkv + kvh;
    if (tid == 0) *flag = atomicAdd(counter, 1u) == S * hsplit - 1 ? 1u : 0u;
    sync256();
    const bool last = *flag != 0;
    sync256();  // the flag word is rewritten by the next item
    if (!last) return;
    __threadfence();
    // Up to 8 splits the per-element combine (its loads in flight together,
    // no block barrier) is faster: at 4 splits 3.8 against 8.0 µs for the
    // staged one; the staged one wins with many splits (batch 1, 4k-32k
    // positions). The same operations in the same split order: the same bits.
    if (a.unstaged_combine || S <= 8) {
        for (uint32_t idx = tid; idx < Gf * HD; idx += kThreads)
            store((size_t)slot * a.out_stride + (size_t)kvh * Gf * HD + idx, combine<true>(part, S, Gf, HD, idx));
    } else {
        combine_staged(part, S, Gf, HD, sm, [&](uint32_t idx, float v) {
            store((size_t)slot * a.out_stride + (size_t)kvh * Gf * HD + idx, v);
        });
    }
    if (tid == 0) *counter = 0;
}

}  // namespace attn
}  // namespace hs
