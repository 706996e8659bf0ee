// Query-block causal GQA attention for prompt prefill on the tensor-core
// path (hs_prefill): model.rs:259-305 for a pass of consecutive prompt
// tokens of one sequence, whose k, v rows the append launch has already
// written to the KV region.
//
// The per-token split-KV item (attn_split.cu) streams a token's whole prefix
// of K/V for every token; here one CTA takes kRows = 64 query rows (the G
// heads of one KV head for floor(64 / G) consecutive tokens) and one
// segment of `seg` cached positions, so every K/V chunk it loads serves 64
// rows. Segments are fixed in absolute positions ([s seg, (s+1) seg), seg
// from max_ctx only), chunks of 64 positions run from the segment's start,
// and each row's products, running maximum, sum and output are its own, so
// a token's bits depend on its position and the KV contents only: never on
// which tokens share its block, on the pass it is in or on the batch. A
// token with one segment (pos < seg) is written normalised by the attend
// kernel; otherwise each segment writes (unnormalised output, max, sum) and
// the combine kernel merges the token's pos / seg + 1 segments in segment
// order (attn::combine_staged, the split items' combine).
//
// Products: fp32 FMA chains on the CUDA cores, register-tiled. Scores: a
// thread holds a 4 (rows) x 4 (positions) tile, q and K read from shared
// memory as float4 along head_dim (q broadcast in the warp, K rows
// swizzled so that a warp's 16 rows hit distinct banks). Online softmax per
// row over the chunk (the 16 lanes holding a row reduce by shuffles).
// P.V: the same thread holds the same 4 rows x head_dim/16 dimensions; P is
// stored transposed [position][row] (swizzled) and read as float4 per
// position, V rows as float4 per 16 lanes.
//
// Pipeline per chunk: K(c) and V(c) are separate commit groups; K(c+1)
// loads while the softmax and P.V of chunk c run, V(c+1) while the scores of
// chunk c+1 run. Shared memory (head_dim 128): q 32 KB + K 32 KB + V 32 KB +
// P 16 KB = 112 KB, two CTAs per SM.
#include <cfloat>

#include "attn_body.cuh"
#include "common.h"
#include "kernels.h"

namespace hs {
namespace {

constexpr uint32_t kRows = 64;  // query rows per CTA
constexpr uint32_t kPCh = 64;   // positions per chunk
constexpr uint32_t kPThreads = 256;

template <int HD>
struct PfGeom {
    static constexpr uint32_t Q = kRows * HD, K = kPCh * HD, V = kPCh * HD, P = kPCh * kRows;
    static constexpr size_t bytes = (size_t)(Q + K + V + P) * sizeof(float);
};

// float4 slot of dimension group k4 in row r of the q and K buffers
__device__ __forceinline__ uint32_t swz(uint32_t k4, uint32_t r) { return k4 ^ (r & 7u); }

__device__ __forceinline__ void store_out(const SplitAttnArgs& a, size_t at, float v) {
    if (a.out_f32) {
        a.out_f32[at] = v;
    } else {
        uint16_t hi, lo;
        attn::split_f16(v, &hi, &lo);
        a.out_hi[at] = hi;
        a.out_lo[at] = lo;
    }
}

template <int HD>
__global__ void __launch_bounds__(kPThreads, 2)
    k_prefill_attend(const SplitAttnArgs a, uint32_t slots, uint32_t qb_tokens, uint32_t seg) {
    using Geo = PfGeom<HD>;
    constexpr uint32_t NK4 = HD / 4, HALF = HD / 2, DJ = HD / 64;  // float4 groups of V per lane
    extern __shared__ __align__(16) float sm[];
    float* Qs = sm;
    float* Ks = Qs + Geo::Q;
    float* Vs = Ks + Geo::K;
    float* Ps = Vs + Geo::V;
    __shared__ uint32_t s_lim[kRows];  // per token of the block: pos + 1, or 0 (no such token)
    __shared__ uint32_t s_max;
    const uint32_t s = blockIdx.x, qb = blockIdx.y, kvh = blockIdx.z, tid = threadIdx.x;
    const uint32_t Gf = a.nh / a.nkv, t0 = qb * qb_tokens;
    const KTrace tr(a.trace, a.trace_slot);
    tr.enter();
    pdl_launch_dependents();
    if (tid < kRows) {  // control blocks are host-written before the launch
        uint32_t lim = 0;
        if (tid < qb_tokens && t0 + tid < slots) {
            const DevCtl* c = a.ctl + t0 + tid;
            const uint32_t pos = attn::ldv(&c->pos);
            if (attn::ldv(&c->active) != 0 && pos < a.max_ctx) lim = pos + 1;
        }
        s_lim[tid] = lim;
    }
    __syncthreads();
    if (tid < 32) {
        uint32_t m = s_lim[tid] > s_lim[tid + 32] ? s_lim[tid] : s_lim[tid + 32];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const uint32_t o = __shfl_xor_sync(0xffffffffu, m, off);
            m = o > m ? o : m;
        }
        if (tid == 0) s_max = m;
    }
    __syncthreads();
    const uint32_t lim_max = s_max, p_begin = s * seg;
    if (lim_max <= p_begin) {  // no token of the block reaches this segment
        tr.exit();
        return;
    }
    const uint32_t p_end = p_begin + seg < lim_max ? p_begin + seg : lim_max;
    const uint32_t nch = (p_end - p_begin + kPCh - 1) / kPCh;
    const float* kv = a.kv[t0];
    const uint32_t layer = a.layer;
    auto load_k = [&](uint32_t c) {
        if (c < nch) {
            const uint32_t c0 = p_begin + c * kPCh, cnt = p_end - c0 < kPCh ? p_end - c0 : kPCh;
            for (uint32_t i = tid; i < cnt * NK4; i += kPThreads) {
                const uint32_t rr = i / NK4, k4 = i % NK4;
                cp_async16(Ks + rr * HD + 4 * swz(k4, rr), kv + attn::kv_row_off(a, layer, kvh, HD, c0 + rr, 0) + 4 * k4);
            }
        }
        attn::cp_commit();
    };
    auto load_v = [&](uint32_t c) {
        if (c < nch) {
            const uint32_t c0 = p_begin + c * kPCh, cnt = p_end - c0 < kPCh ? p_end - c0 : kPCh;
            for (uint32_t i = tid; i < cnt * NK4; i += kPThreads) {
                const uint32_t rr = i / NK4, k4 = i % NK4;
                cp_async16(Vs + rr * HD + 4 * k4, kv + attn::kv_row_off(a, layer, kvh, HD, c0 + rr, 1) + 4 * k4);
            }
            // rows past the chunk's end: zero (their probabilities are 0,
            // and 0 times a stale non-finite value would not be)
            for (uint32_t i = cnt * NK4 + tid; i < kPCh * NK4; i += kPThreads)
                reinterpret_cast<float4*>(Vs)[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        attn::cp_commit();
    };

    // The QKV product and the appended rows come from the previous launches.
    pdl_wait();
    load_k(0);
    load_v(0);

    // q rows of the block: split-K partials in split order, then the bias,
    // then RoPE at the token's position (model.rs:365-373); zero for rows
    // without a token. Job = (row, dimension group k4 < HD/8): the float4
    // pair (k4, k4 + HD/8) that RoPE rotates together.
    for (uint32_t j = tid; j < kRows * (HD / 8); j += kPThreads) {
        const uint32_t r = j / (HD / 8), k4 = j % (HD / 8), t = r / Gf, h = r % Gf;
        float4 x0 = make_float4(0.0f, 0.0f, 0.0f, 0.0f), x1 = x0;
        const uint32_t lim = r < qb_tokens * Gf ? s_lim[t] : 0u;
        if (lim) {
            const uint32_t pos = lim - 1, row = (kvh * Gf + h) * HD + 4 * k4;
            const float* src = a.qkv + (size_t)(t0 + t) * a.qkv_rows + row;
            for (uint32_t q = 0; q < a.n_part; q++) {
                x0 = attn::f4add(x0, __ldcg(reinterpret_cast<const float4*>(src + q * a.part_stride)));
                x1 = attn::f4add(x1, __ldcg(reinterpret_cast<const float4*>(src + q * a.part_stride + HALF)));
            }
            if (a.bias) {
                x0 = attn::f4add(x0, *reinterpret_cast<const float4*>(a.bias + row));
                x1 = attn::f4add(x1, *reinterpret_cast<const float4*>(a.bias + row + HALF));
            }
            const float4 c = *reinterpret_cast<const float4*>(a.rope_cos + (size_t)pos * HALF + 4 * k4);
            const float4 sn = *reinterpret_cast<const float4*>(a.rope_sin + (size_t)pos * HALF + 4 * k4);
            auto rot = [](float& u, float& w, float cc, float ss) {
                const float u0 = u, w0 = w;
                u = __fsub_rn(__fmul_rn(u0, cc), __fmul_rn(w0, ss));
                w = __fadd_rn(__fmul_rn(u0, ss), __fmul_rn(w0, cc));
            };
            rot(x0.x, x1.x, c.x, sn.x);
            rot(x0.y, x1.y, c.y, sn.y);
            rot(x0.z, x1.z, c.z, sn.z);
            rot(x0.w, x1.w, c.w, sn.w);
        }
        reinterpret_cast<float4*>(Qs + r * HD)[swz(k4, r)] = x0;
        reinterpret_cast<float4*>(Qs + r * HD)[swz(k4 + HD / 8, r)] = x1;
    }

    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
    const uint32_t warp = tid >> 5, lane = tid & 31, rl = lane >> 4, cl = lane & 15;
    const uint32_t r0 = warp * 8 + rl * 4, rg = r0 / 4;  // this thread's 4 rows, their float4 slot in P
    uint32_t rlim[4];  // positions < rlim are this row's (0: no token)
#pragma unroll
    for (uint32_t ii = 0; ii < 4; ii++) {
        const uint32_t r = r0 + ii;
        rlim[ii] = r < qb_tokens * Gf ? s_lim[r / Gf] : 0u;
    }
    float m[4], l[4], acc[4][4 * DJ];
#pragma unroll
    for (uint32_t ii = 0; ii < 4; ii++) {
        m[ii] = -FLT_MAX;
        l[ii] = 0.0f;
#pragma unroll
        for (uint32_t d = 0; d < 4 * DJ; d++) acc[ii][d] = 0.0f;
    }

    for (uint32_t c = 0; c < nch; c++) {
        const uint32_t c0 = p_begin + c * kPCh, cnt = p_end - c0 < kPCh ? p_end - c0 : kPCh;
        attn::cp_wait<1>();  // K(c) (V(c) may still be in flight)
        __syncthreads();
        if (c == 0) tr.mark(1);
        float sc[4][4];
#pragma unroll
        for (uint32_t ii = 0; ii < 4; ii++)
#pragma unroll
            for (uint32_t i = 0; i < 4; i++) sc[ii][i] = 0.0f;
#pragma unroll 4
        for (uint32_t k4 = 0; k4 < NK4; k4++) {
            float4 q[4], k[4];
#pragma unroll
            for (uint32_t ii = 0; ii < 4; ii++) q[ii] = reinterpret_cast<const float4*>(Qs + (r0 + ii) * HD)[swz(k4, r0 + ii)];
#pragma unroll
            for (uint32_t i = 0; i < 4; i++) k[i] = reinterpret_cast<const float4*>(Ks + (cl + 16 * i) * HD)[swz(k4, cl)];
#pragma unroll
            for (uint32_t ii = 0; ii < 4; ii++)
#pragma unroll
                for (uint32_t i = 0; i < 4; i++) {
                    float v = sc[ii][i];
                    v = __fmaf_rn(q[ii].x, k[i].x, v);
                    v = __fmaf_rn(q[ii].y, k[i].y, v);
                    v = __fmaf_rn(q[ii].z, k[i].z, v);
                    v = __fmaf_rn(q[ii].w, k[i].w, v);
                    sc[ii][i] = v;
                }
        }
        __syncthreads();  // K(c) consumed
        load_k(c + 1);
        // online softmax of the chunk per row; masked: past the chunk, past
        // the row's position, rows without a token
        float f[4];
#pragma unroll
        for (uint32_t ii = 0; ii < 4; ii++) {
            float mx = -FLT_MAX;
#pragma unroll
            for (uint32_t i = 0; i < 4; i++) {
                const uint32_t rr = cl + 16 * i;
                const bool ok = rr < cnt && c0 + rr < rlim[ii];
                sc[ii][i] = ok ? __fmul_rn(sc[ii][i], scale) : -FLT_MAX;
                mx = fmaxf(mx, sc[ii][i]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            // nothing of this row in the chunk: an exact no-op (f = 1, all
            // probabilities 0, m and l kept). Selects, not a branch: both
            // half-warps (different rows) take every shuffle.
            const bool none = mx == -FLT_MAX;
            const float mn = none ? m[ii] : fmaxf(m[ii], mx);
            float sum = 0.0f;
#pragma unroll
            for (uint32_t i = 0; i < 4; i++) {
                const float e = sc[ii][i] == -FLT_MAX ? 0.0f : __expf(__fsub_rn(sc[ii][i], mn));
                sc[ii][i] = e;
                sum = __fadd_rn(sum, e);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, off));
            f[ii] = none ? 1.0f : (m[ii] == -FLT_MAX ? 0.0f : __expf(__fsub_rn(m[ii], mn)));
            l[ii] = none ? l[ii] : __fadd_rn(__fmul_rn(l[ii], f[ii]), sum);
            m[ii] = mn;
        }
#pragma unroll
        for (uint32_t i = 0; i < 4; i++) {
            const uint32_t col = cl + 16 * i;
            reinterpret_cast<float4*>(Ps + col * kRows)[rg ^ (col & 15u)] =
                make_float4(sc[0][i], sc[1][i], sc[2][i], sc[3][i]);
        }
        attn::cp_wait<1>();  // V(c) (K(c+1) may still be in flight)
        __syncthreads();
#pragma unroll
        for (uint32_t ii = 0; ii < 4; ii++)
#pragma unroll
            for (uint32_t d = 0; d < 4 * DJ; d++) acc[ii][d] = __fmul_rn(acc[ii][d], f[ii]);
#pragma unroll 4
        for (uint32_t j = 0; j < cnt; j++) {
            const float4 p = reinterpret_cast<const float4*>(Ps + j * kRows)[rg ^ (j & 15u)];
            const float pr[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
            for (uint32_t dj = 0; dj < DJ; dj++) {
                const float4 v = reinterpret_cast<const float4*>(Vs + j * HD)[cl + 16 * dj];
#pragma unroll
                for (uint32_t ii = 0; ii < 4; ii++) {
                    acc[ii][4 * dj + 0] = __fmaf_rn(pr[ii], v.x, acc[ii][4 * dj + 0]);
                    acc[ii][4 * dj + 1] = __fmaf_rn(pr[ii], v.y, acc[ii][4 * dj + 1]);
                    acc[ii][4 * dj + 2] = __fmaf_rn(pr[ii], v.z, acc[ii][4 * dj + 2]);
                    acc[ii][4 * dj + 3] = __fmaf_rn(pr[ii], v.w, acc[ii][4 * dj + 3]);
                }
            }
        }
        __syncthreads();  // V(c) and P consumed
        load_v(c + 1);
    }
    attn::cp_wait0();
    tr.mark(2);

    // rows of a token with one segment: the normalised output; otherwise this
    // segment's record (rows whose token does not reach it write nothing)
    const uint32_t rec = attn_record(Gf, HD);
#pragma unroll
    for (uint32_t ii = 0; ii < 4; ii++) {
        const uint32_t r = r0 + ii;
        if (rlim[ii] <= p_begin) continue;
        const uint32_t slot = t0 + r / Gf, h = r % Gf;
        if (rlim[ii] <= seg) {
            const size_t o = (size_t)slot * a.out_stride + (size_t)(kvh * Gf + h) * HD;
#pragma unroll
            for (uint32_t dj = 0; dj < DJ; dj++)
#pragma unroll
                for (uint32_t e = 0; e < 4; e++)
                    store_out(a, o + 4 * (cl + 16 * dj) + e, __fdiv_rn(acc[ii][4 * dj + e], l[ii]));
        } else {
            float* part = a.partials + ((size_t)(slot * a.nkv + kvh) * a.max_splits + s) * rec;
#pragma unroll
            for (uint32_t dj = 0; dj < DJ; dj++)
                reinterpret_cast<float4*>(part + h * HD)[cl + 16 * dj] =
                    make_float4(acc[ii][4 * dj], acc[ii][4 * dj + 1], acc[ii][4 * dj + 2], acc[ii][4 * dj + 3]);
            if (cl == 0) {
                part[Gf * HD + h] = m[ii];
                part[Gf * HD + Gf + h] = l[ii];
            }
        }
    }
    tr.exit();
}

// Merge of a token's segments (pos / seg + 1 of them, when more than one),
// one CTA per (KV head, token).
template <int HD>
__global__ void __launch_bounds__(kPThreads) k_prefill_combine(const SplitAttnArgs a, uint32_t seg) {
    extern __shared__ __align__(16) float sm[];
    const uint32_t kvh = blockIdx.x, slot = blockIdx.y;
    const KTrace tr(a.trace, a.trace_slot);
    tr.enter();
    const DevCtl* c = a.ctl + slot;
    const bool active = attn::ldv(&c->active) != 0;
    const uint32_t pos = attn::ldv(&c->pos);
    pdl_launch_dependents();
    pdl_wait();
    if (active && pos < a.max_ctx && pos >= seg) {
        const uint32_t S = pos / seg + 1, Gf = a.nh / a.nkv;
        const float* part = a.partials + (size_t)(slot * a.nkv + kvh) * a.max_splits * attn_record(Gf, HD);
        const size_t o = (size_t)slot * a.out_stride + (size_t)kvh * Gf * HD;
        attn::combine_staged(part, S, Gf, HD, sm, [&](uint32_t idx, float v) { store_out(a, o + idx, v); });
    }
    tr.exit();
}

// ---------------------------------------------------------------- tensor cores
// The same query blocks, segments and records with both products on the
// tensor cores (mma.sync m16n8k16, f16 operands, f32 accumulate), every
// operand carried as an f16 pair hi = f16(x), lo = f16(x - hi) and every
// product as lo*hi + hi*lo + hi*hi into the same f32 accumulator (about 22
// significant bits of each operand; the f16 range, as the tensor-core GEMMs'
// activation pairs). One CTA: kTcRows = 128 query rows (floor(128 / G)
// tokens), 8 warps of 16 rows; a warp computes its rows' scores for the
// whole 64-position chunk (8 n-tiles), their online softmax, and P.V for all
// head_dim columns, with the probabilities kept in registers (the score
// accumulator layout of two n-tiles is the A-operand layout of one 16-wide
// k-step). Each row's arithmetic is its own, so a token's bits depend on its
// position and the KV contents only.
//
// Per chunk: the f32 K and V rows land by cp.async in staging buffers; all
// threads convert them once into f16 hi/lo K [position][dim] and V^T
// [dim][position] (rows padded by 8 halves: the fragment loads of a warp hit
// 32 distinct banks); the next chunk's rows then load while the warps run
// the products. Shared memory at head_dim 128: q pairs 68 KB + K pairs 34 KB
// + V pairs 36 KB + staging 66 KB = 204 KB, one CTA per SM.
constexpr uint32_t kTcRows = 128;

template <int HD>
struct PfTcGeom {
    static constexpr uint32_t QS = HD + 8, KS = HD + 8, VS = kPCh + 8, SS = HD + 4;  // row strides (halves / floats)
    static constexpr uint32_t Q = kTcRows * QS, K = kPCh * KS, V = HD * VS;        // halves per hi or lo buffer
    static constexpr uint32_t STG = kPCh * SS;                                      // floats per staging buffer
    static constexpr size_t bytes = (size_t)2 * (Q + K + V) * 2 + (size_t)2 * STG * 4;
};

__device__ __forceinline__ void split_h2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(__fsub_rn(x0, hf.x), __fsub_rn(x1, hf.y));
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}
__device__ __forceinline__ void mma_h16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t ld_h2(const uint16_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

template <int HD>
__global__ void __launch_bounds__(kPThreads, 1)
    k_prefill_attend_tc(const SplitAttnArgs a, uint32_t slots, uint32_t qb_tokens, uint32_t seg) {
    using Geo = PfTcGeom<HD>;
    constexpr uint32_t NK4 = HD / 4, HALF = HD / 2, NT = HD / 8, QS = Geo::QS, KS = Geo::KS, VS = Geo::VS,
                       SS = Geo::SS;
    extern __shared__ __align__(16) uint16_t smh[];
    uint16_t* Qh = smh;
    uint16_t* Ql = Qh + Geo::Q;
    uint16_t* Kh = Ql + Geo::Q;
    uint16_t* Kl = Kh + Geo::K;
    uint16_t* Vh = Kl + Geo::K;  // V^T [dim][position]
    uint16_t* Vl = Vh + Geo::V;
    float* Ks = reinterpret_cast<float*>(Vl + Geo::V);  // staging [position][SS]
    float* Vs = Ks + Geo::STG;
    __shared__ uint32_t s_lim[kTcRows];
    __shared__ uint32_t s_max;
    const uint32_t s = blockIdx.x, qb = blockIdx.y, kvh = blockIdx.z, tid = threadIdx.x;
    const uint32_t Gf = a.nh / a.nkv, t0 = qb * qb_tokens;
    const KTrace tr(a.trace, a.trace_slot);
    tr.enter();
    pdl_launch_dependents();
    if (tid < kTcRows) {
        uint32_t lim = 0;
        if (tid < qb_tokens && t0 + tid < slots) {
            const DevCtl* c = a.ctl + t0 + tid;
            const uint32_t pos = attn::ldv(&c->pos);
            if (attn::ldv(&c->active) != 0 && pos < a.max_ctx) lim = pos + 1;
        }
        s_lim[tid] = lim;
    }
    __syncthreads();
    if (tid < 32) {
        uint32_t m = 0;
        for (uint32_t i = tid; i < kTcRows; i += 32) m = s_lim[i] > m ? s_lim[i] : m;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const uint32_t o = __shfl_xor_sync(0xffffffffu, m, off);
            m = o > m ? o : m;
        }
        if (tid == 0) s_max = m;
    }
    __syncthreads();
    const uint32_t lim_max = s_max, p_begin = s * seg;
    if (lim_max <= p_begin) {
        tr.exit();
        return;
    }
    const uint32_t p_end = p_begin + seg < lim_max ? p_begin + seg : lim_max;
    const uint32_t nch = (p_end - p_begin + kPCh - 1) / kPCh;
    const float* kv = a.kv[t0];
    const uint32_t layer = a.layer;
    auto stage = [&](uint32_t c) {  // chunk c's cached rows into the staging buffers, one commit group
        const uint32_t c0 = p_begin + c * kPCh, cnt = p_end - c0 < kPCh ? p_end - c0 : kPCh;
        for (uint32_t i = tid; i < cnt * NK4; i += kPThreads) {
            const uint32_t rr = i / NK4, k4 = i % NK4;
            cp_async16(Ks + rr * SS + 4 * k4, kv + attn::kv_row_off(a, layer, kvh, HD, c0 + rr, 0) + 4 * k4);
            cp_async16(Vs + rr * SS + 4 * k4, kv + attn::kv_row_off(a, layer, kvh, HD, c0 + rr, 1) + 4 * k4);
        }
        attn::cp_commit();
    };

    pdl_wait();
    stage(0);

    // q rows: partials in split order, the bias, RoPE (as k_prefill_attend),
    // then the f16 pairs; zero for rows without a token
    for (uint32_t j = tid; j < kTcRows * (HD / 8); j += kPThreads) {
        const uint32_t r = j / (HD / 8), k4 = j % (HD / 8), t = r / Gf, h = r % Gf;
        float4 x0 = make_float4(0.0f, 0.0f, 0.0f, 0.0f), x1 = x0;
        const uint32_t lim = r < qb_tokens * Gf ? s_lim[t] : 0u;
        if (lim) {
            const uint32_t pos = lim - 1, row = (kvh * Gf + h) * HD + 4 * k4;
            const float* src = a.qkv + (size_t)(t0 + t) * a.qkv_rows + row;
            for (uint32_t q = 0; q < a.n_part; q++) {
                x0 = attn::f4add(x0, __ldcg(reinterpret_cast<const float4*>(src + q * a.part_stride)));
                x1 = attn::f4add(x1, __ldcg(reinterpret_cast<const float4*>(src + q * a.part_stride + HALF)));
            }
            if (a.bias) {
                x0 = attn::f4add(x0, *reinterpret_cast<const float4*>(a.bias + row));
                x1 = attn::f4add(x1, *reinterpret_cast<const float4*>(a.bias + row + HALF));
            }
            const float4 c = *reinterpret_cast<const float4*>(a.rope_cos + (size_t)pos * HALF + 4 * k4);
            const float4 sn = *reinterpret_cast<const float4*>(a.rope_sin + (size_t)pos * HALF + 4 * k4);
            auto rot = [](float& u, float& w, float cc, float ss) {
                const float u0 = u, w0 = w;
                u = __fsub_rn(__fmul_rn(u0, cc), __fmul_rn(w0, ss));
                w = __fadd_rn(__fmul_rn(u0, ss), __fmul_rn(w0, cc));
            };
            rot(x0.x, x1.x, c.x, sn.x);
            rot(x0.y, x1.y, c.y, sn.y);
            rot(x0.z, x1.z, c.z, sn.z);
            rot(x0.w, x1.w, c.w, sn.w);
        }
        uint2 h0, l0, h1, l1;
        split_h2(x0.x, x0.y, h0.x, l0.x);
        split_h2(x0.z, x0.w, h0.y, l0.y);
        split_h2(x1.x, x1.y, h1.x, l1.x);
        split_h2(x1.z, x1.w, h1.y, l1.y);
        *reinterpret_cast<uint2*>(Qh + r * QS + 4 * k4) = h0;
        *reinterpret_cast<uint2*>(Ql + r * QS + 4 * k4) = l0;
        *reinterpret_cast<uint2*>(Qh + r * QS + HALF + 4 * k4) = h1;
        *reinterpret_cast<uint2*>(Ql + r * QS + HALF + 4 * k4) = l1;
    }

    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
    const uint32_t warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
    const uint32_t ra = warp * 16 + g, rb = ra + 8;  // this thread's two rows
    const uint32_t lima = ra < qb_tokens * Gf ? s_lim[ra / Gf] : 0u;
    const uint32_t limb = rb < qb_tokens * Gf ? s_lim[rb / Gf] : 0u;
    float ma = -FLT_MAX, mb = -FLT_MAX, la = 0.0f, lb = 0.0f;
    float O[NT][4];
#pragma unroll
    for (uint32_t n = 0; n < NT; n++) O[n][0] = O[n][1] = O[n][2] = O[n][3] = 0.0f;

    for (uint32_t c = 0; c < nch; c++) {
        const uint32_t c0 = p_begin + c * kPCh, cnt = p_end - c0 < kPCh ? p_end - c0 : kPCh;
        attn::cp_wait0();
        __syncthreads();  // staging holds chunk c; the previous chunk's pairs are consumed
        if (c == 0) tr.mark(1);
        // staging -> f16 pairs: K [position][dim]; V^T [dim][position] with
        // positions past the chunk's end zero (their probabilities are 0, and
        // 0 times a stale non-finite value would not be)
        for (uint32_t i = tid; i < kPCh * NK4; i += kPThreads) {
            const uint32_t rr = i / NK4, k4 = i % NK4;
            float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (rr < cnt) x = *reinterpret_cast<const float4*>(Ks + rr * SS + 4 * k4);
            uint2 h, l;
            split_h2(x.x, x.y, h.x, l.x);
            split_h2(x.z, x.w, h.y, l.y);
            *reinterpret_cast<uint2*>(Kh + rr * KS + 4 * k4) = h;
            *reinterpret_cast<uint2*>(Kl + rr * KS + 4 * k4) = l;
        }
        for (uint32_t i = tid; i < kPCh * NK4; i += kPThreads) {
            const uint32_t rr = i % kPCh, k4 = i / kPCh;  // lanes along positions: the V^T writes are contiguous
            float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (rr < cnt) x = *reinterpret_cast<const float4*>(Vs + rr * SS + 4 * k4);
            const float xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (uint32_t e = 0; e < 4; e++) {
                const __half h = __float2half_rn(xv[e]);
                Vh[(4 * k4 + e) * VS + rr] = __half_as_ushort(h);
                Vl[(4 * k4 + e) * VS + rr] = __half_as_ushort(__float2half_rn(__fsub_rn(xv[e], __half2float(h))));
            }
        }
        __syncthreads();  // pairs ready; staging free
        if (c + 1 < nch) stage(c + 1);

        // scores: 16 rows x 64 positions per warp
        float S[8][4];
#pragma unroll
        for (uint32_t j = 0; j < 8; j++) S[j][0] = S[j][1] = S[j][2] = S[j][3] = 0.0f;
#pragma unroll
        for (uint32_t k0 = 0; k0 < HD; k0 += 16) {
            uint32_t ah[4], al[4];
            ah[0] = ld_h2(Qh + ra * QS + k0 + 2 * t4);
            ah[1] = ld_h2(Qh + rb * QS + k0 + 2 * t4);
            ah[2] = ld_h2(Qh + ra * QS + k0 + 2 * t4 + 8);
            ah[3] = ld_h2(Qh + rb * QS + k0 + 2 * t4 + 8);
            al[0] = ld_h2(Ql + ra * QS + k0 + 2 * t4);
            al[1] = ld_h2(Ql + rb * QS + k0 + 2 * t4);
            al[2] = ld_h2(Ql + ra * QS + k0 + 2 * t4 + 8);
            al[3] = ld_h2(Ql + rb * QS + k0 + 2 * t4 + 8);
            // four n-tiles at a time, each accumulator's three products in
            // the same order, the tiles interleaved (independent MMAs between
            // dependent ones)
#pragma unroll
            for (uint32_t j0 = 0; j0 < 8; j0 += 4) {
                uint32_t bh[4][2], bl[4][2];
#pragma unroll
                for (uint32_t u = 0; u < 4; u++) {
                    const uint32_t kr = (8 * (j0 + u) + g) * KS + k0 + 2 * t4;
                    bh[u][0] = ld_h2(Kh + kr);
                    bh[u][1] = ld_h2(Kh + kr + 8);
                    bl[u][0] = ld_h2(Kl + kr);
                    bl[u][1] = ld_h2(Kl + kr + 8);
                }
#pragma unroll
                for (uint32_t u = 0; u < 4; u++) mma_h16(S[j0 + u], al, bh[u][0], bh[u][1]);
#pragma unroll
                for (uint32_t u = 0; u < 4; u++) mma_h16(S[j0 + u], ah, bl[u][0], bl[u][1]);
#pragma unroll
                for (uint32_t u = 0; u < 4; u++) mma_h16(S[j0 + u], ah, bh[u][0], bh[u][1]);
            }
        }
        // online softmax per row (row a: S[j][0..1], row b: S[j][2..3];
        // positions 8 j + 2 t4 + e); the 4 lanes of a row reduce by shuffles.
        // Selects, not branches: every lane takes every shuffle.
        float mxa = -FLT_MAX, mxb = -FLT_MAX;
#pragma unroll
        for (uint32_t j = 0; j < 8; j++)
#pragma unroll
            for (uint32_t e = 0; e < 2; e++) {
                const uint32_t col = 8 * j + 2 * t4 + e;
                const bool in = col < cnt;
                S[j][e] = in && c0 + col < lima ? __fmul_rn(S[j][e], scale) : -FLT_MAX;
                S[j][2 + e] = in && c0 + col < limb ? __fmul_rn(S[j][2 + e], scale) : -FLT_MAX;
                mxa = fmaxf(mxa, S[j][e]);
                mxb = fmaxf(mxb, S[j][2 + e]);
            }
#pragma unroll
        for (int off = 1; off < 4; off <<= 1) {
            mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, off));
            mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, off));
        }
        const bool nonea = mxa == -FLT_MAX, noneb = mxb == -FLT_MAX;
        const float mna = nonea ? ma : fmaxf(ma, mxa), mnb = noneb ? mb : fmaxf(mb, mxb);
        float suma = 0.0f, sumb = 0.0f;
#pragma unroll
        for (uint32_t j = 0; j < 8; j++)
#pragma unroll
            for (uint32_t e = 0; e < 2; e++) {
                S[j][e] = S[j][e] == -FLT_MAX ? 0.0f : __expf(__fsub_rn(S[j][e], mna));
                S[j][2 + e] = S[j][2 + e] == -FLT_MAX ? 0.0f : __expf(__fsub_rn(S[j][2 + e], mnb));
                suma = __fadd_rn(suma, S[j][e]);
                sumb = __fadd_rn(sumb, S[j][2 + e]);
            }
#pragma unroll
        for (int off = 1; off < 4; off <<= 1) {
            suma = __fadd_rn(suma, __shfl_xor_sync(0xffffffffu, suma, off));
            sumb = __fadd_rn(sumb, __shfl_xor_sync(0xffffffffu, sumb, off));
        }
        const float fa = nonea ? 1.0f : (ma == -FLT_MAX ? 0.0f : __expf(__fsub_rn(ma, mna)));
        const float fb = noneb ? 1.0f : (mb == -FLT_MAX ? 0.0f : __expf(__fsub_rn(mb, mnb)));
        la = nonea ? la : __fadd_rn(__fmul_rn(la, fa), suma);
        lb = noneb ? lb : __fadd_rn(__fmul_rn(lb, fb), sumb);
        ma = mna;
        mb = mnb;
#pragma unroll
        for (uint32_t n = 0; n < NT; n++) {
            O[n][0] = __fmul_rn(O[n][0], fa);
            O[n][1] = __fmul_rn(O[n][1], fa);
            O[n][2] = __fmul_rn(O[n][2], fb);
            O[n][3] = __fmul_rn(O[n][3], fb);
        }
        // P.V: the 16-position slab k = positions 16 q .. +15 is score
        // n-tiles 2q and 2q + 1
#pragma unroll
        for (uint32_t q = 0; q < kPCh / 16; q++) {
            uint32_t ph[4], pl[4];
            split_h2(S[2 * q][0], S[2 * q][1], ph[0], pl[0]);
            split_h2(S[2 * q][2], S[2 * q][3], ph[1], pl[1]);
            split_h2(S[2 * q + 1][0], S[2 * q + 1][1], ph[2], pl[2]);
            split_h2(S[2 * q + 1][2], S[2 * q + 1][3], ph[3], pl[3]);
#pragma unroll
            for (uint32_t n0 = 0; n0 < NT; n0 += 4) {
                uint32_t bh[4][2], bl[4][2];
#pragma unroll
                for (uint32_t u = 0; u < 4; u++) {
                    const uint32_t vr = (8 * (n0 + u) + g) * VS + 16 * q + 2 * t4;
                    bh[u][0] = ld_h2(Vh + vr);
                    bh[u][1] = ld_h2(Vh + vr + 8);
                    bl[u][0] = ld_h2(Vl + vr);
                    bl[u][1] = ld_h2(Vl + vr + 8);
                }
#pragma unroll
                for (uint32_t u = 0; u < 4; u++) mma_h16(O[n0 + u], pl, bh[u][0], bh[u][1]);
#pragma unroll
                for (uint32_t u = 0; u < 4; u++) mma_h16(O[n0 + u], ph, bl[u][0], bl[u][1]);
#pragma unroll
                for (uint32_t u = 0; u < 4; u++) mma_h16(O[n0 + u], ph, bh[u][0], bh[u][1]);
            }
        }
    }
    attn::cp_wait0();
    tr.mark(2);

    const uint32_t rec = attn_record(Gf, HD);
#pragma unroll
    for (uint32_t side = 0; side < 2; side++) {
        const uint32_t r = side ? rb : ra, lim = side ? limb : lima;
        const float m = side ? mb : ma, l = side ? lb : la;
        if (lim <= p_begin) continue;
        const uint32_t slot = t0 + r / Gf, h = r % Gf;
        if (lim <= seg) {
            const size_t o = (size_t)slot * a.out_stride + (size_t)(kvh * Gf + h) * HD;
#pragma unroll
            for (uint32_t n = 0; n < NT; n++) {
                store_out(a, o + 8 * n + 2 * t4, __fdiv_rn(O[n][2 * side], l));
                store_out(a, o + 8 * n + 2 * t4 + 1, __fdiv_rn(O[n][2 * side + 1], l));
            }
        } else {
            float* part = a.partials + ((size_t)(slot * a.nkv + kvh) * a.max_splits + s) * rec;
#pragma unroll
            for (uint32_t n = 0; n < NT; n++)
                *reinterpret_cast<float2*>(part + h * HD + 8 * n + 2 * t4) = make_float2(O[n][2 * side], O[n][2 * side + 1]);
            if (t4 == 0) {
                part[Gf * HD + h] = m;
                part[Gf * HD + Gf + h] = l;
            }
        }
    }
    tr.exit();
}

// The append half of a prefill pass (model.rs:268-275): one warp per
// (token, KV head) rebuilds the token's k and v from the QKV product
// (split-K partials in split order, then the bias: the split items' order,
// so the rows have the same bits), applies RoPE to k (model.rs:365-373),
// writes both rows and, when the region tracks writes, marks their pages
// dirty once the rows are visible.
template <int HD>
__global__ void __launch_bounds__(kPThreads) k_prefill_append(const SplitAttnArgs a, uint32_t slots) {
    constexpr uint32_t HALF = HD / 2;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t item = blockIdx.x * (kPThreads / 32) + warp;
    const KTrace tr(a.trace, a.trace_slot);
    tr.enter();
    pdl_launch_dependents();
    const bool in = item < slots * a.nkv;
    const uint32_t slot = in ? item / a.nkv : 0, kvh = in ? item % a.nkv : 0;
    DevCtl* ctl = a.ctl + slot;
    const bool active = in && attn::ldv(&ctl->active) != 0;
    const uint32_t pos = in ? attn::ldv(&ctl->pos) : 0;
    pdl_wait();
    if (active && pos >= a.max_ctx && lane == 0 && kvh == 0) atomicOr(&ctl->err, ERR_POS);
    if (active && pos < a.max_ctx) {
        float* kv = a.kv[slot];
        const float* src = a.qkv + (size_t)slot * a.qkv_rows;
        const uint32_t krow = a.nh * HD + kvh * HD, vrow = (a.nh + a.nkv) * HD + kvh * HD;
        auto row = [&](uint32_t r) {  // float4 at row offset r: partials in split order, then the bias
            float4 p = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            for (uint32_t q = 0; q < a.n_part; q++)
                p = attn::f4add(p, __ldcg(reinterpret_cast<const float4*>(src + q * a.part_stride + r)));
            if (a.bias) p = attn::f4add(p, *reinterpret_cast<const float4*>(a.bias + r));
            return p;
        };
        if (lane < HALF / 4) {  // k: the float4 pair (lane, lane + HALF/4) that RoPE rotates together
            float4 x0 = row(krow + 4 * lane), x1 = row(krow + HALF + 4 * lane);
            const float4 c = *reinterpret_cast<const float4*>(a.rope_cos + (size_t)pos * HALF + 4 * lane);
            const float4 sn = *reinterpret_cast<const float4*>(a.rope_sin + (size_t)pos * HALF + 4 * lane);
            auto rot = [](float& u, float& w, float cc, float ss) {
                const float u0 = u, w0 = w;
                u = __fsub_rn(__fmul_rn(u0, cc), __fmul_rn(w0, ss));
                w = __fadd_rn(__fmul_rn(u0, ss), __fmul_rn(w0, cc));
            };
            rot(x0.x, x1.x, c.x, sn.x);
            rot(x0.y, x1.y, c.y, sn.y);
            rot(x0.z, x1.z, c.z, sn.z);
            rot(x0.w, x1.w, c.w, sn.w);
            float* kd = kv + attn::kv_row_off(a, a.layer, kvh, HD, pos, 0);
            reinterpret_cast<float4*>(kd)[lane] = x0;
            reinterpret_cast<float4*>(kd + HALF)[lane] = x1;
        }
        if (lane < HD / 4)
            reinterpret_cast<float4*>(kv + attn::kv_row_off(a, a.layer, kvh, HD, pos, 1))[lane] = row(vrow + 4 * lane);
        __syncwarp();
        if (lane < 2 && attn::ldv(a.tracking[slot]) != 0) {  // lane 0: the k row's pages, lane 1: the v row's
            __threadfence();
            const uint64_t off = attn::kv_row_off(a, a.layer, kvh, HD, pos, lane) * 4, last = off + HD * 4 - 1;
            uint64_t* dirty = a.dirty[slot];
            for (uint64_t pg = off >> a.page_shift; pg <= (last >> a.page_shift); pg++)
                atomicOr(reinterpret_cast<unsigned long long*>(&dirty[pg >> 6]), 1ull << (pg & 63));
        }
    }
    tr.exit();
}

// combine_staged's space for at most nseg segments: maxima, sums, weights
// and a tile of min(kCombTile, nseg) segment outputs.
size_t combine_smem(uint32_t hd, uint32_t nseg, uint32_t G) {
    const uint32_t rows = nseg < attn::kCombTile ? nseg : attn::kCombTile;
    return ((size_t)3 * nseg * G + 20 + (size_t)rows * G * hd) * sizeof(float);
}

}  // namespace

// Segment length: 384 positions (6 chunks per CTA; measured on 1,024-token
// passes at 1,023-2,046 positions of the 1.5B shape, attend + merge: 166 µs
// at 384 against 188 at 256, 177 at 512, 195 at 768), longer where max_ctx
// needs more than kPrefillMaxSegs segments.
uint32_t attn_prefill_seg(uint32_t max_ctx) {
    const uint32_t chunks = (max_ctx + kPCh - 1) / kPCh;
    const uint32_t seg = (chunks + kPrefillMaxSegs - 1) / kPrefillMaxSegs * kPCh;
    return seg > 384 ? seg : 384;
}

uint32_t attn_prefill_segs(uint32_t max_ctx) {
    const uint32_t seg = attn_prefill_seg(max_ctx);
    return (max_ctx + seg - 1) / seg;
}

bool attn_prefill_supported(uint32_t head_dim, uint32_t nh, uint32_t nkv) {
    return (head_dim == 64 || head_dim == 128) && nkv && nh % nkv == 0 && nh / nkv <= 8;
}

cudaError_t attn_prefill_set_smem_limits(int optin) {
    const void* fa[] = {(const void*)k_prefill_attend<64>, (const void*)k_prefill_attend<128>,
                        (const void*)k_prefill_attend_tc<64>, (const void*)k_prefill_attend_tc<128>};
    const size_t na[] = {PfGeom<64>::bytes, PfGeom<128>::bytes, PfTcGeom<64>::bytes, PfTcGeom<128>::bytes};
    for (int i = 0; i < 4; i++) {
        if (na[i] > (size_t)optin) continue;
        const cudaError_t e = cudaFuncSetAttribute(fa[i], cudaFuncAttributeMaxDynamicSharedMemorySize, (int)na[i]);
        if (e != cudaSuccess) return e;
    }
    const void* fc[] = {(const void*)k_prefill_combine<64>, (const void*)k_prefill_combine<128>};
    const uint32_t hds[] = {64, 128};
    for (int i = 0; i < 2; i++) {
        const size_t need = combine_smem(hds[i], kPrefillMaxSegs, 8);
        const cudaError_t e = cudaFuncSetAttribute(fc[i], cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)(need < (size_t)optin ? need : (size_t)optin));
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_prefill_append(uint32_t head_dim, const SplitAttnArgs& a, uint32_t slots, cudaStream_t st) {
    if (!attn_prefill_supported(head_dim, a.nh, a.nkv) || slots == 0) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((slots * a.nkv + kPThreads / 32 - 1) / (kPThreads / 32));
    cfg.blockDim = dim3(kPThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return head_dim == 64 ? cudaLaunchKernelEx(&cfg, k_prefill_append<64>, a, slots)
                          : cudaLaunchKernelEx(&cfg, k_prefill_append<128>, a, slots);
}

size_t attn_prefill_smem(uint32_t head_dim, bool tensor_cores) {
    if (tensor_cores) return head_dim == 64 ? PfTcGeom<64>::bytes : PfTcGeom<128>::bytes;
    return head_dim == 64 ? PfGeom<64>::bytes : PfGeom<128>::bytes;
}

cudaError_t launch_attn_prefill(uint32_t head_dim, const SplitAttnArgs& a, uint32_t slots, uint32_t seg,
                                cudaStream_t st, uint32_t trace_slot, bool tensor_cores) {
    if (!attn_prefill_supported(head_dim, a.nh, a.nkv) || seg == 0 || slots == 0 || (!a.out_f32 && !a.out_hi))
        return cudaErrorInvalidValue;
    const uint32_t G = a.nh / a.nkv, qb_tokens = (tensor_cores ? kTcRows : kRows) / G;
    const uint32_t nseg = (a.max_ctx + seg - 1) / seg;
    if (nseg > a.max_splits || nseg > kPrefillMaxSegs) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(nseg, (slots + qb_tokens - 1) / qb_tokens, a.nkv);
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = attn_prefill_smem(head_dim, tensor_cores);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    SplitAttnArgs b = a;
    b.trace_slot = trace_slot;
    cudaError_t e;
    if (tensor_cores)
        e = head_dim == 64 ? cudaLaunchKernelEx(&cfg, k_prefill_attend_tc<64>, b, slots, qb_tokens, seg)
                           : cudaLaunchKernelEx(&cfg, k_prefill_attend_tc<128>, b, slots, qb_tokens, seg);
    else
        e = head_dim == 64 ? cudaLaunchKernelEx(&cfg, k_prefill_attend<64>, b, slots, qb_tokens, seg)
                           : cudaLaunchKernelEx(&cfg, k_prefill_attend<128>, b, slots, qb_tokens, seg);
    if (e != cudaSuccess) return e;
    cfg.gridDim = dim3(a.nkv, slots, 1);
    cfg.dynamicSmemBytes = combine_smem(head_dim, nseg, G);
    b.trace_slot = trace_slot + 1;
    return head_dim == 64 ? cudaLaunchKernelEx(&cfg, k_prefill_combine<64>, b, seg)
                          : cudaLaunchKernelEx(&cfg, k_prefill_combine<128>, b, seg);
}

}  // namespace hs
