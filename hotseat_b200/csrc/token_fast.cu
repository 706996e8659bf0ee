// One decode token of the GPU-native numeric path (HS_NUMERIC_FAST, batch 1)
// as a single persistent kernel: every layer's five phases (QKV, attention,
// O, gate/up, down) and the LM head with no kernel boundary and no grid
// barrier between them (each phase hands its outputs on as tagged entries
// that their readers poll), and the weight stream running ahead of the
// compute.
//
//   warp 8 (producer)  streams this CTA's rows of every weight matrix, in
//                      phase order for the whole token, through a ring of
//                      shared-memory slots with 1-D bulk copies. It never
//                      waits for activations, so the weights of the next
//                      phases arrive while the current phase computes or
//                      waits for its input.
//   warps 0-7          per phase: await and build the input vector (RMSNorm
//                      of x, the attention output or hb), take the weight tiles from
//                      the ring, compute their rows and apply the epilogue
//                      (bias, residual add, SiLU gate); in the attention phase
//                      they run the split-KV attention items (attn_body.cuh).
//
// The arithmetic is that of the per-kernel fast path operation for operation
// (decode_fast.cu k_gemv_fast: threads per row from the row length, chunk
// order, packed FMA chains, xor tree, warp-order combine; attn_split.cu for
// attention), so a token's logits and KV rows are bit-identical to it, and
// nothing depends on the grid size. One CTA per SM, launched cooperatively
// so that all CTAs are resident; every wait is bounded and reports
// ERR_TIMEOUT instead of spinning forever.
#include <algorithm>
#include <cfloat>

#include "attn_body.cuh"
#include "common.h"
#include "kernels.h"

namespace hs {
namespace {

constexpr uint32_t kConsumers = 256;
constexpr uint32_t kThreads = kConsumers + 32;
constexpr uint32_t kPart = 2048;         // warp partials of a phase: this CTA's rows * warps per row
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr uint32_t kMaxNorm = 8;         // RMSNorm gains per consumer thread (d <= 2048)
constexpr uint32_t kReaderCombine = 8;   // up to this many attention splits, every O-phase CTA combines them
constexpr uint32_t kMaxLayers = 64;      // layer table copied to shared memory
// K/V chunk buffers of an attention item: one (its first chunk is
// prefetched; an item has more only past max_splits * 64 positions).
__host__ __device__ constexpr uint32_t attn_buf(uint32_t) { return 1; }

__device__ __forceinline__ uint32_t ldv(const uint32_t* p) { return *(const volatile uint32_t*)p; }
// Bytes of the shared area that holds an attention item or, between
// attention phases, an input vector of up to xmax tagged entries.
__host__ __device__ constexpr size_t att_area(uint32_t hd, uint32_t xmax) {
    return attn::item_smem(hd, attn_buf(hd)) > (size_t)xmax * 8 ? attn::item_smem(hd, attn_buf(hd)) : (size_t)xmax * 8;
}
// Exact f16 -> f32 of both halves of a word.
__device__ __forceinline__ uint64_t widen2(uint32_t v) {
    float a, b;
    asm("{ .reg .b16 lo, hi;\n mov.b32 {lo, hi}, %2;\n add.rn.f32.f16 %0, lo, 0f80000000;\n"
        " add.rn.f32.f16 %1, hi, 0f80000000; }"
        : "=f"(a), "=f"(b)
        : "r"(v));
    return pack2(a, b);
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Block barrier of the 256 consumer threads that also ORs a predicate.
__device__ __forceinline__ bool any256(bool p) {
    uint32_t r;
    asm volatile(
        "{ .reg .pred pi, po;\n setp.ne.u32 pi, %1, 0;\n bar.red.or.pred po, 1, 256, pi;\n selp.u32 %0, 1, 0, po; }"
        : "=r"(r)
        : "r"((uint32_t)p)
        : "memory");
    return r != 0;
}

// Threads per row for rows of length k: the fast GEMV's rule (a power of two
// from 32 with at most 6 chunks of 8 elements per thread, 256 at most).
__host__ __device__ inline uint32_t row_threads(uint32_t k) {
    const uint32_t nchunks = k / 8;
    uint32_t T = 32;
    while (T < 256 && (nchunks + T - 1) / T > 6) T *= 2;
    return T;
}

enum Phase : uint32_t { PH_QKV = 0, PH_O = 1, PH_GU = 2, PH_DOWN = 3, PH_HEAD = 4 };
// Writers of tagged entries, in a layer's order (tag(l, TG_*)).
enum TagPhase : uint32_t { TG_QKV = 0, TG_ATT = 1, TG_O = 2, TG_GU = 3, TG_DOWN = 4 };

// The weights of one phase: `rows` rows of length k, one matrix or the
// gate/up pair (a slot holds the same rows of both, w0's first).
struct Mat {
    const uint16_t *w0, *w1;
    uint32_t rows, k;
};

__device__ __forceinline__ Mat phase_mat(const TokenArgs& a, const TokLayer* layers, uint32_t ph, uint32_t l) {
    if (ph == PH_HEAD) return Mat{a.head_w, nullptr, a.vocab, a.d};
    const TokLayer& L = layers[l];
    switch (ph) {
        case PH_QKV: return Mat{L.wqkv, nullptr, (a.nh + 2 * a.nkv) * a.hd, a.d};
        case PH_O: return Mat{L.wo, nullptr, a.d, a.nh * a.hd};
        case PH_GU: return Mat{L.wgate, L.wup, a.ff, a.d};
        default: return Mat{L.wdown, nullptr, a.d, a.ff};
    }
}
// Rows per ring slot for a phase: as many as fit, rounded down so that a
// tile's rows (both matrices of a pair) are a whole number of passes of the
// CTA's row groups (256 / threads per row) when there are at least that many.
__host__ __device__ inline uint32_t tile_rows(uint32_t slot_bytes, uint32_t k, uint32_t nmat) {
    const uint32_t groups = kConsumers / row_threads(k);
    uint32_t vr = slot_bytes / (k * 2 * nmat) * nmat;
    if (vr >= groups) vr = vr / groups * groups;
    return vr / nmat > 0 ? vr / nmat : 1;
}
__device__ __forceinline__ uint32_t tile_rows(const TokenArgs& a, const Mat& m) {
    return tile_rows(a.slot_bytes, m.k, m.w1 ? 2u : 1u);
}

// Consumer state carried across phases.
struct RowState {
    uint32_t it;             // tiles taken from the ring so far
    bool dead;               // a weight wait ran out: stop waiting
    uint64_t wait_cy, comp_cy, tiles;  // trace mode (CTA 0, thread 0)
};

// One pass of a thread group over up to RB of a tile's rows (rows vr0,
// vr0 + Gp, ...): T threads per row, each over its CM chunks j = tg, tg + T,
// ... (the last only where j < nchunks) in order with packed FMA, then the
// xor tree; lane 0 of each of the row's warps stores its partial. T and CM
// are compile-time so that every load of the pass can be issued up front.
template <uint32_t T, uint32_t CM, uint32_t RB>
__device__ __forceinline__ void tile_pass(const uint8_t* st, const uint64_t (&xp)[CM * 4], float* part, uint32_t k,
                                          uint32_t vr0, uint32_t vrows, uint32_t n, uint32_t base, uint32_t nrows,
                                          uint32_t tg) {
    constexpr uint32_t Gp = kConsumers / T, WG = T / 32;
    const uint32_t nchunks = k / 8, wig = tg / 32;
    const uint8_t* rowp[RB];
    bool okr[RB];
#pragma unroll
    for (uint32_t q = 0; q < RB; q++) {
        okr[q] = vr0 + Gp * q < vrows;
        rowp[q] = st + (size_t)(okr[q] ? vr0 + Gp * q : vr0) * k * 2;
    }
    uint64_t acc[RB];
#pragma unroll
    for (uint32_t q = 0; q < RB; q++) acc[q] = 0;
    const bool tail = tg + T * (CM - 1) < nchunks;
#pragma unroll
    for (uint32_t c = 0; c < CM; c++) {
        const uint32_t j = tg + T * c;
        if (c + 1 < CM || tail) {
            uint4 w[RB];
#pragma unroll
            for (uint32_t q = 0; q < RB; q++)
                if (okr[q]) w[q] = *reinterpret_cast<const uint4*>(rowp[q] + j * 16);
#pragma unroll
            for (uint32_t q = 0; q < RB; q++) {
                if (!okr[q]) continue;
                acc[q] = fma2(widen2(w[q].x), xp[4 * c + 0], acc[q]);
                acc[q] = fma2(widen2(w[q].y), xp[4 * c + 1], acc[q]);
                acc[q] = fma2(widen2(w[q].z), xp[4 * c + 2], acc[q]);
                acc[q] = fma2(widen2(w[q].w), xp[4 * c + 3], acc[q]);
            }
        }
    }
    float v[RB];
#pragma unroll
    for (uint32_t q = 0; q < RB; q++) {
        float p0, p1;
        unpack2(acc[q], &p0, &p1);
        v[q] = p0 + p1;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (uint32_t q = 0; q < RB; q++) v[q] += __shfl_xor_sync(0xffffffffu, v[q], o);
    if ((tg & 31) == 0)
#pragma unroll
        for (uint32_t q = 0; q < RB; q++) {
            if (!okr[q]) continue;
            const uint32_t vr = vr0 + Gp * q, mi = vr < n ? 0u : 1u;
            part[(mi * nrows + base + vr - mi * n) * WG + wig] = v[q];
        }
}

// The tiles of one phase for this CTA (rows [r0, r1) of m), in the
// producer's order: each row's warp partials go to `part` (rows of w1 after
// those of w0); a warp releases a slot as soon as it has read it. T =
// threads per row, CM = chunks per thread for m.k.
template <uint32_t T, uint32_t CM>
__device__ __forceinline__ void phase_tiles(const TokenArgs& a, const Mat m, uint32_t r0, uint32_t r1,
                                         const uint8_t* ring, uint64_t* full, uint64_t* empty, const float* xs,
                                         float* part, RowState& rs, bool tmark) {
    constexpr uint32_t Gp = kConsumers / T;
    const uint32_t tid = threadIdx.x, lane = tid & 31, grp = tid / T, tg = tid % T;
    const uint32_t per = tile_rows(a, m), nmat = m.w1 ? 2 : 1, nrows = r1 - r0, nslot = a.nslot;
    const uint32_t slot_bytes = a.slot_bytes, nchunks = m.k / 8;
    // this thread's slice of x (chunks tg, tg + T, ...), in registers for the phase
    uint64_t xp[CM * 4];
#pragma unroll
    for (uint32_t c = 0; c < CM; c++) {
        const uint32_t j = tg + T * c;
        const float4* src = reinterpret_cast<const float4*>(xs + 8 * (j < nchunks ? j : 0));
        const float4 lo = src[0], hi = src[1];
        xp[4 * c + 0] = pack2(lo.x, lo.y);
        xp[4 * c + 1] = pack2(lo.z, lo.w);
        xp[4 * c + 2] = pack2(hi.x, hi.y);
        xp[4 * c + 3] = pack2(hi.z, hi.w);
    }
    uint32_t it = rs.it, s = it % nslot, parity = (it / nslot) & 1;
    bool dead = rs.dead;
    for (uint32_t r = r0; r < r1; r += per, it++) {
        const uint32_t n = r1 - r < per ? r1 - r : per, vrows = nmat * n;
        const uint64_t c0 = tmark ? clock64() : 0;
        if (!dead && !mbar_wait_bounded(&full[s], parity, kSpinLimit)) {
            atomicOr(&a.ctl->err, ERR_TIMEOUT);
            dead = true;
        }
        const uint64_t c1 = tmark ? clock64() : 0;
        const uint8_t* st = ring + (size_t)s * slot_bytes;
        // one row per group, or passes of two side by side
        if (vrows <= Gp) {
            if (grp < vrows) tile_pass<T, CM, 1>(st, xp, part, m.k, grp, vrows, n, r - r0, nrows, tg);
        } else {
            for (uint32_t vr0 = grp; vr0 < vrows; vr0 += Gp * 2)
                tile_pass<T, CM, 2>(st, xp, part, m.k, vr0, vrows, n, r - r0, nrows, tg);
        }
        __syncwarp();
        // this warp is done with the slot; after a ring timeout it stops
        // releasing slots, so the producer stops filling them
        if (lane == 0 && !dead) mbar_arrive(&empty[s]);
        if (++s == nslot) {
            s = 0;
            parity ^= 1;
        }
        if (tmark) {
            rs.wait_cy += c1 - c0;
            rs.comp_cy += clock64() - c1;
            rs.tiles++;
        }
    }
    rs.it = it;
    rs.dead = dead;
}

// Compiled shape classes: head_dim, and (threads per row, chunks per thread)
// for rows of length d (QKV, O with nh*hd == d, gate/up, head) and ff (down).
struct TokShape {
    uint32_t hd, td, cmd, tf, cmf;
};
constexpr TokShape kShapes[] = {
    {64, 32, 4, 128, 5},   // Qwen2.5-0.5B: d 896, ff 4864
    {128, 32, 6, 256, 5},  // Qwen2.5-1.5B: d 1536, ff 8960
    {128, 64, 4, 256, 6},  // Qwen2.5-3B: d 2048, ff 11008
    {64, 32, 1, 32, 2},    // d 256, ff 512
    {128, 32, 1, 32, 3},   // d 256, ff 768
};

template <int HD, uint32_t TD, uint32_t CMD, uint32_t TF, uint32_t CMF>
__global__ void __launch_bounds__(kThreads, 1) k_token_fast(const __grid_constant__ TokenArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t G = gridDim.x, b = blockIdx.x;
    const uint32_t d = a.d, ff = a.ff, nkv = a.nkv;
    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)a.nslot * a.slot_bytes);
    uint64_t* empty = full + a.nslot;
    float* part = reinterpret_cast<float*>(empty + a.nslot);  // [kPart] warp partials of a phase's rows
    float* red = part + kPart;                                // [64]
    float* xs = red + 64;                                     // [max(d, ff, nh*hd)] input vector
    const uint32_t xn = d > ff ? d : ff;
    const uint32_t xmax = xn > a.nh * a.hd ? xn : a.nh * a.hd;
    float* att_sm = xs + xmax;  // one attention item, or the staged tagged input
    // the layers' weight pointers (read at every phase start)
    TokLayer* lay = reinterpret_cast<TokLayer*>(att_sm + att_area(HD, xmax) / 4);
    const KTrace tr(a.trace, a.trace_slot);
    tr.enter();
    if (tid == 0) {
        for (uint32_t s = 0; s < a.nslot; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumers / 32);  // one arrival per consumer warp
        }
        mbar_init_fence();
    }
    for (uint32_t i = tid; i < a.n_layers * (sizeof(TokLayer) / 8); i += kThreads)
        reinterpret_cast<uint64_t*>(lay)[i] = reinterpret_cast<const uint64_t*>(a.layers)[i];
    __syncthreads();
    DevCtl* ctl = a.ctl;
    const bool run = ldv(&ctl->active) != 0;
    const uint32_t pos = ldv(&ctl->pos), token = ldv(&ctl->token);
    const bool pos_ok = pos < a.attn.max_ctx, tok_ok = token < a.vocab, ok = run && pos_ok && tok_ok;
    if (run && !ok && tid == 0 && b == 0) atomicOr(&ctl->err, pos_ok ? ERR_TOKEN : ERR_POS);

    if (warp == kConsumers / 32) {
        // ---------------------------------------------------------- producer
        uint32_t it = 0;  // tiles put in flight
        if (lane == 0 && ok) {
            bool dead = false;
            for (uint32_t l = 0; l <= a.n_layers && !dead; l++) {
                for (uint32_t pi = 0; pi < (l < a.n_layers ? 4u : 1u) && !dead; pi++) {
                    const uint32_t ph = l < a.n_layers ? pi : (uint32_t)PH_HEAD;  // PH_QKV..PH_DOWN = 0..3
                    const Mat m = phase_mat(a, lay, ph, l);
                    uint32_t r0, r1;
                    split_range(m.rows, G, b, &r0, &r1);
                    const uint32_t per = tile_rows(a, m);
                    for (uint32_t r = r0; r < r1; r += per, it++) {
                        const uint32_t s = it % a.nslot, round = it / a.nslot;
                        if (round > 0 && !mbar_wait_bounded(&empty[s], (round - 1) & 1, kSpinLimit)) {
                            atomicOr(&ctl->err, ERR_TIMEOUT);
                            dead = true;
                            break;
                        }
                        const uint32_t n = r1 - r < per ? r1 - r : per, bytes = n * m.k * 2;
                        uint8_t* dst = ring + (size_t)s * a.slot_bytes;
                        mbar_expect_tx(&full[s], m.w1 ? 2 * bytes : bytes);
                        bulk_load_1d(dst, m.w0 + (size_t)r * m.k, bytes, &full[s]);
                        if (m.w1) bulk_load_1d(dst + bytes, m.w1 + (size_t)r * m.k, bytes, &full[s]);
                    }
                }
            }
        }
        __syncthreads();
        // Every consumer is past the ring. A fill the consumers stopped
        // waiting for (after a ring timeout) may still be landing: wait for
        // the last fill of every slot before the CTA's shared memory goes.
        if (lane == 0)
            for (uint32_t s = 0; s < a.nslot && s < it; s++) {
                const uint32_t last = s + (it - 1 - s) / a.nslot * a.nslot;
                mbar_wait_bounded(&full[s], (last / a.nslot) & 1, kSpinLimit);
            }
        tr.exit();
        return;
    }

    // -------------------------------------------------------------- consumers
    // Phases hand their outputs on as tagged entries (attn_body.cuh): the
    // writes of phase ph of layer l carry tag(l, ph), unique within this
    // launch and different from earlier launches' (the launch counter; the
    // host clears the entries every 2^21 launches, before the counter's
    // part of the tag could repeat), and every reader polls the entries it
    // needs until they carry the tag it waits for. Each phase needs all of the previous phase's outputs
    // (attention only its group's q/k/v rows), so no CTA can overwrite an
    // entry that another still has to read: the buffers are single.
    const uint32_t seq = ldv(a.seq);
    auto tag = [&](uint32_t l, uint32_t t) { return seq * 1024u + l * 5u + t + 1u; };  // t: TG_*
    bool dead = false;  // a wait ran out (the same in every consumer thread after any256)
    auto timed_out = [&](bool got) {
        if (!got && !dead) {
            dead = true;
            atomicOr(&ctl->err, ERR_TIMEOUT);
        }
    };
    uint32_t epoch = 0;  // phase interval (trace)
    RowState rs{0, false, 0, 0, 0};

    // Trace mode: per phase interval (5 a layer: QKV, attention, O,
    // gate/up, down; then the LM head), CTA 0's [input ready, rows done,
    // outputs written, next phase's input ready (%globaltimer ns), SM cycles
    // waiting for weight tiles, tiles, SM cycles computing rows, SM cycles
    // in the epilogue], then over all CTAs [~earliest, latest] outputs
    // written, the input staged and transformed (RMSNorm, or the split
    // combine), then (attention intervals) the clock64 checkpoints of CTA
    // 0's first attention item.
    const bool tmark = a.phase_ts && b == 0 && tid == 0;
    uint64_t epi_cy = 0;
    auto mark = [&](uint32_t k, uint64_t v) {
        if (tmark) a.phase_ts[20 * epoch + k] = v;
    };
    // End of a phase interval: trace words, then the next interval.
    auto phase_end = [&]() {
        attn::sync256();
        if (tid == 0) {
            mark(4, rs.wait_cy);
            mark(5, rs.tiles);
            mark(6, rs.comp_cy);
            mark(7, epi_cy);
            mark(2, tmark ? gtime() : 0);
            if (a.phase_ts) {  // over CTAs: latest, and latest of the complements (earliest)
                const unsigned long long t = gtime();
                atomicMax(reinterpret_cast<unsigned long long*>(a.phase_ts + 20 * epoch + 9), t);
                atomicMax(reinterpret_cast<unsigned long long*>(a.phase_ts + 20 * epoch + 8), ~t);
            }
            rs.wait_cy = rs.tiles = rs.comp_cy = epi_cy = 0;
        }
        epoch++;
    };
    // A phase's RMSNorm gains, loaded before its input is awaited.
    float gv[kMaxNorm];
    auto load_gain = [&](const float* g) {
#pragma unroll
        for (uint32_t k = 0; k < kMaxNorm; k++) {
            const uint32_t i = tid + k * kConsumers;
            gv[k] = i < d ? g[i] : 0.0f;
        }
    };
    // Tagged entries staged in the attention item's shared memory (free
    // outside attention) once every entry carries `want`: n_runs runs of
    // `len` entries (even), run r = g * group + j (j < group) from src +
    // g * group_stride + j * run_stride to stage + r * len; 16-byte
    // asynchronous copies, re-issued for the pairs not yet tagged, all of a
    // round in flight together. False after a.poll_limit rounds (the staged
    // values are then whatever arrived; no copy is left in flight).
    auto stage_tagged = [&](uint64_t* stage, const uint64_t* src, uint32_t n_runs, uint32_t len, uint32_t group,
                            size_t group_stride, size_t run_stride, uint32_t want) -> bool {
        const uint32_t per = len / 2, np = n_runs * per;
        auto from = [&](uint32_t i) {
            const uint32_t r = i / per;
            return src + (size_t)(r / group) * group_stride + (size_t)(r % group) * run_stride + 2 * (i % per);
        };
        for (uint32_t i = tid; i < np; i += kConsumers) cp_async16(stage + 2 * i, from(i));
        attn::cp_commit();
        for (uint32_t round = 0;; round++) {
            attn::cp_wait0();
            bool pending = false;
            for (uint32_t i = tid; i < np; i += kConsumers)
                if ((uint32_t)(stage[2 * i] >> 32) != want || (uint32_t)(stage[2 * i + 1] >> 32) != want) {
                    cp_async16(stage + 2 * i, from(i));
                    pending = true;
                }
            attn::cp_commit();
            if (!pending) return true;
            if (round >= a.poll_limit) {
                attn::cp_wait0();
                return false;
            }
        }
    };
    // n tagged entries into xs once they carry `want`.
    auto await_x = [&](const uint64_t* src, uint32_t n, uint32_t want) {
        uint64_t* stage = reinterpret_cast<uint64_t*>(att_sm);
        if (!dead) timed_out(stage_tagged(stage, src, 1, n, 1, 0, 0, want));
        dead = any256(dead);
        for (uint32_t i = tid; i < n; i += kConsumers) xs[i] = attn::tagged_value(stage[i]);
        attn::sync256();
    };
    // RMSNorm into xs of the embedding row (layer 0) or of x once it
    // carries `want`, with the loaded gains; the sum of squares by one warp
    // in the fast GEMV's order.
    auto norm_x = [&](bool embed, uint32_t want) {
        if (embed) {
            for (uint32_t i = tid; i < d; i += kConsumers) xs[i] = h2f(a.embd[(size_t)token * d + i]);
            attn::sync256();
        } else {
            await_x(a.tx, d, want);
        }
        mark(10, tmark ? gtime() : 0);
        if (tid < 32) {
            float ss = 0.0f;
            for (uint32_t i = tid; i < d; i += 32) ss = __fmaf_rn(xs[i], xs[i], ss);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (tid == 0) red[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)d), a.eps)));
        }
        attn::sync256();
        const float scale = red[0];
#pragma unroll
        for (uint32_t k = 0; k < kMaxNorm; k++) {
            const uint32_t i = tid + k * kConsumers;
            if (i < d) xs[i] = __fmul_rn(__fmul_rn(xs[i], scale), gv[k]);
        }
        attn::sync256();
        mark(11, tmark ? gtime() : 0);
    };
    if (ok) {
        const uint32_t n = pos + 1, Ls = attn_split_len(n, a.attn.max_splits, a.attn.ws_from), S = (n + Ls - 1) / Ls;
        const uint32_t G_ = a.nh / nkv, rec = attn_record(G_, a.hd);
        // attention item i: split i / (nkv * hsp), KV head (i / hsp) % nkv,
        // query-head part i % hsp
        const uint32_t hsp = attn_head_split(a.attn), n_items = S * nkv * hsp;
        // records of the splits, staged as tagged entries, and the per-head
        // weights must fit in the attention item's space
        const uint32_t used = G_ * a.hd + 2 * G_;  // written entries of a record
        const bool reader_combines = S > 1 && S <= kReaderCombine &&
                                     (size_t)nkv * S * used * 8 + a.nh * (S + 1) * 4 <= attn::item_smem(HD, attn_buf(HD));
        const uint32_t qrows = (a.nh + 2 * nkv) * a.hd;
        uint32_t dr0, dr1;  // this CTA's rows of d (O and down)
        split_range(d, G, b, &dr0, &dr1);
        // The residual of row `row` before the O phase of layer l: the
        // embedding at layer 0, else x as this CTA wrote it in the last down
        // phase (and before down: as it wrote it in O).
        auto resid = [&](uint32_t l, uint32_t ph, uint32_t row) -> float {
            return l == 0 && ph == PH_O ? h2f(a.embd[(size_t)token * d + row]) : attn::tagged_value(a.tx[row]);
        };
        load_gain(lay[0].attn_norm);
        // The epilogue operand of this thread's first row, read before the
        // phase's tiles: the QKV bias, or the residual row (O, down).
        float pre = 0.0f;
        // GEMV phases: QKV, O, gate/up, down per layer, then the LM head;
        // attention between QKV and O.
        for (uint32_t step = 0; step <= 4 * a.n_layers; step++) {
            const uint32_t l = step / 4, ph = l < a.n_layers ? step % 4 : (uint32_t)PH_HEAD;
            // ---- input vector
            if (ph == PH_QKV) {
                norm_x(l == 0, l > 0 ? tag(l - 1, TG_DOWN) : 0u);
                // this CTA's first attention item: start loading its cached
                // K/V rows and RoPE row (written by earlier tokens / constant)
                if (b < n_items) {
                    bool ws = false;
                    if constexpr (attn::WsGeom<HD, attn_buf(HD)>::OK) {
                        ws = attn_use_ws(pos + 1, a.attn.ws_from);
                        if (ws) attn::ws_prefetch<HD, attn_buf(HD)>(a.attn, l, b / (nkv * hsp), (b / hsp) % nkv, 0, pos, att_sm);
                    }
                    if (!ws)
                        attn::prefetch<HD, attn_buf(HD)>(a.attn, l, b / (nkv * hsp), (b / hsp) % nkv, 0, pos, att_sm);
                }
                uint32_t r0, r1;
                split_range(qrows, G, b, &r0, &r1);
                pre = tid < r1 - r0 ? lay[l].bqkv[r0 + tid] : 0.0f;
            } else if (ph == PH_O) {
                if (reader_combines) {
                    // the attention output from the splits' tagged records,
                    // as the last split's CTA would combine them: stage them
                    // in shared memory (the attention item's space), combine
                    // in split order
                    // records [kvh][split] of `used` tagged entries (the
                    // written part of each record, a multiple of 2)
                    uint64_t* ps = reinterpret_cast<uint64_t*>(att_sm);
                    const uint32_t gh = G_ * a.hd;
                    // (record (kvh, q) sits at (kvh * max_splits + q) * rec: runs of
                    // S records per KV head, so one run per record)
                    if (!dead)
                        timed_out(stage_tagged(ps, a.trec, nkv * S, used, S, (size_t)a.attn.max_splits * rec, rec,
                                               tag(l, TG_ATT)));
                    mark(10, tmark ? gtime() : 0);
                    // per query head: the split weights exp(m_q - M) and the
                    // rescaled sum, then every output element's weighted sum
                    // (the same operations as attn::combine, shared per head)
                    float* hw = reinterpret_cast<float*>(ps + (size_t)nkv * S * used);  // [nh][S + 1]: weights, sum
                    dead = any256(dead);
                    auto val = [&](uint32_t kvh, uint32_t q, uint32_t e) {
                        return attn::tagged_value(ps[(size_t)(kvh * S + q) * used + e]);
                    };
                    if (tid < a.nh) {
                        const uint32_t kvh = tid / G_, h = tid % G_;
                        float M = -FLT_MAX;
                        for (uint32_t q = 0; q < S; q++) M = fmaxf(M, val(kvh, q, gh + h));
                        float den = 0.0f;
                        for (uint32_t q = 0; q < S; q++) {
                            const float w = __expf(__fsub_rn(val(kvh, q, gh + h), M));
                            hw[tid * (S + 1) + q] = w;
                            den = __fadd_rn(den, __fmul_rn(w, val(kvh, q, gh + G_ + h)));
                        }
                        hw[tid * (S + 1) + S] = den;
                    }
                    attn::sync256();
                    mark(11, tmark ? gtime() : 0);
                    for (uint32_t idx = tid; idx < a.nh * a.hd; idx += kConsumers) {
                        const uint32_t head = idx / a.hd, kvh = head / G_, e = idx - kvh * gh;
                        const float* w = hw + head * (S + 1);
                        float num = 0.0f;
                        for (uint32_t q = 0; q < S; q++) num = __fadd_rn(num, __fmul_rn(w[q], val(kvh, q, e)));
                        xs[idx] = __fdiv_rn(num, w[S]);
                    }
                    attn::sync256();
                } else {
                    await_x(a.tatt, a.nh * a.hd, tag(l, TG_ATT));
                }
            } else if (ph == PH_DOWN) {
                await_x(a.thb, ff, tag(l, TG_GU));
            } else {  // gate/up, head
                norm_x(false, ph == PH_GU ? tag(l, TG_O) : tag(a.n_layers - 1, TG_DOWN));
            }
            mark(0, tmark ? gtime() : 0);
            // ---- rows, then the epilogue for this CTA's rows
            const Mat m = phase_mat(a, lay, ph, l);
            const uint32_t WG = row_threads(m.k) / 32;
            uint32_t r0, r1;
            split_range(m.rows, G, b, &r0, &r1);
            const uint32_t nrows = r1 - r0;
            if (m.k == d)
                phase_tiles<TD, CMD>(a, m, r0, r1, ring, full, empty, xs, part, rs, tmark);
            else
                phase_tiles<TF, CMF>(a, m, r0, r1, ring, full, empty, xs, part, rs, tmark);
            const uint64_t c2 = tmark ? clock64() : 0;
            attn::sync256();
            const float* bias = ph == PH_QKV ? lay[l].bqkv : nullptr;
            for (uint32_t i = tid; i < nrows; i += kConsumers) {
                float v = 0.0f, u = 0.0f;
                for (uint32_t w = 0; w < WG; w++) v += part[i * WG + w];
                if (m.w1)
                    for (uint32_t w = 0; w < WG; w++) u += part[(nrows + i) * WG + w];
                const uint32_t row = r0 + i;
                switch (ph) {
                    case PH_QKV: attn::st_tagged(a.tqkv + row, __fadd_rn(v, i == tid ? pre : bias[row]), tag(l, TG_QKV)); break;
                    case PH_GU: attn::st_tagged(a.thb + row, __fmul_rn(ref_silu(v), u), tag(l, TG_GU)); break;
                    case PH_HEAD: a.logits[row] = v; break;
                    default:  // O, down: the residual added
                        attn::st_tagged(a.tx + row, __fadd_rn(i == tid ? pre : resid(l, ph, row), v),
                                        tag(l, ph == PH_O ? TG_O : TG_DOWN));
                        break;
                }
            }
            if (tmark) epi_cy += clock64() - c2;
            // ---- operands of the next phase that do not wait for its input
            if (ph == PH_O) load_gain(lay[l].ffn_norm);
            if (ph == PH_GU) pre = tid < dr1 - dr0 ? resid(l, PH_DOWN, dr0 + tid) : 0.0f;
            if (ph == PH_DOWN) load_gain(l + 1 < a.n_layers ? lay[l + 1].attn_norm : a.out_norm);
            mark(1, tmark ? gtime() : 0);
            if (ph == PH_HEAD) break;
            phase_end();
            if (ph == PH_QKV) {
                // attention: the items of the S splits of this position
                mark(0, tmark ? gtime() : 0);
                const attn::TagIO tio{a.tqkv, a.tatt, a.trec, tag(l, TG_QKV), tag(l, TG_ATT), a.poll_limit};
                for (uint32_t i = b; i < n_items && !dead; i += G) {
                    attn::item<HD, attn_buf(HD), false>(a.attn, l, i / (nkv * hsp), (i / hsp) % nkv, i % hsp, 0, pos,
                                                        att_sm, i == b ? 1u : 0u, reader_combines,
                                                        tmark && i == b ? a.phase_ts + 20 * epoch + 12 : nullptr,
                                                        &tio);
                    attn::sync256();
                }
                if (b < n_items && dead) attn::cp_wait0();  // the prefetch of an item not run
                pre = tid < dr1 - dr0 ? resid(l, PH_O, dr0 + tid) : 0.0f;
                mark(1, tmark ? gtime() : 0);
                phase_end();
            }
        }
        mark(4, rs.wait_cy);
        mark(5, rs.tiles);
        mark(6, rs.comp_cy);
        mark(7, epi_cy);
        // the next launch's tags: after every CTA has read this launch's
        // counter (each wrote rows this CTA's LM head input needed)
        if (b == 0 && tid == 0) *a.seq = seq + 1;
    } else if (b == 0 && tid == 0) {
        *a.seq = seq + 1;
    }
    __syncthreads();
    tr.exit();
}

size_t fixed_smem(uint32_t d, uint32_t ff, uint32_t nh, uint32_t hd, uint32_t nslot) {
    const uint32_t xmax = std::max(std::max(d, ff), nh * hd);
    return (size_t)2 * nslot * 8 + (kPart + 64) * 4 + (size_t)xmax * 4 + att_area(hd, xmax) +
           kMaxLayers * sizeof(TokLayer);
}

int token_shape(uint32_t hd, uint32_t d, uint32_t ff) {
    const uint32_t td = row_threads(d), tf = row_threads(ff);
    const uint32_t cmd = (d / 8 + td - 1) / td, cmf = (ff / 8 + tf - 1) / tf;
    for (int i = 0; i < (int)(sizeof(kShapes) / sizeof(kShapes[0])); i++) {
        const TokShape& q = kShapes[i];
        if (q.hd == hd && q.td == td && q.cmd == cmd && q.tf == tf && q.cmf == cmf) return i;
    }
    return -1;
}

template <int I>
constexpr auto kernel_of() {
    return k_token_fast<(int)kShapes[I].hd, kShapes[I].td, kShapes[I].cmd, kShapes[I].tf, kShapes[I].cmf>;
}
void (*token_kernel(int i))(TokenArgs) {
    switch (i) {
        case 0: return kernel_of<0>();
        case 1: return kernel_of<1>();
        case 2: return kernel_of<2>();
        case 3: return kernel_of<3>();
        case 4: return kernel_of<4>();
        default: return nullptr;
    }
}

}  // namespace

bool token_fast_plan(TokenPlan* p, uint32_t n_layers, uint32_t d, uint32_t ff, uint32_t nh, uint32_t nkv,
                     uint32_t hd, uint32_t vocab, int n_sm, size_t smem_cap, uint32_t slot_only) {
    if ((hd != 64 && hd != 128) || nkv == 0 || nh % nkv || nh / nkv > 8 || d % 64 || ff % 64 || (nh * hd) % 64 ||
        n_sm <= 0 || n_layers == 0 || n_layers > kMaxLayers)
        return false;
    // a compiled shape class (O rows have the length d)
    if (nh * hd != d || token_shape(hd, d, ff) < 0) return false;
    // a phase's warp partials fit, and its per-row epilogue operands (bias,
    // residual) are one per consumer thread
    const uint32_t G = (uint32_t)n_sm;
    const struct { uint32_t rows, k, nmat; } ph[5] = {
        {(nh + 2 * nkv) * hd, d, 1}, {d, nh * hd, 1}, {ff, d, 2}, {d, ff, 1}, {vocab, d, 1}};
    for (const auto& q : ph)
        if (q.nmat * ((q.rows + G - 1) / G) * (row_threads(q.k) / 32) > kPart) return false;
    if ((ph[0].rows + G - 1) / G > kConsumers || (d + G - 1) / G > kConsumers || d > kMaxNorm * kConsumers)
        return false;
    // Ring slots: the largest ring of at least 4 slots that fits, among slot
    // sizes that hold whole passes of d-long rows (the QKV, O, gate/up and
    // head tiles); ties: larger slots, fewer tiles per phase. Other sizes
    // only when no such slot fits.
    const uint32_t unit = (kConsumers / row_threads(d)) * d * 2;
    bool found = false;
    for (int pass = 0; pass < 2 && !found; pass++) {
        for (uint32_t slot = pass == 0 ? unit : 16384; slot <= 65536; slot += pass == 0 ? unit : 1024) {
            if (slot < 16384 || slot % 16) continue;
            // a slot holds at least one row of every matrix (one of each of the gate/up pair)
            if (slot < 4 * d || slot < 2 * ff || slot < 2 * nh * hd || (slot_only && slot != slot_only)) continue;
            for (uint32_t nslot = 4; nslot <= 12; nslot++) {
                const size_t need = (size_t)nslot * slot + fixed_smem(d, ff, nh, hd, nslot);
                if (need > smem_cap) break;
                const uint64_t ring = (uint64_t)nslot * slot, best = (uint64_t)p->nslot * p->slot_bytes;
                if (!found || ring > best || (ring == best && nslot < p->nslot)) {
                    p->grid = (uint32_t)n_sm;
                    p->shape = token_shape(hd, d, ff);
                    p->slot_bytes = slot;
                    p->nslot = nslot;
                    p->smem = need;
                    found = true;
                }
            }
        }
    }
    return found;
}

bool token_fast_resident(const TokenPlan& p) {
    int per_sm = 0;
    auto k = token_kernel(p.shape);
    if (!k) return false;
    const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, p.smem);
    return e == cudaSuccess && per_sm >= 1;
}

cudaError_t token_fast_set_smem_limits(int optin) {
    for (int i = 0; token_kernel(i); i++) {
        const cudaError_t e = cudaFuncSetAttribute(token_kernel(i), cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_token_fast(const TokenPlan& p, const TokenArgs& a, cudaStream_t st) {
    auto k = token_kernel(p.shape);
    if (!p.grid || !k || a.nslot != p.nslot || a.slot_bytes != p.slot_bytes) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, a);
}

}  // namespace hs
