// Batch-1 token-loop kernels for sm_100a.
//
// Numerics are the reference's, operation for operation (hotseat
// crates/hs-engine/src/model.rs:240-327 and math.rs): every dot product is
// eight strided lanes acc[l] += w[8j+l]*x[8j+l] accumulated in order, folded as
// ((a0+a1)+(a2+a3))+((a4+a5)+(a6+a7)); no FMA anywhere. The GPU therefore
// produces the same bits as the CPU reference for the same weights, which is
// what lets a sequence move between the two.
//
// Performance shape (HBM-bound decode): each GEMV CTA owns a contiguous row
// range, TMA-loads its weight rows (128B-swizzled 64-column slabs) into shared
// memory *before* griddepcontrol.wait, so the weight stream of kernel k+1
// overlaps the tail of kernel k under programmatic dependent launch; after the
// wait it reads the activation and runs the fixed-order lanes out of shared
// memory, one (row, lane-group) per thread.
#include <cfloat>

#include "common.h"
#include "kernels.h"

namespace hs {
namespace {

__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) { return *(const volatile uint32_t*)p; }

// L consecutive f16 weights of one row (one per dot lane), widened to f32.
template <int L>
__device__ __forceinline__ void load_w(const uint8_t* p, float* w) {
    if (L == 1) {
        w[0] = h2f(*reinterpret_cast<const uint16_t*>(p));
    } else if (L == 2) {
        const uint32_t v = *reinterpret_cast<const uint32_t*>(p);
        w[0] = h2f((uint16_t)v);
        w[1] = h2f((uint16_t)(v >> 16));
    } else if (L == 4) {
        const uint2 v = *reinterpret_cast<const uint2*>(p);
        w[0] = h2f((uint16_t)v.x);
        w[1] = h2f((uint16_t)(v.x >> 16));
        w[2] = h2f((uint16_t)v.y);
        w[3] = h2f((uint16_t)(v.y >> 16));
    } else {
        const uint4 v = *reinterpret_cast<const uint4*>(p);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            w[2 * i] = h2f((uint16_t)u[i]);
            w[2 * i + 1] = h2f((uint16_t)(u[i] >> 16));
        }
    }
}

// Fold this thread's L lanes with its row-mates' (8/L consecutive lanes of
// the warp) into the reference's fold tree (math.rs:89-93). IEEE addition is
// commutative, so each partner computing b+a instead of a+b is the same value.
template <int L>
__device__ __forceinline__ float fold_lanes(const float* a) {
    const unsigned full = 0xffffffffu;
    float v;
    if (L == 8) {
        v = __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3])),
                      __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7])));
    } else if (L == 4) {
        v = __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3]));
        v = __fadd_rn(v, __shfl_xor_sync(full, v, 1));
    } else if (L == 2) {
        v = __fadd_rn(a[0], a[1]);
        v = __fadd_rn(v, __shfl_xor_sync(full, v, 1));
        v = __fadd_rn(v, __shfl_xor_sync(full, v, 2));
    } else {
        v = a[0];
        v = __fadd_rn(v, __shfl_xor_sync(full, v, 1));
        v = __fadd_rn(v, __shfl_xor_sync(full, v, 2));
        v = __fadd_rn(v, __shfl_xor_sync(full, v, 4));
    }
    return v;
}

// ------------------------------------------------------------------ GEMV
// y[r] = fold8(W[r] . x) for the CTA's rows, with the prologue/epilogue that
// model.rs fuses around each matvec: rmsnorm (math.rs:200-207) of the
// residual stream (or of the embedding row, model.rs:247-250) on the way in;
// bias (model.rs:255-257), residual add (308-310, 319-321) or SiLU gate
// (315-317) on the way out.
//
// Shared memory: [nst weight stages][xs: n f32][gs: n f32 norm gain]
// [xe: n f16 embedding row][outs: 2*rt][bias_s: rt][red: 32][bars: nst+1].
template <int OUT, int L>
__global__ void __launch_bounds__(512) k_gemv(const __grid_constant__ CUtensorMap tm0,
                                              const __grid_constant__ CUtensorMap tm1, const GemvArgs a,
                                              const int in_mode) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    // Align by offsetting the shared array itself, so every access below
    // stays a shared-space access.
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    constexpr int NMAT = OUT == OUT_SILU ? 2 : 1;
    const uint32_t n = a.n;
    const uint32_t kslabs = n / 64;
    const uint32_t mat_bytes = kslabs * a.slab_stride;
    const uint32_t stage_bytes = NMAT * mat_bytes;
    uint8_t* stages = smem;
    float* xs = reinterpret_cast<float*>(smem + a.nst * stage_bytes);
    float* gs = xs + n;
    uint16_t* xe = reinterpret_cast<uint16_t*>(gs + n);
    float* outs = reinterpret_cast<float*>(xe + n);
    float* bias_s = outs + 2 * a.rt;
    float* red = bias_s + a.rt;
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + 32 + ((a.rt & 1) ? 1 : 0));
    uint64_t* xbar = bars + a.nst;
    const uint32_t tid = threadIdx.x;
    const KTrace tr(a.trace, a.trace_slot);
    tr.enter();

    uint32_t r0, r1;
    split_range(a.rows, gridDim.x, blockIdx.x, &r0, &r1);
    const uint32_t mine = r1 - r0;
    const uint32_t ntiles = (mine + a.rt - 1) / a.rt;
    const uint32_t tx_bytes = NMAT * kslabs * a.rt * 128;

    if (tid == 0) {
        for (uint32_t s = 0; s <= a.nst; s++) mbar_init(&bars[s], 1);
        mbar_init_fence();
    }
    __syncthreads();
    auto issue = [&](uint32_t t) {
        uint32_t s = t % a.nst;
        uint8_t* st = stages + s * stage_bytes;
        mbar_expect_tx(&bars[s], tx_bytes);
        int y = (int)(r0 + t * a.rt);
        for (int m = 0; m < NMAT; m++)
            for (uint32_t k = 0; k < kslabs; k++)
                tma_load_2d(st + m * mat_bytes + k * a.slab_stride, m ? &tm1 : &tm0, (int)(k * 64), y, &bars[s]);
    };
    const uint32_t npre = ntiles < a.nst ? ntiles : a.nst;
    // Everything constant is fetched before waiting on the previous kernel:
    // the weight tiles, the norm gain, the first tile's bias.
    if (tid == 0)
        for (uint32_t t = 0; t < npre; t++) issue(t);
    if (in_mode != IN_PLAIN) {
        const float4* g4 = reinterpret_cast<const float4*>(a.norm_g);
        float4* s4 = reinterpret_cast<float4*>(gs);
#pragma unroll 4
        for (uint32_t i = tid; i < n / 4; i += blockDim.x) s4[i] = g4[i];
    }
    if (OUT == OUT_STORE && a.bias && tid < a.rt && tid < mine) bias_s[tid] = a.bias[r0 + tid];
    // `active` and `token` are set before the graph launch (by the host or the
    // previous step's commit kernel) and stay fixed during it.
    DevCtl* ctl = a.ctl;
    bool run = ld_volatile(&ctl->active) != 0;
    uint32_t token = 0;
    if (run && in_mode == IN_EMBED_NORM) {
        token = ld_volatile(&ctl->token);
        if (token >= ctl->vocab) {
            if (tid == 0 && blockIdx.x == 0) atomicOr(&ctl->err, ERR_TOKEN);
            run = false;
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    tr.waited();
    if (!run) {
        // Never leave with bulk copies in flight into this CTA's shared memory.
        for (uint32_t t = 0; t < npre; t++) mbar_wait_bounded(&bars[t], 0);
        return;
    }

    // ---- activation: one bulk copy (it was just written; it is in L2)
    if (tid == 0) {
        if (in_mode == IN_EMBED_NORM) {
            mbar_expect_tx(xbar, n * 2);
            bulk_load_1d(xe, a.embd + (size_t)token * n, n * 2, xbar);
        } else {
            mbar_expect_tx(xbar, n * 4);
            bulk_load_1d(xs, a.src, n * 4, xbar);
        }
    }
    if (!mbar_wait_bounded(xbar, 0)) {
        if (tid == 0) atomicOr(&ctl->err, ERR_TIMEOUT);
        for (uint32_t t = 0; t < npre; t++) mbar_wait_bounded(&bars[t], 0);
        return;
    }
    tr.mark(1);
    if (in_mode == IN_EMBED_NORM) {
        for (uint32_t i = tid; i < n; i += blockDim.x) {
            const float v = h2f(xe[i]);
            xs[i] = v;
            if (blockIdx.x == 0) a.x_out[i] = v;
        }
        __syncthreads();
    }
    if (in_mode != IN_PLAIN) {
        // rmsnorm: ss = dot_f32(x, x) in the 8-lane shape; scale = 1/sqrt(ss/n + eps);
        // out[i] = x[i] * scale * g[i].
        if (tid < 32) {
            // Thread t < 4 runs lanes 2t and 2t+1 of the 8-lane sum of squares.
            float a0 = 0.0f, a1 = 0.0f;
            if (tid < 4) {
                const uint32_t nj = n / 8;
                const uint64_t* x2 = reinterpret_cast<const uint64_t*>(xs) + tid;
#pragma unroll 16
                for (uint32_t j = 0; j < nj; j++) {
                    const uint64_t v = x2[4 * j];
                    mul_add_pair(&a0, &a1, v, v);
                }
            }
            float v = __fadd_rn(a0, a1);
            v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
            v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
            if (tid == 0) red[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(v, (float)n), a.eps)));
        }
        __syncthreads();
        const float scale = red[0];
        for (uint32_t i = tid; i < n; i += blockDim.x) xs[i] = __fmul_rn(__fmul_rn(xs[i], scale), gs[i]);
        __syncthreads();
    }
    tr.mark(2);

    // ---- fixed-order lanes out of shared memory
    constexpr uint32_t TPR = 8 / L;  // threads per row
    const uint32_t vr = tid / TPR, g = tid % TPR;
    const bool lane_active = vr < NMAT * a.rt;
    const uint32_t m = lane_active ? vr / a.rt : 0, r = lane_active ? vr % a.rt : 0;
    for (uint32_t t = 0; t < ntiles; t++) {
        const uint32_t s = t % a.nst;
        if (!mbar_wait_bounded(&bars[s], (t / a.nst) & 1)) {
            if (tid == 0) atomicOr(&ctl->err, ERR_TIMEOUT);
            return;
        }
        if (t == 0) tr.mark(3);
        float acc[L];
#pragma unroll
        for (int i = 0; i < L; i++) acc[i] = 0.0f;
        if (lane_active) {
            const uint8_t* base = stages + s * stage_bytes + m * mat_bytes + r * 128;
            const uint32_t sw = r & 7;
            if (L == 1) {
#pragma unroll 2
                for (uint32_t k = 0; k < kslabs; k++) {
                    const uint8_t* sb = base + k * a.slab_stride;
                    const float* xk = xs + k * 64 + g;
#pragma unroll
                    for (uint32_t c = 0; c < 8; c++) {
                        float w[1];
                        load_w<1>(sb + (((c ^ sw) << 4) | (g * 2)), w);
                        acc[0] = __fadd_rn(acc[0], __fmul_rn(w[0], xk[c * 8]));
                    }
                }
            } else {
#pragma unroll 2
                for (uint32_t k = 0; k < kslabs; k++) {
                    const uint8_t* sb = base + k * a.slab_stride;
                    const uint64_t* xk = reinterpret_cast<const uint64_t*>(xs + k * 64 + g * L);
#pragma unroll
                    for (uint32_t c = 0; c < 8; c++) {
                        float w[L];
                        load_w<L>(sb + (((c ^ sw) << 4) | (g * L * 2)), w);
#pragma unroll
                        for (int i = 0; i < L / 2; i++)
                            mul_add_pair(&acc[2 * i], &acc[2 * i + 1], pack2(w[2 * i], w[2 * i + 1]), xk[c * 4 + i]);
                    }
                }
            }
        }
        const float v = fold_lanes<L>(acc);
        if (t == 0) tr.mark(4);
        const uint32_t rr = t * a.rt + r;  // row index inside this CTA's range
        if (OUT == OUT_SILU) {
            if (lane_active && g == 0) outs[m * a.rt + r] = v;
            __syncthreads();
            if (tid < a.rt && t * a.rt + tid < mine) {
                const float gv = outs[tid], uv = outs[a.rt + tid];
                a.dst[r0 + t * a.rt + tid] = __fmul_rn(ref_silu(gv), uv);
            }
        } else if (lane_active && g == 0 && rr < mine) {
            const uint32_t row = r0 + rr;
            if (OUT == OUT_STORE) {
                if (a.bias) a.dst[row] = __fadd_rn(v, t == 0 ? bias_s[r] : a.bias[row]);
                else a.dst[row] = v;
            } else {
                a.dst[row] = __fadd_rn(a.dst[row], v);
            }
        }
        __syncthreads();
        if (tid == 0 && t + a.nst < ntiles) {
            fence_proxy_async_smem();
            issue(t + a.nst);
        }
    }
    tr.exit();
}

// ------------------------------------------------------------ attention
// One CTA per query head (model.rs:259-305): RoPE on q and k from the cached
// tables (rope_apply, model.rs:365-373); the head group's first CTA appends
// k, v at `pos` (model.rs:268-275) and marks the touched pages in the dirty
// bitmap; scores p in [0, pos] = dot_f32(q, k_p) * (1/sqrt(hd)); softmax with
// exp_f32, sequential sum and 1/sum (math.rs:210-226); out = sum_p sc[p]*v_p in
// position order (axpy, math.rs:185-190).
//
// Rows p < pos were written by earlier tokens, so up to kAttnPre of them are
// copied into shared memory before griddepcontrol.wait, overlapping the QKV
// kernel; longer contexts stream the remainder in chunks after the wait.
template <int HD>
struct AttnShape {
    static constexpr int RS = HD + 4;          // padded row stride (floats): conflict-free row reads
    static constexpr int PRE = 12288 / HD;     // rows of K and of V prefetched (192 at hd 64)
    static constexpr int CH = 4096 / HD;       // rows per streamed chunk beyond PRE
};

template <int HD>
__global__ void __launch_bounds__(256) k_attention(const AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    using S = AttnShape<HD>;
    constexpr int RS = S::RS, PRE = S::PRE, CH = S::CH, HALF = HD / 2;
    float* q = sm;
    float* kc = q + HD;
    float* vc = kc + HD;
    float* red = vc + HD;
    float* kb = red + 64;       // [PRE][RS]
    float* vb = kb + PRE * RS;  // [PRE][RS]
    float* cb = vb + PRE * RS;  // [CH][RS]
    // [max_ctx] scores: shared memory, or this head's row of a global buffer
    // when max_ctx scores do not fit next to the K/V staging.
    float* sc = a.sc_global ? a.sc_global + (size_t)blockIdx.x * a.max_ctx : cb + CH * RS;
    const uint32_t tid = threadIdx.x;
    const KTrace tr(a.trace, a.trace_slot);
    tr.enter();
    DevCtl* ctl = a.ctl;
    const uint32_t h = blockIdx.x, groups = a.nh / a.nkv, kvh = h / groups;
    const uint64_t plane = (uint64_t)a.max_ctx * a.nkv * HD;
    const uint64_t lbase = (uint64_t)a.layer * 2 * plane;
    auto row_off = [&](uint32_t p, uint32_t is_v) -> uint64_t {
        uint64_t within = a.layout == 0 ? ((uint64_t)p * a.nkv + kvh) * HD : ((uint64_t)kvh * a.max_ctx + p) * HD;
        return lbase + (is_v ? plane : 0) + within;
    };
    // `active` and `pos` were set before this graph launch began (by the host
    // or by the previous step's commit kernel), so they are stable here.
    const bool run = ld_volatile(&ctl->active) != 0;
    const uint32_t pos = ld_volatile(&ctl->pos);
    const bool pos_ok = pos < a.max_ctx;
    const uint32_t npre = run && pos_ok ? min(pos, (uint32_t)PRE) : 0;
    for (uint32_t idx = tid; idx < npre * (HD / 4); idx += blockDim.x) {
        const uint32_t p = idx / (HD / 4), c4 = idx % (HD / 4);
        cp_async16(kb + p * RS + 4 * c4, a.kv + row_off(p, 0) + 4 * c4);
        cp_async16(vb + p * RS + 4 * c4, a.kv + row_off(p, 1) + 4 * c4);
    }
    pdl_launch_dependents();
    pdl_wait();
    tr.waited();
    if (!run || !pos_ok) {
        cp_async_wait_all();
        if (run && tid == 0 && blockIdx.x == 0) atomicOr(&ctl->err, ERR_POS);
        return;
    }
    if (tid < HD) {
        q[tid] = a.qkv[h * HD + tid];
        kc[tid] = a.qkv[a.nh * HD + kvh * HD + tid];
        vc[tid] = a.qkv[(a.nh + a.nkv) * HD + kvh * HD + tid];
    }
    __syncthreads();
    if (tid < HALF) {
        const float c = a.rope_cos[(size_t)pos * HALF + tid], s = a.rope_sin[(size_t)pos * HALF + tid];
        float x0 = q[tid], x1 = q[tid + HALF];
        q[tid] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        q[tid + HALF] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        x0 = kc[tid];
        x1 = kc[tid + HALF];
        kc[tid] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        kc[tid + HALF] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
    __syncthreads();
    if (h % groups == 0) {
        if (tid < HD) {
            a.kv[row_off(pos, 0) + tid] = kc[tid];
            a.kv[row_off(pos, 1) + tid] = vc[tid];
        }
        // Data first, then the mark: a harvester that sees the page dirty
        // also sees the bytes that dirtied it.
        __syncthreads();
        if (tid < 2 && ld_volatile(a.tracking)) {
            __threadfence();
            const uint64_t off = row_off(pos, tid) * 4, last = off + HD * 4 - 1;
            for (uint64_t pg = off >> a.page_shift; pg <= (last >> a.page_shift); pg++)
                atomicOr(reinterpret_cast<unsigned long long*>(&a.dirty[pg >> 6]), 1ull << (pg & 63));
        }
    }
    tr.mark(1);
    cp_async_wait_all();
    __syncthreads();
    tr.mark(2);

    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
    const uint32_t n = pos + 1;
    auto score = [&](const float* kr) -> float {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < HD / 8; j++)
#pragma unroll
            for (int l = 0; l < 8; l++) acc[l] = __fadd_rn(acc[l], __fmul_rn(q[8 * j + l], kr[8 * j + l]));
        const float d = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3])),
                                  __fadd_rn(__fadd_rn(acc[4], acc[5]), __fadd_rn(acc[6], acc[7])));
        return __fmul_rn(d, scale);
    };
    // scores: prefetched rows, the current row, then any streamed remainder
    for (uint32_t p = tid; p < npre; p += blockDim.x) sc[p] = score(kb + p * RS);
    if (tid == 0) sc[pos] = score(kc);
    for (uint32_t c0 = npre; c0 < pos; c0 += CH) {
        const uint32_t cnt = min((uint32_t)CH, pos - c0);
        __syncthreads();
        for (uint32_t idx = tid; idx < cnt * (HD / 4); idx += blockDim.x) {
            const uint32_t rr = idx / (HD / 4), c4 = idx % (HD / 4);
            *reinterpret_cast<float4*>(cb + rr * RS + 4 * c4) =
                *reinterpret_cast<const float4*>(a.kv + row_off(c0 + rr, 0) + 4 * c4);
        }
        __syncthreads();
        if (tid < cnt) sc[c0 + tid] = score(cb + tid * RS);
    }
    __syncthreads();
    // softmax: max (order-free), exp, sequential sum, scale by 1/sum
    float mx = __int_as_float(0xff800000);
    for (uint32_t p = tid; p < n; p += blockDim.x) mx = fmaxf(mx, sc[p]);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (uint32_t w = 1; w < blockDim.x / 32; w++) mx = fmaxf(mx, red[w]);
    for (uint32_t p = tid; p < n; p += blockDim.x) sc[p] = ref_exp(__fsub_rn(sc[p], mx));
    __syncthreads();
    if (tid == 0) {
        float sum = 0.0f;
#pragma unroll 8
        for (uint32_t p = 0; p < n; p++) sum = __fadd_rn(sum, sc[p]);
        red[33] = __fdiv_rn(1.0f, sum);
    }
    __syncthreads();
    const float inv = red[33];
    for (uint32_t p = tid; p < n; p += blockDim.x) sc[p] = __fmul_rn(sc[p], inv);
    __syncthreads();
    tr.mark(3);
    // out[d] = sum over p, in order, of sc[p] * v_p[d]
    float out = 0.0f;
    if (tid < HD) {
#pragma unroll 8
        for (uint32_t p = 0; p < npre; p++) out = __fadd_rn(out, __fmul_rn(sc[p], vb[p * RS + tid]));
    }
    for (uint32_t c0 = npre; c0 < pos; c0 += CH) {
        const uint32_t cnt = min((uint32_t)CH, pos - c0);
        __syncthreads();
        for (uint32_t idx = tid; idx < cnt * (HD / 4); idx += blockDim.x) {
            const uint32_t rr = idx / (HD / 4), c4 = idx % (HD / 4);
            *reinterpret_cast<float4*>(cb + rr * RS + 4 * c4) =
                *reinterpret_cast<const float4*>(a.kv + row_off(c0 + rr, 1) + 4 * c4);
        }
        __syncthreads();
        if (tid < HD)
#pragma unroll 8
            for (uint32_t t = 0; t < cnt; t++) out = __fadd_rn(out, __fmul_rn(sc[c0 + t], cb[t * RS + tid]));
    }
    if (tid < HD) {
        out = __fadd_rn(out, __fmul_rn(sc[pos], vc[tid]));
        a.att[h * HD + tid] = out;
    }
    tr.exit();
}

// -------------------------------------------------------------- sampler
// Stage 1 (k_sample_cand): each CTA takes 1024 logits (8 warps x 128),
// applies the repetition penalty to the history tokens in its slice
// (sampler.rs:103-111: a token is penalised once per occurrence, in history
// order), then either finds its first maximum (greedy, sampler.rs:177-187)
// or orders its slice under cmp_desc and keeps the best kmax keys.
// Stage 2 (k_sample_final): merges the per-CTA lists into the global top-k
// (a merge tree of co-rank searches), computes the temperature weights with
// exp_f32 one per thread, and runs the reference's serial tail on one
// thread: the sums in order, nucleus cut, one next_f32 draw
// (sampler.rs:134-166); in sequence mode it then commits the step exactly
// as seq.rs:273-312 does.
__device__ __forceinline__ bool seq_needs_sample(const DevCtl* c) {
    if (c->mode == 1) return true;
    return c->active && c->filled + 1 == c->n_tokens;
}

// Copy the control block into shared memory with one parallel batch of loads.
// Nothing launched in the same step writes it before the commit kernel, so
// both sampler kernels take this snapshot before waiting on their predecessor.
__device__ __forceinline__ void load_ctl(DevCtl* dst, const DevCtl* src) {
    constexpr uint32_t words = sizeof(DevCtl) / 4;
    static_assert(sizeof(DevCtl) % 4 == 0, "DevCtl is copied as 32-bit words");
    if (threadIdx.x < words)
        reinterpret_cast<uint32_t*>(dst)[threadIdx.x] =
            __ldcg(reinterpret_cast<const unsigned int*>(src) + threadIdx.x);
}

// (value, index) "better" for greedy: larger value, then smaller index; an
// invalid index (0xffffffff) never wins and NaN never compares larger.
__device__ __forceinline__ bool arg_better(float v2, uint32_t i2, float v1, uint32_t i1) {
    if (i2 == 0xffffffffu) return false;
    if (i1 == 0xffffffffu) return true;
    return v2 > v1 || (v2 == v1 && i2 < i1);
}

__device__ __forceinline__ void warp_argbest(float* v, uint32_t* i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, *v, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, *i, o);
        if (arg_better(ov, oi, *v, *i)) {
            *v = ov;
            *i = oi;
        }
    }
}

// Ascending bitonic sort of 128 keys held as k[i] = element i*32 + lane.
__device__ __forceinline__ void warp_sort128(uint64_t k[4], int lane) {
#pragma unroll
    for (int size = 2; size <= 128; size <<= 1) {
#pragma unroll
        for (int j = size >> 1; j > 0; j >>= 1) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int e = i * 32 + lane;
                const bool up = (e & size) == 0;
                if (j >= 32) {
                    const int ii = i ^ (j >> 5);
                    if (ii > i) {
                        const uint64_t x = k[i], y = k[ii];
                        if ((x > y) == up) {
                            k[i] = y;
                            k[ii] = x;
                        }
                    }
                } else {
                    const uint64_t o = __shfl_xor_sync(0xffffffffu, k[i], j);
                    const bool lower = (e & j) == 0;
                    k[i] = (lower == up) ? (o < k[i] ? o : k[i]) : (o > k[i] ? o : k[i]);
                }
            }
        }
    }
}

// Number of keys in sorted list[0..len) smaller than `key`.
// len must be a power of two; fixed step count, no data-dependent loop, so
// several searches interleave.
__device__ __forceinline__ uint32_t lower_bound_u64(const uint64_t* list, uint32_t len, uint64_t key) {
    uint32_t idx = 0;
#pragma unroll
    for (uint32_t step = 128; step > 0; step >>= 1)
        if (step <= len && idx + step <= len && list[idx + step - 1] < key) idx += step;
    return idx;
}

// Slot blockIdx.y of a batched launch: its logits, candidate lists, greedy
// entries, control block and history buffer.
__device__ __forceinline__ SampleArgs slot_args(const SampleArgs& a0) {
    SampleArgs a = a0;
    const uint32_t s = blockIdx.y;
    if (s) {
        a.logits += s * a0.logits_stride;
        a.cand += s * a0.cand_stride;
        a.argbuf += s * a0.n_cta;
        a.ctl += s;
    }
    if (a0.tok_tab) {
        a.tokens = a0.tok_tab[s];
        a.tokens_w = a0.tok_tab[s];
    }
    return a;
}

__global__ void __launch_bounds__(256) k_sample_cand(const SampleArgs a0) {
    const SampleArgs a = slot_args(a0);
    __shared__ uint64_t lists[8][128];
    __shared__ uint32_t win_cnt[kSampleSlice];
    __shared__ float bv_s[8];
    __shared__ uint32_t bi_s[8];
    __shared__ DevCtl cs;
    const uint32_t tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const KTrace tr(a.trace, a.trace_slot);
    tr.enter();
    load_ctl(&cs, a.ctl);
    __syncthreads();
    const DevCtl* c = &cs;
    // The history window is also fixed until the commit: count it now.
    const float pen = c->repeat_penalty;
    const uint64_t nt = c->n_tokens;
    const uint64_t nw = (pen != 1.0f && c->repeat_last_n > 0) ? (c->repeat_last_n < nt ? c->repeat_last_n : nt) : 0;
    const uint32_t cta_base = blockIdx.x * kSampleSlice;
    const bool need = seq_needs_sample(c);
    if (need && nw) {
        for (uint32_t i = tid; i < kSampleSlice; i += blockDim.x) win_cnt[i] = 0;
        __syncthreads();
        for (uint64_t i = nt - nw + tid; i < nt; i += blockDim.x) {
            const uint32_t t = __ldcg(a.tokens + i);
            if (t >= cta_base && t < cta_base + kSampleSlice) atomicAdd(&win_cnt[t - cta_base], 1u);
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    tr.waited();
    if (!need) return;
    __syncthreads();
    const uint32_t base = blockIdx.x * kSampleSlice + w * 128;
    float v[4];
    uint32_t e[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        e[i] = base + i * 32 + lane;
        v[i] = e[i] < a.vocab ? __ldcg(a.logits + e[i]) : 0.0f;
    }
    tr.mark(1);
    // Penalty: each slice token's occurrences in the history window were
    // counted above; apply the reference's update that many times. Every
    // occurrence applies the same operation to the same logit, so this is the
    // sequential loop of sampler.rs:105-110 with the loop order factored out.
    if (nw) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t times = win_cnt[e[i] - cta_base];
            while (times--) v[i] = v[i] > 0.0f ? __fdiv_rn(v[i], pen) : __fmul_rn(v[i], pen);
        }
    }
    if (c->temperature <= 0.0f) {
        float bv = 0.0f;
        uint32_t bi = 0xffffffffu;
#pragma unroll
        for (int i = 0; i < 4; i++)  // index order within the thread
            if (e[i] < a.vocab && !(v[i] != v[i]) && v[i] > __int_as_float(0xff800000) && arg_better(v[i], e[i], bv, bi)) {
                bv = v[i];
                bi = e[i];
            }
        warp_argbest(&bv, &bi);
        if (lane == 0) {
            bv_s[w] = bv;
            bi_s[w] = bi;
        }
        __syncthreads();
        if (tid == 0) {
            float fv = bv_s[0];
            uint32_t fi = bi_s[0];
            for (int k = 1; k < 8; k++)
                if (arg_better(bv_s[k], bi_s[k], fv, fi)) {
                    fv = bv_s[k];
                    fi = bi_s[k];
                }
            a.argbuf[blockIdx.x] = ((uint64_t)__float_as_uint(fv) << 32) | fi;
        }
        return;
    }
    tr.mark(2);
    uint64_t k[4];
#pragma unroll
    for (int i = 0; i < 4; i++) k[i] = e[i] < a.vocab ? cand_key(v[i], e[i]) : ~0ull - e[i];
    warp_sort128(k, (int)lane);
    tr.mark(3);
#pragma unroll
    for (int i = 0; i < 4; i++) lists[w][i * 32 + lane] = k[i];
    __syncthreads();
    // Rank-based merge of the 8 sorted lists: element j of list l has rank
    // j + (keys smaller than it in the other lists); keep ranks < kmax.
    const uint32_t J = a.kmax < 128 ? a.kmax : 128;
    for (uint32_t idx = tid; idx < 8 * J; idx += blockDim.x) {
        const uint32_t l = idx / J, j = idx % J;
        const uint64_t key = lists[l][j];
        uint32_t rank = j;
#pragma unroll
        for (uint32_t o = 0; o < 8; o++)
            if (o != l) rank += lower_bound_u64(lists[o], J, key);
        if (rank < a.kmax) a.cand[(size_t)blockIdx.x * a.kmax + rank] = key;
    }
    tr.exit();
}

// Candidate kernel for wide slices (a multiple of 256 logits per CTA, top
// keys kmax <= 64): the same output as k_sample_cand (the CTA's kmax best
// keys in key order) from an exact radix select instead of sorting. Each
// thread holds slice/256 keys; 8-bit digits of the 64-bit key, most
// significant first, narrow the prefix of the kmax-th smallest key until the
// boundary bin is taken whole; the selected keys (exactly kmax, keys are
// unique) are then ranked against each other.
//
// SORT (sort mode, any top_k): the CTA instead sorts its whole slice of keys
// (bitonic network in shared memory, padded to a power of two) and writes
// all `slice` of them in key order; k_sample_rank then finds each key's
// place among every slice's keys.
template <bool SORT>
__global__ void __launch_bounds__(256) k_sample_cand_wide(const SampleArgs a0) {
    const SampleArgs a = slot_args(a0);
    constexpr uint32_t PER = kMaxSlice / 256;
    __shared__ uint32_t win_cnt[kMaxSlice];
    __shared__ uint32_t hist[256];
    __shared__ uint64_t sel_keys[kMaxTopK];
    __shared__ uint32_t n_sel, sh_digit, sh_need;
    __shared__ float bv_s[8];
    __shared__ uint32_t bi_s[8];
    __shared__ DevCtl cs;
    const uint32_t tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const uint32_t slice = a.slice, per = slice / 256;
    const KTrace tr(a.trace, a.trace_slot);
    tr.enter();
    load_ctl(&cs, a.ctl);
    __syncthreads();
    const DevCtl* c = &cs;
    const float pen = c->repeat_penalty;
    const uint64_t nt = c->n_tokens;
    const uint64_t nw = (pen != 1.0f && c->repeat_last_n > 0) ? (c->repeat_last_n < nt ? c->repeat_last_n : nt) : 0;
    const uint32_t cta_base = blockIdx.x * slice;
    const bool need = seq_needs_sample(c);
    if (need && nw) {
        for (uint32_t i = tid; i < slice; i += blockDim.x) win_cnt[i] = 0;
        __syncthreads();
        for (uint64_t i = nt - nw + tid; i < nt; i += blockDim.x) {
            const uint32_t t = __ldcg(a.tokens + i);
            if (t >= cta_base && t < cta_base + slice) atomicAdd(&win_cnt[t - cta_base], 1u);
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    tr.waited();
    if (!need) return;
    __syncthreads();
    // Element j of thread t is id cta_base + j*256 + t (coalesced loads).
    float v[PER];
#pragma unroll
    for (uint32_t j = 0; j < PER; j++) {
        const uint32_t e = cta_base + j * 256 + tid;
        v[j] = (j < per && e < a.vocab) ? __ldcg(a.logits + e) : 0.0f;
        if (nw && j < per && e < a.vocab) {
            // sampler.rs:105-110, each occurrence in the window once
            uint32_t times = win_cnt[e - cta_base];
            while (times--) v[j] = v[j] > 0.0f ? __fdiv_rn(v[j], pen) : __fmul_rn(v[j], pen);
        }
    }
    if (c->temperature <= 0.0f) {
        float bv = 0.0f;
        uint32_t bi = 0xffffffffu;
#pragma unroll
        for (uint32_t j = 0; j < PER; j++) {
            const uint32_t e = cta_base + j * 256 + tid;
            if (j < per && e < a.vocab && !(v[j] != v[j]) && v[j] > __int_as_float(0xff800000) &&
                arg_better(v[j], e, bv, bi)) {
                bv = v[j];
                bi = e;
            }
        }
        warp_argbest(&bv, &bi);
        if (lane == 0) {
            bv_s[w] = bv;
            bi_s[w] = bi;
        }
        __syncthreads();
        if (tid == 0) {
            float fv = bv_s[0];
            uint32_t fi = bi_s[0];
            for (int k = 1; k < 8; k++)
                if (arg_better(bv_s[k], bi_s[k], fv, fi)) {
                    fv = bv_s[k];
                    fi = bi_s[k];
                }
            a.argbuf[blockIdx.x] = ((uint64_t)__float_as_uint(fv) << 32) | fi;
        }
        return;
    }
    // Keys ascend best-first; ids past the vocabulary (or past the slice) get
    // keys above every real key, as in k_sample_cand.
    uint64_t key[PER];
#pragma unroll
    for (uint32_t j = 0; j < PER; j++) {
        const uint32_t e = cta_base + j * 256 + tid;
        key[j] = (j < per && e < a.vocab) ? cand_key(v[j], e) : ~0ull - e;
    }
    if (SORT) {
        extern __shared__ uint64_t sk[];  // [n2]
        uint32_t n2 = 256;
        while (n2 < slice) n2 <<= 1;
#pragma unroll
        for (uint32_t j = 0; j < PER; j++)
            if (j < per) sk[j * 256 + tid] = key[j];
        for (uint32_t i = slice + tid; i < n2; i += 256) sk[i] = ~0ull;
        __syncthreads();
        for (uint32_t size = 2; size <= n2; size <<= 1) {
            for (uint32_t j = size >> 1; j > 0; j >>= 1) {
                for (uint32_t i = tid; i < n2 / 2; i += 256) {
                    const uint32_t lo = ((i & ~(j - 1)) << 1) | (i & (j - 1)), hi = lo + j;
                    const bool up = (lo & size) == 0;
                    const uint64_t x = sk[lo], y = sk[hi];
                    if ((x > y) == up) {
                        sk[lo] = y;
                        sk[hi] = x;
                    }
                }
                __syncthreads();
            }
        }
        for (uint32_t i = tid; i < slice; i += 256) a.cand[(size_t)blockIdx.x * slice + i] = sk[i];
        tr.exit();
        return;
    }
    const uint32_t K = a.kmax;
    uint64_t prefix = 0, mask = 0;  // bits of the K-th key fixed so far
    uint32_t needk = K;              // keys still to take at or below the prefix
    for (int shift = 56; shift >= 0; shift -= 8) {
        hist[tid] = 0;
        __syncthreads();
#pragma unroll
        for (uint32_t j = 0; j < PER; j++)
            if (j < per && (key[j] & mask) == prefix) atomicAdd(&hist[(key[j] >> shift) & 255], 1u);
        __syncthreads();
        if (w == 0) {
            // Inclusive scan over the 256 bins, 8 per lane, lanes in order.
            uint32_t h8[8], s = 0;
#pragma unroll
            for (int q = 0; q < 8; q++) {
                h8[q] = hist[lane * 8 + q];
                s += h8[q];
            }
            uint32_t incl = s;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= (uint32_t)o) incl += y;
            }
            uint32_t run = incl - s;
#pragma unroll
            for (int q = 0; q < 8; q++) {
                if (run < needk && run + h8[q] >= needk) {
                    sh_digit = lane * 8 + q;
                    sh_need = needk - run;  // keys to take from the boundary bin
                }
                run += h8[q];
            }
        }
        __syncthreads();
        const uint32_t d = sh_digit;
        prefix |= (uint64_t)d << shift;
        mask |= 255ull << shift;
        const bool whole = sh_need == hist[d];
        needk = sh_need;
        __syncthreads();
        if (whole) break;
    }
    // Selected: keys below the prefix's bin, plus the whole boundary bin.
    if (tid == 0) n_sel = 0;
    __syncthreads();
#pragma unroll
    for (uint32_t j = 0; j < PER; j++) {
        if (j >= per) continue;
        const uint64_t kk = key[j];
        if ((kk & mask) < prefix || (kk & mask) == prefix) {
            const uint32_t at = atomicAdd(&n_sel, 1u);
            if (at < kMaxTopK) sel_keys[at] = kk;
        }
    }
    __syncthreads();
    const uint32_t ns = n_sel < K ? n_sel : K;
    for (uint32_t i = tid; i < ns; i += blockDim.x) {
        const uint64_t kk = sel_keys[i];
        uint32_t rank = 0;
        for (uint32_t q = 0; q < ns; q++) rank += sel_keys[q] < kk ? 1u : 0u;
        a.cand[(size_t)blockIdx.x * K + rank] = kk;
    }
    tr.exit();
}

// Sort mode, stage 2: the global top-k of each slot in key order. Thread
// (list l, index j) takes key x = list_l[j] and counts the keys below it in
// every other list (binary search); keys are unique, so j + those counts is
// x's rank among all keys, and the keys of rank < k land in wkeys[rank].
// Only the first min(k, slice) keys of a list can be in the top k, and every
// key below a top-k key is itself within those prefixes, so the searches run
// over the prefixes alone.
__device__ __forceinline__ uint32_t count_below(const uint64_t* list, uint32_t n, uint64_t key) {
    uint32_t lo = 0, hi = n;
    while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        if (__ldcg(list + mid) < key)
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo;
}

__global__ void __launch_bounds__(256) k_sample_rank(const SampleArgs a0) {
    const SampleArgs a = slot_args(a0);
    pdl_launch_dependents();
    pdl_wait();
    const DevCtl* c = a.ctl;
    const uint32_t mode = __ldcg(&c->mode), active = __ldcg(&c->active);
    const uint64_t filled = __ldcg((const unsigned long long*)&c->filled);
    const uint64_t n_tokens = __ldcg((const unsigned long long*)&c->n_tokens);
    const bool need = mode == 1 || (active && filled + 1 == n_tokens);
    if (!need || !(__ldcg(&c->temperature) > 0.0f)) return;
    const uint32_t top_k = __ldcg(&c->top_k);
    const uint32_t k = top_k == 0 ? a.vocab : min(top_k, a.vocab);
    const uint32_t slice = a.kmax, L = min(k, slice);
    const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t l = idx / slice, j = idx % slice;
    if (l >= a.n_cta || j >= L) return;
    const uint64_t key = __ldcg(a.cand + (size_t)l * slice + j);
    uint32_t rank = j;
    for (uint32_t o = 0; o < a.n_cta; o++)
        if (o != l) rank += count_below(a.cand + (size_t)o * slice, L, key);
    if (rank < k) a.wkeys[(size_t)blockIdx.y * a.wide_stride + rank] = key;
}

constexpr uint32_t kFinalThreads = 256;

__global__ void __launch_bounds__(kFinalThreads) k_sample_final(const SampleArgs a0) {
    const SampleArgs a = slot_args(a0);
    extern __shared__ uint64_t sel_lists[];  // [n_sel][kmax]
    __shared__ uint64_t heads[256];
    __shared__ uint32_t sel[64];
    __shared__ uint64_t merged[1024];
    __shared__ float pk[1024];
    __shared__ float bv_s[8];
    __shared__ uint32_t bi_s[8];
    __shared__ uint32_t tok_s;
    __shared__ DevCtl cs;
    const uint32_t tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const KTrace tr(a.trace, a.trace_slot + 1);
    tr.enter();
    load_ctl(&cs, a.ctl);
    pdl_launch_dependents();
    pdl_wait();
    tr.waited();
    __syncthreads();
    DevCtl* c = &cs;
    const bool seq = c->mode == 0;
    if (seq && !c->active) return;
    const bool need = seq_needs_sample(c);
    if (tid == 0) tok_s = 0;
    if (need && c->temperature <= 0.0f) {
        float bv = 0.0f;
        uint32_t bi = 0xffffffffu;
        if (tid < a.n_cta) {
            const uint64_t ent = a.argbuf[tid];
            bv = __uint_as_float((uint32_t)(ent >> 32));
            bi = (uint32_t)ent;
        }
        warp_argbest(&bv, &bi);
        if (lane == 0) {
            bv_s[w] = bv;
            bi_s[w] = bi;
        }
        __syncthreads();
        if (tid == 0) {
            float fv = bv_s[0];
            uint32_t fi = bi_s[0];
            for (uint32_t k = 1; k < kFinalThreads / 32; k++)
                if (arg_better(bv_s[k], bi_s[k], fv, fi)) {
                    fv = bv_s[k];
                    fi = bi_s[k];
                }
            tok_s = fi == 0xffffffffu ? 0u : fi;
        }
    } else if (need && sample_sort_mode(a.n_cta, a.kmax)) {
        // Sort mode: the slot's top-k keys are in wkeys in order. The
        // reference's three passes (sampler.rs:135-166: the sum of the
        // weights, the nucleus scan `acc += p; if acc >= target`, the sum of
        // the kept prefix, and the pick scan `acc += p; if r < acc`) all
        // accumulate the same weights in the same order from zero, so one
        // serial pass that stores every running sum S_i answers them all:
        // sum = S_{k-1}; cut = 1 + the first i with S_i >= top_p * sum; the
        // kept prefix sums to S_{cut-1}; the pick is the first i < cut with
        // r < S_i. The weights are computed in parallel, the running sums on
        // one thread, 1024 at a time through shared memory while the other
        // warps stage the next 1024.
        const uint32_t k = c->top_k == 0 ? a.vocab : min(c->top_k, a.vocab);
        const uint64_t* keys = a.wkeys + (size_t)blockIdx.y * a.wide_stride;
        float* ps = a.wps + (size_t)blockIdx.y * a.wide_stride;
        float* pb = reinterpret_cast<float*>(merged);  // two 1024-float buffers
        __shared__ float run_s, cmp_s;
        __shared__ uint32_t first_s;
        {
            const float inv_t = __fdiv_rn(1.0f, c->temperature);
            const float mx = key_value(__ldcg(keys));
            for (uint32_t i = tid; i < k; i += blockDim.x)
                ps[i] = ref_exp(__fmul_rn(__fsub_rn(key_value(__ldcg(keys + i)), mx), inv_t));
        }
        __syncthreads();
        const uint32_t nch = (k + 1023) / 1024;
        for (uint32_t i = tid; i < min(k, 1024u); i += blockDim.x) pb[i] = __ldcg(ps + i);
        float run = 0.0f;
        __syncthreads();
        for (uint32_t ch = 0; ch < nch; ch++) {
            float* cur = pb + (ch & 1) * 1024;
            const uint32_t base = ch * 1024, cnt = min(1024u, k - base);
            if (tid == 0) {
                for (uint32_t t = 0; t < cnt; t++) {
                    run = __fadd_rn(run, cur[t]);
                    cur[t] = run;
                }
            } else if (tid >= 32 && ch + 1 < nch) {
                float* nxt = pb + ((ch + 1) & 1) * 1024;
                const uint32_t nb = base + 1024, ncnt = min(1024u, k - nb);
                for (uint32_t t = tid - 32; t < ncnt; t += blockDim.x - 32) nxt[t] = __ldcg(ps + nb + t);
            }
            __syncthreads();
            for (uint32_t t = tid; t < cnt; t += blockDim.x) ps[base + t] = cur[t];
            __syncthreads();
        }
        if (tid == 0) {
            run_s = run;
            first_s = 0xffffffffu;
            cmp_s = c->top_p < 1.0f ? __fmul_rn(c->top_p, run) : 0.0f;
        }
        __syncthreads();
        uint32_t cut = k;
        if (c->top_p < 1.0f) {
            const float target = cmp_s;
            for (uint32_t i = tid; i < k; i += blockDim.x)
                if (__ldcg(ps + i) >= target) {
                    atomicMin(&first_s, i);
                    break;
                }
            __syncthreads();
            if (first_s != 0xffffffffu) cut = first_s + 1;
            __syncthreads();
        }
        if (tid == 0) {
            const float sum = c->top_p < 1.0f ? __ldcg(ps + cut - 1) : run_s;
            uint64_t s4[4] = {c->rng[0], c->rng[1], c->rng[2], c->rng[3]};
            const float u = __fmul_rn((float)(rng_next(s4) >> 40), 1.0f / 16777216.0f);
            for (int i = 0; i < 4; i++) c->rng[i] = a.ctl->rng[i] = s4[i];
            c->draws += 1;
            a.ctl->draws = c->draws;
            cmp_s = __fmul_rn(u, sum);
            first_s = 0xffffffffu;
        }
        __syncthreads();
        {
            const float r = cmp_s;
            for (uint32_t i = tid; i < cut; i += blockDim.x)
                if (r < __ldcg(ps + i)) {
                    atomicMin(&first_s, i);
                    break;
                }
        }
        __syncthreads();
        if (tid == 0) tok_s = (uint32_t)__ldcg(keys + (first_s != 0xffffffffu ? first_s : cut - 1));
    } else if (need) {
        const uint32_t k = c->top_k == 0 ? a.vocab : min(c->top_k, a.vocab);
        if (a.n_cta == 1) {
            for (uint32_t i = tid; i < k; i += blockDim.x) merged[i] = a.cand[i];
        } else {
            // Only lists whose best key is among the k best heads can hold a
            // global top-k key (the k best heads are k keys).
            if (tid < a.n_cta) heads[tid] = a.cand[(size_t)tid * a.kmax];
            __syncthreads();
            if (tid < a.n_cta) {
                const uint64_t hk = heads[tid];
                uint32_t rank = 0;
                for (uint32_t o = 0; o < a.n_cta; o++) rank += heads[o] < hk;
                if (rank < k) sel[rank] = tid;
            }
            __syncthreads();
            const uint32_t n_sel = min(k, a.n_cta);
            for (uint32_t idx = tid; idx < n_sel * k; idx += blockDim.x) {
                const uint32_t s = idx / k, j = idx % k;
                sel_lists[s * k + j] = a.cand[(size_t)sel[s] * a.kmax + j];
            }
            __syncthreads();
            tr.mark(1);
            // Merge tree: pairs of sorted lists merged into the first k of
            // their union (output p by a co-rank search: i keys of X and
            // p - i of Y are the p smallest), ping-pong between the two
            // halves of the list buffer, until one list is left. Keys are
            // unique, so this is the exact top-k in order.
            uint64_t* src = sel_lists;
            uint64_t* dst = sel_lists + 64 * 64;
            for (uint32_t m = n_sel; m > 1;) {
                const uint32_t pairs = m / 2, lists = pairs + (m & 1);
                for (uint32_t idx = tid; idx < lists * k; idx += blockDim.x) {
                    const uint32_t pr = idx / k, p = idx % k;
                    const uint64_t* X = src + (size_t)(2 * pr) * k;
                    if (pr == pairs) {  // the odd list out
                        dst[(size_t)pr * k + p] = X[p];
                        continue;
                    }
                    const uint64_t* Y = X + k;
                    uint32_t lo = 0, hi = p;
                    while (lo < hi) {
                        const uint32_t mid = (lo + hi) >> 1;
                        if (X[mid] < Y[p - mid - 1])
                            lo = mid + 1;
                        else
                            hi = mid;
                    }
                    const uint64_t x = X[lo], y = Y[p - lo];
                    dst[(size_t)pr * k + p] = x < y ? x : y;
                }
                __syncthreads();
                uint64_t* t = src;
                src = dst;
                dst = t;
                m = lists;
            }
            for (uint32_t i = tid; i < k; i += blockDim.x) merged[i] = src[i];
        }
        __syncthreads();
        tr.mark(2);
        // sampler.rs:135-141: each weight exp((l - max) / T) on its own
        // thread, then the sums in order on one
        {
            const float inv_t = __fdiv_rn(1.0f, c->temperature);
            const float mx = key_value(merged[0]);
            for (uint32_t i = tid; i < k; i += blockDim.x)
                pk[i] = ref_exp(__fmul_rn(__fsub_rn(key_value(merged[i]), mx), inv_t));
        }
        __syncthreads();
        if (tid == 0) {
            float sum = 0.0f;
            for (uint32_t i = 0; i < k; i++) sum = __fadd_rn(sum, pk[i]);
            uint32_t cut = k;
            if (c->top_p < 1.0f) {
                const float target = __fmul_rn(c->top_p, sum);
                float acc = 0.0f;
                for (uint32_t i = 0; i < k; i++) {
                    acc = __fadd_rn(acc, pk[i]);
                    if (acc >= target) {
                        cut = i + 1;
                        break;
                    }
                }
                sum = 0.0f;
                for (uint32_t i = 0; i < cut; i++) sum = __fadd_rn(sum, pk[i]);
            }
            uint64_t s4[4] = {c->rng[0], c->rng[1], c->rng[2], c->rng[3]};
            const float u = __fmul_rn((float)(rng_next(s4) >> 40), 1.0f / 16777216.0f);
            for (int i = 0; i < 4; i++) c->rng[i] = a.ctl->rng[i] = s4[i];
            c->draws += 1;
            a.ctl->draws = c->draws;
            const float r = __fmul_rn(u, sum);
            uint32_t pick = (uint32_t)merged[cut - 1];
            float acc = 0.0f;
            for (uint32_t i = 0; i < cut; i++) {
                acc = __fadd_rn(acc, pk[i]);
                if (r < acc) {
                    pick = (uint32_t)merged[i];
                    break;
                }
            }
            tok_s = pick;
        }
    }
    __syncthreads();
    tr.mark(3);
    if (tid != 0) return;
    DevCtl* g = a.ctl;
    if (!seq) {
        g->out_token = tok_s;
        return;
    }
    // seq.rs:273-312 commit, then arm the next step (seq.rs:239-268); the
    // decisions use the snapshot, and only the changed fields are stored.
    const uint64_t filled = c->filled + 1;
    uint64_t n_tokens = c->n_tokens;
    uint32_t done = c->done, reason = c->done_reason, err = 0;
    uint32_t next_token = 0;
    if (filled == n_tokens) {
        const uint32_t next = tok_s;
        const uint64_t generated = n_tokens - c->prompt_len;
        if (next == c->eos) {
            done = 1;
            reason = 1;
        } else if (generated >= c->max_tokens) {
            done = 1;
            reason = 2;
        } else if (n_tokens + 1 >= c->max_ctx) {
            done = 1;
            reason = 3;
        } else if (n_tokens >= c->cap) {
            done = 1;
            err |= ERR_CAP;
        } else {
            a.tokens_w[n_tokens] = next;
            n_tokens += 1;
            if (filled == n_tokens - 1) next_token = next;
        }
    }
    uint32_t active = 0;
    if (!done) {
        if (filled >= n_tokens) {
            done = 1;
            err |= ERR_INVARIANT;
        } else if (!(c->stop_at && filled >= c->stop_at)) {
            active = 1;
            // The token at `filled` is the one just appended, or a prompt token
            // already in the history.
            c->token = filled == n_tokens - 1 && n_tokens != c->n_tokens ? next_token : __ldcg(a.tokens + filled);
        }
    }
    g->filled = filled;
    g->n_tokens = n_tokens;
    g->done = done;
    g->done_reason = reason;
    if (err) atomicOr(&g->err, err);
    if (active) {
        g->token = c->token;
        g->pos = (uint32_t)filled;
    }
    g->active = active;
    tr.exit();
}

template <int OUT, int L>
cudaError_t launch_gemv_t(const GemvPlan& p, const GemvArgs& a, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(p.threads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_gemv<OUT, L>, p.tm0, p.tm1, a, p.in_mode);
}

template <typename K, typename A>
cudaError_t launch_pdl(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, const A& args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args);
}

}  // namespace

// Allow each kernel the device's opt-in shared memory minus its static part.
template <typename K>
cudaError_t allow_smem(K kernel, int optin) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
    if (e != cudaSuccess) return e;
    // One carveout for every kernel, so a kernel launched early under PDL
    // never waits for an SM to switch its L1/shared split.
    return cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
}

cudaError_t gemv_set_smem_limits(int optin) {
    cudaError_t e = cudaSuccess;
#define HS_SET(O, L) \
    if (e == cudaSuccess) e = allow_smem(k_gemv<O, L>, optin);
    HS_SET(OUT_STORE, 1) HS_SET(OUT_STORE, 2) HS_SET(OUT_STORE, 4) HS_SET(OUT_STORE, 8)
    HS_SET(OUT_RESID, 1) HS_SET(OUT_RESID, 2) HS_SET(OUT_RESID, 4) HS_SET(OUT_RESID, 8)
    HS_SET(OUT_SILU, 1) HS_SET(OUT_SILU, 2) HS_SET(OUT_SILU, 4) HS_SET(OUT_SILU, 8)
#undef HS_SET
    if (e == cudaSuccess) e = allow_smem(k_attention<64>, optin);
    if (e == cudaSuccess) e = allow_smem(k_attention<128>, optin);
    if (e == cudaSuccess) e = allow_smem(k_sample_final, optin);
    if (e == cudaSuccess) e = allow_smem(k_sample_cand_wide<true>, optin);
    return e;
}

cudaError_t launch_gemv(const GemvPlan& p, const GemvArgs& a, cudaStream_t st) {
    switch (p.out_mode * 16 + p.lanes) {
        case OUT_STORE * 16 + 1: return launch_gemv_t<OUT_STORE, 1>(p, a, st);
        case OUT_STORE * 16 + 2: return launch_gemv_t<OUT_STORE, 2>(p, a, st);
        case OUT_STORE * 16 + 4: return launch_gemv_t<OUT_STORE, 4>(p, a, st);
        case OUT_STORE * 16 + 8: return launch_gemv_t<OUT_STORE, 8>(p, a, st);
        case OUT_RESID * 16 + 1: return launch_gemv_t<OUT_RESID, 1>(p, a, st);
        case OUT_RESID * 16 + 2: return launch_gemv_t<OUT_RESID, 2>(p, a, st);
        case OUT_RESID * 16 + 4: return launch_gemv_t<OUT_RESID, 4>(p, a, st);
        case OUT_RESID * 16 + 8: return launch_gemv_t<OUT_RESID, 8>(p, a, st);
        case OUT_SILU * 16 + 1: return launch_gemv_t<OUT_SILU, 1>(p, a, st);
        case OUT_SILU * 16 + 2: return launch_gemv_t<OUT_SILU, 2>(p, a, st);
        case OUT_SILU * 16 + 4: return launch_gemv_t<OUT_SILU, 4>(p, a, st);
        case OUT_SILU * 16 + 8: return launch_gemv_t<OUT_SILU, 8>(p, a, st);
        default: return cudaErrorInvalidValue;
    }
}

size_t attention_smem(uint32_t head_dim, uint32_t max_ctx) {
    const size_t rs = head_dim + 4, pre = 12288 / head_dim, ch = 4096 / head_dim;
    return (3 * head_dim + 64 + (2 * pre + ch) * rs + max_ctx) * sizeof(float);
}

cudaError_t launch_attention(uint32_t head_dim, uint32_t nh, size_t smem, const AttnArgs& a, cudaStream_t st) {
    if (head_dim == 64) return launch_pdl(k_attention<64>, dim3(nh), dim3(256), smem, st, a);
    if (head_dim == 128) return launch_pdl(k_attention<128>, dim3(nh), dim3(256), smem, st, a);
    return cudaErrorInvalidValue;
}

size_t sample_final_smem(uint32_t n_cta, uint32_t kmax) {
    // Selected lists: at most 64 lists of at most 64 keys (top_k <= 64), and
    // as much again for the merge tree's other half, when there are several
    // CTAs in list mode; none with one CTA or in sort mode.
    return n_cta > 1 && !sample_sort_mode(n_cta, kmax) ? (size_t)2 * 64 * 64 * sizeof(uint64_t) : 16;
}

size_t sample_sort_smem(uint32_t slice) {
    uint32_t n2 = 256;
    while (n2 < slice) n2 <<= 1;
    return (size_t)n2 * sizeof(uint64_t);
}

cudaError_t launch_sample(const SampleArgs& a, cudaStream_t st) {
    const uint32_t slots = a.slots ? a.slots : 1;
    const uint32_t slice = a.slice ? a.slice : kSampleSlice;
    if (sample_sort_mode(a.n_cta, a.kmax)) {
        // any top_k: every slice sorted whole, ranked across slices, then the final kernel
        if (slice % 256 || slice > kMaxSlice || a.kmax != slice || !a.wkeys || !a.wps || a.wide_stride < a.vocab ||
            a.cand_stride < (uint64_t)a.n_cta * slice)
            return cudaErrorInvalidValue;
        SampleArgs s = a;
        s.slice = slice;
        cudaError_t e = launch_pdl(k_sample_cand_wide<true>, dim3(a.n_cta, slots), dim3(256), sample_sort_smem(slice),
                                   st, s);
        if (e != cudaSuccess) return e;
        SampleArgs r = s;
        r.trace = nullptr;
        e = launch_pdl(k_sample_rank, dim3((a.n_cta * slice + 255) / 256, slots), dim3(256), 0, st, r);
        if (e != cudaSuccess) return e;
        return launch_pdl(k_sample_final, dim3(1, slots), dim3(kFinalThreads), sample_final_smem(a.n_cta, a.kmax), st,
                          s);
    }
    const bool wide = a.slice > kSampleSlice;
    if (wide && (a.slice % 256 || a.slice > kMaxSlice || a.kmax > kMaxTopK)) return cudaErrorInvalidValue;
    cudaError_t e = wide ? launch_pdl(k_sample_cand_wide<false>, dim3(a.n_cta, slots), dim3(256), 0, st, a)
                         : launch_pdl(k_sample_cand, dim3(a.n_cta, slots), dim3(256), 0, st, a);
    if (e != cudaSuccess) return e;
    return launch_pdl(k_sample_final, dim3(1, slots), dim3(kFinalThreads), sample_final_smem(a.n_cta, a.kmax), st, a);
}

}  // namespace hs
