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
#include <cfloat>

#include "common.h"
#include "kernels.h"

namespace hs {
namespace {

constexpr uint32_t kThreads = 256;
constexpr uint32_t kCh = 64;  // positions per chunk

__device__ __forceinline__ uint32_t ldv(const uint32_t* p) { return *(const volatile uint32_t*)p; }
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void split_f16(float x, uint16_t* hi, uint16_t* lo) {
    const __half h = __float2half_rn(x);
    *hi = __half_as_ushort(h);
    *lo = __half_as_ushort(__float2half_rn(__fsub_rn(x, __half2float(h))));
}
__device__ __forceinline__ float4 f4add(float4 a, float4 b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

template <int HD>
__global__ void __launch_bounds__(kThreads) k_attn_split(const SplitAttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    constexpr uint32_t RS = HD + 4, HALF = HD / 2;
    constexpr uint32_t HSETS = kThreads / HD, HPT = (8 + HSETS - 1) / HSETS;
    const uint32_t s = blockIdx.x, kvh = blockIdx.y, slot = blockIdx.z;
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t G = a.nh / a.nkv;
    float* qs = sm;                        // [8][HD]
    float* kn = qs + 8 * HD;               // [HD]
    float* vn = kn + HD;                   // [HD]
    float* kb = vn + HD;                   // [2][kCh][RS]
    float* vb = kb + 2 * kCh * RS;         // [2][kCh][RS]
    float* sp = vb + 2 * kCh * RS;         // [8][kCh] scores, then probabilities
    float* hs_m = sp + 8 * kCh;            // [8] running maximum per head
    float* hs_f = hs_m + 8;                // [8] rescale of the running sums this chunk
    float* hs_l = hs_f + 8;                // [8] running sums
    uint32_t* flag = reinterpret_cast<uint32_t*>(hs_l + 8);
    const KTrace tr(a.trace, a.trace_slot);
    tr.enter();
    DevCtl* ctl = a.ctl + slot;
    const bool active = ldv(&ctl->active) != 0;
    const uint32_t pos = ldv(&ctl->pos);
    pdl_launch_dependents();
    pdl_wait();
    if (!active) return;
    if (pos >= a.max_ctx) {
        if (tid == 0 && s == 0 && kvh == 0) atomicOr(&ctl->err, ERR_POS);
        return;
    }
    const uint32_t n = pos + 1, L = attn_split_len(n, a.max_splits), S = (n + L - 1) / L;
    // Prefill runs append (every token's k, v) and attend (reading all rows
    // from memory) as two launches, so tokens of one sequence in one batch
    // see each other's rows.
    const bool append = a.mode != ATTN_ATTEND_ONLY, attend = a.mode != ATTN_APPEND_ONLY;
    if (s >= (attend ? S : 1u)) return;
    const uint32_t p0 = s * L, p1 = p0 + L < n ? p0 + L : n;
    float* kv = a.kv[slot];
    const uint64_t plane = (uint64_t)a.max_ctx * a.nkv * HD;
    const uint64_t lbase = (uint64_t)a.layer * 2 * plane;
    auto row_off = [&](uint32_t p, uint32_t is_v) -> uint64_t {
        const uint64_t within = a.layout == 0 ? ((uint64_t)p * a.nkv + kvh) * HD : ((uint64_t)kvh * a.max_ctx + p) * HD;
        return lbase + (is_v ? plane : 0) + within;
    };

    // q, k, v of this group; split-K partials in split order, then the bias.
    const uint32_t qrow0 = kvh * G * HD, krow0 = a.nh * HD + kvh * HD, vrow0 = (a.nh + a.nkv) * HD + kvh * HD;
    for (uint32_t c = tid; c < (G + 2) * HD / 4; c += kThreads) {
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
    __syncthreads();
    for (uint32_t idx = tid; idx < (G + 1) * HALF; idx += kThreads) {
        const uint32_t h = idx / HALF, i = idx % HALF;
        float* r = h < G ? qs + h * HD : kn;
        const float c = a.rope_cos[(size_t)pos * HALF + i], sn = a.rope_sin[(size_t)pos * HALF + i];
        const float x0 = r[i], x1 = r[i + HALF];
        r[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
        r[i + HALF] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
    if (tid < 8) {
        hs_m[tid] = -FLT_MAX;
        hs_l[tid] = 0.0f;
    }
    __syncthreads();
    if (s == 0 && append) {
        if (tid < HD) {
            kv[row_off(pos, 0) + tid] = kn[tid];
            kv[row_off(pos, 1) + tid] = vn[tid];
        }
        __syncthreads();
        if (tid < 2 && ldv(a.tracking[slot])) {
            __threadfence();
            const uint64_t off = row_off(pos, tid) * 4, last = off + HD * 4 - 1;
            uint64_t* dirty = a.dirty[slot];
            for (uint64_t pg = off >> a.page_shift; pg <= (last >> a.page_shift); pg++)
                atomicOr(reinterpret_cast<unsigned long long*>(&dirty[pg >> 6]), 1ull << (pg & 63));
        }
    }

    if (!attend) return;
    const uint32_t nch = (p1 - p0 + kCh - 1) / kCh;
    auto issue = [&](uint32_t c) {
        if (c < nch) {
            const uint32_t c0 = p0 + c * kCh, cnt = p1 - c0 < kCh ? p1 - c0 : kCh;
            float* kd = kb + (c & 1) * kCh * RS;
            float* vd = vb + (c & 1) * kCh * RS;
            for (uint32_t idx = tid; idx < cnt * (HD / 4); idx += kThreads) {
                const uint32_t r = idx / (HD / 4), c4 = idx % (HD / 4);
                if (c0 + r == pos && append) {
                    *reinterpret_cast<float4*>(kd + r * RS + 4 * c4) = *reinterpret_cast<const float4*>(kn + 4 * c4);
                    *reinterpret_cast<float4*>(vd + r * RS + 4 * c4) = *reinterpret_cast<const float4*>(vn + 4 * c4);
                } else {
                    cp_async16(kd + r * RS + 4 * c4, kv + row_off(c0 + r, 0) + 4 * c4);
                    cp_async16(vd + r * RS + 4 * c4, kv + row_off(c0 + r, 1) + 4 * c4);
                }
            }
        }
        cp_commit();
    };
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
    float o[HPT];
#pragma unroll
    for (uint32_t j = 0; j < HPT; j++) o[j] = 0.0f;
    const uint32_t dd = tid % HD, hs0 = tid / HD;
    issue(0);
    for (uint32_t c = 0; c < nch; c++) {
        issue(c + 1);
        cp_wait1();
        __syncthreads();
        const uint32_t c0 = p0 + c * kCh, cnt = p1 - c0 < kCh ? p1 - c0 : kCh;
        const float* kc = kb + (c & 1) * kCh * RS;
        const float* vc = vb + (c & 1) * kCh * RS;
        // scores: thread t takes position t % 64 and heads t/64, t/64 + 4
        {
            const uint32_t r = tid % kCh;
            for (uint32_t h = tid / kCh; h < G; h += kThreads / kCh) {
                float v = -FLT_MAX;
                if (r < cnt) {
                    const float4* k4 = reinterpret_cast<const float4*>(kc + r * RS);
                    const float4* q4 = reinterpret_cast<const float4*>(qs + h * HD);
                    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
#pragma unroll
                    for (uint32_t d4 = 0; d4 < HD / 4; d4++) {
                        const float4 kk = k4[d4], qq = q4[d4];
                        s0 = __fmaf_rn(qq.x, kk.x, s0);
                        s1 = __fmaf_rn(qq.y, kk.y, s1);
                        s2 = __fmaf_rn(qq.z, kk.z, s2);
                        s3 = __fmaf_rn(qq.w, kk.w, s3);
                    }
                    v = __fmul_rn(__fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3)), scale);
                }
                sp[h * kCh + r] = v;
            }
        }
        __syncthreads();
        // online softmax: warp h owns head h
        if (warp < G) {
            float* sh = sp + warp * kCh;
            const float a0 = sh[lane], a1 = sh[lane + 32];
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
        }
        __syncthreads();
        // P.V: thread t owns dimension t % HD of heads t/HD, t/HD + HSETS, ...
#pragma unroll
        for (uint32_t j = 0; j < HPT; j++) {
            const uint32_t h = hs0 + j * HSETS;
            if (h >= G) break;
            const float* ph = sp + h * kCh;
            float acc = 0.0f;
            for (uint32_t r = 0; r < cnt; r++) acc = __fmaf_rn(ph[r], vc[r * RS + dd], acc);
            o[j] = __fadd_rn(__fmul_rn(o[j], hs_f[h]), acc);
        }
        __syncthreads();
    }
    cp_wait0();

    auto store = [&](uint32_t h, float v) {
        const size_t at = (size_t)slot * a.out_stride + (size_t)(kvh * G + h) * HD + dd;
        if (a.out_f32) {
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
            if (h < G) store(h, __fdiv_rn(o[j], hs_l[h]));
        }
        tr.exit();
        return;
    }
    // Several splits: publish (unnormalised output, max, sum); the last CTA
    // to arrive combines all splits in split order.
    const uint32_t rec = G * HD + 2 * G;
    float* part = a.partials + ((size_t)(slot * a.nkv + kvh) * a.max_splits) * rec;
#pragma unroll
    for (uint32_t j = 0; j < HPT; j++) {
        const uint32_t h = hs0 + j * HSETS;
        if (h < G) part[(size_t)s * rec + h * HD + dd] = o[j];
    }
    if (tid < G) {
        part[(size_t)s * rec + G * HD + tid] = hs_m[tid];
        part[(size_t)s * rec + G * HD + G + tid] = hs_l[tid];
    }
    __threadfence();
    __syncthreads();
    uint32_t* counter = a.counters + slot * a.nkv + kvh;
    if (tid == 0) *flag = atomicAdd(counter, 1u) == S - 1 ? 1u : 0u;
    __syncthreads();
    if (!*flag) return;
    __threadfence();
    for (uint32_t idx = tid; idx < G * HD; idx += kThreads) {
        const uint32_t h = idx / HD;
        float M = -FLT_MAX;
        for (uint32_t q = 0; q < S; q++) M = fmaxf(M, __ldcg(part + (size_t)q * rec + G * HD + h));
        float num = 0.0f, den = 0.0f;
        for (uint32_t q = 0; q < S; q++) {
            const float w = __expf(__fsub_rn(__ldcg(part + (size_t)q * rec + G * HD + h), M));
            num = __fadd_rn(num, __fmul_rn(w, __ldcg(part + (size_t)q * rec + idx)));
            den = __fadd_rn(den, __fmul_rn(w, __ldcg(part + (size_t)q * rec + G * HD + G + h)));
        }
        const size_t at = (size_t)slot * a.out_stride + (size_t)kvh * G * HD + idx;
        const float v = __fdiv_rn(num, den);
        if (a.out_f32) {
            a.out_f32[at] = v;
        } else {
            uint16_t hi, lo;
            split_f16(v, &hi, &lo);
            a.out_hi[at] = hi;
            a.out_lo[at] = lo;
        }
    }
    if (tid == 0) *counter = 0;
    tr.exit();
}

}  // namespace

size_t attn_split_smem(uint32_t head_dim) {
    return (8 * head_dim + 2 * head_dim + 4 * kCh * (head_dim + 4) + 8 * kCh + 3 * 8 + 4) * sizeof(float);
}

uint32_t attn_max_splits(uint32_t max_ctx) {
    const uint32_t chunks = (max_ctx + kCh - 1) / kCh;
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
    cfg.blockDim = dim3(kThreads);
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
