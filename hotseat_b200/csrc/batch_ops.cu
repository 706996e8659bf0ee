// Per-sequence kernels of the tensor-core token loop (numeric path
// HS_NUMERIC_TC), around the GEMMs of batch_tc.cu:
//
//   k_tc_norm       one CTA per sequence: finishes the residual stream
//                   (embedding row at layer 0, or x += the split-K partial
//                   sums of the previous O / down GEMM, added in split
//                   order), then RMSNorm, written as the f16 hi/lo pair the
//                   next GEMM reads (model.rs:247-250, 308-321; math.rs:200-207).
//   k_tc_attention  one CTA per (sequence, KV head): sums the QKV partials
//                   and the bias, RoPE on the group's query heads and the
//                   key (model.rs:259-266, 365-373), appends k and v at
//                   `pos` in the sequence's own KV region and marks the
//                   dirty pages (model.rs:268-275), then scores, softmax
//                   and P.V for every query head of the group over the
//                   cached positions (model.rs:277-305).
//
// Reductions have fixed shapes that depend only on the model, never on the
// slot or the number of sequences in the batch.
#include <cfloat>

#include "common.h"
#include "kernels.h"

namespace hs {
namespace {

__device__ __forceinline__ uint32_t ldv(const uint32_t* p) { return *(const volatile uint32_t*)p; }
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void split_f16(float x, uint16_t* hi, uint16_t* lo) {
    const __half h = __float2half_rn(x);
    *hi = __half_as_ushort(h);
    *lo = __half_as_ushort(__float2half_rn(__fsub_rn(x, __half2float(h))));
}

constexpr uint32_t kNormThreads = 256;
constexpr uint32_t kNormMaxChunks = 2;  // float4 chunks per thread: d <= 2048
constexpr uint32_t kMaxParts = 32;      // split-K partials a consumer adds

__device__ __forceinline__ float4 f4add(float4 a, float4 b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}
// Sum of `n` split partials of one float4 chunk, in split order; the loads
// are issued eight at a time so they overlap.
__device__ __forceinline__ float4 sum_parts(const float* base, uint64_t stride, uint32_t n) {
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (uint32_t s0 = 0; s0 < n; s0 += 8) {
        float4 v[8];
#pragma unroll
        for (uint32_t j = 0; j < 8; j++)
            if (s0 + j < n) v[j] = __ldcg(reinterpret_cast<const float4*>(base + (s0 + j) * stride));
#pragma unroll
        for (uint32_t j = 0; j < 8; j++)
            if (s0 + j < n) acc = f4add(acc, v[j]);
    }
    return acc;
}

// ---------------------------------------------------------------- RMSNorm
// Thread t owns the float4 chunks t and t + 256 of the row.
__global__ void __launch_bounds__(kNormThreads) k_tc_norm(const TcNormArgs a) {
    __shared__ float red[kNormThreads / 32];
    const uint32_t slot = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const KTrace tr(a.trace, a.trace_slot);
    tr.enter();
    DevCtl* ctl = a.ctl + slot;
    const bool active = ldv(&ctl->active) != 0;
    const uint32_t token = a.embd ? ldv(&ctl->token) : 0;
    pdl_launch_dependents();
    pdl_wait();
    if (!active) return;
    if (a.embd && token >= a.vocab) {
        if (tid == 0) atomicOr(&ctl->err, ERR_TOKEN);
        return;
    }
    const uint32_t d4 = a.d / 4;
    float4 v[kNormMaxChunks];
    float ss = 0.0f;
#pragma unroll
    for (uint32_t j = 0; j < kNormMaxChunks; j++) {
        const uint32_t c = tid + j * kNormThreads;
        v[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (c >= d4) continue;
        float4 x;
        if (a.embd) {
            const uint2 e = *reinterpret_cast<const uint2*>(a.embd + (size_t)token * a.d + 4 * c);
            x = make_float4(h2f(e.x & 0xffff), h2f(e.x >> 16), h2f(e.y & 0xffff), h2f(e.y >> 16));
        } else {
            x = *reinterpret_cast<const float4*>(a.x + (size_t)slot * a.d + 4 * c);
            if (a.n_part) x = f4add(x, sum_parts(a.part + (size_t)slot * a.d + 4 * c, a.part_stride, a.n_part));
        }
        if (a.embd || a.n_part) *reinterpret_cast<float4*>(a.x + (size_t)slot * a.d + 4 * c) = x;
        v[j] = x;
        ss = __fmaf_rn(x.x, x.x, ss);
        ss = __fmaf_rn(x.y, x.y, ss);
        ss = __fmaf_rn(x.z, x.z, ss);
        ss = __fmaf_rn(x.w, x.w, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (uint32_t w = 0; w < kNormThreads / 32; w++) tot = __fadd_rn(tot, red[w]);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)a.d), a.eps)));
#pragma unroll
    for (uint32_t j = 0; j < kNormMaxChunks; j++) {
        const uint32_t c = tid + j * kNormThreads;
        if (c >= d4) continue;
        const float4 g = *reinterpret_cast<const float4*>(a.g + 4 * c);
        const float y[4] = {__fmul_rn(__fmul_rn(v[j].x, scale), g.x), __fmul_rn(__fmul_rn(v[j].y, scale), g.y),
                            __fmul_rn(__fmul_rn(v[j].z, scale), g.z), __fmul_rn(__fmul_rn(v[j].w, scale), g.w)};
        uint16_t hi[4], lo[4];
#pragma unroll
        for (int q = 0; q < 4; q++) split_f16(y[q], &hi[q], &lo[q]);
        *reinterpret_cast<uint2*>(a.out_hi + (size_t)slot * a.d + 4 * c) =
            make_uint2(hi[0] | (uint32_t)hi[1] << 16, hi[2] | (uint32_t)hi[3] << 16);
        *reinterpret_cast<uint2*>(a.out_lo + (size_t)slot * a.d + 4 * c) =
            make_uint2(lo[0] | (uint32_t)lo[1] << 16, lo[2] | (uint32_t)lo[3] << 16);
    }
    tr.exit();
}

// ---------------------------------------------------------------- attention
constexpr uint32_t kAttnThreads = 256;
constexpr uint32_t kChunk = 64;  // cached positions per K / V chunk
constexpr uint32_t kNb = 4;      // chunk buffers in flight
__device__ __forceinline__ void cp_wait_nb() { asm volatile("cp.async.wait_group %0;" ::"n"(kNb - 1) : "memory"); }

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) k_tc_attention(const TcAttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    constexpr uint32_t RS = HD + 4;                  // chunk row stride (16-byte rows, conflict-free float4 reads)
    constexpr uint32_t HALF = HD / 2;
    constexpr uint32_t HSETS = kAttnThreads / HD;    // head sets in P.V
    constexpr uint32_t HPT = (8 + HSETS - 1) / HSETS;  // heads per thread in P.V (G <= 8)
    const uint32_t kvh = blockIdx.x, slot = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t G = a.nh / a.nkv;
    float* qs = sm;                                  // [G][HD]
    float* kn = qs + 8 * HD;                         // [HD]
    float* vn = kn + HD;                             // [HD]
    float* buf = vn + HD;                            // [kNb][kChunk][RS]
    // [G][max_ctx] scores: shared memory, or this CTA's block of a global
    // buffer when they do not fit.
    float* sc = a.sc_global ? a.sc_global + ((size_t)blockIdx.y * a.nkv + blockIdx.x) * G * a.max_ctx
                            : buf + kNb * kChunk * RS;
    float* inv = buf + kNb * kChunk * RS + (a.sc_global ? 0 : (size_t)G * a.max_ctx);  // [8]
    const KTrace tr(a.trace, a.trace_slot);
    tr.enter();
    DevCtl* ctl = a.ctl + slot;
    const bool active = ldv(&ctl->active) != 0;
    const uint32_t pos = ldv(&ctl->pos);
    float* kv = a.kv[slot];
    const uint64_t plane = (uint64_t)a.max_ctx * a.nkv * HD;
    const uint64_t lbase = (uint64_t)a.layer * 2 * plane;
    auto row_off = [&](uint32_t p, uint32_t is_v) -> uint64_t {
        const uint64_t within = a.layout == 0 ? ((uint64_t)p * a.nkv + kvh) * HD : ((uint64_t)kvh * a.max_ctx + p) * HD;
        return lbase + (is_v ? plane : 0) + within;
    };
    pdl_launch_dependents();
    pdl_wait();
    if (!active) return;
    if (pos >= a.max_ctx) {
        if (tid == 0) atomicOr(&ctl->err, ERR_POS);
        return;
    }
    // q (G heads), k, v: split-K partials in split order, then the bias.
    const uint32_t qrow0 = kvh * G * HD, krow0 = a.nh * HD + kvh * HD, vrow0 = (a.nh + a.nkv) * HD + kvh * HD;
    for (uint32_t c = tid; c < (G + 2) * HD / 4; c += kAttnThreads) {
        const uint32_t idx = 4 * c;
        const uint32_t row = idx < G * HD ? qrow0 + idx : (idx < (G + 1) * HD ? krow0 + idx - G * HD : vrow0 + idx - (G + 1) * HD);
        float4 p = sum_parts(a.qkv_part + (size_t)slot * a.qkv_rows + row, a.part_stride, a.n_part);
        p = f4add(p, *reinterpret_cast<const float4*>(a.bias + row));
        float* dst = idx < G * HD ? qs + idx : (idx < (G + 1) * HD ? kn + idx - G * HD : vn + idx - (G + 1) * HD);
        *reinterpret_cast<float4*>(dst) = p;
    }
    __syncthreads();
    // RoPE (NeoX pairs i, i + HD/2) on the query heads and the key.
    for (uint32_t idx = tid; idx < (G + 1) * HALF; idx += kAttnThreads) {
        const uint32_t h = idx / HALF, i = idx % HALF;
        float* r = h < G ? qs + h * HD : kn;
        const float c = a.rope_cos[(size_t)pos * HALF + i], s = a.rope_sin[(size_t)pos * HALF + i];
        const float x0 = r[i], x1 = r[i + HALF];
        r[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        r[i + HALF] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
    __syncthreads();
    // KV append at `pos`, then the dirty bits of the pages it touched.
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

    const uint32_t n = pos + 1, nchunks = (n + kChunk - 1) / kChunk, items = 2 * nchunks;
    // One pipeline over all K chunks then all V chunks, kNb buffers deep: item
    // i lands in buf[i % kNb]; the row at `pos` comes from shared memory (this
    // CTA just wrote it). Every iteration commits one cp.async group (empty
    // past the end), so "item i is complete" is wait_group(kNb - 1).
    auto issue = [&](uint32_t it) {
        if (it < items) {
            const uint32_t is_v = it >= nchunks, c = is_v ? it - nchunks : it;
            float* dst = buf + (it % kNb) * kChunk * RS;
            const uint32_t c0 = c * kChunk, cnt = n - c0 < kChunk ? n - c0 : kChunk;
            for (uint32_t idx = tid; idx < cnt * (HD / 4); idx += kAttnThreads) {
                const uint32_t r = idx / (HD / 4), c4 = idx % (HD / 4);
                if (c0 + r == pos) {
                    const float* src = is_v ? vn : kn;
                    *reinterpret_cast<float4*>(dst + r * RS + 4 * c4) = *reinterpret_cast<const float4*>(src + 4 * c4);
                } else {
                    cp_async16(dst + r * RS + 4 * c4, kv + row_off(c0 + r, is_v) + 4 * c4);
                }
            }
        }
        cp_commit();
    };
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
    float acc[HPT];
#pragma unroll
    for (uint32_t j = 0; j < HPT; j++) acc[j] = 0.0f;
    const uint32_t dd = tid % HD, hs0 = tid / HD;
    for (uint32_t it = 0; it + 1 < kNb; it++) issue(it);
    for (uint32_t it = 0; it < items; it++) {
        issue(it + kNb - 1);
        cp_wait_nb();
        __syncthreads();
        const float* cb = buf + (it % kNb) * kChunk * RS;
        if (it < nchunks) {
            // Scores: thread t takes position t % 64 of the chunk and heads t/64, t/64 + 4.
            const uint32_t c0 = it * kChunk, r = tid % kChunk, p = c0 + r;
            if (p < n) {
                const float4* k4 = reinterpret_cast<const float4*>(cb + r * RS);
                for (uint32_t h = tid / kChunk; h < G; h += kAttnThreads / kChunk) {
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
                    sc[(size_t)h * a.max_ctx + p] = __fmul_rn(__fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3)), scale);
                }
            }
        } else {
            if (it == nchunks) {
                // Softmax: warp h owns head h (lane-strided partials, fixed xor tree).
                if (warp < G) {
                    float* sh = sc + (size_t)warp * a.max_ctx;
                    float mx = -FLT_MAX;
                    for (uint32_t p = lane; p < n; p += 32) mx = fmaxf(mx, sh[p]);
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                    float sum = 0.0f;
                    for (uint32_t p = lane; p < n; p += 32) {
                        const float e = __expf(__fsub_rn(sh[p], mx));
                        sh[p] = e;
                        sum = __fadd_rn(sum, e);
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
                    if (lane == 0) inv[warp] = __fdiv_rn(1.0f, sum);
                }
                __syncthreads();
            }
            // P.V: thread t owns dimension t % HD of heads t/HD, t/HD + HSETS, ...
            const uint32_t c0 = (it - nchunks) * kChunk, cnt = n - c0 < kChunk ? n - c0 : kChunk;
#pragma unroll
            for (uint32_t j = 0; j < HPT; j++) {
                const uint32_t h = hs0 + j * HSETS;
                if (h >= G) break;
                const float* ph = sc + (size_t)h * a.max_ctx + c0;
                float sacc = acc[j];
                for (uint32_t r = 0; r < cnt; r++) sacc = __fmaf_rn(ph[r], cb[r * RS + dd], sacc);
                acc[j] = sacc;
            }
        }
        __syncthreads();
    }
    cp_wait_0();
#pragma unroll
    for (uint32_t j = 0; j < HPT; j++) {
        const uint32_t h = hs0 + j * HSETS;
        if (h >= G) break;
        uint16_t hi, lo;
        split_f16(__fmul_rn(acc[j], inv[h]), &hi, &lo);
        const size_t o = (size_t)slot * a.nh * HD + (size_t)(kvh * G + h) * HD + dd;
        a.att_hi[o] = hi;
        a.att_lo[o] = lo;
    }
    tr.exit();
}

cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace

size_t tc_attention_smem(uint32_t head_dim, uint32_t groups, uint32_t max_ctx) {
    const size_t rs = head_dim + 4;
    return (8 * head_dim + 2 * head_dim + kNb * kChunk * rs + (size_t)groups * max_ctx + 8) * sizeof(float);
}

cudaError_t tc_ops_set_smem_limits(int optin) {
    cudaError_t e = cudaFuncSetAttribute(k_tc_attention<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_tc_attention<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
}

cudaError_t launch_tc_norm(const TcNormArgs& a, uint32_t slots, cudaStream_t st) {
    if (a.d % 4 || a.d > kNormThreads * kNormMaxChunks * 4 || a.n_part > kMaxParts) return cudaErrorInvalidValue;
    TcNormArgs c = a;
    void* args[] = {&c};
    return launch_pdl(reinterpret_cast<const void*>(k_tc_norm), dim3(slots), dim3(kNormThreads), 0, st, args);
}

cudaError_t launch_tc_attention(uint32_t head_dim, const TcAttnArgs& a, uint32_t slots, size_t smem, cudaStream_t st) {
    if (a.nkv == 0 || a.nh % a.nkv || a.nh / a.nkv > 8) return cudaErrorInvalidValue;
    TcAttnArgs c = a;
    void* args[] = {&c};
    if (head_dim == 64)
        return launch_pdl(reinterpret_cast<const void*>(k_tc_attention<64>), dim3(a.nkv, slots), dim3(kAttnThreads), smem,
                          st, args);
    if (head_dim == 128)
        return launch_pdl(reinterpret_cast<const void*>(k_tc_attention<128>), dim3(a.nkv, slots), dim3(kAttnThreads),
                          smem, st, args);
    return cudaErrorInvalidValue;
}

}  // namespace hs
