// Batch-1 token-loop kernels in the GPU-native numeric order ("fast" mode).
//
// Same model and the same fused prologues/epilogues as decode.cu (RMSNorm on
// the way in; bias, residual add or SiLU gate on the way out), but every
// reduction uses a fixed parallel shape instead of the reference's eight
// serial lanes:
//
//   GEMV row r:  a group of T threads (T = 32..256, from the row length only);
//                thread t owns the 16-byte weight chunks t, t+T, t+2T, ... and
//                the matching slice of x, held in registers for the whole
//                kernel; it accumulates with packed FMA (fma.rn.f32x2) in chunk
//                order; the group then reduces by a fixed xor tree and a fixed
//                warp order.
//   RMSNorm:     sum of squares over 32 lanes, xor tree.
//   attention:   split-KV with an online softmax (attn_split.cu).
//
// token_fast.cu runs the same arithmetic as one persistent kernel per token.
//
// Each choice depends only on the tensor shapes, never on the SM count or on
// the batch, so the result for a sequence is bit-identical on every B200 and
// across a migration between GPUs. It is not bit-identical to the CPU
// reference (the serial lane order is what makes that path slow on a GPU);
// the token loop holds it to logits within 1e-2 of the CPU path.
#include "common.h"
#include "kernels.h"

namespace hs {
namespace {

__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) { return *(const volatile uint32_t*)p; }

// Exact f16 -> f32 of both halves of a word (a mixed-precision add of -0.0
// runs on the FP32 pipe and keeps the sign of zero).
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

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ------------------------------------------------------------------ GEMV
// Shared memory: [nst weight stages][xs: n f32][gs: n f32][xe: n f16]
// [part: 2*rt*8 f32][bias_s: rt][red: 32][bars: nst+1]. `a.lanes` carries T.
template <int OUT, int CMAX>
__global__ void __launch_bounds__(256) k_gemv_fast(const __grid_constant__ CUtensorMap tm0,
                                                   const __grid_constant__ CUtensorMap tm1, const GemvArgs a,
                                                   const int in_mode) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    constexpr int NMAT = OUT == OUT_SILU ? 2 : 1;
    const uint32_t n = a.n, kslabs = n / 64, nchunks = n / 8;
    const uint32_t mat_bytes = kslabs * a.slab_stride;
    const uint32_t stage_bytes = NMAT * mat_bytes;
    uint8_t* stages = smem;
    float* xs = reinterpret_cast<float*>(smem + a.nst * stage_bytes);
    float* gs = xs + n;
    uint16_t* xe = reinterpret_cast<uint16_t*>(gs + n);
    float* part = reinterpret_cast<float*>(xe + n);
    float* bias_s = part + 2 * a.rt * 8;
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
    if (tid == 0)
        for (uint32_t t = 0; t < npre; t++) issue(t);
    if (in_mode != IN_PLAIN) {
        const float4* g4 = reinterpret_cast<const float4*>(a.norm_g);
        float4* s4 = reinterpret_cast<float4*>(gs);
#pragma unroll 4
        for (uint32_t i = tid; i < n / 4; i += blockDim.x) s4[i] = g4[i];
    }
    if (OUT == OUT_STORE && a.bias && tid < a.rt && tid < mine) bias_s[tid] = a.bias[r0 + tid];
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
        for (uint32_t t = 0; t < npre; t++) mbar_wait_bounded(&bars[t], 0);
        return;
    }
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
        if (tid < 32) {
            float ss = 0.0f;
            for (uint32_t i = tid; i < n; i += 32) ss = __fmaf_rn(xs[i], xs[i], ss);
            ss = warp_sum(ss);
            if (tid == 0) red[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), a.eps)));
        }
        __syncthreads();
        const float scale = red[0];
        for (uint32_t i = tid; i < n; i += blockDim.x) xs[i] = __fmul_rn(__fmul_rn(xs[i], scale), gs[i]);
        __syncthreads();
    }
    tr.mark(2);

    // This thread's slice of x, in registers for every row.
    const uint32_t T = a.lanes, G = blockDim.x / T, grp = tid / T, tg = tid % T, WG = T / 32, wig = tg / 32;
    uint64_t xp[CMAX * 4];
#pragma unroll
    for (int m = 0; m < CMAX; m++) {
        const uint32_t j = tg + T * m;
        const float4* src = reinterpret_cast<const float4*>(xs + 8 * (j < nchunks ? j : 0));
        const float4 lo = src[0], hi = src[1];
        xp[4 * m + 0] = pack2(lo.x, lo.y);
        xp[4 * m + 1] = pack2(lo.z, lo.w);
        xp[4 * m + 2] = pack2(hi.x, hi.y);
        xp[4 * m + 3] = pack2(hi.z, hi.w);
    }
    const uint32_t vrows = NMAT * a.rt;
    constexpr uint32_t RB = 4;  // rows a thread group runs side by side (independent chains)
    for (uint32_t t = 0; t < ntiles; t++) {
        const uint32_t s = t % a.nst;
        if (!mbar_wait_bounded(&bars[s], (t / a.nst) & 1)) {
            if (tid == 0) atomicOr(&ctl->err, ERR_TIMEOUT);
            return;
        }
        if (t == 0) tr.mark(3);
        const uint8_t* st = stages + s * stage_bytes;
        // Rows go round-robin over the thread groups; each group runs up to RB
        // of its rows side by side.
        for (uint32_t vr0 = grp; vr0 < vrows; vr0 += G * RB) {
            const uint8_t* rowp[RB];
            uint32_t sw[RB];
            bool ok[RB];
#pragma unroll
            for (uint32_t b = 0; b < RB; b++) {
                ok[b] = vr0 + G * b < vrows;
                const uint32_t vr = ok[b] ? vr0 + G * b : vr0;
                const uint32_t mm = vr / a.rt, r = vr % a.rt;
                rowp[b] = st + mm * mat_bytes + r * 128;
                sw[b] = r & 7;
            }
            uint64_t acc[RB];
#pragma unroll
            for (uint32_t b = 0; b < RB; b++) acc[b] = 0;
#pragma unroll
            for (int m = 0; m < CMAX; m++) {
                const uint32_t j = tg + T * m;
                if (j < nchunks) {
                    uint4 w[RB];
#pragma unroll
                    for (uint32_t b = 0; b < RB; b++)
                        if (ok[b])
                            w[b] = *reinterpret_cast<const uint4*>(rowp[b] + (j >> 3) * a.slab_stride +
                                                                    (((j & 7) ^ sw[b]) << 4));
#pragma unroll
                    for (uint32_t b = 0; b < RB; b++) {
                        if (!ok[b]) continue;
                        acc[b] = fma2(widen2(w[b].x), xp[4 * m + 0], acc[b]);
                        acc[b] = fma2(widen2(w[b].y), xp[4 * m + 1], acc[b]);
                        acc[b] = fma2(widen2(w[b].z), xp[4 * m + 2], acc[b]);
                        acc[b] = fma2(widen2(w[b].w), xp[4 * m + 3], acc[b]);
                    }
                }
            }
            float v[RB];
#pragma unroll
            for (uint32_t b = 0; b < RB; b++) {
                float p0, p1;
                unpack2(acc[b], &p0, &p1);
                v[b] = p0 + p1;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (uint32_t b = 0; b < RB; b++) v[b] += __shfl_xor_sync(0xffffffffu, v[b], o);
            if ((tg & 31) == 0)
#pragma unroll
                for (uint32_t b = 0; b < RB; b++)
                    if (ok[b]) part[(vr0 + G * b) * WG + wig] = v[b];
        }
        __syncthreads();
        if (t == 0) tr.mark(4);
        // Combine each row's warp partials in warp order, then the epilogue.
        const uint32_t base_row = t * a.rt;
        if (OUT == OUT_SILU) {
            if (tid < a.rt && base_row + tid < mine) {
                float gv = 0.0f, uv = 0.0f;
                for (uint32_t w = 0; w < WG; w++) {
                    gv += part[tid * WG + w];
                    uv += part[(a.rt + tid) * WG + w];
                }
                a.dst[r0 + base_row + tid] = __fmul_rn(ref_silu(gv), uv);
            }
        } else if (tid < a.rt && base_row + tid < mine) {
            float v = 0.0f;
            for (uint32_t w = 0; w < WG; w++) v += part[tid * WG + w];
            const uint32_t row = r0 + base_row + tid;
            if (OUT == OUT_STORE) {
                if (a.bias) v = __fadd_rn(v, t == 0 ? bias_s[tid] : a.bias[row]);
                a.dst[row] = v;
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

template <int OUT, int CMAX>
cudaError_t launch_fast_t(const GemvPlan& p, const GemvArgs& a, cudaStream_t st) {
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
    return cudaLaunchKernelEx(&cfg, k_gemv_fast<OUT, CMAX>, p.tm0, p.tm1, a, p.in_mode);
}

template <typename K>
cudaError_t allow_smem_fast(K kernel, int optin) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
}

}  // namespace

// Chunks per thread the fast GEMV instantiates (registers hold 8*CMAX floats of x).
uint32_t fast_cmax_for(uint32_t chunks_per_thread) {
    const uint32_t opts[] = {1, 2, 3, 4, 5, 6, 8};
    for (uint32_t c : opts)
        if (chunks_per_thread <= c) return c;
    return 0;
}

cudaError_t fast_set_smem_limits(int optin) {
    cudaError_t e = cudaSuccess;
#define HS_SETF(O, C) \
    if (e == cudaSuccess) e = allow_smem_fast(k_gemv_fast<O, C>, optin);
#define HS_SETF_ALL(O) HS_SETF(O, 1) HS_SETF(O, 2) HS_SETF(O, 3) HS_SETF(O, 4) HS_SETF(O, 5) HS_SETF(O, 6) HS_SETF(O, 8)
    HS_SETF_ALL(OUT_STORE) HS_SETF_ALL(OUT_RESID) HS_SETF_ALL(OUT_SILU)
#undef HS_SETF_ALL
#undef HS_SETF
    return e;
}

cudaError_t launch_gemv_fast(const GemvPlan& p, const GemvArgs& a, cudaStream_t st) {
#define HS_CASE(O, C) \
    case O * 16 + C: return launch_fast_t<O, C>(p, a, st);
    switch (p.out_mode * 16 + p.cmax) {
        HS_CASE(OUT_STORE, 1) HS_CASE(OUT_STORE, 2) HS_CASE(OUT_STORE, 3) HS_CASE(OUT_STORE, 4)
        HS_CASE(OUT_STORE, 5) HS_CASE(OUT_STORE, 6) HS_CASE(OUT_STORE, 8)
        HS_CASE(OUT_RESID, 1) HS_CASE(OUT_RESID, 2) HS_CASE(OUT_RESID, 3) HS_CASE(OUT_RESID, 4)
        HS_CASE(OUT_RESID, 5) HS_CASE(OUT_RESID, 6) HS_CASE(OUT_RESID, 8)
        HS_CASE(OUT_SILU, 1) HS_CASE(OUT_SILU, 2) HS_CASE(OUT_SILU, 3) HS_CASE(OUT_SILU, 4)
        HS_CASE(OUT_SILU, 5) HS_CASE(OUT_SILU, 6) HS_CASE(OUT_SILU, 8)
        default: return cudaErrorInvalidValue;
    }
#undef HS_CASE
}

}  // namespace hs
