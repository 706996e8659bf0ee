// RMSNorm of the tensor-core token loop (numeric path HS_NUMERIC_TC),
// between the GEMMs of batch_tc.cu (attention is attn_split.cu):
//
//   k_tc_norm  one CTA per sequence: finishes the residual stream (embedding
//              row at layer 0, or x += the split-K partial sums of the
//              previous O / down GEMM, added in split order), then RMSNorm,
//              written as the f16 hi/lo pair the next GEMM reads
//              (model.rs:247-250, 308-321; math.rs:200-207).
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
// of B partials at a time (up to 24) are issued before the first add so they
// overlap in one round trip.
template <uint32_t B>
__device__ __forceinline__ float4 sum_parts(const float* base, uint64_t stride, uint32_t n) {
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (uint32_t s0 = 0; s0 < n; s0 += B) {
        float4 v[B];
#pragma unroll
        for (uint32_t j = 0; j < B; j++)
            if (s0 + j < n) v[j] = __ldcg(reinterpret_cast<const float4*>(base + (s0 + j) * stride));
#pragma unroll
        for (uint32_t j = 0; j < B; j++)
            if (s0 + j < n) acc = f4add(acc, v[j]);
    }
    return acc;
}

// ---------------------------------------------------------------- RMSNorm
// Thread t owns the float4 chunks t and t + 256 of the row. B: partials
// loaded per round (24 for the many-split decode GEMMs; 8 keeps a CTA small
// enough for several per SM when a prompt pass launches one per token).
template <uint32_t B>
__device__ __forceinline__ void tc_norm_body(const TcNormArgs a) {
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
            if (a.n_part) x = f4add(x, sum_parts<B>(a.part + (size_t)slot * a.d + 4 * c, a.part_stride, a.n_part));
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

// The decode path's many-split consumers (one CTA per sequence, few CTAs),
// and the prompt pass's few-split ones held to 64 registers (four CTAs per SM
// for one CTA per token).
__global__ void __launch_bounds__(kNormThreads) k_tc_norm24(const TcNormArgs a) { tc_norm_body<24>(a); }
__global__ void __launch_bounds__(kNormThreads, 4) k_tc_norm8(const TcNormArgs a) { tc_norm_body<8>(a); }

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

cudaError_t launch_tc_norm(const TcNormArgs& a, uint32_t slots, cudaStream_t st) {
    if (a.d % 4 || a.d > kNormThreads * kNormMaxChunks * 4 || a.n_part > kMaxParts) return cudaErrorInvalidValue;
    TcNormArgs c = a;
    void* args[] = {&c};
    const void* fn = a.n_part > 8 ? reinterpret_cast<const void*>(k_tc_norm24) : reinterpret_cast<const void*>(k_tc_norm8);
    return launch_pdl(fn, dim3(slots), dim3(kNormThreads), 0, st, args);
}

}  // namespace hs
