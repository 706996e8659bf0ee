// The perplexity harness's per-token score (hs-engine examples/ppl.rs:35-43)
// on the device: the negative log-likelihood of the next token under a row
// of logits, max-shifted: the maximum (f32::max semantics: a NaN operand is
// skipped), the sum of exp_f32(l - max) in f64, then
// -((l[next] - max) - ln(sum)) in f64. The sum runs in a fixed tree order
// (per-thread strided f64 sums, then a fixed xor tree and the warps in
// order), so a row gives the same bits on any B200; it differs from the
// reference's sequential f64 sum only by f64 rounding.
#include <cfloat>

#include "common.h"
#include "kernels.h"

namespace hs {
namespace {

constexpr uint32_t kNllThreads = 1024;

__global__ void __launch_bounds__(kNllThreads) k_logits_nll(const float* logits, uint64_t stride,
                                                            const uint32_t* next, uint32_t vocab, double* out) {
    __shared__ float wmax[32];
    __shared__ double wsum[32];
    const float* l = logits + (size_t)blockIdx.x * stride;
    const uint32_t tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    float mx = -INFINITY;
    for (uint32_t i = tid; i < vocab; i += kNllThreads) mx = fmaxf(mx, l[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) wmax[w] = mx;
    __syncthreads();
    mx = wmax[0];
    for (uint32_t i = 1; i < kNllThreads / 32; i++) mx = fmaxf(mx, wmax[i]);
    double s = 0.0;
    for (uint32_t i = tid; i < vocab; i += kNllThreads) s += (double)ref_exp(__fsub_rn(l[i], mx));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) wsum[w] = s;
    __syncthreads();
    if (tid == 0) {
        double sum = 0.0;
        for (uint32_t i = 0; i < kNllThreads / 32; i++) sum += wsum[i];
        const uint32_t t = next[blockIdx.x];
        const float lt = t < vocab ? l[t] : NAN;
        out[blockIdx.x] = -((double)__fsub_rn(lt, mx) - log(sum));
    }
}

}  // namespace

cudaError_t launch_logits_nll(const float* logits, uint64_t stride, const uint32_t* next, uint32_t rows,
                              uint32_t vocab, double* out, cudaStream_t st) {
    if (rows == 0) return cudaSuccess;
    k_logits_nll<<<rows, kNllThreads, 0, st>>>(logits, stride, next, vocab, out);
    return cudaGetLastError();
}

}  // namespace hs
