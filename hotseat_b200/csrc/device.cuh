// Device-side building blocks shared by the kernels: exact IEEE helpers that
// restate hotseat's numerics (crates/hs-engine/src/math.rs, f16.rs), the
// xoshiro256** stream (sampler.rs:47-80), and thin PTX wrappers for mbarrier,
// TMA and programmatic dependent launch on sm_100a.
//
// Every float operation that must match the reference bit for bit is written
// with an explicit round-to-nearest intrinsic (__fmul_rn, __fadd_rn, ...), so
// nvcc can never contract a multiply and an add into one FMA; the library is
// also built with -fmad=false.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hs {

// Error bits a kernel may set in DevCtl::err (read back by the host).
enum : uint32_t {
    ERR_TIMEOUT = 1u,     // a bounded wait ran out
    ERR_TOKEN = 2u,       // token id >= vocab
    ERR_POS = 4u,         // pos >= max_ctx
    ERR_CAP = 8u,         // token history buffer full
    ERR_INVARIANT = 16u,  // filled >= n_tokens at a token boundary (seq.rs:258-266)
};

// Device control block of one decode thread (hs_scratch): the step the
// forward kernels run, and the SeqState + sampler state the commit kernel
// advances (seq.rs:35-61, sampler.rs:38-44).
struct DevCtl {
    uint32_t token, pos, active, mode;  // mode 0: seq commit; 1: sample only
    uint64_t n_tokens, filled, prompt_len, max_tokens, cap, stop_at;
    uint32_t done, done_reason, out_token, err;
    uint64_t rng[4];
    uint64_t draws;
    float temperature, top_p, repeat_penalty;
    uint32_t top_k, repeat_last_n;
    uint32_t eos, max_ctx, vocab, err_info;
};

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h_rn(float f) { return __half_as_ushort(__float2half_rn(f)); }

// 2^k from the exponent field (math.rs:65-75).
__device__ __forceinline__ float pow2i(int k) {
    int e = k + 127;
    if (e <= 0) return e <= -23 ? 0.0f : __uint_as_float(1u << (22 + e));
    return __uint_as_float((uint32_t)e << 23);
}

// exp_f32 (math.rs:39-61), operation for operation.
__device__ __forceinline__ float ref_exp(float x) {
    if (isnan(x)) return x;
    if (x >= 89.0f) return __int_as_float(0x7f800000);
    if (x <= -104.0f) return 0.0f;
    float kf = roundf(__fmul_rn(x, 1.44269504f));  // half away from zero, like Rust round()
    float r = __fsub_rn(__fsub_rn(x, __fmul_rn(kf, 0.693359375f)), __fmul_rn(kf, -2.1219444e-4f));
    float p = __fadd_rn(0.00833333f, __fmul_rn(r, 0.001388889f));
    p = __fadd_rn(0.04166667f, __fmul_rn(r, p));
    p = __fadd_rn(0.16666667f, __fmul_rn(r, p));
    p = __fadd_rn(0.5f, __fmul_rn(r, p));
    p = __fadd_rn(1.0f, __fmul_rn(r, p));
    p = __fadd_rn(1.0f, __fmul_rn(r, p));
    int k = (int)kf;
    int k1 = k >> 1;
    return __fmul_rn(__fmul_rn(p, pow2i(k1)), pow2i(k - k1));
}

// silu (math.rs:79-81): x / (1 + e^-x).
__device__ __forceinline__ float ref_silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, ref_exp(-x))); }

// xoshiro256** (sampler.rs:60-80).
__device__ __forceinline__ uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }
__device__ __forceinline__ uint64_t rng_next(uint64_t* s) {
    uint64_t result = rotl64(s[1] * 5ull, 7) * 9ull;
    uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl64(s[3], 45);
    return result;
}

// Key that sorts ascending as (value descending by f32::total_cmp, id
// ascending): the order of cmp_desc (sampler.rs:170-175).
__device__ __forceinline__ uint64_t cand_key(float v, uint32_t id) {
    int32_t b = __float_as_int(v);
    b ^= (int32_t)(((uint32_t)(b >> 31)) >> 1);  // total_cmp's integer image
    uint32_t u = (uint32_t)b ^ 0x80000000u;      // as unsigned, same order
    return ((uint64_t)(~u) << 32) | id;
}
__device__ __forceinline__ float key_value(uint64_t k) {
    uint32_t u = ~(uint32_t)(k >> 32);
    int32_t b = (int32_t)(u ^ 0x80000000u);
    b ^= (int32_t)(((uint32_t)(b >> 31)) >> 1);
    return __int_as_float(b);
}

// ---- PTX wrappers ---------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: gives up after `limit` polls (each poll itself suspends for a
// hardware-chosen interval) and reports false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t limit = 1u << 24) {
    for (uint32_t i = 0; i < limit; i++)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 2-D tiled TMA load (no multicast) of box {x: 64 cols, y: rows} into smem.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
// 1-D bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// 16-byte asynchronous copy global -> shared (completion via cp.async.wait_all).
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src))
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Programmatic dependent launch: let the next kernel in the stream start its
// prologue (weight prefetch) now; wait until the previous kernel finished.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Optional launch timeline (trace mode): per launch slot, 8 u64 of
// %globaltimer ns: [first CTA entry (min), CTA 0 past the PDL wait,
// last CTA exit (max), last CTA entry (max), checkpoints 1-4 (max over CTAs)].
__device__ __forceinline__ uint64_t gtime() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
struct KTrace {
    uint64_t* p;
    __device__ __forceinline__ KTrace(uint64_t* base, uint32_t slot) : p(base ? base + 8 * slot : nullptr) {}
    __device__ __forceinline__ void enter() const {
        if (p && threadIdx.x == 0) {
            const unsigned long long t = gtime();
            atomicMin(reinterpret_cast<unsigned long long*>(p), t);
            atomicMax(reinterpret_cast<unsigned long long*>(p + 3), t);
        }
    }
    __device__ __forceinline__ void waited() const {
        if (p && threadIdx.x == 0 && blockIdx.x == 0) p[1] = gtime();
    }
    __device__ __forceinline__ void mark(int i) const {
        if (p && threadIdx.x == 0) atomicMax(reinterpret_cast<unsigned long long*>(p + 3 + i), (unsigned long long)gtime());
    }
    __device__ __forceinline__ void exit() const {
        if (p && threadIdx.x == 0) atomicMax(reinterpret_cast<unsigned long long*>(p + 2), (unsigned long long)gtime());
    }
};

// Packed pairs of f32 (sm_100 f32x2 ALU ops). The packed multiply is exact
// lane-wise IEEE; the adds stay scalar add.rn, which is never contracted, so
// `acc + w*x` keeps its two roundings. (A packed multiply feeding only a
// packed add can be fused into a packed FMA by the assembler, which would
// change the bits; this form avoids it.)
__device__ __forceinline__ uint64_t pack2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float* a, float* b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(*a), "=f"(*b) : "l"(v));
}
__device__ __forceinline__ void mul_add_pair(float* acc0, float* acc1, uint64_t w, uint64_t x) {
    uint64_t p;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(p) : "l"(w), "l"(x));
    float p0, p1;
    unpack2(p, &p0, &p1);
    *acc0 = __fadd_rn(*acc0, p0);
    *acc1 = __fadd_rn(*acc1, p1);
}

// pool.rs:139-145 split: contiguous balanced ranges.
__device__ __forceinline__ void split_range(uint32_t rows, uint32_t n, uint32_t tid, uint32_t* a, uint32_t* b) {
    uint32_t per = rows / n, rem = rows % n;
    uint32_t start = tid * per + (tid < rem ? tid : rem);
    *a = start;
    *b = start + per + (tid < rem ? 1u : 0u);
}

}  // namespace hs
