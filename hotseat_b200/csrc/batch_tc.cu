// Tensor-core token loop (numeric path HS_NUMERIC_TC): the same layer as
// decode.cu / decode_fast.cu, computed for up to 128 sequences at once.
//
// Every matrix product of the layer (QKV+bias, O+residual, gate/up+SiLU,
// down+residual, tied LM head) is one tcgen05 GEMM
//
//     D[slot][row] = sum_k A[slot][k] * W[row][k]
//
// with A = the activations of all sequences (M = 128 slots, K-major f16,
// rows past the live slots ignored) and B = a tile of weight rows (N = 16..256
// rows, K-major f16 exactly as dequantised). Operands arrive by TMA
// (SWIZZLE_128B, 64-column boxes) into a ring of shared-memory stages; one
// thread issues tcgen05.mma into a TMEM accumulator (two buffers, so the
// epilogue of one weight tile overlaps the MMAs of the next); four warps read
// TMEM back with tcgen05.ld and apply the fused epilogue.
//
// Activations are f32 in the reference. The f16 tensor-core operands carry
// them as a pair hi = f16(x), lo = f16(x - hi) and every k-step issues two
// MMAs into the same f32 accumulator (W*hi + W*lo): products are exact in
// f32 and the pair holds ~22 significant bits of x, so the result tracks the
// f32 GEMV to accumulation-order rounding.
//
// A sequence's results depend only on its own activation row and the model
// (every accumulator element is formed the same way whatever the slot or the
// batch size), so a sequence decoded alone, in a batch of 64, or after a
// migration to another B200 produces the same bits.
#include <cfloat>

#include "common.h"
#include "kernels.h"

namespace hs {
namespace {

// ---------------------------------------------------------------- tcgen05 PTX

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D (TMEM) (+)= A (smem desc) x B (smem desc); kind::f16, both operands f16.
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on an mbarrier once every MMA this thread issued so far completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* m) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (the layout a 64-column SWIZZLE_128B TMA box writes).
__device__ __forceinline__ uint64_t sw128_desc(const void* p) {
    const uint64_t addr = smem_u32(p);
    return ((addr >> 4) & 0x3FFFull) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor: D f32, A and B f16, both K-major, M x N.
__host__ __device__ constexpr uint32_t tc_idesc(uint32_t m, uint32_t n) {
    return (1u << 4) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__device__ __forceinline__ void split_f16(float x, uint16_t* hi, uint16_t* lo) {
    const __half h = __float2half_rn(x);
    *hi = __half_as_ushort(h);
    *lo = __half_as_ushort(__float2half_rn(__fsub_rn(x, __half2float(h))));
}

// TMEM accumulator arrangement for an N-column tile: `nacc` independent
// accumulators (quarter kk of every 64-wide k-step feeds accumulator
// kk % nacc, so consecutive MMAs do not wait on each other) times `nbuf`
// tile buffers (the epilogue of one tile overlaps the MMAs of the next).
// `ncols` covers the farthest 32-column epilogue load; a power of two.
struct TcAcc {
    uint32_t nacc, nbuf, ncols;
};
// A CTA that owns several tiles prefers two buffers; one with a single tile
// prefers more accumulators.
__host__ __device__ inline TcAcc tc_acc(uint32_t nmat, uint32_t nt, bool multi) {
    const uint32_t n = nmat * nt, r32 = (nt + 31) / 32 * 32;
    const uint32_t opts_multi[6][2] = {{4, 2}, {2, 2}, {1, 2}, {4, 1}, {2, 1}, {1, 1}};
    const uint32_t opts_single[6][2] = {{4, 1}, {2, 1}, {1, 1}, {1, 1}, {1, 1}, {1, 1}};
    for (int i = 0; i < 6; i++) {
        const uint32_t na = multi ? opts_multi[i][0] : opts_single[i][0];
        const uint32_t nb = multi ? opts_multi[i][1] : opts_single[i][1];
        const uint32_t reach = (nb - 1) * na * n + (na - 1) * n + (nmat - 1) * nt + r32;
        const uint32_t need = nb * na * n > reach ? nb * na * n : reach;
        if (need <= 512) {
            uint32_t c = 32;
            while (c < need) c <<= 1;
            return TcAcc{na, nb, c};
        }
    }
    return TcAcc{0, 0, 0};
}

// Trace checkpoint i (1-4) from any thread: latest time over CTAs.
__device__ __forceinline__ void tr_mark(uint64_t* trace, uint32_t slot, int i) {
    if (trace) atomicMax(reinterpret_cast<unsigned long long*>(trace + 8 * slot + 3 + i), (unsigned long long)gtime());
}

// 32 consecutive 32-bit TMEM columns of this thread's lane; complete at tmem_wait().
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Named barrier for the four epilogue warps only.
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Sum of this lane's 32 columns over the tile's accumulators, in a fixed
// order: ((a0 + a1) + (a2 + a3)).
__device__ __forceinline__ void acc_sum32(uint32_t taddr, uint32_t stride, uint32_t nacc, float* out) {
    uint32_t r0[32], r1[32];
    tmem_ld32(taddr, r0);
    if (nacc > 1) tmem_ld32(taddr + stride, r1);
    tmem_wait();
    if (nacc == 1) {
#pragma unroll
        for (int j = 0; j < 32; j++) out[j] = __uint_as_float(r0[j]);
        return;
    }
#pragma unroll
    for (int j = 0; j < 32; j++) out[j] = __fadd_rn(__uint_as_float(r0[j]), __uint_as_float(r1[j]));
    if (nacc == 4) {
        tmem_ld32(taddr + 2 * stride, r0);
        tmem_ld32(taddr + 3 * stride, r1);
        tmem_wait();
#pragma unroll
        for (int j = 0; j < 32; j++)
            out[j] = __fadd_rn(out[j], __fadd_rn(__uint_as_float(r0[j]), __uint_as_float(r1[j])));
    }
}

// SiLU for the tensor-core path: x / (1 + e^-x) with the fast exponential
// (a fixed instruction sequence, so the same bits on every B200).
__device__ __forceinline__ float tc_silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

constexpr uint32_t kTcThreads = 192;  // warps 0-3 epilogue, warp 4 TMA, warp 5 MMA
constexpr uint32_t kLimit = 1u << 24;
constexpr uint32_t kMaxStages = 16;
constexpr uint32_t kXchgStride = 33;  // floats per slot row of the hi/lo exchange buffer

// ---------------------------------------------------------------- GEMM
// One MMA covers 64 slots twice: A rows 0-63 are the hi halves and rows
// 64-127 the lo halves of the same 64 activation rows, so D lanes 0-63 hold
// W*hi and lanes 64-127 hold W*lo, summed in the epilogue. For the SiLU
// epilogue the B operand stacks the gate tile over the up tile (N = 2*nt).
//
// Work unit = (weight-row tile of n_tile rows, K split). A CTA takes units
// blockIdx.x, +gridDim.x, ...; blockIdx.y picks the 64-slot group. With
// m_loop (prompt passes: many 64-slot groups) the grid is one row and a CTA
// walks items = (unit, group) i = blockIdx.x, +gridDim.x, ... (unit i %
// units, group i / units), so the CTAs sweep the groups together and each
// item's epilogue overlaps the next item's MMAs.
// Shared memory: [nst stages: A hi | A lo | W0 (| W1)][xchg][barriers][tmem slot].
template <int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_tc_gemm(const __grid_constant__ CUtensorMap tm_ahi, const __grid_constant__ CUtensorMap tm_alo,
              const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
              const TcGemmArgs a) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    constexpr uint32_t NMAT = EPI == TC_SILU ? 2 : 1;
    constexpr uint32_t a_half = 64 * 128;           // one 64-column box of 64 slots
    const uint32_t nt = a.n_tile, N = NMAT * nt;
    const uint32_t w_bytes = nt * 128;              // one 64-column box of nt rows
    const bool wres = a.wres != 0;
    // stages: activation boxes (+ weight boxes unless resident)
    const uint32_t stage_bytes = 2 * a_half + (wres ? 0 : NMAT * w_bytes);
    const uint32_t nst = a.nst;
    const uint32_t kw = wres ? (a.K / 64 + a.splits - 1) / a.splits : 0;  // resident k-blocks
    uint8_t* wreg = smem + nst * stage_bytes;       // resident weight boxes, NMAT per k-block
    float* xchg = reinterpret_cast<float*>(wreg + kw * NMAT * w_bytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(xchg + 64 * kXchgStride * NMAT + 2);
    uint64_t* full = bars;
    uint64_t* empty = bars + nst;
    uint64_t* tfull = bars + 2 * nst;
    uint64_t* tempty = tfull + 2;
    uint64_t* wfull = tempty + 2;                   // resident weights landed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(wfull + 1);
    volatile uint32_t* epi_flag = tmem_slot + 1;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const KTrace tr(a.trace, a.trace_slot);
    tr.enter();

    const uint32_t kt_n = a.K / 64, S = a.splits, n_units = a.n_tiles * S;
    const uint32_t n_items = a.m_loop ? n_units * ((a.slots + 63) / 64) : n_units;
    auto item_m0 = [&](uint32_t i) -> uint32_t { return a.m_loop ? i / n_units * 64 : blockIdx.y * 64; };
    // The accumulator arrangement sets the order of a tile's sums, so it must
    // not depend on the pass: walking CTAs always take the several-items form.
    const TcAcc acc = tc_acc(NMAT, nt, a.m_loop ? true : n_items > gridDim.x);
    const uint32_t buf_cols = acc.nacc * N;
    auto k_range = [&](uint32_t split, uint32_t* k0, uint32_t* k1) {
        *k0 = split * kt_n / S;
        *k1 = (split + 1) * kt_n / S;
    };
    uint32_t total_its = 0;
    for (uint32_t i = blockIdx.x; i < n_items; i += gridDim.x) {
        uint32_t k0, k1;
        k_range(i % n_units % S, &k0, &k1);
        total_its += k1 - k0;
    }

    if (tid == 0) {
        for (uint32_t s = 0; s < nst; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 128);
        }
        mbar_init(wfull, 1);
        mbar_init_fence();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, acc.ncols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 4) {
        // TMA producer. Weight boxes do not depend on earlier kernels, so the
        // first nst stages' weights are requested before the dependency wait
        // and their activation boxes right after it.
        pdl_launch_dependents();
        if (lane == 0) {
            prefetch_tmap(&tm_w0);
            if (NMAT == 2) prefetch_tmap(&tm_w1);
            prefetch_tmap(&tm_ahi);
            prefetch_tmap(&tm_alo);
            uint32_t it = 0, deferred[kMaxStages], deferred_m[kMaxStages];
            bool waited = false;
            auto a_load = [&](uint32_t s, uint32_t kt, uint32_t m0) {
                uint8_t* st = smem + s * stage_bytes;
                tma_load_2d(st, &tm_ahi, (int)(kt * 64), (int)m0, &full[s]);
                tma_load_2d(st + a_half, &tm_alo, (int)(kt * 64), (int)m0, &full[s]);
            };
            if (wres) {
                // The CTA's one unit: all its weight boxes now, then the
                // activation boxes through the ring after the wait.
                const uint32_t u = blockIdx.x;
                if (u < n_units) {
                    const uint32_t tile = u / S;
                    uint32_t k0, k1;
                    k_range(u % S, &k0, &k1);
                    mbar_expect_tx(wfull, (k1 - k0) * NMAT * w_bytes);
                    for (uint32_t kt = k0; kt < k1; kt++) {
                        uint8_t* dst = wreg + (kt - k0) * NMAT * w_bytes;
                        tma_load_2d(dst, &tm_w0, (int)(kt * 64), (int)(tile * nt), wfull);
                        if (NMAT == 2) tma_load_2d(dst + w_bytes, &tm_w1, (int)(kt * 64), (int)(tile * nt), wfull);
                    }
                    pdl_wait();
                    if (a.trace && blockIdx.x == 0 && blockIdx.y == 0) a.trace[8 * a.trace_slot + 1] = gtime();
                    for (uint32_t kt = k0; kt < k1; kt++, it++) {
                        const uint32_t s = it % nst, r = it / nst;
                        if (r > 0 && !mbar_wait_bounded(&empty[s], (r - 1) & 1, kLimit)) {
                            ok = false;
                            break;
                        }
                        mbar_expect_tx(&full[s], stage_bytes);
                        a_load(s, kt, item_m0(u));
                    }
                }
                waited = true;
            }
            for (uint32_t i = blockIdx.x; i < n_items && ok && !wres; i += gridDim.x) {
                const uint32_t u = i % n_units, tile = u / S, m0 = item_m0(i);
                uint32_t k0, k1;
                k_range(u % S, &k0, &k1);
                for (uint32_t kt = k0; kt < k1; kt++, it++) {
                    const uint32_t s = it % nst, r = it / nst;
                    if (r > 0 && !mbar_wait_bounded(&empty[s], (r - 1) & 1, kLimit)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&full[s], stage_bytes);
                    uint8_t* st = smem + s * stage_bytes + 2 * a_half;
                    tma_load_2d(st, &tm_w0, (int)(kt * 64), (int)(tile * nt), &full[s]);
                    if (NMAT == 2) tma_load_2d(st + w_bytes, &tm_w1, (int)(kt * 64), (int)(tile * nt), &full[s]);
                    if (waited) {
                        a_load(s, kt, m0);
                    } else {
                        deferred[it] = kt;
                        deferred_m[it] = m0;
                        if (it + 1 == nst || it + 1 == total_its) {
                            pdl_wait();
                            if (a.trace && blockIdx.x == 0 && blockIdx.y == 0) a.trace[8 * a.trace_slot + 1] = gtime();
                            waited = true;
                            for (uint32_t j = 0; j <= it; j++) a_load(j, deferred[j], deferred_m[j]);
                        }
                    }
                }
            }
            if (!waited) pdl_wait();
        }
    } else if (warp == 5) {
        pdl_launch_dependents();
        if (lane == 0) {
            const uint32_t idesc = tc_idesc(128, N);
            uint32_t it = 0, t = 0;
            if (wres && blockIdx.x < n_units && !mbar_wait_bounded(wfull, 0, kLimit)) ok = false;
            for (uint32_t i = blockIdx.x; i < n_items && ok; i += gridDim.x, t++) {
                const uint32_t u = i % n_units;
                const uint32_t b = t % acc.nbuf, use = t / acc.nbuf;
                if (use > 0 && !mbar_wait_bounded(&tempty[b], (use - 1) & 1, kLimit)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t dbase = tmem + b * buf_cols;
                uint32_t k0, k1;
                k_range(u % S, &k0, &k1);
                for (uint32_t kt = k0; kt < k1; kt++, it++) {
                    const uint32_t s = it % nst, r = it / nst;
                    if (!mbar_wait_bounded(&full[s], r & 1, kLimit)) {
                        ok = false;
                        break;
                    }
                    if (it == 0) tr_mark(a.trace, a.trace_slot, 1);
                    tc_fence_after();
                    const uint8_t* st = smem + s * stage_bytes;
                    const uint64_t da = sw128_desc(st);
                    const uint64_t dw = sw128_desc(wres ? wreg + (kt - k0) * NMAT * w_bytes : st + 2 * a_half);
#pragma unroll
                    for (uint32_t kk = 0; kk < 4; kk++) {
                        // +32 bytes along K per 16-element step, inside the swizzle atom
                        const uint32_t ai = kk % acc.nacc;
                        const uint32_t first = (kt == k0 && kk < acc.nacc) ? 1u : 0u;
                        tc_mma(dbase + ai * N, da + 2 * kk, dw + 2 * kk, idesc, first ? 0u : 1u);
                    }
                    tc_commit(&empty[s]);
                }
                if (ok) tc_commit(&tfull[b]);
                tr_mark(a.trace, a.trace_slot, 2);
            }
        }
    } else {
        // Epilogue warps 0-3: warp w reads TMEM lanes 32w..32w+31. Warps 0-1
        // hold W*hi for slots m0+32w+lane, warps 2-3 hold W*lo for slots
        // m0+32(w-2)+lane; the lo warps hand their sums over through `xchg`.
        pdl_launch_dependents();
        pdl_wait();
        const bool hi_warp = warp < 2;
        const uint32_t sl = (warp & 1) * 32 + lane;  // slot within the 64-slot group
        const bool vec = (a.ld & 3) == 0;
        uint32_t t = 0;
        for (uint32_t i = blockIdx.x; i < n_items; i += gridDim.x, t++) {
            const uint32_t u = i % n_units, slot = item_m0(i) + sl;
            const bool live = slot < a.slots;
            const uint32_t b = t % acc.nbuf, use = t / acc.nbuf;
            // One thread waits; the named barrier makes the outcome (and the
            // accumulator) visible to all four warps, which then leave or
            // continue together, so no warp is left alone at a barrier.
            if (tid == 0) *epi_flag = mbar_wait_bounded(&tfull[b], use & 1, kLimit) ? 1u : 0u;
            epi_sync();
            if (!*epi_flag) {
                ok = false;
                break;
            }
            tc_fence_after();
            if (tid == 0) tr_mark(a.trace, a.trace_slot, 3);
            const uint32_t tile = u / S, split = u % S, row0 = tile * nt;
            const uint32_t tbase = tmem + ((warp * 32) << 16) + b * buf_cols;
            for (uint32_t c0 = 0; c0 < nt; c0 += 32) {
                float v[32], w[32];
                acc_sum32(tbase + c0, N, acc.nacc, v);
                if (EPI == TC_SILU) acc_sum32(tbase + nt + c0, N, acc.nacc, w);
                if (!hi_warp) {
                    float* x = xchg + sl * kXchgStride;
#pragma unroll
                    for (int j = 0; j < 32; j++) x[j] = v[j];
                    if (EPI == TC_SILU) {
                        float* xu = xchg + (64 + sl) * kXchgStride;
#pragma unroll
                        for (int j = 0; j < 32; j++) xu[j] = w[j];
                    }
                }
                epi_sync();
                if (hi_warp) {
                    const float* x = xchg + sl * kXchgStride;
#pragma unroll
                    for (int j = 0; j < 32; j++) v[j] = __fadd_rn(v[j], x[j]);
                    if (EPI == TC_SILU) {
                        const float* xu = xchg + (64 + sl) * kXchgStride;
#pragma unroll
                        for (int j = 0; j < 32; j++) w[j] = __fadd_rn(w[j], xu[j]);
                    }
                    const uint32_t cn = nt - c0 < 32 ? nt - c0 : 32;
#pragma unroll
                    for (uint32_t c8 = 0; c8 < 32; c8 += 8) {
                        const uint32_t row = row0 + c0 + c8;
                        if (!live || c8 >= cn || row >= a.rows) break;
                        const uint32_t nv = a.rows - row < 8 ? a.rows - row : 8;
                        if (EPI == TC_SILU) {
                            uint16_t hi[8], lo[8];
#pragma unroll
                            for (int j = 0; j < 8; j++) split_f16(__fmul_rn(tc_silu(v[c8 + j]), w[c8 + j]), &hi[j], &lo[j]);
                            uint16_t* ph = a.out_hi + (size_t)slot * a.ld + row;
                            uint16_t* pl = a.out_lo + (size_t)slot * a.ld + row;
                            if (nv == 8 && (a.ld & 7) == 0) {
                                uint4 h4, l4;
                                h4.x = hi[0] | (uint32_t)hi[1] << 16;
                                h4.y = hi[2] | (uint32_t)hi[3] << 16;
                                h4.z = hi[4] | (uint32_t)hi[5] << 16;
                                h4.w = hi[6] | (uint32_t)hi[7] << 16;
                                l4.x = lo[0] | (uint32_t)lo[1] << 16;
                                l4.y = lo[2] | (uint32_t)lo[3] << 16;
                                l4.z = lo[4] | (uint32_t)lo[5] << 16;
                                l4.w = lo[6] | (uint32_t)lo[7] << 16;
                                *reinterpret_cast<uint4*>(ph) = h4;
                                *reinterpret_cast<uint4*>(pl) = l4;
                            } else {
                                for (uint32_t j = 0; j < nv; j++) {
                                    ph[j] = hi[j];
                                    pl[j] = lo[j];
                                }
                            }
                        } else {
                            float* po = a.out + (EPI == TC_PART ? (size_t)split * a.part_stride : 0) +
                                        (size_t)slot * a.ld + row;
                            if (nv == 8 && vec) {
                                reinterpret_cast<float4*>(po)[0] =
                                    make_float4(v[c8], v[c8 + 1], v[c8 + 2], v[c8 + 3]);
                                reinterpret_cast<float4*>(po)[1] =
                                    make_float4(v[c8 + 4], v[c8 + 5], v[c8 + 6], v[c8 + 7]);
                            } else {
                                for (uint32_t j = 0; j < nv; j++) po[j] = v[c8 + j];
                            }
                        }
                    }
                }
                epi_sync();
            }
            tc_fence_before();
            mbar_arrive(&tempty[b]);
        }
        if (tid == 0) tr_mark(a.trace, a.trace_slot, 4);
    }
    if (!ok) atomicOr(a.err, ERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, acc.ncols);
    tr.exit();
}

}  // namespace

size_t tc_gemm_smem(uint32_t n_tile, uint32_t nst, bool silu) {
    const uint32_t nmat = silu ? 2 : 1;
    const size_t stage = 2 * 64 * 128 + nmat * (size_t)n_tile * 128;
    return 1024 + nst * stage + (64 * kXchgStride * nmat + 2) * 4 + (2 * nst + 5) * 8 + 16;
}

size_t tc_gemm_smem_wres(uint32_t n_tile, uint32_t nst, bool silu, uint32_t kw) {
    const uint32_t nmat = silu ? 2 : 1;
    return 1024 + nst * (size_t)(2 * 64 * 128) + (size_t)kw * nmat * n_tile * 128 + (64 * kXchgStride * nmat + 2) * 4 +
           (2 * nst + 5) * 8 + 16;
}

bool tc_tile_ok(uint32_t n_tile, bool silu) {
    const uint32_t nmat = silu ? 2 : 1;
    return n_tile >= 8 && n_tile % 8 == 0 && nmat * n_tile <= 256 && nmat * n_tile % 16 == 0 &&
           tc_acc(nmat, n_tile, true).nacc != 0 && tc_acc(nmat, n_tile, false).nacc != 0;
}

cudaError_t tc_set_smem_limits(int optin) {
    cudaError_t e;
#define HS_TC_ATTR(K)                                                                                   \
    e = cudaFuncSetAttribute(K, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);                    \
    if (e != cudaSuccess) return e;
    HS_TC_ATTR(k_tc_gemm<TC_STORE>)
    HS_TC_ATTR(k_tc_gemm<TC_PART>)
    HS_TC_ATTR(k_tc_gemm<TC_SILU>)
#undef HS_TC_ATTR
    return cudaSuccess;
}

cudaError_t launch_tc_gemm(const TcGemmPlan& p, const CUtensorMap& ahi, const CUtensorMap& alo, const TcGemmArgs& a,
                           cudaStream_t st) {
    const bool silu = p.epi == TC_SILU;
    if (p.nst == 0 || p.nst > kMaxStages || !tc_tile_ok(p.n_tile, silu) || p.K % 64 || p.splits == 0 ||
        p.splits > p.K / 64 || (silu && p.splits != 1) || a.n_tile != p.n_tile || a.splits != p.splits ||
        a.nst != p.nst || a.K != p.K || a.wres != (p.wres ? 1u : 0u) ||
        (p.wres && p.n_tiles * p.splits > p.grid) ||  // weights resident: one unit per CTA
        a.m_loop != (p.m_loop ? 1u : 0u) || (p.m_loop && (p.wres || p.m_tiles != 1)))
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(p.grid, p.m_tiles);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    switch (p.epi) {
        case TC_STORE: return cudaLaunchKernelEx(&cfg, k_tc_gemm<TC_STORE>, ahi, alo, p.tm0, p.tm1, a);
        case TC_PART: return cudaLaunchKernelEx(&cfg, k_tc_gemm<TC_PART>, ahi, alo, p.tm0, p.tm1, a);
        case TC_SILU: return cudaLaunchKernelEx(&cfg, k_tc_gemm<TC_SILU>, ahi, alo, p.tm0, p.tm1, a);
    }
    return cudaErrorInvalidValue;
}

}  // namespace hs
