// Load-time dequantisation kernels: GGML block formats -> f16 bits, bit-exact
// with hotseat's quant.rs:18-206. Tensors are flat streams of blocks that may
// straddle rows (model.rs:375-396), so block b always lands at elements
// [b*QK, (b+1)*QK) of the output regardless of the row length.
//
// Roofline: HBM. Per element, Q4_K reads 144/256 B and writes 2 B; Q6_K reads
// 210/256 B and writes 2 B.
#include "common.h"
#include "device.cuh"

namespace hs {
namespace {

__device__ __forceinline__ float ld_half(const uint8_t* p) {
    return h2f((uint16_t)(p[0] | ((uint16_t)p[1] << 8)));
}

// scale_min_k4 (quant.rs:101-107).
__device__ __forceinline__ void scale_min(int j, const uint8_t* q, float* sc, float* m) {
    uint32_t s, mm;
    if (j < 4) {
        s = q[j] & 63;
        mm = q[j + 4] & 63;
    } else {
        s = (q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4);
        mm = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
    *sc = (float)s;
    *m = (float)mm;
}

// Q4_K: one warp per 144-byte super-block; lane t writes elements 8t..8t+7
// as one 16-byte store. quant.rs:109-139: v = d1*q - mm1 with d1 = d*sc,
// mm1 = dmin*m, rounded to f16 (RNE).
__global__ void __launch_bounds__(256) k_dequant_q4k(const uint8_t* __restrict__ src, uint16_t* __restrict__ dst,
                                                      uint64_t n_blocks) {
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x >> 5);
    for (uint64_t b = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < n_blocks; b += warps) {
        const uint8_t* blk = src + b * 144;
        float d = ld_half(blk), dmin = ld_half(blk + 2);
        int g = lane >> 3;             // 64-element group
        int o = (lane * 8) & 63;       // offset inside the group
        int hi = o >= 32;              // high nibbles carry the second sub-block
        float sc, m;
        scale_min(2 * g + hi, blk + 4, &sc, &m);
        float dd = __fmul_rn(d, sc), mm = __fmul_rn(dmin, m);
        uint2 qv = *reinterpret_cast<const uint2*>(blk + 16 + g * 32 + (o & 31));
        uint32_t q8[2] = {qv.x, qv.y};
        uint16_t out[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            uint32_t byte = (q8[i >> 2] >> ((i & 3) * 8)) & 0xff;
            uint32_t q = hi ? (byte >> 4) : (byte & 0x0f);
            out[i] = f2h_rn(__fsub_rn(__fmul_rn(dd, (float)q), mm));
        }
        uint4 w;
        w.x = out[0] | ((uint32_t)out[1] << 16);
        w.y = out[2] | ((uint32_t)out[3] << 16);
        w.z = out[4] | ((uint32_t)out[5] << 16);
        w.w = out[6] | ((uint32_t)out[7] << 16);
        *reinterpret_cast<uint4*>(dst + b * 256 + lane * 8) = w;
    }
}

// Q6_K: one warp per 210-byte super-block (quant.rs:178-206): element
// h*128 + c*32 + l takes its low nibble from ql[h*64 + l + 32*(c&1)] (nibble
// c>>1), its top two bits from qh[h*32 + l] (bits 2c), scale sc[h*8 + l/16 + 2c];
// v = (d * sc) * (q - 32).
__global__ void __launch_bounds__(256) k_dequant_q6k(const uint8_t* __restrict__ src, uint16_t* __restrict__ dst,
                                                      uint64_t n_blocks) {
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x >> 5);
    for (uint64_t b = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < n_blocks; b += warps) {
        const uint8_t* blk = src + b * 210;
        float d = ld_half(blk + 208);
        int h = lane >> 4, c = (lane >> 2) & 3, l0 = (lane & 3) * 8;
        float scv = (float)(int8_t)blk[192 + h * 8 + (l0 >> 4) + 2 * c];
        float ds = __fmul_rn(d, scv);
        const uint8_t* ql = blk + h * 64 + 32 * (c & 1) + l0;
        const uint8_t* qh = blk + 128 + h * 32 + l0;
        uint16_t out[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            uint32_t lo = (ql[i] >> (4 * (c >> 1))) & 0x0f;
            uint32_t hb = (qh[i] >> (2 * c)) & 3;
            int q = (int)(lo | (hb << 4)) - 32;
            out[i] = f2h_rn(__fmul_rn(ds, (float)q));
        }
        uint4 w;
        w.x = out[0] | ((uint32_t)out[1] << 16);
        w.y = out[2] | ((uint32_t)out[3] << 16);
        w.z = out[4] | ((uint32_t)out[5] << 16);
        w.w = out[6] | ((uint32_t)out[7] << 16);
        *reinterpret_cast<uint4*>(dst + b * 256 + lane * 8) = w;
    }
}

// The remaining formats, one thread per element (quant.rs:21-31, 64-96, 143-176).
__global__ void k_dequant_generic(uint32_t ty, const uint8_t* __restrict__ src, uint16_t* __restrict__ dst,
                                  uint64_t n) {
    uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += stride) {
        uint16_t r = 0;
        if (ty == 1) {
            r = (uint16_t)(src[2 * e] | ((uint16_t)src[2 * e + 1] << 8));
        } else if (ty == 0) {
            uint32_t u = (uint32_t)src[4 * e] | ((uint32_t)src[4 * e + 1] << 8) | ((uint32_t)src[4 * e + 2] << 16) |
                         ((uint32_t)src[4 * e + 3] << 24);
            r = f2h_rn(__uint_as_float(u));
        } else if (ty == 8) {  // Q8_0
            const uint8_t* blk = src + (e / 32) * 34;
            r = f2h_rn(__fmul_rn(ld_half(blk), (float)(int8_t)blk[2 + (e % 32)]));
        } else if (ty == 6) {  // Q5_0: byte j holds elements j and j+16
            const uint8_t* blk = src + (e / 32) * 22;
            uint32_t i = e % 32, j = i & 15;
            uint32_t qh = blk[2] | (blk[3] << 8) | (blk[4] << 16) | ((uint32_t)blk[5] << 24);
            uint32_t x;
            if (i < 16) x = (blk[6 + j] & 0x0F) | (((qh >> j) << 4) & 0x10);
            else x = (blk[6 + j] >> 4) | ((qh >> (j + 12)) & 0x10);
            r = f2h_rn(__fmul_rn(ld_half(blk), (float)((int)x - 16)));
        } else if (ty == 13) {  // Q5_K
            const uint8_t* blk = src + (e / 256) * 176;
            uint32_t i = e % 256, g = i / 64, within = i % 64, l = within % 32, hi = within >= 32;
            float sc, m;
            scale_min((int)(2 * g + hi), blk + 4, &sc, &m);
            float dd = __fmul_rn(ld_half(blk), sc), mm = __fmul_rn(ld_half(blk + 2), m);
            uint32_t qb = blk[48 + g * 32 + l];
            uint32_t q = hi ? (qb >> 4) : (qb & 0x0F);
            uint32_t bit = 1u << (2 * g + hi);
            if (blk[16 + l] & bit) q += 16;
            r = f2h_rn(__fsub_rn(__fmul_rn(dd, (float)q), mm));
        } else if (ty == 12) {  // Q4_K (scalar form, for odd sizes)
            const uint8_t* blk = src + (e / 256) * 144;
            uint32_t i = e % 256, g = i / 64, within = i % 64, l = within % 32, hi = within >= 32;
            float sc, m;
            scale_min((int)(2 * g + hi), blk + 4, &sc, &m);
            float dd = __fmul_rn(ld_half(blk), sc), mm = __fmul_rn(ld_half(blk + 2), m);
            uint32_t qb = blk[16 + g * 32 + l];
            r = f2h_rn(__fsub_rn(__fmul_rn(dd, (float)(hi ? qb >> 4 : qb & 0x0F)), mm));
        } else if (ty == 14) {  // Q6_K (scalar form)
            const uint8_t* blk = src + (e / 256) * 210;
            uint32_t i = e % 256, h = i / 128, c = (i % 128) / 32, l = i % 32;
            uint32_t lo = (blk[h * 64 + l + 32 * (c & 1)] >> (4 * (c >> 1))) & 0x0f;
            uint32_t hb = (blk[128 + h * 32 + l] >> (2 * c)) & 3;
            float ds = __fmul_rn(ld_half(blk + 208), (float)(int8_t)blk[192 + h * 8 + l / 16 + 2 * c]);
            r = f2h_rn(__fmul_rn(ds, (float)((int)(lo | (hb << 4)) - 32)));
        }
        dst[e] = r;
    }
}

}  // namespace

// Enqueue the dequantisation of n elements. Q4_K and Q6_K take the
// warp-per-block kernels when the source is 8-byte aligned.
int launch_dequant(uint32_t ty, const void* src, uint64_t n, void* dst, cudaStream_t st, int n_sm) {
    uint64_t be, bb;
    if (!ggml_block(ty, &be, &bb)) return fail(HS_E_UNSUPPORTED, "unknown ggml type " + std::to_string(ty));
    if (n % be) return fail(HS_E_ARG, "element count is not a whole number of blocks");
    if (n == 0) return HS_OK;
    const uint8_t* s = static_cast<const uint8_t*>(src);
    uint16_t* d = static_cast<uint16_t*>(dst);
    uint64_t nb = n / be;
    bool aligned16 = ((uintptr_t)dst & 15) == 0;
    if (ty == 12 && aligned16 && ((uintptr_t)src & 7) == 0) {
        uint64_t grid = (nb + 7) / 8;
        if (grid > (uint64_t)n_sm * 16) grid = (uint64_t)n_sm * 16;
        k_dequant_q4k<<<(unsigned)grid, 256, 0, st>>>(s, d, nb);
    } else if (ty == 14 && aligned16) {
        uint64_t grid = (nb + 7) / 8;
        if (grid > (uint64_t)n_sm * 16) grid = (uint64_t)n_sm * 16;
        k_dequant_q6k<<<(unsigned)grid, 256, 0, st>>>(s, d, nb);
    } else {
        uint64_t grid = (n + 255) / 256;
        if (grid > (uint64_t)n_sm * 32) grid = (uint64_t)n_sm * 32;
        k_dequant_generic<<<(unsigned)grid, 256, 0, st>>>(ty, s, d, n);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(HS_E_CUDA, std::string("dequant launch: ") + cudaGetErrorString(e));
    return HS_OK;
}

}  // namespace hs
