// KV byte-run transfers: one kernel moves a table of (source offset,
// destination offset, length) runs between two byte arrays. It serves the
// three data paths of a hand-over:
//   - gather of a region's runs into a packed staging buffer, read back to
//     the host in one copy (hs-wire send_page_bytes, lib.rs:338-361);
//   - scatter of a packed host buffer into a region (recv_page_bytes,
//     lib.rs:377-396);
//   - region to region, the destination on another GPU written through its
//     peer mapping over NVLink (the pre-copy rounds of migrate.rs:234-473
//     without the TCP hop).
// The host splits long runs into pieces of at most kXferPiece bytes, so a
// CTA per piece keeps every SM busy whatever the run lengths.
#include "common.h"
#include "kernels.h"

namespace hs {
namespace {

__global__ void __launch_bounds__(256) k_copy_runs(const uint8_t* src, uint8_t* dst, const XferRun* runs,
                                                   uint32_t n) {
    for (uint32_t r = blockIdx.x; r < n; r += gridDim.x) {
        const XferRun x = runs[r];
        const uint8_t* s = src + x.src_off;
        uint8_t* d = dst + x.dst_off;
        if ((((uintptr_t)s | (uintptr_t)d | x.len) & 15) == 0) {
            const uint4* s4 = reinterpret_cast<const uint4*>(s);
            uint4* d4 = reinterpret_cast<uint4*>(d);
            const uint32_t n4 = (uint32_t)(x.len / 16);
            for (uint32_t i = threadIdx.x; i < n4; i += blockDim.x) d4[i] = s4[i];
        } else if ((((uintptr_t)s | (uintptr_t)d | x.len) & 3) == 0) {
            const uint32_t* s1 = reinterpret_cast<const uint32_t*>(s);
            uint32_t* d1 = reinterpret_cast<uint32_t*>(d);
            for (uint32_t i = threadIdx.x; i < x.len / 4; i += blockDim.x) d1[i] = s1[i];
        } else {
            for (uint32_t i = threadIdx.x; i < x.len; i += blockDim.x) d[i] = s[i];
        }
    }
}

}  // namespace

cudaError_t launch_copy_runs(const uint8_t* src, uint8_t* dst, const XferRun* runs, uint32_t n, int n_sm,
                             cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const uint32_t grid = n < (uint32_t)(4 * n_sm) ? n : (uint32_t)(4 * n_sm);
    k_copy_runs<<<grid, 256, 0, st>>>(src, dst, runs, n);
    return cudaGetLastError();
}

}  // namespace hs
