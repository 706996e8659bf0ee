// hs_sample_noalloc: the device sampler (the same two kernels hs_sample runs)
// over logits that already sit in the caller's device memory, with every byte
// of working memory taken from one fixed array compiled into this library.
//
// Why: hs_sample needs an hs_scratch, and making one allocates device memory
// (cudaMalloc). Some callers cannot do that at the point where they sample:
//  - a serving loop that has sized its KV pages to fill HBM has no room left,
//    and a failed allocation in the middle of a step is not recoverable there;
//  - cudaFree synchronises the whole device, which stalls every other stream
//    of a pipelined decode, so a caller that samples between two in-flight
//    steps cannot create and drop a scratch around the call;
//  - a caller whose device memory belongs to another allocator (a framework's
//    caching pool) may not go around it with its own cudaMalloc.
// This entry point calls no cudaMalloc/cudaFree and no routine that allocates.
//
// Limits (checked before any device work; larger inputs are refused with
// HS_E_ARG and a message naming the limit):
//  - vocab <= kNaMaxVocab (262144 logits, 256 candidate CTAs of 1024);
//  - the penalty window, min(repeat_last_n, n_hist) when the penalty is on,
//    <= kNaMaxWindow (4096 tokens).
// The array holds 149,760 bytes per device.
//
// Set-up: the first call on a device makes that device current and looks up
// the array's device address once (cudaGetSymbolAddress, which may load this
// library's device code); make that first call before any stream capture
// begins. Each call waits for its own result on `stream`.
//
// Nothing in the array has to start at zero: every call writes the control
// block and the history window from the host before its kernels run, the
// candidate kernel writes every per-CTA key list and greedy entry it owns
// before the final kernel reads them, and the final kernel reads nothing
// else. There is ONE array per device: calls that overlap on the same device
// (from two host threads, or on two streams without ordering between them)
// race on it and may return wrong tokens. Serialise them.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>

#include "common.h"
#include "kernels.h"

namespace hs {
namespace {

constexpr uint32_t kNaMaxCta = 256;
constexpr uint32_t kNaMaxVocab = kNaMaxCta * kSampleSlice;  // 262144
constexpr uint32_t kNaMaxWindow = 4096;
constexpr int kNaMaxDevices = 64;

// Byte layout of the array: control block, per-CTA greedy entries, per-CTA
// top-k key lists (kMaxTopK each with several CTAs; up to kSampleSlice keys
// when one CTA covers the whole vocabulary), the history window.
constexpr size_t kOffCtl = 0;
constexpr size_t kOffArg = 256;
constexpr size_t kOffCand = kOffArg + (size_t)kNaMaxCta * 8;
constexpr size_t kCandBytes = (size_t)kNaMaxCta * kMaxTopK * 8 > (size_t)kSampleSlice * 8
                                  ? (size_t)kNaMaxCta * kMaxTopK * 8
                                  : (size_t)kSampleSlice * 8;
constexpr size_t kOffHist = kOffCand + kCandBytes;
constexpr size_t kNaBytes = kOffHist + (size_t)kNaMaxWindow * 4;
static_assert(sizeof(DevCtl) <= kOffArg, "control block does not fit its slot");
static_assert(kOffCand % 256 == 0 && kOffHist % 256 == 0, "regions are 256-byte aligned");
static_assert(kNaBytes == 149760, "stated size of the array");

static __device__ __align__(256) unsigned char g_sample_scratch[kNaBytes];

std::mutex g_na_mu;
unsigned char* g_na_ptr[kNaMaxDevices];

// Device address of the array on `device`, which the caller made current.
int na_scratch(int device, unsigned char** out) {
    std::lock_guard<std::mutex> lock(g_na_mu);
    if (!g_na_ptr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_sample_scratch);
        if (e != cudaSuccess)
            return fail(HS_E_CUDA, std::string("cudaGetSymbolAddress(sampler scratch): ") + cudaGetErrorString(e));
        g_na_ptr[device] = static_cast<unsigned char*>(p);
    }
    *out = g_na_ptr[device];
    return HS_OK;
}

// Puts the caller's current device back on every return path.
struct DeviceRestore {
    int prev = -1;
    ~DeviceRestore() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace
}  // namespace hs

using namespace hs;

extern "C" int hs_sample_noalloc(int device, const float* logits, uint32_t vocab, const hs_sampler_cfg* cfg,
                                 hs_rng* rng, const uint32_t* hist, uint64_t n_hist, void* stream, uint32_t* out) {
    if (!logits || !cfg || !rng || !out || (!hist && n_hist)) return fail(HS_E_ARG, "null argument");
    if (device < 0 || device >= kNaMaxDevices) return fail(HS_E_ARG, "device ordinal out of range");
    if (vocab == 0) return fail(HS_E_ARG, "empty vocabulary");
    if (vocab > kNaMaxVocab)
        return fail(HS_E_ARG, "vocab " + std::to_string(vocab) + " exceeds the no-allocation sampler's maximum of " +
                                  std::to_string(kNaMaxVocab));
    const uint32_t n_cta = (vocab + kSampleSlice - 1) / kSampleSlice;
    // Same top_k support as hs_sample: any top_k with one candidate CTA, else
    // top_k <= kMaxTopK when sampling.
    const uint32_t k = cfg->top_k == 0 ? vocab : (cfg->top_k < vocab ? cfg->top_k : vocab);
    if (cfg->temperature > 0.0f && (k > kSampleSlice || (n_cta > 1 && k > kMaxTopK)))
        return fail(HS_E_UNSUPPORTED, "device sampler supports top_k <= " + std::to_string(kMaxTopK) +
                                          " (or any top_k when vocab <= " + std::to_string(kSampleSlice) + ")");
    uint32_t kmax = n_cta > 1 ? kMaxTopK : kSampleSlice;
    if (kmax > vocab) kmax = vocab;
    // Only the tail the penalty reads is used (sampler.rs:103-111).
    const uint64_t win =
        (cfg->repeat_penalty != 1.0f && cfg->repeat_last_n > 0) ? (cfg->repeat_last_n < n_hist ? cfg->repeat_last_n : n_hist)
                                                                 : 0;
    if (win > kNaMaxWindow)
        return fail(HS_E_ARG, "penalty window of " + std::to_string(win) +
                                  " tokens exceeds the no-allocation sampler's maximum of " +
                                  std::to_string(kNaMaxWindow));
    const uint32_t* w = hist ? hist + (n_hist - win) : nullptr;
    for (uint64_t i = 0; i < win; i++)
        if (w[i] >= vocab) return fail(HS_E_ARG, "history token out of range");

    DeviceRestore restore;
    HS_CUDA_TRY(cudaGetDevice(&restore.prev));
    HS_CUDA_TRY(cudaSetDevice(device));
    unsigned char* base = nullptr;
    int rc = na_scratch(device, &base);
    if (rc) return rc;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);

    DevCtl h;
    std::memset(&h, 0, sizeof(h));
    h.mode = 1;  // sample only: the final kernel writes out_token, rng and draws
    h.n_tokens = win;
    h.vocab = vocab;
    h.max_ctx = kNaMaxWindow;
    h.temperature = cfg->temperature;
    h.top_p = cfg->top_p;
    h.top_k = cfg->top_k;
    h.repeat_penalty = cfg->repeat_penalty;
    h.repeat_last_n = cfg->repeat_last_n;
    for (int i = 0; i < 4; i++) h.rng[i] = rng->s[i];
    h.draws = rng->draws;

    DevCtl* ctl = reinterpret_cast<DevCtl*>(base + kOffCtl);
    uint32_t* tokens = reinterpret_cast<uint32_t*>(base + kOffHist);
    if (win) HS_CUDA_TRY(cudaMemcpyAsync(tokens, w, win * 4, cudaMemcpyHostToDevice, st));
    HS_CUDA_TRY(cudaMemcpyAsync(ctl, &h, sizeof(DevCtl), cudaMemcpyHostToDevice, st));

    SampleArgs a{};
    a.logits = logits;
    a.tokens = tokens;
    a.tokens_w = tokens;
    a.cand = reinterpret_cast<uint64_t*>(base + kOffCand);
    a.argbuf = reinterpret_cast<uint64_t*>(base + kOffArg);
    a.ctl = ctl;
    a.vocab = vocab;
    a.n_cta = n_cta;
    a.kmax = kmax;
    a.trace = nullptr;
    a.trace_slot = 0;
    cudaError_t e = launch_sample(a, st);
    if (e != cudaSuccess) return fail(HS_E_CUDA, std::string("sampler launch: ") + cudaGetErrorString(e));

    DevCtl r;
    HS_CUDA_TRY(cudaMemcpyAsync(&r, ctl, sizeof(DevCtl), cudaMemcpyDeviceToHost, st));
    HS_CUDA_TRY(cudaStreamSynchronize(st));
    if (r.err) return fail(HS_E_CUDA, "device sampler reported error bits " + std::to_string(r.err));
    *out = r.out_token;
    for (int i = 0; i < 4; i++) rng->s[i] = r.rng[i];
    rng->draws = r.draws;
    return HS_OK;
}
