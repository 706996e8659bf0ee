/*
 * hotseat.h — C ABI of the B200 token loop (libhotseat.so).
 *
 * This replaces the Rust API that hotseat's hs-worker and hs-wire call on
 * hs-engine (crates/hs-engine/src). Each entry point names the reference
 * interface it stands in for. Conventions:
 *   - every call returns an int status: HS_OK (0) or a negative HS_E_* code;
 *     hs_last_error() gives the message of the calling thread's last failure;
 *   - no exception or abort crosses the ABI: conditions on which the reference
 *     panics (pos >= max_ctx, model.rs:242; a KV shape mismatch, model.rs:243)
 *     return HS_E_ARG instead;
 *   - plain pointers and sizes only; host buffers are owned by the caller;
 *   - an hs_kv / hs_scratch is used by one thread at a time (the reference's
 *     one decode thread per sequence, hs-worker seq.rs:223-318).
 */
#ifndef HOTSEAT_H
#define HOTSEAT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HS_OK 0
#define HS_E_ARG (-1)         /* bad argument, out-of-range pos/token, shape mismatch */
#define HS_E_IO (-2)          /* file or GGUF format error (gguf.rs Error variants) */
#define HS_E_CUDA (-3)        /* CUDA error, no device, or a kernel reported a fault */
#define HS_E_STATE (-4)       /* sequence invariant broken (seq.rs:258-266) */
#define HS_E_NOMEM (-5)       /* device or host allocation failed */
#define HS_E_UNSUPPORTED (-6) /* shape or option this build does not implement */

/* Message for the calling thread's most recent failing call. */
const char* hs_last_error(void);

/* KV layouts (kv.rs:29-33). */
#define HS_LAYOUT_TOKEN_MAJOR 0u
#define HS_LAYOUT_HEAD_MAJOR 1u

/* Model configuration plus the load-time facts the worker needs
 * (model.rs:21-33 Config, model.rs:62-68 fingerprint, tok.rs eos). */
typedef struct {
    uint32_t n_layers, n_heads, n_kv_heads, head_dim, d_model, d_ff, vocab;
    float eps, rope_base;
    uint32_t train_ctx, max_ctx, eos;
    uint64_t fingerprint;
    uint32_t numeric; /* HS_NUMERIC_* the model was loaded with */
} hs_config;

/* Numeric paths. A sequence must use one path for its whole life; the path is
 * part of the fingerprint, so workers on different paths refuse a handover
 * exactly as the reference refuses different weights (migrate.rs:497-505).
 *   REFERENCE: every reduction in hs-engine's order (eight serial lanes and
 *              one fold, no FMA): bit-identical to the CPU reference, and the
 *              fingerprint equals the reference's (model.rs:145-156).
 *   FAST:      fixed GPU-native reduction shapes (warp trees, packed FMA):
 *              bit-identical across B200s and migrations, logits within 1e-2
 *              of the CPU reference. */
#define HS_NUMERIC_REFERENCE 0u
#define HS_NUMERIC_FAST 1u
/* Tensor-core path: every matrix product runs as a tcgen05 GEMM over a batch
 * of sequences (activations carried as f16 hi/lo pairs, f32 accumulation).
 * Same tolerance contract as FAST; a sequence's bits do not depend on the
 * batch it runs in. Models loaded with it decode through hs_batch_*. */
#define HS_NUMERIC_TC 2u

typedef struct hs_model hs_model;
typedef struct hs_kv hs_kv;
typedef struct hs_scratch hs_scratch;

/* ---- model (replaces Model::load, model.rs:110-215) ------------------------ */

/* Parse the GGUF, copy the quantised tensors to `device` and dequantise them
 * there to f16 (Q4_K/Q6_K/Q5_K/Q5_0/Q8_0/F16/F32, quant.rs:18-206), build the
 * RoPE tables with the reference's own exp/ln/sincos (model.rs:187-201). */
int hs_model_load(const char* path, uint32_t max_ctx, int device, hs_model** out);
/* hs_model_load with an explicit numeric path (hs_model_load uses REFERENCE). */
int hs_model_load_ex(const char* path, uint32_t max_ctx, int device, uint32_t numeric, hs_model** out);
/* Model{cfg, fingerprint} and tok.eos (model.rs:62-78). */
int hs_model_config(const hs_model* m, hs_config* out);
void hs_model_free(hs_model* m);
/* Copy one loaded tensor back to the host: f16 bits for 2-D weights (as
 * Layer::wq etc. hold them, model.rs:47-60), f32 for norms and biases.
 * *dtype_out = 1 (f16) or 0 (f32). For parity checks. */
int hs_model_tensor(const hs_model* m, const char* name, void* host, uint64_t bytes, uint32_t* dtype_out);

/* ---- KV cache (replaces hs-track Region + Kv::from_raw, kv.rs:196-274) ---- */

typedef struct {
    uint32_t n_layers, n_kv_heads, head_dim, max_ctx, layout;
} hs_kv_spec;

/* Device KV region with the reference's exact byte layout (KvSpec::row_off,
 * kv.rs:96-104) and a device dirty-page bitmap of `page_size`-byte pages in
 * PageSet's word/bit format (hs-track pageset.rs:10-34). */
int hs_kv_alloc(const hs_model* m, uint32_t layout, uint32_t page_size, hs_kv** out);
int hs_kv_info(const hs_kv* kv, hs_kv_spec* spec, uint64_t* bytes, uint32_t* page_size, uint64_t* n_pages);
/* Cross-process hand-over on one node (the destination worker is another
 * process, e.g. one rank per GPU): the owner exports its region with
 * hs_kv_ipc_handle (a CUDA IPC handle, HS_IPC_HANDLE_BYTES bytes); the source
 * process opens it with hs_kv_open_ipc on its own model and GPU, which maps
 * the remote region for hs_kv_peer_copy / hs_kv_copy_runs / hs_migrate_* as
 * a destination (stores over NVLink). A view is never decoded into; the
 * owner must keep its region alive until the view is freed (hs_kv_free). No
 * counterpart in the reference, whose hand-over crosses a TCP socket
 * (hs-wire lib.rs:338-396). */
#define HS_IPC_HANDLE_BYTES 64
int hs_kv_ipc_handle(hs_kv* kv, void* out, uint64_t out_bytes);
int hs_kv_open_ipc(const hs_model* m, const void* handle, uint32_t layout, uint32_t page_size, hs_kv** out);
/* The fingerprint of the model the region was allocated for (the Hello
 * field model_fingerprint, hs-wire lib.rs / migrate.rs:250-258). */
int hs_kv_fingerprint(const hs_kv* kv, uint64_t* out);
void hs_kv_free(hs_kv* kv);
/* Byte-range staging between the device region and host memory (the hs-wire
 * send_page_bytes / recv_page_bytes path, hs-wire lib.rs:339-396). */
int hs_kv_read(hs_kv* kv, uint64_t off, uint64_t len, void* host);
int hs_kv_write(hs_kv* kv, uint64_t off, uint64_t len, const void* host);
/* Kv::hash (kv.rs:267-274): hash::Wide over live_ranges(n_pos). */
int hs_kv_hash(hs_kv* kv, uint32_t n_pos, uint64_t* out);
/* Dirty-page tracking (Tracker::arm/harvest/disarm, hs-track lib.rs:75-170).
 * The KV-append kernel marks pages as it stores; harvest atomically takes and
 * clears the set into `words` (ceil(n_pages/64) u64 words). */
int hs_kv_arm(hs_kv* kv);
int hs_kv_harvest(hs_kv* kv, uint64_t* words, uint64_t n_words);
int hs_kv_disarm(hs_kv* kv);
/* Run-list staging for the hs-wire TCP path (hs-wire lib.rs:338-396,
 * Conn::send_page_bytes / recv_page_bytes): the bytes of `runs` ((off, len)
 * pairs) packed back to back in run order, moved between the device region
 * and `host` (host_bytes >= the runs' total) in one stream-ordered pass: a
 * gather (or scatter) kernel over a device staging buffer and one copy each
 * way. Both return once the bytes are in place. */
int hs_kv_read_runs(hs_kv* kv, const uint64_t* runs, uint64_t n_runs, void* host, uint64_t host_bytes);
int hs_kv_write_runs(hs_kv* kv, const uint64_t* runs, uint64_t n_runs, const void* host, uint64_t host_bytes);
/* Copy byte runs from one KV region to another (the pre-copy data path of
 * hs-worker migrate.rs:234-473 without the TCP hop): one kernel on the
 * source's GPU reads the runs and stores them into the destination, through
 * its peer mapping over NVLink when it lives on another GPU. Enqueued on
 * `stream` (a cudaStream_t of the source's device; NULL = the source
 * region's own stream) and not waited for. The copy sees the source bytes as
 * of its turn on `stream`: to take a residue after the decode loop's last
 * append, park the loop first or make `stream` wait on an event recorded
 * after it. Specs must match. */
int hs_kv_peer_copy(hs_kv* src, hs_kv* dst, const uint64_t* runs, uint64_t n_runs, void* stream);
/* hs_kv_peer_copy on the source region's stream, waited for. */
int hs_kv_copy_runs(hs_kv* src, hs_kv* dst, const uint64_t* runs, uint64_t n_runs);

/* ---- pre-copy migration (replaces hs-worker migrate.rs:45-166, 234-630) --
 * The source half of migrate_out with the destination's Hello checks, for
 * two device KV regions on one node (the bytes move by hs_kv_copy_runs).
 * The decode loop and the sequence's FinalState stay the caller's:
 *   hs_migrate_begin   fingerprint / KV spec / page size must match (else
 *                      HS_E_STATE "destination refused: ..." before any byte
 *                      moves, migrate.rs:486-518); arms the source; round 0
 *                      copies every live byte of positions [0, upper + 1)
 *   hs_migrate_round   while the sequence keeps decoding: the pages dirtied
 *                      since the last harvest, clipped to [low, upper + 1);
 *                      *more = 0 once the rounds stop (nothing left, a round
 *                      within target_bytes, not shrinking, or max_rounds;
 *                      migrate.rs:293-346); the next round starts at
 *                      low = filled.
 *   `filled`: a count of positions known complete (seen at a token boundary
 *   at or before the call); `upper`: the last position the decode loop may
 *   have written by the call (filled when it is parked; filled + the steps
 *   in flight otherwise). The reference reads one value after its harvest
 *   for both (migrate.rs:307-313).
 *   hs_migrate_finish  with the decode loop parked at `filled` (no append in
 *                      flight): the residue, then with verify both KV hashes
 *                      inside the window (HS_E_STATE if they differ: keep
 *                      decoding on the source); fills the report. park_us is
 *                      the caller's measured park time, added to stw_us.
 * tokens_now / tokens_total: the sequence's token count, for tokens_during. */
#define HS_MIGRATE_MAX_ROUNDS 34
typedef struct {
    uint32_t max_rounds;   /* Opts::max_rounds (8); at most HS_MIGRATE_MAX_ROUNDS - 2 */
    uint64_t target_bytes; /* Opts::target_bytes (1 MiB) */
    uint32_t verify;       /* Opts::verify (0) */
} hs_migrate_opts;
typedef struct { /* RoundStat, migrate.rs:70-78 */
    uint32_t index;
    uint64_t bytes, runs;
    double ms;
    uint64_t tokens_during;
} hs_migrate_round_stat;
typedef struct { /* Report, migrate.rs:80-110 (tracker fields: the device bitmap has no faults) */
    hs_migrate_round_stat rounds[HS_MIGRATE_MAX_ROUNDS];
    uint32_t n_rounds;
    uint64_t precopy_bytes;
    double precopy_ms, park_us, stw_us, stw_send_us, dest_resume_us;
    uint64_t final_bytes, live_bytes, filled, tokens_total, kv_hash_src, kv_hash_dst;
    uint32_t verified, converged;
    char stop_reason[160];
} hs_migrate_report;
typedef struct hs_migration hs_migration;
void hs_migrate_opts_default(hs_migrate_opts* o);
int hs_migrate_begin(hs_kv* src, hs_kv* dst, const hs_migrate_opts* opts, uint64_t filled, uint64_t upper,
                     uint64_t tokens_now, hs_migration** out);
int hs_migrate_round(hs_migration* g, uint64_t filled, uint64_t upper, uint64_t tokens_now, int* more);
int hs_migrate_finish(hs_migration* g, uint64_t filled, uint64_t tokens_total, double park_us,
                      hs_migrate_report* out);
void hs_migrate_free(hs_migration* g);

/* Host-only mirrors of the reference's range logic (no device needed).
 * Output is (off, len) pairs; return value is the number of pairs, which may
 * exceed `cap` (then only cap pairs were written). */
uint64_t hs_kv_live_ranges_between(const hs_kv_spec* s, uint32_t from, uint32_t to, uint64_t* out, uint64_t cap);
uint64_t hs_runs_to_byte_runs(const uint64_t* words, uint64_t n_pages, uint64_t page_size, const uint64_t* live,
                              uint64_t n_live, uint64_t* out, uint64_t cap);

/* ---- forward (replaces Model::scratch / Model::forward, model.rs:221-327) - */

int hs_scratch_new(const hs_model* m, hs_scratch** out);
void hs_scratch_free(hs_scratch* s);
/* One token at `pos`: appends its K/V to `kv` (marking dirty pages) and
 * leaves the next-token logits on the device. Blocks until done. */
int hs_forward(const hs_model* m, hs_kv* kv, uint32_t token, uint32_t pos, hs_scratch* s);
/* Scratch::logits (model.rs:341) copied to the host. */
int hs_scratch_logits(hs_scratch* s, float* host, uint64_t n);
/* Overwrite Scratch::logits from the host (the field is public in the
 * reference, so a caller may sample from logits it supplies). */
int hs_scratch_set_logits(hs_scratch* s, const float* host, uint64_t n);
/* The perplexity harness's score (hs-engine examples/ppl.rs:35-43) of the
 * scratch's logits: -((l[next] - max) - ln(sum of exp_f32(l - max))), the
 * sum in f64 (in a fixed tree order on the device). */
int hs_scratch_nll(hs_scratch* s, uint32_t next, double* out);

/* ---- sampling (replaces sampler.rs:12-187, seq.rs:321-330) ------------- */

typedef struct {
    float temperature, top_p;
    uint32_t top_k;
    float repeat_penalty;
    uint32_t repeat_last_n;
    uint64_t seed;
} hs_sampler_cfg;

typedef struct {
    uint64_t s[4];
    uint64_t draws;
} hs_rng;

void hs_sampler_cfg_default(hs_sampler_cfg* cfg); /* SamplerCfg::default, sampler.rs:22-33 */
void hs_rng_seed(uint64_t seed, hs_rng* r);        /* Rng::seed, sampler.rs:47-58 */
/* Sampler::sample over the scratch's logits on the device: penalty, top-k
 * by (value desc, id asc), temperature softmax, nucleus, one RNG draw
 * (none at temperature <= 0). `rng` is read and written back. */
int hs_sample(hs_scratch* s, const hs_sampler_cfg* cfg, hs_rng* rng, const uint32_t* hist, uint64_t n_hist,
              uint32_t* out);
/* argmax (sampler.rs:177-187) of the scratch's logits. */
int hs_argmax(hs_scratch* s, uint32_t* out);
/* hs_sample over `vocab` f32 logits in the caller's device memory on
 * `device`, with no allocation: its working memory is one fixed array per
 * device inside this library. No counterpart in the reference (its sampler
 * reads host logits); it serves callers that cannot allocate device memory
 * where they sample. Limits: vocab <= 262144; penalty window (min of
 * repeat_last_n and n_hist, when the penalty is on) <= 4096 tokens; larger
 * inputs return HS_E_ARG. The first call on a device does the set-up and must
 * come before any stream capture; each call waits for its result on `stream`
 * (cudaStream_t or NULL). Overlapping calls on one device race: serialise
 * them. Same tokens and RNG state as hs_sample on the same logits. */
int hs_sample_noalloc(int device, const float* logits, uint32_t vocab, const hs_sampler_cfg* cfg, hs_rng* rng,
                      const uint32_t* hist, uint64_t n_hist, void* stream, uint32_t* out);

/* ---- the decode loop (replaces hs-worker seq.rs:230-318 `run`) ---------- */

/* SeqState fields that a handover carries (seq.rs:35-61, hs-wire FinalState).
 * done_reason: 0 running, 1 eos, 2 max_tokens, 3 context full. */
typedef struct {
    uint64_t prompt_len, filled, max_tokens;
    uint32_t done, done_reason;
} hs_seq_state;

/* Run the sequence until it stops or `filled` reaches stop_at_filled (0 =
 * never), entirely on the device: forward, commit, sample and the stop
 * checks of seq.rs:273-312 run as kernels, with no host round trip per
 * token. tokens[0..*n_tokens) is the history on entry (prompt plus anything
 * generated before a handover); on return it holds the full history. */
int hs_seq_run(const hs_model* m, hs_kv* kv, hs_scratch* s, uint32_t* tokens, uint64_t* n_tokens, uint64_t cap,
               hs_seq_state* st, const hs_sampler_cfg* cfg, hs_rng* rng, uint64_t stop_at_filled);

/* The same loop split into its stream-ordered parts, for callers that keep
 * the history resident on the device between calls (and for timing):
 * begin uploads the state, step enqueues n forward+commit steps without
 * synchronising, end downloads the state. */
int hs_seq_begin(hs_scratch* s, hs_kv* kv, const uint32_t* tokens, uint64_t n_tokens, uint64_t cap,
                 const hs_seq_state* st, const hs_sampler_cfg* cfg, const hs_rng* rng, uint64_t stop_at_filled);
int hs_seq_step(hs_scratch* s, uint32_t n_steps);
int hs_seq_end(hs_scratch* s, uint32_t* tokens, uint64_t* n_tokens, uint64_t cap, hs_seq_state* st, hs_rng* rng);
/* ---- batched decode (HS_NUMERIC_TC models; one worker, many sequences) --
 * The reference decodes each Seq on its own thread (seq.rs:223-318); a B200
 * worker keeps up to 128 sequences in one hs_batch and advances them together,
 * one token each per step, with the same per-sequence semantics: own KV
 * region, history, SeqState, sampler config and RNG. No counterpart type in
 * the reference. */
typedef struct hs_batch hs_batch;
int hs_batch_new(const hs_model* m, uint32_t max_seqs, hs_batch** out); /* max_seqs 1..4096 (sequences, or prompt tokens per prefill pass) */
void hs_batch_free(hs_batch* b);
/* One Model::forward for each of n sequences: tokens[i] at pos[i], appending
 * to kvs[i] (all regions of one layout and page size). Blocks until done. */
int hs_forward_batch(const hs_model* m, hs_kv* const* kvs, const uint32_t* tokens, const uint32_t* pos, uint32_t n,
                     hs_batch* b);
/* Prompt prefill: Model::forward for tokens[0..n) of ONE sequence at
 * positions pos0.., appended to `kv`, with the tokens as the rows of each
 * GEMM (up to the batch capacity per pass) instead of one token per step.
 * No logits. Its GEMMs use wide tiles without the decode steps' K splits,
 * so the KV rows match single-token steps within the path's tolerance (and
 * are bit-identical however the prompt is cut into calls). Follow
 * with hs_batch_seq_run from filled = pos0 + n: the sequence's next
 * (last prompt) token then produces the logits of the first sample. */
int hs_prefill(const hs_model* m, hs_kv* kv, const uint32_t* tokens, uint32_t n, uint32_t pos0, hs_batch* b);
/* Logits of sequence `slot` from the last hs_forward_batch. */
int hs_batch_logits(hs_batch* b, uint32_t slot, float* host, uint64_t n);
/* hs_scratch_nll for slots 0..n-1 of the last hs_forward_batch: out[i] =
 * the score of next[i] under slot i's logits. */
int hs_batch_nll(hs_batch* b, const uint32_t* next, uint32_t n, double* out);
/* hs_seq_run for n sequences at once: sequence i uses kvs[i], its history
 * tokens[i] (n_tokens[i] valid, capacity cap each), st[i], cfg[i], rng[i];
 * all advance until each stops (or reaches stop_at_filled, 0 = never). */
int hs_batch_seq_run(const hs_model* m, hs_kv* const* kvs, hs_batch* b, uint32_t n, uint32_t* const* tokens,
                     uint64_t* n_tokens, uint64_t cap, hs_seq_state* st, const hs_sampler_cfg* cfg, hs_rng* rng,
                     uint64_t stop_at_filled);
/* The same in parts (device-resident stepping, for timing): begin uploads the
 * state, step enqueues n_steps batched decode steps, end syncs and reads back. */
int hs_batch_seq_begin(hs_batch* b, hs_kv* const* kvs, uint32_t n, uint32_t* const* tokens, const uint64_t* n_tokens,
                       uint64_t cap, const hs_seq_state* st, const hs_sampler_cfg* cfg, const hs_rng* rng,
                       uint64_t stop_at_filled);
int hs_batch_seq_step(hs_batch* b, uint32_t n_steps);
int hs_batch_seq_end(hs_batch* b, uint32_t* const* tokens, uint64_t* n_tokens, uint64_t cap, hs_seq_state* st,
                     hs_rng* rng);
/* The batch's CUDA stream (cudaStream_t), and kernels launched per step. */
void* hs_batch_stream(hs_batch* b);
int hs_batch_launches_per_step(hs_batch* b, uint32_t* out);
/* Launch timeline of the last batched forward or step (HS_TRACE=1 in the
 * environment when the batch is created), in the layout of hs_scratch_trace. */
int hs_batch_trace(hs_batch* b, uint64_t* out, uint64_t n_slots, uint64_t* used);

/* The scratch's CUDA stream (cudaStream_t), for event timing. */
void* hs_scratch_stream(hs_scratch* s);
/* Kernel launches one hs_seq_step(s, 1) enqueues. */
int hs_seq_launches_per_step(hs_scratch* s, uint32_t* out);
/* Launch timeline of the last hs_seq_step (profiling; enabled by HS_TRACE=1
 * in the environment when the scratch is created): 8 u64 per launch, in
 * launch order, %globaltimer ns: first CTA entry, CTA 0 past its wait on the
 * previous kernel, last CTA exit, last CTA entry, then four kernel-specific
 * checkpoints (latest CTA). *used = number of launch slots. */
int hs_scratch_trace(hs_scratch* s, uint64_t* out, uint64_t n_slots, uint64_t* used);

/* ---- load-time dequantisation as a standalone op (quant.rs:18-38) ------ */

/* Dequantise n elements of ggml type `ggml_type` from device memory `src`
 * into f16 bits at device memory `dst`, on `stream` (cudaStream_t or NULL). */
int hs_dequant_f16(uint32_t ggml_type, const void* src, uint64_t n, void* dst, void* stream);

#ifdef __cplusplus
}
#endif
#endif
