/*
 * hs_oracle.h — CPU restatement of hotseat's hs-engine token loop.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker: only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may load
 * it. The product (hotseat_b200/libhotseat.so) never links or calls it.
 *
 * The reference (Rust, crates/hs-engine) cannot be compiled in this image (no
 * cargo/rustc), so every function here restates the reference's arithmetic in
 * C++, operation for operation, and is compiled with -ffp-contract=off so no
 * multiply-add is ever fused (Rust never fuses them either). Each definition in
 * hs_oracle.cpp cites the reference file:line it follows. The restatement is
 * pinned by the reference's own known-answer tests (tests/test_oracle_kat.py)
 * and cross-checked by an independent numpy forward; end-to-end logits and
 * transcripts are parity unpinned against the Rust binary itself, which
 * cannot be built here and ships no golden vectors.
 */
#ifndef HS_ORACLE_H
#define HS_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* f16.rs */
float hso_f16_to_f32(uint16_t h);
uint16_t hso_f32_to_f16(float f);

/* math.rs */
float hso_exp_f32(float x);
float hso_ln_f32(float x);
void hso_sincos_f32(float x, float* s, float* c);
float hso_silu(float x);
float hso_dot_f16(const uint16_t* w, const float* x, size_t n);
float hso_dot_f32(const float* a, const float* b, size_t n);
void hso_rmsnorm(float* out, const float* x, const float* g, size_t n, float eps);
void hso_softmax(float* x, size_t n);
double hso_nll(const float* logits, size_t n, uint32_t next); /* examples/ppl.rs:35-43 */

/* quant.rs: ggml type ids 0,1,6,8,12,13,14. Returns 0, or -1 on unknown type. */
int hso_dequant_f16(uint32_t ggml_type, const uint8_t* src, size_t n, uint16_t* dst);
/* scale_min_k4 (quant.rs:101-107); packs (sc << 8) | m. */
uint32_t hso_scale_min_k4(uint32_t j, const uint8_t* q12);

/* hash.rs */
uint64_t hso_fnv1a(const uint8_t* p, size_t n);
uint64_t hso_wide(const uint8_t* p, size_t n);

/* sampler.rs */
typedef struct {
    float temperature;
    float top_p;
    uint32_t top_k;
    float repeat_penalty;
    uint32_t repeat_last_n;
    uint64_t seed;
} hso_sampler_cfg;

typedef struct {
    uint64_t s[4];
    uint64_t draws;
} hso_rng;

void hso_sampler_cfg_default(hso_sampler_cfg* cfg);
void hso_rng_seed(uint64_t seed, hso_rng* r);
uint64_t hso_rng_next_u64(hso_rng* r);
float hso_rng_next_f32(hso_rng* r);
/* Sampler::sample. `logits` is modified in place, as in the reference. */
uint32_t hso_sample(const hso_sampler_cfg* cfg, hso_rng* rng, float* logits, size_t n,
                    const uint32_t* hist, size_t n_hist);
uint32_t hso_argmax(const float* logits, size_t n);
/* seq.rs penalised_argmax */
uint32_t hso_penalised_argmax(const hso_sampler_cfg* cfg, float* logits, size_t n,
                              const uint32_t* hist, size_t n_hist);

/* pool.rs split */
void hso_split(size_t rows, size_t n, size_t tid, size_t* a, size_t* b);

/* kv.rs. layout 0 = TokenMajor, 1 = HeadMajor. Ranges are (byte_off, byte_len)
 * pairs written into out[2*i], out[2*i+1]; returns the count (may exceed cap,
 * in which case only cap pairs are written). */
typedef struct {
    uint64_t n_layers, n_kv_heads, head_dim, max_ctx;
    uint32_t layout;
} hso_kv_spec;
uint64_t hso_kv_row_off(const hso_kv_spec* s, uint64_t layer, int is_v, uint64_t pos, uint64_t head);
size_t hso_kv_written_ranges(const hso_kv_spec* s, uint64_t pos, uint64_t* out, size_t cap);
size_t hso_kv_live_ranges_between(const hso_kv_spec* s, uint64_t from, uint64_t to, uint64_t* out,
                                  size_t cap);
uint64_t hso_kv_hash(const hso_kv_spec* s, const void* kv_base, uint64_t n_pos);

/* hs-track pageset.rs runs + hs-wire lib.rs runs_to_byte_runs. `words` is a
 * PageSet bitmap (bit p%64 of word p/64). Outputs (off, len) pairs. */
size_t hso_pageset_runs(const uint64_t* words, size_t n_pages, uint64_t* out, size_t cap);
size_t hso_runs_to_byte_runs(const uint64_t* words, size_t n_pages, uint64_t page_size,
                             const uint64_t* live, size_t n_live, uint64_t* out, size_t cap);

/* model.rs */
typedef struct {
    uint64_t n_layers, n_heads, n_kv_heads, head_dim, d_model, d_ff, vocab;
    float eps, rope_base;
    uint64_t train_ctx;
    uint64_t fingerprint;
    uint32_t eos;
    uint64_t max_ctx;
} hso_config;

typedef struct hso_model hso_model;

/* Returns 0, or a negative code with a message available from hso_last_error(). */
int hso_model_load(const char* path, uint64_t max_ctx, uint32_t threads, hso_model** out);
void hso_model_free(hso_model* m);
void hso_model_config(const hso_model* m, hso_config* out);
const char* hso_last_error(void);
/* Dequantised f16 weights of one tensor as the reference holds them
 * (`Layer::wq` and friends); NULL if absent. */
const uint16_t* hso_model_tensor_f16(const hso_model* m, const char* name, size_t* n);
const float* hso_model_tensor_f32(const hso_model* m, const char* name, size_t* n);
const float* hso_model_rope_cos(const hso_model* m);
const float* hso_model_rope_sin(const hso_model* m);

/* Model::forward with the KV in `kv` (spec from the model, TokenMajor unless
 * layout says otherwise). Leaves logits in `logits[vocab]`. If `trace` is not
 * NULL it receives the residual stream x after every layer (n_layers*d_model). */
int hso_forward(hso_model* m, float* kv, uint32_t layout, uint32_t token, uint64_t pos,
                float* logits, float* trace);

/* The seq.rs decode loop (`run`, seq.rs:230-318), for one sequence, until it
 * stops or `filled` reaches `stop_at_filled` (0 = never). tokens[] has room for
 * cap entries; *n_tokens holds the prompt (and anything generated before).
 * done_reason: 0 running/paused, 1 eos, 2 max_tokens, 3 context full. */
typedef struct {
    uint64_t prompt_len;
    uint64_t filled;
    uint64_t max_tokens;
    uint32_t done;
    uint32_t done_reason;
} hso_seq_state;

int hso_seq_run(hso_model* m, float* kv, uint32_t layout, uint32_t* tokens, uint64_t* n_tokens,
                uint64_t cap, hso_seq_state* st, const hso_sampler_cfg* cfg, hso_rng* rng,
                uint64_t stop_at_filled);

#ifdef __cplusplus
}
#endif
#endif
