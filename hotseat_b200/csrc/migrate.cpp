// Pre-copy migration of a live sequence between two device KV regions: the
// source half of hs-worker's migrate.rs (migrate_out, migrate.rs:234-473)
// with the destination's checks (migrate_in, 476-630), for regions on the
// same or different GPUs of one node. The page bytes move by
// hs_kv_copy_runs (one kernel, peer stores over NVLink across GPUs) instead
// of a TCP stream; the sequence's FinalState (tokens, SeqState, RNG,
// sampler config) is the caller's to hand over, as the decode loop that
// owns it is the caller's (hs_seq_* or hs_batch_seq_*).
//
//   hs_migrate_begin   Hello checks (fingerprint, KV spec, page size), arm
//                      the source's dirty bitmap, round 0: every live byte
//                      of positions [0, filled + 1)
//   hs_migrate_round   one iterative round while the sequence decodes: the
//                      pages dirtied since the last harvest, clipped to
//                      positions [low, upper + 1); the convergence rules of
//                      migrate.rs:293-346 decide whether another follows
//
// The reference reads `filled` once after each harvest and uses it as both
// the low-water mark of the next round (positions below it are complete)
// and the clip (nothing past filled + 1 can have been written). A caller
// here may run a round while decode steps are in flight and not know
// `filled` exactly, so the two are separate arguments: `filled`, a count
// known complete, and `upper`, the last position the loop may have written
// by the harvest (filled itself at a token boundary).
//   hs_migrate_finish  with the decode loop parked: the residue, the KV
//                      hashes, the report (migrate.rs:347-473)
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <memory>
#include <string>
#include <vector>

#include "common.h"

namespace {

using Clock = std::chrono::steady_clock;

double us_since(Clock::time_point t) {
    return std::chrono::duration<double, std::micro>(Clock::now() - t).count();
}

std::string fmt_bytes(uint64_t b) {  // migrate.rs:184-198
    static const char* U[4] = {"B", "KiB", "MiB", "GiB"};
    double v = (double)b;
    int i = 0;
    while (v >= 1024.0 && i < 3) {
        v /= 1024.0;
        i++;
    }
    char s[64];
    if (i == 0)
        std::snprintf(s, sizeof s, "%llu B", (unsigned long long)b);
    else
        std::snprintf(s, sizeof s, "%.2f %s", v, U[i]);
    return s;
}

}  // namespace

struct hs_migration {
    hs_kv* src = nullptr;
    hs_kv* dst = nullptr;
    hs_migrate_opts opts{};
    hs_kv_spec spec{};
    uint64_t bytes = 0, n_pages = 0, n_words = 0;
    uint32_t page_size = 0;
    std::vector<uint64_t> dirty;  // pages harvested and not yet sent (PageSet)
    uint64_t low = 0;             // positions below are on the destination for good
    uint64_t prev = ~0ull;        // last round's bytes
    uint64_t t_mark = 0;          // tokens at the start of the round
    bool rounds_done = false;
    Clock::time_point precopy_start;
    hs_migrate_report rep{};
};

namespace {

int live_runs(const hs_migration* g, const uint64_t* words, uint64_t from, uint64_t to, std::vector<uint64_t>* runs) {
    std::vector<uint64_t> live(2 * (size_t)(2 * g->spec.n_layers * g->spec.n_kv_heads + 2));
    uint64_t n_live = hs_kv_live_ranges_between(&g->spec, (uint32_t)from, (uint32_t)to, live.data(), live.size() / 2);
    if (n_live > live.size() / 2) {
        live.resize(2 * n_live);
        n_live = hs_kv_live_ranges_between(&g->spec, (uint32_t)from, (uint32_t)to, live.data(), n_live);
    }
    runs->assign(2 * (size_t)std::max<uint64_t>(n_live, 1) + 2, 0);
    uint64_t n = hs_runs_to_byte_runs(words, g->n_pages, g->page_size, live.data(), n_live, runs->data(),
                                      runs->size() / 2);
    if (n > runs->size() / 2) {
        runs->assign(2 * n, 0);
        n = hs_runs_to_byte_runs(words, g->n_pages, g->page_size, live.data(), n_live, runs->data(), n);
    }
    runs->resize(2 * n);
    return HS_OK;
}

uint64_t total_bytes(const std::vector<uint64_t>& runs) {
    uint64_t t = 0;
    for (size_t i = 1; i < runs.size(); i += 2) t += runs[i];
    return t;
}

void set_reason(hs_migrate_report* r, const std::string& why) {
    std::snprintf(r->stop_reason, sizeof r->stop_reason, "%s", why.c_str());
}

int push_round(hs_migration* g, uint32_t index, const std::vector<uint64_t>& runs, uint64_t tokens_now) {
    const auto t0 = Clock::now();
    int rc = hs_kv_copy_runs(g->src, g->dst, runs.data(), runs.size() / 2);
    if (rc) return rc;
    hs_migrate_report& r = g->rep;
    if (r.n_rounds < HS_MIGRATE_MAX_ROUNDS) {
        hs_migrate_round_stat& s = r.rounds[r.n_rounds++];
        s.index = index;
        s.bytes = total_bytes(runs);
        s.runs = runs.size() / 2;
        s.ms = us_since(t0) / 1000.0;
        s.tokens_during = tokens_now >= g->t_mark ? tokens_now - g->t_mark : 0;
    }
    g->t_mark = tokens_now;
    r.precopy_bytes += total_bytes(runs);
    return HS_OK;
}

}  // namespace

extern "C" {

void hs_migrate_opts_default(hs_migrate_opts* o) {
    if (!o) return;
    o->max_rounds = 8;          // migrate.rs:66
    o->target_bytes = 1 << 20;
    o->verify = 0;
}

int hs_migrate_begin(hs_kv* src, hs_kv* dst, const hs_migrate_opts* opts, uint64_t filled, uint64_t upper,
                     uint64_t tokens_now, hs_migration** out) {
    using hs::fail;
    if (!src || !dst || !out) return fail(HS_E_ARG, "null argument");
    *out = nullptr;
    hs_migrate_opts o;
    hs_migrate_opts_default(&o);
    if (opts) o = *opts;
    if (o.max_rounds > HS_MIGRATE_MAX_ROUNDS - 2)
        return fail(HS_E_ARG, "max_rounds above " + std::to_string(HS_MIGRATE_MAX_ROUNDS - 2));
    auto g = std::make_unique<hs_migration>();
    g->src = src;
    g->dst = dst;
    g->opts = o;
    hs_kv_spec ds{};
    uint64_t dbytes = 0, dpages = 0;
    uint32_t dpage = 0;
    int rc = hs_kv_info(src, &g->spec, &g->bytes, &g->page_size, &g->n_pages);
    if (!rc) rc = hs_kv_info(dst, &ds, &dbytes, &dpage, &dpages);
    if (rc) return rc;
    // The destination's checks before any byte moves (migrate.rs:486-518):
    // each mismatch would give fluent, wrong output rather than an error.
    uint64_t fs = 0, fd = 0;
    if ((rc = hs_kv_fingerprint(src, &fs)) || (rc = hs_kv_fingerprint(dst, &fd))) return rc;
    if (fs != fd) {
        char m[160];
        std::snprintf(m, sizeof m, "destination refused: model fingerprint %#018llx != local %#018llx",
                      (unsigned long long)fs, (unsigned long long)fd);
        return fail(HS_E_STATE, m);
    }
    if (std::memcmp(&ds, &g->spec, sizeof ds) != 0) return fail(HS_E_STATE, "destination refused: KV spec mismatch");
    if (dpage != g->page_size) return fail(HS_E_STATE, "destination refused: page size mismatch");
    if (filled >= g->spec.max_ctx || upper < filled) return fail(HS_E_ARG, "filled past max_ctx or above upper");
    g->n_words = (g->n_pages + 63) / 64;
    g->dirty.assign(g->n_words, 0);
    g->rep.converged = 1;
    // From here on every write the model makes is observed.
    if ((rc = hs_kv_arm(src))) return rc;
    g->precopy_start = Clock::now();
    g->t_mark = tokens_now;
    // Round 0: everything the sequence occupies right now, up to one
    // position past the last one it may have started (a position may be
    // partly written; its other layers are dirtied after the arm and arrive
    // later; migrate.rs:200-213, 271-297).
    const uint64_t clip = std::min<uint64_t>(upper + 1, g->spec.max_ctx);
    std::vector<uint64_t> all(g->n_words, ~0ull), runs;
    live_runs(g.get(), all.data(), 0, clip, &runs);
    if ((rc = push_round(g.get(), 0, runs, tokens_now))) return rc;
    g->low = filled;
    *out = g.release();
    return HS_OK;
}

int hs_migrate_round(hs_migration* g, uint64_t filled, uint64_t upper, uint64_t tokens_now, int* more) {
    using hs::fail;
    if (!g || !more) return fail(HS_E_ARG, "null argument");
    if (upper < filled || filled < g->low) return fail(HS_E_ARG, "need low <= filled <= upper");
    *more = 0;
    if (g->rounds_done) return HS_OK;
    const uint32_t round = g->rep.n_rounds;  // round 0 was the first entry
    if (round > g->opts.max_rounds) {
        g->rounds_done = true;
        return HS_OK;
    }
    // harvest ORs into the carried set: a round harvested and then
    // abandoned keeps its pages (migrate.rs:300-306)
    std::vector<uint64_t> w(g->n_words);
    int rc = hs_kv_harvest(g->src, w.data(), w.size());
    if (rc) return rc;
    for (uint64_t i = 0; i < g->n_words; i++) g->dirty[i] |= w[i];
    // Every page harvested holds writes of positions below `clip`, so the
    // set can be cleared once these runs are sent.
    const uint64_t clip = std::min<uint64_t>(upper + 1, g->spec.max_ctx);
    std::vector<uint64_t> runs;
    live_runs(g, g->dirty.data(), g->low, clip, &runs);
    const uint64_t bytes = total_bytes(runs);
    hs_migrate_report& r = g->rep;
    if (bytes == 0) {
        set_reason(&r, "nothing left to send");
        g->rounds_done = true;
        return HS_OK;
    }
    if (bytes >= g->prev) {  // not shrinking: stop and take the pause (migrate.rs:319-329)
        r.converged = 0;
        set_reason(&r, "round " + std::to_string(round) + " would send " + fmt_bytes(bytes) + " after " +
                           fmt_bytes(g->prev) + ", no smaller -- link cannot outrun the sequence");
        g->rounds_done = true;
        return HS_OK;
    }
    if ((rc = push_round(g, round, runs, tokens_now))) return rc;
    std::fill(g->dirty.begin(), g->dirty.end(), 0);  // these pages are now on the far side
    g->low = filled;
    if (bytes <= g->opts.target_bytes) {
        set_reason(&r, "round fits in the " + fmt_bytes(g->opts.target_bytes) + " budget");
        g->rounds_done = true;
        return HS_OK;
    }
    g->prev = bytes;
    if (round == g->opts.max_rounds) {
        set_reason(&r, "round budget of " + std::to_string(g->opts.max_rounds) + " used up");
        g->rounds_done = true;
        return HS_OK;
    }
    *more = 1;
    return HS_OK;
}

int hs_migrate_finish(hs_migration* g, uint64_t filled, uint64_t tokens_total, double park_us,
                      hs_migrate_report* out) {
    using hs::fail;
    if (!g || !out) return fail(HS_E_ARG, "null argument");
    if (filled > g->spec.max_ctx || filled < g->low) return fail(HS_E_ARG, "filled below the pre-copy or past max_ctx");
    hs_migrate_report& r = g->rep;
    r.precopy_ms = us_since(g->precopy_start) / 1000.0;
    r.park_us = park_us;
    // ---- stop and copy: the loop is parked at a token boundary, so
    // nothing is half-written and `filled` is exact (migrate.rs:347-394)
    const auto t_parked = Clock::now();
    std::vector<uint64_t> w(g->n_words);
    int rc = hs_kv_harvest(g->src, w.data(), w.size());
    if (rc) return rc;
    for (uint64_t i = 0; i < g->n_words; i++) g->dirty[i] |= w[i];
    std::vector<uint64_t> runs;
    live_runs(g, g->dirty.data(), g->low, filled, &runs);
    const auto t_send = Clock::now();
    if ((rc = hs_kv_copy_runs(g->src, g->dst, runs.data(), runs.size() / 2))) return rc;
    r.stw_send_us = us_since(t_send);
    r.final_bytes = total_bytes(runs);
    // Destination: with verify, hash both live caches before taking over
    // (migrate.rs:582-594); the window includes it. Without verify no hash
    // is taken (each is a device-to-host read of the whole live cache) and
    // the report's hashes stay 0.
    const auto t_dest = Clock::now();
    r.verified = g->opts.verify ? 1 : 0;
    if (g->opts.verify) {
        if ((rc = hs_kv_hash(g->dst, (uint32_t)filled, &r.kv_hash_dst))) return rc;
        if ((rc = hs_kv_hash(g->src, (uint32_t)filled, &r.kv_hash_src))) return rc;
    }
    r.dest_resume_us = us_since(t_dest);
    r.stw_us = us_since(t_parked) + park_us;
    std::vector<uint64_t> live(2 * (size_t)(2 * g->spec.n_layers * g->spec.n_kv_heads + 2));
    uint64_t n_live = hs_kv_live_ranges_between(&g->spec, 0, (uint32_t)filled, live.data(), live.size() / 2);
    r.live_bytes = 0;
    for (uint64_t i = 0; i < std::min<uint64_t>(n_live, live.size() / 2); i++) r.live_bytes += live[2 * i + 1];
    r.filled = filled;
    r.tokens_total = tokens_total;
    if ((rc = hs_kv_disarm(g->src))) return rc;
    *out = r;
    if (r.kv_hash_src != r.kv_hash_dst) {
        char m[160];
        std::snprintf(m, sizeof m, "KV cache differs after transfer: source %#018llx, destination %#018llx",
                      (unsigned long long)r.kv_hash_src, (unsigned long long)r.kv_hash_dst);
        return fail(HS_E_STATE, m);
    }
    return HS_OK;
}

void hs_migrate_free(hs_migration* g) { delete g; }

}  // extern "C"
