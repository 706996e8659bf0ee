"""Data-parallel batched decode on the GPUs of one node, every sequence live-
migrated to another GPU by dirty-page pre-copy over NVLink (the 8-GPU
serving configuration: 64 sequences per GPU, 64-token uniform-random
prompts, 200 decode steps at temperature 0.8; sequence j, homed on GPU
j // 64, moves to GPU (home + 1) % N once it holds `at_j` positions, at_j
drawn from the seed in [40, 160]).

    python -m hotseat_b200.serve --gpus N [--seqs 64] [--prompt 64] [--steps 200] [--seed 7] [--round-tokens 8]
                                [--verify]

One process drives all N GPUs (one model replica, one batch and one worker
thread per GPU) in lockstep rounds: each round every GPU advances its
resident sequences by up to `round_tokens` tokens (hs_batch_seq_begin / step
/ end on the tensor-core path; the host sees the sequences only between
rounds). The run is made twice from the same seeds: unmigrated (every
sequence stays home) and migrated. A migration is hs_migrate_* (the
pre-copy of migrate.rs): at `at_j` the source KV region is armed and round 0
copies its live bytes to a region on the destination GPU; while the next
rounds' decode steps are in flight the pages dirtied since the last harvest
are copied (migrate.rs's convergence rules decide when the rounds stop, at
most MAX_ROUNDS); then, with the loop parked at a token boundary, the
residue is copied, the state (tokens, SeqState, RNG) is handed over and the
sequence continues on the destination. `--verify` hashes both KV caches
inside every hand-over (Opts::verify, off by default as in the reference).
Batched results do not depend on the batch a sequence is in, so every
migrated transcript, RNG state and KV hash must equal the unmigrated run's.

Prints one JSON line: aggregate decode tok/s of the migrated run (host-driven
rounds, so the host loop's overhead is included), the unmigrated run's, the
equality checks, the bytes moved per pre-copy round and the stop-the-world
window of the hand-overs (migrate.rs Report). With N = 1 the destination is
a second region on the same GPU.
"""
import argparse
import json
import os
import sys
import tempfile
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

import hotseat_b200 as hs

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from tests.golden.synth import QWEN05, write_synthetic_gguf  # noqa: E402  (fixture writer)

MAX_ROUNDS = 3  # pre-copy rounds after round 0 before the hand-over at the latest


def _sequences(n_gpus, per_gpu, prompt_len, steps, seed, at_range, vocab):
    g = np.random.default_rng(seed)
    seqs = []
    for j in range(n_gpus * per_gpu):
        prompt = [int(t) for t in g.integers(0, vocab, size=prompt_len)]
        at = int(g.integers(at_range[0], at_range[1] + 1))
        seqs.append(dict(j=j, home=j // per_gpu, at=at, tokens=prompt, prompt_len=prompt_len, max_tokens=steps,
                         cfg=hs.SamplerCfg.default(temperature=0.8, seed=seed * 1000 + j),
                         rng=hs.Rng.seed(seed * 1000 + j), filled=0, done=0, done_reason=0))
    return seqs


def _launch(batch, resident, n_tokens):
    """Enqueue up to n_tokens tokens for every resident sequence of one GPU."""
    if resident:
        batch.begin([q["kv"] for q in resident], resident)
        batch.step(n_tokens)


def _park(batch, resident):
    """Wait for the GPU's round and take the sequences' state back."""
    if not resident:
        return
    for q, (toks, st, rng) in zip(resident, batch.end()):
        q["tokens"] = [int(t) for t in toks]
        q["filled"], q["done"], q["done_reason"] = st.filled, st.done, st.done_reason
        q["rng"] = rng


def run(models, batches, seqs, migrate, pool, round_tokens, verify=False):
    n = len(models)
    for q in seqs:
        q["gpu"], q["kv"] = q["home"], models[q["home"]].kv()
        q["mig"] = "none" if migrate else "off"
    reports = []
    generated = 0
    t0 = time.perf_counter()
    while True:
        live = [q for q in seqs if not q["done"]]
        if not live:
            break
        before = {q["j"]: len(q["tokens"]) for q in live}
        resident = [[q for q in live if q["gpu"] == g] for g in range(n)]
        list(pool.map(lambda g: _launch(batches[g], resident[g], round_tokens), range(n)))
        # pre-copy rounds of the sequences being migrated, while their
        # decode steps are in flight (positions up to filled + round_tokens
        # may be written meanwhile)
        for q in live:
            if q["mig"] == "precopy":
                upper = min(q["filled"] + round_tokens, q["max_ctx"] - 1)
                q["more"] = q["m"].round(q["filled"], len(q["tokens"]), upper=upper)
        list(pool.map(lambda g: _park(batches[g], resident[g]), range(n)))
        generated += sum(len(q["tokens"]) - before[q["j"]] for q in live)
        if not migrate:
            continue
        # every decode loop is parked here: hand-overs, then new migrations
        for q in live:
            if q["mig"] == "precopy" and (not q["more"] or q["done"]):
                t_park = time.perf_counter()
                rep = q["m"].finish(q["filled"], len(q["tokens"]), park_us=0.0)
                q["m"].close()
                q["kv"].close()
                q["kv"], q["gpu"], q["mig"] = q["dst"], q["dst_gpu"], "done"
                rep["handover_us"] = (time.perf_counter() - t_park) * 1e6
                reports.append(rep)
                del q["dst"], q["m"]
            elif q["mig"] == "none" and q["filled"] >= q["at"] and not q["done"]:
                dst_gpu = (q["gpu"] + 1) % n
                q["dst_gpu"], q["dst"] = dst_gpu, models[dst_gpu].kv()
                q["m"] = hs.Migration(q["kv"], q["dst"], q["filled"], len(q["tokens"]), max_rounds=MAX_ROUNDS,
                                      verify=verify)
                q["mig"], q["more"] = "precopy", True
    seconds = time.perf_counter() - t0
    out = {q["j"]: (list(q["tokens"]), tuple(q["rng"].s), q["rng"].draws, q["kv"].hash(q["filled"])) for q in seqs}
    for q in seqs:
        q["kv"].close()
    return out, generated, seconds, reports


def serve(path, n_gpus, per_gpu, prompt, steps, seed, at_range=(40, 160), round_tokens=8, verify=False):
    """Both runs on the GGUF at `path`; returns the result record."""
    max_ctx = prompt + steps + 8
    models = [hs.Model.load(path, max_ctx=max_ctx, device=g, numeric=hs.NUMERIC_TC) for g in range(n_gpus)]
    # room for the home sequences and the ones migrating in
    batches = [hs.Batch(models[g], 2 * per_gpu) for g in range(n_gpus)]
    results = {}
    try:
        with ThreadPoolExecutor(max_workers=n_gpus) as pool:
            for migrate in (False, True):
                seqs = _sequences(n_gpus, per_gpu, prompt, steps, seed, at_range, models[0].cfg.vocab)
                for q in seqs:
                    q["max_ctx"] = max_ctx
                results[migrate] = run(models, batches, seqs, migrate, pool, round_tokens, verify)
    finally:
        for b in batches:
            b.close()
        for m in models:
            m.close()
    ref, gen0, sec0, _ = results[False]
    got, gen1, sec1, reports = results[True]
    by_round = {}
    for r in reports:
        for st in r["rounds"]:
            by_round.setdefault(st["index"], []).append(st["bytes"])
        by_round.setdefault("final", []).append(r["final_bytes"])

    def pct(key, q):
        v = [r[key] for r in reports]
        return float(np.percentile(v, q)) if v else None

    return {
        "bench": "serve_migrate", "n_gpus": n_gpus, "sequences": n_gpus * per_gpu, "prompt": prompt,
        "steps": steps, "numeric": "tc", "round_tokens": round_tokens, "verify": verify,
        "tok_s_migrated": gen1 / sec1, "tok_s_unmigrated": gen0 / sec0, "generated_tokens": gen1,
        "migrations": len(reports), "max_rounds": MAX_ROUNDS,
        "bytes_per_migration_by_round": {str(k): float(np.mean(v)) for k, v in by_round.items()},
        "stw_us": {"p50": pct("stw_us", 50), "p90": pct("stw_us", 90), "max": pct("stw_us", 100)},
        "stw_send_us_p50": pct("stw_send_us", 50), "handover_us_p50": pct("handover_us", 50),
        "precopy_ms_p50": pct("precopy_ms", 50),
        "converged": sum(r["converged"] for r in reports),
        "stop_reasons": sorted({r["stop_reason"] for r in reports}),
        "transcripts_equal": all(got[j][0] == ref[j][0] for j in ref),
        "rng_equal": all(got[j][1:3] == ref[j][1:3] for j in ref),
        "kv_hash_equal": all(got[j][3] == ref[j][3] for j in ref),
        "timing": "host wall clock over lockstep rounds; pre-copy rounds run while the decode steps are in flight; "
                  "stw_us = the hand-over's residue harvest + copy (+ both KV hashes with verify), the loop parked",
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--seqs", type=int, default=64, help="sequences per GPU")
    ap.add_argument("--prompt", type=int, default=64)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--seed", type=int, default=7)
    ap.add_argument("--round-tokens", type=int, default=8, help="tokens per lockstep round")
    ap.add_argument("--verify", action="store_true", help="hash both KV caches inside every hand-over")
    args = ap.parse_args()
    td = tempfile.mkdtemp(prefix="hsserve")
    path = os.path.join(td, "q05.gguf")
    write_synthetic_gguf(path, seed=1234, **QWEN05)
    try:
        rec = serve(path, args.gpus, args.seqs, args.prompt, args.steps, args.seed, round_tokens=args.round_tokens,
                    verify=args.verify)
    finally:
        os.remove(path)
        os.rmdir(td)
    print(json.dumps(rec), flush=True)
    if not (rec["transcripts_equal"] and rec["rng_equal"] and rec["kv_hash_equal"]):
        raise SystemExit(1)


if __name__ == "__main__":
    main()
