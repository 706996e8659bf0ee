"""Data-parallel batched decode on the GPUs of one node, every sequence live-
migrated to another GPU by dirty-page pre-copy over NVLink (the 8-GPU
serving configuration: 64 sequences per GPU, 64-token uniform-random
prompts, 200 decode steps at temperature 0.8; sequence j, homed on GPU
j // 64, moves to GPU (home + 1) % N once it holds `at_j` positions, at_j
drawn from the seed in [40, 160]).

    python -m hotseat_b200.serve --gpus N [--seqs 64] [--prompt 64] [--steps 200] [--seed 7] [--round-tokens 8]

One process drives all N GPUs (one model replica, one batch and one worker
thread per GPU) in lockstep rounds: each round every GPU advances its
resident sequences by up to `round_tokens` tokens (hs_batch_seq_begin / step
/ end on the tensor-core path; the host sees the sequences only between
rounds). The run is made twice from the same seeds: unmigrated
(every sequence stays home) and migrated. A migration follows migrate.rs's
pre-copy: at `at_j` the source KV region is armed and its live bytes copied
to a region on the destination GPU while the sequence keeps decoding on the
source; after each of the next rounds the pages it dirtied are copied; after
the third the sequence is parked at a token boundary, the residue is copied,
its state (tokens, SeqState, RNG) is handed over and it continues on the
destination. Batched results do not depend on the batch a sequence is in,
so every migrated transcript, RNG state and KV hash must equal the
unmigrated run's.

Prints one JSON line: aggregate decode tok/s of the migrated run (host-driven
rounds, so the host loop's overhead is included), the unmigrated run's, the
equality checks, and the bytes moved per pre-copy round. With N = 1 the
destination is a second region on the same GPU.
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

PRECOPY_ROUNDS = 3  # rounds the source keeps decoding between the first copy and the hand-over


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


def _round(batch, resident, n_tokens):
    """Up to n_tokens tokens for every resident sequence of one GPU."""
    if not resident:
        return
    batch.begin([q["kv"] for q in resident], resident)
    batch.step(n_tokens)
    for q, (toks, st, rng) in zip(resident, batch.end()):
        q["tokens"] = [int(t) for t in toks]
        q["filled"], q["done"], q["done_reason"] = st.filled, st.done, st.done_reason
        q["rng"] = rng


def run(models, batches, seqs, migrate, pool, round_tokens):
    n = len(models)
    spec = {g: models[g].kv_spec(hs.TOKEN_MAJOR) for g in range(n)}
    for q in seqs:
        q["gpu"], q["kv"] = q["home"], models[q["home"]].kv()
        q["mig"] = "none" if migrate else "off"
    sent = {}  # pre-copy round -> bytes moved by each migration in that round
    generated = 0
    t0 = time.perf_counter()
    while True:
        live = [q for q in seqs if not q["done"]]
        if not live:
            break
        before = {q["j"]: len(q["tokens"]) for q in live}
        list(pool.map(lambda g: _round(batches[g], [q for q in live if q["gpu"] == g], round_tokens), range(n)))
        generated += sum(len(q["tokens"]) - before[q["j"]] for q in live)
        if not migrate:
            continue
        # pre-copy steps between rounds (every loop is parked at a token boundary here)
        for q in live:
            src = q["kv"]
            if q["mig"] == "none" and q["filled"] >= q["at"]:
                dst_gpu = (q["gpu"] + 1) % n
                q["dst_gpu"], q["dst"] = dst_gpu, models[dst_gpu].kv()
                q["all_pages"] = np.full(src.n_words, ~np.uint64(0), dtype=np.uint64)
                src.arm()
                clip = min(q["filled"] + 1, models[q["gpu"]].cfg.max_ctx)
                runs = hs.runs_to_byte_runs(q["all_pages"], src.n_pages, src.page_size,
                                            hs.live_ranges_between(spec[q["gpu"]], 0, clip))
                src.copy_runs_to(q["dst"], runs)
                sent.setdefault(0, []).append(sum(r[1] for r in runs))
                q["low"], q["mig"], q["rounds"] = clip - 1, "precopy", 0
            elif q["mig"] == "precopy":
                dirty = src.harvest()
                q["rounds"] += 1
                if q["rounds"] < PRECOPY_ROUNDS and not q["done"]:
                    clip = min(q["filled"] + 1, models[q["gpu"]].cfg.max_ctx)
                    runs = hs.runs_to_byte_runs(dirty, src.n_pages, src.page_size,
                                                hs.live_ranges_between(spec[q["gpu"]], q["low"], clip))
                    q["low"] = clip - 1
                else:
                    # parked: the residue, then the hand-over
                    runs = hs.runs_to_byte_runs(dirty, src.n_pages, src.page_size,
                                                hs.live_ranges_between(spec[q["gpu"]], q["low"], q["filled"]))
                src.copy_runs_to(q["dst"], runs)
                sent.setdefault(q["rounds"], []).append(sum(r[1] for r in runs))
                if q["rounds"] >= PRECOPY_ROUNDS or q["done"]:
                    src.disarm()
                    if src.hash(q["filled"]) != q["dst"].hash(q["filled"]):
                        raise RuntimeError(f"sequence {q['j']}: destination KV differs after the hand-over")
                    src.close()
                    q["kv"], q["gpu"], q["mig"] = q["dst"], q["dst_gpu"], "done"
                    del q["dst"]
    seconds = time.perf_counter() - t0
    out = {q["j"]: (list(q["tokens"]), tuple(q["rng"].s), q["rng"].draws, q["kv"].hash(q["filled"])) for q in seqs}
    for q in seqs:
        q["kv"].close()
    return out, generated, seconds, sent


def serve(path, n_gpus, per_gpu, prompt, steps, seed, at_range=(40, 160), round_tokens=8):
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
                results[migrate] = run(models, batches, seqs, migrate, pool, round_tokens)
    finally:
        for b in batches:
            b.close()
        for m in models:
            m.close()
    ref, gen0, sec0, _ = results[False]
    got, gen1, sec1, sent = results[True]
    return {
        "bench": "serve_migrate", "n_gpus": n_gpus, "sequences": n_gpus * per_gpu, "prompt": prompt,
        "steps": steps, "numeric": "tc", "round_tokens": round_tokens,
        "tok_s_migrated": gen1 / sec1, "tok_s_unmigrated": gen0 / sec0, "generated_tokens": gen1,
        "migrations": len(sent.get(0, [])), "precopy_rounds": PRECOPY_ROUNDS,
        "bytes_per_migration_by_round": {str(k): float(np.mean(v)) for k, v in sorted(sent.items())},
        "transcripts_equal": all(got[j][0] == ref[j][0] for j in ref),
        "rng_equal": all(got[j][1:3] == ref[j][1:3] for j in ref),
        "kv_hash_equal": all(got[j][3] == ref[j][3] for j in ref),
        "timing": "host wall clock over lockstep rounds (begin/step/end per GPU per round)",
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--seqs", type=int, default=64, help="sequences per GPU")
    ap.add_argument("--prompt", type=int, default=64)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--seed", type=int, default=7)
    ap.add_argument("--round-tokens", type=int, default=8, help="tokens per lockstep round")
    args = ap.parse_args()
    td = tempfile.mkdtemp(prefix="hsserve")
    path = os.path.join(td, "q05.gguf")
    write_synthetic_gguf(path, seed=1234, **QWEN05)
    try:
        rec = serve(path, args.gpus, args.seqs, args.prompt, args.steps, args.seed, round_tokens=args.round_tokens)
    finally:
        os.remove(path)
        os.rmdir(td)
    print(json.dumps(rec), flush=True)
    if not (rec["transcripts_equal"] and rec["rng_equal"] and rec["kv_hash_equal"]):
        raise SystemExit(1)


if __name__ == "__main__":
    main()
