"""Data-parallel serving with live migration across processes: one rank per
GPU (torch.distributed), each decoding its own sequences on the tensor-core
path, every sequence migrated once to the next rank's GPU by hs_migrate_*
(the pre-copy of hs-worker migrate.rs) into a KV region that the next rank
owns and exported by CUDA IPC (hs_kv_ipc_handle / hs_kv_open_ipc): the
source writes the destination's memory over NVLink.

Protocol, the same steps on every rank in the same order:
  set-up   rank r makes its home sequences (global id j = r * per + i, seeded
           prompt and migration point at_j) and `per` inbound regions, one per
           home sequence of rank r - 1; the handles are all-gathered and rank r
           opens rank r + 1's inbound regions as its destinations (with one
           rank, its own).
  round    launch the resident sequences' next `round_tokens` tokens; while
           they run, one pre-copy round of every outgoing migration
           (upper = filled + round_tokens); park; hand over the migrations whose
           rounds stopped (the residue with the loop parked, then the state
           record: id, tokens, SeqState, RNG, inbound slot); start a migration
           for every sequence that reached at_j; all-gather the hand-over
           records (each rank adopts those addressed to it) and the count of
           unfinished sequences, which ends the loop on every rank at once.
A run without migrations follows the same rounds, so the two runs' transcripts,
RNG states and KV hashes must be equal.

The engine is an argument: `GpuEngine` drives libhotseat; the multi-rank
tests drive the same protocol on CPU ranks with a stand-in engine.
"""
import numpy as np


class GpuEngine:
    """One rank's device side: a tensor-core model and batch on `device`."""

    def __init__(self, path, device, max_ctx, capacity):
        import hotseat_b200 as hs
        self.hs = hs
        self.model = hs.Model.load(path, max_ctx=max_ctx, device=device, numeric=hs.NUMERIC_TC)
        self.batch = hs.Batch(self.model, capacity)
        self.vocab = self.model.cfg.vocab

    def new_kv(self):
        return self.model.kv()

    def export(self, kv):
        return kv.ipc_handle()

    def open_remote(self, handle):
        return self.hs.Kv.open_ipc(self.model, handle)

    def sampler(self, seed):
        return self.hs.SamplerCfg.default(temperature=0.8, seed=seed), self.hs.Rng.seed(seed)

    def launch(self, seqs, n_tokens):
        if seqs:
            self.batch.begin([q["kv"] for q in seqs], seqs)
            self.batch.step(n_tokens)

    def park(self, seqs):
        if not seqs:
            return
        for q, (toks, st, rng) in zip(seqs, self.batch.end()):
            q["tokens"] = [int(t) for t in toks]
            q["filled"], q["done"], q["done_reason"] = st.filled, st.done, st.done_reason
            q["rng"] = rng

    def migration(self, src, dst, filled, tokens_now, max_rounds, verify):
        return self.hs.Migration(src, dst, filled, tokens_now, max_rounds=max_rounds, verify=verify)

    def rng_state(self, rng):
        return [int(x) for x in rng.s], int(rng.draws)

    def rng_from(self, state):
        r = self.hs.Rng()
        r.s[:] = state[0]
        r.draws = state[1]
        return r

    def kv_hash(self, kv, n_pos):
        return kv.hash(n_pos)

    def start_clock(self):
        import torch
        self._ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        self._ev[0].record(torch.cuda.ExternalStream(self.batch.stream))

    def stop_clock(self):
        import torch
        self._ev[1].record(torch.cuda.ExternalStream(self.batch.stream))
        self._ev[1].synchronize()
        return self._ev[0].elapsed_time(self._ev[1]) / 1000.0

    def close(self):
        self.batch.close()
        self.model.close()


def home_sequences(rank, per, prompt_len, steps, seed, at_range, vocab, max_ctx):
    """Rank `rank`'s home sequences, each a pure function of (seed, global id)."""
    out = []
    for i in range(per):
        j = rank * per + i
        g = np.random.default_rng([seed, j])
        prompt = [int(t) for t in g.integers(0, vocab, size=prompt_len)]
        at = int(g.integers(at_range[0], at_range[1] + 1))
        out.append(dict(j=j, slot=i, at=at, tokens=prompt, prompt_len=prompt_len, max_tokens=steps, filled=0,
                        done=0, done_reason=0, seed=seed * 100003 + j, max_ctx=max_ctx))
    return out


def run_rank(engine, dist, rank, world, per, prompt_len, steps, seed, migrate, max_ctx, round_tokens=8,
             max_rounds=3, verify=False, at_range=(40, 160)):
    """The protocol above on one rank. Returns (results of the sequences that
    finished here: {j: (tokens, rng state, kv hash)}, tokens generated here,
    seconds on this rank's device clock, hand-over reports of the migrations
    this rank sent)."""
    seqs = home_sequences(rank, per, prompt_len, steps, seed, at_range, engine.vocab, max_ctx)
    for q in seqs:
        q["cfg"], q["rng"] = engine.sampler(q["seed"])
        q["kv"] = engine.new_kv()
        q["mig"] = "none" if migrate else "off"
    inbound = [engine.new_kv() for _ in range(per)]
    handles = [None] * world
    dist.all_gather_object(handles, [engine.export(kv) for kv in inbound])
    nxt = (rank + 1) % world
    dests = inbound if nxt == rank else [engine.open_remote(h) for h in handles[nxt]]
    resident = list(seqs)
    finished = {}
    reports = []
    generated = 0
    engine.start_clock()
    while True:
        live = [q for q in resident if not q["done"]]
        before = {q["j"]: len(q["tokens"]) for q in live}
        engine.launch(live, round_tokens)
        for q in live:  # pre-copy rounds while the steps are in flight
            if q["mig"] == "precopy":
                upper = min(q["filled"] + round_tokens, q["max_ctx"] - 1)
                q["more"] = q["m"].round(q["filled"], len(q["tokens"]), upper=upper)
        engine.park(live)
        generated += sum(len(q["tokens"]) - before[q["j"]] for q in live)
        records = []
        for q in live:
            if q["mig"] == "precopy" and (not q["more"] or q["done"]):
                rep = q["m"].finish(q["filled"], len(q["tokens"]))
                q["m"].close()
                reports.append(rep)
                records.append(dict(to=nxt, j=q["j"], slot=q["slot"], tokens=list(q["tokens"]),
                                    prompt_len=q["prompt_len"], max_tokens=q["max_tokens"], filled=q["filled"],
                                    done=q["done"], done_reason=q["done_reason"], seed=q["seed"],
                                    rng=engine.rng_state(q["rng"])))
                q["mig"] = "gone"
            elif q["mig"] == "none" and q["filled"] >= q["at"] and not q["done"]:
                q["m"] = engine.migration(q["kv"], dests[q["slot"]], q["filled"], len(q["tokens"]), max_rounds,
                                          verify)
                q["mig"], q["more"] = "precopy", True
        for q in resident:
            if q["done"] and q["mig"] in ("none", "off", "arrived"):
                finished[q["j"]] = (list(q["tokens"]), engine.rng_state(q["rng"]),
                                    engine.kv_hash(q["kv"], q["filled"]))
        resident = [q for q in resident if not (q["done"] and q["mig"] in ("none", "off", "arrived"))
                    and q["mig"] != "gone"]
        gathered = [None] * world
        dist.all_gather_object(gathered, (records, sum(1 for q in resident if not q["done"]) + len(records)))
        for recs, _ in gathered:
            for r in recs:
                if r["to"] != rank:
                    continue
                cfg, _ = engine.sampler(r["seed"])
                resident.append(dict(j=r["j"], slot=r["slot"], at=0, tokens=r["tokens"], prompt_len=r["prompt_len"],
                                     max_tokens=r["max_tokens"], filled=r["filled"], done=r["done"],
                                     done_reason=r["done_reason"], seed=r["seed"], cfg=cfg,
                                     rng=engine.rng_from(r["rng"]), kv=inbound[r["slot"]], mig="arrived",
                                     max_ctx=max_ctx))
        if sum(n for _, n in gathered) == 0:
            break
    for q in resident:  # sequences that arrived already finished
        if q["mig"] == "arrived" and q["done"]:
            finished[q["j"]] = (list(q["tokens"]), engine.rng_state(q["rng"]), engine.kv_hash(q["kv"], q["filled"]))
    seconds = engine.stop_clock()
    return finished, generated, seconds, reports


def serve_dist(engine, dist, rank, world, per=64, prompt_len=64, steps=200, seed=7, round_tokens=8, max_rounds=3,
               verify=False, at_range=(40, 160)):
    """Both runs (without and with migrations) on every rank; rank 0 returns
    the record (others None). Times are each rank's device clock, maximum
    over ranks."""
    max_ctx = prompt_len + steps + 8
    out = {}
    for migrate in (False, True):
        fin, gen, sec, reps = run_rank(engine, dist, rank, world, per, prompt_len, steps, seed, migrate, max_ctx,
                                       round_tokens, max_rounds, verify, at_range)
        allv = [None] * world
        dist.all_gather_object(allv, (fin, gen, sec, [(r["stw_us"], r["final_bytes"], r["precopy_bytes"],
                                                       r["converged"]) for r in reps]))
        out[migrate] = allv
    if rank != 0:
        return None

    def merge(run):
        fin = {}
        for f, _, _, _ in run:
            fin.update(f)
        return fin, sum(g for _, g, _, _ in run), max(s for _, _, s, _ in run), [x for *_, r in run for x in r]

    ref, gen0, sec0, _ = merge(out[False])
    got, gen1, sec1, reps = merge(out[True])
    stw = [r[0] for r in reps]
    return {
        "workload": f"{per} sequences per GPU, prompt {prompt_len}, {steps} steps, temp 0.8, every sequence migrated "
                    f"once to the next rank's GPU (pre-copy, CUDA IPC peer stores)",
        "n_gpus": world, "sequences": world * per, "round_tokens": round_tokens,
        "tok_s_unmigrated": gen0 / sec0, "tok_s_migrated": gen1 / sec1, "migrations": len(reps),
        "stw_us_p50": float(np.percentile(stw, 50)) if stw else None,
        "stw_us_max": float(max(stw)) if stw else None,
        "bytes_per_migration": float(np.mean([r[1] + r[2] for r in reps])) if reps else None,
        "converged": sum(r[3] for r in reps),
        "transcripts_equal": len(ref) == world * per and all(got.get(j, (None,))[0] == ref[j][0] for j in ref),
        "rng_equal": all(got.get(j, (None, None))[1] == ref[j][1] for j in ref),
        "kv_hash_equal": all(got.get(j, (None, None, None))[2] == ref[j][2] for j in ref),
        "timing": "each rank's device clock over its lockstep rounds (host-driven), maximum over ranks",
    }


class Solo:
    """The object collective of a single process (no process group)."""

    @staticmethod
    def all_gather_object(out, obj):
        out[0] = obj


def main():
    """python -m hotseat_b200.serve_dist [--seqs 64] [--prompt 64] [--steps 200]
    under torchrun (one rank per GPU) or alone (one GPU)."""
    import argparse
    import datetime
    import json
    import os
    import sys
    import tempfile

    import torch
    import torch.distributed as dist
    ap = argparse.ArgumentParser()
    ap.add_argument("--seqs", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=64)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--round-tokens", type=int, default=8)
    ap.add_argument("--verify", action="store_true")
    args = ap.parse_args()
    rank, world, local = (int(os.environ.get(k, d)) for k, d in (("RANK", 0), ("WORLD_SIZE", 1), ("LOCAL_RANK", 0)))
    torch.cuda.set_device(local)
    group = Solo
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
        group = dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from tests.golden.synth import QWEN05, write_synthetic_gguf
    td = tempfile.mkdtemp(prefix="hsserve")
    path = os.path.join(td, "q05.gguf")
    if rank == 0:
        write_synthetic_gguf(path, seed=1234, **QWEN05)
    if world > 1:
        paths = [path]
        dist.broadcast_object_list(paths, src=0)
        path = paths[0]
        dist.barrier()
    eng = GpuEngine(path, local, args.prompt + args.steps + 8, 2 * args.seqs)
    try:
        rec = serve_dist(eng, group, rank, world, per=args.seqs, prompt_len=args.prompt, steps=args.steps,
                         round_tokens=args.round_tokens, verify=args.verify)
        if world > 1:
            dist.barrier()
        if rank == 0:
            print(json.dumps(rec), flush=True)
    finally:
        eng.close()
        if world > 1:
            dist.destroy_process_group()
        if rank == 0:
            os.remove(path)
            os.rmdir(td)


if __name__ == "__main__":
    main()
