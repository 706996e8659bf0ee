"""Decode throughput of the hotseat token loop on B200.

Headline workload (the batch-64 configuration of the metric): the seeded
random-init Qwen2.5-0.5B-shape GGUF (24 layers, d 896, 14/2 heads, ff 4864,
vocab 151936, Q6_K embedding, Q4_K weights, f32 norms/biases), 64 independent
sequences, each with a 128-token uniform-random prompt, 256 generated tokens
at temperature 0.8 with seed 99+i, f32 KV, decoded together on the
tensor-core path (HS_NUMERIC_TC). One step = the 256-token decode phase of
all 64 sequences (16,384 tokens: batched forward, device sampling and
seq.rs commit per token) from their post-prompt state, restored before
each step. `value` is decode tok/s with that state already in HBM; `e2e` is
the same through hs_batch_seq_run with host token buffers.

The batch-1 configuration of the metric (36-token prompt, 120 tokens,
temperature 0.8, seed 99, GPU-native numeric path) is measured in the same
run and reported under "batch1".

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Under torchrun each rank decodes its own 64 sequences on its own GPU
(independent sequences shard with no collective); value = all ranks' tokens
/ max time over ranks.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s per GPU, Qwen2.5-0.5B-shape, batch 1/64; % of HBM roofline"
UNIT = "tok/s"
MODEL_SEED = 1234
SEED, TEMP = 99, 0.8
B64_SEQS, B64_PROMPT, B64_GEN, B64_CTX = 64, 128, 256, 512
B1_PROMPT, B1_GEN, B1_CTX = 36, 120, 2048
CTL_BYTES = 160  # sizeof(DevCtl), the device control block copied each way per sequence
D, FF, NH, NKV, HD, L, V = 896, 4864, 14, 2, 64, 24, 151936
KV_ROW = L * 2 * NKV * HD * 4  # bytes of K and V one position adds across the layers (24,576)
WEIGHT_BYTES = L * 2 * ((NH + 2 * NKV) * HD * D + D * NH * HD + 3 * FF * D) + V * D * 2
SMALL_BYTES = L * 4 * (2 * D + (NH + 2 * NKV) * HD) + D * 4


def workload_config(world=1):
    return {"workload": "qwen2.5-0.5b-shape batched decode: 64 sequences per GPU, prompt 128, gen 256, temp 0.8, "
                        "seed 99+i, f32 KV",
            "model_shape": "24L d896 14/2h hd64 ff4864 vocab151936 Q6_K-embd Q4_K-weights",
            "global_batch": B64_SEQS * world, "max_ctx": B64_CTX,
            "l2": "weights 0.99 GB stream per decode step > 126 MB L2 (no flush needed)"}


def b64_bytes_per_step():
    """Algorithmic HBM bytes of one batched decode step (64 tokens), averaged
    over the decode phase: f16 weights + norms/biases once, each sequence's KV
    read (pos+1 rows) and write, and the logits written and read back."""
    kv = np.mean([B64_SEQS * ((p + 1) * KV_ROW + KV_ROW) for p in range(B64_PROMPT, B64_PROMPT + B64_GEN)])
    logits = B64_SEQS * V * 4 * 2
    return WEIGHT_BYTES + SMALL_BYTES + kv + logits


def b1_bytes_per_token():
    kv = np.mean([(p + 1) * KV_ROW + KV_ROW for p in range(B1_PROMPT, B1_PROMPT + B1_GEN)])
    return WEIGHT_BYTES + SMALL_BYTES + kv


def make_model(path):
    from tests.golden.synth import QWEN05, write_synthetic_gguf
    write_synthetic_gguf(path, seed=MODEL_SEED, **QWEN05)


def b64_prompts():
    return [[int(t) for t in np.random.default_rng(128 + i).integers(0, V, size=B64_PROMPT)] for i in range(B64_SEQS)]


def b1_prompt():
    return [int(t) for t in np.random.default_rng(36).integers(0, V, size=B1_PROMPT)]


class ClockSampler:
    """nvidia-smi clocks and throttle reasons while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = []
        for line in (self.out or "").strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"]}
        loaded = [r for r in rows if r[2] > 200.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "samples": len(loaded), "power_w_max": max(r[2] for r in rows), "reasons": reasons}


def cpu_sample(path, prompt, max_ctx, n_decode, threads):
    """The CPU restatement of the reference path (oracle/, test infrastructure
    used here only as the baseline): prompt forwarded untimed, then `n_decode`
    tokens timed. The reference decodes each sequence on its own thread over
    one shared pool, so its throughput with many sequences is this rate."""
    from oracle import ffi
    o = ffi.Model(path, max_ctx=max_ctx, threads=threads)
    kv = o.new_kv()
    cfg = ffi.default_cfg(temperature=TEMP, seed=SEED)
    rng = ffi.seeded_rng(SEED)
    toks, st, rng = o.run_seq(kv, prompt, 10 ** 6, cfg, rng, stop_at_filled=len(prompt))
    t0 = time.perf_counter()
    o.run_seq(kv, toks, 10 ** 6, cfg, rng, state=st, stop_at_filled=len(prompt) + n_decode)
    return n_decode / (time.perf_counter() - t0)


CPU_SAMPLE = "12 decode tokens of sequence 0 (128-token prompt forwarded untimed) on all host threads"


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU algorithm (its C++ restatement;
    rustc is not available to build the Rust original) on the host cores,
    on a bounded sample of the batch-64 workload."""
    if rank != 0:
        return
    from oracle import ffi
    ffi.build()
    threads = os.cpu_count() or 1
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "qwen05.gguf")
        make_model(path)
        prompt = b64_prompts()[0]
        vals = []
        for i in range(args.warmup + args.steps):
            v = cpu_sample(path, prompt, B64_CTX, 12, threads)
            if i >= args.warmup:
                vals.append(v)
    value = float(np.mean(vals))
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * 12 / value,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (f16 weights)",
            "data": "synthetic", "config": workload_config(),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": CPU_SAMPLE},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def max_over_ranks(x, world, torch, dist):
    """The largest x over the ranks (a device tensor under NCCL, a host one
    under gloo)."""
    if world == 1:
        return x
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def weak_value(world, units_per_rank, total_ms):
    """Whole-job throughput under weak scaling: every rank processed
    units_per_rank units; total_ms is the slowest rank's time."""
    return world * units_per_rank / (total_ms / 1000.0)


def _copy_rng(hs, r):
    c = hs.Rng()
    c.s[:] = list(r.s)
    c.draws = r.draws
    return c


def bench_batch64(hs, torch, dist, path, local, world, args):
    m = hs.Model.load(path, max_ctx=B64_CTX, device=local, numeric=hs.NUMERIC_TC)
    b = hs.Batch(m, B64_SEQS)
    kvs = [m.kv() for _ in range(B64_SEQS)]
    cfg = hs.SamplerCfg.default(temperature=TEMP, seed=SEED)
    seqs = [dict(tokens=p, prompt_len=B64_PROMPT, max_tokens=B64_GEN, cfg=cfg, rng=hs.Rng.seed(SEED + i))
            for i, p in enumerate(b64_prompts())]
    # Prompt (untimed): the post-prompt state is every step's starting point.
    pre = b.run_seqs(kvs, seqs, stop_at_filled=B64_PROMPT)
    snap = [dict(tokens=list(t), prompt_len=B64_PROMPT, max_tokens=B64_GEN, cfg=cfg, rng=_copy_rng(hs, r),
                 filled=st.filled) for t, st, r in pre]
    n_steps = B64_PROMPT + B64_GEN - min(q["filled"] for q in snap)
    stream = torch.cuda.ExternalStream(b.stream)

    def fresh():
        return [dict(q, rng=_copy_rng(hs, q["rng"])) for q in snap]

    if args.profile_step:
        for _ in range(3):
            b.begin(kvs, fresh())
            b.step(1)
            b.end()
        b.begin(kvs, fresh())
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("decode_step")
        b.step(1)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        b.end()
        print(json.dumps({"profile_step": "done", "workload": "batch64", "launches": b.launches_per_step()}))
        return None

    def one(ev=None):
        b.begin(kvs, fresh())
        if ev:
            ev[0].record(stream)
        b.step(n_steps)
        if ev:
            ev[1].record(stream)
        return b.end()

    for _ in range(args.warmup):
        ref = one()
    gen_tokens = sum(len(t) for t, _, _ in ref) - sum(len(q["tokens"]) for q in snap)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        outs = [one(evs[i]) for i in range(args.steps)]
        torch.cuda.synchronize()
    for o in outs:
        assert all(list(x[0]) == list(y[0]) for x, y in zip(o, ref)), "batched decode is not deterministic"
    total_ms = max_over_ranks(float(sum(a.elapsed_time(z) for a, z in evs)), world, torch, dist)
    if world > 1:
        dist.barrier()
    ms_per_step = total_ms / args.steps
    value = weak_value(world, gen_tokens * args.steps, total_ms)

    # end to end through hs_batch_seq_run with host buffers
    e2e_ms = []
    for _ in range(args.steps):
        a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        out = b.run_seqs(kvs, fresh())
        z.record(stream)
        z.synchronize()
        e2e_ms.append(a.elapsed_time(z))
        assert all(list(x[0]) == list(y[0]) for x, y in zip(out, ref))
    e2e_total = max_over_ranks(float(sum(e2e_ms)), world, torch, dist)
    e2e_value = weak_value(world, gen_tokens * args.steps, e2e_total)
    h2d = sum(len(q["tokens"]) * 4 + CTL_BYTES for q in snap)
    d2h = sum(len(t) * 4 + 2 * CTL_BYTES for t, _, _ in ref)
    launches = b.launches_per_step()
    res = dict(value=value, ms_per_step=ms_per_step, gen_tokens=gen_tokens, n_steps=n_steps, e2e_value=e2e_value,
               h2d=h2d, d2h=d2h, gpu_launches=launches * n_steps * args.steps, launches_per_decode_step=launches,
               clocks=clk.summary())
    b.close()
    m.close()
    return res


def bench_batch1(hs, torch, dist, path, local, world, args):
    import ctypes as C
    m = hs.Model.load(path, max_ctx=B1_CTX, device=local, numeric=hs.NUMERIC_FAST)
    kv, s = m.kv(), m.scratch()
    cfg = hs.SamplerCfg.default(temperature=TEMP, seed=SEED)
    toks, st, rng = hs.run_seq(m, kv, s, b1_prompt(), B1_PROMPT, B1_GEN, cfg, hs.Rng.seed(SEED),
                               stop_at_filled=B1_PROMPT)
    snap_toks, snap_rng = np.array(toks, dtype=np.uint32), _copy_rng(hs, rng)
    snap_state = (st.prompt_len, st.filled, st.max_tokens)
    stream = torch.cuda.ExternalStream(s.stream)
    lib = hs.lib()

    def begin():
        r = _copy_rng(hs, snap_rng)
        sst = hs.SeqState(*snap_state, 0, 0)
        hs._check(lib.hs_seq_begin(s._h, kv._h, hs._ptr(snap_toks), len(snap_toks), B1_CTX + 1, C.byref(sst),
                                   C.byref(cfg), C.byref(r), 0))

    def end():
        out = np.zeros(B1_CTX + 1, dtype=np.uint32)
        n = C.c_uint64()
        sst, r = hs.SeqState(), hs.Rng()
        hs._check(lib.hs_seq_end(s._h, hs._ptr(out), C.byref(n), out.size, C.byref(sst), C.byref(r)))
        return out[: n.value]

    n_steps = B1_PROMPT + B1_GEN - snap_state[1]
    if args.profile_step:
        for _ in range(3):
            begin()
            hs._check(lib.hs_seq_step(s._h, 1))
            end()
        begin()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("decode_step")
        hs._check(lib.hs_seq_step(s._h, 1))
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        end()
        print(json.dumps({"profile_step": "done", "workload": "batch1", "launches": s.launches_per_step()}))
        return None
    for _ in range(args.warmup):
        begin()
        hs._check(lib.hs_seq_step(s._h, n_steps))
        ref = end()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        begin()
        evs[i][0].record(stream)
        hs._check(lib.hs_seq_step(s._h, n_steps))
        evs[i][1].record(stream)
    torch.cuda.synchronize()
    assert list(end()) == list(ref), "decode is not deterministic across steps"
    total_ms = max_over_ranks(float(sum(a.elapsed_time(z) for a, z in evs)), world, torch, dist)
    value = weak_value(world, B1_GEN * args.steps, total_ms)
    e2e_ms = []
    for _ in range(args.steps):
        a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        out, _, _ = hs.run_seq(m, kv, s, snap_toks, snap_state[0], snap_state[2], cfg, _copy_rng(hs, snap_rng),
                               filled=snap_state[1])
        z.record(stream)
        z.synchronize()
        e2e_ms.append(a.elapsed_time(z))
        assert list(out) == list(ref)
    e2e_total = max_over_ranks(float(sum(e2e_ms)), world, torch, dist)
    res = dict(value=value, ms_per_step=total_ms / args.steps,
               e2e_value=weak_value(world, B1_GEN * args.steps, e2e_total),
               gpu_launches=s.launches_per_step() * n_steps * args.steps)
    for o in (s, kv):
        o.close()
    m.close()
    return res


def bench_extra(q05_path):
    """The other configurations, timed on the device (one GPU):
    c3 - Qwen2.5-1.5B shape, 16 sequences x 2048-token prefill (tensor-core
         roofline: 2 x weights x tokens FLOPs) then 512 greedy steps at batch
         16 (HBM roofline);
    c4 - Q4_K/Q6_K dequantisation of 4864x896, 896x4864 and 151936x896
         tensors (L2 flushed between launches), and GQA decode attention at
         1k-32k context, batch 1 and 64 (HBM roofline)."""
    from hotseat_b200 import microbench as mb
    out = {}
    pre, dec = mb.bench_prefill()
    out["c3"] = {"workload": "qwen2.5-1.5b-shape: 16 x 2048-token prefill, then 512 greedy steps at batch 16",
                 "prefill": {k: pre[k] for k in ("pass_tokens", "ms", "tok/s", "gemm_TFLOP/s", "peak_TFLOP/s", "frac",
                                                 "peak_source", "note")},
                 "decode": {k: dec[k] for k in ("ms", "tok/s", "GB/s", "frac", "generated", "note")}}
    out["c4"] = {
        "dequant": [{k: r[k] for k in ("type", "shape", "us", "GB/s", "frac")} for r in mb.bench_dequant(q05_path=q05_path)],
        "attention": [{k: r[k] for k in ("batch", "context", "us_per_layer", "GB/s", "frac")}
                      for r in mb.bench_attention(q05_path=q05_path)],
        "peak_GB/s": mb._peak()[0],
    }
    return out


def bench_c5(path, rank, world, local, dist):
    """c5 - serving with live migration on the job's GPUs: 64 sequences per
    GPU, 64-token prompts, 200 steps at temperature 0.8; every sequence is
    migrated once, at a seeded position in [40, 160], to the next rank's GPU
    (pre-copy into a region that rank owns, mapped by CUDA IPC; with one GPU
    a second region on it), then the same run without migrations: aggregate
    tok/s of both, the hand-overs' stop-the-world window, and whether every
    transcript, RNG state and KV hash is unchanged. Host-driven lockstep
    rounds of 8 tokens, so the rate is below the graph-driven headline."""
    from hotseat_b200 import serve_dist
    eng = serve_dist.GpuEngine(path, local, 64 + 200 + 8, 128)
    try:
        return serve_dist.serve_dist(eng, dist if world > 1 else serve_dist.Solo, rank, world, per=64,
                                     prompt_len=64, steps=200, seed=7, round_tokens=8)
    finally:
        eng.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="hotseat", choices=["hotseat", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batch1", action="store_true", help="skip the batch-1 items")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the 1.5B prefill/decode (c3) and kernel microbenchmark (c4) sub-objects")
    ap.add_argument("--profile-step", choices=["batch64", "batch1"],
                    help="reach the post-prompt state, run ONE decode step inside the NVTX range 'decode_step', exit")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    import hotseat_b200 as hs

    td = tempfile.mkdtemp(prefix="hsbench")
    path = os.path.join(td, "qwen05.gguf")
    make_model(path)
    try:
        if args.profile_step == "batch1":
            bench_batch1(hs, torch, dist, path, local, world, args)
            return
        b64 = bench_batch64(hs, torch, dist, path, local, world, args)
        if args.profile_step:
            return
        b1 = None if args.no_batch1 else bench_batch1(hs, torch, dist, path, local, world, args)
        extra = {}
        if world == 1 and not args.no_extra:
            extra = bench_extra(path)
        if not args.no_extra:
            c5 = bench_c5(path, rank, world, local, dist)
            if rank == 0:
                extra["c5"] = c5
        if rank == 0:
            peaks = {}
            try:
                peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
            except (OSError, ValueError):
                pass
            peak, peak_src = peaks.get("hbm_gbs"), "measured"
            if not peak:
                peak, peak_src = 6650.0, "fallback"
            step_bytes = b64_bytes_per_step()
            step_s = b64["ms_per_step"] / 1000.0 / b64["n_steps"]  # one batched decode step (one graph)
            achieved = step_bytes / step_s / 1e9
            traffic = None
            tp = os.path.join(ROOT, "profiles", "batch64_step_traffic.txt")
            if os.path.exists(tp):
                for ln in open(tp):
                    if ln.startswith("dram_bytes_per_step"):
                        traffic = float(ln.split()[1])
            cpu = None
            if not args.no_cpu_baseline:
                threads = os.cpu_count() or 1
                cv = cpu_sample(path, b64_prompts()[0], B64_CTX, 12, threads)
                cpu = {"value": cv, "unit": UNIT, "cores": threads, "kind": "port", "sample": CPU_SAMPLE}
            line = {
                "metric": METRIC, "value": b64["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": b64["ms_per_step"], "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None,
                "dtype": "f32 activations as f16 hi/lo pairs on tcgen05, f32 accumulate (f16 weights)",
                "data": "synthetic",
                "config": dict(workload_config(world), parallelism=f"independent sequences x{world} GPUs" if world > 1
                               else "1 GPU", numeric="tc", decode_steps_per_step=b64["n_steps"]),
                "roofline": {"bound": "hbm",
                             "kernel": "one batched decode step (graph of %d kernels)" % b64["launches_per_decode_step"],
                             "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                             "peak_source": peak_src, "traffic": traffic, "bytes_per_decode_step": step_bytes,
                             "frac_of_8TBps_nominal": achieved / 8000.0},
                "cpu_baseline": cpu,
                "e2e": {"value": b64["e2e_value"], "unit": UNIT, "h2d_bytes_per_step": b64["h2d"],
                        "d2h_bytes_per_step": b64["d2h"]},
                "gpu_launches": b64["gpu_launches"] + (b1["gpu_launches"] if b1 else 0),
                "clocks": b64["clocks"],
            }
            if b1:
                b1_ach = b1_bytes_per_token() * b1["value"] / world / 1e9
                line["batch1"] = {"workload": "1 sequence, prompt 36, gen 120, temp 0.8, seed 99, numeric fast",
                                  "value": b1["value"], "unit": UNIT, "ms_per_step": b1["ms_per_step"],
                                  "e2e": b1["e2e_value"],
                                  "roofline": {"achieved": b1_ach, "peak": peak, "unit": "GB/s",
                                               "frac": b1_ach / peak, "bytes_per_token": b1_bytes_per_token()}}
            line.update(extra)
            print(json.dumps(line), flush=True)
    finally:
        try:
            os.remove(path)
            os.rmdir(td)
        except OSError:
            pass
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
