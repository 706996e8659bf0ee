"""Decode throughput of the hotseat token loop on B200.

Workload (the batch-1 configuration the metric is quoted on): the seeded
random-init Qwen2.5-0.5B-shape GGUF (24 layers, d 896, 14/2 heads, ff 4864,
vocab 151936, Q6_K embedding, Q4_K weights, f32 norms/biases), a 36-token
uniform-random prompt, temperature 0.8, seed 99, 120 generated tokens, f32 KV.

One step = the 120-token decode phase of that sequence (forward + device
sampling + seq.rs commit per token) from its post-prefill state, which is
restored before each step. `value` is decode tok/s with the state already in
HBM; `e2e` is the same through hs_seq_run with host token buffers.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Under torchrun each rank runs its own sequence on its own GPU (independent
sequences shard with no collective); value = all ranks' tokens / max time.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s per GPU, Qwen2.5-0.5B-shape, batch 1/64; % of HBM roofline"
UNIT = "tok/s"
PROMPT_LEN, GEN, SEED, TEMP, MAX_CTX = 36, 120, 99, 0.8, 2048
MODEL_SEED = 1234
CTL_BYTES = 160  # sizeof(DevCtl), the device control block hs_seq_* copies each way


def workload_config():
    return {"workload": "qwen2.5-0.5b-shape decode, batch 1, prompt 36, gen 120, temp 0.8, seed 99, f32 KV",
            "model_shape": "24L d896 14/2h hd64 ff4864 vocab151936 Q6_K-embd Q4_K-weights",
            "max_ctx": MAX_CTX, "l2": "weights 0.99 GB stream per token > 126 MB L2 (no flush needed)"}


def bytes_per_token_avg():
    """Algorithmic HBM bytes per decode token, averaged over positions 36..155:
    f16 weights + f32 norms/biases + KV read (pos+1 rows) + KV write."""
    d, ff, nh, nkv, hd, L, V = 896, 4864, 14, 2, 64, 24, 151936
    w = L * 2 * ((nh + 2 * nkv) * hd * d + d * nh * hd + 3 * ff * d) + V * d * 2
    small = L * 4 * (2 * d + (nh + 2 * nkv) * hd) + d * 4
    kv_row = L * 2 * nkv * hd * 4
    kv = np.mean([(p + 1) * kv_row + kv_row for p in range(PROMPT_LEN, PROMPT_LEN + GEN)])
    return w + small + kv


def make_model(path):
    import hotseat_b200 as hs
    hs.write_synthetic_gguf(path, seed=MODEL_SEED, **hs.QWEN05)


def prompt_tokens():
    rng = np.random.default_rng(36)
    return [int(t) for t in rng.integers(0, 151936, size=PROMPT_LEN)]


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


def cpu_baseline(path, n_decode, threads):
    """The CPU restatement of the reference path (oracle/, test infrastructure
    used here only as the baseline): prefill untimed, `n_decode` tokens timed."""
    from oracle import ffi
    o = ffi.Model(path, max_ctx=MAX_CTX, threads=threads)
    kv = o.new_kv()
    cfg = ffi.default_cfg(temperature=TEMP, seed=SEED)
    rng = ffi.seeded_rng(SEED)
    prompt = prompt_tokens()
    toks, st, rng = o.run_seq(kv, prompt, GEN, cfg, rng, stop_at_filled=PROMPT_LEN)
    t0 = time.perf_counter()
    toks, st, rng = o.run_seq(kv, toks, GEN, cfg, rng, state=st, stop_at_filled=PROMPT_LEN + n_decode)
    dt = time.perf_counter() - t0
    return n_decode / dt, toks


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU algorithm (its C++ restatement;
    rustc is not available to build the Rust original) on the host cores."""
    if rank != 0:
        return
    from oracle import ffi
    ffi.build()
    threads = os.cpu_count() or 1
    sample = 12
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "qwen05.gguf")
        make_model(path)
        vals = []
        for i in range(args.warmup + args.steps):
            v, _ = cpu_baseline(path, sample, threads)
            if i >= args.warmup:
                vals.append(v)
    value = float(np.mean(vals))
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * sample / value,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (f16 weights)",
            "data": "synthetic", "config": workload_config(),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{sample} decode tokens per step after an untimed 36-token prefill"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="hotseat", choices=["hotseat", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--numeric", default="fast", choices=["fast", "reference"],
                    help="fast: GPU-native reduction order (logits within 1e-2 of the CPU path); "
                         "reference: bit-identical to the CPU reference")
    ap.add_argument("--profile-step", action="store_true",
                    help="prefill, then run one decode token inside the NVTX range 'decode_step' and exit")
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
    numeric = hs.NUMERIC_FAST if args.numeric == "fast" else hs.NUMERIC_REFERENCE
    m = hs.Model.load(path, max_ctx=MAX_CTX, device=local, numeric=numeric)
    kv, s = m.kv(), m.scratch()
    cfg = hs.SamplerCfg.default(temperature=TEMP, seed=SEED)
    prompt = prompt_tokens()
    # Prefill (untimed): the post-prefill state is every step's starting point.
    toks, st, rng = hs.run_seq(m, kv, s, prompt, PROMPT_LEN, GEN, cfg, hs.Rng.seed(SEED), stop_at_filled=PROMPT_LEN)
    snap_toks, snap_rng = np.array(toks, dtype=np.uint32), hs.Rng()
    snap_rng.s[:] = list(rng.s)
    snap_rng.draws = rng.draws
    snap_state = (st.prompt_len, st.filled, st.max_tokens)
    stream = torch.cuda.ExternalStream(s.stream)
    lib = hs.lib()
    import ctypes as C

    def begin():
        r = hs.Rng()
        r.s[:] = list(snap_rng.s)
        r.draws = snap_rng.draws
        sst = hs.SeqState(*snap_state, 0, 0)
        hs._check(lib.hs_seq_begin(s._h, kv._h, hs._ptr(snap_toks), len(snap_toks), MAX_CTX + 1, C.byref(sst),
                                   C.byref(cfg), C.byref(r), 0))

    def end_check():
        out = np.zeros(MAX_CTX + 1, dtype=np.uint32)
        n = C.c_uint64()
        sst, r = hs.SeqState(), hs.Rng()
        hs._check(lib.hs_seq_end(s._h, hs._ptr(out), C.byref(n), out.size, C.byref(sst), C.byref(r)))
        return out[: n.value], sst

    n_steps = PROMPT_LEN + GEN - snap_state[1]  # forwards in the decode phase
    if args.profile_step:
        for _ in range(3):
            begin()
            hs._check(lib.hs_seq_step(s._h, 1))
            end_check()
        begin()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("decode_step")
        hs._check(lib.hs_seq_step(s._h, 1))
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        end_check()
        print(json.dumps({"profile_step": "done", "launches": s.launches_per_step()}))
        return
    for _ in range(args.warmup):
        begin()
        hs._check(lib.hs_seq_step(s._h, n_steps))
        ref_toks, ref_st = end_check()
    assert len(ref_toks) == PROMPT_LEN + GEN and ref_st.done_reason == 2

    # ---- device-resident timing
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms = []
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            begin()
            evs[i][0].record(stream)
            hs._check(lib.hs_seq_step(s._h, n_steps))
            evs[i][1].record(stream)
        torch.cuda.synchronize()
    ms = [a.elapsed_time(b) for a, b in evs]
    final_toks, _ = end_check()
    assert list(final_toks) == list(ref_toks), "decode is not deterministic across steps"
    total_ms = float(sum(ms))
    if world > 1:
        t = torch.tensor([total_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
        dist.barrier()
    ms_per_step = total_ms / args.steps
    tokens_per_step = GEN
    value = world * tokens_per_step * args.steps / (total_ms / 1000.0)

    # ---- end to end through the C ABI with host buffers
    e2e_ms = []
    for i in range(args.steps):
        r = hs.Rng()
        r.s[:] = list(snap_rng.s)
        r.draws = snap_rng.draws
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        out_toks, out_st, _ = hs.run_seq(m, kv, s, snap_toks, snap_state[0], snap_state[2], cfg, r,
                                         filled=snap_state[1])
        b.record(stream)
        b.synchronize()
        e2e_ms.append(a.elapsed_time(b))
        assert list(out_toks) == list(ref_toks)
    e2e_total = float(sum(e2e_ms))
    if world > 1:
        t = torch.tensor([e2e_total], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_total = float(t.item())
    e2e_value = world * tokens_per_step * args.steps / (e2e_total / 1000.0)

    if rank == 0:
        peaks = {}
        try:
            peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        except (OSError, ValueError):
            pass
        peak = peaks.get("hbm_gbs")
        peak_src = "measured"
        if not peak:
            peak, peak_src = 6650.0, "fallback"
        bpt = bytes_per_token_avg()
        achieved = bpt * (tokens_per_step / (ms_per_step / 1000.0)) / 1e9
        traffic = None
        tp = os.path.join(ROOT, "profiles", "decode_step_traffic.txt")
        if os.path.exists(tp):
            try:
                for ln in open(tp):
                    if ln.startswith("dram_bytes_per_token"):
                        traffic = float(ln.split()[1])
            except (OSError, ValueError, IndexError):
                traffic = None
        cpu = None
        if not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            cv, _ = cpu_baseline(path, 24, threads)
            cpu = {"value": cv, "unit": UNIT, "cores": threads, "kind": "port",
                   "sample": "24 decode tokens of the same sequence after an untimed 36-token prefill"}
        launches = s.launches_per_step() * n_steps * args.steps
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32 (f16 weights)", "data": "synthetic",
            "config": dict(workload_config(), parallelism=f"replicas x{world}" if world > 1 else "1 GPU",
                           numeric=args.numeric),
            "roofline": {"bound": "hbm", "kernel": "decode step (k_gemv x121, k_attention x24, sampler x2)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": peak_src, "traffic": traffic,
                         "bytes_per_token": bpt, "frac_of_8TBps_nominal": achieved / 8000.0},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": len(snap_toks) * 4 + CTL_BYTES,
                    "d2h_bytes_per_step": (PROMPT_LEN + GEN) * 4 + 2 * CTL_BYTES},
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    for o in (s, kv):
        o.close()
    m.close()
    try:
        os.remove(path)
        os.rmdir(td)
    except OSError:
        pass
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
