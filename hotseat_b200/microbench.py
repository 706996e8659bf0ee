"""Kernel microbenchmarks of the token loop's building blocks (B200).

    python -m hotseat_b200.microbench dequant     # Q4_K/Q6_K -> f16 load-time dequantisation
    python -m hotseat_b200.microbench attention   # GQA decode attention at 1k-32k context
    python -m hotseat_b200.microbench prefill     # 1.5B shape: 16 x 2048-token prefill, 512 greedy steps
    python -m hotseat_b200.microbench token       # batch-1 persistent token kernel: phase timeline
    python -m hotseat_b200.microbench batch       # batch-64 tensor-core step: per-kernel timeline

dequant: the tensors of the seeded Qwen2.5-0.5B-shape GGUF (ffn_gate 4864x896
and ffn_down 896x4864 in Q4_K, token_embd 151936x896 in Q6_K) plus the same
embedding written in Q4_K, dequantised by hs_dequant_f16 from device memory;
L2 is flushed (256 MB written) between timed launches. Bytes = quantised
blocks read + 2 bytes per element written.

attention: one forward of the 0.5B-shape model at position P (KV regions as
allocated, so every cached row is read), batch 1 on the GPU-native path (its
per-kernel form, HS_TOKEN_KERNEL=0, so that attention is a launch of its
own) and batch 64 on the tensor-core path, with the launch timeline
(HS_TRACE=1). The
attention time of a layer is its kernel's exit minus the QKV kernel's exit
(the work it adds after its input is ready), averaged over the 24 layers.
Bytes = (P+1) x 1024 B of K and V read + 1024 B written per sequence and
layer (14 query / 2 KV heads, head_dim 64, f32).

prefill: the seeded Qwen2.5-1.5B-shape GGUF (28 layers, d 1536, 12/2 heads,
head_dim 128, ff 8960, vocab 151936), 16 sequences with 2048-token
uniform-random prompts, each prefilled by hs_prefill (2047 tokens as GEMM rows,
up to 512 per pass), then the 16 decoded together for 512 greedy tokens
(temperature 0, penalty 1.1). FLOPs = 2 x (non-embedding weights) per token
for the GEMMs (the tensor cores execute twice that: f16 hi and lo halves).

token: one sequence of the 0.5B shape (36-token prompt, sampled at temperature 0.8, seed
99) decoded to 60 and to 120 tokens by the persistent token kernel with the
trace on; the kernel's timeline of its last step, from CTA 0 (per phase of
layers 1-23, averaged: input wait and its parts, rows, tiles) and over all
CTAs (phase-end spread), plus the LM head and the sampler.

batch: 64 sequences of the 0.5B shape (128-token prompts, 140 tokens at
temperature 0.8) decoded together on the tensor-core path with the trace
on; the last step's launch timeline: per kernel role of layers 1-22, the
time from the previous kernel's last exit to its own last exit, and for the
four GEMMs their trace marks (latest CTA): dependency wait released, first
stage landed, MMAs issued, accumulator ready, epilogue done, exit.

Each line printed is one JSON object; peaks are the measured copy bandwidth
in MEASURED_PEAKS.json when present.
"""
import json
import os
import struct
import sys
import tempfile

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from tests.golden.synth import QWEN05, QWEN15, write_synthetic_gguf  # noqa: E402  (fixture writer)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _peak():
    try:
        return float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError):
        return 6650.0, "fallback"


def gguf_tensors(path):
    """name -> (ggml type, element count, absolute byte offset) of a GGUF v3 file."""
    with open(path, "rb") as f:
        data = f.read(1 << 26)
    off = 0

    def take(fmt):
        nonlocal off
        v = struct.unpack_from("<" + fmt, data, off)
        off += struct.calcsize("<" + fmt)
        return v[0] if len(v) == 1 else v

    def string():
        nonlocal off
        n = take("Q")
        s = data[off: off + n].decode()
        off += n
        return s

    sizes = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}

    def skip_value(t):
        nonlocal off
        if t == 8:
            string()
        elif t == 9:
            et, n = take("I"), take("Q")
            for _ in range(n):
                skip_value(et)
        else:
            off += sizes[t]

    assert data[:4] == b"GGUF"
    off = 4
    take("I")
    n_t, n_kv = take("Q"), take("Q")
    align = 32
    for _ in range(n_kv):
        key = string()
        t = take("I")
        if key == "general.alignment" and t == 4:
            align = take("I")
        else:
            skip_value(t)
    infos = []
    for _ in range(n_t):
        name = string()
        nd = take("I")
        n = 1
        for _ in range(nd):
            n *= take("Q")
        infos.append((name, take("I"), n, take("Q")))
    base = (off + align - 1) // align * align
    return {name: (t, n, base + o) for name, t, n, o in infos}


def block_bytes(t):
    return {12: 144, 14: 210, 13: 176, 8: 34, 6: 22}[t]


def bench_dequant(reps=10, q05_path=None):
    """Returns one record per tensor; q05_path: an existing 0.5B-shape file
    (seed 1234) to read the Q4_K/Q6_K tensors from."""
    import torch
    import hotseat_b200 as hs
    peak, src = _peak()
    td = tempfile.mkdtemp(prefix="hsmicro")
    a = q05_path or os.path.join(td, "q6.gguf")
    b = os.path.join(td, "q4.gguf")
    if not q05_path:
        write_synthetic_gguf(a, seed=1234, **QWEN05)
    write_synthetic_gguf(b, seed=1234, embd_type=12, **dict(QWEN05, n_layers=1))
    out = []
    cases = [(a, "blk.0.ffn_gate.weight", "4864x896"), (a, "blk.0.ffn_down.weight", "896x4864"),
             (b, "token_embd.weight", "151936x896"), (a, "token_embd.weight", "151936x896")]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    for path, name, shape in cases:
        t, n, at = gguf_tensors(path)[name]
        nbytes = n // 256 * block_bytes(t)
        with open(path, "rb") as f:
            f.seek(at)
            raw = np.frombuffer(f.read(nbytes), dtype=np.uint8)
        src_d = torch.from_numpy(raw.copy()).cuda()
        dst = torch.empty(n, dtype=torch.float16, device="cuda")
        ms = []
        for i in range(3 + reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            hs.dequant_f16(t, src_d.data_ptr(), n, dst.data_ptr(), stream.cuda_stream)
            e1.record(stream)
            e1.synchronize()
            if i >= 3:
                ms.append(e0.elapsed_time(e1))
        us = 1000.0 * float(np.median(ms))
        moved = nbytes + 2 * n
        gbs = moved / us / 1e3
        out.append({"bench": "dequant", "type": {12: "Q4_K", 14: "Q6_K"}[t], "shape": shape,
                    "bytes": moved, "us": us, "GB/s": gbs, "frac": gbs / peak, "peak": peak,
                    "peak_source": src, "l2": "flushed between launches"})
    for p in ((b,) if q05_path else (a, b)):
        os.remove(p)
    os.rmdir(td)
    return out


def _att_times(trace, per_layer, att_slot, layers):
    t = trace.astype(np.int64)
    out = []
    for l in range(layers):
        s = l * per_layer + att_slot
        out.append((t[s, 2] - t[s - 1, 2]) / 1000.0)
    return float(np.mean(out))


def bench_attention(ctxs=(1024, 4096, 16384, 32767), q05_path=None):
    """Returns one record per (batch, context); tracing is on only for the
    models this function creates."""
    old_trace = os.environ.get("HS_TRACE")
    os.environ["HS_TRACE"] = "1"
    import hotseat_b200 as hs
    peak, src = _peak()
    td = tempfile.mkdtemp(prefix="hsmicro")
    path = q05_path or os.path.join(td, "q05.gguf")
    if not q05_path:
        write_synthetic_gguf(path, seed=1234, **QWEN05)
    recs = []
    max_ctx = max(ctxs) + 8
    layers, row = 24, 2 * 2 * 64 * 4
    for batch, numeric in ((1, hs.NUMERIC_FAST), (64, hs.NUMERIC_TC)):
        os.environ["HS_TOKEN_KERNEL"] = "0"
        m = hs.Model.load(path, max_ctx=max_ctx, numeric=numeric)
        del os.environ["HS_TOKEN_KERNEL"]
        kvs = [m.kv() for _ in range(batch)]
        if batch == 1:
            s = m.scratch()
        else:
            bt = hs.Batch(m, batch)
        for p in ctxs:
            res = []
            for _ in range(3):
                if batch == 1:
                    m.forward(kvs[0], 17, p, s)
                    res.append(_att_times(s.trace(), 5, 1, layers))
                else:
                    bt.forward(kvs, list(range(17, 17 + batch)), [p] * batch)
                    res.append(_att_times(bt.trace(), 7, 2, layers))
            us = float(np.median(res[1:]))
            moved = batch * ((p + 1) * row + row)
            gbs = moved / us / 1e3
            recs.append({"bench": "attention", "batch": batch, "context": p + 1,
                         "numeric": "fast" if batch == 1 else "tc", "bytes_per_layer": moved,
                         "us_per_layer": us, "GB/s": gbs, "frac": gbs / peak, "peak": peak,
                         "peak_source": src})
        for k in kvs:
            k.close()
        if batch == 1:
            s.close()
        else:
            bt.close()
        m.close()
    if not q05_path:
        os.remove(path)
    os.rmdir(td)
    if old_trace is None:
        del os.environ["HS_TRACE"]
    else:
        os.environ["HS_TRACE"] = old_trace
    return recs


def bench_prefill(n_seqs=16, prompt=2048, gen=512, pass_tokens=2048):
    import torch
    import hotseat_b200 as hs
    peak_bw, _ = _peak()
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        tflops, tsrc = float(peaks["bf16_tflops"]), "measured"
    except (OSError, ValueError, KeyError):
        tflops, tsrc = 1590.0, "fallback"
    td = tempfile.mkdtemp(prefix="hsmicro")
    path = os.path.join(td, "q15.gguf")
    write_synthetic_gguf(path, seed=1234, **QWEN15)
    c = QWEN15
    hd = c["d_model"] // c["n_heads"]
    qrows = (c["n_heads"] + 2 * c["n_kv_heads"]) * hd
    layer_w = c["d_model"] * qrows + c["d_model"] * c["d_model"] + 3 * c["d_model"] * c["d_ff"]
    m = hs.Model.load(path, max_ctx=prompt + gen + 8, numeric=hs.NUMERIC_TC)
    kvs = [m.kv() for _ in range(n_seqs)]
    prompts = [[int(t) for t in np.random.default_rng(2048 + i).integers(0, c["vocab"], size=prompt)]
               for i in range(n_seqs)]
    pb = hs.Batch(m, pass_tokens)
    stream = torch.cuda.ExternalStream(pb.stream)
    pb.prefill(kvs[0], prompts[0][:pass_tokens])  # warm-up (graphs)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for kv, p in zip(kvs, prompts):
        pb.prefill(kv, p[:-1])
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    toks = n_seqs * (prompt - 1)
    flops = 2.0 * c["n_layers"] * layer_w * toks
    tf = flops / (ms / 1000.0) / 1e12
    recs = [{"bench": "prefill", "model": "qwen2.5-1.5b-shape", "sequences": n_seqs, "prompt": prompt,
             "pass_tokens": pass_tokens, "ms": ms, "tok/s": toks / (ms / 1000.0), "gemm_TFLOP/s": tf,
             "peak_TFLOP/s": tflops,
             "frac": tf / tflops, "peak_source": tsrc,
             "note": "algorithmic 2*weights*tokens; the tensor cores run twice that (hi/lo halves)"}]
    cfg = hs.SamplerCfg.default(temperature=0.0)
    db = hs.Batch(m, n_seqs)
    seqs = [dict(tokens=p, prompt_len=prompt, max_tokens=gen, cfg=cfg, rng=hs.Rng.seed(i), filled=prompt - 1)
            for i, p in enumerate(prompts)]
    dstream = torch.cuda.ExternalStream(db.stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(dstream)
    out = db.run_seqs(kvs, seqs)
    e1.record(dstream)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    gen_toks = sum(len(t) - prompt for t, _, _ in out)
    step_bytes = c["n_layers"] * layer_w * 2 + c["vocab"] * c["d_model"] * 2
    steps = max(len(t) - prompt for t, _, _ in out) + 1
    kv_row = c["n_layers"] * 2 * c["n_kv_heads"] * hd * 4
    kv_bytes = n_seqs * kv_row * np.mean([p + 1 for p in range(prompt - 1, prompt + gen - 1)])
    gbs = (step_bytes + kv_bytes) * steps / (ms / 1000.0) / 1e9
    recs.append({"bench": "decode", "model": "qwen2.5-1.5b-shape", "batch": n_seqs, "context_from": prompt,
                 "generated": gen_toks, "ms": ms, "tok/s": gen_toks / (ms / 1000.0), "GB/s": gbs,
                 "frac": gbs / peak_bw, "note": "hs_batch_seq_run end to end, greedy, penalty 1.1"})
    for k in kvs:
        k.close()
    pb.close()
    db.close()
    m.close()
    os.remove(path)
    os.rmdir(td)
    return recs


def bench_token():
    os.environ["HS_TRACE"] = "1"
    import hotseat_b200 as hs
    td = tempfile.mkdtemp(prefix="hsmicro")
    path = os.path.join(td, "q05.gguf")
    write_synthetic_gguf(path, seed=1234, **QWEN05)
    m = hs.Model.load(path, max_ctx=256, numeric=hs.NUMERIC_FAST)
    s = m.scratch()
    if s.launches_per_step() != 3:
        raise RuntimeError("the persistent token kernel is not in use for this model")
    rng = np.random.default_rng(36)
    prompt = [int(t) for t in rng.integers(0, QWEN05["vocab"], size=36)]
    cfg = hs.SamplerCfg.default(temperature=0.8, seed=99)
    L, ghz = 24, 1.965
    for ntok in (60, 120):
        kv = m.kv()
        hs.run_seq(m, kv, s, prompt, 36, ntok, cfg, hs.Rng.seed(99))
        kv.close()
        t = s.trace()
        k = t[0].astype(np.int64)
        # timeline words after the 3 launch slots: 20 per barrier interval
        flat = t[3:].reshape(-1)[: 20 * (5 * L + 1)].reshape(5 * L + 1, 20)
        body = flat[: 5 * L].astype(np.int64).reshape(L, 5, 20)
        # per interval: CTA 0's input ready (0), rows done (1), outputs written
        # (2); over CTAs the earliest (~8) and latest (9) outputs written
        seq_end = np.concatenate([[k[0]], body.reshape(-1, 20)[:-1, 2]]).reshape(L, 5)
        latest_prev = np.concatenate([[k[0]], flat[: 5 * L - 1, 9].astype(np.int64)]).reshape(L, 5)
        earliest = (~flat[: 5 * L, 8]).astype(np.int64).reshape(L, 5)
        latest = flat[: 5 * L, 9].astype(np.int64).reshape(L, 5)
        sl = slice(1, L)
        phases = {}
        for i, name in enumerate(["qkv", "attention", "o", "gate_up", "down"]):
            phases[name] = {
                "input_us": float(((body[sl, i, 0] - seq_end[sl, i]) / 1e3).mean()),
                "detect_us": float(((body[sl, i, 0] - latest_prev[sl, i]) / 1e3).mean()),
                "rows_us": float(((body[sl, i, 1] - body[sl, i, 0]) / 1e3).mean()),
                "tiles": float(body[sl, i, 5].mean()),
                "tile_wait_us": float((body[sl, i, 4] / ghz / 1e3).mean()),
                "tile_compute_us": float((body[sl, i, 6] / ghz / 1e3).mean()),
                "end_spread_us": float(((latest[sl, i] - earliest[sl, i]) / 1e3).mean()),
                # input staged (word 10) and transformed (word 11: RMSNorm, or the
                # split combine) after the latest previous-phase end (not attention)
                "staged_us": float(((body[sl, i, 10] - latest_prev[sl, i]) / 1e3).mean()) if i != 1 else 0.0,
                "transformed_us": float(((body[sl, i, 11] - body[sl, i, 10]) / 1e3).mean()) if i != 1 else 0.0,
            }
        # one CTA's first attention item: SM clock at each checkpoint
        # (the last writer's), cumulative from the item's start
        probe = body[sl, 1, 12:20].astype(np.int64)
        item = {name: float(((probe[:, i] - probe[:, 0]) / ghz / 1e3).mean())
                for i, name in enumerate(["start", "qkv_gathered", "rope_done", "chunk0_ready", "scores_done",
                                          "softmax_done", "loop_done"]) if i > 0}
        h = flat[5 * L].astype(np.int64)
        print(json.dumps({"bench": "token_kernel", "prompt": 36, "max_tokens": ntok, "kernel_us": float((k[2] - k[0]) / 1e3),
                          "per_layer": phases, "attention_item_us": item, "lm_head_us": float((h[1] - h[0]) / 1e3),
                          "lm_head_tiles": int(h[5]),
                          "sampler_us": [float((int(t[i][2]) - int(t[i][0])) / 1e3) for i in (1, 2)],
                          # token kernel's end to: candidates' first CTA start, their last exit,
                          # the final kernel's wait released, its exit
                          "sampler_path_us": [float((int(x) - int(k[2])) / 1e3)
                                              for x in (t[1][0], t[1][2], t[2][1], t[2][2])],
                          # the final kernel after its wait: candidate lists loaded, merged,
                          # token picked, exit (%globaltimer marks, last CTA)
                          "sampler_final_us": [float((int(t[2][j]) - int(t[2][1])) / 1e3) for j in (4, 5, 6, 2)]}),
              flush=True)
    s.close()
    m.close()
    os.remove(path)
    os.rmdir(td)


def bench_batch(shape="q05"):
    """The last decode step's launch timeline: q05 = 64 sequences of the 0.5B
    shape (128-token prompts, 140 tokens); q15 = 16 sequences of the 1.5B
    shape decoding after a 2,047-token prefill (16 tokens)."""
    os.environ["HS_TRACE"] = "1"
    import hotseat_b200 as hs
    td = tempfile.mkdtemp(prefix="hsmicro")
    c = QWEN05 if shape == "q05" else QWEN15
    path = os.path.join(td, shape + ".gguf")
    write_synthetic_gguf(path, seed=1234, **c)
    B, prompt, gen, max_ctx = (64, 128, 140, 512) if shape == "q05" else (16, 2048, 16, 2568)
    m = hs.Model.load(path, max_ctx=max_ctx, numeric=hs.NUMERIC_TC)
    b = hs.Batch(m, B)
    kvs = [m.kv() for _ in range(B)]
    seqs = []
    pb = hs.Batch(m, prompt) if shape != "q05" else None
    for i in range(B):
        g = np.random.default_rng(99 + i)
        p = [int(t) for t in g.integers(0, c["vocab"], size=prompt)]
        filled = 0
        if pb is not None:
            pb.prefill(kvs[i], p[:-1])
            filled = prompt - 1
        seqs.append(dict(tokens=p, prompt_len=prompt, max_tokens=gen, filled=filled, rng=hs.Rng.seed(99 + i),
                         cfg=hs.SamplerCfg.default(temperature=0.8, seed=99 + i)))
    if pb is not None:
        pb.close()
    b.run_seqs(kvs, seqs)
    n = b.launches_per_step()
    t = b.trace().astype(np.int64)[:n]
    L = c["n_layers"]
    names = ["norm", "qkv", "attention", "o", "ffn_norm", "gate_up", "down"]
    per = {}
    for j, k in enumerate(names):
        per[k] = float(np.mean([(t[l * 7 + j, 2] - t[l * 7 + j - 1, 2]) / 1e3 for l in range(1, L - 1)]))
    gemm = {}
    for j, k in [(1, "qkv"), (3, "o"), (5, "gate_up"), (6, "down")]:
        rows = [t[l * 7 + j] for l in range(1, L - 1)]
        prev = [t[l * 7 + j - 1, 2] for l in range(1, L - 1)]
        gemm[k] = {
            "wait_released": float(np.mean([r[1] - p for r, p in zip(rows, prev)]) / 1e3),
            "first_stage": float(np.mean([r[4] - r[1] for r in rows]) / 1e3),
            "mmas_issued": float(np.mean([r[5] - r[4] for r in rows]) / 1e3),
            "accumulator_ready": float(np.mean([r[6] - r[5] for r in rows]) / 1e3),
            "epilogue_done": float(np.mean([r[7] - r[6] for r in rows]) / 1e3),
            "exit": float(np.mean([r[2] - r[7] for r in rows]) / 1e3),
        }
    # attention item checkpoints (SM cycles from the item's start, maximum over
    # CTAs): RoPE done, first chunk (or warp 0's first block) ready, the
    # positions done, the item's end
    att = [t[l * 7 + 2] for l in range(1, L - 1)]
    item = {k: float(np.mean([r[4 + i] for r in att]) / 1965.0) for i, k in
            enumerate(["rope_done", "first_ready", "positions_done", "end"])}
    print(json.dumps({"bench": "batch_step", "model": shape, "sequences": B, "launches": int(n),
                      "exit_to_exit_us": per, "layer_us": sum(per.values()), "gemm_marks_us": gemm,
                      "attention_item_us": item}), flush=True)
    for kv in kvs:
        kv.close()
    b.close()
    m.close()
    os.remove(path)
    os.rmdir(td)


def bench_prefill_trace(prompt=2048, pass_tokens=1024):
    """One prefill pass of the 1.5B shape at the end of a 2048-token prompt
    (positions prompt-1-pass_tokens .. prompt-2) with the launch timeline:
    per kernel role of layers 1-26, previous kernel's last exit to its own."""
    os.environ["HS_TRACE"] = "1"
    import hotseat_b200 as hs
    td = tempfile.mkdtemp(prefix="hsmicro")
    path = os.path.join(td, "q15.gguf")
    write_synthetic_gguf(path, seed=1234, **QWEN15)
    c = QWEN15
    m = hs.Model.load(path, max_ctx=prompt + 8, numeric=hs.NUMERIC_TC)
    kv = m.kv()
    toks = [int(t) for t in np.random.default_rng(2048).integers(0, c["vocab"], size=prompt)]
    b = hs.Batch(m, pass_tokens)
    head = prompt - 1 - pass_tokens
    b.prefill(kv, toks[:head])
    b.prefill(kv, toks[head:prompt - 1], pos0=head)
    t = b.trace().astype(np.int64)
    L = c["n_layers"]
    names = ["norm", "qkv", "append", "attend", "o", "ffn_norm", "gate_up", "down"]
    if os.environ.get("HS_PREFILL_ATTN", "1") != "0":  # query-block attend, then the segments' merge
        names.insert(4, "combine")
    P = len(names)
    per = {}
    for j, k in enumerate(names):
        per[k] = float(np.mean([(t[l * P + j, 2] - t[l * P + j - 1, 2]) / 1e3 for l in range(1, L - 1)]))
    print(json.dumps({"bench": "prefill_pass", "model": "qwen2.5-1.5b-shape", "positions": [head, prompt - 2],
                      "exit_to_exit_us": per, "layer_us": sum(per.values()),
                      "pass_ms": float((t[L * P - 1, 2] - t[0, 0]) / 1e6)}), flush=True)
    kv.close()
    b.close()
    m.close()
    os.remove(path)
    os.rmdir(td)


if __name__ == "__main__":
    which = sys.argv[1] if len(sys.argv) > 1 else "all"
    if which in ("dequant", "all"):
        for r in bench_dequant():
            print(json.dumps(r), flush=True)
    if which in ("attention", "all"):
        for r in bench_attention():
            print(json.dumps(r), flush=True)
    if which in ("prefill", "all"):
        for r in bench_prefill(pass_tokens=int(sys.argv[2]) if which == "prefill" and len(sys.argv) > 2 else 2048):
            print(json.dumps(r), flush=True)
    if which in ("token", "all"):
        bench_token()
    if which in ("batch", "all"):
        bench_batch()
    if which == "batch15":
        bench_batch("q15")
    if which == "prefill_trace":
        bench_prefill_trace(pass_tokens=int(sys.argv[2]) if len(sys.argv) > 2 else 1024)
