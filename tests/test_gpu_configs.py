"""The benchmarked configurations themselves against the CPU restatement.

- The batch-64 decode workload exactly as bench.py times it (64 sequences of
  128-token prompts from default_rng(128+i), seeds 99+i, temperature 0.8,
  256 generated tokens, max_ctx 512, the tensor-core path): sequences decoded
  inside the full 64-sequence batch give the CPU path's transcripts, SeqState
  and RNG state, and KV rows within the token loop's 1e-2.
- The Qwen2.5-1.5B shape (28 layers, d 1536, 12/2 heads, head_dim 128, ff
  8960) on the tensor-core path: logits within 1e-2 at every position of a
  prompt and greedy tokens identical to the CPU path's.
- hs_prefill followed by one decode forward gives the logits of the CPU path
  after the whole prompt (0.5B and 1.5B shapes).
- EOS as a stop reason (seq.rs:290-293) on all three numeric paths.
"""
import numpy as np
import pytest

import hotseat_b200 as hs
from oracle import ffi
from tests.golden.synth import QWEN05, QWEN15, write_synthetic_gguf

import bench
from conftest import TINY

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2
TC = hs.NUMERIC_TC


def _seq(tokens, max_tokens, cfg, seed, **kw):
    return dict(tokens=list(tokens), prompt_len=len(tokens), max_tokens=max_tokens, cfg=cfg, rng=hs.Rng.seed(seed),
                **kw)


def test_c2_bench_workload_matches_the_oracle(fixture_dir):
    """bench.py's headline inputs, all 64 sequences decoded together; four
    of them (first, two inner, last slot) replayed on the CPU path."""
    path = str(fixture_dir / "qwen05_bench.gguf")
    bench.make_model(path)
    prompts = bench.b64_prompts()
    assert len(prompts) == 64 and all(len(p) == 128 for p in prompts)
    m = hs.Model.load(path, max_ctx=bench.B64_CTX, numeric=TC)
    kvs = [m.kv() for _ in prompts]
    cfg = hs.SamplerCfg.default(temperature=bench.TEMP, seed=bench.SEED)
    seqs = [_seq(p, bench.B64_GEN, cfg, bench.SEED + i) for i, p in enumerate(prompts)]
    got = hs.Batch(m, 64).run_seqs(kvs, seqs)
    picks = [0, 21, 42, 63]
    # one CPU model, sequences one after another on all host threads (the
    # restatement's model and pool serve one decode loop at a time)
    o = ffi.Model(path, max_ctx=bench.B64_CTX)
    want = []
    for i in picks:
        okv = o.new_kv()
        toks, st, rng = o.run_seq(okv, prompts[i], bench.B64_GEN,
                                  ffi.default_cfg(temperature=bench.TEMP, seed=bench.SEED),
                                  ffi.seeded_rng(bench.SEED + i))
        want.append((toks, st, rng, okv))
    for i, (toks, st, rng, okv) in zip(picks, want):
        g_toks, g_st, g_rng = got[i]
        assert list(g_toks) == list(toks), i
        assert (g_st.filled, g_st.done, g_st.done_reason) == (st.filled, st.done, st.done_reason), i
        assert list(g_rng.s) == list(rng.s) and g_rng.draws == rng.draws, i
        n = int(g_st.filled) * o.cfg.n_kv_heads * o.cfg.head_dim
        spec = o.cfg
        gk = kvs[i].floats().reshape(spec.n_layers, 2, spec.max_ctx, -1)[:, :, : g_st.filled]
        ok = okv.reshape(spec.n_layers, 2, spec.max_ctx, -1)[:, :, : st.filled]
        assert n > 0 and float(np.max(np.abs(gk - ok))) <= LOGIT_TOL, i


@pytest.fixture(scope="module")
def q15_oracle(q15_gguf):
    return ffi.Model(q15_gguf, max_ctx=256)


def test_qwen15_shape_logits_and_greedy_tokens(q15_gguf, q15_oracle):
    o = q15_oracle
    m = hs.Model.load(q15_gguf, max_ctx=256, numeric=TC)
    assert (m.cfg.n_layers, m.cfg.d_model, m.cfg.head_dim, m.cfg.d_ff) == (28, 1536, 128, 8960)
    b = hs.Batch(m, 1)
    kv, okv = m.kv(), o.new_kv()
    toks = [int(t) for t in np.random.default_rng(15).integers(0, QWEN15["vocab"], size=10)]
    worst = 0.0
    for pos, tok in enumerate(toks):
        b.forward([kv], [tok], [pos])
        err = float(np.max(np.abs(b.logits(0) - o.forward(okv, tok, pos))))
        worst = max(worst, err)
        assert err <= LOGIT_TOL, (pos, err)
    assert float(np.max(np.abs(kv.floats() - okv))) <= LOGIT_TOL
    cfg = hs.SamplerCfg.default(temperature=0.0)
    got = hs.Batch(m, 2).run_seqs([m.kv()], [_seq(toks, 8, cfg, 1)])[0]
    want, _, _ = o.run_seq(o.new_kv(), toks, 8, ffi.default_cfg(temperature=0.0), ffi.seeded_rng(1))
    assert list(got[0]) == list(want)
    print(f"1.5B shape: worst logit error {worst:.3g}")


@pytest.mark.parametrize("shape", ["q05", "q15"])
def test_prefill_then_one_forward_gives_the_oracle_logits(shape, q05_gguf, q15_gguf):
    path, vocab, n = {"q05": (q05_gguf, QWEN05["vocab"], 96), "q15": (q15_gguf, QWEN15["vocab"], 40)}[shape]
    prompt = [int(t) for t in np.random.default_rng(77).integers(0, vocab, size=n)]
    m = hs.Model.load(path, max_ctx=256, numeric=TC)
    kv = m.kv()
    hs.Batch(m, 128).prefill(kv, prompt[:-1])
    b = hs.Batch(m, 1)
    b.forward([kv], [prompt[-1]], [n - 1])
    o = ffi.Model(path, max_ctx=256)
    okv = o.new_kv()
    for pos, tok in enumerate(prompt):
        want = o.forward(okv, tok, pos)
    err = float(np.max(np.abs(b.logits(0) - want)))
    assert err <= LOGIT_TOL, err
    c = o.cfg
    gk = kv.floats().reshape(c.n_layers, 2, c.max_ctx, -1)[:, :, :n]
    ok = okv.reshape(c.n_layers, 2, c.max_ctx, -1)[:, :, :n]
    assert float(np.max(np.abs(gk - ok))) <= LOGIT_TOL
    print(f"{shape}: prefill of {n - 1} tokens, next-token logit error {err:.3g}")


def test_eos_stops_the_sequence_on_every_path(fixture_dir):
    """A fixture whose eos_token_id is the token greedy decoding picks at its
    fourth step (same weights: the values depend only on the seed and the
    tensor names). Every numeric path must stop there with reason "eos",
    without appending the token, exactly like the CPU path."""
    prompt = [5, 77, 300, 12, 640, 9]
    base = str(fixture_dir / "eos_base.gguf")
    write_synthetic_gguf(base, **TINY)
    o = ffi.Model(base, max_ctx=64, threads=2)
    free, _, _ = o.run_seq(o.new_kv(), prompt, 12, ffi.default_cfg(temperature=0.0), ffi.seeded_rng(1))
    eos = int(free[len(prompt) + 3])
    path = str(fixture_dir / "eos_at_4.gguf")
    write_synthetic_gguf(path, eos=eos, **TINY)
    o = ffi.Model(path, max_ctx=64, threads=2)
    want, wst, _ = o.run_seq(o.new_kv(), prompt, 12, ffi.default_cfg(temperature=0.0), ffi.seeded_rng(1))
    assert wst.done and wst.done_reason == 1 and eos not in list(want[len(prompt):])
    cfg = hs.SamplerCfg.default(temperature=0.0)
    for numeric in (hs.NUMERIC_REFERENCE, hs.NUMERIC_FAST):
        m = hs.Model.load(path, max_ctx=64, numeric=numeric)
        assert m.eos == eos
        toks, st, _ = hs.run_seq(m, m.kv(), m.scratch(), prompt, len(prompt), 12, cfg, hs.Rng.seed(1))
        assert list(toks) == list(want), numeric
        assert st.done and st.done_reason == 1 and st.filled == wst.filled, numeric
    m = hs.Model.load(path, max_ctx=64, numeric=TC)
    toks, st, _ = hs.Batch(m, 3).run_seqs([m.kv()], [_seq(prompt, 12, cfg, 1)])[0]
    assert list(toks) == list(want)
    assert st.done and st.done_reason == 1 and st.filled == wst.filled
