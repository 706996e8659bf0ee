"""The on-device sampler against Sampler::sample (sampler.rs:100-187): same
token and same RNG state for the same logits, history and configuration."""
import ctypes as C

import numpy as np
import pytest

import hotseat_b200 as hs
from tests.golden.synth import QWEN05
from oracle import ffi

from conftest import TINY

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny_scratch(tiny_gguf):
    m = hs.Model.load(tiny_gguf, max_ctx=64)
    return m, m.scratch()


@pytest.fixture(scope="module")
def big_scratch(q05_gguf):
    m = hs.Model.load(q05_gguf, max_ctx=64)
    return m, m.scratch()


def oracle_sample(cfg, rng_state, logits, hist):
    ocfg = ffi.SamplerCfg(cfg.temperature, cfg.top_p, cfg.top_k, cfg.repeat_penalty, cfg.repeat_last_n, cfg.seed)
    r = ffi.Rng()
    r.s[:] = list(rng_state.s)
    r.draws = rng_state.draws
    l = logits.copy()
    h = np.ascontiguousarray(hist, dtype=np.uint32)
    tok = ffi.lib().hso_sample(C.byref(ocfg), C.byref(r), ffi.ptr(l), l.size, ffi.ptr(h) if h.size else None, h.size)
    return tok, list(r.s), r.draws


def device_sample(scratch, cfg, rng, logits, hist):
    scratch.set_logits(logits)
    smp = hs.Sampler(cfg, hs.Rng())
    smp.rng.s[:] = list(rng.s)
    smp.rng.draws = rng.draws
    tok = smp.sample(scratch, hist)
    return tok, list(smp.rng.s), smp.rng.draws


def check(scratch, cfg, logits, hist, seed=5):
    rng = hs.Rng.seed(seed)
    got = device_sample(scratch, cfg, rng, logits, hist)
    want = oracle_sample(cfg, rng, logits, hist)
    assert got == want


def test_reference_cases_on_the_device(tiny_scratch):
    m, s = tiny_scratch
    v = TINY["vocab"]
    # greedy_sampling_ignores_the_rng (sampler.rs:235-242)
    l = np.full(v, -10.0, dtype=np.float32)
    l[:4] = [0.1, 5.0, -3.0, 4.9]
    cfg = hs.SamplerCfg.default(temperature=0.0)
    smp = hs.Sampler(cfg)
    s.set_logits(l)
    assert smp.sample(s, []) == 1 and smp.rng.draws == 0
    # top_k_one_is_greedy_even_with_temperature (244-258)
    cfg = hs.SamplerCfg.default(temperature=2.0, top_k=1, top_p=1.0, repeat_penalty=1.0)
    smp = hs.Sampler(cfg)
    for _ in range(20):
        assert smp.sample(s, []) == 1
    # repetition_penalty_pushes_logits_down (275-284)
    l2 = np.full(v, -10.0, dtype=np.float32)
    l2[:4] = [0.0, 10.0, 9.0, 0.0]
    s.set_logits(l2)
    cfg = hs.SamplerCfg.default(temperature=0.0, repeat_penalty=2.0, repeat_last_n=8)
    assert hs.Sampler(cfg).sample(s, [1]) == 2


def test_same_state_gives_the_same_token_on_the_device(tiny_scratch):
    m, s = tiny_scratch
    logits = np.array([((i * 37 % 91) / 13.0) for i in range(TINY["vocab"])], dtype=np.float32)
    cfg = hs.SamplerCfg.default(temperature=1.0, top_k=0, top_p=1.0, repeat_penalty=1.0)
    s.set_logits(logits)
    a = hs.Sampler(cfg)
    for _ in range(20):
        a.sample(s)
    b = hs.Sampler(cfg, hs.Rng())
    b.rng.s[:] = list(a.rng.s)
    b.rng.draws = a.rng.draws
    assert a.sample(s) == b.sample(s)


@pytest.mark.parametrize("trial", range(12))
def test_random_configs_match_the_oracle_tiny(tiny_scratch, trial):
    m, s = tiny_scratch
    rng = np.random.default_rng(trial)
    v = TINY["vocab"]
    logits = (rng.standard_normal(v) * rng.choice([0.3, 1.0, 4.0])).astype(np.float32)
    if trial % 3 == 0:  # exact ties: the id must break them
        logits[rng.integers(0, v, 50)] = logits.max()
    hist = rng.integers(0, v, size=int(rng.integers(0, 100))).astype(np.uint32)
    cfg = hs.SamplerCfg.default(temperature=float(rng.choice([0.0, 0.3, 0.8, 1.5])),
                                top_p=float(rng.choice([0.5, 0.9, 0.95, 1.0])),
                                top_k=int(rng.choice([0, 1, 5, 40, 64, 200])),
                                repeat_penalty=float(rng.choice([1.0, 1.1, 1.3])),
                                repeat_last_n=int(rng.choice([0, 8, 64])))
    for seed in range(3):
        check(s, cfg, logits, hist, seed)


@pytest.mark.parametrize("trial", range(8))
def test_random_configs_match_the_oracle_full_vocab(big_scratch, trial):
    m, s = big_scratch
    rng = np.random.default_rng(100 + trial)
    v = QWEN05["vocab"]
    logits = (rng.standard_normal(v) * 0.6).astype(np.float32)
    if trial % 2 == 0:
        logits[rng.integers(0, v, 200)] = np.float32(np.sort(logits)[-30])
    hist = rng.integers(0, v, size=int(rng.integers(1, 300))).astype(np.uint32)
    hist[-5:] = np.argsort(logits)[-5:]
    cfg = hs.SamplerCfg.default(temperature=float(rng.choice([0.0, 0.8, 1.2])),
                                top_k=int(rng.choice([1, 20, 40, 64])),
                                top_p=float(rng.choice([0.8, 0.95, 1.0])))
    for seed in range(3):
        check(s, cfg, logits, hist, seed)


@pytest.mark.parametrize("top_k", [0, 65, 100, 1000, 4097, 40000, 200000])
def test_any_top_k_matches_the_oracle_full_vocab(big_scratch, top_k):
    """top_k beyond the per-slice lists (sort mode): 0 (the whole
    vocabulary, sampler.rs:120-124), just past 64, across a slice boundary
    and past the vocabulary; with and without the nucleus cut, with exact
    ties at the cut, the penalty on."""
    m, s = big_scratch
    rng = np.random.default_rng(700 + top_k % 997)
    v = QWEN05["vocab"]
    for trial in range(3):
        logits = (rng.standard_normal(v) * float(rng.choice([0.3, 1.0, 3.0]))).astype(np.float32)
        if trial == 1:
            logits[rng.integers(0, v, 500)] = np.float32(np.sort(logits)[-max(2, min(top_k or v, v) // 2)])
        hist = rng.integers(0, v, size=int(rng.integers(1, 300))).astype(np.uint32)
        cfg = hs.SamplerCfg.default(temperature=float(rng.choice([0.7, 1.0, 1.5])), top_k=top_k,
                                    top_p=float([0.95, 1.0, 0.5][trial]))
        check(s, cfg, logits, hist, seed=trial)


@pytest.mark.parametrize("top_k", [0, 65, 700, 1500])
def test_any_top_k_matches_the_oracle_two_slices(tiny128_gguf, top_k):
    """A 1500-token vocabulary: two 1024-logit candidate CTAs."""
    m = hs.Model.load(tiny128_gguf, max_ctx=64)
    s = m.scratch()
    rng = np.random.default_rng(top_k)
    v = 1500
    for trial in range(4):
        logits = (rng.standard_normal(v) * 2.0).astype(np.float32)
        if trial % 2:
            logits[rng.integers(0, v, 40)] = logits.max()
        hist = rng.integers(0, v, size=20).astype(np.uint32)
        cfg = hs.SamplerCfg.default(temperature=0.9, top_k=top_k, top_p=float([0.9, 1.0][trial % 2]))
        check(s, cfg, logits, hist, seed=trial)


def test_sequences_with_large_top_k_match_the_oracle(q05_gguf):
    """Decode loops with top_k = 0 and 1000 (sort mode inside the per-token
    graph) on the bit-exact numeric path: transcripts and RNG states equal
    the CPU path's. (Over the whole vocabulary the pick depends on running
    sums of ~150k nearly equal weights, so only bit-identical logits give
    identical transcripts; the GPU-native paths are held to the sampler's
    exactness on their own logits by the tests above.)"""
    rng = np.random.default_rng(5)
    prompt = [int(t) for t in rng.integers(0, QWEN05["vocab"], size=12)]
    m = hs.Model.load(q05_gguf, max_ctx=128, numeric=hs.NUMERIC_REFERENCE)
    o = ffi.Model(q05_gguf, max_ctx=128)
    for top_k in (0, 1000):
        cfg = hs.SamplerCfg.default(temperature=0.8, top_k=top_k, seed=3)
        s = m.scratch()
        toks, st, r = hs.run_seq(m, m.kv(), s, prompt, len(prompt), 10, cfg, hs.Rng.seed(3))
        assert s.launches_per_step() == 24 * 5 + 1 + 3
        want, _, orng = o.run_seq(o.new_kv(), prompt, 10, ffi.default_cfg(temperature=0.8, top_k=top_k, seed=3),
                                  ffi.seeded_rng(3))
        assert list(toks) == list(want), top_k
        assert list(r.s) == list(orng.s) and r.draws == orng.draws


def test_batch_with_mixed_top_k(q05_gguf):
    """One tensor-core batch whose sequences sample with top_k 0, 1000 and
    40 and one greedy: the step graph runs sort mode for all of them. Every
    sequence equals itself decoded alone (tokens, RNG), and the top_k 40 and
    greedy ones equal the CPU path's transcripts."""
    rng = np.random.default_rng(8)
    v = QWEN05["vocab"]
    m = hs.Model.load(q05_gguf, max_ctx=128, numeric=hs.NUMERIC_TC)
    o = ffi.Model(q05_gguf, max_ctx=128)
    cases = [(0, 0.8), (1000, 1.0), (40, 0.8), (40, 0.0)]
    prompts = [[int(t) for t in rng.integers(0, v, size=10 + 3 * i)] for i in range(len(cases))]

    def seqs():
        return [dict(tokens=p, prompt_len=len(p), max_tokens=8, rng=hs.Rng.seed(20 + i),
                     cfg=hs.SamplerCfg.default(temperature=t, top_k=k, seed=20 + i))
                for i, (p, (k, t)) in enumerate(zip(prompts, cases))]

    b = hs.Batch(m, len(cases))
    got = b.run_seqs([m.kv() for _ in cases], seqs())
    assert b.launches_per_step() == 24 * 7 + 2 + 3
    for i, q in enumerate(seqs()):
        alone = hs.Batch(m, 1).run_seqs([m.kv()], [q])[0]
        assert list(got[i][0]) == list(alone[0]) and list(got[i][2].s) == list(alone[2].s), i
    for i in (2, 3):
        k, t = cases[i]
        want, _, orng = o.run_seq(o.new_kv(), prompts[i], 8, ffi.default_cfg(temperature=t, top_k=k, seed=20 + i),
                                  ffi.seeded_rng(20 + i))
        assert list(got[i][0]) == list(want), i
        assert list(got[i][2].s) == list(orng.s) and got[i][2].draws == orng.draws, i
