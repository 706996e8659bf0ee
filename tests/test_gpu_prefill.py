"""Prompt prefill on the tensor-core path (hs_prefill): the prompt's tokens as
the rows of every GEMM, K/V appended for all of them before any attends.

Prefill GEMMs use wide weight tiles and no K split (the prompt's tokens
give the parallelism), so their sums are ordered differently from the decode
steps': the KV rows match token-by-token decoding within the path's
tolerance, greedy continuations are identical, prefill in pieces is
bit-identical to one call, and the greedy tokens match the CPU path."""
import numpy as np
import pytest

import hotseat_b200 as hs
from tests.golden.synth import QWEN05
from oracle import ffi

from conftest import TINY

pytestmark = pytest.mark.gpu

TC = hs.NUMERIC_TC


def state(tokens, prompt_len, max_tokens, cfg, seed, filled=0):
    return dict(tokens=list(tokens), prompt_len=prompt_len, max_tokens=max_tokens, cfg=cfg, rng=hs.Rng.seed(seed),
                filled=filled)


@pytest.mark.parametrize("cap", [1, 64, 128])
def test_prefill_then_decode_matches_token_by_token(tiny_gguf, cap):
    m = hs.Model.load(tiny_gguf, max_ctx=256, numeric=TC)
    g = np.random.default_rng(cap)
    prompt = [int(t) for t in g.integers(0, TINY["vocab"], size=150)]
    cfg = hs.SamplerCfg.default(temperature=0.0)
    kv_a = m.kv()
    ref = hs.Batch(m, 1).run_seqs([kv_a], [state(prompt, 150, 20, cfg, 5)])[0]
    kv_b = m.kv()
    b = hs.Batch(m, cap)
    b.prefill(kv_b, prompt[:-1])
    got = hs.Batch(m, 1).run_seqs([kv_b], [state(prompt, 150, 20, cfg, 5, filled=149)])[0]
    assert list(got[0]) == list(ref[0])
    assert float(np.max(np.abs(kv_a.floats() - kv_b.floats()))) <= 1e-3


def test_prefill_in_pieces_equals_one_call(tiny_gguf):
    m = hs.Model.load(tiny_gguf, max_ctx=256, numeric=TC)
    prompt = [int(t) for t in np.random.default_rng(3).integers(0, TINY["vocab"], size=100)]
    b = hs.Batch(m, 64)
    one, two = m.kv(), m.kv()
    b.prefill(one, prompt)
    b.prefill(two, prompt[:37])
    b.prefill(two, prompt[37:], pos0=37)
    assert one.hash(100) == two.hash(100)


def test_prefill_greedy_continuation_matches_the_oracle(q05_gguf):
    g = np.random.default_rng(12)
    prompt = [int(t) for t in g.integers(0, QWEN05["vocab"], size=80)]
    cfg = hs.SamplerCfg.default(temperature=0.0)
    m = hs.Model.load(q05_gguf, max_ctx=256, numeric=TC)
    kv = m.kv()
    hs.Batch(m, 128).prefill(kv, prompt[:-1])
    got = hs.Batch(m, 1).run_seqs([kv], [state(prompt, 80, 16, cfg, 1, filled=79)])[0]
    o = ffi.Model(q05_gguf, max_ctx=256)
    want, _, _ = o.run_seq(o.new_kv(), prompt, 16, ffi.default_cfg(temperature=0.0), ffi.seeded_rng(1))
    assert list(got[0]) == list(want)


def test_prefill_rejects_bad_input(tiny_gguf):
    m = hs.Model.load(tiny_gguf, max_ctx=64, numeric=TC)
    b = hs.Batch(m, 64)
    kv = m.kv()
    with pytest.raises(hs.HotseatError):
        b.prefill(kv, [1] * 65)
    with pytest.raises(hs.HotseatError):
        b.prefill(kv, [1, 2, TINY["vocab"]])
    with pytest.raises(hs.HotseatError):
        b.prefill(kv, [1, 2], pos0=63)
