"""Model::forward on the GPU against the CPU restatement.

The batch-1 kernels keep the reference's accumulation order, so the bar here
is bit equality of logits and of the KV bytes. The tolerance the token loop is
held to (logits within 1e-2 max-abs of the CPU path) is asserted as well, so a
deliberate change of numeric path would still be checked against it."""
import numpy as np
import pytest

import hotseat_b200 as hs
from tests.golden.synth import QWEN05
from oracle import ffi

from conftest import TINY, TINY128

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2


def compare_run(path, vocab, n_pos, max_ctx, layout=0, seed=0):
    rng = np.random.default_rng(seed)
    toks = [int(t) for t in rng.integers(0, vocab, size=n_pos)]
    m = hs.Model.load(path, max_ctx=max_ctx)
    o = ffi.Model(path, max_ctx=max_ctx)
    assert m.fingerprint == o.cfg.fingerprint and m.eos == o.cfg.eos
    kv, s = m.kv(layout), m.scratch()
    okv = o.new_kv(layout)
    for pos, tok in enumerate(toks):
        m.forward(kv, tok, pos, s)
        got = s.logits()
        want = o.forward(okv, tok, pos, layout=layout)
        assert np.max(np.abs(got - want)) <= LOGIT_TOL, pos
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (pos, np.max(np.abs(got - want)))
    assert np.array_equal(kv.floats().view(np.uint32), okv.view(np.uint32))
    assert kv.hash(n_pos) == ffi.kv_hash(o.kv_spec(layout), okv, n_pos)
    return m, kv, s


@pytest.mark.parametrize("layout", [0, 1])
def test_tiny_logits_and_kv_bit_exact(tiny_gguf, layout):
    compare_run(tiny_gguf, TINY["vocab"], 40, 64, layout)


def test_head_dim_128_logits_bit_exact(tiny128_gguf):
    compare_run(tiny128_gguf, TINY128["vocab"], 24, 48)


def test_long_context_crosses_attention_chunks(tiny_gguf):
    # 300 positions: several 128-position staging chunks in the attention kernel.
    compare_run(tiny_gguf, TINY["vocab"], 300, 320, seed=3)


def test_05b_shape_logits_bit_exact(q05_gguf):
    compare_run(q05_gguf, QWEN05["vocab"], 5, 64)


def test_forward_rejects_out_of_range_inputs(tiny_gguf):
    m = hs.Model.load(tiny_gguf, max_ctx=16)
    kv, s = m.kv(), m.scratch()
    with pytest.raises(hs.HotseatError) as e:
        m.forward(kv, 1, 16, s)
    assert e.value.code == hs.HS_E_ARG and "max_ctx" in str(e.value)
    with pytest.raises(hs.HotseatError) as e:
        m.forward(kv, TINY["vocab"], 0, s)
    assert e.value.code == hs.HS_E_ARG
    m2 = hs.Model.load(tiny_gguf, max_ctx=32)
    with pytest.raises(hs.HotseatError) as e:
        m2.forward(kv, 1, 0, m2.scratch())  # KV shaped for another max_ctx
    assert "shape" in str(e.value)
