"""The fast path's persistent token kernel (one launch per token: all layers'
phases between grid barriers, the weights streamed through a shared-memory
ring) against the same path's per-kernel launches (HS_TOKEN_KERNEL=0 at model
load).

Both run the same arithmetic (the fast GEMV's row order, split-KV attention),
so logits, KV rows, sampled tokens and RNG state must be bit-identical, at
short contexts (one attention split), a few splits (the last-CTA combine) and
long contexts (more attention items than CTAs)."""
import numpy as np
import pytest

import hotseat_b200 as hs
from tests.golden.synth import QWEN05

from conftest import TINY, TINY128

pytestmark = pytest.mark.gpu

FAST = hs.NUMERIC_FAST


def load(path, max_ctx, token_kernel, monkeypatch):
    monkeypatch.setenv("HS_TOKEN_KERNEL", "1" if token_kernel else "0")
    return hs.Model.load(path, max_ctx=max_ctx, numeric=FAST)


def test_token_kernel_is_one_launch_per_forward(tiny_gguf, monkeypatch):
    one = load(tiny_gguf, 64, True, monkeypatch).scratch()
    many = load(tiny_gguf, 64, False, monkeypatch).scratch()
    assert one.launches_per_step() == 1 + 2  # the token kernel + the two sampler kernels
    assert many.launches_per_step() == 5 * TINY["n_layers"] + 1 + 2


@pytest.mark.parametrize("which", ["tiny", "tiny128", "q05"])
def test_token_kernel_forward_is_bit_identical(which, tiny_gguf, tiny128_gguf, q05_gguf, monkeypatch):
    path, vocab, n_pos, max_ctx = {"tiny": (tiny_gguf, TINY["vocab"], 200, 512),
                                   "tiny128": (tiny128_gguf, TINY128["vocab"], 150, 512),
                                   "q05": (q05_gguf, QWEN05["vocab"], 80, 256)}[which]
    rng = np.random.default_rng(5)
    toks = [int(t) for t in rng.integers(0, vocab, size=n_pos)]
    a = load(path, max_ctx, True, monkeypatch)
    b = load(path, max_ctx, False, monkeypatch)
    assert a.fingerprint == b.fingerprint
    kva, kvb, sa, sb = a.kv(), b.kv(), a.scratch(), b.scratch()
    for pos, tok in enumerate(toks):
        a.forward(kva, tok, pos, sa)
        b.forward(kvb, tok, pos, sb)
        la, lb = sa.logits(), sb.logits()
        assert np.array_equal(la, lb), (pos, float(np.max(np.abs(la - lb))))
    assert np.array_equal(kva.floats(), kvb.floats())


def test_token_kernel_sampled_sequence_is_bit_identical(q05_gguf, monkeypatch):
    rng = np.random.default_rng(36)
    prompt = [int(t) for t in rng.integers(0, QWEN05["vocab"], size=24)]
    cfg = hs.SamplerCfg.default(temperature=0.8, seed=99)
    out = []
    for tk in (True, False):
        m = load(q05_gguf, 512, tk, monkeypatch)
        kv = m.kv()
        toks, st, r = hs.run_seq(m, kv, m.scratch(), prompt, len(prompt), 96, cfg, hs.Rng.seed(99))
        out.append((list(toks), list(r.s), r.draws, kv.hash(st.filled)))
    assert out[0] == out[1]


def test_token_kernel_long_context_is_bit_identical(tiny_gguf, monkeypatch):
    """40,000 positions: 128 attention splits of up to 320 positions, so a
    CTA runs several attention items and each item several chunks."""
    max_ctx = 40000
    a = load(tiny_gguf, max_ctx, True, monkeypatch)
    b = load(tiny_gguf, max_ctx, False, monkeypatch)
    kva, kvb = a.kv(), b.kv()
    g = np.random.default_rng(11)
    init = g.normal(0.0, 0.5, size=kva.floats().size).astype(np.float32)
    kva.write(0, init.view(np.uint8))
    kvb.write(0, init.view(np.uint8))
    sa, sb = a.scratch(), b.scratch()
    for pos, tok in ((1000, 17), (16000, 403), (max_ctx - 3, 999)):
        a.forward(kva, tok, pos, sa)
        b.forward(kvb, tok, pos, sb)
        assert np.array_equal(sa.logits(), sb.logits()), pos
    assert np.array_equal(kva.floats(), kvb.floats())


def test_token_kernel_reports_bad_input(tiny_gguf, monkeypatch):
    m = load(tiny_gguf, 32, True, monkeypatch)
    kv, s = m.kv(), m.scratch()
    with pytest.raises(hs.HotseatError):
        m.forward(kv, TINY["vocab"], 0, s)
    with pytest.raises(hs.HotseatError):
        m.forward(kv, 1, 32, s)
    # still usable afterwards
    m.forward(kv, 1, 0, s)
    assert np.all(np.isfinite(s.logits()))


def test_token_kernel_head_split_keeps_the_bits(q05_gguf, monkeypatch):
    """Attention items over parts of a group's query heads (more CTAs per
    split) give the same logits as whole groups."""
    rng = np.random.default_rng(8)
    toks = [int(t) for t in rng.integers(0, QWEN05["vocab"], size=150)]
    out = []
    for hsplit in ("1", "2"):
        monkeypatch.setenv("HS_ATTN_HEAD_SPLIT", hsplit)
        m = load(q05_gguf, 256, True, monkeypatch)
        kv, s = m.kv(), m.scratch()
        rows = []
        for pos, tok in enumerate(toks):
            m.forward(kv, tok, pos, s)
            if pos % 10 == 9:
                rows.append(s.logits())
        out.append((np.stack(rows), kv.floats()))
    assert np.array_equal(out[0][0], out[1][0]) and np.array_equal(out[0][1], out[1][1])
