"""Prompt prefill on the tensor-core path (hs_prefill): the prompt's tokens as
the rows of every GEMM, K/V appended for all of them before any attends.

Prefill GEMMs use wide weight tiles and no K split (the prompt's tokens
give the parallelism), so their sums are ordered differently from the decode
steps': the KV rows match token-by-token decoding within the path's
tolerance, greedy continuations are identical, prefill in pieces is
bit-identical to one call, and the greedy tokens match the CPU path.

Prefill attention runs by query blocks over fixed segments of cached
positions (attn_prefill.cu), its products on the tensor cores (f16 hi/lo
operands); HS_PREFILL_ATTN=1 at model load runs the blocks on the CUDA cores
and 0 the per-token split items. All three agree within tolerance on prompts
that span several segments, and a token's bits do not depend on the pass it
is in."""
import os

import numpy as np
import pytest

import hotseat_b200 as hs
from tests.golden.synth import QWEN05
from oracle import ffi

from conftest import TINY, TINY128

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


QBLOCK_TC, QBLOCK_CUDA_CORES, PER_TOKEN = "2", "1", "0"


def _load(path, max_ctx, mode):
    old = os.environ.get("HS_PREFILL_ATTN")
    os.environ["HS_PREFILL_ATTN"] = mode
    try:
        return hs.Model.load(path, max_ctx=max_ctx, numeric=TC)
    finally:
        if old is None:
            del os.environ["HS_PREFILL_ATTN"]
        else:
            os.environ["HS_PREFILL_ATTN"] = old


@pytest.mark.parametrize("mode", [QBLOCK_TC, QBLOCK_CUDA_CORES])
@pytest.mark.parametrize("shape,n", [("tiny", 700), ("tiny128", 700), ("q05", 600), ("tiny128", 200)])
def test_query_block_prefill_matches_the_per_token_items(shape, n, mode, request):
    """Several 384-position segments (and one, at 200): the same KV rows and
    next-token logits as the per-token split items within tolerance."""
    path, vocab = {"tiny": ("tiny_gguf", TINY["vocab"]), "tiny128": ("tiny128_gguf", TINY128["vocab"]),
                   "q05": ("q05_gguf", QWEN05["vocab"])}[shape]
    path = request.getfixturevalue(path)
    prompt = [int(t) for t in np.random.default_rng(n).integers(0, vocab, size=n)]
    got = []
    for md in (mode, PER_TOKEN):
        m = _load(path, 1024, md)
        kv = m.kv()
        hs.Batch(m, 256).prefill(kv, prompt[:-1])
        b = hs.Batch(m, 1)
        b.forward([kv], [prompt[-1]], [n - 1])
        got.append((kv.floats(), b.logits(0)))
    kv_err = float(np.max(np.abs(got[0][0] - got[1][0])))
    logit_err = float(np.max(np.abs(got[0][1] - got[1][1])))
    print(f"{shape}, {n - 1} prompt tokens, mode {mode}: KV {kv_err:.3g}, logits {logit_err:.3g}")
    assert kv_err <= 1e-3 and logit_err <= 1e-2


@pytest.mark.parametrize("mode", [QBLOCK_TC, QBLOCK_CUDA_CORES])
def test_query_block_prefill_in_pieces_equals_one_call_across_segments(tiny128_gguf, mode):
    """Passes cut at 301 and at multiples of 128 put the tokens in different
    query blocks: the KV region is bit-identical."""
    m = _load(tiny128_gguf, 1024, mode)
    prompt = [int(t) for t in np.random.default_rng(31).integers(0, TINY128["vocab"], size=700)]
    b = hs.Batch(m, 128)
    one, two = m.kv(), m.kv()
    b.prefill(one, prompt)
    b.prefill(two, prompt[:301])
    b.prefill(two, prompt[301:], pos0=301)
    assert one.hash(700) == two.hash(700)


def test_query_block_prefill_then_decode_matches_token_by_token(tiny128_gguf):
    m = hs.Model.load(tiny128_gguf, max_ctx=1024, numeric=TC)
    prompt = [int(t) for t in np.random.default_rng(5).integers(0, TINY128["vocab"], size=600)]
    cfg = hs.SamplerCfg.default(temperature=0.0)
    kv_a = m.kv()
    ref = hs.Batch(m, 1).run_seqs([kv_a], [state(prompt, 600, 16, cfg, 2)])[0]
    kv_b = m.kv()
    hs.Batch(m, 512).prefill(kv_b, prompt[:-1])
    got = hs.Batch(m, 1).run_seqs([kv_b], [state(prompt, 600, 16, cfg, 2, filled=599)])[0]
    assert list(got[0]) == list(ref[0])
    assert float(np.max(np.abs(kv_a.floats() - kv_b.floats()))) <= 1e-3


@pytest.mark.parametrize("layout", [hs.TOKEN_MAJOR, hs.HEAD_MAJOR])
def test_prefill_marks_exactly_the_pages_it_writes(tiny128_gguf, layout):
    """An armed region: the prefill append marks the pages of every k, v row
    it writes, the same bits as the per-token items."""
    prompt = [int(t) for t in np.random.default_rng(9).integers(0, TINY128["vocab"], size=300)]
    got = []
    for md in (QBLOCK_TC, PER_TOKEN):
        m = _load(tiny128_gguf, 1024, md)
        kv = m.kv(layout=layout, page_size=4096)
        kv.arm()
        hs.Batch(m, 128).prefill(kv, prompt, pos0=0)
        got.append(kv.harvest())
        kv.disarm()
    c = m.cfg
    hd, nkv, T = c.head_dim, c.n_kv_heads, c.max_ctx
    want = np.zeros_like(got[0])
    for layer in range(c.n_layers):
        for is_v in (0, 1):
            for kvh in range(nkv):
                for p in range(len(prompt)):
                    within = (p * nkv + kvh) * hd if layout == hs.TOKEN_MAJOR else (kvh * T + p) * hd
                    off = ((layer * 2 + is_v) * T * nkv * hd + within) * 4
                    for pg in range(off // 4096, (off + hd * 4 - 1) // 4096 + 1):
                        want[pg >> 6] |= np.uint64(1) << np.uint64(pg & 63)
    assert np.array_equal(got[0], want) and np.array_equal(got[1], want)


def test_one_2048_token_pass_equals_128_token_passes(tiny128_gguf):
    """A batch of 2,048 slots prefills a 2,000-token prompt in one pass; the
    KV region is bit-identical to passes of 128 tokens."""
    m = hs.Model.load(tiny128_gguf, max_ctx=2048, numeric=TC)
    prompt = [int(t) for t in np.random.default_rng(41).integers(0, TINY128["vocab"], size=2000)]
    one, many = m.kv(), m.kv()
    hs.Batch(m, 2048).prefill(one, prompt)
    hs.Batch(m, 128).prefill(many, prompt)
    assert one.hash(2000) == many.hash(2000)
