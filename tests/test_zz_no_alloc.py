"""hs_sample_noalloc, the sampler entry point that allocates nothing, against
hs_sample (and, above any model's vocabulary, the CPU sampler).

Both run the same two kernels, so the bar is exact: the same token, RNG state
and draw count, on two calls in a row that reuse the library's one fixed
array. Collected last so it also runs after everything else on the device."""
import ctypes as C

import numpy as np
import pytest
import torch

import hotseat_b200 as hs
from tests.golden.synth import QWEN05
from oracle import ffi

from conftest import TINY, TINY128

pytestmark = pytest.mark.gpu

MAX_VOCAB = 262144
MAX_WINDOW = 4096


def noalloc(dev_logits, vocab, cfg, rng, hist, stream=None):
    h = np.ascontiguousarray(hist, dtype=np.uint32)
    out = C.c_uint32()
    rc = hs.lib().hs_sample_noalloc(0, C.c_void_p(dev_logits.data_ptr()), vocab, C.byref(cfg), C.byref(rng),
                                    h.ctypes.data_as(C.c_void_p) if h.size else None, h.size, stream, C.byref(out))
    return rc, out.value


def on_device(logits):
    t = torch.from_numpy(np.ascontiguousarray(logits, dtype=np.float32)).to("cuda:0")
    torch.cuda.synchronize()
    return t


def draw_logits(rng, vocab):
    x = rng.normal(0.0, 3.0, size=vocab).astype(np.float32)
    x[rng.integers(0, vocab, size=8)] += 9.0  # a few clear leaders, like real logits
    return x


CFGS = {
    "sampled": dict(temperature=0.8, top_p=0.95, top_k=40, repeat_penalty=1.1, repeat_last_n=64),
    "greedy": dict(temperature=0.0, repeat_penalty=1.1, repeat_last_n=64),
    "plain": dict(temperature=1.0, top_p=1.0, top_k=0, repeat_penalty=1.0),
}


@pytest.mark.parametrize("which", ["tiny", "tiny128", "q05"])
@pytest.mark.parametrize("mode", list(CFGS))
def test_noalloc_matches_hs_sample_twice_in_a_row(which, mode, tiny_gguf, tiny128_gguf, q05_gguf):
    path, vocab = {"tiny": (tiny_gguf, TINY["vocab"]), "tiny128": (tiny128_gguf, TINY128["vocab"]),
                   "q05": (q05_gguf, QWEN05["vocab"])}[which]
    kw = dict(CFGS[mode])
    if mode == "plain" and vocab > 1024:
        kw["top_k"] = 64  # any top_k needs a single candidate CTA
    cfg = hs.SamplerCfg.default(**kw)
    m = hs.Model.load(path, max_ctx=128)
    s = m.scratch()
    g = np.random.default_rng(["tiny", "tiny128", "q05"].index(which) * 10 + list(CFGS).index(mode))
    rng_ref, rng_new = hs.Rng.seed(77), hs.Rng.seed(77)
    for call in range(2):
        logits = draw_logits(g, vocab)
        hist = g.integers(0, vocab, size=100).astype(np.uint32)
        hist[-20:] = np.argsort(logits)[-20:]  # the penalty must bite on the leaders
        s.set_logits(logits)
        want = hs.Sampler(cfg, rng_ref).sample(s, hist)
        dev = on_device(logits)
        rc, got = noalloc(dev, vocab, cfg, rng_new, hist, stream=s.stream if call else None)
        assert rc == hs.HS_OK, hs.lib().hs_last_error().decode()
        assert got == want, (call, got, want)
        assert list(rng_new.s) == list(rng_ref.s) and rng_new.draws == rng_ref.draws


def test_noalloc_at_its_maximum_sizes_matches_the_cpu_sampler():
    g = np.random.default_rng(5)
    for kw in (CFGS["sampled"], CFGS["greedy"]):
        kw = dict(kw, repeat_last_n=MAX_WINDOW)
        cfg = hs.SamplerCfg.default(**kw)
        ocfg = ffi.default_cfg(**kw)
        rng, orng = hs.Rng.seed(3), ffi.seeded_rng(3)
        for _ in range(2):
            logits = draw_logits(g, MAX_VOCAB)
            hist = g.integers(0, MAX_VOCAB, size=MAX_WINDOW + 50).astype(np.uint32)
            hist[-30:] = np.argsort(logits)[-30:]
            rc, got = noalloc(on_device(logits), MAX_VOCAB, cfg, rng, hist)
            assert rc == hs.HS_OK, hs.lib().hs_last_error().decode()
            want = ffi.lib().hso_sample(C.byref(ocfg), C.byref(orng), ffi.ptr(logits), logits.size, ffi.ptr(hist),
                                        hist.size)
            assert got == want
            assert list(rng.s) == list(orng.s) and rng.draws == orng.draws


def test_noalloc_refuses_sizes_beyond_its_array():
    dev = on_device(np.zeros(16, dtype=np.float32))
    cfg = hs.SamplerCfg.default()
    rc, _ = noalloc(dev, MAX_VOCAB + 1, cfg, hs.Rng.seed(1), [])
    assert rc == hs.HS_E_ARG and "262144" in hs.lib().hs_last_error().decode()
    cfg = hs.SamplerCfg.default(repeat_penalty=1.1, repeat_last_n=MAX_WINDOW + 1)
    rc, _ = noalloc(dev, 16, cfg, hs.Rng.seed(1), np.zeros(MAX_WINDOW + 1, dtype=np.uint32))
    assert rc == hs.HS_E_ARG and "4096" in hs.lib().hs_last_error().decode()
    # a long history with a short window is fine: only the window is used
    cfg = hs.SamplerCfg.default(repeat_penalty=1.1, repeat_last_n=64)
    rc, _ = noalloc(dev, 16, cfg, hs.Rng.seed(1), np.zeros(MAX_WINDOW * 4, dtype=np.uint32))
    assert rc == hs.HS_OK, hs.lib().hs_last_error().decode()
