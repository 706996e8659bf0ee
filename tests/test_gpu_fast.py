"""The GPU-native numeric path (HS_NUMERIC_FAST) against the CPU restatement,
in both of its forms: the persistent token kernel (tensor-core rows, the
default where it fits) and the per-kernel launches (HS_TOKEN_KERNEL=0).

Its reductions use fixed GPU shapes instead of the reference's eight serial
lanes, so the bar is the token loop's: logits within 1e-2 max-abs of the CPU
path, identical greedy tokens (near-ties reported with their margin), and
bit-exact results GPU-to-GPU, including across a migration."""
import numpy as np
import pytest

import hotseat_b200 as hs
from tests.golden.synth import QWEN05
from oracle import ffi

from conftest import TINY, TINY128

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2
FAST = hs.NUMERIC_FAST


@pytest.fixture(autouse=True, params=["token_kernel", "per_kernel"])
def form(request, monkeypatch):
    monkeypatch.setenv("HS_TOKEN_KERNEL", "1" if request.param == "token_kernel" else "0")
    return request.param


def load(path, max_ctx):
    return hs.Model.load(path, max_ctx=max_ctx, numeric=FAST)


@pytest.mark.parametrize("which", ["tiny", "tiny128", "q05"])
def test_fast_logits_within_tolerance(which, tiny_gguf, tiny128_gguf, q05_gguf):
    path, vocab, n_pos = {"tiny": (tiny_gguf, TINY["vocab"], 40), "tiny128": (tiny128_gguf, TINY128["vocab"], 24),
                          "q05": (q05_gguf, QWEN05["vocab"], 6)}[which]
    rng = np.random.default_rng(2)
    toks = [int(t) for t in rng.integers(0, vocab, size=n_pos)]
    m = load(path, 64)
    o = ffi.Model(path, max_ctx=64)
    kv, s, okv = m.kv(), m.scratch(), o.new_kv()
    worst = 0.0
    for pos, tok in enumerate(toks):
        m.forward(kv, tok, pos, s)
        got, want = s.logits(), o.forward(okv, tok, pos)
        err = float(np.max(np.abs(got - want)))
        worst = max(worst, err)
        assert err <= LOGIT_TOL, (pos, err)
    # the KV rows are within the same kind of tolerance
    kv_err = float(np.max(np.abs(kv.floats() - okv)))
    assert kv_err <= LOGIT_TOL
    print(f"{which}: worst logit error {worst:.3g}, KV {kv_err:.3g}")


def test_fast_path_has_its_own_fingerprint(tiny_gguf):
    a = hs.Model.load(tiny_gguf, max_ctx=16)
    b = load(tiny_gguf, 16)
    assert a.fingerprint == ffi.Model(tiny_gguf, max_ctx=16).cfg.fingerprint
    assert b.fingerprint != a.fingerprint and b.cfg.numeric == FAST


def run(m, prompt, max_tokens, cfg, seed, kv=None, s=None):
    kv = kv or m.kv()
    s = s or m.scratch()
    toks, st, rng = hs.run_seq(m, kv, s, prompt, len(prompt), max_tokens, cfg, hs.Rng.seed(seed))
    return list(toks), st, rng, kv.hash(st.filled)


def test_fast_greedy_tokens_match_the_oracle(q05_gguf):
    """Greedy decode (temperature 0, penalty 1.1) of the 0.5B shape: the GPU
    path must pick the CPU path's token at every step. A disagreement is
    reported with the CPU logits' top-1/top-2 margin at that step."""
    rng = np.random.default_rng(36)
    prompt = [int(t) for t in rng.integers(0, QWEN05["vocab"], size=36)]
    cfg = hs.SamplerCfg.default(temperature=0.0)
    m = load(q05_gguf, 256)
    got = run(m, prompt, 48, cfg, 1)[0]
    o = ffi.Model(q05_gguf, max_ctx=256)
    okv = o.new_kv()
    ocfg = ffi.default_cfg(temperature=0.0)
    want, _, _ = o.run_seq(okv, prompt, 48, ocfg, ffi.seeded_rng(1))
    want = list(want)
    if got != want:
        i = next(k for k in range(min(len(got), len(want))) if got[k] != want[k])
        o2 = ffi.Model(q05_gguf, max_ctx=256)
        kv2 = o2.new_kv()
        for p in range(i):
            logits = o2.forward(kv2, want[p], p)
        top = np.sort(logits)[-2:]
        pytest.fail(f"first divergence at index {i}: gpu {got[i]} cpu {want[i]}, cpu top-2 margin {top[1] - top[0]:.3g}")


def test_fast_sampled_c1_transcript_matches_the_oracle(q05_gguf):
    rng = np.random.default_rng(36)
    prompt = [int(t) for t in rng.integers(0, QWEN05["vocab"], size=36)]
    cfg = hs.SamplerCfg.default(temperature=0.8, seed=99)
    m = load(q05_gguf, 2048)
    g = run(m, prompt, 120, cfg, 99)
    o = ffi.Model(q05_gguf, max_ctx=2048)
    okv = o.new_kv()
    want, ost, orng = o.run_seq(okv, prompt, 120, ffi.default_cfg(temperature=0.8, seed=99), ffi.seeded_rng(99))
    assert g[0] == list(want)
    assert list(g[2].s) == list(orng.s) and g[2].draws == orng.draws


def test_fast_path_is_deterministic_gpu_to_gpu(tiny_gguf):
    m = load(tiny_gguf, 96)
    cfg = hs.SamplerCfg.default()
    prompt = list(range(40, 52))
    a = run(m, prompt, 40, cfg, 4)
    b = run(m, prompt, 40, cfg, 4)
    assert a[0] == b[0] and a[3] == b[3] and list(a[2].s) == list(b[2].s)
    # a second model instance (fresh load, fresh plans) gives the same bits
    m2 = load(tiny_gguf, 96)
    c = run(m2, prompt, 40, cfg, 4)
    assert a[0] == c[0] and a[3] == c[3]


def test_fast_migration_reproduces_the_unmigrated_transcript(tiny_gguf):
    from test_gpu_seq import precopy_migrate
    m = load(tiny_gguf, 96)
    cfg = hs.SamplerCfg.default()
    prompt = list(range(500, 512))
    ref = run(m, prompt, 40, cfg, 8)
    src_kv, dst_kv = m.kv(), m.kv()
    toks, st, rng, _ = precopy_migrate(m, src_kv, dst_kv, m.scratch(), prompt, 40, cfg, hs.Rng.seed(8), 18)
    t2, st2, _ = hs.run_seq(m, dst_kv, m.scratch(), toks, len(prompt), 40, cfg, rng, filled=st.filled)
    assert list(t2) == ref[0] and dst_kv.hash(st2.filled) == ref[3]
