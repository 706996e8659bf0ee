"""The perplexity harness (hotseat_b200.ppl, examples/ppl.rs) against the CPU
restatement: the same windows and scored positions, each token's score from
the oracle's logits and ppl.rs's formula (hso_nll). The bit-exact numeric
path gives the same mean NLL to f64 rounding (the device sums the
exponentials in a fixed tree order, the reference in sequence); the
GPU-native and tensor-core paths within the token loop's logit tolerance."""
import ctypes as C

import numpy as np
import pytest

import hotseat_b200 as hs
from hotseat_b200 import ppl
from oracle import ffi

from conftest import TINY

pytestmark = pytest.mark.gpu


def oracle_ppl(path, ids, ctx):
    o = ffi.Model(path, max_ctx=ctx, threads=2)
    nll, counted = 0.0, 0
    for c in range(len(ids) // ctx):
        w = ids[c * ctx:(c + 1) * ctx]
        kv = o.new_kv()
        for p, t in enumerate(w):
            logits = o.forward(kv, t, p)
            if p >= ctx // 2 and p + 1 < len(w):
                nll += ffi.lib().hso_nll(ffi.ptr(logits), logits.size, w[p + 1])
                counted += 1
    return nll / counted, counted


@pytest.mark.parametrize("numeric, tol", [(hs.NUMERIC_REFERENCE, 1e-12), (hs.NUMERIC_FAST, 1e-2),
                                          (hs.NUMERIC_TC, 1e-2)])
def test_ppl_matches_the_oracle(tiny_gguf, numeric, tol):
    ctx = 32
    ids = [int(t) for t in np.random.default_rng(17).integers(0, TINY["vocab"], size=3 * ctx + 7)]
    want, counted = oracle_ppl(tiny_gguf, ids, ctx)
    m = hs.Model.load(tiny_gguf, max_ctx=ctx, numeric=numeric)
    r = ppl.score(m, ids, ctx)
    assert r["windows"] == 3 and r["scored"] == counted == 3 * (ctx // 2 - 1)
    assert abs(r["mean_nll"] - want) <= tol * max(1.0, abs(want)), (r["mean_nll"], want)


def test_nll_of_one_row_matches_the_formula(tiny_gguf):
    m = hs.Model.load(tiny_gguf, max_ctx=16)
    s = m.scratch()
    rng = np.random.default_rng(2)
    for scale in (0.1, 3.0, 30.0):
        logits = (rng.standard_normal(TINY["vocab"]) * scale).astype(np.float32)
        s.set_logits(logits)
        for nxt in (0, 17, TINY["vocab"] - 1):
            want = ffi.lib().hso_nll(ffi.ptr(logits), logits.size, nxt)
            assert abs(s.nll(nxt) - want) <= 1e-12 * max(1.0, abs(want))
