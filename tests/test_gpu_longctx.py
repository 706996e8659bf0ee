"""Attention over long contexts (scores past the shared-memory budget move to
a global buffer), on all three numeric paths, against the CPU restatement.

Filling 40,000 positions one forward at a time would take minutes on the
CPU, so both sides start from the same random KV bytes and run one forward
at a late position: the reference path must match bit for bit, the fast and
tensor-core paths within the token loop's 1e-2."""
import numpy as np
import pytest

import hotseat_b200 as hs
from oracle import ffi

from conftest import TINY

pytestmark = pytest.mark.gpu

MAX_CTX = 40000
LOGIT_TOL = 1e-2


@pytest.mark.parametrize("numeric", [hs.NUMERIC_REFERENCE, hs.NUMERIC_FAST, hs.NUMERIC_TC])
def test_long_context_forward_matches_the_oracle(tiny_gguf, numeric):
    m = hs.Model.load(tiny_gguf, max_ctx=MAX_CTX, numeric=numeric)
    o = ffi.Model(tiny_gguf, max_ctx=MAX_CTX)
    okv = o.new_kv()
    g = np.random.default_rng(11)
    okv[:] = g.normal(0.0, 0.5, size=okv.size).astype(np.float32)
    kv = m.kv()
    kv.write(0, okv.view(np.uint8))
    b = hs.Batch(m, 1) if numeric == hs.NUMERIC_TC else None
    s = None if b else m.scratch()
    for pos, tok in ((1000, 17), (16000, 403), (MAX_CTX - 3, 999)):
        want = o.forward(okv, tok, pos)
        if b:
            b.forward([kv], [tok], [pos])
            got = b.logits(0)
        else:
            m.forward(kv, tok, pos, s)
            got = s.logits()
        if numeric == hs.NUMERIC_REFERENCE:
            assert np.array_equal(got, want), pos
        else:
            err = float(np.max(np.abs(got - want)))
            assert err <= LOGIT_TOL, (pos, err)
    # the KV rows written at those positions match too
    got_kv = kv.floats()
    if numeric == hs.NUMERIC_REFERENCE:
        assert np.array_equal(got_kv, okv)
    else:
        assert float(np.max(np.abs(got_kv - okv))) <= LOGIT_TOL
