"""Failure detection without a GPU fault.

Device side: the persistent token kernel's readers poll tagged entries that
other CTAs write, and every poll is bounded. With the test knob
HS_POLL_LIMIT=0 (read when a scratch is created) a reader gives up at the
first round whose data is not there yet; the launch must then finish, the
call must return HS_E_CUDA naming the bounded wait, and the GPU, the model
and a fresh scratch must keep working (the next forwards match the CPU
path). The weight ring's waits keep their normal limit, so no copy is left
in flight when a CTA gives up.

Host side: a KV byte run corrupted in transit is caught by the hand-over's
KV-hash check, and a destination whose model fingerprint differs refuses the
hand-over before any byte moves (migrate.rs:486-518, 583-594)."""
import numpy as np
import pytest

import hotseat_b200 as hs
from oracle import ffi

pytestmark = pytest.mark.gpu


def test_token_kernel_poll_timeout_is_reported_and_the_device_recovers(tiny_gguf, monkeypatch):
    m = hs.Model.load(tiny_gguf, max_ctx=64, numeric=hs.NUMERIC_FAST)
    monkeypatch.setenv("HS_POLL_LIMIT", "0")
    bad = m.scratch()
    monkeypatch.delenv("HS_POLL_LIMIT")
    assert bad.launches_per_step() == 3  # the persistent token kernel runs
    kv = m.kv()
    errors = []
    for pos, tok in enumerate([11, 22, 33]):
        try:
            m.forward(kv, tok, pos, bad)
        except hs.HotseatError as e:
            errors.append(e)
    assert errors, "no reader gave up with a zero poll limit"
    assert all(e.code == hs.HS_E_CUDA and "bounded-wait-timeout" in str(e) for e in errors)
    # the same model on a scratch with the normal limit: still the CPU path's logits
    good = m.scratch()
    o = ffi.Model(tiny_gguf, max_ctx=64, threads=2)
    kv2, okv = m.kv(), o.new_kv()
    for pos, tok in enumerate([11, 22, 33, 44, 55]):
        m.forward(kv2, tok, pos, good)
        assert float(np.max(np.abs(good.logits() - o.forward(okv, tok, pos)))) <= 1e-2
    # a decode loop on a fresh scratch after the failures: the CPU path's transcript
    bad.close()
    cfg = hs.SamplerCfg.default(temperature=0.0)
    toks = hs.run_seq(m, m.kv(), m.scratch(), [5, 6, 7], 3, 6, cfg, hs.Rng.seed(1))[0]
    want = o.run_seq(o.new_kv(), [5, 6, 7], 6, ffi.default_cfg(temperature=0.0), ffi.seeded_rng(1))[0]
    assert list(toks) == list(want)
