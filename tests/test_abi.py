"""The C ABI without a GPU: the library loads, exports every entry point that
include/hotseat.h declares, and its host-side logic (KV range arithmetic,
dirty-page runs, RNG seeding, the synthetic GGUF writer) agrees with the CPU
restatement of the reference."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import hotseat_b200 as hs
from oracle import ffi
from tests.golden.synth import write_synthetic_gguf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "hotseat.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hs_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_entry_point():
    names = declared_functions()
    assert len(names) >= 30
    lib = C.CDLL(hs.LIB_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(hs.EXPORTED)


def test_errors_are_reported_not_raised_without_a_device(tiny_gguf):
    # A bad path is an I/O error from the GGUF reader, before any CUDA call.
    with pytest.raises(hs.HotseatError) as e:
        hs.Model.load("/nonexistent/model.gguf", 64)
    assert e.value.code == hs.HS_E_IO


def test_gguf_format_errors_are_reported(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGML" + b"\0" * 60)
    with pytest.raises(hs.HotseatError) as e:
        hs.Model.load(str(p), 64)
    assert e.value.code == hs.HS_E_IO and "magic" in str(e.value)
    p.write_bytes(struct_pack_header(9))
    with pytest.raises(hs.HotseatError) as e:
        hs.Model.load(str(p), 64)
    assert "version" in str(e.value)


def struct_pack_header(version):
    import struct
    return struct.pack("<IIQQ", 0x46554747, version, 0, 0)


def test_sampler_defaults_and_seeding_match_the_reference():
    c = hs.SamplerCfg.default()
    o = ffi.default_cfg()
    for k in ("temperature", "top_p", "top_k", "repeat_penalty", "repeat_last_n", "seed"):
        assert getattr(c, k) == getattr(o, k)
    for seed in (0, 1, 42, 99, 0xC0FFEE0012345678, 2 ** 64 - 1):
        a, b = hs.Rng.seed(seed), ffi.seeded_rng(seed)
        assert list(a.s) == list(b.s) and a.draws == 0


@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("shape", [(3, 2, 8, 16), (24, 2, 64, 2048), (28, 2, 128, 4096)])
def test_live_ranges_match_the_reference(layout, shape):
    s = hs.KvSpec(*shape, layout)
    o = ffi.kv_spec(*shape, layout)
    for a, b in [(0, 0), (0, 1), (0, 7), (3, 10), (5, 5), (9, 3), (0, shape[3]), (shape[3] - 1, shape[3])]:
        assert hs.live_ranges_between(s, a, b) == ffi.live_ranges_between(o, a, b)


def test_byte_runs_match_the_reference_on_random_sets():
    rng = np.random.default_rng(11)
    for trial in range(60):
        n_pages = int(rng.integers(1, 700))
        dens = rng.choice([0.02, 0.3, 0.9])
        bits = rng.random(n_pages) < dens
        w = np.zeros((n_pages + 63) // 64, dtype=np.uint64)
        for p in np.nonzero(bits)[0]:
            w[p // 64] |= np.uint64(1) << np.uint64(p % 64)
        ps = int(rng.choice([256, 4096, 16384]))
        live = []
        for _ in range(int(rng.integers(0, 6))):
            off = int(rng.integers(0, n_pages * ps))
            live.append((off, int(rng.integers(1, 3 * ps))))
        assert hs.runs_to_byte_runs(w, n_pages, ps, live) == ffi.runs_to_byte_runs(w, n_pages, ps, live)


def test_reference_byte_run_cases_on_the_product():
    def words(n, marks):
        w = np.zeros((n + 63) // 64, dtype=np.uint64)
        for p in marks:
            w[p // 64] |= np.uint64(1) << np.uint64(p % 64)
        return w
    # hs-wire lib.rs:457-503
    assert hs.runs_to_byte_runs(words(100, range(100)), 100, 4096, [(0, 10_000)]) == [(0, 10_000)]
    assert hs.runs_to_byte_runs(words(100, range(3, 8)), 100, 4096, [(0, 100 * 4096)]) == [(3 * 4096, 5 * 4096)]
    assert hs.runs_to_byte_runs(words(8, [2]), 8, 16384, [(2 * 16384, 512)]) == [(2 * 16384, 512)]
    live = [(0, 8192), (40 * 4096, 8192)]
    assert hs.runs_to_byte_runs(words(64, range(64)), 64, 4096, live) == live
    assert hs.runs_to_byte_runs(words(64, []), 64, 4096, [(0, 1 << 20)]) == []


def test_synthetic_writer_is_deterministic_across_thread_counts(tmp_path):
    a, b = str(tmp_path / "a.gguf"), str(tmp_path / "b.gguf")
    spec = dict(n_layers=1, d_model=128, n_heads=2, n_kv_heads=1, d_ff=256, vocab=300, seed=3)
    write_synthetic_gguf(a, threads=1, **spec)
    write_synthetic_gguf(b, threads=7, **spec)
    assert open(a, "rb").read() == open(b, "rb").read()


def test_synthetic_model_has_the_requested_distribution(tiny_gguf):
    m = ffi.Model(tiny_gguf, max_ctx=16, threads=2)
    w = m.tensor_f16("blk.1.ffn_up.weight").view(np.float16).astype(np.float32)
    assert abs(w.std() - 0.02) < 0.002 and abs(w.mean()) < 0.001
    assert np.all(m.tensor_f32("blk.0.ffn_norm.weight") == 1.0)
    b = m.tensor_f32("blk.0.attn_q.bias")
    assert abs(b.std() - 0.02) < 0.005
    assert m.tensor_f16("output.weight") is None  # tied head


def test_synthetic_writer_rejects_bad_shapes(tmp_path):
    with pytest.raises(RuntimeError):
        write_synthetic_gguf(str(tmp_path / "x.gguf"), n_layers=1, d_model=100, n_heads=3, n_kv_heads=1,
                                d_ff=256, vocab=300, seed=1)
