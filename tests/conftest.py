import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA path)")


def _build_all():
    from oracle import ffi as oracle_ffi
    oracle_ffi.build()
    from tests.golden import synth
    synth.build()
    import importlib.util
    spec = importlib.util.spec_from_file_location("hs_build", os.path.join(ROOT, "hotseat_b200", "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build()  # no-op when the library is newer than every source; raises if nvcc fails


_build_all()

from tests.golden.synth import QWEN05, QWEN15, write_synthetic_gguf  # noqa: E402

TINY = dict(n_layers=2, d_model=256, n_heads=4, n_kv_heads=2, d_ff=512, vocab=1000, seed=7)
TINY128 = dict(n_layers=2, d_model=256, n_heads=2, n_kv_heads=1, d_ff=768, vocab=1500, seed=11)


def gpu_count():
    try:
        import torch
        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0


@pytest.fixture(scope="session")
def fixture_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("gguf")


@pytest.fixture(scope="session")
def tiny_gguf(fixture_dir):
    p = str(fixture_dir / "tiny.gguf")
    write_synthetic_gguf(p, **TINY)
    return p


@pytest.fixture(scope="session")
def tiny128_gguf(fixture_dir):
    p = str(fixture_dir / "tiny128.gguf")
    write_synthetic_gguf(p, **TINY128)
    return p


@pytest.fixture(scope="session")
def q05_gguf(fixture_dir):
    """The Qwen2.5-0.5B-shape seeded model (Q6_K embedding, Q4_K weights)."""
    p = str(fixture_dir / "qwen05.gguf")
    write_synthetic_gguf(p, seed=1234, **QWEN05)
    return p


@pytest.fixture(scope="session")
def q15_gguf(fixture_dir):
    """The Qwen2.5-1.5B-shape seeded model (28 layers, d 1536, 12/2 heads,
    head_dim 128, ff 8960; Q6_K embedding, Q4_K weights)."""
    p = str(fixture_dir / "qwen15.gguf")
    write_synthetic_gguf(p, seed=1234, **QWEN15)
    return p
