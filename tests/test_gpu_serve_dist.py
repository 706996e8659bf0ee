"""Serving with live migration across processes on the GPUs
(hotseat_b200.serve_dist): one GPU (the destination a second region on it),
and two ranks under torchrun over NCCL where two GPUs exist (the source
writes the next rank's region, mapped by CUDA IPC, over NVLink). Every
sequence migrates once; transcripts, RNG states and KV hashes equal the
unmigrated run's."""
import json
import os
import subprocess
import sys

import pytest

from hotseat_b200 import serve_dist

from conftest import gpu_count

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("verify", [False, True])
def test_one_gpu(tiny_gguf, verify):
    eng = serve_dist.GpuEngine(tiny_gguf, 0, 12 + 30 + 8, 12)
    try:
        rec = serve_dist.serve_dist(eng, serve_dist.Solo, 0, 1, per=6, prompt_len=12, steps=30, seed=5, round_tokens=3,
                                    verify=verify, at_range=(14, 30))
    finally:
        eng.close()
    assert rec["migrations"] == 6
    assert rec["transcripts_equal"] and rec["rng_equal"] and rec["kv_hash_equal"], rec


def test_two_ranks_over_nvlink():
    if gpu_count() < 2:
        pytest.skip("needs two GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr",
           "127.0.0.1", "--master-port", "29611", "-m", "hotseat_b200.serve_dist", "--seqs", "8", "--prompt", "64",
           "--steps", "120", "--round-tokens", "4"]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    rec = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1])
    assert rec["migrations"] == 16 and rec["n_gpus"] == 2
    assert rec["transcripts_equal"] and rec["rng_equal"] and rec["kv_hash_equal"], rec
