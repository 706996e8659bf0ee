"""Data-parallel batched decode with every sequence live-migrated mid-run
(hotseat_b200.serve, the 8-GPU serving configuration at small sizes): on one
GPU the destination is a second KV region, on two GPUs the other GPU over
NVLink. Migrated transcripts, RNG states and KV hashes must equal the
unmigrated run's."""
import pytest

from hotseat_b200 import serve

from conftest import gpu_count

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n_gpus,round_tokens,verify", [(1, 1, True), (1, 3, False), (2, 1, False), (2, 3, True)])
def test_every_sequence_migrates_and_reproduces_its_transcript(tiny_gguf, n_gpus, round_tokens, verify):
    if gpu_count() < n_gpus:
        pytest.skip("needs two GPUs")
    rec = serve.serve(tiny_gguf, n_gpus, per_gpu=6, prompt=12, steps=30, seed=3, at_range=(14, 30),
                      round_tokens=round_tokens, verify=verify)
    assert rec["migrations"] == 6 * n_gpus
    assert rec["transcripts_equal"] and rec["rng_equal"] and rec["kv_hash_equal"], rec
    by_round = rec["bytes_per_migration_by_round"]
    assert by_round["0"] > 0 and "final" in by_round
    assert rec["stw_us"]["p50"] is not None and rec["stw_us"]["p50"] > 0
