"""The cross-process serving protocol (hotseat_b200.serve_dist) on CPU ranks:
two and three gloo ranks drive the same rounds, migrations and hand-over
records as the GPU ranks do, with a stand-in engine whose "decode" is a
deterministic function of the sequence's history and whose KV regions are
shared-memory segments that the next rank maps and writes (as the GPU ranks
map each other's regions by CUDA IPC). Every sequence must migrate once and
the migrated run's transcripts, RNG states and KV hashes must equal the
unmigrated run's; a stand-in that drops the RNG on hand-over must be caught."""
import hashlib
import json
import os
import socket
import sys
import time
from multiprocessing import shared_memory

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

REC = 16  # bytes a position writes


class _Kv:
    def __init__(self, n_pos, name=None):
        self.shm = shared_memory.SharedMemory(name=name, create=name is None, size=n_pos * REC)
        self.buf = np.ndarray((n_pos * REC,), dtype=np.uint8, buffer=self.shm.buf)
        if name is None:
            self.buf[:] = 0


class _Mig:
    def __init__(self, src, dst, filled, upper, max_rounds):
        self.src, self.dst, self.max_rounds, self.rounds = src, dst, max_rounds, 0
        self.low = 0
        self._copy(0, upper + 1)
        self.low = filled
        self.sent = (upper + 1) * REC

    def _copy(self, a, b):
        self.dst.buf[a * REC:b * REC] = self.src.buf[a * REC:b * REC]

    def round(self, filled, tokens_now, upper=None):
        upper = filled if upper is None else upper
        self._copy(self.low, upper + 1)
        self.sent += (upper + 1 - self.low) * REC
        self.low = filled
        self.rounds += 1
        return self.rounds < self.max_rounds

    def finish(self, filled, tokens_total):
        self._copy(self.low, filled)
        return {"stw_us": 1.0, "final_bytes": (filled - self.low) * REC, "precopy_bytes": self.sent, "converged": 1}

    def close(self):
        pass


class FakeEngine:
    """Deterministic stand-in: the token after position p is a hash of the
    history and the RNG draw count; position p writes REC bytes of its token."""

    vocab = 1000

    def __init__(self, max_ctx, drop_rng=False):
        self.max_ctx, self.drop_rng, self.kvs = max_ctx, drop_rng, []

    def new_kv(self):
        kv = _Kv(self.max_ctx)
        self.kvs.append(kv)
        return kv

    def export(self, kv):
        return kv.shm.name

    def open_remote(self, name):
        kv = _Kv(self.max_ctx, name)
        self.kvs.append(kv)
        return kv

    def sampler(self, seed):
        return None, {"s": seed, "draws": 0}

    def launch(self, seqs, n_tokens):
        for q in seqs:
            for _ in range(n_tokens):
                if q["done"]:
                    break
                p = q["filled"]
                q["kv"].buf[p * REC:(p + 1) * REC] = np.frombuffer(
                    hashlib.sha256(f"{q['tokens'][p]}@{p}".encode()).digest()[:REC], dtype=np.uint8)
                q["filled"] += 1
                if q["filled"] == len(q["tokens"]):
                    h = hashlib.sha256(f"{q['tokens'][-8:]}|{q['rng']['s']}|{q['rng']['draws']}".encode()).digest()
                    q["rng"]["draws"] += 1
                    if len(q["tokens"]) - q["prompt_len"] >= q["max_tokens"]:
                        q["done"], q["done_reason"] = 1, 2
                    else:
                        q["tokens"].append(int.from_bytes(h[:4], "little") % self.vocab)

    def park(self, seqs):
        pass

    def migration(self, src, dst, filled, tokens_now, max_rounds, verify):
        return _Mig(src, dst, filled, filled, max_rounds)

    def rng_state(self, rng):
        return [rng["s"], rng["draws"]]

    def rng_from(self, state):
        return {"s": state[0] + (1 if self.drop_rng else 0), "draws": state[1]}

    def kv_hash(self, kv, n_pos):
        return hashlib.sha256(bytes(kv.buf[:n_pos * REC])).hexdigest()

    def start_clock(self):
        self._t = time.perf_counter()

    def stop_clock(self):
        return max(1e-6, time.perf_counter() - self._t)

    def close(self):
        for kv in self.kvs:
            kv.shm.close()
            try:
                kv.shm.unlink()
            except FileNotFoundError:
                pass


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_dir, drop_rng):
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    from hotseat_b200 import serve_dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    eng = FakeEngine(max_ctx=6 + 30 + 8, drop_rng=drop_rng)
    try:
        rec = serve_dist.serve_dist(eng, dist, rank, world, per=5, prompt_len=6, steps=30, seed=3, round_tokens=3,
                                    max_rounds=2, at_range=(8, 20))
        dist.barrier()
        if rank == 0:
            with open(os.path.join(out_dir, "rec.json"), "w") as f:
                json.dump(rec, f)
    finally:
        eng.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2, 3])
def test_every_sequence_migrates_and_reproduces_the_unmigrated_run(tmp_path, world):
    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path), False), nprocs=world, start_method="spawn",
                       join=True)
    rec = json.load(open(tmp_path / "rec.json"))
    assert rec["migrations"] == 5 * world and rec["sequences"] == 5 * world
    assert rec["transcripts_equal"] and rec["rng_equal"] and rec["kv_hash_equal"], rec


def test_a_hand_over_that_drops_the_rng_is_caught(tmp_path):
    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path), True), nprocs=2, start_method="spawn", join=True)
    rec = json.load(open(tmp_path / "rec.json"))
    assert rec["migrations"] == 10
    assert not (rec["transcripts_equal"] and rec["rng_equal"])
