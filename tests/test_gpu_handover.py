"""The hand-over data path and the pre-copy migration state machine.

- Run-list staging (hs_kv_read_runs / hs_kv_write_runs: hs-wire
  send_page_bytes / recv_page_bytes, lib.rs:338-396) round-trips random run
  lists, aligned or not, and leaves the bytes outside the runs alone.
- hs_kv_peer_copy is stream-ordered and copies exactly the runs.
- The migration (hs_migrate_*: migrate.rs:234-630) with a pre-copy round
  taken while decode steps are in flight on the batch's stream, then the
  residue after parking: the destination's KV hash equals the source's and
  the sequence continued on the destination equals the unmigrated run
  (tokens, RNG state, final KV hash).
- Host-side failure injection: a destination of another model is refused
  before any byte moves; a byte corrupted on the destination after the
  pre-copy is caught by the verified hand-over's KV-hash check.
"""
import numpy as np
import pytest

import hotseat_b200 as hs

pytestmark = pytest.mark.gpu

TC = hs.NUMERIC_TC


def random_runs(rng, total, n, align):
    cuts = np.sort(rng.choice(np.arange(0, total // align), size=2 * n, replace=False)) * align
    runs = [(int(cuts[2 * i]), int(cuts[2 * i + 1] - cuts[2 * i])) for i in range(n)]
    return [r for r in runs if r[1] > 0]


@pytest.mark.parametrize("align", [1, 4, 16, 512])
def test_run_staging_round_trips(tiny_gguf, align):
    m = hs.Model.load(tiny_gguf, max_ctx=64)
    kv = m.kv()
    rng = np.random.default_rng(align)
    base = rng.integers(0, 256, size=kv.bytes, dtype=np.uint8)
    kv.write(0, base.tobytes())
    runs = random_runs(rng, kv.bytes, 37, align) + [(kv.bytes - 300, 300)]
    runs = sorted(set(runs))
    # non-overlapping: drop any run that overlaps its predecessor
    keep = []
    for r in runs:
        if not keep or r[0] >= keep[-1][0] + keep[-1][1]:
            keep.append(r)
    got = kv.read_runs(keep)
    want = np.concatenate([base[o:o + n] for o, n in keep])
    assert np.array_equal(got, want)
    new = rng.integers(0, 256, size=want.size, dtype=np.uint8)
    kv.write_runs(keep, new.tobytes())
    after = kv.read(0, kv.bytes)
    expect = base.copy()
    at = 0
    for o, n in keep:
        expect[o:o + n] = new[at:at + n]
        at += n
    assert np.array_equal(after, expect)


def test_peer_copy_is_stream_ordered_and_exact(tiny_gguf):
    import torch
    m = hs.Model.load(tiny_gguf, max_ctx=64)
    a, b = m.kv(), m.kv()
    rng = np.random.default_rng(3)
    src = rng.integers(0, 256, size=a.bytes, dtype=np.uint8)
    a.write(0, src.tobytes())
    runs = [(0, 4096), (5000, 1000), (a.bytes - 16, 16), (70000, 3)]
    s = torch.cuda.Stream()
    a.peer_copy(b, runs, stream=s.cuda_stream)
    s.synchronize()
    got = b.read(0, b.bytes)
    expect = np.zeros(b.bytes, dtype=np.uint8)
    for o, n in runs:
        expect[o:o + n] = src[o:o + n]
    assert np.array_equal(got, expect)


def test_bad_runs_are_refused(tiny_gguf):
    m = hs.Model.load(tiny_gguf, max_ctx=64)
    kv = m.kv()
    with pytest.raises(hs.HotseatError) as e:
        kv.read_runs([(kv.bytes - 8, 16)])
    assert e.value.code == hs.HS_E_ARG
    with pytest.raises(hs.HotseatError):
        kv.write_runs([(0, 100)], b"x" * 50)


def _seq(prompt, max_tokens, seed, **kw):
    return dict(tokens=list(prompt), prompt_len=len(prompt), max_tokens=max_tokens,
                cfg=hs.SamplerCfg.default(temperature=0.8, seed=seed), rng=hs.Rng.seed(seed), **kw)


def _copy_rng(r):
    c = hs.Rng()
    c.s[:] = list(r.s)
    c.draws = r.draws
    return c


@pytest.mark.parametrize("verify", [True, False])
def test_migration_with_a_round_during_decode_equals_the_unmigrated_run(tiny_gguf, verify):
    m = hs.Model.load(tiny_gguf, max_ctx=128, numeric=TC)
    prompt = [int(t) for t in np.random.default_rng(21).integers(0, 1000, size=20)]
    ref_kv = m.kv()
    ref = hs.Batch(m, 1).run_seqs([ref_kv], [_seq(prompt, 60, 7)])[0]
    src, dst = m.kv(), m.kv()
    b = hs.Batch(m, 1)
    toks, st, rng = b.run_seqs([src], [_seq(prompt, 60, 7)], stop_at_filled=30)[0]
    assert st.filled == 30
    mig = hs.Migration(src, dst, filled=30, tokens_now=len(toks), verify=verify)
    # ten more steps in flight on the batch's stream while a round harvests
    # and copies on the region's stream
    q = dict(tokens=[int(t) for t in toks], prompt_len=len(prompt), max_tokens=60, cfg=_seq(prompt, 60, 7)["cfg"],
             rng=_copy_rng(rng), filled=st.filled, done=st.done, done_reason=st.done_reason)
    b.begin([src], [q], stop_at_filled=40)
    b.step(10)
    more = mig.round(filled=30, tokens_now=len(toks), upper=40)
    toks, st, rng = b.end()[0]  # parked at 40
    assert st.filled == 40
    if more:
        mig.round(filled=40, tokens_now=len(toks))
    rep = mig.finish(filled=40, tokens_total=len(toks), park_us=0.0)
    assert rep["filled"] == 40 and rep["rounds"][0]["bytes"] > 0 and rep["verified"] == int(verify)
    if verify:
        assert rep["kv_hash_src"] == rep["kv_hash_dst"] == src.hash(40)
    assert dst.hash(40) == src.hash(40)
    # the sequence continues on the destination
    q = dict(tokens=[int(t) for t in toks], prompt_len=len(prompt), max_tokens=60, cfg=_seq(prompt, 60, 7)["cfg"],
             rng=_copy_rng(rng), filled=st.filled, done=st.done, done_reason=st.done_reason)
    fin = hs.Batch(m, 1).run_seqs([dst], [q])[0]
    assert list(fin[0]) == list(ref[0])
    assert list(fin[2].s) == list(ref[2].s) and fin[2].draws == ref[2].draws
    assert dst.hash(fin[1].filled) == ref_kv.hash(ref[1].filled)


def test_destination_of_another_model_is_refused_before_any_byte_moves(tiny_gguf):
    a = hs.Model.load(tiny_gguf, max_ctx=64, numeric=TC)
    f = hs.Model.load(tiny_gguf, max_ctx=64, numeric=hs.NUMERIC_FAST)
    src, dst = a.kv(), f.kv()
    src.write(0, np.full(src.bytes, 7, dtype=np.uint8).tobytes())
    with pytest.raises(hs.HotseatError) as e:
        hs.Migration(src, dst, filled=10, tokens_now=11)
    assert e.value.code == hs.HS_E_STATE and "fingerprint" in str(e.value)
    assert not np.any(dst.read(0, dst.bytes))
    other = hs.Model.load(tiny_gguf, max_ctx=32, numeric=TC)  # another KV spec
    with pytest.raises(hs.HotseatError) as e:
        hs.Migration(src, other.kv(), filled=10, tokens_now=11)
    assert e.value.code == hs.HS_E_STATE


def test_corrupted_byte_is_caught_by_the_verified_hand_over(tiny_gguf):
    m = hs.Model.load(tiny_gguf, max_ctx=64, numeric=TC)
    prompt = [int(t) for t in np.random.default_rng(4).integers(0, 1000, size=16)]
    src, dst = m.kv(), m.kv()
    toks, st, _ = hs.Batch(m, 1).run_seqs([src], [_seq(prompt, 30, 3)], stop_at_filled=24)[0]
    mig = hs.Migration(src, dst, filled=24, tokens_now=len(toks), verify=True)
    # one byte of a live position flipped on the destination side of the link
    row = dst.read(1000, 4)
    dst.write(1000, bytes([row[0] ^ 0x40]) + bytes(row[1:]))
    with pytest.raises(hs.HotseatError) as e:
        mig.finish(filled=24, tokens_total=len(toks))
    assert e.value.code == hs.HS_E_STATE and "differs" in str(e.value)
    assert mig.report["kv_hash_src"] != mig.report["kv_hash_dst"]
