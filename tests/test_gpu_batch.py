"""The tensor-core batched path (HS_NUMERIC_TC) against the CPU restatement.

Every matrix product runs as a tcgen05 GEMM over all sequences of the batch,
with activations carried as f16 hi/lo pairs. The bar is the token loop's:
logits and KV rows within 1e-2 max-abs of the CPU path, identical greedy
tokens, and the same bits for a sequence whatever batch it runs in (alone,
in another slot, in a batch of more than 64), so batched transcripts equal
single ones and a migration reproduces the unmigrated run."""
import numpy as np
import pytest

import hotseat_b200 as hs
from tests.golden.synth import QWEN05
from oracle import ffi

from conftest import TINY, TINY128

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2
TC = hs.NUMERIC_TC


def load(path, max_ctx):
    return hs.Model.load(path, max_ctx=max_ctx, numeric=TC)


def seq(tokens, max_tokens, cfg, seed, **kw):
    return dict(tokens=list(tokens), prompt_len=len(tokens), max_tokens=max_tokens, cfg=cfg, rng=hs.Rng.seed(seed),
                **kw)


@pytest.mark.parametrize("which", ["tiny", "tiny128", "q05"])
def test_tc_logits_within_tolerance(which, tiny_gguf, tiny128_gguf, q05_gguf):
    path, vocab, n_pos = {"tiny": (tiny_gguf, TINY["vocab"], 40), "tiny128": (tiny128_gguf, TINY128["vocab"], 24),
                          "q05": (q05_gguf, QWEN05["vocab"], 6)}[which]
    rng = np.random.default_rng(2)
    toks = [int(t) for t in rng.integers(0, vocab, size=n_pos)]
    m = load(path, 64)
    b = hs.Batch(m, 1)
    o = ffi.Model(path, max_ctx=64)
    kv, okv = m.kv(), o.new_kv()
    worst = 0.0
    for pos, tok in enumerate(toks):
        b.forward([kv], [tok], [pos])
        got, want = b.logits(0), o.forward(okv, tok, pos)
        err = float(np.max(np.abs(got - want)))
        worst = max(worst, err)
        assert err <= LOGIT_TOL, (pos, err)
    kv_err = float(np.max(np.abs(kv.floats() - okv)))
    assert kv_err <= LOGIT_TOL
    print(f"{which}: worst logit error {worst:.3g}, KV {kv_err:.3g}")


def test_tc_model_has_its_own_fingerprint_and_refuses_the_single_scratch(tiny_gguf):
    a = hs.Model.load(tiny_gguf, max_ctx=16)
    f = hs.Model.load(tiny_gguf, max_ctx=16, numeric=hs.NUMERIC_FAST)
    t = load(tiny_gguf, 16)
    assert len({a.fingerprint, f.fingerprint, t.fingerprint}) == 3 and t.cfg.numeric == TC
    with pytest.raises(hs.HotseatError) as e:
        t.scratch()
    assert e.value.code == hs.HS_E_UNSUPPORTED
    with pytest.raises(hs.HotseatError):
        hs.Batch(a, 4)


@pytest.mark.parametrize("n, slot", [(7, 5), (70, 66)])
def test_tc_results_do_not_depend_on_the_batch(tiny_gguf, n, slot):
    """A sequence alone and the same sequence in slot `slot` of an n-sequence
    batch (other slots random) give bit-identical logits and KV bytes."""
    m = load(tiny_gguf, 64)
    b1, bn = hs.Batch(m, 1), hs.Batch(m, n)
    g = np.random.default_rng(9)
    seq_a = [int(t) for t in g.integers(0, TINY["vocab"], size=20)]
    kv_a = m.kv()
    kvs = [m.kv() for _ in range(n)]
    for pos in range(20):
        b1.forward([kv_a], [seq_a[pos]], [pos])
        toks = [int(t) for t in g.integers(0, TINY["vocab"], size=n)]
        toks[slot] = seq_a[pos]
        bn.forward(kvs, toks, [pos] * n)
        assert np.array_equal(bn.logits(slot), b1.logits(0)), pos
    assert kv_a.hash(20) == kvs[slot].hash(20)


def test_tc_greedy_tokens_match_the_oracle(q05_gguf):
    """Four greedy sequences (temperature 0, penalty 1.1) of the 0.5B shape
    decoded together; each must pick the CPU path's token at every step."""
    g = np.random.default_rng(36)
    prompts = [[int(t) for t in g.integers(0, QWEN05["vocab"], size=12 + 4 * i)] for i in range(4)]
    cfg = hs.SamplerCfg.default(temperature=0.0)
    m = load(q05_gguf, 256)
    b = hs.Batch(m, 4)
    kvs = [m.kv() for _ in prompts]
    got = b.run_seqs(kvs, [seq(p, 24, cfg, 1) for p in prompts])
    o = ffi.Model(q05_gguf, max_ctx=256)
    for i, p in enumerate(prompts):
        want, _, _ = o.run_seq(o.new_kv(), p, 24, ffi.default_cfg(temperature=0.0), ffi.seeded_rng(1))
        assert list(got[i][0]) == list(want), i


def test_tc_sampled_c1_transcript_matches_the_oracle(q05_gguf):
    rng = np.random.default_rng(36)
    prompt = [int(t) for t in rng.integers(0, QWEN05["vocab"], size=36)]
    cfg = hs.SamplerCfg.default(temperature=0.8, seed=99)
    m = load(q05_gguf, 2048)
    b = hs.Batch(m, 1)
    toks, st, r = b.run_seqs([m.kv()], [seq(prompt, 120, cfg, 99)])[0]
    o = ffi.Model(q05_gguf, max_ctx=2048)
    want, ost, orng = o.run_seq(o.new_kv(), prompt, 120, ffi.default_cfg(temperature=0.8, seed=99),
                                ffi.seeded_rng(99))
    assert list(toks) == list(want)
    assert list(r.s) == list(orng.s) and r.draws == orng.draws == 121


def test_tc_batched_transcripts_equal_single_runs(tiny_gguf):
    """Six sequences with different prompts, lengths, budgets, temperatures
    and seeds, run together, equal each one run alone: tokens, SeqState, RNG
    and KV hash."""
    m = load(tiny_gguf, 96)
    g = np.random.default_rng(4)
    seqs = []
    for i in range(6):
        cfg = hs.SamplerCfg.default(temperature=0.0 if i % 3 == 0 else 0.7 + 0.1 * i, top_k=40)
        p = [int(t) for t in g.integers(0, TINY["vocab"], size=5 + 3 * i)]
        seqs.append(seq(p, 10 + 7 * i, cfg, 100 + i))
    kvs = [m.kv() for _ in seqs]
    together = hs.Batch(m, len(seqs)).run_seqs(kvs, seqs)
    for i, q in enumerate(seqs):
        q2 = dict(q, rng=hs.Rng.seed(100 + i))
        kv1 = m.kv()
        alone = hs.Batch(m, 1).run_seqs([kv1], [q2])[0]
        assert list(together[i][0]) == list(alone[0]), i
        assert together[i][1].filled == alone[1].filled and together[i][1].done_reason == alone[1].done_reason
        assert list(together[i][2].s) == list(alone[2].s)
        assert kvs[i].hash(together[i][1].filled) == kv1.hash(alone[1].filled)


def test_tc_batch_of_more_than_1024_sequences_equals_single_runs(tiny_gguf):
    """1,100 sequences in one batch (a capacity of 1,152 slots: 18 groups of
    64): sampled transcripts, RNG and KV hashes of the first, a middle and the
    last sequence equal each one run alone."""
    m = load(tiny_gguf, 32)
    g = np.random.default_rng(11)
    n = 1100
    seqs = [seq([int(t) for t in g.integers(0, TINY["vocab"], size=4 + i % 5)], 6,
                hs.SamplerCfg.default(temperature=0.8, top_k=40), 500 + i) for i in range(n)]
    kvs = [m.kv() for _ in range(n)]
    together = hs.Batch(m, n).run_seqs(kvs, seqs)
    for i in (0, 517, n - 1):
        q2 = dict(seqs[i], rng=hs.Rng.seed(500 + i))
        kv1 = m.kv()
        alone = hs.Batch(m, 1).run_seqs([kv1], [q2])[0]
        assert list(together[i][0]) == list(alone[0]), i
        assert list(together[i][2].s) == list(alone[2].s)
        assert kvs[i].hash(together[i][1].filled) == kv1.hash(alone[1].filled)
    for kv in kvs:
        kv.close()


def test_tc_batch_marks_exactly_the_written_pages(tiny_gguf):
    m = load(tiny_gguf, 96)
    b = hs.Batch(m, 3)
    for layout in (0, 1):
        kvs = [m.kv(layout, page_size=1024) for _ in range(3)]
        for kv in kvs:
            kv.arm()
        b.forward(kvs, [3, 4, 5], [0, 0, 0])
        for kv in kvs:
            kv.harvest()
        for pos in (1, 17, 40):
            b.forward(kvs, [3, 4, 5], [pos, pos + 1, pos + 2])
            for i, kv in enumerate(kvs):
                w = kv.harvest()
                got = {j for j in range(kv.n_pages) if (int(w[j // 64]) >> (j % 64)) & 1}
                want = set()
                for off, nb in ffi.written_ranges(ffi.kv_spec(m.cfg.n_layers, m.cfg.n_kv_heads, m.cfg.head_dim,
                                                              m.cfg.max_ctx, layout), pos + i):
                    want.update(range(off // 1024, (off + nb - 1) // 1024 + 1))
                assert got == want, (layout, pos, i)


def test_tc_migration_between_batches_reproduces_the_transcript(tiny_gguf):
    """Sequence 0 of a 3-sequence batch stops at filled=18; its KV bytes move
    by dirty-page pre-copy rounds to a fresh region, and it finishes there in
    a different batch (slot 1 of 2). Tokens and KV hash equal the unmigrated
    run."""
    m = load(tiny_gguf, 96)
    g = np.random.default_rng(8)
    cfg = hs.SamplerCfg.default()
    prompts = [[int(t) for t in g.integers(0, TINY["vocab"], size=12)] for _ in range(3)]
    ref = hs.Batch(m, 1).run_seqs([m.kv()], [seq(prompts[0], 40, cfg, 8)])[0]

    spec = m.kv_spec(0)
    src = [m.kv() for _ in range(3)]
    dst = m.kv()
    b3 = hs.Batch(m, 3)
    part = b3.run_seqs(src, [seq(p, 40, cfg, 8 + i) for i, p in enumerate(prompts)], stop_at_filled=10)
    src[0].arm()
    all_pages = np.full(src[0].n_words, ~np.uint64(0), dtype=np.uint64)
    runs = hs.runs_to_byte_runs(all_pages, src[0].n_pages, src[0].page_size, hs.live_ranges_between(spec, 0, 11))
    src[0].copy_runs_to(dst, runs)
    # source keeps decoding to 18 while armed, then the residue moves
    state = [dict(tokens=list(t), prompt_len=12, max_tokens=40, cfg=cfg, rng=r, filled=s.filled)
             for t, s, r in part]
    part2 = b3.run_seqs(src, state, stop_at_filled=18)
    dirty = src[0].harvest()
    runs = hs.runs_to_byte_runs(dirty, src[0].n_pages, src[0].page_size, hs.live_ranges_between(spec, 10, 18))
    src[0].copy_runs_to(dst, runs)
    src[0].disarm()
    toks, st, r = part2[0]
    assert src[0].hash(st.filled) == dst.hash(st.filled)
    other = m.kv()
    b2 = hs.Batch(m, 2)
    fin = b2.run_seqs([other, dst], [seq(prompts[1][:5], 6, cfg, 77),
                                     dict(tokens=list(toks), prompt_len=12, max_tokens=40, cfg=cfg, rng=r,
                                          filled=st.filled)])
    assert list(fin[1][0]) == list(ref[0])
    kv_ref = m.kv()
    hs.Batch(m, 1).run_seqs([kv_ref], [seq(prompts[0], 40, cfg, 8)])
    assert dst.hash(fin[1][1].filled) == kv_ref.hash(fin[1][1].filled)


@pytest.mark.parametrize("env", [{"HS_ATTN_HEAD_SPLIT": "2"}, {"HS_ATTN_HEAD_SPLIT": "3", "HS_ATTN_NBUF": "2"},
                                 {"HS_ATTN_NBUF": "3"}, {"HS_ATTN_HEAD_SPLIT": "7"}])
def test_tc_attention_work_split_keeps_the_bits(env, q05_gguf, monkeypatch):
    """Splitting a (split, KV head) item's query heads over several CTAs, or
    changing how many K/V chunks load ahead, leaves every head's arithmetic
    as it was: transcripts, RNG and KV hashes equal the default launch's.
    (At head_dim 64 the default is the tensor-core warp-split form, which
    stages its own blocks: the chunk-buffer count does not reach it.)"""
    def run():
        m = load(q05_gguf, 256)
        g = np.random.default_rng(12)
        seqs = [seq([int(t) for t in g.integers(0, QWEN05["vocab"], size=70 + 9 * i)], 24,
                    hs.SamplerCfg.default(temperature=0.8, seed=5 + i), 5 + i) for i in range(3)]
        kvs = [m.kv() for _ in seqs]
        out = hs.Batch(m, len(seqs)).run_seqs(kvs, seqs)
        return [(list(t), list(r.s), kv.hash(st.filled)) for (t, st, r), kv in zip(out, kvs)]

    ref = run()
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    assert run() == ref
