"""The reference's own known-answer tests, run against the CPU restatement.

Each test restates one #[test] of hotseat (file:line in crates/...), with the
same inputs and expected values, so the oracle is pinned to the reference's
published behaviour before anything is compared against it.
"""
import ctypes as C
import math
import struct

import numpy as np
import pytest

from oracle import ffi

L = ffi.lib()


def h2f(h):
    return L.hso_f16_to_f32(h)


def f2h(f):
    return L.hso_f32_to_f16(f)


# ---- hs-engine/src/f16.rs:75-104 -------------------------------------------

def test_f16_round_trip_exact_values():
    for v in [0.0, -0.0, 1.0, -1.0, 0.5, 2.0, 65504.0, -65504.0, 6.1035156e-5]:
        got = h2f(f2h(v))
        assert got == np.float32(v)
        assert math.copysign(1, got) == math.copysign(1, v)


def test_f16_saturates_and_underflows():
    assert f2h(1.0e30) & 0x7FFF == 0x7C00
    assert f2h(-1.0e30) == 0xFC00
    assert f2h(1.0e-30) == 0x0000
    assert math.isnan(h2f(f2h(float("nan"))))


def test_f16_subnormals_survive_the_round_trip():
    for k in range(1, 16):
        assert f2h(h2f(k)) == k


def test_f16_rounds_to_nearest_even():
    assert h2f(f2h(2049.0)) == 2048.0
    assert h2f(f2h(2051.0)) == 2052.0


def test_f16_matches_numpy_everywhere():
    # Independent check: numpy's IEEE half conversion, every f16 pattern, and
    # a sweep of f32 values including ties, subnormals and overflow.
    hs = np.arange(65536, dtype=np.uint16)
    ours = np.array([h2f(int(h)) for h in hs[::7]], dtype=np.float32)
    ref = hs[::7].view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(ours[~nan].view(np.uint32), ref[~nan].view(np.uint32))
    rng = np.random.default_rng(3)
    fs = np.concatenate([rng.standard_normal(4000).astype(np.float32) * s for s in (1e-7, 1e-5, 1e-2, 1, 1e4, 7e4)])
    ties = (np.arange(1, 2000, dtype=np.float32) + 0.5) * np.float32(2.0 ** -24)
    fs = np.concatenate([fs, ties, -ties])
    ours = np.array([f2h(float(f)) for f in fs], dtype=np.uint16)
    assert np.array_equal(ours, fs.astype(np.float16).view(np.uint16))


# ---- hs-engine/src/math.rs:301-364 (math.rs test module) -------------------

def lcg_vectors(n):
    w = np.zeros(n, dtype=np.uint16)
    x = np.zeros(n, dtype=np.float32)
    s = 0x12345678
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        a = np.float32(s >> 8) / np.float32(8388608.0) - np.float32(1.0)
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        b = np.float32(s >> 8) / np.float32(8388608.0) - np.float32(1.0)
        w[i] = f2h(float(a))
        x[i] = b
    return w, x


def eight_lane_dot(w, x):
    """numpy float32 restatement of dot_f16_scalar's accumulation shape."""
    wf = w.view(np.float16).astype(np.float32).reshape(-1, 8)
    xf = x.reshape(-1, 8)
    acc = np.zeros(8, dtype=np.float32)
    for j in range(wf.shape[0]):
        acc = acc + wf[j] * xf[j]  # elementwise f32 mul then add, no FMA
    l = (acc[0] + acc[1]) + (acc[2] + acc[3])
    r = (acc[4] + acc[5]) + (acc[6] + acc[7])
    return np.float32(l + r)


def test_dot_matches_an_independent_eight_lane_restatement():
    # math.rs:306-325 uses this vector pair to tie the NEON dot to the scalar
    # one; here it ties the oracle's dot to a numpy restatement, bit for bit.
    w, x = lcg_vectors(8960)
    got = np.float32(L.hso_dot_f16(ffi.ptr(w), ffi.ptr(x), len(w)))
    assert got.view(np.uint32) == eight_lane_dot(w, x).view(np.uint32)


def test_exp_is_accurate():
    for x in [0.0, 1.0, -1.0, 0.5, -12.25, 30.0, -30.0, 80.0, 88.5, -95.0, 1e-8]:
        ours = L.hso_exp_f32(x)
        libm = np.float32(math.exp(np.float32(x)))
        if libm == 0.0 or not np.isfinite(libm):
            continue
        assert abs((ours - libm) / libm) < 2e-7, x
    assert L.hso_exp_f32(0.0) == 1.0
    assert math.isinf(L.hso_exp_f32(1000.0))
    assert L.hso_exp_f32(-1000.0) == 0.0


def test_ln_is_accurate():
    for x in [1.0, 2.0, 0.5, 10000.0, 1e-6, 1.0e6, 1.414, 0.708]:
        assert abs(L.hso_ln_f32(x) - np.float32(math.log(np.float32(x)))) < 1e-5, x


def test_sincos_is_accurate_at_large_arguments():
    for x in [0.0, 0.3, 1.7, -2.5, 100.0, 5000.0, 31999.0]:
        s, c = C.c_float(), C.c_float()
        L.hso_sincos_f32(x, C.byref(s), C.byref(c))
        xf = float(np.float32(x))
        assert abs(s.value - math.sin(xf)) < 3e-5, x
        assert abs(c.value - math.cos(xf)) < 3e-5, x


def test_softmax_sums_to_one():
    v = np.array([1.0, 2.0, 3.0, -40.0, 0.0, 12.5, -1.0, 7.0], dtype=np.float32)
    L.hso_softmax(ffi.ptr(v), len(v))
    assert abs(float(v.sum()) - 1.0) < 1e-6
    assert (v >= 0).all()


# ---- hs-engine/src/quant.rs:212-306 -----------------------------------------

def half_bytes(f):
    return struct.pack("<H", f2h(f))


def test_q8_0_round_trips_a_known_block():
    blk = bytearray(34)
    blk[0:2] = half_bytes(0.5)
    for l in range(32):
        blk[2 + l] = (l - 16) & 0xFF
    out = ffi.dequant_f16(8, blk, 32)
    for l in range(32):
        assert h2f(int(out[l])) == 0.5 * (l - 16)


def test_q4_k_scale_min_unpacking_matches_reference():
    q = np.array([0b11_000001, 0b10_000010, 0b01_000011, 0b00_000100, 0x55, 0x66, 0x77, 0x88, 0x9A, 0xBC, 0xDE,
                  0xF0], dtype=np.uint8)

    def sm(j):
        v = L.hso_scale_min_k4(j, ffi.ptr(q))
        return (v >> 8, v & 0xFF)

    assert sm(0) == (1, 0x55 & 63)
    assert sm(3) == (4, 0x88 & 63)
    assert sm(4) == ((0x9A & 0x0F) | (0b11 << 4), (0x9A >> 4) | ((0x55 >> 6) << 4))
    assert sm(7) == ((0xF0 & 0x0F) | (0b00 << 4), (0xF0 >> 4) | ((0x88 >> 6) << 4))


def test_q4_k_block_is_affine_in_the_nibble():
    blk = bytearray(144)
    blk[0:2] = half_bytes(1.0)
    blk[2:4] = half_bytes(0.0)
    blk[4] = 3
    for l in range(128):
        blk[16 + l] = 0x21
    out = ffi.dequant_f16(12, blk, 256)
    assert h2f(int(out[0])) == 3.0
    assert h2f(int(out[31])) == 3.0
    assert h2f(int(out[32])) == 0.0
    assert h2f(int(out[64])) == 0.0


def test_q5_0_interleaves_its_halves_and_uses_the_fifth_bit():
    blk = bytearray(22)
    blk[0:2] = half_bytes(1.0)
    blk[2] = 0b0000_0001
    blk[4] = 0b0000_0001
    for j in range(16):
        blk[6 + j] = 0x10
    out = ffi.dequant_f16(6, blk, 32)
    assert h2f(int(out[0])) == 0 + 16 - 16
    assert h2f(int(out[1])) == 0 - 16
    assert h2f(int(out[16])) == 1 + 16 - 16
    assert h2f(int(out[17])) == 1 - 16


def test_q5_k_adds_sixteen_when_the_high_bit_is_set():
    blk = bytearray(176)
    blk[0:2] = half_bytes(1.0)
    blk[2:4] = half_bytes(0.0)
    blk[4] = 1
    blk[16] = 0b0000_0001
    for l in range(128):
        blk[48 + l] = 0x03
    out = ffi.dequant_f16(13, blk, 256)
    assert h2f(int(out[0])) == 19.0
    assert h2f(int(out[1])) == 3.0


def test_q6_k_centres_on_zero():
    blk = bytearray(210)
    for i in range(16):
        blk[192 + i] = 1
    blk[208:210] = half_bytes(0.25)
    out = ffi.dequant_f16(14, blk, 256)
    assert all(h2f(int(v)) == -8.0 for v in out)


# ---- hs-engine/src/hash.rs:132-176 ------------------------------------------

def test_fnv_matches_published_vectors():
    assert ffi.fnv1a(b"") == 0xCBF29CE484222325
    assert ffi.fnv1a(b"a") == 0xAF63DC4C8601EC8C
    assert ffi.fnv1a(b"foobar") == 0x85944171F73967E8


def test_wide_hash_detects_single_bit_flips():
    data = bytearray((i * 31) & 0xFF for i in range(100_000))
    a = ffi.wide(data)
    for at in [0, 1, 7, 8, 31, 32, 99_999]:
        data[at] ^= 1
        assert ffi.wide(data) != a, at
        data[at] ^= 1
    assert ffi.wide(data) == a


def test_wide_hash_is_length_sensitive():
    assert ffi.wide(bytes(64)) != ffi.wide(bytes(96))
    assert ffi.wide(b"") != ffi.wide(b"\0")


def test_wide_streaming_matches_one_shot_on_aligned_chunks():
    # Kv::hash streams over live ranges; each TokenMajor range is a multiple
    # of 32 bytes, so hashing range by range equals hashing their concatenation.
    spec = ffi.kv_spec(3, 2, 8, 16, 0)
    kv = np.arange(3 * 2 * 16 * 2 * 8, dtype=np.float32) * 0.5
    ranges = ffi.live_ranges_between(spec, 0, 10)
    raw = kv.view(np.uint8)
    cat = b"".join(bytes(raw[o:o + n]) for o, n in ranges)
    assert all(n % 32 == 0 for _, n in ranges)
    assert ffi.kv_hash(spec, kv, 10) == ffi.wide(cat)


# ---- hs-engine/src/sampler.rs:193-284 ---------------------------------------

def test_rng_matches_the_reference_stream():
    r = ffi.Rng()
    r.s[:] = [1, 2, 3, 4]
    got = [L.hso_rng_next_u64(C.byref(r)) for _ in range(5)]
    assert got == [11520, 0, 1509978240, 1215971899390074240, 1216172134540287360]
    assert r.draws == 5


def test_rng_state_fully_determines_the_future():
    a = ffi.seeded_rng(42)
    for _ in range(1000):
        L.hso_rng_next_u64(C.byref(a))
    snap = ffi.Rng()
    C.memmove(C.byref(snap), C.byref(a), C.sizeof(a))
    want = [L.hso_rng_next_u64(C.byref(a)) for _ in range(50)]
    got = [L.hso_rng_next_u64(C.byref(snap)) for _ in range(50)]
    assert want == got and list(a.s) == list(snap.s)


def test_next_f32_stays_in_range():
    r = ffi.seeded_rng(7)
    for _ in range(100_000):
        v = L.hso_rng_next_f32(C.byref(r))
        assert 0.0 <= v < 1.0


def test_greedy_sampling_ignores_the_rng():
    cfg = ffi.default_cfg(temperature=0.0)
    r = ffi.seeded_rng(cfg.seed)
    l = np.array([0.1, 5.0, -3.0, 4.9], dtype=np.float32)
    assert L.hso_sample(C.byref(cfg), C.byref(r), ffi.ptr(l), 4, None, 0) == 1
    assert r.draws == 0


def test_top_k_one_is_greedy_even_with_temperature():
    cfg = ffi.default_cfg(temperature=2.0, top_k=1, top_p=1.0, repeat_penalty=1.0)
    r = ffi.seeded_rng(cfg.seed)
    for _ in range(100):
        l = np.array([0.1, 5.0, -3.0, 4.9], dtype=np.float32)
        assert L.hso_sample(C.byref(cfg), C.byref(r), ffi.ptr(l), 4, None, 0) == 1


def test_same_state_gives_the_same_token():
    cfg = ffi.default_cfg(temperature=1.0, top_k=0, top_p=1.0, repeat_penalty=1.0)
    logits = np.array([((i * 37 % 91) / 13.0) for i in range(512)], dtype=np.float32)
    a = ffi.seeded_rng(cfg.seed)
    for _ in range(20):
        L.hso_sample(C.byref(cfg), C.byref(a), ffi.ptr(logits.copy()), 512, None, 0)
    b = ffi.Rng()
    C.memmove(C.byref(b), C.byref(a), C.sizeof(a))
    x = L.hso_sample(C.byref(cfg), C.byref(a), ffi.ptr(logits.copy()), 512, None, 0)
    y = L.hso_sample(C.byref(cfg), C.byref(b), ffi.ptr(logits.copy()), 512, None, 0)
    assert x == y


def test_repetition_penalty_pushes_logits_down():
    cfg = ffi.default_cfg(temperature=0.0, repeat_penalty=2.0, repeat_last_n=8)
    r = ffi.seeded_rng(cfg.seed)
    h = np.array([1], dtype=np.uint32)
    l = np.array([0.0, 10.0, 9.0, 0.0], dtype=np.float32)
    assert L.hso_sample(C.byref(cfg), C.byref(r), ffi.ptr(l), 4, ffi.ptr(h), 1) == 2
    l2 = np.array([0.0, -1.0, -2.0, 0.0], dtype=np.float32)
    L.hso_sample(C.byref(cfg), C.byref(r), ffi.ptr(l2), 4, ffi.ptr(h), 1)
    assert l2[1] == -2.0


# ---- hs-engine/src/kv.rs:281-422 --------------------------------------------

def spec(layout):
    return ffi.kv_spec(3, 2, 8, 16, layout)


@pytest.mark.parametrize("layout", [0, 1])
def test_kv_rows_are_disjoint_and_in_bounds(layout):
    s = spec(layout)
    floats = 3 * 2 * 16 * 2 * 8
    seen = np.zeros(floats, dtype=np.int64)
    tag = 0
    for l in range(3):
        for p in range(16):
            for h in range(2):
                for is_v in (0, 1):
                    tag += 1
                    off = L.hso_kv_row_off(C.byref(s), l, is_v, p, h)
                    assert (seen[off:off + 8] == 0).all()
                    seen[off:off + 8] = tag
    assert (seen != 0).all()


@pytest.mark.parametrize("layout", [0, 1])
def test_kv_written_ranges_cover_exactly_the_step(layout):
    s = spec(layout)
    mem = np.zeros(3 * 2 * 16 * 2 * 8, dtype=np.float32)
    pos = 5
    for l in range(3):
        for h in range(2):
            for is_v in (0, 1):
                off = L.hso_kv_row_off(C.byref(s), l, is_v, pos, h)
                mem[off:off + 8] = 1.0
    ranges = ffi.written_ranges(s, pos)
    covered = np.zeros_like(mem, dtype=bool)
    for off, n in ranges:
        covered[off // 4: off // 4 + n // 4] = True
    assert sum(n // 4 for _, n in ranges) == int((mem != 0).sum())
    assert np.array_equal(mem != 0, covered)


@pytest.mark.parametrize("layout", [0, 1])
def test_kv_live_ranges_cover_every_written_position(layout):
    s = spec(layout)
    mem = np.zeros(3 * 2 * 16 * 2 * 8, dtype=np.float32)
    for p in range(7):
        for l in range(3):
            for h in range(2):
                for is_v in (0, 1):
                    off = L.hso_kv_row_off(C.byref(s), l, is_v, p, h)
                    mem[off:off + 8] = p + 1.0
    covered = np.zeros_like(mem, dtype=bool)
    for off, n in ffi.live_ranges_between(s, 0, 7):
        covered[off // 4: off // 4 + n // 4] = True
    assert covered[mem != 0].all()


@pytest.mark.parametrize("layout", [0, 1])
def test_kv_live_ranges_between_is_a_suffix_of_live_ranges(layout):
    s = spec(layout)
    full = ffi.live_ranges_between(s, 0, 10)
    head = ffi.live_ranges_between(s, 0, 4)
    tail = ffi.live_ranges_between(s, 4, 10)
    assert len(full) == len(head) == len(tail)
    for f, h, t in zip(full, head, tail):
        assert h[0] == f[0] and h[0] + h[1] == t[0] and t[0] + t[1] == f[0] + f[1]


def test_kv_empty_and_degenerate_intervals_are_empty():
    s = spec(0)
    assert ffi.live_ranges_between(s, 5, 5) == []
    assert ffi.live_ranges_between(s, 9, 3) == []
    assert ffi.live_ranges_between(s, 0, 0) == []


def test_token_major_dirties_fewer_pages_per_step():
    page = 16384

    def pages(layout):
        s = ffi.kv_spec(28, 2, 128, 2048, layout)
        out = set()
        for off, n in ffi.written_ranges(s, 1000):
            out.update(range(off // page, (off + n - 1) // page + 1))
        return len(out)

    assert pages(0) < pages(1)


# ---- hs-engine/src/pool.rs:202-218 ------------------------------------------

def test_pool_ranges_tile_exactly():
    a, b = C.c_size_t(), C.c_size_t()
    for rows in [0, 1, 7, 8, 1536, 151936]:
        for n in range(1, 10):
            prev = 0
            for tid in range(n):
                L.hso_split(rows, n, tid, C.byref(a), C.byref(b))
                assert a.value == prev
                prev = b.value
            assert prev == rows


# ---- hs-track/src/pageset.rs:140-176 and hs-wire/src/lib.rs:457-503 ---------

def words_of(n_pages, marks):
    w = np.zeros((n_pages + 63) // 64, dtype=np.uint64)
    for p in marks:
        w[p // 64] |= np.uint64(1) << np.uint64(p % 64)
    return w


def test_pageset_runs_coalesce_across_word_boundaries():
    w = words_of(200, list(range(60, 70)) + [100, 102])
    assert ffi.pageset_runs(w, 200) == [(60, 10), (100, 1), (102, 1)]


def test_pageset_full_set_is_one_run():
    assert ffi.pageset_runs(words_of(130, range(130)), 130) == [(0, 130)]


def test_pageset_runs_reconstruct_the_membership_exactly():
    want = np.zeros(500, dtype=bool)
    x = 12345
    for p in range(500):
        x = (x * 6364136223846793005 + 1442695040888963407) & (2 ** 64 - 1)
        if x >> 62 == 0:
            want[p] = True
    got = np.zeros(500, dtype=bool)
    for first, n in ffi.pageset_runs(words_of(500, np.nonzero(want)[0]), 500):
        assert not got[first:first + n].any()
        got[first:first + n] = True
    assert np.array_equal(got, want)


def test_byte_runs_are_clipped_to_the_live_prefix():
    assert ffi.runs_to_byte_runs(words_of(100, range(100)), 100, 4096, [(0, 10_000)]) == [(0, 10_000)]


def test_byte_runs_merge_adjacent_pages():
    w = words_of(100, list(range(3, 7)) + [7])
    assert ffi.runs_to_byte_runs(w, 100, 4096, [(0, 100 * 4096)]) == [(3 * 4096, 5 * 4096)]


def test_a_dirty_page_only_costs_its_live_bytes():
    ps = 16384
    assert ffi.runs_to_byte_runs(words_of(8, [2]), 8, ps, [(2 * ps, 512)]) == [(2 * 16384, 512)]


def test_byte_runs_handle_several_live_stripes():
    ps = 4096
    live = [(0, 8192), (40 * ps, 8192)]
    assert ffi.runs_to_byte_runs(words_of(64, range(64)), 64, ps, live) == [(0, 8192), (40 * 4096, 8192)]


def test_a_clean_set_sends_nothing():
    assert ffi.runs_to_byte_runs(words_of(64, []), 64, 4096, [(0, 1 << 20)]) == []
