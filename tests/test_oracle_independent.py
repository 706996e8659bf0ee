"""Independent checks of the CPU restatement, beyond the reference's KATs.

- dequantisation against gguf-py (llama.cpp's own Python package, installed in
  the image) on random blocks of every format the reference loads;
- the model fingerprint against a tensor table parsed by gguf-py;
- a whole forward pass against a float64 numpy Qwen2 written from the
  architecture (RMSNorm, NeoX RoPE, GQA, SwiGLU, tied head) — not from the
  reference's code — on the same dequantised weights.
"""
import struct

import numpy as np
import pytest

from oracle import ffi

gguf = pytest.importorskip("gguf")
from gguf import GGMLQuantizationType as Q  # noqa: E402
from gguf.quants import dequantize  # noqa: E402

from conftest import TINY, TINY128  # noqa: E402


@pytest.mark.parametrize("qtype,bs,be", [(Q.Q4_K, 144, 256), (Q.Q6_K, 210, 256), (Q.Q8_0, 34, 32),
                                         (Q.Q5_0, 22, 32), (Q.Q5_K, 176, 256)])
def test_dequant_matches_gguf_py(qtype, bs, be):
    rng = np.random.default_rng(int(qtype))
    nb = 1500
    r = rng.integers(0, 256, size=(nb, bs), dtype=np.uint8)
    offs = {Q.Q4_K: (0, 2), Q.Q5_K: (0, 2), Q.Q6_K: (208,)}.get(qtype, (0,))
    for off in offs:
        r[:, off:off + 2] = (rng.standard_normal(nb) * 0.01).astype(np.float16).view(np.uint8).reshape(nb, 2)
    ref = dequantize(r.reshape(-1), qtype).reshape(-1).astype(np.float32).astype(np.float16).view(np.uint16)
    ours = ffi.dequant_f16(int(qtype), r.tobytes(), nb * be)
    assert np.array_equal(ours, ref)


def _enum_index(t):
    return {0: 0, 1: 1, 6: 2, 8: 3, 12: 4, 13: 5, 14: 6}[int(t)]


def test_fingerprint_matches_a_gguf_py_parse(tiny_gguf):
    import os
    r = gguf.GGUFReader(tiny_gguf)
    h = 0xCBF29CE484222325

    def put(b):
        nonlocal h
        for x in b:
            h = ((h ^ x) * 0x100000001B3) & (2 ** 64 - 1)

    put(struct.pack("<Q", os.path.getsize(tiny_gguf)))
    for t in r.tensors:
        put(t.name.encode())
        put(struct.pack("<I", _enum_index(t.tensor_type)))
        put(struct.pack("<Q", t.data_offset))
        put(struct.pack("<Q", t.n_bytes))
    m = ffi.Model(tiny_gguf, max_ctx=16, threads=2)
    assert m.cfg.fingerprint == h


def numpy_qwen2(path, tokens):
    """float64 Qwen2 decode on gguf-py-dequantised f16 weights; returns logits per step."""
    r = gguf.GGUFReader(path)
    f = lambda k: r.fields[k].parts[-1][0]
    L_, d, dff = int(f("qwen2.block_count")), int(f("qwen2.embedding_length")), int(f("qwen2.feed_forward_length"))
    nh, nkv = int(f("qwen2.attention.head_count")), int(f("qwen2.attention.head_count_kv"))
    eps, base = float(f("qwen2.attention.layer_norm_rms_epsilon")), float(f("qwen2.rope.freq_base"))
    hd = d // nh
    T = {}
    for t in r.tensors:
        v = dequantize(t.data, t.tensor_type).reshape(-1).astype(np.float32)
        if len(t.shape) == 2:
            v = v.astype(np.float16).astype(np.float32)  # the engine keeps f16 weights
            v = v.reshape(int(t.shape[1]), int(t.shape[0]))
        T[t.name] = v.astype(np.float64)

    def rms(x, g):
        return x / np.sqrt(np.mean(x * x) + eps) * g

    inv = base ** (-np.arange(0, hd, 2) / hd)
    K = [[] for _ in range(L_)]
    V = [[] for _ in range(L_)]
    outs = []
    for pos, tok in enumerate(tokens):
        x = T["token_embd.weight"][tok].copy()
        c, s = np.cos(pos * inv), np.sin(pos * inv)

        def rope(v):
            a, b = v[..., : hd // 2], v[..., hd // 2:]
            return np.concatenate([a * c - b * s, a * s + b * c], axis=-1)

        for l in range(L_):
            p = f"blk.{l}."
            xb = rms(x, T[p + "attn_norm.weight"])
            q = (T[p + "attn_q.weight"] @ xb + T[p + "attn_q.bias"]).reshape(nh, hd)
            k = (T[p + "attn_k.weight"] @ xb + T[p + "attn_k.bias"]).reshape(nkv, hd)
            v = (T[p + "attn_v.weight"] @ xb + T[p + "attn_v.bias"]).reshape(nkv, hd)
            q, k = rope(q), rope(k)
            K[l].append(k)
            V[l].append(v)
            Ks, Vs = np.stack(K[l]), np.stack(V[l])  # [ctx, nkv, hd]
            att = np.zeros((nh, hd))
            for h in range(nh):
                g = h // (nh // nkv)
                sc = Ks[:, g, :] @ q[h] / np.sqrt(hd)
                w = np.exp(sc - sc.max())
                w /= w.sum()
                att[h] = w @ Vs[:, g, :]
            x = x + T[p + "attn_output.weight"] @ att.reshape(-1)
            xb = rms(x, T[p + "ffn_norm.weight"])
            gt = T[p + "ffn_gate.weight"] @ xb
            hb = gt / (1 + np.exp(-gt)) * (T[p + "ffn_up.weight"] @ xb)
            x = x + T[p + "ffn_down.weight"] @ hb
        xb = rms(x, T["output_norm.weight"])
        head = T.get("output.weight", T["token_embd.weight"])
        outs.append(head @ xb)
    return outs


@pytest.mark.parametrize("which", ["tiny", "tiny128"])
def test_forward_matches_float64_numpy(which, tiny_gguf, tiny128_gguf):
    path = tiny_gguf if which == "tiny" else tiny128_gguf
    spec = TINY if which == "tiny" else TINY128
    rng = np.random.default_rng(5)
    tokens = [int(t) for t in rng.integers(0, spec["vocab"], size=12)]
    ref = numpy_qwen2(path, tokens)
    m = ffi.Model(path, max_ctx=32, threads=4)
    kv = m.new_kv()
    for pos, tok in enumerate(tokens):
        ours = m.forward(kv, tok, pos).astype(np.float64)
        err = np.max(np.abs(ours - ref[pos]))
        # f32 accumulation over d=256..768 against float64: a few ulps of |logit| ~ 0.3-1
        assert err < 2e-5, (pos, err)
        assert int(np.argmax(ours)) == int(np.argmax(ref[pos])) or np.sort(ref[pos])[-1] - np.sort(ref[pos])[-2] < 1e-5
