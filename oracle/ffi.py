"""ctypes binding for the CPU restatement in oracle/hs_oracle.cpp.

Test infrastructure only: tests/, __graft_entry__.smoke() and bench.py's CPU
baseline use it as the checker. The product package never imports it.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "libhs_oracle.so")


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


class SamplerCfg(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_uint32),
                ("repeat_penalty", C.c_float), ("repeat_last_n", C.c_uint32), ("seed", C.c_uint64)]


class Rng(C.Structure):
    _fields_ = [("s", C.c_uint64 * 4), ("draws", C.c_uint64)]


class KvSpec(C.Structure):
    _fields_ = [("n_layers", C.c_uint64), ("n_kv_heads", C.c_uint64), ("head_dim", C.c_uint64),
                ("max_ctx", C.c_uint64), ("layout", C.c_uint32)]


class Config(C.Structure):
    _fields_ = [("n_layers", C.c_uint64), ("n_heads", C.c_uint64), ("n_kv_heads", C.c_uint64),
                ("head_dim", C.c_uint64), ("d_model", C.c_uint64), ("d_ff", C.c_uint64),
                ("vocab", C.c_uint64), ("eps", C.c_float), ("rope_base", C.c_float),
                ("train_ctx", C.c_uint64), ("fingerprint", C.c_uint64), ("eos", C.c_uint32),
                ("max_ctx", C.c_uint64)]


class SeqState(C.Structure):
    _fields_ = [("prompt_len", C.c_uint64), ("filled", C.c_uint64), ("max_tokens", C.c_uint64),
                ("done", C.c_uint32), ("done_reason", C.c_uint32)]


_lib = None


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    L = C.CDLL(LIB_PATH)
    P = C.c_void_p
    sig = {
        "hso_f16_to_f32": (C.c_float, [C.c_uint16]),
        "hso_f32_to_f16": (C.c_uint16, [C.c_float]),
        "hso_exp_f32": (C.c_float, [C.c_float]),
        "hso_ln_f32": (C.c_float, [C.c_float]),
        "hso_sincos_f32": (None, [C.c_float, C.POINTER(C.c_float), C.POINTER(C.c_float)]),
        "hso_silu": (C.c_float, [C.c_float]),
        "hso_dot_f16": (C.c_float, [P, P, C.c_size_t]),
        "hso_dot_f32": (C.c_float, [P, P, C.c_size_t]),
        "hso_rmsnorm": (None, [P, P, P, C.c_size_t, C.c_float]),
        "hso_softmax": (None, [P, C.c_size_t]),
        "hso_dequant_f16": (C.c_int, [C.c_uint32, P, C.c_size_t, P]),
        "hso_scale_min_k4": (C.c_uint32, [C.c_uint32, P]),
        "hso_fnv1a": (C.c_uint64, [P, C.c_size_t]),
        "hso_wide": (C.c_uint64, [P, C.c_size_t]),
        "hso_sampler_cfg_default": (None, [C.POINTER(SamplerCfg)]),
        "hso_rng_seed": (None, [C.c_uint64, C.POINTER(Rng)]),
        "hso_rng_next_u64": (C.c_uint64, [C.POINTER(Rng)]),
        "hso_rng_next_f32": (C.c_float, [C.POINTER(Rng)]),
        "hso_sample": (C.c_uint32, [C.POINTER(SamplerCfg), C.POINTER(Rng), P, C.c_size_t, P, C.c_size_t]),
        "hso_argmax": (C.c_uint32, [P, C.c_size_t]),
        "hso_penalised_argmax": (C.c_uint32, [C.POINTER(SamplerCfg), P, C.c_size_t, P, C.c_size_t]),
        "hso_nll": (C.c_double, [P, C.c_size_t, C.c_uint32]),
        "hso_split": (None, [C.c_size_t, C.c_size_t, C.c_size_t, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
        "hso_kv_row_off": (C.c_uint64, [C.POINTER(KvSpec), C.c_uint64, C.c_int, C.c_uint64, C.c_uint64]),
        "hso_kv_written_ranges": (C.c_size_t, [C.POINTER(KvSpec), C.c_uint64, P, C.c_size_t]),
        "hso_kv_live_ranges_between": (C.c_size_t, [C.POINTER(KvSpec), C.c_uint64, C.c_uint64, P, C.c_size_t]),
        "hso_kv_hash": (C.c_uint64, [C.POINTER(KvSpec), P, C.c_uint64]),
        "hso_pageset_runs": (C.c_size_t, [P, C.c_size_t, P, C.c_size_t]),
        "hso_runs_to_byte_runs": (C.c_size_t, [P, C.c_size_t, C.c_uint64, P, C.c_size_t, P, C.c_size_t]),
        "hso_model_load": (C.c_int, [C.c_char_p, C.c_uint64, C.c_uint32, C.POINTER(P)]),
        "hso_model_free": (None, [P]),
        "hso_model_config": (None, [P, C.POINTER(Config)]),
        "hso_last_error": (C.c_char_p, []),
        "hso_model_tensor_f16": (P, [P, C.c_char_p, C.POINTER(C.c_size_t)]),
        "hso_model_tensor_f32": (P, [P, C.c_char_p, C.POINTER(C.c_size_t)]),
        "hso_model_rope_cos": (P, [P]),
        "hso_model_rope_sin": (P, [P]),
        "hso_forward": (C.c_int, [P, P, C.c_uint32, C.c_uint32, C.c_uint64, P, P]),
        "hso_seq_run": (C.c_int, [P, P, C.c_uint32, P, C.POINTER(C.c_uint64), C.c_uint64,
                                  C.POINTER(SeqState), C.POINTER(SamplerCfg), C.POINTER(Rng), C.c_uint64]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def ptr(a):
    return a.ctypes.data_as(C.c_void_p)


def default_cfg(**kw):
    c = SamplerCfg()
    lib().hso_sampler_cfg_default(C.byref(c))
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def seeded_rng(seed):
    r = Rng()
    lib().hso_rng_seed(seed, C.byref(r))
    return r


def dequant_f16(ggml_type, raw, n):
    out = np.zeros(n, dtype=np.uint16)
    raw = np.ascontiguousarray(np.frombuffer(bytes(raw), dtype=np.uint8))
    rc = lib().hso_dequant_f16(ggml_type, ptr(raw), n, ptr(out))
    if rc != 0:
        raise ValueError(f"unknown ggml type {ggml_type}")
    return out


def fnv1a(b):
    a = np.frombuffer(bytes(b), dtype=np.uint8) if len(b) else np.zeros(1, np.uint8)
    return lib().hso_fnv1a(ptr(a), len(b))


def wide(b):
    a = np.frombuffer(bytes(b), dtype=np.uint8) if len(b) else np.zeros(1, np.uint8)
    return lib().hso_wide(ptr(a), len(b))


def _pairs(fn, *args, cap=1 << 16):
    out = np.zeros(2 * cap, dtype=np.uint64)
    n = fn(*args, ptr(out), cap)
    assert n <= cap
    return [(int(out[2 * i]), int(out[2 * i + 1])) for i in range(n)]


def kv_spec(n_layers, n_kv_heads, head_dim, max_ctx, layout=0):
    return KvSpec(n_layers, n_kv_heads, head_dim, max_ctx, layout)


def written_ranges(spec, pos):
    return _pairs(lib().hso_kv_written_ranges, C.byref(spec), pos)


def live_ranges_between(spec, a, b):
    return _pairs(lib().hso_kv_live_ranges_between, C.byref(spec), a, b)


def kv_hash(spec, kv, n_pos):
    return lib().hso_kv_hash(C.byref(spec), ptr(kv), n_pos)


def pageset_runs(words, n_pages):
    w = np.ascontiguousarray(words, dtype=np.uint64)
    return _pairs(lib().hso_pageset_runs, ptr(w), n_pages)


def runs_to_byte_runs(words, n_pages, page_size, live):
    w = np.ascontiguousarray(words, dtype=np.uint64)
    lv = np.array([x for r in live for x in r] or [0], dtype=np.uint64)
    return _pairs(lib().hso_runs_to_byte_runs, ptr(w), n_pages, page_size, ptr(lv), len(live))


class Model:
    """Model::load + Model::forward (model.rs:110-327) on the host CPU."""

    def __init__(self, path, max_ctx=2048, threads=0):
        threads = threads or os.cpu_count() or 1
        h = C.c_void_p()
        rc = lib().hso_model_load(path.encode(), max_ctx, threads, C.byref(h))
        if rc != 0:
            raise RuntimeError(lib().hso_last_error().decode())
        self.h = h
        self.cfg = Config()
        lib().hso_model_config(h, C.byref(self.cfg))
        self.threads = threads

    def __del__(self):
        if getattr(self, "h", None):
            lib().hso_model_free(self.h)
            self.h = None

    def kv_spec(self, layout=0):
        c = self.cfg
        return kv_spec(c.n_layers, c.n_kv_heads, c.head_dim, c.max_ctx, layout)

    def new_kv(self, layout=0):
        c = self.cfg
        return np.zeros(c.n_layers * 2 * c.max_ctx * c.n_kv_heads * c.head_dim, dtype=np.float32)

    def forward(self, kv, token, pos, layout=0, trace=False):
        c = self.cfg
        logits = np.zeros(c.vocab, dtype=np.float32)
        tr = np.zeros(c.n_layers * c.d_model, dtype=np.float32) if trace else None
        rc = lib().hso_forward(self.h, ptr(kv), layout, token, pos, ptr(logits),
                               ptr(tr) if trace else None)
        if rc != 0:
            raise RuntimeError(lib().hso_last_error().decode())
        return (logits, tr.reshape(c.n_layers, c.d_model)) if trace else logits

    def tensor_f16(self, name):
        n = C.c_size_t()
        p = lib().hso_model_tensor_f16(self.h, name.encode(), C.byref(n))
        if not p:
            return None
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint16)), shape=(n.value,)).copy()

    def tensor_f32(self, name):
        n = C.c_size_t()
        p = lib().hso_model_tensor_f32(self.h, name.encode(), C.byref(n))
        if not p:
            return None
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_float)), shape=(n.value,)).copy()

    def rope_tables(self):
        c = self.cfg
        n = c.max_ctx * (c.head_dim // 2)
        cs = np.ctypeslib.as_array(C.cast(lib().hso_model_rope_cos(self.h), C.POINTER(C.c_float)), shape=(n,))
        sn = np.ctypeslib.as_array(C.cast(lib().hso_model_rope_sin(self.h), C.POINTER(C.c_float)), shape=(n,))
        return cs.copy(), sn.copy()

    def run_seq(self, kv, prompt, max_tokens, cfg, rng, layout=0, stop_at_filled=0, state=None, tokens=None,
                cap=None):
        """seq.rs run loop. Returns (tokens, state, rng)."""
        cap = cap or (len(prompt) + max_tokens + 8)
        buf = np.zeros(cap, dtype=np.uint32)
        src = prompt if tokens is None else tokens
        buf[: len(src)] = src
        n = C.c_uint64(len(src))
        st = state or SeqState(len(prompt), 0, max_tokens, 0, 0)
        rc = lib().hso_seq_run(self.h, ptr(kv), layout, ptr(buf), C.byref(n), cap, C.byref(st), C.byref(cfg),
                               C.byref(rng), stop_at_filled)
        if rc != 0:
            raise RuntimeError(lib().hso_last_error().decode())
        return buf[: n.value].copy(), st, rng
