"""hotseat_b200 — the hotseat token loop on B200 (sm_100a), behind a C ABI.

This module is a thin ctypes binding of include/hotseat.h, shaped like the
Rust API that hotseat's worker calls on hs-engine (crates/hs-engine/src):

    Model.load(path, max_ctx)         model.rs:110   Model::load
    model.cfg / .fingerprint / .eos   model.rs:62-78
    model.scratch()                   model.rs:221   Model::scratch
    model.forward(kv, tok, pos, s)    model.rs:240   Model::forward
    model.kv(layout, page_size)       hs-track Region + kv.rs Kv::from_raw
    kv.hash(n_pos)                    kv.rs:267      Kv::hash
    Sampler(cfg).sample(s, history)   sampler.rs:100 Sampler::sample
    argmax(s)                         sampler.rs:177 argmax
    run_seq(...)                      hs-worker seq.rs:230 run

All compute runs in libhotseat.so on the GPU. There is no CPU fallback: if the
library is missing the import fails, and a call without a GPU raises.
"""
import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libhotseat.so")

HS_OK = 0
HS_E_ARG, HS_E_IO, HS_E_CUDA, HS_E_STATE, HS_E_NOMEM, HS_E_UNSUPPORTED = -1, -2, -3, -4, -5, -6
TOKEN_MAJOR, HEAD_MAJOR = 0, 1
NUMERIC_REFERENCE, NUMERIC_FAST, NUMERIC_TC = 0, 1, 2
DONE_REASONS = {0: "", 1: "eos", 2: "max_tokens", 3: "context full"}

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is not built; run `python hotseat_b200/build.py` (needs nvcc)")
_lib = C.CDLL(LIB_PATH)


class HotseatError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class Config(C.Structure):
    _fields_ = [("n_layers", C.c_uint32), ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32),
                ("head_dim", C.c_uint32), ("d_model", C.c_uint32), ("d_ff", C.c_uint32), ("vocab", C.c_uint32),
                ("eps", C.c_float), ("rope_base", C.c_float), ("train_ctx", C.c_uint32), ("max_ctx", C.c_uint32),
                ("eos", C.c_uint32), ("fingerprint", C.c_uint64), ("numeric", C.c_uint32)]


class KvSpec(C.Structure):
    _fields_ = [("n_layers", C.c_uint32), ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
                ("max_ctx", C.c_uint32), ("layout", C.c_uint32)]


class SamplerCfg(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_uint32),
                ("repeat_penalty", C.c_float), ("repeat_last_n", C.c_uint32), ("seed", C.c_uint64)]

    @classmethod
    def default(cls, **kw):
        c = cls()
        _lib.hs_sampler_cfg_default(C.byref(c))
        for k, v in kw.items():
            setattr(c, k, v)
        return c


class Rng(C.Structure):
    _fields_ = [("s", C.c_uint64 * 4), ("draws", C.c_uint64)]

    @classmethod
    def seed(cls, seed):
        r = cls()
        _lib.hs_rng_seed(C.c_uint64(seed), C.byref(r))
        return r

    def state(self):
        return [int(x) for x in self.s], int(self.draws)


class SeqState(C.Structure):
    _fields_ = [("prompt_len", C.c_uint64), ("filled", C.c_uint64), ("max_tokens", C.c_uint64),
                ("done", C.c_uint32), ("done_reason", C.c_uint32)]


MIGRATE_MAX_ROUNDS = 34


class MigrateOpts(C.Structure):
    _fields_ = [("max_rounds", C.c_uint32), ("target_bytes", C.c_uint64), ("verify", C.c_uint32)]


class MigrateRoundStat(C.Structure):
    _fields_ = [("index", C.c_uint32), ("bytes", C.c_uint64), ("runs", C.c_uint64), ("ms", C.c_double),
                ("tokens_during", C.c_uint64)]


class MigrateReport(C.Structure):
    _fields_ = [("rounds", MigrateRoundStat * MIGRATE_MAX_ROUNDS), ("n_rounds", C.c_uint32),
                ("precopy_bytes", C.c_uint64), ("precopy_ms", C.c_double), ("park_us", C.c_double),
                ("stw_us", C.c_double), ("stw_send_us", C.c_double), ("dest_resume_us", C.c_double),
                ("final_bytes", C.c_uint64), ("live_bytes", C.c_uint64), ("filled", C.c_uint64),
                ("tokens_total", C.c_uint64), ("kv_hash_src", C.c_uint64), ("kv_hash_dst", C.c_uint64),
                ("verified", C.c_uint32), ("converged", C.c_uint32), ("stop_reason", C.c_char * 160)]

    def as_dict(self):
        d = {f: getattr(self, f) for f, _ in self._fields_ if f not in ("rounds", "stop_reason")}
        d["rounds"] = [dict(index=r.index, bytes=r.bytes, runs=r.runs, ms=r.ms, tokens_during=r.tokens_during)
                       for r in self.rounds[: self.n_rounds]]
        d["stop_reason"] = self.stop_reason.decode(errors="replace")
        return d


_P = C.c_void_p
_U64P = C.POINTER(C.c_uint64)
_SIGS = {
    "hs_last_error": (C.c_char_p, []),
    "hs_model_load": (C.c_int, [C.c_char_p, C.c_uint32, C.c_int, C.POINTER(_P)]),
    "hs_model_load_ex": (C.c_int, [C.c_char_p, C.c_uint32, C.c_int, C.c_uint32, C.POINTER(_P)]),
    "hs_model_config": (C.c_int, [_P, C.POINTER(Config)]),
    "hs_model_free": (None, [_P]),
    "hs_model_tensor": (C.c_int, [_P, C.c_char_p, _P, C.c_uint64, C.POINTER(C.c_uint32)]),
    "hs_kv_alloc": (C.c_int, [_P, C.c_uint32, C.c_uint32, C.POINTER(_P)]),
    "hs_kv_info": (C.c_int, [_P, C.POINTER(KvSpec), _U64P, C.POINTER(C.c_uint32), _U64P]),
    "hs_kv_free": (None, [_P]),
    "hs_kv_read": (C.c_int, [_P, C.c_uint64, C.c_uint64, _P]),
    "hs_kv_write": (C.c_int, [_P, C.c_uint64, C.c_uint64, _P]),
    "hs_kv_hash": (C.c_int, [_P, C.c_uint32, _U64P]),
    "hs_kv_arm": (C.c_int, [_P]),
    "hs_kv_harvest": (C.c_int, [_P, _P, C.c_uint64]),
    "hs_kv_disarm": (C.c_int, [_P]),
    "hs_kv_copy_runs": (C.c_int, [_P, _P, _P, C.c_uint64]),
    "hs_kv_fingerprint": (C.c_int, [_P, _U64P]),
    "hs_kv_ipc_handle": (C.c_int, [_P, _P, C.c_uint64]),
    "hs_kv_open_ipc": (C.c_int, [_P, C.c_char_p, C.c_uint32, C.c_uint32, C.POINTER(_P)]),
    "hs_migrate_opts_default": (None, [C.POINTER(MigrateOpts)]),
    "hs_migrate_begin": (C.c_int, [_P, _P, C.POINTER(MigrateOpts), C.c_uint64, C.c_uint64, C.c_uint64,
                                   C.POINTER(_P)]),
    "hs_migrate_round": (C.c_int, [_P, C.c_uint64, C.c_uint64, C.c_uint64, C.POINTER(C.c_int)]),
    "hs_migrate_finish": (C.c_int, [_P, C.c_uint64, C.c_uint64, C.c_double, C.POINTER(MigrateReport)]),
    "hs_migrate_free": (None, [_P]),
    "hs_kv_peer_copy": (C.c_int, [_P, _P, _P, C.c_uint64, _P]),
    "hs_kv_read_runs": (C.c_int, [_P, _P, C.c_uint64, _P, C.c_uint64]),
    "hs_kv_write_runs": (C.c_int, [_P, _P, C.c_uint64, _P, C.c_uint64]),
    "hs_kv_live_ranges_between": (C.c_uint64, [C.POINTER(KvSpec), C.c_uint32, C.c_uint32, _P, C.c_uint64]),
    "hs_runs_to_byte_runs": (C.c_uint64, [_P, C.c_uint64, C.c_uint64, _P, C.c_uint64, _P, C.c_uint64]),
    "hs_scratch_new": (C.c_int, [_P, C.POINTER(_P)]),
    "hs_scratch_free": (None, [_P]),
    "hs_forward": (C.c_int, [_P, _P, C.c_uint32, C.c_uint32, _P]),
    "hs_scratch_logits": (C.c_int, [_P, _P, C.c_uint64]),
    "hs_scratch_set_logits": (C.c_int, [_P, _P, C.c_uint64]),
    "hs_scratch_nll": (C.c_int, [_P, C.c_uint32, C.POINTER(C.c_double)]),
    "hs_batch_nll": (C.c_int, [_P, _P, C.c_uint32, _P]),
    "hs_sampler_cfg_default": (None, [C.POINTER(SamplerCfg)]),
    "hs_rng_seed": (None, [C.c_uint64, C.POINTER(Rng)]),
    "hs_sample": (C.c_int, [_P, C.POINTER(SamplerCfg), C.POINTER(Rng), _P, C.c_uint64, C.POINTER(C.c_uint32)]),
    "hs_argmax": (C.c_int, [_P, C.POINTER(C.c_uint32)]),
    "hs_sample_noalloc": (C.c_int, [C.c_int, _P, C.c_uint32, C.POINTER(SamplerCfg), C.POINTER(Rng), _P, C.c_uint64,
                                    _P, C.POINTER(C.c_uint32)]),
    "hs_seq_run": (C.c_int, [_P, _P, _P, _P, _U64P, C.c_uint64, C.POINTER(SeqState), C.POINTER(SamplerCfg),
                             C.POINTER(Rng), C.c_uint64]),
    "hs_seq_begin": (C.c_int, [_P, _P, _P, C.c_uint64, C.c_uint64, C.POINTER(SeqState), C.POINTER(SamplerCfg),
                               C.POINTER(Rng), C.c_uint64]),
    "hs_seq_step": (C.c_int, [_P, C.c_uint32]),
    "hs_seq_end": (C.c_int, [_P, _P, _U64P, C.c_uint64, C.POINTER(SeqState), C.POINTER(Rng)]),
    "hs_scratch_stream": (_P, [_P]),
    "hs_seq_launches_per_step": (C.c_int, [_P, C.POINTER(C.c_uint32)]),
    "hs_scratch_trace": (C.c_int, [_P, _P, C.c_uint64, _U64P]),
    "hs_dequant_f16": (C.c_int, [C.c_uint32, _P, C.c_uint64, _P, _P]),
    "hs_batch_new": (C.c_int, [_P, C.c_uint32, C.POINTER(_P)]),
    "hs_batch_free": (None, [_P]),
    "hs_forward_batch": (C.c_int, [_P, _P, _P, _P, C.c_uint32, _P]),
    "hs_batch_logits": (C.c_int, [_P, C.c_uint32, _P, C.c_uint64]),
    "hs_prefill": (C.c_int, [_P, _P, _P, C.c_uint32, C.c_uint32, _P]),
    "hs_batch_seq_run": (C.c_int, [_P, _P, _P, C.c_uint32, _P, _U64P, C.c_uint64, C.POINTER(SeqState),
                                   C.POINTER(SamplerCfg), C.POINTER(Rng), C.c_uint64]),
    "hs_batch_seq_begin": (C.c_int, [_P, _P, C.c_uint32, _P, _U64P, C.c_uint64, C.POINTER(SeqState),
                                     C.POINTER(SamplerCfg), C.POINTER(Rng), C.c_uint64]),
    "hs_batch_seq_step": (C.c_int, [_P, C.c_uint32]),
    "hs_batch_seq_end": (C.c_int, [_P, _P, _U64P, C.c_uint64, C.POINTER(SeqState), C.POINTER(Rng)]),
    "hs_batch_stream": (_P, [_P]),
    "hs_batch_launches_per_step": (C.c_int, [_P, C.POINTER(C.c_uint32)]),
    "hs_batch_trace": (C.c_int, [_P, _P, C.c_uint64, _U64P]),
}
for _name, (_res, _args) in _SIGS.items():
    _f = getattr(_lib, _name)
    _f.restype = _res
    _f.argtypes = _args

EXPORTED = tuple(_SIGS)


def _check(rc):
    if rc != HS_OK:
        raise HotseatError(rc, _lib.hs_last_error().decode(errors="replace"))


def _ptr(a):
    return a.ctypes.data_as(C.c_void_p)


def lib():
    return _lib


class Model:
    """A loaded model on one GPU (Model::load, model.rs:110-215)."""

    def __init__(self, handle):
        self._h = handle
        self.cfg = Config()
        _check(_lib.hs_model_config(handle, C.byref(self.cfg)))

    @classmethod
    def load(cls, path, max_ctx=2048, device=0, numeric=NUMERIC_REFERENCE):
        """numeric: NUMERIC_REFERENCE (bit-identical to the CPU reference) or
        NUMERIC_FAST (GPU-native reduction order, deterministic across GPUs)."""
        h = C.c_void_p()
        _check(_lib.hs_model_load_ex(os.fsencode(path), max_ctx, device, numeric, C.byref(h)))
        return cls(h)

    @property
    def fingerprint(self):
        return int(self.cfg.fingerprint)

    @property
    def eos(self):
        return int(self.cfg.eos)

    def close(self):
        if getattr(self, "_h", None):
            _lib.hs_model_free(self._h)
            self._h = None

    __del__ = close

    def tensor(self, name):
        """A loaded tensor copied back: f16 bits (uint16) or f32."""
        dt = C.c_uint32()
        _check(_lib.hs_model_tensor(self._h, name.encode(), None, 0, C.byref(dt)))
        c = self.cfg
        hd = c.head_dim
        shapes = {
            "token_embd.weight": c.vocab * c.d_model, "output.weight": c.vocab * c.d_model,
            "output_norm.weight": c.d_model,
        }
        base = name.split(".", 2)[-1] if name.startswith("blk.") else name
        per = {
            "attn_norm.weight": c.d_model, "ffn_norm.weight": c.d_model,
            "attn_q.weight": c.n_heads * hd * c.d_model, "attn_k.weight": c.n_kv_heads * hd * c.d_model,
            "attn_v.weight": c.n_kv_heads * hd * c.d_model, "attn_output.weight": c.d_model * c.n_heads * hd,
            "attn_q.bias": c.n_heads * hd, "attn_k.bias": c.n_kv_heads * hd, "attn_v.bias": c.n_kv_heads * hd,
            "ffn_gate.weight": c.d_ff * c.d_model, "ffn_up.weight": c.d_ff * c.d_model,
            "ffn_down.weight": c.d_model * c.d_ff,
        }
        count = shapes.get(name) if not name.startswith("blk.") else per[base]
        out = np.zeros(count, dtype=np.uint16 if dt.value == 1 else np.float32)
        _check(_lib.hs_model_tensor(self._h, name.encode(), _ptr(out), out.nbytes, None))
        return out

    def kv_spec(self, layout=TOKEN_MAJOR):
        c = self.cfg
        return KvSpec(c.n_layers, c.n_kv_heads, c.head_dim, c.max_ctx, layout)

    def kv(self, layout=TOKEN_MAJOR, page_size=4096):
        return Kv.alloc(self, layout, page_size)

    def scratch(self):
        return Scratch(self)

    def forward(self, kv, token, pos, scratch):
        """One token through every layer; appends its K/V to `kv`."""
        _check(_lib.hs_forward(self._h, kv._h, token, pos, scratch._h))


class Kv:
    """Device KV region in the reference's byte layout, with a dirty-page bitmap."""

    def __init__(self, handle, model):
        self._h = handle
        self.model = model
        self.spec = KvSpec()
        b, ps, npg = C.c_uint64(), C.c_uint32(), C.c_uint64()
        _check(_lib.hs_kv_info(handle, C.byref(self.spec), C.byref(b), C.byref(ps), C.byref(npg)))
        self.bytes, self.page_size, self.n_pages = b.value, ps.value, npg.value
        self.n_words = (self.n_pages + 63) // 64

    @classmethod
    def alloc(cls, model, layout=TOKEN_MAJOR, page_size=4096):
        h = C.c_void_p()
        _check(_lib.hs_kv_alloc(model._h, layout, page_size, C.byref(h)))
        return cls(h, model)

    def ipc_handle(self):
        """The region's CUDA IPC handle (bytes) for another process's open_ipc."""
        buf = C.create_string_buffer(64)
        _check(_lib.hs_kv_ipc_handle(self._h, buf, 64))
        return buf.raw

    @classmethod
    def open_ipc(cls, model, handle, layout=TOKEN_MAJOR, page_size=4096):
        """Map another process's region (same spec) on `model`'s GPU as a
        hand-over destination."""
        h = C.c_void_p()
        _check(_lib.hs_kv_open_ipc(model._h, bytes(handle), layout, page_size, C.byref(h)))
        return cls(h, model)

    def close(self):
        if getattr(self, "_h", None):
            _lib.hs_kv_free(self._h)
            self._h = None

    __del__ = close

    def read(self, off, length):
        out = np.zeros(length, dtype=np.uint8)
        _check(_lib.hs_kv_read(self._h, off, length, _ptr(out)))
        return out

    def write(self, off, data):
        data = np.ascontiguousarray(np.frombuffer(bytes(data), dtype=np.uint8))
        _check(_lib.hs_kv_write(self._h, off, data.size, _ptr(data)))

    def floats(self):
        return self.read(0, self.bytes).view(np.float32)

    def hash(self, n_pos):
        out = C.c_uint64()
        _check(_lib.hs_kv_hash(self._h, n_pos, C.byref(out)))
        return out.value

    def arm(self):
        _check(_lib.hs_kv_arm(self._h))

    def harvest(self):
        w = np.zeros(self.n_words, dtype=np.uint64)
        _check(_lib.hs_kv_harvest(self._h, _ptr(w), w.size))
        return w

    def disarm(self):
        _check(_lib.hs_kv_disarm(self._h))

    @staticmethod
    def _runs(runs):
        return np.array([x for run in runs for x in run] or [0], dtype=np.uint64)

    def copy_runs_to(self, dst, runs):
        """Blocking copy of byte runs into `dst` (same spec, any GPU)."""
        r = self._runs(runs)
        _check(_lib.hs_kv_copy_runs(self._h, dst._h, _ptr(r), len(runs)))

    def peer_copy(self, dst, runs, stream=None):
        """Enqueue the copy of byte runs into `dst` on `stream` (a stream of
        this region's GPU; None = this region's own stream); not waited for."""
        r = self._runs(runs)
        _check(_lib.hs_kv_peer_copy(self._h, dst._h, _ptr(r), len(runs), C.c_void_p(stream) if stream else None))

    def read_runs(self, runs):
        """The bytes of `runs` packed back to back (hs-wire send_page_bytes)."""
        r = self._runs(runs)
        out = np.zeros(max(1, sum(int(x[1]) for x in runs)), dtype=np.uint8)
        _check(_lib.hs_kv_read_runs(self._h, _ptr(r), len(runs), _ptr(out), out.size))
        return out[: sum(int(x[1]) for x in runs)]

    def write_runs(self, runs, data):
        """Scatter packed bytes into `runs` (hs-wire recv_page_bytes)."""
        r = self._runs(runs)
        d = np.ascontiguousarray(np.frombuffer(bytes(data), dtype=np.uint8))
        _check(_lib.hs_kv_write_runs(self._h, _ptr(r), len(runs), _ptr(d) if d.size else None, d.size))


class Migration:
    """Pre-copy migration of a live sequence from KV region `src` to `dst`
    (hs-worker migrate.rs migrate_out + migrate_in's checks): construction
    runs the Hello checks and round 0; round() is one iterative round while
    the sequence keeps decoding (False once the rounds stop); finish(), with
    the decode loop parked, copies the residue and returns the report. The
    sequence's tokens, SeqState and RNG are the caller's to hand over."""

    def __init__(self, src, dst, filled, tokens_now, upper=None, max_rounds=8, target_bytes=1 << 20,
                 verify=False):
        o = MigrateOpts()
        _lib.hs_migrate_opts_default(C.byref(o))
        o.max_rounds, o.target_bytes, o.verify = max_rounds, target_bytes, 1 if verify else 0
        h = C.c_void_p()
        _check(_lib.hs_migrate_begin(src._h, dst._h, C.byref(o), filled, filled if upper is None else upper,
                                     tokens_now, C.byref(h)))
        self._h = h

    def round(self, filled, tokens_now, upper=None):
        """filled: positions known complete; upper: the last position the
        decode loop may have written (filled when parked)."""
        more = C.c_int()
        _check(_lib.hs_migrate_round(self._h, filled, filled if upper is None else upper, tokens_now,
                                     C.byref(more)))
        return bool(more.value)

    def finish(self, filled, tokens_total, park_us=0.0):
        r = MigrateReport()
        rc = _lib.hs_migrate_finish(self._h, filled, tokens_total, park_us, C.byref(r))
        self.report = r.as_dict()
        _check(rc)
        return self.report

    def close(self):
        if getattr(self, "_h", None):
            _lib.hs_migrate_free(self._h)
            self._h = None

    __del__ = close


def live_ranges_between(spec, a, b):
    n = _lib.hs_kv_live_ranges_between(C.byref(spec), a, b, None, 0)
    out = np.zeros(2 * max(n, 1), dtype=np.uint64)
    _lib.hs_kv_live_ranges_between(C.byref(spec), a, b, _ptr(out), n)
    return [(int(out[2 * i]), int(out[2 * i + 1])) for i in range(n)]


def runs_to_byte_runs(words, n_pages, page_size, live):
    w = np.ascontiguousarray(words, dtype=np.uint64)
    lv = np.array([x for r in live for x in r] or [0], dtype=np.uint64)
    n = _lib.hs_runs_to_byte_runs(_ptr(w), n_pages, page_size, _ptr(lv), len(live), None, 0)
    out = np.zeros(2 * max(n, 1), dtype=np.uint64)
    _lib.hs_runs_to_byte_runs(_ptr(w), n_pages, page_size, _ptr(lv), len(live), _ptr(out), n)
    return [(int(out[2 * i]), int(out[2 * i + 1])) for i in range(n)]


class Scratch:
    """Per-decode-thread device state: activations, logits, stream, graphs."""

    def __init__(self, model):
        h = C.c_void_p()
        _check(_lib.hs_scratch_new(model._h, C.byref(h)))
        self._h = h
        self.model = model

    def close(self):
        if getattr(self, "_h", None):
            _lib.hs_scratch_free(self._h)
            self._h = None

    __del__ = close

    def logits(self):
        out = np.zeros(self.model.cfg.vocab, dtype=np.float32)
        _check(_lib.hs_scratch_logits(self._h, _ptr(out), out.size))
        return out

    def set_logits(self, logits):
        a = np.ascontiguousarray(logits, dtype=np.float32)
        _check(_lib.hs_scratch_set_logits(self._h, _ptr(a), a.size))

    def nll(self, next_token):
        """examples/ppl.rs's score of next_token under the current logits."""
        out = C.c_double()
        _check(_lib.hs_scratch_nll(self._h, next_token, C.byref(out)))
        return out.value

    @property
    def stream(self):
        return _lib.hs_scratch_stream(self._h)

    def trace(self):
        """Launch timeline of the last decode step (needs HS_TRACE=1 at creation):
        array [slots, 8]: entry, past-wait, exit, last entry, checkpoints 1-4 (ns)."""
        used = C.c_uint64()
        _check(_lib.hs_scratch_trace(self._h, None, 0, C.byref(used)))
        out = np.zeros((used.value, 8), dtype=np.uint64)
        _check(_lib.hs_scratch_trace(self._h, _ptr(out), used.value, C.byref(used)))
        return out

    def launches_per_step(self):
        n = C.c_uint32()
        _check(_lib.hs_seq_launches_per_step(self._h, C.byref(n)))
        return n.value


class Sampler:
    """Sampler{cfg, rng} (sampler.rs:85-167); sampling runs on the device."""

    def __init__(self, cfg=None, rng=None):
        self.cfg = cfg or SamplerCfg.default()
        self.rng = rng or Rng.seed(self.cfg.seed)

    def sample(self, scratch, history=()):
        h = np.ascontiguousarray(history, dtype=np.uint32)
        out = C.c_uint32()
        _check(_lib.hs_sample(scratch._h, C.byref(self.cfg), C.byref(self.rng), _ptr(h) if h.size else None, h.size,
                              C.byref(out)))
        return out.value


def argmax(scratch):
    out = C.c_uint32()
    _check(_lib.hs_argmax(scratch._h, C.byref(out)))
    return out.value


def run_seq(model, kv, scratch, tokens, prompt_len, max_tokens, cfg, rng, filled=0, stop_at_filled=0, done=0,
            done_reason=0):
    """The seq.rs decode loop on the device. Returns (tokens, SeqState, Rng)."""
    cap = model.cfg.max_ctx + 1
    buf = np.zeros(cap, dtype=np.uint32)
    buf[: len(tokens)] = tokens
    n = C.c_uint64(len(tokens))
    st = SeqState(prompt_len, filled, max_tokens, done, done_reason)
    _check(_lib.hs_seq_run(model._h, kv._h, scratch._h, _ptr(buf), C.byref(n), cap, C.byref(st), C.byref(cfg),
                           C.byref(rng), stop_at_filled))
    return buf[: n.value].copy(), st, rng


class Batch:
    """Working memory for decoding up to `max_seqs` sequences together
    (models loaded with NUMERIC_TC)."""

    def __init__(self, model, max_seqs):
        h = C.c_void_p()
        _check(_lib.hs_batch_new(model._h, max_seqs, C.byref(h)))
        self._h = h
        self.model = model
        self.max_seqs = max_seqs

    def close(self):
        if getattr(self, "_h", None):
            _lib.hs_batch_free(self._h)
            self._h = None

    __del__ = close

    @staticmethod
    def _kv_table(kvs):
        return (C.c_void_p * len(kvs))(*[k._h.value for k in kvs])

    def forward(self, kvs, tokens, pos):
        """One forward per sequence: tokens[i] at pos[i] into kvs[i]."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = np.ascontiguousarray(pos, dtype=np.uint32)
        _check(_lib.hs_forward_batch(self.model._h, self._kv_table(kvs), _ptr(t), _ptr(p), len(kvs), self._h))

    def prefill(self, kv, tokens, pos0=0):
        """Forward a prompt's tokens (one sequence) as GEMM rows; fills its KV."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        _check(_lib.hs_prefill(self.model._h, kv._h, _ptr(t), t.size, pos0, self._h))

    def logits(self, slot):
        out = np.zeros(self.model.cfg.vocab, dtype=np.float32)
        _check(_lib.hs_batch_logits(self._h, slot, _ptr(out), out.size))
        return out

    def nll(self, next_tokens):
        """examples/ppl.rs's score per slot of the last forward."""
        t = np.ascontiguousarray(next_tokens, dtype=np.uint32)
        out = np.zeros(max(1, t.size), dtype=np.float64)
        _check(_lib.hs_batch_nll(self._h, _ptr(t), t.size, _ptr(out)))
        return out[: t.size]

    @property
    def stream(self):
        return _lib.hs_batch_stream(self._h)

    def launches_per_step(self):
        n = C.c_uint32()
        _check(_lib.hs_batch_launches_per_step(self._h, C.byref(n)))
        return n.value

    def trace(self):
        """Launch timeline of the last forward/step (needs HS_TRACE=1 at creation):
        array [slots, 8]: entry, past-wait, exit, last entry, checkpoints 1-4 (ns)."""
        used = C.c_uint64()
        _check(_lib.hs_batch_trace(self._h, None, 0, C.byref(used)))
        out = np.zeros((used.value, 8), dtype=np.uint64)
        _check(_lib.hs_batch_trace(self._h, _ptr(out), used.value, C.byref(used)))
        return out

    def _state(self, seqs, stop_at_filled):
        """seqs: list of dicts with tokens, prompt_len, max_tokens, cfg, rng, filled, done, done_reason."""
        n = len(seqs)
        cap = self.model.cfg.max_ctx + 1
        bufs = [np.zeros(cap, dtype=np.uint32) for _ in range(n)]
        for b, q in zip(bufs, seqs):
            b[: len(q["tokens"])] = q["tokens"]
        tabs = (C.c_void_p * n)(*[b.ctypes.data for b in bufs])
        nt = (C.c_uint64 * n)(*[len(q["tokens"]) for q in seqs])
        st = (SeqState * n)(*[SeqState(q["prompt_len"], q.get("filled", 0), q["max_tokens"], q.get("done", 0),
                                       q.get("done_reason", 0)) for q in seqs])
        cfg = (SamplerCfg * n)(*[q["cfg"] for q in seqs])
        rng = (Rng * n)(*[q["rng"] for q in seqs])
        return bufs, tabs, nt, st, cfg, rng, cap

    def run_seqs(self, kvs, seqs, stop_at_filled=0):
        """hs_batch_seq_run: every sequence to its stop. Returns [(tokens, SeqState, Rng)]."""
        bufs, tabs, nt, st, cfg, rng, cap = self._state(seqs, stop_at_filled)
        _check(_lib.hs_batch_seq_run(self.model._h, self._kv_table(kvs), self._h, len(seqs), tabs, nt, cap, st, cfg,
                                     rng, stop_at_filled))
        return [(bufs[i][: nt[i]].copy(), st[i], rng[i]) for i in range(len(seqs))]

    def begin(self, kvs, seqs, stop_at_filled=0):
        self._pending = self._state(seqs, stop_at_filled)
        bufs, tabs, nt, st, cfg, rng, cap = self._pending
        _check(_lib.hs_batch_seq_begin(self._h, self._kv_table(kvs), len(seqs), tabs, nt, cap, st, cfg, rng,
                                       stop_at_filled))

    def step(self, n_steps):
        _check(_lib.hs_batch_seq_step(self._h, n_steps))

    def end(self):
        bufs, tabs, nt, st, cfg, rng, cap = self._pending
        _check(_lib.hs_batch_seq_end(self._h, tabs, nt, cap, st, rng))
        return [(bufs[i][: nt[i]].copy(), st[i], rng[i]) for i in range(len(bufs))]


def dequant_f16(ggml_type, src_dev_ptr, n, dst_dev_ptr, stream=None):
    _check(_lib.hs_dequant_f16(ggml_type, C.c_void_p(src_dev_ptr), n, C.c_void_p(dst_dev_ptr),
                               C.c_void_p(stream) if stream else None))

