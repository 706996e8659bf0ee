"""Seeded synthetic Qwen2 GGUF fixtures (test and benchmark input generator).

`write_synthetic_gguf(path, **shape, seed=...)` writes a GGUF v3 file of the
Qwen2 architecture with N(0, 0.02) weights and biases and unit norm gains,
quantised as the reference's loader expects (Q6_K token embedding, Q4_K
other 2-D weights, flat block streams; model.rs:110-185, 375-396). The writer
is C++ (`synth.cpp` beside this file) compiled with g++ into
`_build/libhs_synth.so`; it is not part of libhotseat.so, so a process that
only runs the CPU restatement of the reference maps none of the product's
code.

Shapes: QWEN05 (Qwen2.5-0.5B architecture) and QWEN15 (Qwen2.5-1.5B).
"""
import ctypes as C
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "synth.cpp")
LIB = os.path.join(HERE, "_build", "libhs_synth.so")

QWEN05 = dict(n_layers=24, d_model=896, n_heads=14, n_kv_heads=2, d_ff=4864, vocab=151936)
QWEN15 = dict(n_layers=28, d_model=1536, n_heads=12, n_kv_heads=2, d_ff=8960, vocab=151936)


class SynthSpec(C.Structure):
    _fields_ = [("n_layers", C.c_uint32), ("d_model", C.c_uint32), ("n_heads", C.c_uint32),
                ("n_kv_heads", C.c_uint32), ("d_ff", C.c_uint32), ("vocab", C.c_uint32),
                ("context_length", C.c_uint32), ("eos", C.c_uint32), ("eps", C.c_float), ("rope_base", C.c_float),
                ("weight_std", C.c_float), ("bias_std", C.c_float), ("embd_type", C.c_uint32),
                ("weight_type", C.c_uint32), ("tied", C.c_uint32), ("threads", C.c_uint32), ("seed", C.c_uint64)]


def build(force=False):
    """Compile the writer (g++, seconds); a no-op when the library is current."""
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-o", LIB, SRC, "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"building the fixture writer failed:\n{r.stdout}\n{r.stderr}")
    return LIB


_lib = None


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        lib = C.CDLL(LIB)
        lib.hs_synth_write.restype = C.c_int
        lib.hs_synth_write.argtypes = [C.c_char_p, C.POINTER(SynthSpec)]
        lib.hs_synth_last_error.restype = C.c_char_p
        lib.hs_synth_last_error.argtypes = []
        _lib = lib
    return _lib


def write_synthetic_gguf(path, n_layers, d_model, n_heads, n_kv_heads, d_ff, vocab, seed, context_length=32768,
                         eos=None, eps=1e-6, rope_base=1e6, weight_std=0.02, bias_std=0.02, embd_type=14,
                         weight_type=12, tied=True, threads=0):
    """Seeded random-init Qwen2-architecture GGUF; returns `path`.

    eos defaults to 151643 (Qwen2's <|endoftext|>) when the vocabulary holds
    it, else the last id. Raises RuntimeError on a bad shape or an I/O error.
    """
    if eos is None:
        eos = 151643 if vocab > 151643 else vocab - 1
    spec = SynthSpec(n_layers, d_model, n_heads, n_kv_heads, d_ff, vocab, context_length, eos, eps, rope_base,
                     weight_std, bias_std, embd_type, weight_type, 1 if tied else 0, threads or (os.cpu_count() or 1),
                     seed)
    lib = _load()
    rc = lib.hs_synth_write(os.fsencode(path), C.byref(spec))
    if rc != 0:
        raise RuntimeError(f"[{rc}] {lib.hs_synth_last_error().decode(errors='replace')}")
    return path
