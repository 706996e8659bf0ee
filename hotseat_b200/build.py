"""Build libhotseat.so in-tree for sm_100a.

    python hotseat_b200/build.py [--force] [-v]

Compiles every source under hotseat_b200/csrc with nvcc (host files through
nvcc's host compiler) and links hotseat_b200/libhotseat.so with the CUDA
runtime linked statically, so the library loads on a host without a GPU and
fails only at the first call that needs one.

Floating point: -fmad=false and -ffp-contract=off keep every multiply and add
separately rounded, as the reference's arithmetic is; nothing is compiled
with fast-math.
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libhotseat.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC,-ffp-contract=off,-fno-fast-math",
          "-I" + os.path.join(HERE, "..", "include")]
SOURCES = ["engine.cu", "decode.cu", "decode_fast.cu", "batch_tc.cu", "batch_ops.cu", "attn_split.cu", "attn_prefill.cu", "token_fast.cu", "dequant.cu", "sample_noalloc.cu", "kv_xfer.cu", "migrate.cpp", "nll.cu", "gguf.cpp", "hostmath.cpp"]
HEADERS = ["common.h", "device.cuh", "kernels.h", "gguf.h", "attn_body.cuh"]


def _newer(src, dst, deps):
    if not os.path.exists(dst):
        return True
    t = os.path.getmtime(dst)
    return any(os.path.getmtime(p) > t for p in [src] + deps)


def _compile(src, verbose):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    deps = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(HERE, "..", "include", "hotseat.h")]
    if not _newer(src, obj, deps):
        return obj, False
    cmd = [NVCC] + ARCH + COMMON + ["-c", src, "-o", obj]
    if src.endswith(".cu") and verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        sys.stderr.write(r.stderr)
    return obj, True


def up_to_date():
    """True when libhotseat.so is newer than every source and header."""
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(HERE, "..", "include", "hotseat.h"),
                                                                   os.path.abspath(__file__)]
    return all(os.path.getmtime(p) <= t for p in deps)


def build(force=False, verbose=False):
    if not force and not verbose and up_to_date():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    if force:
        for s in srcs:
            o = os.path.join(BUILD, os.path.basename(s) + ".o")
            if os.path.exists(o):
                os.remove(o)
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), srcs))
    objs = [o for o, _ in results]
    if any(changed for _, changed in results) or not os.path.exists(LIB) or force:
        cmd = [NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
