"""Build libkessie_cuda.so for B200 (sm_100a) in-tree.

    python -m kessie_b200.build [--force] [--jobs N]

Outputs kessie_b200/build/libkessie_cuda.so and a copy named
libkessie_hip.so -- the file name the reference's ctypes loader searches
for (kessie_hip_ctypes.py:44-52) -- so the drop-in KeSSieKernels finds it
unchanged.  Objects go to kessie_b200/_build/.  nvcc cross-compiles without
a GPU.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "build")
LIB = os.path.join(OUT, "libkessie_cuda.so")
LEGACY = os.path.join(OUT, "libkessie_hip.so")

SOURCES = ["status.cu", "page_ops.cu", "fog_decode.cu", "fog_decode_f32.cu", "cp_exchange.cu", "fog_bias.cu", "index_query.cu", "tiered_cache.cu", "fog_prefill.cu", "fog_prefill_tc.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2", "-I" + os.path.join(ROOT, "include"),
                "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(ROOT, "include", "kessie_capi.h"))
    return hs


def _stale(src, obj, headers):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or any(os.path.getmtime(h) > t for h in headers)


def _compile(src, obj, verbose):
    cmd = [NVCC] + FLAGS + ["-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(force: bool = False, jobs: int = 8, verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(OUT, exist_ok=True)
    headers = _headers()
    objs, todo = [], []
    for s in SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(OBJ, s.replace(".cu", ".o"))
        objs.append(obj)
        if force or _stale(src, obj, headers):
            todo.append((src, obj))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
            for msg in ex.map(lambda a: _compile(a[0], a[1], verbose), todo):
                if msg and ("warning" in msg or "spill" in msg.lower()) and verbose:
                    print(msg, file=sys.stderr)
    if todo or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [NVCC] + ARCH + ["-shared", "-o", tmp] + objs + ["-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
        shutil.copyfile(LIB, LEGACY + ".tmp")
        os.replace(LEGACY + ".tmp", LEGACY)
    return LIB


BINDING_SRC = os.path.join(CSRC, "kessie_hip_binding.cpp")
BINDING = os.path.join(OUT, "kessie_hip.so")


def build_binding(force: bool = False, verbose: bool = False) -> str:
    """The torch extension module `kessie_hip` (the reference's pybind11
    boundary, over this library's C ABI), built in-tree with torch's
    extension builder: kessie_b200/build/kessie_hip.so.  Needs
    libkessie_cuda.so (its launchers are resolved from it at import)."""
    hdr = os.path.join(ROOT, "include", "kessie_capi.h")
    if (not force and os.path.exists(BINDING) and os.path.getmtime(BINDING) >= os.path.getmtime(BINDING_SRC)
            and os.path.getmtime(BINDING) >= os.path.getmtime(hdr)):
        return BINDING
    import ctypes
    from torch.utils.cpp_extension import load
    ctypes.CDLL(LIB, mode=ctypes.RTLD_GLOBAL)          # the launchers the module links against
    bdir = os.path.join(OBJ, "binding")
    os.makedirs(bdir, exist_ok=True)
    load(name="kessie_hip", sources=[BINDING_SRC], build_directory=bdir, with_cuda=True,
         extra_cflags=["-O2"], verbose=verbose)
    shutil.copyfile(os.path.join(bdir, "kessie_hip.so"), BINDING + ".tmp")
    os.replace(BINDING + ".tmp", BINDING)
    return BINDING


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.verbose))
    print(build_binding(a.force, a.verbose))
