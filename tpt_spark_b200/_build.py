"""In-tree build of the native libraries.

``lib/libtptc.so``     the engine: CUDA kernels for sm_100a + C++ host runtime + C ABI
                       (``include/tptc.h``), compiled with nvcc, cudart linked statically.
``lib/libtptsynth.so`` synthetic-model encoder (plain C, OpenMP).

Objects go to ``_build/`` at the repository root; the .so files are written into the
package so they travel with the source tree.  Rebuilds are incremental on mtimes (any
header change rebuilds every object of its library).
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import hashlib
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "lib")
BUILD = os.path.join(ROOT, "_build")
INCLUDE = os.path.join(ROOT, "include")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
HOST_CC = "/usr/bin/gcc"
HOST_CXX = "/usr/bin/g++"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-ccbin", HOST_CXX, "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
                     "-I" + INCLUDE, "-I" + CSRC, "-DTPTC_BUILD"]


def lib_path(name: str) -> str:
    return os.path.join(LIBDIR, name)


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def build_synth(verbose=False) -> str:
    src = os.path.join(CSRC, "synth.c")
    out = lib_path("libtptsynth.so")
    stamp = out + ".srchash"
    digest = _source_hash([src])
    if os.path.exists(out) and os.path.exists(stamp) and open(stamp).read().strip() == digest:
        return out
    os.makedirs(LIBDIR, exist_ok=True)
    _run([HOST_CC, "-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", "-std=c11",
          "-ffp-contract=off", "-o", out, src, "-lm"])
    with open(stamp, "w") as fh:
        fh.write(digest)
    if verbose:
        print("built", out)
    return out


def _source_hash(files) -> str:
    h = hashlib.sha1()
    for f in sorted(files):
        h.update(os.path.basename(f).encode())
        with open(f, "rb") as fh:
            h.update(fh.read())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def build_tptc(verbose=False, jobs=None) -> str:
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    headers = (glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
               + glob.glob(os.path.join(INCLUDE, "*.h")))
    out = lib_path("libtptc.so")
    stamp = out + ".srchash"
    digest = _source_hash(srcs + headers)
    if os.path.exists(out) and os.path.exists(stamp) and open(stamp).read().strip() == digest:
        return out  # built from exactly these sources (mtimes may differ in a copied tree)
    objdir = os.path.join(BUILD, "tptc")
    os.makedirs(objdir, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    objs, todo = [], []
    for s in srcs:
        o = os.path.join(objdir, os.path.basename(s) + ".o")
        objs.append(o)
        if _newer(o, [s] + headers):
            todo.append((s, o))

    def compile_one(so):
        s, o = so
        lang = ["-x", "cu"] if s.endswith(".cpp") else []  # host files share the .cuh helpers
        return _run([NVCC] + NVCC_FLAGS + lang + ["-Xptxas", "-v" if verbose else "-O3", "-c", s, "-o", o])

    if todo:
        with cf.ThreadPoolExecutor(jobs or min(8, os.cpu_count() or 4)) as ex:
            for (s, _), log in zip(todo, ex.map(compile_one, todo)):
                if verbose:
                    print("compiled", os.path.basename(s))
                    if log.strip():
                        print(log)
    if todo or _newer(out, objs):
        _run([NVCC] + ARCH + ["-shared", "-ccbin", HOST_CXX, "-cudart", "static", "-o", out] + objs
             + ["-ldl", "-lpthread", "-lrt"])
        if verbose:
            print("linked", out)
    with open(stamp, "w") as fh:
        fh.write(digest)
    return out


def build(verbose=False) -> None:
    build_synth(verbose)
    build_tptc(verbose)


def clean() -> None:
    shutil.rmtree(os.path.join(BUILD, "tptc"), ignore_errors=True)
    for f in glob.glob(os.path.join(LIBDIR, "*.so")):
        os.remove(f)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
