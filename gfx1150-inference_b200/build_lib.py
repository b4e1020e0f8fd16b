"""Build recipe for libkvcache.so (sm_100a) — the native side of this package.

Compiles csrc/*.cu and csrc/*.cpp with nvcc for ``-gencode
arch=compute_100a,code=sm_100a`` and links them, with the CUDA runtime linked
statically, into ``libkvcache.so`` next to this file, where ``kvcache_ffi``
loads it.  Objects go to ``_build/`` (git-ignored).  Run as a script or call
``build()``; rebuilds only when a source or header is newer than the library.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.abspath(os.path.join(HERE, "..", "include"))
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libkvcache.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
          "-I", CSRC, "-I", INCLUDE]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libkvcache.so")
    return cand


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _headers():
    out = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    out += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return out


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in _sources() + _headers() + [__file__])


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile libkvcache.so if needed; return its path."""
    if not force and not _stale():
        return LIB
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    objs = []
    jobs = []
    for src in _sources():
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        cmd = [nvcc, *ARCH, *COMMON, "-x", "cu", "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        jobs.append(cmd)

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r.stdout + r.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
        logs = list(ex.map(run, jobs))
    if verbose:
        for log in logs:
            sys.stdout.write(log)
    tmp = LIB + ".tmp"
    run([nvcc, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-lpthread", "-ldl", "-lrt"])
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
