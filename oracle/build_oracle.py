"""Build + load recipe of the C oracle (oracle/gqa_online.c) — TEST INFRASTRUCTURE.

``build()`` compiles ``oracle/liboracle.so`` with gcc and OpenMP; ``load()``
returns it through ctypes with argument types set.  Only tests/, smoke() and
bench.py's CPU baseline use it.

The reference's own kernel (src/kernels/attention.hip) is HIP C++ for gfx1150
and cannot be compiled here (no ROCm / hipcc), so there is no oracle/_ref
build; its algorithm is restated in gqa_online.c instead.
"""

from __future__ import annotations

import ctypes
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "gqa_online.c")
LIB = os.path.join(HERE, "liboracle.so")
FLAGS = ["-O3", "-std=gnu11", "-fPIC", "-shared", "-fopenmp", "-mavx2", "-mfma", "-mf16c",
         "-fno-math-errno"]


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC) \
            and os.path.getmtime(LIB) >= os.path.getmtime(__file__):
        return LIB
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("gcc is required to build the C oracle")
    tmp = LIB + ".tmp"
    subprocess.run([cc, *FLAGS, SRC, "-o", tmp, "-lm"], check=True)
    os.replace(tmp, LIB)
    return LIB


_lib = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(build())
        vp, ci, cf = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        for name in ("gqa_online_f16", "gqa_online_f32"):
            fn = getattr(lib, name)
            fn.restype = ci
            fn.argtypes = [vp, vp, vp, vp, ci, ci, ci, ci, ci, ci, cf, ci, ci]
        lib.gqa_decode_batch_f16.restype = ci
        lib.gqa_decode_batch_f16.argtypes = [ci, vp, ctypes.POINTER(vp), ctypes.POINTER(vp),
                                             ctypes.POINTER(ci), vp, ci, ci, ci, cf, ci]
        lib.gqa_max_threads.restype = ci
        lib.gqa_max_threads.argtypes = []
        _lib = lib
    return _lib


def gqa_online(Q, K, V, start_pos=0, scale=0.0, causal=True, threads=0):
    """numpy wrapper: fp16 or fp32 arrays, Q (q_len, H, D), K/V (kv_len, Hkv, D)."""
    import numpy as np

    lib = load()
    Q = np.ascontiguousarray(Q)
    K = np.ascontiguousarray(K)
    V = np.ascontiguousarray(V)
    q_len, H, D = Q.shape
    kv_len, Hkv, _ = K.shape
    out = np.empty_like(Q)
    fn = lib.gqa_online_f16 if Q.dtype == np.float16 else lib.gqa_online_f32
    rc = fn(Q.ctypes.data, K.ctypes.data, V.ctypes.data, out.ctypes.data, q_len, kv_len, H, Hkv, D,
            int(start_pos), float(scale), int(bool(causal)), int(threads or lib.gqa_max_threads()))
    if rc != 0:
        raise ValueError("invalid attention arguments")
    return out


if __name__ == "__main__":
    print(build(force=True))
