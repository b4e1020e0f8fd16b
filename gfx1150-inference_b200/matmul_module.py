"""Drop-in replacement for the KV-cache entry points of gfx1150-inference's
pybind11 extension ``matmul_module`` (src/python_bindings/bindings.cpp).

Same names, positional order, defaults and error classes as the reference
(module definitions at bindings.cpp:775-791 and :801-831), backed by the
sm_100a library libkvcache.so through ``kvcache_ffi``:

  kv_cache_init(num_layers, max_seq_len, num_kv_heads, head_dim)        bindings.cpp:468-472
  kv_cache_free()                                                        bindings.cpp:474-478
  gqa_attention_cached(Q, K_new, V_new, Out, layer_idx, q_len, start_pos,
                       num_heads, num_kv_heads, head_dim, scale=0.0, causal=True)
                                                                         bindings.cpp:480-514
  gqa_attention(Q, K, V, Out, q_len, kv_len, num_heads, num_kv_heads, head_dim,
                start_pos=0, scale=0.0, causal=True)                     bindings.cpp:414-447

Array checks follow check_fp16_contiguous (bindings.cpp:20-38): a 2-byte float
dtype, C-contiguous, ``Out`` writeable, and at least the expected number of
elements, else ValueError.  Extension: a pool created with
``kv_cache_init_ex(..., dtype=numpy.float32)`` takes float32 arrays, and
``gqa_attention`` takes float32 arrays when all four are float32.

Only the KV-cache path lives here; the reference module's matmul, dequant,
norm, RoPE and SwiGLU kernels are not part of this library.
"""

from __future__ import annotations

import numpy as np

import kvcache_ffi as _ffi

__all__ = [
    "kv_cache_init",
    "kv_cache_init_ex",
    "kv_cache_free",
    "kv_cache_dtype",
    "kv_cache_gather",
    "gqa_attention_cached",
    "gqa_attention",
]


def _check_array(arr, name: str, min_elems: int, expect: np.dtype, require_writeable: bool = False):
    """check_fp16_contiguous (bindings.cpp:20-38), generalised to the pool dtype."""
    if not isinstance(arr, np.ndarray):
        if require_writeable:
            raise ValueError(f"{name} must be a writeable array.")
        arr = np.asarray(arr)
    if arr.dtype.kind != "f" or arr.dtype.itemsize != expect.itemsize:
        if expect == np.float16:
            raise ValueError(f"{name} must be a 2-byte FP16 (numpy.float16) array.")
        raise ValueError(f"{name} must be a {expect.itemsize}-byte {expect.name} array.")
    if not arr.flags["C_CONTIGUOUS"]:
        raise ValueError(f"{name} must be a C-contiguous array.")
    if require_writeable and not arr.flags["WRITEABLE"]:
        raise ValueError(f"{name} must be a writeable array.")
    if arr.size < min_elems:
        raise ValueError(f"{name} buffer is smaller than expected dimensions.")
    return arr


# Geometry of the live process-wide pool (for kv_cache_gather's output shape).
_POOL_SHAPE = {"num_kv_heads": None, "head_dim": None}


def kv_cache_init(num_layers: int, max_seq_len: int, num_kv_heads: int, head_dim: int) -> None:
    """Allocate GPU-resident GQA KV cache pool for all transformer layers (fp16)."""
    _ffi.check(_ffi.lib.kvc_cache_init(int(num_layers), int(max_seq_len), int(num_kv_heads),
                                       int(head_dim)))
    _POOL_SHAPE.update(num_kv_heads=int(num_kv_heads), head_dim=int(head_dim))


def kv_cache_init_ex(num_layers: int, max_seq_len: int, num_kv_heads: int, head_dim: int,
                     dtype=np.float16, page_size: int = 16) -> None:
    """kv_cache_init with a storage dtype (float16 / float32) and page size."""
    code = _ffi.dtype_code_of(np.dtype(dtype))
    _ffi.check(_ffi.lib.kvc_cache_init_ex(int(num_layers), int(max_seq_len), int(num_kv_heads),
                                          int(head_dim), code, int(page_size)))
    _POOL_SHAPE.update(num_kv_heads=int(num_kv_heads), head_dim=int(head_dim))


def kv_cache_free() -> None:
    """Free GPU-resident GQA KV cache pool."""
    _ffi.check(_ffi.lib.kvc_cache_free())
    _POOL_SHAPE.update(num_kv_heads=None, head_dim=None)


def kv_cache_dtype():
    """numpy dtype of the live pool, or None."""
    code = _ffi.lib.kvc_cache_dtype()
    return None if code < 0 else _ffi.np_dtype_of(code)


def _pool_dtype() -> np.dtype:
    code = _ffi.lib.kvc_cache_dtype()
    return _ffi.np_dtype_of(code) if code >= 0 else np.dtype(np.float16)


def gqa_attention_cached(Q, K_new, V_new, Out, layer_idx: int, q_len: int, start_pos: int,
                         num_heads: int, num_kv_heads: int, head_dim: int, scale: float = 0.0,
                         causal: bool = True) -> None:
    """Update GPU-resident KV cache at start_pos and run GQA online-softmax attention."""
    dt = _pool_dtype()
    q_elems = int(q_len) * int(num_heads) * int(head_dim)
    kv_new_elems = int(q_len) * int(num_kv_heads) * int(head_dim)
    Q = _check_array(Q, "Q", q_elems, dt)
    K_new = _check_array(K_new, "K_new", kv_new_elems, dt)
    V_new = _check_array(V_new, "V_new", kv_new_elems, dt)
    Out = _check_array(Out, "Out", q_elems, dt, require_writeable=True)
    _ffi.check(_ffi.lib.kvc_gqa_attention_cached(
        _ffi.np_ptr(Q), _ffi.np_ptr(K_new), _ffi.np_ptr(V_new), _ffi.np_ptr(Out),
        int(layer_idx), int(q_len), int(start_pos), int(num_heads), int(num_kv_heads),
        int(head_dim), float(scale), int(bool(causal))))


def gqa_attention(Q, K, V, Out, q_len: int, kv_len: int, num_heads: int, num_kv_heads: int,
                  head_dim: int, start_pos: int = 0, scale: float = 0.0,
                  causal: bool = True) -> None:
    """Grouped-Query Attention (GQA) with online softmax over host-resident K/V."""
    arr = Q if isinstance(Q, np.ndarray) else np.asarray(Q)
    dt = np.dtype(np.float32) if arr.dtype == np.float32 else np.dtype(np.float16)
    q_elems = int(q_len) * int(num_heads) * int(head_dim)
    kv_elems = int(kv_len) * int(num_kv_heads) * int(head_dim)
    Q = _check_array(Q, "Q", q_elems, dt)
    K = _check_array(K, "K", kv_elems, dt)
    V = _check_array(V, "V", kv_elems, dt)
    Out = _check_array(Out, "Out", q_elems, dt, require_writeable=True)
    _ffi.check(_ffi.lib.kvc_gqa_attention_ex(
        _ffi.np_ptr(Q), _ffi.np_ptr(K), _ffi.np_ptr(V), _ffi.np_ptr(Out), int(q_len), int(kv_len),
        int(num_heads), int(num_kv_heads), int(head_dim), int(start_pos), float(scale),
        int(bool(causal)), _ffi.dtype_code_of(dt)))


def rope(x_in, x_out, seq_len: int, num_heads: int, head_dim: int, pos_offset: int = 0,
         freq_base: float = 10000.0, neox_style: bool = False) -> None:
    """Rotary Positional Embeddings (bindings.cpp:392-412, defaults :763-774) on
    host fp16 arrays (seq_len, num_heads, head_dim); x_out may not alias x_in."""
    total = int(seq_len) * int(num_heads) * int(head_dim)
    x_in = _check_array(x_in, "x_in", total, np.dtype(np.float16))
    x_out = _check_array(x_out, "x_out", total, np.dtype(np.float16), require_writeable=True)
    _ffi.check(_ffi.lib.kvc_rope_host(_ffi.np_ptr(x_in), _ffi.np_ptr(x_out), int(seq_len),
                                      int(num_heads), int(head_dim), int(pos_offset),
                                      float(freq_base), int(bool(neox_style))))


def kv_cache_gather(layer_idx: int, start: int, count: int):
    """Copy positions [start, start+count) of a layer out of the pool as
    (count, num_kv_heads, head_dim) K and V arrays (bit-exact pool checks)."""
    code = _ffi.lib.kvc_cache_dtype()
    if code < 0 or _POOL_SHAPE["num_kv_heads"] is None:
        raise RuntimeError("Device KV cache not initialized. Call kv_cache_init first.")
    shape = (int(count), _POOL_SHAPE["num_kv_heads"], _POOL_SHAPE["head_dim"])
    k = np.empty(shape, dtype=_ffi.np_dtype_of(code))
    v = np.empty_like(k)
    _ffi.check(_ffi.lib.kvc_cache_gather(int(layer_idx), int(start), int(count), _ffi.np_ptr(k),
                                         _ffi.np_ptr(v)))
    return k, v
