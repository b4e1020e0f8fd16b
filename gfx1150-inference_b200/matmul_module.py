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
  forward_layer_cached(x_in, x_out, attn_norm_w, wq, wq_type, ..., rope_neox, scale)
                                                                         bindings.cpp:562-627
  rope(x_in, x_out, seq_len, num_heads, head_dim, pos_offset=0,
       freq_base=10000.0, neox_style=False)                              bindings.cpp:392-412

Array checks follow check_fp16_contiguous (bindings.cpp:20-38): a 2-byte float
dtype, C-contiguous, ``Out`` writeable, and at least the expected number of
elements, else ValueError.  Extension: a pool created with
``kv_cache_init_ex(..., dtype=numpy.float32)`` takes float32 arrays, and
``gqa_attention`` takes float32 arrays when all four are float32.

The KV-cache path and the layer that drives it live here; the reference
module's standalone host-buffer matmul, dequant, norm and SwiGLU entry points
(used by the per-op layer path) are not part of this library.
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


# GGML weight types forward_layer_cached takes: id -> (weights per block, bytes per block, name)
_WTYPES = {1: (1, 2, "F16"), 2: (32, 18, "Q4_0"), 8: (32, 34, "Q8_0"), 12: (256, 144, "Q4_K"),
           14: (256, 210, "Q6_K")}


def _check_weight_buffer(buf, w_type: int, n: int, k: int, name: str):
    """check_weight_buffer (bindings.cpp:518-557): C-contiguous buffer, known type,
    k divisible by the type's block, at least n · k / per · bytes bytes."""
    arr = buf if isinstance(buf, np.ndarray) else np.frombuffer(memoryview(buf), dtype=np.uint8)
    if arr.ndim > 0 and not arr.flags["C_CONTIGUOUS"]:
        raise ValueError(f"{name} buffer must be C-contiguous.")
    w_type = int(w_type)
    if w_type not in _WTYPES:
        raise ValueError(f"{name} has unsupported ggml_type.")
    per, nbytes, tname = _WTYPES[w_type]
    if w_type != 1 and (k <= 0 or k % per != 0):
        raise ValueError(f"{name} K must be divisible by {per} for {tname}.")
    expected = n * k * 2 if w_type == 1 else n * (k // per) * nbytes
    if arr.nbytes < expected:
        raise ValueError(f"{name} weight buffer is smaller than required.")
    return arr


def forward_layer_cached(x_in, x_out, attn_norm_w, wq, wq_type: int, wk, wk_type: int, wv,
                         wv_type: int, wo, wo_type: int, ffn_norm_w, wgate, wgate_type: int, wup,
                         wup_type: int, wdown, wdown_type: int, layer_idx: int, seq_len: int,
                         pos_offset: int, hidden_size: int, intermediate_size: int,
                         num_heads: int, num_kv_heads: int, head_dim: int, rms_norm_eps: float,
                         rope_freq_base: float, rope_neox: bool, scale: float) -> None:
    """Execute a full transformer layer on-device with the GPU-resident KV cache
    (bindings.cpp:562-627 ⇒ attention.hip:603-695): RMSNorm, q/k/v projections,
    RoPE, cached GQA attention (appending the rotated K rows and the V rows at
    pos_offset), output projection, residual + RMSNorm, SwiGLU FFN, residual.
    fp16 activations (seq_len, hidden_size); weights of GGML types F16 / Q4_0 /
    Q8_0 / Q4_K / Q6_K, copied to the device on every call like the reference."""
    hidden_elems = int(seq_len) * int(hidden_size)
    f16 = np.dtype(np.float16)
    x_in = _check_array(x_in, "x_in", hidden_elems, f16)
    x_out = _check_array(x_out, "x_out", hidden_elems, f16, require_writeable=True)
    attn_norm_w = _check_array(attn_norm_w, "attn_norm_w", int(hidden_size), f16)
    ffn_norm_w = _check_array(ffn_norm_w, "ffn_norm_w", int(hidden_size), f16)
    q_dim = int(num_heads) * int(head_dim)
    kv_dim = int(num_kv_heads) * int(head_dim)
    hs, inter = int(hidden_size), int(intermediate_size)
    ws = [
        _check_weight_buffer(wq, wq_type, q_dim, hs, "wq"),
        _check_weight_buffer(wk, wk_type, kv_dim, hs, "wk"),
        _check_weight_buffer(wv, wv_type, kv_dim, hs, "wv"),
        _check_weight_buffer(wo, wo_type, hs, q_dim, "wo"),
        _check_weight_buffer(wgate, wgate_type, inter, hs, "wgate"),
        _check_weight_buffer(wup, wup_type, inter, hs, "wup"),
        _check_weight_buffer(wdown, wdown_type, hs, inter, "wdown"),
    ]
    p = [_ffi.np_ptr(w) for w in ws]
    _ffi.check(_ffi.lib.kvc_forward_layer_cached(
        _ffi.np_ptr(x_in), _ffi.np_ptr(x_out), _ffi.np_ptr(attn_norm_w),
        p[0], int(wq_type), p[1], int(wk_type), p[2], int(wv_type), p[3], int(wo_type),
        _ffi.np_ptr(ffn_norm_w), p[4], int(wgate_type), p[5], int(wup_type), p[6], int(wdown_type),
        int(layer_idx), int(seq_len), int(pos_offset), hs, inter, int(num_heads),
        int(num_kv_heads), int(head_dim), float(rms_norm_eps), float(rope_freq_base),
        int(bool(rope_neox)), float(scale)))
