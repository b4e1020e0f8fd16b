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

Host-streamed KV (``--offload-kv-cpu`` / ``--kv-mmap-dir``).  The reference's
KVCacheManager keeps K and V in two host arrays (num_layers, max_seq_len,
num_kv_heads, head_dim) (numpy, or memory-mapped files), writes each new row
there itself, and calls ``gqa_attention`` with the layer's view
``k_host[layer]`` and kv_len = start_pos + q_len (src/kv_cache.py:219-239).
``gqa_attention`` recognises such a pair of layer views (each a C-contiguous
(max_seq_len, num_kv_heads, head_dim) slice of one contiguous buffer of at least
two layers) and serves it from the library's offload engine (kvc_offload_*):
the host buffers are page-locked once (bounce buffers when they cannot be), the
layer's rows stream to the GPU on a copy stream, the next layer is prefetched
while this one attends, and rows below start_pos that an earlier call on the
layer already moved are reused (they are the KV history, which the manager
never rewrites).  Outputs are bit-identical to the stateless path and to the
GPU-resident pool.  A caller that rewrites history rows of such a buffer in
place calls ``offload_invalidate()`` afterwards; ``KVC_OFFLOAD_STREAM=0`` turns
the engine off (every call then copies its whole [0, kv_len) like the
reference).  The engine lives as long as both host arrays: it is released when
either is freed.  ``set_offload_mirror_bytes(n)`` (or ``KVC_OFFLOAD_MIRROR_BYTES``)
lets engines keep as many layers as n bytes of HBM hold resident on the device
(a B200's 180 GB often holds what a smaller GPU had to offload).

The KV-cache path and the layer that drives it live here; the reference
module's standalone host-buffer matmul, dequant, norm and SwiGLU entry points
(used by the per-op layer path) are not part of this library.
"""

from __future__ import annotations

import ctypes
import os
import threading
import weakref

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
    "rope",
    "forward_layer_cached",
    "offload_stats",
    "offload_invalidate",
    "set_offload_mirror_bytes",
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
    eng = _offload_engine_for(K, V, int(q_len), int(kv_len), int(start_pos), int(num_heads),
                              int(num_kv_heads), int(head_dim), dt)
    if eng is not None:
        eng.attend(Q, Out, int(q_len), int(start_pos), int(num_heads), float(scale),
                   bool(causal))
        return
    _ffi.check(_ffi.lib.kvc_gqa_attention_ex(
        _ffi.np_ptr(Q), _ffi.np_ptr(K), _ffi.np_ptr(V), _ffi.np_ptr(Out), int(q_len), int(kv_len),
        int(num_heads), int(num_kv_heads), int(head_dim), int(start_pos), float(scale),
        int(bool(causal)), _ffi.dtype_code_of(dt)))


# ---- host-streamed KV: layer views of a (num_layers, max_seq_len, Hkv, D) buffer ----
_ENGINES = {}                 # (id(K owner), id(V owner)) -> _OffloadEngine
_ENGINES_LOCK = threading.Lock()
_MIRROR_BYTES = [int(os.environ.get("KVC_OFFLOAD_MIRROR_BYTES", "0") or 0)]


def _owner(a: np.ndarray) -> np.ndarray:
    """The outermost ndarray of a view chain (the array whose memory ``a`` views)."""
    o = a
    while isinstance(o.base, np.ndarray):
        o = o.base
    return o


def host_layer_view(a, num_kv_heads: int, head_dim: int):
    """(owner, layer, num_layers, max_seq_len) when ``a`` is layer ``layer`` of a
    contiguous host buffer of num_layers >= 2 layers of (max_seq_len,
    num_kv_heads, head_dim) rows, the shape of KVCacheManager's host arrays
    (src/kv_cache.py:97) and of its views k_host[layer]; else None."""
    if (not isinstance(a, np.ndarray) or a.ndim != 3 or a.base is None
            or a.shape[1:] != (num_kv_heads, head_dim) or not a.flags["C_CONTIGUOUS"]
            or a.nbytes == 0):
        return None
    o = _owner(a)
    if o is a or not o.flags["C_CONTIGUOUS"]:
        return None
    # an (L, S, Hkv, D) array must be sliced along L; a flat buffer (the mmap
    # mode's np.frombuffer) is cut into whole layers of the view's size
    if o.ndim > 1 and (o.ndim != 4 or tuple(o.shape[1:]) != a.shape):
        return None
    off = a.ctypes.data - o.ctypes.data
    lb = a.nbytes
    if off < 0 or off % lb or o.nbytes % lb or off + lb > o.nbytes:
        return None
    n_layers = o.nbytes // lb
    if n_layers < 2:
        return None
    return o, off // lb, n_layers, a.shape[0]


class _OffloadEngine:
    """kvc_offload_* over a K / V pair of host buffers, released with either."""

    def __init__(self, ok: np.ndarray, ov: np.ndarray, num_layers: int, max_seq_len: int,
                 num_kv_heads: int, head_dim: int, dt: np.dtype, key):
        h = ctypes.c_void_p()
        _ffi.check(_ffi.lib.kvc_offload_create(
            ok.ctypes.data, ov.ctypes.data, num_layers, max_seq_len, num_kv_heads, head_dim,
            _ffi.dtype_code_of(dt), _ffi.OFFLOAD_REGISTER, -1, ctypes.byref(h)))
        self.handle = h
        self.key = key
        self.geom = (num_layers, max_seq_len, num_kv_heads, head_dim, dt)
        self.k_ptr, self.v_ptr = ok.ctypes.data, ov.ctypes.data
        self.lock = threading.Lock()
        if _MIRROR_BYTES[0] > 0:
            self.set_mirror(_MIRROR_BYTES[0])
        # released when either host array is freed (weak references only: holding
        # the arrays would keep memory-mapped files from being closed)
        self._refs = (weakref.ref(ok, self._gone), weakref.ref(ov, self._gone))

    def _gone(self, _ref=None):
        with _ENGINES_LOCK:
            if _ENGINES.get(self.key) is self:
                del _ENGINES[self.key]
        self.close()

    def close(self):
        with self.lock:
            if self.handle is None:
                return
            # the host arrays may be about to be freed: wait (again) while the
            # engine's copies are still in flight rather than leave them running
            for _ in range(1000):
                rc = _ffi.lib.kvc_offload_destroy(self.handle)
                if rc != _ffi.KVC_ERR_TIMEOUT:
                    break
            self.handle = None

    def set_mirror(self, budget: int) -> int:
        n = ctypes.c_int()
        with self.lock:
            _ffi.check(_ffi.lib.kvc_offload_set_mirror(self.handle, int(budget), ctypes.byref(n)))
        return n.value

    def attend(self, Q, Out, layer, q_len, start_pos, num_heads, scale, causal):
        with self.lock:
            _ffi.check(_ffi.lib.kvc_offload_attend(
                self.handle, _ffi.np_ptr(Q), None, None, _ffi.np_ptr(Out), layer, q_len,
                start_pos, num_heads, scale, int(causal)))

    def stats(self) -> dict:
        b, ms = ctypes.c_double(), ctypes.c_double()
        hits, calls = ctypes.c_int64(), ctypes.c_int64()
        nl, mb = ctypes.c_int(), ctypes.c_double()
        with self.lock:
            _ffi.check(_ffi.lib.kvc_offload_stats(self.handle, ctypes.byref(b), ctypes.byref(ms),
                                                  ctypes.byref(hits), ctypes.byref(calls)))
            _ffi.check(_ffi.lib.kvc_offload_mirror_stats(self.handle, ctypes.byref(nl),
                                                         ctypes.byref(mb)))
        return {"h2d_bytes": b.value, "h2d_ms": ms.value, "prefetch_hits": hits.value,
                "attend_calls": calls.value, "mirror_layers": nl.value,
                "mirror_bytes": mb.value}


def _offload_engine_for(K, V, q_len, kv_len, start_pos, num_heads, num_kv_heads, head_dim, dt):
    """The offload engine serving this gqa_attention call, or None for the
    stateless path (any other array layout, a non-cached call shape, or
    KVC_OFFLOAD_STREAM=0)."""
    if os.environ.get("KVC_OFFLOAD_STREAM", "1") == "0":
        return None
    if (q_len <= 0 or start_pos < 0 or kv_len != start_pos + q_len or num_kv_heads <= 0
            or num_heads <= 0 or num_heads % num_kv_heads or not 0 < head_dim <= 256):
        return None
    kv = host_layer_view(K, num_kv_heads, head_dim)
    vv = host_layer_view(V, num_kv_heads, head_dim)
    if kv is None or vv is None:
        return None
    (ok, layer, n_layers, max_seq), (ov, vlayer, vn_layers, vmax_seq) = kv, vv
    if (layer, n_layers, max_seq) != (vlayer, vn_layers, vmax_seq) or ok is ov:
        return None
    if kv_len > max_seq:
        return None
    key = (id(ok), id(ov))
    with _ENGINES_LOCK:
        eng = _ENGINES.get(key)
        if eng is not None and (eng.geom != (n_layers, max_seq, num_kv_heads, head_dim, dt)
                                or (eng.k_ptr, eng.v_ptr) != (ok.ctypes.data, ov.ctypes.data)):
            del _ENGINES[key]
            eng.close()
            eng = None
        if eng is None:
            eng = _OffloadEngine(ok, ov, n_layers, max_seq, num_kv_heads, head_dim, dt, key)
            _ENGINES[key] = eng
    return _EngineCall(eng, layer)


class _EngineCall:
    __slots__ = ("eng", "layer")

    def __init__(self, eng, layer):
        self.eng, self.layer = eng, layer

    def attend(self, Q, Out, q_len, start_pos, num_heads, scale, causal):
        self.eng.attend(Q, Out, self.layer, q_len, start_pos, num_heads, scale, causal)


def _engine_of(K):
    if K is None:
        with _ENGINES_LOCK:
            return list(_ENGINES.values())
    o = _owner(K) if isinstance(K, np.ndarray) else None
    with _ENGINES_LOCK:
        return [e for k, e in _ENGINES.items() if o is not None and k[0] == id(o)]


def offload_stats(K=None) -> dict:
    """Counters of the offload engine serving the host K buffer ``K`` (the
    (num_layers, ...) array or any of its layer views): bytes and copy-engine
    time of the streamed layers, prefetch hits, attend calls, mirrored layers and
    the bytes uploaded into the mirror.  Without ``K``: summed over all engines."""
    engines = _engine_of(K)
    tot = {"h2d_bytes": 0.0, "h2d_ms": 0.0, "prefetch_hits": 0, "attend_calls": 0,
           "mirror_layers": 0, "mirror_bytes": 0.0, "engines": len(engines)}
    for e in engines:
        for k, v in e.stats().items():
            tot[k] += v
    return tot


def offload_invalidate(K=None) -> None:
    """Forget the rows the offload engines hold for the host buffer ``K`` (all
    engines without it): call after rewriting KV history rows in place."""
    for e in _engine_of(K):
        with e.lock:
            _ffi.check(_ffi.lib.kvc_offload_invalidate(e.handle))


def set_offload_mirror_bytes(budget: int) -> None:
    """HBM budget of the offload engines' device mirror (0: none): applies to the
    engines alive now and to the ones created later."""
    budget = int(budget)
    if budget < 0:
        raise ValueError("the mirror budget must be non-negative")
    _MIRROR_BYTES[0] = budget
    for e in _engine_of(None):
        e.set_mirror(budget)


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
