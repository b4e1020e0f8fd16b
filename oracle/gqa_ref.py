"""CPU oracle for the KV-cache decode path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this module, and only as the checker (or the timed CPU baseline); the product
path never calls it.

Restatements of the reference's own CPU code for this path
(KupipiKuki/gfx1150-inference):

* ``ref_gqa_attention`` — tests/test_layer.py:76-105, the numpy oracle the
  reference's GPU tests compare against: fp32 math per (query m, q-head h),
  kv_h = h // group, causal bound min(kv_len, start_pos + m + 1), max-subtracted
  softmax, result cast to fp16 (``out_dtype=np.float16``, the reference) or kept
  in fp32 (``out_dtype=np.float32``, used for the fp32 configuration whose
  tolerance is 1e-5).  Like the reference function, ``scale == 0`` selects
  1/sqrt(head_dim) (test_layer.py:87-88).
* ``online_softmax_attention`` — the serial online-softmax recurrence of the
  reference HIP kernel gqa_online_softmax_kernel (src/kernels/attention.hip:
  35-123), vectorised over heads: it uses ``scale`` exactly as given (0 means
  equal scores, attention.hip:99) and returns 0 when nothing is attended
  (attention.hip:115).
* ``append_rows`` — the host-mode append of KVCacheManager.attend
  (src/kv_cache.py:222-225): plain slice assignment into (L, S, Hkv, D) arrays.
* ``ref_rope`` — tests/test_layer.py:44-73, the numpy oracle of the reference's
  rope kernel (src/kernels/rope.hip:21-55): fp32 inv_freq = 1 / base^(2i/D),
  angle = position * inv_freq, pairs (2i, 2i+1) or (i, i+D/2) for NeoX, result
  cast to fp16.  ``positions`` extends it to one position per token (a batch of
  sequences at different positions), which the reference has no call for.

Pinning: tests/test_oracle_golden.py checks ``ref_gqa_attention``,
``online_softmax_attention`` and ``ref_rope`` against golden vectors produced by
importing the reference's own ``ref_gqa_attention`` and ``ref_rope``
(tests/golden/make_golden.py).
"""

from __future__ import annotations

import math

import numpy as np


def ref_gqa_attention(Q, K, V, start_pos: int = 0, scale: float = 0.0, causal: bool = True,
                      out_dtype=np.float16) -> np.ndarray:
    """tests/test_layer.py:76-105 restated; Q (q_len, H, D), K/V (kv_len, Hkv, D)."""
    q_len, num_heads, head_dim = Q.shape
    kv_len, num_kv_heads, _ = K.shape
    group_size = num_heads // num_kv_heads
    if scale == 0.0:
        scale = 1.0 / math.sqrt(head_dim)
    q = np.asarray(Q, dtype=np.float32)
    k = np.asarray(K, dtype=np.float32)
    v = np.asarray(V, dtype=np.float32)
    out = np.zeros(q.shape, dtype=np.float32)
    for m in range(q_len):
        max_kv = min(kv_len, start_pos + m + 1) if causal else kv_len
        for h in range(num_heads):
            kv_h = h // group_size
            scores = (k[:max_kv, kv_h, :] @ q[m, h, :]) * np.float32(scale)
            scores -= np.max(scores)
            probs = np.exp(scores)
            probs /= np.sum(probs)
            out[m, h, :] = probs @ v[:max_kv, kv_h, :]
    return out.astype(out_dtype)


def online_softmax_attention(Q, K, V, start_pos: int = 0, scale: float = 0.0,
                             causal: bool = True, out_dtype=np.float32) -> np.ndarray:
    """gqa_online_softmax_kernel (attention.hip:35-123): serial online softmax."""
    q_len, num_heads, head_dim = Q.shape
    kv_len, num_kv_heads, _ = K.shape
    group = num_heads // num_kv_heads
    q = np.asarray(Q, dtype=np.float32)
    k = np.asarray(K, dtype=np.float32)
    v = np.asarray(V, dtype=np.float32)
    out = np.zeros(q.shape, dtype=np.float32)
    sc = np.float32(scale)
    for m in range(q_len):
        max_kv = min(kv_len, start_pos + m + 1) if causal else kv_len
        for h in range(num_heads):
            kv_h = h // group
            m_prev = np.float32(-np.finfo(np.float32).max)
            l_prev = np.float32(0.0)
            acc = np.zeros(head_dim, dtype=np.float32)
            for s in range(max_kv):
                score = np.float32(np.dot(q[m, h], k[s, kv_h])) * sc
                m_new = max(m_prev, score)
                e_prev = np.float32(math.exp(m_prev - m_new))
                e_cur = np.float32(math.exp(score - m_new))
                l_prev = l_prev * e_prev + e_cur
                acc = acc * e_prev + e_cur * v[s, kv_h]
                m_prev = m_new
            inv_l = np.float32(1.0) / l_prev if l_prev > 0 else np.float32(0.0)
            out[m, h] = acc * inv_l
    return out.astype(out_dtype)


def append_rows(k_host: np.ndarray, v_host: np.ndarray, layer: int, start_pos: int,
                k_new: np.ndarray, v_new: np.ndarray) -> None:
    """kv_cache.py:222-225: k_layer[start_pos:total] = k_new (and V)."""
    total = start_pos + k_new.shape[0]
    k_host[layer][start_pos:total] = k_new
    v_host[layer][start_pos:total] = v_new


def batched_decode(q, ks, vs, ctx_lens, scale: float, out_dtype=np.float32) -> np.ndarray:
    """One decode step for a batch of independent sequences: query i attends over
    positions [0, ctx_lens[i]) of its own K/V (the reference processes the same
    sequences one at a time, src/inference.py:435-447)."""
    n, num_heads, head_dim = q.shape
    out = np.zeros((n, num_heads, head_dim), dtype=np.float32)
    for i in range(n):
        c = int(ctx_lens[i])
        out[i] = ref_gqa_attention(q[i:i + 1], ks[i][:c], vs[i][:c], start_pos=c - 1,
                                   scale=scale, causal=True, out_dtype=np.float32)[0]
    return out.astype(out_dtype)


def ref_rope(x, pos_offset: int = 0, freq_base: float = 10000.0, neox_style: bool = False,
             positions=None, out_dtype=np.float16, inv_freq=None) -> np.ndarray:
    """tests/test_layer.py:44-73 restated; x (tokens, heads, D).  Token t sits at
    positions[t] when given, else pos_offset + t.  ``inv_freq`` replaces the
    numpy power table (e.g. with the libm ``powf`` table rope.hip:79-83 builds on
    the host: the two differ by an ulp in some entries, which a large position
    turns into a visible angle difference)."""
    n, heads, head_dim = x.shape
    half = head_dim // 2
    xf = x.astype(np.float32)
    i = np.arange(half, dtype=np.float32)
    if inv_freq is None:
        inv_freq = np.float32(1.0) / (np.float32(freq_base) ** (np.float32(2.0) * i / np.float32(head_dim)))
    inv_freq = np.asarray(inv_freq, dtype=np.float32)
    if positions is None:
        pos = np.arange(pos_offset, pos_offset + n, dtype=np.float32)
    else:
        pos = np.asarray(positions, dtype=np.float32)
    ang = pos[:, None] * inv_freq[None, :]
    cs = np.cos(ang)[:, None, :]
    sn = np.sin(ang)[:, None, :]
    if neox_style:
        v0, v1 = xf[:, :, :half], xf[:, :, half:]
    else:
        v0, v1 = xf[:, :, 0::2], xf[:, :, 1::2]
    r0 = v0 * cs - v1 * sn
    r1 = v0 * sn + v1 * cs
    out = np.empty_like(xf)
    if neox_style:
        out[:, :, :half], out[:, :, half:] = r0, r1
    else:
        out[:, :, 0::2], out[:, :, 1::2] = r0, r1
    return out.astype(out_dtype)


def libm_inv_freq(freq_base: float, head_dim: int) -> np.ndarray:
    """inv_freq[i] = 1 / powf(freq_base, 2i / head_dim) with the C library's powf,
    the host table of rope.hip:79-83."""
    import ctypes
    import ctypes.util

    libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
    libm.powf.restype = ctypes.c_float
    libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    out = np.empty(head_dim // 2, dtype=np.float32)
    for i in range(head_dim // 2):
        e = np.float32(np.float32(2 * i) / np.float32(head_dim))
        out[i] = np.float32(1.0) / np.float32(libm.powf(float(freq_base), float(e)))
    return out
