"""CPU oracle for the layer pipeline (forward_layer_cached) — TEST INFRASTRUCTURE ONLY.

Imported by tests/ (and the smoke check) as the checker; never by the product
path.  Parity pinned: tests/golden/layer_golden.npz holds outputs of the
reference's own numpy functions (gguf_parser.py dequantizers and quantizers,
tests/test_layer.py ref_rmsnorm / ref_rope / ref_gqa_attention / ref_swiglu),
made by tests/golden/make_layer_golden.py, and tests/test_oracle_golden.py
checks this module against them (dequantizers bit-exact).

What it restates:
  * GGML block formats and their dequantizers (gguf_parser.py:374-590): Q4_0
    (32 weights: fp16 d, 16 bytes of nibbles, w = d·(q − 8)), Q8_0 (32 weights:
    fp16 d, 32 int8, w = d·q), Q4_K (256 weights: fp16 d, fp16 dmin, 12 bytes of
    6-bit scales and mins, 128 bytes of nibbles; w = d·sc·q − dmin·m per 32),
    Q6_K (256 weights: 128 bytes low nibbles, 64 bytes high 2-bit pairs, 16
    int8 scales, fp16 d; w = d·sc·(q − 32) per 16).  Each computes in fp32 and
    rounds to fp16 like the reference.
  * The layer of launch_forward_layer_cached_fp16 (attention.hip:603-695) as
    the reference's CPU layer check composes it (test_layer.py:258-277):
    RMSNorm, q/k/v projections (fp32 products of fp16 activations and fp16
    dequantized weights, fp16 results), RoPE on q and k, cached GQA attention,
    output projection, residual + RMSNorm, SwiGLU FFN, residual.
"""

from __future__ import annotations

import numpy as np

import gqa_ref

# GGML type ids (the w_type arguments of forward_layer_cached, bindings.cpp:518-557)
F16, Q4_0, Q8_0, Q4_K, Q6_K = 1, 2, 8, 12, 14
BLOCK = {F16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}


def weight_bytes(w_type: int, n: int, k: int) -> int:
    """Bytes of an (n, k) weight matrix of w_type (bindings.cpp:518-557)."""
    per, nbytes = BLOCK[w_type]
    if k % per:
        raise ValueError(f"K must be divisible by {per} for type {w_type}")
    return n * (k // per) * nbytes


def _f16(raw: np.ndarray) -> np.ndarray:
    """Little-endian fp16 fields (..., 2) bytes → float32 (...)."""
    return np.ascontiguousarray(raw).view(np.float16)[..., 0].astype(np.float32)


def dequant_q4_0(raw: np.ndarray, n_elem: int) -> np.ndarray:
    b = np.frombuffer(raw, np.uint8, count=n_elem // 32 * 18).reshape(-1, 18)
    d = _f16(b[:, 0:2])[:, None]
    qs = b[:, 2:18]
    q = np.concatenate([qs & 0x0F, qs >> 4], axis=1).astype(np.float32) - 8.0
    return (q * d).reshape(-1).astype(np.float16)


def dequant_q8_0(raw: np.ndarray, n_elem: int) -> np.ndarray:
    b = np.frombuffer(raw, np.uint8, count=n_elem // 32 * 34).reshape(-1, 34)
    d = _f16(b[:, 0:2])[:, None]
    q = b[:, 2:34].view(np.int8).astype(np.float32)
    return (q * d).reshape(-1).astype(np.float16)


def q4_k_scales(sc12: np.ndarray):
    """6-bit scales and mins of the eight 32-weight groups (GGML's packing)."""
    s = sc12.astype(np.int32)
    sc = np.empty(s.shape[:-1] + (8,), np.float32)
    mn = np.empty_like(sc)
    for j in range(4):
        sc[..., j] = s[..., j] & 63
        mn[..., j] = s[..., j + 4] & 63
        sc[..., j + 4] = (s[..., j + 8] & 0x0F) | ((s[..., j] >> 6) << 4)
        mn[..., j + 4] = (s[..., j + 8] >> 4) | ((s[..., j + 4] >> 6) << 4)
    return sc, mn


def dequant_q4_k(raw: np.ndarray, n_elem: int) -> np.ndarray:
    b = np.frombuffer(raw, np.uint8, count=n_elem // 256 * 144).reshape(-1, 144)
    d = _f16(b[:, 0:2])[:, None]
    dmin = _f16(b[:, 2:4])[:, None]
    sc, mn = q4_k_scales(b[:, 4:16])
    qs = b[:, 16:144].reshape(-1, 4, 32)
    # group 2c takes the low nibbles of bytes 32c..32c+31, group 2c+1 the high ones
    q = np.stack([qs & 0x0F, qs >> 4], axis=2).reshape(-1, 8, 32).astype(np.float32)
    w = (d * sc)[:, :, None] * q - (dmin * mn)[:, :, None]
    return w.reshape(-1).astype(np.float16)


def dequant_q6_k(raw: np.ndarray, n_elem: int) -> np.ndarray:
    b = np.frombuffer(raw, np.uint8, count=n_elem // 256 * 210).reshape(-1, 210)
    ql = b[:, 0:128].astype(np.int32)
    qh = b[:, 128:192].astype(np.int32)
    sc = b[:, 192:208].view(np.int8).astype(np.float32)
    d = _f16(b[:, 208:210])[:, None]
    out = np.empty((b.shape[0], 256), np.float32)
    for h in range(2):  # two halves of 128 weights
        lo = ql[:, 64 * h: 64 * h + 64]
        hi = qh[:, 32 * h: 32 * h + 32]
        for t in range(4):  # quarter t: 32 weights
            nib = (lo[:, 32 * (t & 1): 32 * (t & 1) + 32] >> (4 * (t >> 1))) & 0x0F
            q = (nib | (((hi >> (2 * t)) & 0x03) << 4)) - 32
            for s in range(2):  # 16-weight groups with their own scale
                g = 8 * h + 2 * t + s
                out[:, 128 * h + 32 * t + 16 * s: 128 * h + 32 * t + 16 * s + 16] = (
                    d * sc[:, g:g + 1] * q[:, 16 * s: 16 * s + 16].astype(np.float32))
    return out.reshape(-1).astype(np.float16)


def dequantize(raw: np.ndarray, w_type: int, n: int, k: int) -> np.ndarray:
    """(n, k) fp16 weights from raw bytes of w_type."""
    if w_type == F16:
        return np.frombuffer(raw, np.float16, count=n * k).reshape(n, k).copy()
    fn = {Q4_0: dequant_q4_0, Q8_0: dequant_q8_0, Q4_K: dequant_q4_k, Q6_K: dequant_q6_k}[w_type]
    return fn(raw, n * k).reshape(n, k)


def linear(x: np.ndarray, raw: np.ndarray, w_type: int, n: int) -> np.ndarray:
    """x (M, K) fp16 @ W^T, W (n, K) dequantized to fp16; fp32 sums, fp16 out."""
    k = x.shape[-1]
    w = dequantize(raw, w_type, n, k).astype(np.float32)
    return (x.astype(np.float32) @ w.T).astype(np.float16)


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """rmsnorm.hip:23-74: x / sqrt(mean(x²) + eps) · w in fp32, fp16 out."""
    xf = x.astype(np.float32)
    rms = np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + np.float32(eps))
    return ((xf / rms) * w.astype(np.float32)).astype(np.float16)


def residual_add(x: np.ndarray, r: np.ndarray) -> np.ndarray:
    return (x.astype(np.float32) + r.astype(np.float32)).astype(np.float16)


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """mlp.hip:18-31: g / (1 + exp(-g)) · u in fp32, fp16 out."""
    g = gate.astype(np.float32)
    return (g / (np.float32(1.0) + np.exp(-g)) * up.astype(np.float32)).astype(np.float16)


class LayerWeights:
    """One layer's host buffers, as forward_layer_cached takes them."""

    def __init__(self, attn_norm, wq, wk, wv, wo, ffn_norm, wgate, wup, wdown):
        self.attn_norm, self.ffn_norm = attn_norm, ffn_norm
        self.w = {"q": wq, "k": wk, "v": wv, "o": wo, "gate": wgate, "up": wup, "down": wdown}


def layer_forward(x: np.ndarray, lw: LayerWeights, k_cache: np.ndarray, v_cache: np.ndarray,
                  pos_offset: int, num_heads: int, num_kv_heads: int, head_dim: int,
                  inter: int, eps: float, rope_base: float, neox: bool, scale: float):
    """One layer for x (seq, hidden) fp16 at positions pos_offset..; k_cache /
    v_cache (max_seq, Hkv, D) fp16 hold the earlier positions and receive the
    new rotated K rows and V rows (like the pool).  w entries are (raw, type)."""
    seq, hidden = x.shape
    H, Hkv, D = num_heads, num_kv_heads, head_dim
    nx = rmsnorm(x, lw.attn_norm, eps)
    q = linear(nx, *lw.w["q"], H * D).reshape(seq, H, D)
    k = linear(nx, *lw.w["k"], Hkv * D).reshape(seq, Hkv, D)
    v = linear(nx, *lw.w["v"], Hkv * D).reshape(seq, Hkv, D)
    inv_freq = gqa_ref.libm_inv_freq(rope_base, D)
    q_r = gqa_ref.ref_rope(q, pos_offset, rope_base, neox, inv_freq=inv_freq)
    k_r = gqa_ref.ref_rope(k, pos_offset, rope_base, neox, inv_freq=inv_freq)
    total = pos_offset + seq
    k_cache[pos_offset:total] = k_r
    v_cache[pos_offset:total] = v
    attn = gqa_ref.ref_gqa_attention(q_r, k_cache[:total], v_cache[:total], start_pos=pos_offset,
                                     scale=scale, causal=True)
    proj = linear(attn.reshape(seq, H * D).astype(np.float16), *lw.w["o"], hidden)
    h = residual_add(x, proj)
    nh = rmsnorm(h, lw.ffn_norm, eps)
    gate = linear(nh, *lw.w["gate"], inter)
    up = linear(nh, *lw.w["up"], inter)
    down = linear(swiglu(gate, up), *lw.w["down"], hidden)
    return residual_add(h, down)


def random_weight(rng: np.random.Generator, w_type: int, n: int, k: int,
                  scale: float = 1.0) -> np.ndarray:
    """Seeded raw bytes of an (n, k) weight of w_type whose weights are ~scale·N(0,1)/sqrt(k)
    in magnitude: random quants, fp16 block scales drawn so the dequantized values stay
    in range (every bit pattern of the quants and the 6-bit scale packing is exercised)."""
    per, nb = BLOCK[w_type]
    nblk = n * (k // per)
    s = scale / np.sqrt(k)
    if w_type == F16:
        return (rng.standard_normal((n, k), dtype=np.float32) * s).astype(np.float16).view(np.uint8).reshape(-1)
    raw = rng.integers(0, 256, size=(nblk, nb), dtype=np.uint8)

    def put_f16(col, vals):
        raw[:, col:col + 2] = np.asarray(vals, np.float16).reshape(-1, 1).view(np.uint8).reshape(-1, 2)

    if w_type == Q4_0:
        put_f16(0, rng.uniform(0.5, 1.5, nblk) * s / 4.0)
    elif w_type == Q8_0:
        put_f16(0, rng.uniform(0.5, 1.5, nblk) * s / 64.0)
    elif w_type == Q4_K:
        put_f16(0, rng.uniform(0.5, 1.5, nblk) * s / (8.0 * 32.0))
        put_f16(2, rng.uniform(0.5, 1.5, nblk) * s / 32.0)
    elif w_type == Q6_K:
        put_f16(208, rng.uniform(0.5, 1.5, nblk) * s / (32.0 * 64.0))
    return raw.reshape(-1)
