"""Seeded input generators of the golden cases (shared by make_golden.py and the tests).

Each case regenerates its inputs from a numpy seed exactly like the reference's
GPU tests do (``rng.standard_normal(shape, dtype=np.float32) * 0.5`` then a
cast, tests/test_layer.py:164-166, tests/test_full_model.py:89-91); the golden
file stores the reference outputs and a SHA-256 of the regenerated inputs, so a
change in the generator cannot pass silently.
"""

from __future__ import annotations

import hashlib
import math
import os

import numpy as np

GOLDEN_FILE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "gqa_golden.npz")


def _draw(rng, shape, scale, dtype):
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)).astype(dtype)


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def layer_cases():
    """tests/test_layer.py:155-184: H=16, Hkv=4, D=64, seed 30, 0.5 * N(0,1) fp16;
    case A causal prefill (q=12, kv=12, start 0), case B decode (q=1, kv=25, start 24)."""
    rng = np.random.default_rng(30)
    H, Hkv, D = 16, 4, 64
    out = []
    for q_len, kv_len, start in [(12, 12, 0), (1, 25, 24)]:
        Q = _draw(rng, (q_len, H, D), 0.5, np.float16)
        K = _draw(rng, (kv_len, Hkv, D), 0.5, np.float16)
        V = _draw(rng, (kv_len, Hkv, D), 0.5, np.float16)
        out.append(dict(Q=Q, K=K, V=V, q_len=q_len, kv_len=kv_len, start_pos=start,
                        scale=1.0 / math.sqrt(D), causal=True))
    return out


def kv_manager_case():
    """tests/test_full_model.py:78-129: L=2, S=32, H=8, Hkv=2, D=32, seed 19,
    6 positions per layer of 0.5 * N(0,1) fp16."""
    rng = np.random.default_rng(19)
    L, T, H, Hkv, D = 2, 6, 8, 2, 32
    Q = _draw(rng, (L, T, H, D), 0.5, np.float16)
    K = _draw(rng, (L, T, Hkv, D), 0.5, np.float16)
    V = _draw(rng, (L, T, Hkv, D), 0.5, np.float16)
    return dict(Q=Q, K=K, V=V, num_layers=L, max_seq_len=32, num_heads=H, num_kv_heads=Hkv,
                head_dim=D, scale=1.0 / math.sqrt(D))


def config1_case():
    """benchmark config 1 (TinyLlama-1.1B geometry, one layer): 32 q-heads, 4 KV
    heads, D=64, batch 1, 511 cached + 1 appended positions, fp32 N(0,1), scale
    1/sqrt(64), causal over 512 positions (seed 1)."""
    rng = np.random.default_rng(1)
    H, Hkv, D, P = 32, 4, 64, 512
    Q = _draw(rng, (1, H, D), 1.0, np.float32)
    K = _draw(rng, (P, Hkv, D), 1.0, np.float32)
    V = _draw(rng, (P, Hkv, D), 1.0, np.float32)
    return dict(Q=Q, K=K, V=V, q_len=1, kv_len=P, start_pos=P - 1, scale=1.0 / math.sqrt(D),
                causal=True)


# name -> (H, Hkv, D, q_len, kv_len, start_pos, scale or None (= 1/sqrt(D)), causal, seed, dtype)
EDGE_CASES = {
    "mha_g1_d128": (4, 4, 128, 1, 300, 299, None, True, 101, np.float16),
    "g8_d128_decode": (16, 2, 128, 1, 777, 776, None, True, 102, np.float16),
    "noncausal_prefill": (8, 2, 64, 5, 40, 35, None, False, 103, np.float16),
    "scale_custom": (8, 2, 64, 1, 97, 96, 0.3, True, 104, np.float16),
    "prefill_engine_dims": (4, 2, 32, 20, 20, 0, None, True, 105, np.float16),
    "split_boundary_1025": (8, 2, 128, 1, 1025, 1024, None, True, 106, np.float16),
    "g8_d64_fp32": (16, 2, 64, 1, 600, 599, None, True, 107, np.float32),
    "d256_decode": (4, 1, 256, 1, 130, 129, None, True, 108, np.float16),
}


def edge_case(name):
    H, Hkv, D, q_len, kv_len, start, scale, causal, seed, dtype = EDGE_CASES[name]
    rng = np.random.default_rng(seed)
    Q = _draw(rng, (q_len, H, D), 0.5, dtype)
    K = _draw(rng, (kv_len, Hkv, D), 0.5, dtype)
    V = _draw(rng, (kv_len, Hkv, D), 0.5, dtype)
    return dict(Q=Q, K=K, V=V, q_len=q_len, kv_len=kv_len, start_pos=start,
                scale=(1.0 / math.sqrt(D)) if scale is None else scale, causal=causal)


# Ragged batch: one decode query per sequence, lengths straddling page (16) and
# split (512) boundaries; H=8, Hkv=2, D=128, fp16, seed 7.
RAGGED_LENS = [1, 2, 15, 16, 17, 255, 511, 512, 513, 1100]


def ragged_case():
    rng = np.random.default_rng(7)
    H, Hkv, D = 8, 2, 128
    q = _draw(rng, (len(RAGGED_LENS), H, D), 0.5, np.float16)
    ks = [_draw(rng, (c, Hkv, D), 0.5, np.float16) for c in RAGGED_LENS]
    vs = [_draw(rng, (c, Hkv, D), 0.5, np.float16) for c in RAGGED_LENS]
    return dict(q=q, ks=ks, vs=vs, ctx=list(RAGGED_LENS), scale=1.0 / math.sqrt(D), H=H,
                Hkv=Hkv, D=D)


def load_golden():
    return dict(np.load(GOLDEN_FILE, allow_pickle=False))


def rope_cases():
    """tests/test_layer.py:134-152: seed 20, 16 heads x 64, N(0,1) fp16, interleaved
    and NeoX, (seq 8, offset 0) and (seq 1, offset 17); plus long-context decode
    positions (one token at 4095, 32768, 131072) and head_dim 128 (seed 21)."""
    out = []
    rng = np.random.default_rng(20)
    for neox in (False, True):
        for seq_len, pos in [(8, 0), (1, 17)]:
            x = _draw(rng, (seq_len, 16, 64), 1.0, np.float16)
            out.append(dict(x=x, pos_offset=pos, freq_base=10000.0, neox=neox))
    rng = np.random.default_rng(21)
    for neox in (False, True):
        for pos, base in [(4095, 10000.0), (32768, 500000.0), (131072, 500000.0)]:
            x = _draw(rng, (1, 8, 128), 1.0, np.float16)
            out.append(dict(x=x, pos_offset=pos, freq_base=base, neox=neox))
    return out
