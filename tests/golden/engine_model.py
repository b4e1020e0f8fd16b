"""A small seeded Llama-style model for the engine-level fixtures — TEST
INFRASTRUCTURE.

``model_tensors(seed)`` returns every tensor of a 2-layer model by its GGUF name
(``token_embd.weight``, ``blk.{l}.attn_q.weight``, ..., ``output.weight``) as
(raw bytes, GGML type id, (n, k) row-major shape): GGML-block weights drawn by
the oracle's ``random_weight`` (quantized types exercise every bit pattern of
their blocks), fp16 norm weights and an fp16 token-embedding table.  The same
function runs where the fixture is made (tests/golden/make_engine_golden.py, with
the reference) and where it is checked (the GPU tests), and ``digest`` pins the
bytes, so a change in the generator cannot pass silently.
"""

from __future__ import annotations

import hashlib

import numpy as np

import layer_ref as L

MODEL = dict(layers=2, hidden=128, intermediate=256, heads=4, kv_heads=2, vocab=64,
             eps=1e-5, rope_base=10000.0, neox=False)
# GGML type of each projection: q, k, v, o, gate, up, down; and of the LM head
TYPES = {"attn_q": L.Q4_0, "attn_k": L.Q4_0, "attn_v": L.Q8_0, "attn_output": L.Q4_0,
         "ffn_gate": L.Q4_0, "ffn_up": L.Q8_0, "ffn_down": L.Q8_0}
HEAD_TYPE = L.Q8_0
PROJ = ["attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"]


def proj_shape(name: str, m=MODEL):
    """(n, k) of a projection: rows of the output by the input width."""
    d = m["hidden"] // m["heads"]
    q_dim, kv_dim = m["heads"] * d, m["kv_heads"] * d
    return {"attn_q": (q_dim, m["hidden"]), "attn_k": (kv_dim, m["hidden"]),
            "attn_v": (kv_dim, m["hidden"]), "attn_output": (m["hidden"], q_dim),
            "ffn_gate": (m["intermediate"], m["hidden"]), "ffn_up": (m["intermediate"], m["hidden"]),
            "ffn_down": (m["hidden"], m["intermediate"])}[name]


def model_tensors(seed: int, m=MODEL):
    rng = np.random.default_rng(seed)
    t = {}
    hid = m["hidden"]
    emb = (rng.standard_normal((m["vocab"], hid), dtype=np.float32) * 0.5).astype(np.float16)
    t["token_embd.weight"] = (emb.view(np.uint8).reshape(-1), L.F16, (m["vocab"], hid))
    for layer in range(m["layers"]):
        p = f"blk.{layer}."
        for norm in ("attn_norm", "ffn_norm"):
            w = rng.uniform(0.8, 1.2, hid).astype(np.float16)
            t[p + norm + ".weight"] = (w.view(np.uint8), L.F16, (hid,))
        for name in PROJ:
            n, k = proj_shape(name, m)
            t[p + name + ".weight"] = (L.random_weight(rng, TYPES[name], n, k), TYPES[name], (n, k))
    w = rng.uniform(0.8, 1.2, hid).astype(np.float16)
    t["output_norm.weight"] = (w.view(np.uint8), L.F16, (hid,))
    t["output.weight"] = (L.random_weight(rng, HEAD_TYPE, m["vocab"], hid, scale=4.0), HEAD_TYPE,
                          (m["vocab"], hid))
    return t


def digest(tensors) -> str:
    h = hashlib.sha256()
    for name in sorted(tensors):
        raw, typ, shape = tensors[name]
        h.update(name.encode())
        h.update(str((typ, tuple(shape))).encode())
        h.update(np.ascontiguousarray(raw).tobytes())
    return h.hexdigest()
