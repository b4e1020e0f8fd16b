"""Generate tests/golden/engine_golden.npz by running the REFERENCE's engine.

Usage:  PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_engine_golden.py --reference <checkout>

The reference's unchanged ``LlamaInferenceEngine`` (src/inference.py) runs
greedy ``generate_batch_ids`` — its sequential loop over the prompts,
src/inference.py:415-457 — on a GGUF file written with the reference's own
``write_synthetic_gguf`` from the seeded model of tests/golden/engine_model.py.
The ``matmul_module`` it imports is a CPU stand-in computing with this
repository's oracle (oracle/layer_ref.py, pinned to the reference's numpy
functions): ``forward_layer_cached`` (the GPU-mode layer, layer.py:221-263)
keeps a numpy KV cache per layer, and ``rmsnorm`` / ``matmul_*`` serve the final
norm and the LM head (inference.py:233-253).

Stored: the seed and the model digest, the prompts, the reference's generated
token ids, the smallest top-1 / top-2 logit gap seen (seeds are tried until it is
large enough that the GPU's rounding cannot flip a token), and every
``forward_layer_cached`` call layer.py made (activations in, the oracle's output,
and the scalar arguments), for the GPU replay of that call site.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import engine_model as EM  # noqa: E402
import layer_ref as LR  # noqa: E402

OUT = os.path.join(HERE, "engine_golden.npz")
PROMPTS = [[3, 17, 42, 5, 9], [11, 2, 60], [7, 7, 30, 31, 4, 50, 23], [1]]
MAX_NEW = 8
MIN_GAP = 0.05


class OracleMatmulModule:
    """CPU stand-in for matmul_module, computing with the oracle; records the
    forward_layer_cached calls it receives."""

    def __init__(self):
        self.k = self.v = None
        self.calls = []

    def kv_cache_init(self, L, S, Hkv, D):
        self.k = np.zeros((L, S, Hkv, D), np.float16)
        self.v = np.zeros((L, S, Hkv, D), np.float16)

    def kv_cache_free(self):
        self.k = self.v = None

    def forward_layer_cached(self, x_in, x_out, attn_norm_w, wq, wq_type, wk, wk_type, wv,
                             wv_type, wo, wo_type, ffn_norm_w, wgate, wgate_type, wup, wup_type,
                             wdown, wdown_type, layer_idx, seq_len, pos_offset, hidden_size,
                             intermediate_size, num_heads, num_kv_heads, head_dim, rms_norm_eps,
                             rope_freq_base, rope_neox, scale):
        def raw(w):
            return np.frombuffer(memoryview(np.ascontiguousarray(w)), dtype=np.uint8)

        lw = LR.LayerWeights(np.asarray(attn_norm_w, np.float16), (raw(wq), wq_type),
                             (raw(wk), wk_type), (raw(wv), wv_type), (raw(wo), wo_type),
                             np.asarray(ffn_norm_w, np.float16), (raw(wgate), wgate_type),
                             (raw(wup), wup_type), (raw(wdown), wdown_type))
        x = np.asarray(x_in, np.float16).reshape(seq_len, hidden_size)
        y = LR.layer_forward(x, lw, self.k[layer_idx], self.v[layer_idx], pos_offset, num_heads,
                             num_kv_heads, head_dim, intermediate_size, rms_norm_eps,
                             rope_freq_base, bool(rope_neox), scale)
        x_out[...] = y.reshape(x_out.shape)
        self.calls.append(dict(
            x_in=x.copy(), out=y.copy(),
            args=[int(layer_idx), int(seq_len), int(pos_offset), int(hidden_size),
                  int(intermediate_size), int(num_heads), int(num_kv_heads), int(head_dim),
                  float(rms_norm_eps), float(rope_freq_base), bool(rope_neox), float(scale)],
            types=[int(wq_type), int(wk_type), int(wv_type), int(wo_type), int(wgate_type),
                   int(wup_type), int(wdown_type)]))

    def rmsnorm(self, x, w, out, rows, hidden, eps):
        out[...] = LR.rmsnorm(np.asarray(x, np.float16).reshape(rows, hidden),
                              np.asarray(w, np.float16), eps).reshape(out.shape)

    def _mm(self, w_type, x, w, out, M, N, K):
        raw = np.frombuffer(memoryview(np.ascontiguousarray(w)), dtype=np.uint8)
        out[...] = LR.linear(np.asarray(x, np.float16).reshape(M, K), raw, w_type, N).reshape(out.shape)

    def matmul_q4_0(self, *a):
        self._mm(LR.Q4_0, *a)

    def matmul_q8_0(self, *a):
        self._mm(LR.Q8_0, *a)

    def matmul_q4_k(self, *a):
        self._mm(LR.Q4_K, *a)

    def matmul_q6_k(self, *a):
        self._mm(LR.Q6_K, *a)

    def matmul_nt(self, *a):
        self._mm(LR.F16, *a)


def write_model(path, tensors, gg, m=EM.MODEL):
    V = gg.GGUFValueType
    meta = {
        "general.architecture": (V.STRING, "llama"),
        "llama.block_count": (V.UINT32, m["layers"]),
        "llama.embedding_length": (V.UINT32, m["hidden"]),
        "llama.feed_forward_length": (V.UINT32, m["intermediate"]),
        "llama.attention.head_count": (V.UINT32, m["heads"]),
        "llama.attention.head_count_kv": (V.UINT32, m["kv_heads"]),
        "llama.rope.dimension_count": (V.UINT32, m["hidden"] // m["heads"]),
        "llama.attention.layer_norm_rms_epsilon": (V.FLOAT32, m["eps"]),
        "llama.rope.freq_base": (V.FLOAT32, m["rope_base"]),
    }
    items = []
    for name, (raw, typ, shape) in tensors.items():
        dims = tuple(reversed(shape))  # GGUF lists the fastest dimension first
        items.append((name, dims, gg.GGMLType(typ), np.ascontiguousarray(raw).tobytes()))
    with open(path, "wb") as f:
        gg.write_synthetic_gguf(f, meta, items)


class _Dispatch:
    """The ``matmul_module`` the reference's modules import once: forwards to the
    stand-in of the current run."""

    target = None

    def __getattr__(self, name):
        return getattr(type(self).target, name)


def run_reference(root, seed):
    stub = OracleMatmulModule()
    _Dispatch.target = stub
    if not isinstance(sys.modules.get("matmul_module"), _Dispatch):
        sys.modules["matmul_module"] = _Dispatch()
    if os.path.join(root, "src") not in sys.path:
        sys.path.insert(0, os.path.join(root, "src"))
    import gguf_parser as gg  # the reference's
    import inference  # the reference's engine, unchanged

    tensors = EM.model_tensors(seed)
    gaps = []
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "model.gguf")
        write_model(path, tensors, gg)
        with inference.LlamaInferenceEngine(path, max_seq_len=32) as eng:
            assert eng.kv_cache.mode == "gpu" and eng.layer_cfg.head_dim == 32
            fwd = eng.forward_tokens

            def forward_tokens(*a, **k):  # the logits every sampling step sees
                logits = fwd(*a, **k)
                if logits is not None:
                    top = np.sort(logits.astype(np.float32))[-2:]
                    gaps.append(float(top[1] - top[0]))
                return logits

            eng.forward_tokens = forward_tokens
            outs, _ = eng.generate_batch_ids(PROMPTS, max_new_tokens=MAX_NEW, temperature=0.0,
                                             stop_on_eos=False)
    return tensors, outs, min(gaps), stub.calls


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="gfx1150-inference source checkout")
    args = ap.parse_args()
    root = os.path.abspath(args.reference)
    for seed in range(100):
        tensors, outs, gap, calls = run_reference(root, seed)
        if gap >= MIN_GAP:
            break
    else:
        raise SystemExit("no seed gives a safe logit gap")
    g = {"meta": np.array(json.dumps({
        "seed": seed, "digest": EM.digest(tensors), "model": EM.MODEL, "prompts": PROMPTS,
        "max_new_tokens": MAX_NEW, "tokens": outs, "min_logit_gap": gap,
        "calls": [dict(args=c["args"], types=c["types"]) for c in calls],
        "source": "reference src/inference.py generate_batch_ids (greedy), src/layer.py "
                  "forward_layer_cached call site; matmul_module = oracle/layer_ref.py"}))}
    for i, c in enumerate(calls):
        g[f"call{i}_x"] = c["x_in"]
        g[f"call{i}_out"] = c["out"]
    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT}: seed {seed}, tokens {outs}, min gap {gap:.4f}, {len(calls)} layer calls, "
          f"{os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    main()
