"""generate_batch_ids on the paged pool, and the layer.py call site, against the
reference's own engine.

tests/golden/engine_golden.npz (tests/golden/make_engine_golden.py) holds what
the reference's unchanged LlamaInferenceEngine did on a seeded 2-layer model:
the greedy tokens of ``generate_batch_ids`` (its sequential loop over the
prompts, src/inference.py:415-457) and every ``forward_layer_cached`` call its
layer.py made (src/layer.py:221-263) with the oracle's output.  Here:

* ``batch_generate.BatchGenerator`` — all prompts advancing together through
  ``kvc_forward_layer_paged`` — yields exactly the reference's tokens, with whole
  and chunked prefill, and with EOS stopping;
* the recorded layer.py calls replayed in order through this repository's
  ``matmul_module.forward_layer_cached`` (the reference's argument order) match
  the oracle's outputs within the layer tests' bound, 5e-3 * max(1, max|ref|).
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import HAS_GPU

pytestmark = pytest.mark.gpu

if HAS_GPU:
    import torch

    import batch_generate as BG
    import engine_model as EM
    import kvcache_ffi as ffi
    import matmul_module

GOLDEN = None


def _golden():
    global GOLDEN
    if GOLDEN is None:
        import os

        path = os.path.join(os.path.dirname(__file__), "golden", "engine_golden.npz")
        z = np.load(path)
        GOLDEN = (json.loads(str(z["meta"])), z)
    return GOLDEN


def _model():
    meta, _ = _golden()
    tensors = EM.model_tensors(meta["seed"])
    assert EM.digest(tensors) == meta["digest"], "the seeded model changed"
    m = meta["model"]
    cfg = BG.ModelConfig(layers=m["layers"], hidden=m["hidden"], intermediate=m["intermediate"],
                         heads=m["heads"], kv_heads=m["kv_heads"],
                         head_dim=m["hidden"] // m["heads"], vocab=m["vocab"], eps=m["eps"],
                         rope_base=m["rope_base"], rope_neox=m["neox"])
    return cfg, tensors


@pytest.fixture(autouse=True)
def _clean(cuda_device):
    yield
    matmul_module.kv_cache_free()
    torch.cuda.synchronize()
    assert ffi.device_error(0, clear=True) == (0, 0)


def test_batched_generation_yields_the_reference_sequential_tokens():
    meta, _ = _golden()
    cfg, tensors = _model()
    model = BG.BatchModel.from_tensors(cfg, tensors)
    gen = BG.BatchGenerator(model, max_batch=4, max_seq_len=32)
    try:
        want = meta["tokens"]
        got, m = gen.generate_batch_ids(meta["prompts"], max_new_tokens=meta["max_new_tokens"],
                                        temperature=0.0, stop_on_eos=False)
        assert got == want
        assert m["batch_size"] == 4 and m["total_tokens_generated"] == sum(map(len, want))
        # chunked prefill (prefill_tokens' chunk_size) gives the same tokens
        got, _ = gen.generate_batch_ids(meta["prompts"], max_new_tokens=meta["max_new_tokens"],
                                        temperature=0.0, stop_on_eos=False, prefill_chunk_size=2)
        assert got == want
        # EOS: a sequence stops right after emitting it (generate_ids' loop)
        model.cfg.eos_token_id = 37
        got, _ = gen.generate_batch_ids(meta["prompts"], max_new_tokens=meta["max_new_tokens"],
                                        temperature=0.0, stop_on_eos=True)
        expect = [w[:w.index(37) + 1] if 37 in w else w for w in want]
        assert got == expect
        # the reference's argument checks
        with pytest.raises(ValueError):
            gen.generate_batch_ids([[]], max_new_tokens=2)
        with pytest.raises(ValueError):
            gen.generate_batch_ids([[1] * 30], max_new_tokens=8)
        with pytest.raises(ValueError):
            gen.generate_batch_ids(meta["prompts"], temperature=0.7)  # needs a sampler
    finally:
        gen.close()


def test_layer_py_call_site_replays_through_forward_layer_cached():
    meta, z = _golden()
    cfg, tensors = _model()
    calls = meta["calls"]
    matmul_module.kv_cache_init(cfg.layers, 32, cfg.kv_heads, cfg.head_dim)
    for i, c in enumerate(calls):
        (layer, seq_len, pos, hidden, inter, H, Hkv, D, eps, base, neox, scale) = c["args"]
        p = f"blk.{layer}."

        def w(name):
            raw, typ, _ = tensors[p + name + ".weight"]
            return raw, typ

        norm = {n: tensors[p + n + ".weight"][0].view(np.float16) for n in ("attn_norm", "ffn_norm")}
        x = z[f"call{i}_x"]
        out = np.empty_like(x)
        (wq, tq), (wk, tk), (wv, tv), (wo, to), (wg, tg), (wu, tu), (wd, td) = (
            w(n) for n in EM.PROJ)
        assert [tq, tk, tv, to, tg, tu, td] == c["types"]
        matmul_module.forward_layer_cached(
            x, out, norm["attn_norm"], wq, tq, wk, tk, wv, tv, wo, to, norm["ffn_norm"], wg, tg,
            wu, tu, wd, td, layer, seq_len, pos, hidden, inter, H, Hkv, D, eps, base, neox, scale)
        ref = z[f"call{i}_out"].astype(np.float32)
        err = float(np.max(np.abs(out.astype(np.float32) - ref)))
        assert err <= 5e-3 * max(1.0, float(np.abs(ref).max())), (i, c["args"], err)
