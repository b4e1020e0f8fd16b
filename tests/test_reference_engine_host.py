"""The batched-generation adapter under the reference's engine, on the CPU.

With a reference checkout present (this container; skipped elsewhere), the
reference's unchanged LlamaInferenceEngine opens the seeded model of
tests/golden/engine_model.py written as a GGUF file by the reference's own
writer (cpu-offload mode: nothing touches a GPU while it is built), and
``batch_generate.tensors_from_reference_engine`` reads back the configuration,
every tensor and the embedding rows exactly as the model holds them.  Without
a checkout, the committed fixture is still checked against the seeded model.
"""

from __future__ import annotations

import importlib
import json
import os
import sys
import tempfile

import numpy as np
import pytest

import engine_model as EM

REF = "/root/reference"


def test_fixture_matches_the_seeded_model():
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "engine_golden.npz"))
    meta = json.loads(str(z["meta"]))
    assert EM.digest(EM.model_tensors(meta["seed"])) == meta["digest"]
    assert len(meta["tokens"]) == len(meta["prompts"])
    assert meta["min_logit_gap"] >= 0.05
    assert len(meta["calls"]) == EM.MODEL["layers"] * sum(meta["max_new_tokens"]
                                                           for _ in meta["prompts"])


def test_adapter_reads_the_reference_engine():
    if not os.path.isdir(os.path.join(REF, "src")):
        pytest.skip("no reference checkout here")
    sys.dont_write_bytecode = True
    import make_engine_golden as MG
    import matmul_module  # this repository's, imported by the reference's modules

    src = os.path.join(REF, "src")
    if src not in sys.path:
        sys.path.insert(0, src)
    try:
        gg = importlib.import_module("gguf_parser")
        inference = importlib.import_module("inference")
        assert inference.matmul_module is matmul_module
        import batch_generate as BG

        tensors = EM.model_tensors(5)
        with tempfile.TemporaryDirectory() as tmp:
            path = os.path.join(tmp, "m.gguf")
            MG.write_model(path, tensors, gg)
            with inference.LlamaInferenceEngine(path, max_seq_len=16,
                                                offload_kv_to_cpu=True) as eng:
                cfg, got, emb = BG.tensors_from_reference_engine(eng)
        m = EM.MODEL
        assert (cfg.layers, cfg.hidden, cfg.intermediate, cfg.heads, cfg.kv_heads,
                cfg.head_dim, cfg.vocab) == (m["layers"], m["hidden"], m["intermediate"],
                                             m["heads"], m["kv_heads"], m["hidden"] // m["heads"],
                                             m["vocab"])
        assert set(got) == set(tensors)
        for name, (raw, typ, shape) in tensors.items():
            graw, gtyp, gshape = got[name]
            assert gtyp == typ and tuple(gshape) == tuple(shape), name
            np.testing.assert_array_equal(graw, raw, err_msg=name)
        np.testing.assert_array_equal(emb, tensors["token_embd.weight"][0].view(np.float16)
                                      .reshape(m["vocab"], m["hidden"]))
    finally:
        sys.dont_write_bytecode = False
