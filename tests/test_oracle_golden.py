"""Pin the CPU oracle (oracle/) to the reference's own outputs (CPU only).

The golden file holds outputs of the reference's ``ref_gqa_attention`` and ``ref_rope``
(tests/test_layer.py:76-105 of gfx1150-inference), produced by
tests/golden/make_golden.py.  Every oracle used by the GPU tests must agree
with it before it is trusted as a checker.
"""

from __future__ import annotations

import numpy as np
import pytest

import build_oracle
import cases
import gqa_ref

G = cases.load_golden()


def _edge_ids():
    return list(cases.EDGE_CASES)


def test_input_digests_match():
    for i, c in enumerate(cases.layer_cases()):
        assert cases.digest(c["Q"], c["K"], c["V"]) == str(G[f"layer{i}_digest"])
    c = cases.kv_manager_case()
    assert cases.digest(c["Q"], c["K"], c["V"]) == str(G["kvm_digest"])
    c = cases.config1_case()
    assert cases.digest(c["Q"], c["K"], c["V"]) == str(G["config1_digest"])
    for name in cases.EDGE_CASES:
        c = cases.edge_case(name)
        assert cases.digest(c["Q"], c["K"], c["V"]) == str(G[f"{name}_digest"]), name
    c = cases.ragged_case()
    assert cases.digest(c["q"], *c["ks"], *c["vs"]) == str(G["ragged_digest"])


def test_numpy_restatement_is_bit_exact():
    """gqa_ref.ref_gqa_attention reproduces the reference function exactly."""
    for i, c in enumerate(cases.layer_cases()):
        out = gqa_ref.ref_gqa_attention(c["Q"], c["K"], c["V"], c["start_pos"], c["scale"],
                                        c["causal"])
        np.testing.assert_array_equal(out, G[f"layer{i}_out"])
    c = cases.config1_case()
    kw = dict(start_pos=c["start_pos"], scale=c["scale"], causal=True)
    np.testing.assert_array_equal(gqa_ref.ref_gqa_attention(c["Q"], c["K"], c["V"], **kw),
                                  G["config1_out_f16"])
    np.testing.assert_array_equal(
        gqa_ref.ref_gqa_attention(c["Q"], c["K"], c["V"], out_dtype=np.float32, **kw),
        G["config1_out_f32"])
    for name in cases.EDGE_CASES:
        c = cases.edge_case(name)
        od = np.float32 if c["Q"].dtype == np.float32 else np.float16
        out = gqa_ref.ref_gqa_attention(c["Q"], c["K"], c["V"], c["start_pos"], c["scale"],
                                        c["causal"], out_dtype=od)
        np.testing.assert_array_equal(out, G[f"{name}_out"], err_msg=name)


def test_online_softmax_restatement_matches_reference():
    """The serial recurrence of the HIP kernel agrees with the reference oracle."""
    c = cases.layer_cases()[1]
    out = gqa_ref.online_softmax_attention(c["Q"], c["K"], c["V"], c["start_pos"], c["scale"])
    assert np.max(np.abs(out - G["layer1_out"].astype(np.float32))) < 1e-3
    c = cases.edge_case("noncausal_prefill")
    out = gqa_ref.online_softmax_attention(c["Q"], c["K"], c["V"], c["start_pos"], c["scale"],
                                           causal=False)
    assert np.max(np.abs(out - G["noncausal_prefill_out"].astype(np.float32))) < 1e-3


def test_c_oracle_fp32_config1_within_1e5():
    c = cases.config1_case()
    out = build_oracle.gqa_online(c["Q"], c["K"], c["V"], c["start_pos"], c["scale"], True)
    assert out.dtype == np.float32
    assert np.max(np.abs(out - G["config1_out_f32"])) <= 1e-5


@pytest.mark.parametrize("name", _edge_ids())
def test_c_oracle_edge_cases(name):
    c = cases.edge_case(name)
    out = build_oracle.gqa_online(c["Q"], c["K"], c["V"], c["start_pos"], c["scale"],
                                  c["causal"])
    ref = G[f"{name}_out"].astype(np.float32)
    tol = 1e-5 if c["Q"].dtype == np.float32 else 2e-3
    assert np.max(np.abs(out.astype(np.float32) - ref)) <= tol


def test_c_oracle_reference_layer_cases():
    for i, c in enumerate(cases.layer_cases()):
        out = build_oracle.gqa_online(c["Q"], c["K"], c["V"], c["start_pos"], c["scale"], True)
        assert np.max(np.abs(out.astype(np.float32) - G[f"layer{i}_out"].astype(np.float32))) < 2e-3


def test_c_oracle_batch_matches_ragged_golden():
    import ctypes

    c = cases.ragged_case()
    lib = build_oracle.load()
    n = len(c["ctx"])
    ks = [np.ascontiguousarray(k) for k in c["ks"]]
    vs = [np.ascontiguousarray(v) for v in c["vs"]]
    kp = (ctypes.c_void_p * n)(*[k.ctypes.data for k in ks])
    vp = (ctypes.c_void_p * n)(*[v.ctypes.data for v in vs])
    ctx = (ctypes.c_int * n)(*c["ctx"])
    out = np.empty_like(c["q"])
    assert lib.gqa_decode_batch_f16(n, c["q"].ctypes.data, kp, vp, ctx, out.ctypes.data, c["H"],
                                    c["Hkv"], c["D"], c["scale"], 2) == 0
    assert np.max(np.abs(out.astype(np.float32) - G["ragged_out"].astype(np.float32))) < 2e-3


def test_scale_zero_semantics():
    """The HIP kernel uses scale as given (attention.hip:99): scale 0 averages V.
    The numpy oracle maps 0 to 1/sqrt(D) (test_layer.py:87-88).  The B200 path
    follows the kernel; this pins the difference."""
    c = cases.edge_case("scale_custom")
    out = gqa_ref.online_softmax_attention(c["Q"], c["K"], c["V"], c["start_pos"], 0.0)
    mean_v = c["V"].astype(np.float32).mean(axis=0)  # (Hkv, D)
    group = c["Q"].shape[1] // c["K"].shape[1]
    expect = np.repeat(mean_v, group, axis=0)[None]
    assert np.max(np.abs(out - expect)) < 1e-5
    ref_default = gqa_ref.ref_gqa_attention(c["Q"], c["K"], c["V"], c["start_pos"], 0.0)
    assert np.max(np.abs(ref_default.astype(np.float32) - expect)) > 1e-3


def test_c_oracle_rejects_reference_invalid_args():
    c = cases.edge_case("scale_custom")
    with pytest.raises(ValueError):
        build_oracle.gqa_online(c["Q"][:, :7], c["K"], c["V"], c["start_pos"], c["scale"])


def test_append_rows_is_slice_assignment():
    L, S, Hkv, D = 2, 10, 2, 8
    k = np.zeros((L, S, Hkv, D), np.float16)
    v = np.zeros_like(k)
    rows = np.arange(3 * Hkv * D, dtype=np.float16).reshape(3, Hkv, D)
    gqa_ref.append_rows(k, v, 1, 4, rows, -rows)
    assert np.array_equal(k[1, 4:7], rows) and np.array_equal(v[1, 4:7], -rows)
    assert not k[0].any() and not k[1, :4].any() and not k[1, 7:].any()


def test_rope_restatement_matches_reference():
    """gqa_ref.ref_rope against the reference's ref_rope outputs (test_layer.py:44-73):
    bit for bit on every case, including positions up to 131072."""
    for i, c in enumerate(cases.rope_cases()):
        assert cases.digest(c["x"]) == str(G[f"rope{i}_digest"])
        got = gqa_ref.ref_rope(c["x"], pos_offset=c["pos_offset"], freq_base=c["freq_base"],
                               neox_style=c["neox"])
        np.testing.assert_array_equal(got, G[f"rope{i}_out"], err_msg=f"case {i}")
        # per-token positions: the same rotation when they equal pos_offset + t
        pos = np.arange(c["pos_offset"], c["pos_offset"] + c["x"].shape[0])
        again = gqa_ref.ref_rope(c["x"], freq_base=c["freq_base"], neox_style=c["neox"],
                                 positions=pos)
        np.testing.assert_array_equal(again, got)


# ---- layer pipeline oracle (oracle/layer_ref.py) vs the reference's numpy code ----
_LAYER_TYPES = {"q4_0": 2, "q8_0": 8, "q4_k": 12, "q6_k": 14}


@pytest.mark.parametrize("name", sorted(_LAYER_TYPES))
@pytest.mark.parametrize("kind", ["deq", "deqr"])
def test_dequantizers_bit_exact(name, kind):
    """gguf_parser.py dequantize_*_cpu outputs on quantizer-made and on random blocks."""
    import layer_ref
    from make_layer_golden import OUT

    g = np.load(OUT)
    raw, out = g[f"{kind}_{name}_raw"], g[f"{kind}_{name}_out"]
    mine = layer_ref.dequantize(raw, _LAYER_TYPES[name], 4, 512).reshape(-1)
    assert np.array_equal(mine.view(np.uint16), out.view(np.uint16))


def test_layer_oracle_matches_reference_composition():
    """Prefill of 4 tokens then a decode step through layer_forward equals the
    reference's CPU layer check composed from its own functions (bit-exact)."""
    import math

    import layer_ref as L
    from make_layer_golden import LAYER as C, OUT

    g = np.load(OUT)
    t = C["types"]
    lw = L.LayerWeights(g["layer_attn_norm"], *[(g[f"layer_w_{n}"], t[n]) for n in "qkvo"],
                        g["layer_ffn_norm"],
                        *[(g[f"layer_w_{n}"], t[n]) for n in ("gate", "up", "down")])
    kc = np.zeros((16, C["Hkv"], C["D"]), np.float16)
    vc = np.zeros_like(kc)
    kw = dict(num_heads=C["H"], num_kv_heads=C["Hkv"], head_dim=C["D"], inter=C["inter"],
              eps=C["eps"], rope_base=C["base"], neox=C["neox"], scale=1 / math.sqrt(C["D"]))
    x = g["layer_x"]
    out = np.concatenate([L.layer_forward(x[:4], lw, kc, vc, 0, **kw),
                          L.layer_forward(x[4:5], lw, kc, vc, 4, **kw)])
    assert np.array_equal(out, g["layer_out"])
    assert np.array_equal(kc[:5], g["layer_k_rot"]) and np.array_equal(vc[:5], g["layer_v"])


def test_weight_sizes_match_block_layouts():
    import layer_ref as L

    assert L.weight_bytes(L.Q4_0, 4096, 4096) == 4096 * 128 * 18
    assert L.weight_bytes(L.Q6_K, 1024, 4096) == 1024 * 16 * 210
    with pytest.raises(ValueError):
        L.weight_bytes(L.Q4_K, 16, 96)
