"""Generate tests/golden/gqa_golden.npz from the REFERENCE's own oracle.

Usage:  PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference <checkout>

<checkout> is a gfx1150-inference source tree.  This script imports its
``tests/test_layer.py`` and calls its ``ref_gqa_attention`` (test_layer.py:
76-105) and ``ref_rope`` (test_layer.py:44-73) on the inputs of
tests/golden/cases.py.  Importing that module pulls
in ``layer`` / ``kv_cache``, which import the native ``matmul_module``; a stub
namespace stands in for it (the same trick as the reference's own CPU suite,
tests/test_cpu_only.py:391-400), since no attention kernel is called.

For the fp32 configuration the reference function's final
``out.astype(np.float16)`` would hide the 1e-5 tolerance, so it is also run
with its module globals' ``np.float16`` replaced by ``np.float32`` — the
reference's own code, without the cast.  Both variants are stored.

The file holds reference OUTPUTS plus a SHA-256 of each case's regenerated
inputs; the tests regenerate the inputs and check the digest first.
"""

from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402


class _NpNoHalf:
    """numpy namespace whose float16 is float32 (drops the final cast only)."""

    def __getattr__(self, name):
        if name == "float16":
            return np.float32
        return getattr(np, name)


def load_reference_oracle(ref_root: str):
    sys.modules.setdefault("matmul_module", types.SimpleNamespace(
        kv_cache_init=lambda *a, **k: None, kv_cache_free=lambda *a, **k: None))
    sys.path.insert(0, os.path.join(ref_root, "src"))
    sys.path.insert(0, os.path.join(ref_root, "tests"))
    import test_layer  # the reference's module

    ref = test_layer.ref_gqa_attention
    ref_f32 = types.FunctionType(ref.__code__, dict(ref.__globals__, np=_NpNoHalf()),
                                 "ref_gqa_attention_f32", ref.__defaults__)
    return ref, ref_f32, test_layer.ref_rope


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="gfx1150-inference source checkout")
    args = ap.parse_args()
    ref, ref_f32, ref_rope = load_reference_oracle(os.path.abspath(args.reference))
    g = {}

    for i, c in enumerate(cases.layer_cases()):
        key = f"layer{i}"
        g[f"{key}_digest"] = np.array(cases.digest(c["Q"], c["K"], c["V"]))
        g[f"{key}_out"] = ref(c["Q"], c["K"], c["V"], start_pos=c["start_pos"], scale=c["scale"],
                              causal=c["causal"])

    c = cases.kv_manager_case()
    g["kvm_digest"] = np.array(cases.digest(c["Q"], c["K"], c["V"]))
    for l in range(c["num_layers"]):
        g[f"kvm_prefill_l{l}"] = ref(c["Q"][l, :4], c["K"][l, :4], c["V"][l, :4], start_pos=0,
                                     scale=c["scale"])
        for pos in (4, 5):
            g[f"kvm_decode_l{l}_p{pos}"] = ref(c["Q"][l, pos:pos + 1], c["K"][l, :pos + 1],
                                               c["V"][l, :pos + 1], start_pos=pos,
                                               scale=c["scale"])

    c = cases.config1_case()
    g["config1_digest"] = np.array(cases.digest(c["Q"], c["K"], c["V"]))
    kw = dict(start_pos=c["start_pos"], scale=c["scale"], causal=True)
    g["config1_out_f16"] = ref(c["Q"], c["K"], c["V"], **kw)
    g["config1_out_f32"] = ref_f32(c["Q"], c["K"], c["V"], **kw)
    assert g["config1_out_f32"].dtype == np.float32

    for name in cases.EDGE_CASES:
        c = cases.edge_case(name)
        g[f"{name}_digest"] = np.array(cases.digest(c["Q"], c["K"], c["V"]))
        fn = ref_f32 if c["Q"].dtype == np.float32 else ref
        g[f"{name}_out"] = fn(c["Q"], c["K"], c["V"], start_pos=c["start_pos"],
                              scale=c["scale"], causal=c["causal"])

    c = cases.ragged_case()
    g["ragged_digest"] = np.array(cases.digest(c["q"], *c["ks"], *c["vs"]))
    g["ragged_out"] = np.concatenate([
        ref(c["q"][i:i + 1], c["ks"][i], c["vs"][i], start_pos=n - 1, scale=c["scale"])
        for i, n in enumerate(c["ctx"])])

    for i, c in enumerate(cases.rope_cases()):
        g[f"rope{i}_digest"] = np.array(cases.digest(c["x"]))
        g[f"rope{i}_out"] = ref_rope(c["x"], pos_offset=c["pos_offset"], freq_base=c["freq_base"],
                                     neox_style=c["neox"])

    np.savez_compressed(cases.GOLDEN_FILE, **g)
    print(f"wrote {cases.GOLDEN_FILE}: {len(g)} arrays, "
          f"{os.path.getsize(cases.GOLDEN_FILE)} bytes")


if __name__ == "__main__":
    main()
