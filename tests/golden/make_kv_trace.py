"""Generate tests/golden/kv_trace.npz by running the REFERENCE's KVCacheManager.

Usage:  PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_kv_trace.py --reference <checkout>

<checkout> is a gfx1150-inference source tree.  Its ``src/kv_cache.py`` runs
unchanged with a ``kv_trace.Recorder`` installed as ``matmul_module`` (the
module it imports, kv_cache.py:26-40); expected outputs come from the
reference's own numpy oracle ``ref_gqa_attention`` (tests/test_layer.py:76-105).
Scenarios (small shapes, seeded inputs drawn like the reference's GPU tests):

* ``full_model_gpu`` — tests/test_full_model.py:78-129: gpu mode, L=2, S=32,
  H=8, Hkv=2, D=32, seed 19; a 4-token prefill per layer, then decode steps at
  positions 4 and 5; current_seq_len == 6 afterwards.
* ``modes_gpu`` / ``modes_cpu`` / ``modes_mmap`` — the KV-path part of
  tests/test_phase5_scale.py:188-271 (the same greedy tokens in gpu, cpu-offload
  and mmap modes, with full and chunked prefill): L=3, S=64, H=8, Hkv=2, D=64;
  prompt A prefilled in chunks of 3 (8 positions) and decoded 3 steps; reset();
  prompt B prefilled whole (5 positions) and decoded 2 steps, all through
  KVCacheManager.attend in the named mode.  The three traces carry the same
  inputs; a drop-in must give bit-identical outputs in all three.
* ``prefill_whole_gpu`` — prompt A of the modes scenarios prefilled in one call
  (8 positions) instead of chunks of 3, then the same decode steps
  (tests/test_phase5_scale.py:199-206 compares full and chunked prefill).
* ``rollback_gpu`` — kv_cache.py:146-161: kv_cache_init fails (injected), the
  manager rolls its singleton guard back and calls kv_cache_free.
"""

from __future__ import annotations

import argparse
import math
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import kv_trace  # noqa: E402


class _Dispatch:
    """The ``matmul_module`` the reference imports: forwards to the current recorder."""

    rec = None

    def __getattr__(self, name):
        return getattr(type(self).rec, name)


def _draw(rng, shape):
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.5)).astype(np.float16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="gfx1150-inference source checkout")
    args = ap.parse_args()
    root = os.path.abspath(args.reference)
    disp = _Dispatch()
    sys.modules["matmul_module"] = disp
    sys.path.insert(0, os.path.join(root, "src"))
    sys.path.insert(0, os.path.join(root, "tests"))
    import kv_cache  # the reference's, unchanged
    import test_layer  # the reference's numpy oracle

    def ref(q, k, v, start_pos, scale, causal):
        return test_layer.ref_gqa_attention(q, k, v, start_pos=start_pos, scale=scale,
                                            causal=causal)

    KVCacheManager = kv_cache.KVCacheManager
    scenarios = {}

    # -- tests/test_full_model.py:78-129 ------------------------------------------
    rec = _Dispatch.rec = kv_trace.Recorder(ref)
    rng = np.random.default_rng(19)
    L, S, H, Hkv, D, T = 2, 32, 8, 2, 32, 6
    scale = 1.0 / math.sqrt(D)
    Q, K, V = _draw(rng, (L, T, H, D)), _draw(rng, (L, T, Hkv, D)), _draw(rng, (L, T, Hkv, D))
    with KVCacheManager(L, S, Hkv, D) as kv:
        for l in range(L):
            out = np.zeros((4, H, D), np.float16)
            kv.attend(Q[l, :4], K[l, :4], V[l, :4], out, layer_idx=l, q_len=4, start_pos=0,
                      num_heads=H, scale=scale, causal=True)
        for pos in (4, 5):
            for l in range(L):
                out = np.zeros((1, H, D), np.float16)
                kv.attend(Q[l, pos:pos + 1], K[l, pos:pos + 1], V[l, pos:pos + 1], out,
                          layer_idx=l, q_len=1, start_pos=pos, num_heads=H, scale=scale,
                          causal=True)
        assert kv.current_seq_len == 6
    scenarios["full_model_gpu"] = rec

    # -- modes: gpu / cpu / mmap, chunked prefill, reset, second prompt -------------
    rng = np.random.default_rng(77)
    L, S, H, Hkv, D = 3, 64, 8, 2, 64
    scale = 0.125
    prompts = []
    for T in (11, 7):
        prompts.append((_draw(rng, (L, T, H, D)), _draw(rng, (L, T, Hkv, D)),
                        _draw(rng, (L, T, Hkv, D))))
    # (prompt, spans): A = chunks of 3 over 8 positions + 3 decode steps; B = 5 + 2
    plan = [(0, [(0, 3), (3, 6), (6, 8), (8, 9), (9, 10), (10, 11)]),
            (1, [(0, 5), (5, 6), (6, 7)])]
    with tempfile.TemporaryDirectory() as tmp:
        for mode in ("gpu", "cpu", "mmap"):
            rec = _Dispatch.rec = kv_trace.Recorder(ref)
            kw = {"gpu": {}, "cpu": {"offload_to_cpu": True},
                  "mmap": {"mmap_dir": os.path.join(tmp, "kv")}}[mode]
            with KVCacheManager(L, S, Hkv, D, **kw) as kv:
                assert kv.mode == mode
                for p, spans in plan:
                    q, k, v = prompts[p]
                    kv.reset()
                    rec.mark(f"prompt {p}")
                    for s, e in spans:
                        for l in range(L):
                            out = np.zeros((e - s, H, D), np.float16)
                            kv.attend(q[l, s:e], k[l, s:e], v[l, s:e], out, layer_idx=l,
                                      q_len=e - s, start_pos=s, num_heads=H, scale=scale,
                                      causal=True)
                    assert kv.current_seq_len == spans[-1][1]
            scenarios[f"modes_{mode}"] = rec

    # -- prompt A again, prefilled whole (tests/test_phase5_scale.py:199-206 compares
    #    full and chunked prefill) ----------------------------------------------------
    rec = _Dispatch.rec = kv_trace.Recorder(ref)
    with KVCacheManager(L, S, Hkv, D) as kv:
        q, k, v = prompts[0]
        for s_, e in [(0, 8), (8, 9), (9, 10), (10, 11)]:
            for l in range(L):
                out = np.zeros((e - s_, H, D), np.float16)
                kv.attend(q[l, s_:e], k[l, s_:e], v[l, s_:e], out, layer_idx=l, q_len=e - s_,
                          start_pos=s_, num_heads=H, scale=scale, causal=True)
    scenarios["prefill_whole_gpu"] = rec

    # -- kv_cache.py:146-161: a failed kv_cache_init is rolled back ------------------
    rec = _Dispatch.rec = kv_trace.Recorder(ref)
    rec.fail_init = True
    try:
        KVCacheManager(2, 16, 2, 32)
        raise AssertionError("the injected failure did not propagate")
    except RuntimeError:
        pass
    assert not KVCacheManager._active_gpu_instance
    scenarios["rollback_gpu"] = rec

    kv_trace.save(scenarios, meta={
        "source": "reference src/kv_cache.py (unchanged) + tests/test_layer.py ref_gqa_attention",
        "generator": "tests/golden/make_kv_trace.py"})
    n = sum(len(r.events) for r in scenarios.values())
    print(f"wrote {kv_trace.TRACE_FILE}: {len(scenarios)} scenarios, {n} events, "
          f"{os.path.getsize(kv_trace.TRACE_FILE)} bytes")


if __name__ == "__main__":
    main()
