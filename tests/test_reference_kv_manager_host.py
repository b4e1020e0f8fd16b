"""The drop-in boundary under the reference's KVCacheManager, on the CPU.

* The recorded trace (tests/golden/kv_trace.npz, what the reference's unchanged
  src/kv_cache.py passed to ``matmul_module``) replays against a CPU stand-in
  built on this repository's oracle: every output equals the reference oracle's
  recorded output bit for bit (so the trace and ``gqa_ref`` agree, and the replay
  rebuilds the exact arguments: host arrays, appended rows, layer views), and
  ``matmul_module.host_layer_view`` recognises every K / V view the manager
  passed in its cpu and mmap modes, with the right layer.
* With a reference checkout present (this container; skipped elsewhere), the
  reference's kv_cache.py is imported with this repository's ``matmul_module``
  as the module it imports: its host arrays' layer views are recognised in the
  cpu and mmap modes, and without a GPU its gpu-mode constructor fails in
  kv_cache_init and rolls its singleton guard back (kv_cache.py:146-161).
"""

from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import pytest

import gqa_ref  # oracle: checker only
import kv_trace
import matmul_module

REF_SRC = "/root/reference/src/kv_cache.py"


class _OracleModule:
    """CPU stand-in for matmul_module that computes with the oracle and checks
    that every host-array view is recognised as the manager's layer view."""

    def __init__(self):
        self.pool = None
        self.views = []

    def kv_cache_init(self, L, S, Hkv, D):
        self.pool = (np.zeros((L, S, Hkv, D), np.float16), np.zeros((L, S, Hkv, D), np.float16))

    def kv_cache_free(self):
        self.pool = None

    def gqa_attention_cached(self, Q, K_new, V_new, Out, layer, q_len, start, H, Hkv, D,
                             scale=0.0, causal=True):
        kp, vp = self.pool
        kp[layer, start:start + q_len] = K_new
        vp[layer, start:start + q_len] = V_new
        Out[...] = gqa_ref.ref_gqa_attention(Q, kp[layer, :start + q_len],
                                             vp[layer, :start + q_len], start, scale, causal)

    def gqa_attention(self, Q, K, V, Out, q_len, kv_len, H, Hkv, D, start_pos=0, scale=0.0,
                      causal=True):
        kv = matmul_module.host_layer_view(K, Hkv, D)
        vv = matmul_module.host_layer_view(V, Hkv, D)
        # (layer, layers, max_seq_len) only: a reference to the host array would keep
        # the manager's memory-mapped file from closing
        self.views.append((kv and kv[1:], vv and vv[1:], K.shape))
        Out[...] = gqa_ref.ref_gqa_attention(Q, K[:kv_len], V[:kv_len], start_pos, scale, causal)


@pytest.mark.parametrize("scenario", ["full_model_gpu", "modes_gpu", "modes_cpu", "modes_mmap",
                                      "prefill_whole_gpu"])
def test_trace_replays_to_the_reference_oracle_bit_for_bit(scenario, tmp_path):
    trace = kv_trace.load()
    mod = _OracleModule()
    res = kv_trace.replay(trace, scenario, mod, tmpdir=str(tmp_path))
    n = 0
    for ev, out, expect, exc in res.calls:
        assert exc is None, exc
        if expect is not None:
            np.testing.assert_array_equal(out, expect.reshape(out.shape))
            n += 1
    assert n == {"full_model_gpu": 6, "prefill_whole_gpu": 12}.get(scenario, 27)
    if scenario in ("modes_cpu", "modes_mmap"):
        assert len(mod.views) == 27
        attn = [ev for ev, *_ in res.calls if ev["fn"] == "gqa_attention"]
        for (kv, vv, shape), ev in zip(mod.views, attn):
            assert kv is not None and vv is not None, "a host layer view was not recognised"
            layer = ev["args"][1]["at"] // int(np.prod(shape))
            assert kv == vv == (layer, 3, 64)


def test_rollback_scenario_is_recorded():
    trace = kv_trace.load()
    evs = [e for e in trace.scenarios["rollback_gpu"] if e["op"] == "call"]
    assert [e["fn"] for e in evs] == ["kv_cache_init", "kv_cache_free"]
    assert evs[0]["raises"] == "RuntimeError"


def test_host_layer_view_rejects_other_layouts():
    a = np.zeros((3, 10, 2, 8), np.float16)
    assert matmul_module.host_layer_view(a[1], 2, 8)[1:] == (1, 3, 10)
    assert matmul_module.host_layer_view(a[1], 4, 4) is None          # other head geometry
    assert matmul_module.host_layer_view(a[1, :5], 2, 8) is None      # not a whole layer
    assert matmul_module.host_layer_view(np.zeros((10, 2, 8), np.float16), 2, 8) is None
    one = np.zeros((1, 10, 2, 8), np.float16)
    assert matmul_module.host_layer_view(one[0], 2, 8) is None        # a single layer
    assert matmul_module.host_layer_view(a[:, 0], 2, 8) is None       # strided


def _load_reference_kv_cache():
    if not os.path.exists(REF_SRC):
        pytest.skip("no reference checkout here")
    spec = importlib.util.spec_from_file_location("reference_kv_cache", REF_SRC)
    mod = importlib.util.module_from_spec(spec)
    old = sys.dont_write_bytecode
    sys.dont_write_bytecode = True  # nothing is written next to the reference's sources
    try:
        assert sys.modules.get("matmul_module") is matmul_module
        spec.loader.exec_module(mod)
    finally:
        sys.dont_write_bytecode = old
    assert mod.matmul_module is matmul_module
    return mod


@pytest.mark.parametrize("mode", ["cpu", "mmap"])
def test_reference_manager_host_arrays_are_recognised(mode, tmp_path):
    ref = _load_reference_kv_cache()
    kw = {"offload_to_cpu": True} if mode == "cpu" else {"mmap_dir": str(tmp_path)}
    with ref.KVCacheManager(3, 20, 2, 16, **kw) as kv:
        assert kv.mode == mode
        # only (layer, layers, max_seq_len) is kept: a reference to a host array
        # would keep the manager from closing its memory-mapped files
        found = [(matmul_module.host_layer_view(kv._k_host[l], 2, 16) or (None,))[1:]
                 + (matmul_module.host_layer_view(kv._v_host[l], 2, 16) or (None,))[1:]
                 for l in range(3)]
    assert found == [(l, 3, 20, l, 3, 20) for l in range(3)]


def test_reference_gpu_manager_rolls_back_when_init_fails_without_a_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present: kv_cache_init would succeed")
    ref = _load_reference_kv_cache()
    ref.KVCacheManager._active_gpu_instance = False
    with pytest.raises(RuntimeError):
        ref.KVCacheManager(2, 16, 2, 32)
    assert not ref.KVCacheManager._active_gpu_instance
