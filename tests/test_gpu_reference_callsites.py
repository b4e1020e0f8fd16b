"""The drop-in under the reference's own KVCacheManager (src/kv_cache.py).

tests/golden/kv_trace.npz holds what the reference's unchanged KVCacheManager
passed to ``matmul_module`` in each scenario (tests/golden/make_kv_trace.py
recorded it by running the reference's file): the calls, their arguments, the
views of its host arrays with the host appends it made, and the reference
oracle's expected outputs.  These tests replay that sequence against this
repository's ``matmul_module`` on a B200:

* the GPU-resident manager test of the reference (tests/test_full_model.py:
  78-129) within its 1e-3 and within the fp16 bound, pool rows bit-exact;
* the gpu / cpu-offload / mmap modes (tests/test_phase5_scale.py:188-271 at the
  attention level: chunked prefill, decode, reset, a second prompt) bit-identical
  to one another, the host modes served by the streaming engine behind
  ``gqa_attention``; whole vs chunked prefill bit-identical;
* the HBM mirror, an invalidation mid-sequence, the engine turned off, and a
  refused page-locking (copies from pageable memory): all bit-identical;
* failure handling: a device allocation that fails inside kv_cache_init under
  the manager's rollback (kv_cache.py:146-161); host waits that run out
  (KVC_ERR_TIMEOUT -> TimeoutError) and leave the library usable.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import HAS_GPU, assert_attention_close

pytestmark = pytest.mark.gpu

if HAS_GPU:
    import torch

    import kv_trace
    import kvcache_ffi as ffi
    import matmul_module
    import paged

TRACE = kv_trace.load() if HAS_GPU else None


@pytest.fixture(autouse=True)
def _clean(cuda_device):
    yield
    for site in (ffi.FAULT_DEVICE_ALLOC, ffi.FAULT_HOST_ALLOC, ffi.FAULT_HOST_REGISTER,
                 ffi.FAULT_WAIT):
        ffi.inject_failure(site, 0)
    ffi.set_host_wait_limit(60.0)
    matmul_module.set_offload_mirror_bytes(0)
    matmul_module.kv_cache_free()
    torch.cuda.synchronize()
    code, info = ffi.device_error(0, clear=True)
    assert code == 0, f"device error word left set: {code} {info}"


def _attention_outputs(res):
    out = []
    for ev, got, expect, exc in res.calls:
        if ev["fn"] in ("gqa_attention", "gqa_attention_cached"):
            assert exc is None, f"{ev['fn']} raised {exc!r}"
            out.append((ev, got, expect))
    return out


def _check_against_oracle(calls, what, ref_abs=None):
    for i, (ev, got, expect) in enumerate(calls):
        assert_attention_close(got, expect, f"{what} call {i}")
        if ref_abs is not None:  # the reference test's own max-abs tolerance
            err = float(np.max(np.abs(got.astype(np.float32) - expect.astype(np.float32))))
            assert err < ref_abs, (i, err)


def test_reference_full_model_kv_manager_sequence():
    """tests/test_full_model.py:78-129 as the reference's KVCacheManager ran it."""
    rows = {}

    def after(ev, out, exc):
        if ev["fn"] == "gqa_attention_cached":
            layer, q_len, start = ev["args"][4], ev["args"][5], ev["args"][6]
            rows[layer] = max(rows.get(layer, 0), start + q_len)
            if layer == 1 and start == 5:  # last call: pool rows before kv_cache_free
                for l in rows:
                    k, v = matmul_module.kv_cache_gather(l, 0, rows[l])
                    after.pool[l] = (k, v)

    after.pool = {}
    res = kv_trace.replay(TRACE, "full_model_gpu", matmul_module, after_call=after)
    calls = _attention_outputs(res)
    assert len(calls) == 6
    _check_against_oracle(calls, "full_model_gpu", ref_abs=1e-3)
    # the pool holds exactly the rows the manager appended (K_new / V_new arguments)
    k_in = {l: [] for l in after.pool}
    v_in = {l: [] for l in after.pool}
    for ev, _, _ in calls:
        l = ev["args"][4]
        k_in[l].append(TRACE.array("full_model_gpu", ev["args"][1]["array"]))
        v_in[l].append(TRACE.array("full_model_gpu", ev["args"][2]["array"]))
    for l, (k, v) in after.pool.items():
        np.testing.assert_array_equal(k, np.concatenate(k_in[l]).reshape(k.shape))
        np.testing.assert_array_equal(v, np.concatenate(v_in[l]).reshape(v.shape))


def _replay_outputs(name, **kw):
    res = kv_trace.replay(TRACE, name, matmul_module, **kw)
    return _attention_outputs(res)


def _assert_same(a, b, what):
    assert len(a) == len(b)
    for i, ((_, x, _), (_, y, _)) in enumerate(zip(a, b)):
        np.testing.assert_array_equal(x, y, err_msg=f"{what}: call {i}")


def test_storage_modes_bit_identical_through_the_reference_manager():
    stats = {}

    def grab(ev, out, exc):
        stats.update(matmul_module.offload_stats())

    gpu = _replay_outputs("modes_gpu")
    cpu = _replay_outputs("modes_cpu", after_call=grab)
    assert stats["engines"] == 1 and stats["attend_calls"] == 27
    assert stats["prefetch_hits"] >= 20 and stats["h2d_bytes"] > 0
    mm = _replay_outputs("modes_mmap")
    assert matmul_module.offload_stats()["engines"] == 0  # released with the host arrays
    _check_against_oracle(gpu, "modes_gpu")
    _assert_same(cpu, gpu, "cpu offload vs gpu")
    _assert_same(mm, gpu, "mmap vs gpu")


def test_whole_and_chunked_prefill_bit_identical():
    def by_position(calls):
        rows = {}
        for ev, out, _ in calls:
            layer, q_len, start = ev["args"][4], ev["args"][5], ev["args"][6]
            for m in range(q_len):
                rows.setdefault((layer, start + m), out[m])
        return rows

    whole = by_position(_replay_outputs("prefill_whole_gpu"))
    chunked = by_position(_replay_outputs("modes_gpu")[:18])  # prompt A: 6 spans x 3 layers
    assert set(whole) == set(chunked)
    for key in whole:
        np.testing.assert_array_equal(whole[key], chunked[key], err_msg=str(key))


def test_hbm_mirror_uploads_only_new_rows_and_stays_bit_identical():
    gpu = _replay_outputs("modes_gpu")
    row = 2 * 64 * 2                          # Hkv x D fp16 bytes
    layer_bytes = 2 * 4 * 2 * 16 * 64 * 2     # K and V pages of one layer (64 positions)
    for budget, layers in ((2 * layer_bytes, 2), (10 * layer_bytes, 3)):
        matmul_module.set_offload_mirror_bytes(budget)
        stats = {}
        got = _replay_outputs("modes_cpu",
                              after_call=lambda *a: stats.update(matmul_module.offload_stats()))
        _assert_same(got, gpu, f"mirror of {layers} layers")
        assert stats["mirror_layers"] == layers
        # prompt A: 11 rows per mirrored layer; reset; prompt B re-uploads from 0: 7
        assert stats["mirror_bytes"] == 2 * row * layers * (11 + 7)
        if layers == 3:
            assert stats["h2d_bytes"] == 0    # nothing streamed
    matmul_module.set_offload_mirror_bytes(0)


def test_invalidate_engine_off_and_refused_page_locking_stay_bit_identical(monkeypatch):
    gpu = _replay_outputs("modes_gpu")
    n = [0]

    def invalidate_midway(ev, out, exc):
        n[0] += 1
        if n[0] in (7, 20):
            matmul_module.offload_invalidate()

    _assert_same(_replay_outputs("modes_cpu", after_call=invalidate_midway), gpu, "invalidate")
    # page-locking refused: the engine copies from pageable memory (the driver stages it)
    ffi.inject_failure(ffi.FAULT_HOST_REGISTER, count=1)
    _assert_same(_replay_outputs("modes_cpu"), gpu, "bounce buffers")
    monkeypatch.setenv("KVC_OFFLOAD_STREAM", "0")  # stateless: whole layer copied per call
    _assert_same(_replay_outputs("modes_cpu"), gpu, "engine off")


def test_rollback_after_injected_allocation_failure():
    """kv_cache.py:146-161 with a cudaMalloc that fails inside kv_cache_init: the
    call raises RuntimeError (as the reference's HIP_CHECK would), the manager's
    kv_cache_free succeeds, and a later pool works."""
    ffi.inject_failure(ffi.FAULT_DEVICE_ALLOC, count=1)
    res = kv_trace.replay(TRACE, "rollback_gpu", matmul_module)
    (init_ev, _, _, init_exc), (free_ev, _, _, free_exc) = res.calls
    assert init_ev["fn"] == "kv_cache_init" and init_ev["raises"] == "RuntimeError"
    assert isinstance(init_exc, RuntimeError) and "cudaMalloc" in str(init_exc)
    assert free_ev["fn"] == "kv_cache_free" and free_exc is None
    assert matmul_module.kv_cache_dtype() is None
    out = _replay_outputs("full_model_gpu")
    _check_against_oracle(out, "after rollback")


def test_host_wait_limit_runs_out_and_library_stays_usable():
    H, Hkv, D, ps = 8, 2, 64, 16
    ctx = [300, 41]
    table, total = paged.random_block_tables(ctx, ps, 3)
    pool = paged.PagedKVCache(1, total, ps, Hkv, D)
    pool.fill_normal(seed=5)
    bt = torch.from_numpy(table).cuda()
    plan = pool.plan(ctx, H)
    rng = np.random.default_rng(2)
    hq = torch.from_numpy(rng.standard_normal((2, H, D), dtype=np.float32)).half().pin_memory()
    hk = torch.from_numpy(rng.standard_normal((2, Hkv, D), dtype=np.float32)).half().pin_memory()
    hv = torch.from_numpy(rng.standard_normal((2, Hkv, D), dtype=np.float32)).half().pin_memory()
    ho = torch.zeros_like(hq).pin_memory()
    stream = torch.cuda.current_stream()
    pool.decode_host(plan, 0, hq, hk, hv, ho, bt, 0.125, stream=stream)
    expect = ho.clone()
    # (a) a real run-out: the stream is busy with a bounded spin kernel for ~0.3 s
    ffi.set_host_wait_limit(0.02)
    torch.cuda._sleep(600_000_000)
    with pytest.raises(TimeoutError):
        pool.decode_host(plan, 0, hq, hk, hv, ho, bt, 0.125, stream=stream)
    torch.cuda.synchronize()
    ffi.set_host_wait_limit(60.0)
    assert torch.equal(ho, expect)  # the queued work finished after the timeout
    # (b) an injected run-out in the offload engine's wait for its copies, then recovery
    res = {"calls": 0}

    def on_call(ev, out, exc):
        res["calls"] += 1
        if res["calls"] == 3:  # this call's copies are still being timed
            ffi.inject_failure(ffi.FAULT_WAIT, count=1)
            try:
                matmul_module.offload_stats()
            except TimeoutError:
                res["timed_out"] = True
            ffi.inject_failure(ffi.FAULT_WAIT, 0)
            res["stats"] = matmul_module.offload_stats()

    got = _replay_outputs("modes_cpu", after_call=on_call)
    _assert_same(got, _replay_outputs("modes_gpu"), "after an injected offload timeout")
    assert res.get("timed_out") and res["stats"]["attend_calls"] == 3
    pool.decode_host(plan, 0, hq, hk, hv, ho, bt, 0.125, stream=stream)
    assert torch.equal(ho, expect)
    plan.close()
    pool.close()
