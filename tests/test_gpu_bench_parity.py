"""Parity of the exact code paths the benchmark times, against the CPU oracle.

``bench.DecodeWorkload`` is the benchmark's own set-up (seeded workload, paged
pool with a random page permutation, the plan flagged KV-stable, the fused
append + decode step); these tests run a few of its layers and compare every
output row with the reference's numpy path (``ref_gqa_attention``,
tests/test_layer.py:76-105 of the reference) on the gathered pool contents:

* config 3 (Llama-3-8B batched: 32 ragged sequences up to 8,193 positions),
  the step launched directly, then recorded into a CUDA graph and replayed
  (bit-identical to the direct launch), and the growing decode loop (plan
  rebuilt every step);
* config 4 (Llama-3-70B geometry, 8 x 32,769 positions): the full batch's
  multi-wave plan with tail quartering, and the one-wave plans of the 2- and
  8-way KV-head shards;
* config 2 (Llama-2-7B MHA, 4,096 positions);
* the reference's device-pointer cached entry
  (launch_gqa_attention_cached_fp16_device, attention.hip:376-440) against the
  host-buffer entry and the oracle.

Bound (fp16 storage, fp32 accumulate): per query row, max|got - ref| <=
2e-3 * max|ref| (conftest.assert_attention_close); appended pool rows
bit-exact.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest

from conftest import HAS_GPU, assert_attention_close

pytestmark = pytest.mark.gpu

if HAS_GPU:
    import torch

    import bench
    import gqa_ref  # oracle: checker only
    import kvcache_ffi as ffi
    import matmul_module
    import paged


def _oracle_layer(pool, bt, layer, ctx, q, scale, k_new=None, v_new=None):
    """Reference outputs of one layer's queries (one per sequence), from the pool's
    gathered rows; with k_new / v_new, also the appended rows checked bit-exact."""
    ref = np.empty(q.shape, dtype=np.float16)
    qn = q.cpu().numpy()
    for i, c in enumerate(ctx):
        k, v = pool.gather(layer, bt, i, 0, int(c))
        k, v = k.cpu().numpy(), v.cpu().numpy()
        if k_new is not None:
            assert np.array_equal(k[-1], k_new[i].cpu().numpy()), (layer, i)
            assert np.array_equal(v[-1], v_new[i].cpu().numpy()), (layer, i)
        ref[i] = gqa_ref.ref_gqa_attention(qn[i:i + 1], k, v, int(c) - 1, scale)[0]
    return ref


def _check_workload(wl, got, what):
    for l in range(wl.L):
        ref = _oracle_layer(wl.pool, wl.bt, l, wl.current_ctx(), wl.q[l], wl.scale,
                            wl.kn[l], wl.vn[l])
        assert_attention_close(got[l].cpu().numpy(), ref, f"{what} layer {l}")


def _graph_equals_direct(wl, direct):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        wl.step(s=torch.cuda.current_stream())
    for _ in range(2):
        wl.out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert ffi.device_error(0) == (0, 0)
        for l in range(wl.L):
            assert torch.equal(wl.out[l], direct[l]), f"graph replay differs at layer {l}"
    g.reset()


def test_config3_benchmark_step_direct_and_graph(cuda_device):
    wl = bench.DecodeWorkload("3", layers=2)
    try:
        assert wl.plan.info().n_items > 200  # the benchmark's ragged split plan
        got = {}
        wl.step(results=got)
        torch.cuda.synchronize()
        assert ffi.device_error(0) == (0, 0)
        _check_workload(wl, got, "config 3 direct")
        _graph_equals_direct(wl, got)
    finally:
        wl.close()


def test_config3_growing_decode_loop(cuda_device):
    wl = bench.DecodeWorkload("3", layers=2, grow_extra=4)
    try:
        got = {}
        for _ in range(3):
            got = {}
            wl.step(grow=True, results=got)
        torch.cuda.synchronize()
        assert ffi.device_error(0) == (0, 0)
        assert int(wl.current_ctx().max()) == int(wl.ctx.max()) + 3
        _check_workload(wl, got, "config 3 growing loop")
    finally:
        wl.close()


def test_config3_graphed_growing_loop_with_restarts(cuda_device):
    # The headline measurement: the plan rebuilt every step, the step's launches
    # replayed from one graph, contexts back to the configured lengths at every
    # timed pass.  The replayed outputs must equal the oracle after growth and
    # after a restart, with no capture after the first.
    wl = bench.DecodeWorkload("3", layers=2, grow_extra=6)
    try:
        for _ in range(4):
            wl.step_graphed()
        torch.cuda.synchronize()
        assert ffi.device_error(0) == (0, 0)
        assert int(wl.current_ctx().max()) == int(wl.ctx.max()) + 4
        _check_workload(wl, {l: wl.out[l].clone() for l in range(wl.L)}, "graphed growing loop")
        wl.restart_growth()
        for _ in range(2):
            wl.step_graphed()
        torch.cuda.synchronize()
        assert ffi.device_error(0) == (0, 0)
        assert int(wl.current_ctx().max()) == int(wl.ctx.max()) + 2
        _check_workload(wl, {l: wl.out[l].clone() for l in range(wl.L)},
                        "graphed growing loop after a restart")
        assert wl.captures == 1
    finally:
        wl.close()


def _expected_quartered(ctx, C, ups, warps):
    full = sum(c // C for c in ctx) * ups
    part = sum(c % C for c in ctx) * ups
    r = full % warps
    if full > warps and 0 < r < warps * 6 // 10 and part * 20 < C * warps:
        return (r + ups - 1) // ups
    return 0


def _split_tokens(ctx, H, Hkv, sms):
    arr = np.ascontiguousarray(np.asarray(ctx, dtype=np.int32))
    out = ctypes.c_int()
    ffi.check(ffi.lib.kvc_plan_split_tokens(ffi.np_ptr(arr), len(arr), H, Hkv, 16, sms,
                                            ctypes.byref(out)))
    return out.value


def test_config4_full_batch_multiwave_plan_with_tail_quartering(cuda_device):
    wl = bench.DecodeWorkload("4", layers=1)
    try:
        sms = torch.cuda.get_device_properties(0).multi_processor_count
        ctx = [int(c) for c in wl.ctx]
        C = _split_tokens(ctx, wl.H, wl.Hkv, sms)
        ups = wl.Hkv * ((wl.H // wl.Hkv + 7) // 8)
        n_q = _expected_quartered(ctx, C, ups, sms * 8)
        base = sum(math.ceil(c / C) for c in ctx)
        info = wl.plan.info()
        assert info.n_items == base + 3 * n_q
        assert base * ups > sms * 8  # several waves
        got = {}
        wl.step(results=got)
        torch.cuda.synchronize()
        assert ffi.device_error(0) == (0, 0)
        _check_workload(wl, got, f"config 4 full batch ({info.n_items} splits, "
                                 f"{n_q} quartered)")
        _graph_equals_direct(wl, got)
    finally:
        wl.close()


@pytest.mark.parametrize("ways", [2, 8])
def test_config4_head_shard_one_wave_plan(cuda_device, ways):
    """One rank's shard of config 4 split by KV head: 8 x 32,769 positions on
    8 / ways KV heads and their q-heads, a one-wave plan."""
    cfg = bench.CONFIGS["4"]
    Hkv = cfg["Hkv"] // ways
    H = cfg["H"] // ways
    D, B, S = cfg["D"], cfg["batch"], cfg["lens"][1] + 1
    ctx = [S] * B
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    table, total = paged.random_block_tables(ctx, 16, 44 + ways)
    pool = paged.PagedKVCache(1, total, 16, Hkv, D)
    pool.fill_normal(seed=ways, stddev=1.0)
    bt = torch.from_numpy(table).cuda()
    g = torch.Generator(device="cuda")
    g.manual_seed(ways)
    q = torch.randn((B, H, D), generator=g, device="cuda").half()
    kn = torch.randn((B, Hkv, D), generator=g, device="cuda").half()
    vn = torch.randn((B, Hkv, D), generator=g, device="cuda").half()
    out = torch.zeros_like(q)
    plan = pool.plan(ctx, H)
    plan.set_kv_stable(True)
    try:
        info = plan.info()
        C = _split_tokens(ctx, H, Hkv, sms)
        units = info.n_items * Hkv * ((H // Hkv + 7) // 8)
        assert units <= sms * 8, (C, info)  # one wave of equal units
        scale = 1.0 / math.sqrt(D)
        pool.append_decode(plan, 0, q, kn, vn, out, bt, scale)
        torch.cuda.synchronize()
        assert ffi.device_error(0) == (0, 0)
        ref = _oracle_layer(pool, bt, 0, ctx, q, scale, kn, vn)
        assert_attention_close(out.cpu().numpy(), ref,
                               f"config 4, one rank of {ways}-way head split ({C}-position splits)")
    finally:
        plan.close()
        pool.close()


def test_config2_mha_4096(cuda_device):
    wl = bench.DecodeWorkload("2", layers=2)
    try:
        got = {}
        wl.step(results=got)
        torch.cuda.synchronize()
        assert ffi.device_error(0) == (0, 0)
        _check_workload(wl, got, "config 2 direct")
        _graph_equals_direct(wl, got)
    finally:
        wl.close()


# ---------------------------------------------------------------------------
# launch_gqa_attention_cached_fp16_device (attention.hip:376-440)
# ---------------------------------------------------------------------------
def _cached_device(q, k, v, out, layer, q_len, start, H, Hkv, D, scale, stream):
    return ffi.lib.kvc_gqa_attention_cached_device(
        int(q.data_ptr()), int(k.data_ptr()), int(v.data_ptr()), int(out.data_ptr()), layer,
        q_len, start, H, Hkv, D, float(scale), 1, int(stream.cuda_stream) or None)


def test_cached_device_entry_matches_host_entry_and_oracle(cuda_device):
    """A prefill of 5 positions then decode steps at 5 and 6, in two layers, through
    the device-pointer entry on a side stream; the same calls through the
    host-buffer entry on a fresh pool give bit-identical outputs, and both are
    within the bound of the oracle on the accumulated K/V."""
    L, S, H, Hkv, D = 2, 64, 8, 2, 64
    scale = 1.0 / math.sqrt(D)
    rng = np.random.default_rng(23)
    calls = [(0, 5), (5, 1), (6, 1)]  # (start_pos, q_len)
    data = []
    for start, n in calls:
        for l in range(L):
            data.append((l, start, n,
                         (rng.standard_normal((n, H, D), dtype=np.float32) * 0.5).astype(np.float16),
                         (rng.standard_normal((n, Hkv, D), dtype=np.float32) * 0.5).astype(np.float16),
                         (rng.standard_normal((n, Hkv, D), dtype=np.float32) * 0.5).astype(np.float16)))
    # device entry, side stream
    matmul_module.kv_cache_init(L, S, Hkv, D)
    s = torch.cuda.Stream()
    dev_out = []
    try:
        for l, start, n, q, k, v in data:
            qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k, v))
            od = torch.full((n, H, D), float("nan"), dtype=torch.float16, device="cuda")
            torch.cuda.current_stream().synchronize()
            rc = _cached_device(qd, kd, vd, od, l, n, start, H, Hkv, D, scale, s)
            assert rc == 0, ffi.last_error()
            s.synchronize()
            dev_out.append(od.cpu().numpy())
        assert ffi.device_error(0) == (0, 0)
        # the validation of attention.hip:316-329 on the device entry
        qd = torch.zeros((1, H, D), dtype=torch.float16, device="cuda")
        kd = torch.zeros((1, Hkv, D), dtype=torch.float16, device="cuda")
        assert _cached_device(qd, kd, kd, qd, L, 1, 0, H, Hkv, D, scale, s) == ffi.KVC_ERR_OUT_OF_RANGE
        assert _cached_device(qd, kd, kd, qd, 0, 1, S, H, Hkv, D, scale, s) == ffi.KVC_ERR_OUT_OF_RANGE
        assert _cached_device(qd, kd, kd, qd, 0, 1, 0, H, Hkv + 1, D, scale, s) == ffi.KVC_ERR_INVALID_ARG
    finally:
        matmul_module.kv_cache_free()
    # host entry on a fresh pool
    matmul_module.kv_cache_init(L, S, Hkv, D)
    try:
        kh = np.zeros((L, S, Hkv, D), np.float16)
        vh = np.zeros((L, S, Hkv, D), np.float16)
        for i, (l, start, n, q, k, v) in enumerate(data):
            out = np.empty((n, H, D), np.float16)
            matmul_module.gqa_attention_cached(q, k, v, out, l, n, start, H, Hkv, D, scale, True)
            assert np.array_equal(out, dev_out[i]), f"call {i}: device and host entries differ"
            gqa_ref.append_rows(kh, vh, l, start, k, v)
            ref = gqa_ref.ref_gqa_attention(q, kh[l, :start + n], vh[l, :start + n], start, scale)
            assert_attention_close(out, ref, f"cached entries call {i} (layer {l}, start {start})")
    finally:
        matmul_module.kv_cache_free()
