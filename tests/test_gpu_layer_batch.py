"""Batched layer decode on the paged pool (kvc_forward_layer_paged, paged.BatchDecoder)
against the pinned layer oracle (oracle/layer_ref.py).

The reference decodes a batch one sequence at a time (generate_batch_ids,
src/inference.py:435-447), each token through forward_layer_cached
(attention.hip:603-695).  Here every sequence of a batch advances one token per
layer call; the oracle runs the reference's layer for each sequence alone, on its
own cache, and every batched row must match it.

Tolerances (the layer tests' own): whole layer max-abs <= 5e-3 * max(1, max|ref|)
(the reference's layer check, test_layer.py:307); pool rows <= 2e-3 * max(1,
max|ref|), the projections' bound (rotated K and V rows come out of the fp16
projections); BatchDecoder against the same calls made one by one: bit-exact.
"""

from __future__ import annotations

import math

import numpy as np
import pytest

import layer_ref as L
from conftest import HAS_GPU

pytestmark = pytest.mark.gpu

if HAS_GPU:
    import torch

    import kvcache_ffi as ffi
    import paged

HID, INTER, H, HKV, D, PS = 512, 1024, 8, 2, 64, 16
EPS, BASE = 1e-5, 500000.0
NAMES = ("q", "k", "v", "o", "gate", "up", "down")
TYPES = {"q": L.Q4_K, "k": L.Q4_K, "v": L.Q6_K, "o": L.Q4_K, "gate": L.Q4_K, "up": L.Q4_K,
         "down": L.Q6_K}


@pytest.fixture(autouse=True)
def _clean(cuda_device):
    yield
    code, info = ffi.device_error(0, clear=True)
    assert code == 0, f"device error word left set: {code} {info}"


def _maxerr(a, b):
    return float(np.max(np.abs(a.astype(np.float32) - b.astype(np.float32))))


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _layer(rng, types=TYPES):
    qd, kd = H * D, HKV * D
    shapes = {"q": (qd, HID), "k": (kd, HID), "v": (kd, HID), "o": (HID, qd),
              "gate": (INTER, HID), "up": (INTER, HID), "down": (HID, INTER)}
    raws = {n: L.random_weight(rng, types[n], *shapes[n]) for n in NAMES}
    an = (1.0 + 0.05 * rng.standard_normal(HID, dtype=np.float32)).astype(np.float16)
    fn = (1.0 + 0.05 * rng.standard_normal(HID, dtype=np.float32)).astype(np.float16)
    lw = L.LayerWeights(an, *[(raws[n], types[n]) for n in NAMES[:4]], fn,
                        *[(raws[n], types[n]) for n in NAMES[4:]])
    dlw = paged.DeviceLayerWeights(_dev(an), _dev(fn), [_dev(raws[n]) for n in NAMES],
                                   [types[n] for n in NAMES], HID, INTER)
    return lw, dlw


def _oracle(x, lw, kc, vc, pos, neox):
    return L.layer_forward(x, lw, kc, vc, pos, num_heads=H, num_kv_heads=HKV, head_dim=D,
                           inter=INTER, eps=EPS, rope_base=BASE, neox=neox,
                           scale=1.0 / math.sqrt(D))


def _tol(ref):
    return 5e-3 * max(1.0, float(np.abs(ref.astype(np.float32)).max()))


def _tol_rows(ref):
    # the projections' bound: rows reach |x| ~ 3-4, where one or two fp16 spacings
    # (2e-3 each) separate the kernels' exact block scale from the oracle's fp16 weights
    return 2e-3 * max(1.0, float(np.abs(ref.astype(np.float32)).max()))


@pytest.mark.parametrize("neox", [False, True])
def test_forward_layer_paged_matches_oracle(neox):
    """Two layers, twelve sequences with ragged cached prefixes (0 .. 150 positions,
    pages in a random permutation): a causal prefill chunk per sequence through the
    same entry point (queries sharing a block-table row; chunks of 1-150 tokens),
    then two batched decode steps of 12 tokens.  Every row against the oracle run
    on that sequence alone; the pool rows against the oracle's cache."""
    rng = np.random.default_rng(2024 + neox)
    n_layers = 2
    pre = [36, 0, 89, 150, 17, 25, 31, 5, 64, 9, 1, 40]
    steps = 2
    table, total = paged.random_block_tables([p + steps for p in pre], PS, seed=3)
    pool = paged.PagedKVCache(n_layers, total, PS, HKV, D)
    bt = _dev(table)
    layers = [_layer(rng) for _ in range(n_layers)]
    S = max(pre) + steps
    kc = [[np.zeros((S, HKV, D), np.float16) for _ in pre] for _ in range(n_layers)]
    vc = [[np.zeros((S, HKV, D), np.float16) for _ in pre] for _ in range(n_layers)]
    plan = paged.DecodePlan()
    # prefill: sequence i's chunk as len(chunk) queries on row i, ctx 1..pre[i]
    for i, p in enumerate(pre):
        if p == 0:
            continue
        x = (rng.standard_normal((p, HID), dtype=np.float32) * 0.5).astype(np.float16)
        pool.plan(np.arange(1, p + 1), H, rows=[i] * p, plan=plan)
        for layer, (lw, dlw) in enumerate(layers):
            out = torch.empty((p, HID), dtype=torch.float16, device="cuda")
            pool.forward_layer(plan, layer, _dev(x), out, dlw, bt, EPS, BASE, neox)
            torch.cuda.synchronize()
            ref = _oracle(x, lw, kc[layer][i], vc[layer][i], 0, neox)
            got = out.cpu().numpy()
            assert _maxerr(got, ref) <= _tol(ref), ("prefill", i, layer, _maxerr(got, ref))
    # batched decode steps: one token per sequence at position ctx_i - 1
    ctx = np.asarray(pre) + 1
    for step in range(steps):
        x = (rng.standard_normal((len(pre), HID), dtype=np.float32) * 0.5).astype(np.float16)
        pool.plan(ctx, H, plan=plan)
        for layer, (lw, dlw) in enumerate(layers):
            out = torch.empty((len(pre), HID), dtype=torch.float16, device="cuda")
            pool.forward_layer(plan, layer, _dev(x), out, dlw, bt, EPS, BASE, neox)
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            for i in range(len(pre)):
                ref = _oracle(x[i:i + 1], lw, kc[layer][i], vc[layer][i], int(ctx[i]) - 1, neox)
                err = _maxerr(got[i:i + 1], ref)
                assert err <= _tol(ref), ("decode", step, i, layer, err)
        ctx += 1
    for layer in range(n_layers):
        for i, p in enumerate(pre):
            k, v = pool.gather(layer, bt, i, 0, p + steps)
            torch.cuda.synchronize()
            kr, vr = kc[layer][i][:p + steps], vc[layer][i][:p + steps]
            assert _maxerr(k.cpu().numpy(), kr) <= _tol_rows(kr), (layer, i)
            assert _maxerr(v.cpu().numpy(), vr) <= _tol_rows(vr), (layer, i)
    plan.close()
    pool.close()


def test_batch_decoder_equals_layer_calls():
    """BatchDecoder (prefill chunks, then decode steps through every layer) gives
    bit for bit what the same kvc_forward_layer_paged calls give one by one, on a
    second pool with the same pages; a mixed-type layer (F16, Q8_0, Q4_0 and the K
    types, gate and up of different types) takes the separate SwiGLU path."""
    rng = np.random.default_rng(7)
    mixed = {"q": L.F16, "k": L.Q8_0, "v": L.Q4_0, "o": L.Q6_K, "gate": L.Q4_0, "up": L.Q8_0,
             "down": L.Q4_K}
    layers = [_layer(rng), _layer(rng, mixed), _layer(rng)]
    pre = [20, 64, 3]
    steps = 3
    table, total = paged.random_block_tables([p + steps for p in pre], PS, seed=11)
    bt = _dev(table)
    pools = [paged.PagedKVCache(len(layers), total, PS, HKV, D) for _ in range(2)]
    dec = paged.BatchDecoder(pools[0], [d for _, d in layers], bt, H, [0] * len(pre), EPS, BASE)
    xs_pre = [(rng.standard_normal((p, HID), dtype=np.float32) * 0.5).astype(np.float16)
              for p in pre]
    xs = [(rng.standard_normal((len(pre), HID), dtype=np.float32) * 0.5).astype(np.float16)
          for _ in range(steps)]
    got = []
    for i, x in enumerate(xs_pre):
        got.append(dec.prefill(i, _dev(x)).cpu().numpy())
    for x in xs:
        got.append(dec.step(_dev(x)).cpu().numpy())
    assert list(dec.ctx) == [p + steps for p in pre]
    # the same calls by hand on the second pool
    plan = paged.DecodePlan()
    want = []

    def run(xdev):
        cur = xdev
        for layer, (_, dlw) in enumerate(layers):
            nxt = torch.empty_like(cur)
            pools[1].forward_layer(plan, layer, cur, nxt, dlw, bt, EPS, BASE)
            cur = nxt
        return cur.cpu().numpy()

    for i, (p, x) in enumerate(zip(pre, xs_pre)):
        pools[1].plan(np.arange(1, p + 1), H, rows=[i] * p, plan=plan)
        want.append(run(_dev(x)))
    ctx = np.asarray(pre) + 1
    for x in xs:
        pools[1].plan(ctx, H, plan=plan)
        want.append(run(_dev(x)))
        ctx += 1
    for g, w in zip(got, want):
        assert np.array_equal(g, w)
    for layer in range(len(layers)):
        for i, p in enumerate(pre):
            ka, va = pools[0].gather(layer, bt, i, 0, p + steps)
            kb, vb = pools[1].gather(layer, bt, i, 0, p + steps)
            assert torch.equal(ka, kb) and torch.equal(va, vb)
    dec.close()
    plan.close()
    for p in pools:
        p.close()


def test_forward_layer_paged_validation():
    """Status codes of kvc_forward_layer_paged: layer out of range (IndexError), an
    fp32 pool, a plan of another geometry, a query without a new row and an
    unsupported weight type (ValueError); nothing is launched for a rejected call."""
    rng = np.random.default_rng(1)
    _, dlw = _layer(rng)
    table, total = paged.random_block_tables([40, 17], PS, seed=2)
    bt = _dev(table)
    pool = paged.PagedKVCache(2, total, PS, HKV, D)
    plan = pool.plan([40, 17], H)
    x = torch.zeros((2, HID), dtype=torch.float16, device="cuda")
    out = torch.empty_like(x)
    with pytest.raises(IndexError):
        pool.forward_layer(plan, 2, x, out, dlw, bt)
    bad = paged.DeviceLayerWeights(dlw.attn_norm, dlw.ffn_norm, dlw.w,
                                   [99] + list(dlw.types[1:]), HID, INTER)
    with pytest.raises(ValueError):
        pool.forward_layer(plan, 0, x, out, bad, bt)
    other = paged.PagedKVCache(1, total, PS, HKV, 2 * D)
    with pytest.raises(ValueError):
        pool.forward_layer(other.plan([40, 17], H), 0, x, out, dlw, bt)
    f32 = paged.PagedKVCache(1, total, PS, HKV, D, dtype=torch.float32)
    with pytest.raises(ValueError):
        f32.forward_layer(f32.plan([40, 17], H), 0, x, out, dlw, bt)
    with pytest.raises(ValueError):
        pool.forward_layer(pool.plan([40, 0], H), 0, x, out, dlw, bt)
    torch.cuda.synchronize()
    for p in (pool, other, f32):
        p.close()
