"""kvc_decode_noalloc: the decode for callers that cannot allocate device memory.

Some hosts of this library (a runtime that owns all device memory through its
own arena, a plugin that may not call cudaMalloc) can hand over their KV pages,
q and out but cannot let the library allocate plan and split scratch.  This
entry point keeps that scratch in a fixed device array inside the library.  The
tests call it through the C ABI twice in a row and compare each result with the
regular kvc_decode on the same pages (same kernels and split partition, so the
results agree to the fp16 bound of the other tests; in practice they are
identical) and with the CPU oracle on the gathered pool contents; an
even-context batch of several waves checks that it cuts the splits exactly as
kvc_plan_decode does (tail quartering); a capturing stream is refused cleanly.
The file name makes pytest collect it last.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import HAS_GPU, assert_attention_close

pytestmark = pytest.mark.gpu

if HAS_GPU:
    import torch

    import gqa_ref  # oracle: checker only
    import kvcache_ffi as ffi
    import paged


def _noalloc(pool, layer, bt, ctx, num_heads, q, out, scale, stream=None):
    info = pool.info()
    k = info["k"] + layer * info["bytes_per_layer"]
    v = info["v"] + layer * info["bytes_per_layer"]
    ctx_np = np.ascontiguousarray(np.asarray(ctx, dtype=np.int32))
    stream = torch.cuda.current_stream() if stream is None else stream
    return ffi.lib.kvc_decode_noalloc(
        k, v, pool.num_pages, pool.page_size, pool.num_kv_heads, pool.head_dim, ffi.DTYPE_F16,
        int(bt.data_ptr()), int(bt.shape[-1]), ffi.np_ptr(ctx_np), len(ctx_np), num_heads,
        int(q.data_ptr()), int(out.data_ptr()), float(scale), int(stream.cuda_stream) or None)


def _oracle(pool, layer, bt, ctx, q, scale):
    ks, vs = [], []
    for i, c in enumerate(ctx):
        k, v = pool.gather(layer, bt, i, 0, c)
        ks.append(k.cpu().numpy())
        vs.append(v.cpu().numpy())
    return gqa_ref.batched_decode(q.cpu().numpy(), ks, vs, ctx, scale, out_dtype=np.float16)


def test_noalloc_matches_kvc_decode_twice(cuda_device):
    rng = np.random.default_rng(31)
    H, Hkv, D, ps = 32, 8, 128, 16
    ctx = [1500, 1, 700, 2049, 33, 512, 513, 4000]
    table, total = paged.random_block_tables(ctx, ps, 5)
    pool = paged.PagedKVCache(2, total, ps, Hkv, D)
    pool.fill_normal(seed=9)
    bt = torch.from_numpy(table).cuda()
    scale = 1.0 / np.sqrt(D)
    plan = pool.plan(ctx, H)
    for call, layer in enumerate((1, 0)):
        q = torch.from_numpy(rng.standard_normal((len(ctx), H, D), dtype=np.float32)).half().cuda()
        expect = torch.zeros_like(q)
        pool.decode(plan, layer, q, expect, bt, scale)
        got = torch.full_like(q, float("nan"))
        rc = _noalloc(pool, layer, bt, ctx, H, q, got, scale)
        assert rc == 0, ffi.last_error()
        torch.cuda.synchronize()
        assert ffi.device_error(0) == (0, 0)
        assert_attention_close(got.cpu().numpy(), expect.cpu().numpy(),
                               f"noalloc call {call} vs kvc_decode")
        if call == 0:
            assert_attention_close(got.cpu().numpy(), _oracle(pool, layer, bt, ctx, q, scale),
                                   "noalloc vs oracle (ragged batch)")
    plan.close()
    pool.close()


def test_noalloc_even_multiwave_batch_uses_the_plan_partition(cuda_device):
    """40 sequences x 2048 positions, 8 KV heads: 1,280 full 512-position units on
    148 x 8 warps, so the last wave would be 96 units; kvc_plan_decode quarters
    12 full splits (196 split slots) and kvc_decode_noalloc must cut the same."""
    rng = np.random.default_rng(77)
    H, Hkv, D, ps = 32, 8, 128, 16
    ctx = [2048] * 40
    table, total = paged.random_block_tables(ctx, ps, 8)
    pool = paged.PagedKVCache(1, total, ps, Hkv, D)
    pool.fill_normal(seed=10)
    bt = torch.from_numpy(table).cuda()
    scale = 1.0 / np.sqrt(D)
    plan = pool.plan(ctx, H)
    info = plan.info()
    assert info.n_items == 40 * 4 + 3 * 12, info  # tail quartering is in this plan
    for call in range(2):
        q = torch.from_numpy(rng.standard_normal((len(ctx), H, D), dtype=np.float32)).half().cuda()
        expect = torch.zeros_like(q)
        pool.decode(plan, 0, q, expect, bt, scale)
        got = torch.full_like(q, float("nan"))
        rc = _noalloc(pool, 0, bt, ctx, H, q, got, scale)
        assert rc == 0, ffi.last_error()
        torch.cuda.synchronize()
        assert ffi.device_error(0) == (0, 0)
        assert_attention_close(got.cpu().numpy(), expect.cpu().numpy(),
                               f"noalloc even multi-wave call {call} vs kvc_decode")
        if call == 1:
            assert_attention_close(got.cpu().numpy(), _oracle(pool, 0, bt, ctx, q, scale),
                                   "noalloc vs oracle (even multi-wave batch)")
    plan.close()
    pool.close()


def test_noalloc_refuses_a_capturing_stream(cuda_device):
    H, Hkv, D, ps = 8, 2, 64, 16
    ctx = [40, 17]
    table, total = paged.random_block_tables(ctx, ps, 2)
    pool = paged.PagedKVCache(1, total, ps, Hkv, D)
    pool.fill_normal(seed=3)
    bt = torch.from_numpy(table).cuda()
    q = torch.zeros((len(ctx), H, D), dtype=torch.float16, device="cuda")
    out = torch.zeros_like(q)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.graph(graph, stream=s):
        rc = _noalloc(pool, 0, bt, ctx, H, q, out, 0.125, stream=s)
        out.add_(1.0)  # the capture itself stays valid
    assert rc == ffi.KVC_ERR_INVALID_ARG
    assert "captured" in ffi.last_error()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.all(out == 1.0)
    # outside the capture the same call runs
    rc = _noalloc(pool, 0, bt, ctx, H, q, out, 0.125)
    assert rc == 0, ffi.last_error()
    torch.cuda.synchronize()
    assert ffi.device_error(0) == (0, 0)
    del graph
    pool.close()


def test_noalloc_rejects_requests_beyond_its_scratch(cuda_device):
    H, Hkv, D, ps = 64, 8, 128, 16
    ctx = [32768] * 8  # 8 x 64 splits x 64 heads of fp32 partials: far beyond 16 MiB
    table, total = paged.random_block_tables(ctx, ps, 1)
    pool = paged.PagedKVCache(1, total, ps, Hkv, D)
    bt = torch.from_numpy(table).cuda()
    q = torch.zeros((len(ctx), H, D), dtype=torch.float16, device="cuda")
    out = torch.zeros_like(q)
    rc = _noalloc(pool, 0, bt, ctx, H, q, out, 0.1)
    assert rc == ffi.KVC_ERR_INVALID_ARG
    assert "scratch" in ffi.last_error()
    with pytest.raises(ValueError):
        ffi.check(rc)
    pool.close()
