"""kvc_decode_noalloc: the decode for callers that cannot allocate device memory.

Some hosts of this library (a runtime that owns all device memory through its
own arena, a plugin that may not call cudaMalloc) can hand over their KV pages,
q and out but cannot let the library allocate plan and split scratch.  This
entry point keeps that scratch in a fixed device array inside the library.  The
test calls it through the C ABI twice in a row and compares each result with
the regular kvc_decode on the same pages (same kernels and split partition, so
the results agree to the fp16 tolerance of the other tests; in practice they
are identical).  The file name makes pytest collect it last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import HAS_GPU

pytestmark = pytest.mark.gpu

if HAS_GPU:
    import torch

    import kvcache_ffi as ffi
    import paged


def _noalloc(pool, layer, bt, ctx, num_heads, q, out, scale):
    info = pool.info()
    k = info["k"] + layer * info["bytes_per_layer"]
    v = info["v"] + layer * info["bytes_per_layer"]
    ctx_np = np.ascontiguousarray(np.asarray(ctx, dtype=np.int32))
    stream = torch.cuda.current_stream()
    return ffi.lib.kvc_decode_noalloc(
        k, v, pool.num_pages, pool.page_size, pool.num_kv_heads, pool.head_dim, ffi.DTYPE_F16,
        int(bt.data_ptr()), int(bt.shape[-1]), ffi.np_ptr(ctx_np), len(ctx_np), num_heads,
        int(q.data_ptr()), int(out.data_ptr()), float(scale), int(stream.cuda_stream) or None)


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
        err = (got.float() - expect.float()).abs().max().item()
        tol = 2e-3 * max(1.0, expect.float().abs().max().item())
        assert err <= tol, f"call {call}: max-abs difference {err}"


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
