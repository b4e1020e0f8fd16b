"""Every head dim and group shape of the tensor-core decode, fp16 and bf16.

The persistent decode kernel is instantiated per head dim (32 ... 256) and
handles q-head groups in chunks of eight; these cases run each instantiation on
a ragged batch whose contexts cross split boundaries (so the split merge runs)
and compare with the oracle on the gathered pool contents.  Tolerances, per
query row relative to its largest |ref| (conftest.assert_attention_close):
fp16 storage 2e-3 as in the other parity tests; bf16 (8-bit mantissa) 1.6e-2.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import HAS_GPU, assert_attention_close

pytestmark = pytest.mark.gpu

if HAS_GPU:
    import torch

    import gqa_ref
    import paged

HEAD_DIMS = [32, 64, 96, 128, 160, 192, 256]
GROUPS = [1, 3, 8, 16]


def _run(D, group, dtype, seed):
    rng = np.random.default_rng(seed)
    Hkv = 2
    H = group * Hkv
    ctx = [1, 600, 1500, 129]
    table, total = paged.random_block_tables(ctx, 16, seed)
    pool = paged.PagedKVCache(1, total, 16, Hkv, D, dtype=dtype)
    pool.fill_normal(seed=seed, stddev=0.5)
    bt = torch.from_numpy(table).cuda()
    q = torch.from_numpy(rng.standard_normal((len(ctx), H, D), dtype=np.float32) * 0.5)
    q = q.to(dtype).cuda()
    out = torch.zeros_like(q)
    scale = 1.0 / np.sqrt(D)
    plan = pool.plan(ctx, H)
    pool.decode(plan, 0, q, out, bt, scale)
    torch.cuda.synchronize()
    ks, vs = [], []
    for i, c in enumerate(ctx):
        k, v = pool.gather(0, bt, i, 0, c)
        ks.append(k.float().cpu().numpy())
        vs.append(v.float().cpu().numpy())
    ref = gqa_ref.batched_decode(q.float().cpu().numpy(), ks, vs, ctx, scale)
    got = out.float().cpu().numpy()
    return got, ref


@pytest.mark.parametrize("D", HEAD_DIMS)
def test_head_dims_fp16(D):
    got, ref = _run(D, 4, torch.float16, 40 + D)
    assert_attention_close(got, ref, f"fp16 head_dim {D}")


@pytest.mark.parametrize("group", GROUPS)
def test_group_sizes_fp16(group):
    got, ref = _run(128, group, torch.float16, 70 + group)
    assert_attention_close(got, ref, f"fp16 group {group}")


@pytest.mark.parametrize("D", [64, 128, 256])
def test_head_dims_bf16(D):
    got, ref = _run(D, 8, torch.bfloat16, 90 + D)
    assert_attention_close(got, ref, f"bf16 head_dim {D}", rel=1.6e-2)
