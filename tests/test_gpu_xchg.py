"""Head exchange (kvc_xchg_*, sharding.HeadShardedDecode transport "p2p") on GPUs.

One-GPU tests call the C ABI with the exchange connected to its own buffer
(kvc_xchg_connect_ptrs), which runs the whole push + publish + wait chain on one
device.  The two-GPU test (skipped with fewer GPUs) splits KV heads over two
processes and checks that the p2p transport and the NCCL all-gather transport
hand every rank the same outputs.
"""

from __future__ import annotations

import ctypes
import os
import socket

import numpy as np
import pytest

from conftest import HAS_GPU, assert_attention_close

pytestmark = pytest.mark.gpu

if HAS_GPU:
    import torch

    import gqa_ref
    import kvcache_ffi as ffi
    import paged


def _xchg(world, rank, slot_bytes, n_slots=2):
    h = ctypes.c_void_p()
    ffi.check(ffi.lib.kvc_xchg_create(0, rank, world, slot_bytes, n_slots, ctypes.byref(h)))
    return h


def _slot(h, i, shape):
    p = ctypes.c_void_p()
    ffi.check(ffi.lib.kvc_xchg_slot(h, i, ctypes.byref(p)))

    class _A:
        __cuda_array_interface__ = {"shape": shape, "typestr": "<f2", "data": (p.value, False),
                                    "version": 3, "strides": None}

    return torch.as_tensor(_A(), device="cuda:0")


def _connect_self(h, world):
    base = ctypes.c_void_p()
    ffi.check(ffi.lib.kvc_xchg_base(h, ctypes.byref(base)))
    arr = (ctypes.c_void_p * world)(*([base.value] * world))
    ffi.check(ffi.lib.kvc_xchg_connect_ptrs(h, arr))


def _case(seed=12, ctx=(700, 1, 2049, 33, 4000, 16)):
    H, Hkv, D, ps = 32, 8, 128, 16
    table, total = paged.random_block_tables(list(ctx), ps, seed)
    pool = paged.PagedKVCache(1, total, ps, Hkv, D)
    pool.fill_normal(seed=seed)
    bt = torch.from_numpy(table).cuda()
    rng = np.random.default_rng(seed)
    q = torch.from_numpy(rng.standard_normal((len(ctx), H, D), dtype=np.float32)).half().cuda()
    return H, Hkv, D, list(ctx), pool, bt, q


def test_xchg_one_rank_matches_decode_and_oracle(cuda_device):
    H, Hkv, D, ctx, pool, bt, q = _case()
    plan = pool.plan(ctx, H)
    scale = 1.0 / np.sqrt(D)
    expect = torch.zeros_like(q)
    pool.decode(plan, 0, q, expect, bt, scale)
    total = 2 * H  # this rank's heads sit at [H, 2H) of a wider output row
    h = _xchg(1, 0, len(ctx) * total * D * 2)
    try:
        _connect_self(h, 1)
        for call, slot in enumerate((0, 1, 0)):
            view = _slot(h, slot, (len(ctx), total, D))
            view.fill_(float("nan"))
            pool.append_decode_xchg(plan, 0, q, None, None, h, slot, total, H, bt, scale)
            torch.cuda.synchronize()
            assert ffi.device_error(0) == (0, 0)
            got = view[:, H:].float()
            assert torch.isnan(view[:, :H].float()).all(), "heads outside the rank's range were written"
            assert_attention_close(got.cpu().numpy(), expect.float().cpu().numpy(),
                                   f"exchange slot call {call} vs kvc_decode")
        # and against the oracle, per sequence
        info = pool.info()
        for i, c in enumerate(ctx):
            k, v = pool.gather(0, bt, i, 0, c)
            ref = gqa_ref.ref_gqa_attention(q[i:i + 1].cpu().numpy(), k.cpu().numpy(),
                                            v.cpu().numpy(), start_pos=c - 1, scale=scale,
                                            out_dtype=np.float32)[0]
            assert_attention_close(got[i].cpu().numpy(), ref, f"exchange slot vs oracle, query {i}")
        assert info["k"]
    finally:
        ffi.lib.kvc_xchg_destroy(h)


def test_xchg_fused_append_matches_append_decode(cuda_device):
    H, Hkv, D, ctx, pool, bt, q = _case(seed=5, ctx=(1025, 64, 3000))
    _, _, _, _, pool2, _, _ = _case(seed=5, ctx=(1025, 64, 3000))
    plan = pool.plan(ctx, H)
    plan2 = pool2.plan(ctx, H)
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    kn = torch.randn((len(ctx), Hkv, D), generator=g, device="cuda").half()
    vn = torch.randn((len(ctx), Hkv, D), generator=g, device="cuda").half()
    scale = 1.0 / np.sqrt(D)
    expect = torch.zeros_like(q)
    pool.append_decode(plan, 0, q, kn, vn, expect, bt, scale)
    h = _xchg(1, 0, len(ctx) * H * D * 2, n_slots=1)
    try:
        _connect_self(h, 1)
        pool2.append_decode_xchg(plan2, 0, q, kn, vn, h, 0, H, 0, bt, scale)
        torch.cuda.synchronize()
        got = _slot(h, 0, (len(ctx), H, D))
        assert_attention_close(got.float().cpu().numpy(), expect.float().cpu().numpy(),
                               "exchange with fused append vs append_decode")
        # the appended rows are in the pool, bit for bit
        for i, c in enumerate(ctx):
            k2, v2 = pool2.gather(0, bt, i, c - 1, 1)
            assert torch.equal(k2[0], kn[i]) and torch.equal(v2[0], vn[i])
    finally:
        ffi.lib.kvc_xchg_destroy(h)


def test_xchg_wait_gives_up_when_a_rank_never_publishes(cuda_device):
    """Rank 1's flag is never written (nothing plays rank 1): the exchange wait must
    give up after its limit, report it, and leave the context usable."""
    H, Hkv, D, ctx, pool, bt, q = _case(seed=8, ctx=(300, 40))
    plan = pool.plan(ctx, H)
    scale = 1.0 / np.sqrt(D)
    h = _xchg(2, 0, len(ctx) * H * D * 2)
    try:
        _connect_self(h, 2)  # "rank 1" is this buffer too; its flag word stays 0
        ffi.check(ffi.lib.kvc_xchg_set_wait_limit(h, 0.05))
        ffi.device_error(0)  # clear
        pool.append_decode_xchg(plan, 0, q, None, None, h, 0, H, 0, bt, scale)
        torch.cuda.synchronize()
        code, info = ffi.device_error(0)
        assert code == 2 and info == 0x10001, (code, info)
        # the GPU keeps working: a plain decode afterwards is correct and clean
        out = torch.zeros_like(q)
        pool.decode(plan, 0, q, out, bt, scale)
        torch.cuda.synchronize()
        assert ffi.device_error(0) == (0, 0)
        assert torch.isfinite(out.float()).all()
    finally:
        ffi.lib.kvc_xchg_destroy(h)


def test_xchg_rejects_bad_arguments(cuda_device):
    H, Hkv, D, ctx, pool, bt, q = _case(seed=9, ctx=(40,))
    plan = pool.plan(ctx, H)
    h = _xchg(1, 0, H * D * 2)
    try:
        with pytest.raises(ValueError):  # not connected yet
            pool.append_decode_xchg(plan, 0, q, None, None, h, 0, H, 0, bt, 0.1)
        _connect_self(h, 1)
        with pytest.raises(IndexError):
            pool.append_decode_xchg(plan, 0, q, None, None, h, 2, H, 0, bt, 0.1)
        with pytest.raises(ValueError):  # heads beyond total
            pool.append_decode_xchg(plan, 0, q, None, None, h, 0, H, 1, bt, 0.1)
        with pytest.raises(ValueError):  # slot too small for the wider row
            pool.append_decode_xchg(plan, 0, q, None, None, h, 0, 2 * H, H, bt, 0.1)
    finally:
        ffi.lib.kvc_xchg_destroy(h)
    bad = ctypes.c_void_p()
    assert ffi.lib.kvc_xchg_create(0, 0, 9, 64, 1, ctypes.byref(bad)) == ffi.KVC_ERR_INVALID_ARG
    assert ffi.lib.kvc_xchg_create(0, 2, 2, 64, 1, ctypes.byref(bad)) == ffi.KVC_ERR_INVALID_ARG


# ---- two GPUs: p2p transport == NCCL transport --------------------------------------
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_main(rank, port, results):
    import datetime

    import torch.distributed as dist

    import sharding

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        H, Hkv, D, ps, L = 32, 8, 128, 16, 2
        ctx = [900, 17, 2500, 4096, 1]
        h0, h1 = sharding.shard_heads(Hkv, 2, rank)
        q0, q1 = sharding.q_heads_for(H, Hkv, (h0, h1))
        table, total = paged.random_block_tables(ctx, ps, 4)
        bt = torch.from_numpy(table).cuda()
        pools = [paged.PagedKVCache(L, total, ps, h1 - h0, D, device=rank) for _ in range(2)]
        for p in pools:
            p.fill_normal(seed=100 + rank)
        g = torch.Generator(device="cuda")
        g.manual_seed(11)
        q = torch.randn((L, len(ctx), H, D), generator=g, device="cuda").half()[:, :, q0:q1]
        q = q.contiguous()
        kn = torch.randn((L, len(ctx), Hkv, D), generator=g, device="cuda").half()[:, :, h0:h1]
        vn = torch.randn((L, len(ctx), Hkv, D), generator=g, device="cuda").half()[:, :, h0:h1]
        kn, vn = kn.contiguous(), vn.contiguous()
        scale = 1.0 / np.sqrt(D)
        p2p = sharding.HeadShardedDecode(pools[0], H, Hkv, transport="p2p",
                                         num_queries=len(ctx))
        nccl = sharding.HeadShardedDecode(pools[1], H, Hkv, transport="nccl")
        plans = [p.plan(ctx, q1 - q0) for p in pools]
        worst = 0.0
        for step in range(3):
            for l in range(L):
                a = p2p.append_decode(plans[0], l, q[l], kn[l], vn[l], None, bt, scale).clone()
                b = nccl.append_decode(plans[1], l, q[l], kn[l], vn[l], None, bt, scale)
                torch.cuda.synchronize()
                # per query row: max|p2p - nccl| / max|nccl| (the fp16 bound's form)
                d = (a.float() - b.float()).abs().amax(dim=(1, 2))
                m = b.float().abs().amax(dim=(1, 2)).clamp_min(1e-30)
                worst = max(worst, (d / m).max().item())
        code, info = ffi.device_error(rank)
        p2p.close()
        results[rank] = (worst, code, info)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not HAS_GPU or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_p2p_exchange_matches_nccl_all_gather():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_two_rank_main, args=(r, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        if p.is_alive():
            p.kill()
    assert [p.exitcode for p in procs] == [0, 0]
    for rank in (0, 1):
        worst, code, info = results[rank]
        assert code == 0, (rank, code, info)
        assert worst <= 2e-3, (rank, worst)
