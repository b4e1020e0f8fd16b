"""Multi-GPU host logic on CPU: two gloo ranks, oracle arithmetic.

The CUDA decode cannot run here, so each rank computes its shard with the oracle
(the checker) and the test exercises what the multi-GPU path adds on top of the
single-GPU kernel: which KV heads / q-heads / sequences a rank owns, and the
per-layer all-gather that puts every rank's heads back in the unsharded order.
Sharded results must equal the unsharded oracle result exactly (per-head and
per-sequence arithmetic is independent of the split).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import gqa_ref
import sharding

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case():
    rng = np.random.default_rng(77)
    H, Hkv, D = 8, 4, 32
    ctx = np.array([5, 1, 40, 17, 64], dtype=np.int64)
    q = rng.standard_normal((len(ctx), H, D)).astype(np.float32)
    ks = [rng.standard_normal((c, Hkv, D)).astype(np.float32) for c in ctx]
    vs = [rng.standard_normal((c, Hkv, D)).astype(np.float32) for c in ctx]
    return H, Hkv, D, ctx, q, ks, vs


def _rank_main(rank: int, port: int, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        H, Hkv, D, ctx, q, ks, vs = _case()
        scale = 1.0 / np.sqrt(D)
        full = gqa_ref.batched_decode(q, ks, vs, ctx, scale)

        # --- KV-head sharding: local heads, then the all-gather ---
        h0, h1 = sharding.shard_heads(Hkv, WORLD, rank)
        q0, q1 = sharding.q_heads_for(H, Hkv, (h0, h1))
        local = gqa_ref.batched_decode(q[:, q0:q1], [k[:, h0:h1] for k in ks],
                                       [v[:, h0:h1] for v in vs], ctx, scale)
        out = torch.full((len(ctx), H, D), float("nan"))
        sharding.gather_head_outputs(torch.from_numpy(local), out)
        heads_ok = bool(np.array_equal(out.numpy(), full))

        # --- sequence sharding: whole sequences per rank, no data exchange ---
        s0, s1 = sharding.shard_sequences(len(ctx), WORLD, rank)
        mine = gqa_ref.batched_decode(q[s0:s1], ks[s0:s1], vs[s0:s1], ctx[s0:s1], scale)
        # checking only: collect every rank's rows to compare with the full batch
        pad = np.zeros((len(ctx), H, D), dtype=np.float32)
        pad[s0:s1] = mine
        t = torch.from_numpy(pad)
        dist.all_reduce(t)
        seqs_ok = bool(np.array_equal(t.numpy(), full))
        results[rank] = (heads_ok, seqs_ok, (h0, h1), (q0, q1), (s0, s1))
    finally:
        dist.destroy_process_group()


def test_two_rank_head_and_sequence_sharding_match_unsharded():
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, results)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = dict(results)
    assert set(got) == {0, 1}
    for rank, (heads_ok, seqs_ok, kv, qh, seq) in got.items():
        assert heads_ok, f"rank {rank}: gathered heads differ from the unsharded result"
        assert seqs_ok, f"rank {rank}: sequence shards differ from the unsharded result"
    assert got[0][2] == (0, 2) and got[1][2] == (2, 4)
    assert got[0][3] == (0, 4) and got[1][3] == (4, 8)
    assert got[0][4] == (0, 3) and got[1][4] == (3, 5)


def test_shard_ranges_cover_everything_once():
    for world in (1, 2, 4, 8):
        heads = [sharding.shard_heads(8, world, r) for r in range(world)]
        assert heads[0][0] == 0 and heads[-1][1] == 8
        assert all(a[1] == b[0] for a, b in zip(heads, heads[1:]))
        for n in (0, 1, 7, 8, 33):
            seqs = [sharding.shard_sequences(n, world, r) for r in range(world)]
            assert seqs[0][0] == 0 and seqs[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(seqs, seqs[1:]))
            sizes = [b - a for a, b in seqs]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.shard_heads(8, 3, 0)
    with pytest.raises(ValueError):
        sharding.shard_heads(8, 2, 2)
    with pytest.raises(ValueError):
        sharding.q_heads_for(12, 8, (0, 1))


def test_gather_rejects_wrong_output_shape():
    port = _free_port()
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        local = torch.zeros((2, 4, 8))
        with pytest.raises(ValueError):
            sharding.gather_head_outputs(local, torch.zeros((2, 8, 8)))
        out = torch.zeros((2, 4, 8))
        sharding.gather_head_outputs(local + 1, out)
        assert torch.equal(out, local + 1)
    finally:
        dist.destroy_process_group()


def _failing_rank_main(rank: int, port: int, mode: str, results):
    # Rank 1 fails between two layers of a KV-head-sharded decode (it raises, or its
    # process ends without a word); rank 0 goes on to the next layer's head gather.
    # With a short process-group timeout that gather must end with an error on
    # rank 0, so a serving loop learns of the lost rank instead of waiting for good.
    import datetime
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=3))
    B, hl, D = 3, 4, 16
    local = torch.full((B, hl, D), float(rank))
    out = torch.empty((B, WORLD * hl, D))
    sharding.gather_head_outputs(local, out)              # layer 0: both ranks present
    results[(rank, "layer0")] = bool(torch.equal(out[:, hl:], torch.ones((B, hl, D))))
    if rank == 1:
        if mode == "raise":
            results[(rank, "left")] = True
            raise RuntimeError("rank 1 failed between layers (planted on the host)")
        results[(rank, "left")] = True
        os._exit(0)                                       # ends without a word
    t0 = time.monotonic()
    try:
        sharding.gather_head_outputs(local, out)          # layer 1: rank 1 never comes
        results[(rank, "error")] = None
    except Exception as e:  # noqa: BLE001 - the backend's error type varies by version
        results[(rank, "error")] = type(e).__name__
    results[(rank, "waited_s")] = time.monotonic() - t0
    os._exit(0)  # the group cannot be torn down collectively without the lost rank


@pytest.mark.parametrize("mode", ["raise", "exit"])
def test_lost_rank_ends_the_survivors_next_gather_with_an_error(mode):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank_main, args=(r, port, mode, results))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    got = dict(results)
    assert got.get((0, "layer0")) and got.get((1, "layer0")), got
    assert got.get((1, "left")), got
    assert procs[0].exitcode == 0, procs[0].exitcode
    assert got.get((0, "error")) is not None, "the survivor's gather returned without its peer"
    assert got[(0, "waited_s")] < 60.0, got
