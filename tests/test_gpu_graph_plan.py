"""Graph-stable decode plans (KVC_PLAN_GRAPH) on a B200.

A decode loop whose contexts grow by one position per step rebuilds its plan
every step.  With a graph-stable plan the step's launches are captured once in a
CUDA graph and replayed after each rebuild: the kernels read the plan's counts
from its device header, so the replay follows the new partition.  These tests
grow a ragged batch across split boundaries, multi-split thresholds and the
merge's warps-per-head steps, and check every replayed step bit for bit against
direct launches of an ordinary plan of the same contexts (the partition and
every addition order are the same), and against the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

import gqa_ref
from conftest import HAS_GPU, assert_attention_close

pytestmark = pytest.mark.gpu

if HAS_GPU:
    import torch

    import kvcache_ffi as ffi
    import paged


def _oracle(pool, layer, bt, ctx, q, scale):
    ks, vs = [], []
    for i, c in enumerate(ctx):
        k, v = pool.gather(layer, bt, i, 0, int(c))
        ks.append(k.cpu().numpy())
        vs.append(v.cpu().numpy())
    return gqa_ref.batched_decode(q.cpu().numpy(), ks, vs, [int(c) for c in ctx], scale,
                                  out_dtype=np.float16)


def _setup(ctx_max, H, Hkv, D, layers=2, ps=16, seed=3):
    table, total = paged.random_block_tables(ctx_max, ps, seed)
    pool = paged.PagedKVCache(layers, total, ps, Hkv, D)
    pool.fill_normal(seed=seed + 1)
    bt = torch.from_numpy(table).cuda()
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = torch.randn((layers, len(ctx_max), H, D), generator=g, device="cuda").half()
    return pool, bt, q


def test_graph_replay_follows_rebuilt_plans_bit_for_bit(cuda_device):
    H, Hkv, D = 16, 4, 128
    start = np.array([1, 15, 16, 17, 300, 511, 513, 1024, 2000, 48], dtype=np.int32)
    steps, stride = 24, 40          # +40 positions per step: many split boundaries crossed
    pool, bt, q = _setup(start + steps * stride, H, Hkv, D)
    scale = 1.0 / np.sqrt(D)
    s = torch.cuda.current_stream()
    out = torch.zeros((2, len(start), H, D), dtype=torch.float16, device="cuda")
    ref = torch.zeros_like(out)
    gplan = paged.DecodePlan()
    gplan.set_kv_stable(True)
    gplan.set_graph_stable(True)
    plain = paged.DecodePlan()
    graph, gen, captures, n_units_seen, checked = None, None, 0, set(), 0
    for step in range(steps):
        ctx = start + step * stride
        pool.plan(ctx, H, plan=gplan, stream=s)
        if graph is None or gplan.generation != gen:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for layer in range(2):
                    pool.decode(gplan, layer, q[layer], out[layer], bt, scale,
                                stream=torch.cuda.current_stream())
            gen, captures = gplan.generation, captures + 1
        graph.replay()
        pool.plan(ctx, H, plan=plain, stream=s)
        for layer in range(2):
            pool.decode(plain, layer, q[layer], ref[layer], bt, scale, stream=s)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"step {step}: replayed graph differs from direct launches"
        n_units_seen.add(plain.info().n_ctas)
        if step in (0, steps // 2, steps - 1):
            for layer in range(2):
                assert_attention_close(out[layer].cpu().numpy(),
                                       _oracle(pool, layer, bt, ctx, q[layer], scale),
                                       f"graph replay, step {step}, layer {layer}")
            checked += 1
    assert checked == 3
    assert len(n_units_seen) > 5          # the partition really changed under the graph
    assert captures < steps // 2          # rebuilds within capacity kept the captured launches
    code, info = ffi.device_error(0, clear=True)
    assert code == 0, (code, info)


def test_graph_plan_generation_and_validation(cuda_device):
    H, Hkv, D = 8, 2, 128
    pool, bt, q = _setup(np.array([4000, 4000]), H, Hkv, D, layers=1)
    p = paged.DecodePlan()
    p.set_graph_stable(True)
    s = torch.cuda.current_stream()
    pool.plan([100, 200], H, plan=p, stream=s)
    g0 = p.generation
    pool.plan([101, 201], H, plan=p, stream=s)      # same capacity: same layout
    assert p.generation == g0
    pool.plan([4000, 4000], H, plan=p, stream=s)    # far more splits: the layout grows
    assert p.generation > g0
    g1 = p.generation
    pool.plan([4000], H, plan=p, stream=s)          # another query count: new launch shape
    assert p.generation > g1
    # switching the flag lays the plan out again
    g2 = p.generation
    p.set_graph_stable(False)
    assert p.generation > g2
    # an fp32 pool has no graph-stable form
    pool32 = paged.PagedKVCache(1, 8, 16, 2, 128, dtype=torch.float32)
    p32 = paged.DecodePlan()
    p32.set_graph_stable(True)
    with pytest.raises(ValueError):
        pool32.plan([16], H, plan=p32, stream=s)
    for x in (p, p32):
        x.close()
    pool.close()
    pool32.close()


def test_graph_replay_past_table_width_reports_bad_page(cuda_device):
    # A replayed launch does not repeat the host's check of the contexts against
    # the block-table width (a rebuild only uploads the plan): a context grown past
    # the table's row is reported by the kernels as a bad page, and the entries
    # past the row's end are never read.
    H, Hkv, D = 8, 2, 128
    pool, bt, q = _setup(np.array([64, 64]), H, Hkv, D, layers=1)
    assert bt.shape[-1] == 4                       # 4 pages of 16 positions per row
    scale = 1.0 / np.sqrt(D)
    s = torch.cuda.current_stream()
    out = torch.zeros((2, H, D), dtype=torch.float16, device="cuda")
    p = paged.DecodePlan()
    p.set_graph_stable(True)
    ffi.device_error(0, clear=True)
    # a first build at longer contexts sizes the plan's block and scratch, so the
    # rebuilds below stay within them and keep the captured launch's addresses
    pool.plan([200, 200], H, plan=p, stream=s)
    pool.plan([60, 60], H, plan=p, stream=s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        pool.decode(p, 0, q[0], out, bt, scale, stream=torch.cuda.current_stream())
    gen = p.generation
    graph.replay()
    torch.cuda.synchronize()
    assert ffi.device_error(0, clear=True)[0] == 0
    pool.plan([80, 80], H, plan=p, stream=s)       # 5 pages: one past the row
    assert p.generation == gen                     # the captured launch stays valid
    graph.replay()
    torch.cuda.synchronize()
    code, _ = ffi.device_error(0, clear=True)
    assert code == 1                               # KVC_DEVERR_BAD_PAGE
    # the context stays usable: back within the table, the replay is clean
    pool.plan([60, 60], H, plan=p, stream=s)
    graph.replay()
    torch.cuda.synchronize()
    assert ffi.device_error(0, clear=True)[0] == 0
    assert_attention_close(out.cpu().numpy(), _oracle(pool, 0, bt, [60, 60], q[0], scale),
                           "graph replay back within the table")
    del graph
    p.close()
    pool.close()
