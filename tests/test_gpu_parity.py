"""CUDA parity tests (B200): every entry point against the pinned oracle.

Tolerances (the path's parity targets and the reference's own tests):
  fp32 storage                 max-abs <= 1e-5
  fp16 storage, fp32 accumulate per query row max|got - ref| <= 2e-3 * max|ref|
                               (conftest.assert_attention_close); the reference's own
                               tests use max-abs 2e-3 (test_layer.py:179) and 1e-3
                               (test_full_model.py:104/124)
  pool contents, fused vs separate calls: bit-exact.
The reference's KVCacheManager flows (gpu / cpu / mmap modes, offload engine)
are replayed in tests/test_gpu_reference_callsites.py.
"""

from __future__ import annotations

import numpy as np
import pytest

import cases
import gqa_ref
from conftest import HAS_GPU, assert_attention_close

pytestmark = pytest.mark.gpu

if HAS_GPU:
    import torch

    import kvcache_ffi as ffi
    import matmul_module
    import paged

G = cases.load_golden() if HAS_GPU else {}


def _maxerr(a, b):
    return float(np.max(np.abs(a.astype(np.float32) - b.astype(np.float32))))


@pytest.fixture(autouse=True)
def _clean(cuda_device):
    yield
    matmul_module.kv_cache_free()
    code, info = ffi.device_error(0, clear=True)
    assert code == 0, f"device error word left set: {code} {info}"


# ---------------------------------------------------------------------------
# host full-KV entry (matmul_module.gqa_attention, attention.hip:228-284)
# ---------------------------------------------------------------------------
def test_reference_layer_cases_gqa_attention():
    """tests/test_layer.py:155-184 through the drop-in gqa_attention."""
    for i, c in enumerate(cases.layer_cases()):
        out = np.zeros_like(c["Q"])
        matmul_module.gqa_attention(c["Q"], c["K"], c["V"], out, c["q_len"], c["kv_len"], 16, 4,
                                    64, c["start_pos"], c["scale"], True)
        assert _maxerr(out, G[f"layer{i}_out"]) < 2e-3  # the reference test's tolerance
        assert_attention_close(out, G[f"layer{i}_out"], f"reference layer case {i}")


@pytest.mark.parametrize("name", list(cases.EDGE_CASES))
def test_edge_cases_gqa_attention(name):
    c = cases.edge_case(name)
    ref = G[f"{name}_out"]
    out = np.zeros_like(c["Q"])
    H, D = c["Q"].shape[1], c["Q"].shape[2]
    Hkv = c["K"].shape[1]
    matmul_module.gqa_attention(c["Q"], c["K"], c["V"], out, c["q_len"], c["kv_len"], H, Hkv, D,
                                c["start_pos"], c["scale"], c["causal"])
    if c["Q"].dtype == np.float32:
        assert _maxerr(out, ref) <= 1e-5
    else:
        assert_attention_close(out, ref, f"edge case {name}")


def test_scale_zero_follows_the_kernel():
    """scale = 0 gives equal scores (attention.hip:99): output = mean of V."""
    c = cases.edge_case("scale_custom")
    out = np.zeros_like(c["Q"])
    matmul_module.gqa_attention(c["Q"], c["K"], c["V"], out, 1, c["kv_len"], 8, 2, 64,
                                c["start_pos"], 0.0, True)
    expect = gqa_ref.online_softmax_attention(c["Q"], c["K"], c["V"], c["start_pos"], 0.0)
    assert_attention_close(out, expect, "scale 0 (equal scores)")


def test_empty_context_gives_zeros():
    """kv_len = 0: nothing attended -> zero rows (attention.hip:115)."""
    q = np.ones((2, 4, 32), np.float16)
    out = np.full_like(q, 7)
    k = np.zeros((0, 2, 32), np.float16)
    matmul_module.gqa_attention(q, k, k, out, 2, 0, 4, 2, 32, 0, 0.2, False)
    assert not out.any()


# ---------------------------------------------------------------------------
# GPU-resident pool (kv_cache_init / gqa_attention_cached / KVCacheManager)
# ---------------------------------------------------------------------------
def test_config1_fp32_pool_within_1e5():
    """benchmark config 1: fp32 pool, 511 cached + 1 appended, max-abs 1e-5."""
    c = cases.config1_case()
    P, H, Hkv, D = c["kv_len"], 32, 4, 64
    matmul_module.kv_cache_init_ex(1, P, Hkv, D, dtype=np.float32)
    q_pre = np.zeros((P - 1, H, D), np.float32)  # prefill rows (outputs unused)
    out_pre = np.zeros_like(q_pre)
    matmul_module.gqa_attention_cached(q_pre, c["K"][:P - 1], c["V"][:P - 1], out_pre, 0, P - 1,
                                       0, H, Hkv, D, c["scale"], True)
    out = np.zeros((1, H, D), np.float32)
    matmul_module.gqa_attention_cached(c["Q"], c["K"][P - 1:], c["V"][P - 1:], out, 0, 1, P - 1,
                                       H, Hkv, D, c["scale"], True)
    assert _maxerr(out, G["config1_out_f32"]) <= 1e-5
    k, v = matmul_module.kv_cache_gather(0, 0, P)
    np.testing.assert_array_equal(k, c["K"])
    np.testing.assert_array_equal(v, c["V"])


def test_cached_prefill_matches_host_attention_bit_exact():
    """The cached path and the full-KV host path share kernels and splits."""
    c = cases.edge_case("split_boundary_1025")
    H, Hkv, D, P = 8, 2, 128, c["kv_len"]
    matmul_module.kv_cache_init(1, 2048, Hkv, D)
    rng = np.random.default_rng(5)
    qp = (rng.standard_normal((P - 1, H, D), dtype=np.float32) * 0.5).astype(np.float16)
    outp = np.zeros_like(qp)
    matmul_module.gqa_attention_cached(qp, c["K"][:P - 1], c["V"][:P - 1], outp, 0, P - 1, 0, H,
                                       Hkv, D, c["scale"], True)
    out = np.zeros_like(c["Q"])
    matmul_module.gqa_attention_cached(c["Q"], c["K"][P - 1:], c["V"][P - 1:], out, 0, 1, P - 1,
                                       H, Hkv, D, c["scale"], True)
    assert_attention_close(out, G["split_boundary_1025_out"], "cached decode at the 1025 split boundary")
    out2 = np.zeros_like(c["Q"])
    matmul_module.gqa_attention(c["Q"], c["K"], c["V"], out2, 1, P, H, Hkv, D, P - 1, c["scale"])
    np.testing.assert_array_equal(out, out2)
    # Prefill row m of the cached call vs the same queries asked alone.  The two
    # calls have different sizes, so the plan may cut their contexts into splits
    # of different lengths (512 for the 1024-query prefill, 128 for 3 queries):
    # the results agree to rounding, not bit for bit.
    outp2 = np.zeros_like(qp[:3])
    matmul_module.gqa_attention(qp[600:603], c["K"][:603], c["V"][:603], outp2, 3, 603, H, Hkv,
                                D, 600, c["scale"])
    assert_attention_close(outp[600:603], outp2, "prefill rows vs the same queries alone")
    ref = gqa_ref.ref_gqa_attention(qp[600:603], c["K"][:603], c["V"][:603], 600, c["scale"])
    assert_attention_close(outp[600:603], ref, "cached prefill rows 600-602")


def test_validation_matches_reference_exception_classes():
    matmul_module.kv_cache_init(2, 16, 2, 32)
    q = np.zeros((1, 4, 32), np.float16)
    kn = np.zeros((1, 2, 32), np.float16)
    out = np.zeros_like(q)
    with pytest.raises(IndexError, match="layer_idx"):
        matmul_module.gqa_attention_cached(q, kn, kn, out, 2, 1, 0, 4, 2, 32)
    with pytest.raises(IndexError, match="max_seq_len"):
        matmul_module.gqa_attention_cached(q, kn, kn, out, 0, 1, 16, 4, 2, 32)
    with pytest.raises(IndexError, match="max_seq_len"):
        matmul_module.gqa_attention_cached(q, kn, kn, out, 0, 1, -1, 4, 2, 32)
    with pytest.raises(ValueError, match="mismatch"):
        matmul_module.gqa_attention_cached(q, kn, kn, out, 0, 1, 0, 4, 1, 32)
    with pytest.raises(ValueError, match="FP16"):
        matmul_module.gqa_attention_cached(q.astype(np.float32), kn, kn, out, 0, 1, 0, 4, 2, 32)
    with pytest.raises(ValueError, match="C-contiguous"):
        matmul_module.gqa_attention_cached(np.zeros((1, 4, 64), np.float16)[:, :, ::2], kn, kn,
                                           out, 0, 1, 0, 4, 2, 32)
    ro = out.copy()
    ro.flags.writeable = False
    with pytest.raises(ValueError, match="writeable"):
        matmul_module.gqa_attention_cached(q, kn, kn, ro, 0, 1, 0, 4, 2, 32)
    with pytest.raises(ValueError, match="smaller"):
        matmul_module.gqa_attention_cached(q, kn, kn, out[:, :2], 0, 1, 0, 4, 2, 32)
    # grow-only re-init keeps working; free + call -> RuntimeError
    matmul_module.kv_cache_init(1, 8, 2, 32)
    matmul_module.gqa_attention_cached(q, kn, kn, out, 0, 1, 0, 4, 2, 32)
    matmul_module.kv_cache_free()
    with pytest.raises(RuntimeError, match="not initialized"):
        matmul_module.gqa_attention_cached(q, kn, kn, out, 0, 1, 0, 4, 2, 32)


# ---------------------------------------------------------------------------
# paged batched decode
# ---------------------------------------------------------------------------
def _ragged_pool(page_size=16, dtype=None, seed=3):
    dtype = dtype or torch.float16
    c = cases.ragged_case()
    n, H, Hkv, D = len(c["ctx"]), c["H"], c["Hkv"], c["D"]
    table, total = paged.random_block_tables(c["ctx"], page_size, seed)
    pool = paged.PagedKVCache(1, total + 3, page_size, Hkv, D, dtype=dtype)
    bt = torch.from_numpy(table).cuda()
    for i, ctx in enumerate(c["ctx"]):
        k = torch.from_numpy(c["ks"][i]).cuda().to(dtype)
        v = torch.from_numpy(c["vs"][i]).cuda().to(dtype)
        pos = torch.arange(ctx, dtype=torch.int32, device="cuda")
        rows = torch.full((ctx,), i, dtype=torch.int32, device="cuda")
        pool.append(0, k, v, bt, pos, rows)
    torch.cuda.synchronize()
    return c, pool, bt


def test_paged_ragged_batch_decode_and_pool_bit_exact():
    c, pool, bt = _ragged_pool()
    plan = pool.plan(c["ctx"], c["H"])
    q = torch.from_numpy(c["q"]).cuda()
    out = torch.zeros_like(q)
    pool.decode(plan, 0, q, out, bt, c["scale"])
    res = out.cpu().numpy()
    assert_attention_close(res, G["ragged_out"], "paged ragged batch")
    for i, ctx in enumerate(c["ctx"]):
        k, v = pool.gather(0, bt, i, 0, ctx)
        np.testing.assert_array_equal(k.cpu().numpy(), c["ks"][i])
        np.testing.assert_array_equal(v.cpu().numpy(), c["vs"][i])
    # one batched call == one call per sequence (the reference's sequential batch).
    # The split length is chosen per batch, so a one-sequence plan may add its
    # splits in another grouping: equal to the fp16 tolerance, not bit for bit.
    for i, ctx in enumerate(c["ctx"]):
        p1 = pool.plan([ctx], c["H"], rows=[i])
        o1 = torch.zeros_like(q[i:i + 1])
        pool.decode(p1, 0, q[i:i + 1].contiguous(), o1, bt, c["scale"])
        ref = out[i].float().cpu().numpy()
        assert_attention_close(o1[0].cpu().numpy(), ref, f"one-sequence plan, query {i}")
        # the same one-sequence plan twice: bit for bit
        o2 = torch.zeros_like(o1)
        pool.decode(p1, 0, q[i:i + 1].contiguous(), o2, bt, c["scale"])
        assert torch.equal(o1, o2)


@pytest.mark.parametrize("page_size", [32, 64])
def test_page_size_does_not_change_results(page_size):
    c, pool16, bt16 = _ragged_pool(16)
    c, poolp, btp = _ragged_pool(page_size, seed=11)
    q = torch.from_numpy(c["q"]).cuda()
    o16, op = torch.zeros_like(q), torch.zeros_like(q)
    pool16.decode(pool16.plan(c["ctx"], c["H"]), 0, q, o16, bt16, c["scale"])
    poolp.decode(poolp.plan(c["ctx"], c["H"]), 0, q, op, btp, c["scale"])
    # splits are whole pages, so the partition may differ with the page size
    ref = o16.float().cpu().numpy()
    assert_attention_close(op.cpu().numpy(), ref, f"page size {page_size} vs page size 16")
    assert_attention_close(op.cpu().numpy(), G["ragged_out"], f"page size {page_size} vs golden")


def test_append_decode_fused_equals_separate_and_host_call():
    rng = np.random.default_rng(9)
    H, Hkv, D, ps = 32, 8, 128, 16
    ctx = [1000, 1, 2049, 17, 512]
    table, total = paged.random_block_tables(ctx, ps, 4)
    pool = paged.PagedKVCache(2, total, ps, Hkv, D)
    pool.fill_normal(seed=1)
    bt = torch.from_numpy(table).cuda()
    n = len(ctx)
    q = torch.from_numpy(rng.standard_normal((n, H, D), dtype=np.float32)).half().cuda()
    kn = torch.from_numpy(rng.standard_normal((n, Hkv, D), dtype=np.float32)).half().cuda()
    vn = torch.from_numpy(rng.standard_normal((n, Hkv, D), dtype=np.float32)).half().cuda()
    plan = pool.plan(ctx, H)
    o_fused = torch.zeros_like(q)
    pool.append_decode(plan, 1, q, kn, vn, o_fused, bt, 0.088)
    pos = torch.tensor([c - 1 for c in ctx], dtype=torch.int32, device="cuda")
    rows = torch.arange(n, dtype=torch.int32, device="cuda")
    pool.append(1, kn, vn, bt, pos, rows)
    o_sep = torch.zeros_like(q)
    pool.decode(plan, 1, q, o_sep, bt, 0.088)
    assert torch.equal(o_fused, o_sep)
    hq, hk, hv = q.cpu().pin_memory(), kn.cpu().pin_memory(), vn.cpu().pin_memory()
    ho = torch.zeros_like(hq).pin_memory()
    pool.decode_host(plan, 1, hq, hk, hv, ho, bt, 0.088)  # staged inputs, direct output
    assert torch.equal(ho, o_fused.cpu())
    ho2 = torch.zeros_like(ho, pin_memory=False)
    pool.decode_host(plan, 1, q.cpu(), kn.cpu(), vn.cpu(), ho2, bt, 0.088)  # pageable: copies
    assert torch.equal(ho2, o_fused.cpu())
    # against the oracle, from the gathered pool contents
    for i, c in enumerate(ctx):
        k, v = pool.gather(1, bt, i, 0, c)
        assert torch.equal(k[c - 1], kn[i]) and torch.equal(v[c - 1], vn[i])
        ref = gqa_ref.ref_gqa_attention(q[i:i + 1].cpu().numpy(), k.cpu().numpy(),
                                        v.cpu().numpy(), c - 1, 0.088)
        assert_attention_close(o_fused[i:i + 1].cpu().numpy(), ref, f"fused append + decode, query {i}")


def test_bf16_pool_against_fp32_reference():
    rng = np.random.default_rng(12)
    H, Hkv, D, ps = 16, 2, 128, 16
    ctx = [700, 33]
    table, total = paged.random_block_tables(ctx, ps, 2)
    pool = paged.PagedKVCache(1, total, ps, Hkv, D, dtype=torch.bfloat16)
    bt = torch.from_numpy(table).cuda()
    ks = [torch.from_numpy(rng.standard_normal((c, Hkv, D), dtype=np.float32)).bfloat16().cuda()
          for c in ctx]
    vs = [torch.from_numpy(rng.standard_normal((c, Hkv, D), dtype=np.float32)).bfloat16().cuda()
          for c in ctx]
    for i, c in enumerate(ctx):
        pool.append(0, ks[i], vs[i], bt, torch.arange(c, dtype=torch.int32, device="cuda"),
                    torch.full((c,), i, dtype=torch.int32, device="cuda"))
    q = torch.from_numpy(rng.standard_normal((2, H, D), dtype=np.float32)).bfloat16().cuda()
    out = torch.zeros_like(q)
    pool.decode(pool.plan(ctx, H), 0, q, out, bt, 0.09)
    for i, c in enumerate(ctx):
        ref = gqa_ref.ref_gqa_attention(q[i:i + 1].float().cpu().numpy(),
                                        ks[i].float().cpu().numpy(), vs[i].float().cpu().numpy(),
                                        c - 1, 0.09, out_dtype=np.float32)
        assert _maxerr(out[i:i + 1].float().cpu().numpy(), ref) < 2e-2


def test_head_dim_80_uses_cuda_core_path():
    rng = np.random.default_rng(13)
    H, Hkv, D, P = 8, 2, 80, 333
    Q = (rng.standard_normal((1, H, D), dtype=np.float32) * 0.5).astype(np.float16)
    K = (rng.standard_normal((P, Hkv, D), dtype=np.float32) * 0.5).astype(np.float16)
    V = (rng.standard_normal((P, Hkv, D), dtype=np.float32) * 0.5).astype(np.float16)
    out = np.zeros_like(Q)
    matmul_module.gqa_attention(Q, K, V, out, 1, P, H, Hkv, D, P - 1, 0.11)
    ref = gqa_ref.ref_gqa_attention(Q, K, V, P - 1, 0.11)
    assert_attention_close(out, ref, "head_dim 80 (CUDA-core path)")


def test_bad_block_table_is_reported_and_context_survives():
    H, Hkv, D, ps = 8, 2, 64, 16
    pool = paged.PagedKVCache(1, 8, ps, Hkv, D)
    pool.fill_normal(seed=2)
    bt = torch.tensor([[0, 1, 99, 3]], dtype=torch.int32, device="cuda")  # 99 >= num_pages
    q = torch.ones((1, H, D), dtype=torch.float16, device="cuda")
    out = torch.zeros_like(q)
    pool.decode(pool.plan([60], H), 0, q, out, bt, 0.1)
    torch.cuda.synchronize()
    code, info = ffi.device_error(0, clear=True)
    assert code == 1 and info == 99  # KVC_DEVERR_BAD_PAGE
    bt[0, 2] = 2
    pool.decode(pool.plan([60], H), 0, q, out, bt, 0.1)
    torch.cuda.synchronize()
    assert ffi.device_error(0, clear=True) == (0, 0)
    assert torch.isfinite(out).all()
    # the host-buffer call learns of it from the copy of the error word its split
    # merge stores (no copy of its own), then the word is clear again
    plan = pool.plan([40, 60], H)
    bt2 = torch.tensor([[0, 1, 3, 4], [5, 6, 99, 7]], dtype=torch.int32, device="cuda")
    hq = torch.ones((2, H, D), dtype=torch.float16).pin_memory()
    hk = torch.zeros((2, Hkv, D), dtype=torch.float16).pin_memory()
    ho = torch.zeros_like(hq).pin_memory()
    with pytest.raises(ffi.KVCacheDeviceError, match="block table"):
        pool.decode_host(plan, 0, hq, hk, hk, ho, bt2, 0.1)
    assert ffi.device_error(0, clear=True) == (0, 0)
    bt2[1, 2] = 2
    pool.decode_host(plan, 0, hq, hk, hk, ho, bt2, 0.1)  # no stale error
    assert torch.isfinite(ho).all()


# ---- rotary position embedding (rope.hip:21-55; ref_rope, test_layer.py:44-73) --------
def _rope_bound(x, pos):
    """2e-3 (the reference's own rope test, test_layer.py:145-150) plus what an ulp
    of difference in one inv_freq entry (numpy's float32 power vs the libm powf
    table rope.hip:79-83 builds) makes of the angle at position pos."""
    return 2e-3 + 2.0 * float(np.max(np.abs(x.astype(np.float32)))) * pos * 2.0 ** -23


def test_rope_host_matches_reference_golden():
    """matmul_module.rope vs the reference's ref_rope outputs (positions up to
    131072), and vs the oracle on the same libm inv_freq table within the
    reference test's 2e-3 at every position."""
    import matmul_module

    for i, c in enumerate(cases.rope_cases()):
        x = c["x"]
        out = np.zeros_like(x)
        matmul_module.rope(x, out, x.shape[0], x.shape[1], x.shape[2], c["pos_offset"],
                           c["freq_base"], c["neox"])
        last = c["pos_offset"] + x.shape[0] - 1
        err = _maxerr(out, G[f"rope{i}_out"])
        assert err < _rope_bound(x, last), (i, err)
        same_table = gqa_ref.ref_rope(x, pos_offset=c["pos_offset"], neox_style=c["neox"],
                                      inv_freq=gqa_ref.libm_inv_freq(c["freq_base"], x.shape[2]))
        err = _maxerr(out, same_table)
        assert err < 2e-3, (i, err)
    with pytest.raises(ValueError):
        matmul_module.rope(np.zeros((1, 2, 7), np.float16), np.zeros((1, 2, 7), np.float16),
                           1, 2, 7)
    with pytest.raises(ValueError):
        matmul_module.rope(np.zeros((1, 2, 8), np.float32), np.zeros((1, 2, 8), np.float16),
                           1, 2, 8)


def test_rope_device_per_token_positions_and_dtypes():
    rng = np.random.default_rng(5)
    pos = np.array([0, 1, 4095, 32768, 131072, 7], dtype=np.int32)
    for neox in (False, True):
        x = rng.standard_normal((len(pos), 8, 128), dtype=np.float32).astype(np.float16)
        table = gqa_ref.libm_inv_freq(500000.0, 128)
        ref = gqa_ref.ref_rope(x, neox_style=neox, positions=pos, inv_freq=table)
        xt = torch.from_numpy(x).cuda()
        out = torch.empty_like(xt)
        paged.rope(xt, out, positions=torch.from_numpy(pos).cuda(), freq_base=500000.0, neox=neox)
        assert _maxerr(out.cpu().numpy(), ref) < 2e-3
        ref32 = gqa_ref.ref_rope(x.astype(np.float32), neox_style=neox, positions=pos,
                                 out_dtype=np.float32, inv_freq=table)
        x32 = xt.float()
        o32 = torch.empty_like(x32)
        paged.rope(x32, o32, positions=torch.from_numpy(pos).cuda(), freq_base=500000.0, neox=neox)
        assert _maxerr(o32.cpu().numpy(), ref32) < 1e-4


def test_append_decode_rope_equals_rope_then_append_decode():
    """The fused rotate + append + attend chain == kvc_rope of q and k at the plan
    positions followed by kvc_append_decode, bit for bit; the pool holds the
    rotated K row; and the output matches the oracle on the rotated inputs."""
    rng = np.random.default_rng(14)
    H, Hkv, D, ps = 32, 8, 128, 16
    ctx = [700, 1, 2049, 33]
    for neox in (False, True):
        table, total = paged.random_block_tables(ctx, ps, 6)
        pools = [paged.PagedKVCache(1, total, ps, Hkv, D) for _ in range(2)]
        for p in pools:
            p.fill_normal(seed=3)
        bt = torch.from_numpy(table).cuda()
        n = len(ctx)
        q = torch.from_numpy(rng.standard_normal((n, H, D), dtype=np.float32)).half().cuda()
        kn = torch.from_numpy(rng.standard_normal((n, Hkv, D), dtype=np.float32)).half().cuda()
        vn = torch.from_numpy(rng.standard_normal((n, Hkv, D), dtype=np.float32)).half().cuda()
        plans = [p.plan(ctx, H) for p in pools]
        o1 = torch.zeros_like(q)
        pools[0].append_decode_rope(plans[0], 0, q, kn, vn, o1, bt, 0.088, 500000.0, neox)
        pos = torch.tensor([c - 1 for c in ctx], dtype=torch.int32, device="cuda")
        qr, kr = torch.empty_like(q), torch.empty_like(kn)
        paged.rope(q, qr, positions=pos, freq_base=500000.0, neox=neox)
        paged.rope(kn, kr, positions=pos, freq_base=500000.0, neox=neox)
        o2 = torch.zeros_like(q)
        pools[1].append_decode(plans[1], 0, qr, kr, vn, o2, bt, 0.088)
        torch.cuda.synchronize()
        assert torch.equal(o1, o2)
        for i, c in enumerate(ctx):
            k, v = pools[0].gather(0, bt, i, 0, c)
            assert torch.equal(k[c - 1], kr[i]) and torch.equal(v[c - 1], vn[i])
            ref = gqa_ref.ref_gqa_attention(qr[i:i + 1].cpu().numpy(), k.cpu().numpy(),
                                            v.cpu().numpy(), c - 1, 0.088)
            assert_attention_close(o1[i:i + 1].cpu().numpy(), ref, f"rope + append + decode, query {i}")
        # rotated q/k against the oracle rotation
        ref_k = gqa_ref.ref_rope(kn.cpu().numpy(), neox_style=neox, positions=pos.cpu().numpy(),
                                 inv_freq=gqa_ref.libm_inv_freq(500000.0, D))
        assert _maxerr(kr.cpu().numpy(), ref_k) < 2e-3


def test_paged_decode_loop_with_growing_contexts():
    """A serving loop: four decode steps over two layers, every step appending one
    row per sequence at its next position and re-planning (contexts cross split
    boundaries); each output against the oracle on the rows appended so far."""
    rng = np.random.default_rng(23)
    H, Hkv, D, ps, L, steps = 16, 4, 128, 16, 2, 4
    start = np.array([510, 1, 1023, 47, 2047], dtype=np.int64)   # cached before the loop
    table, total = paged.random_block_tables(start + steps, ps, 8)
    pool = paged.PagedKVCache(L, total, ps, Hkv, D)
    bt = torch.from_numpy(table).cuda()
    n = len(start)
    ks = [[rng.standard_normal((int(start[i]) + steps, Hkv, D), dtype=np.float32).astype(np.float16)
           for i in range(n)] for _ in range(L)]
    vs = [[rng.standard_normal((int(start[i]) + steps, Hkv, D), dtype=np.float32).astype(np.float16)
           for i in range(n)] for _ in range(L)]
    for l in range(L):  # the cached prefix
        for i in range(n):
            c = int(start[i])
            pool.append(l, torch.from_numpy(ks[l][i][:c]).cuda(), torch.from_numpy(vs[l][i][:c]).cuda(),
                        bt, torch.arange(c, dtype=torch.int32, device="cuda"),
                        torch.full((c,), i, dtype=torch.int32, device="cuda"))
    plan = None
    for s in range(steps):
        ctx = start + s + 1
        plan = pool.plan(ctx, H, plan=plan)
        for l in range(L):
            q = rng.standard_normal((n, H, D), dtype=np.float32).astype(np.float16)
            kn = np.stack([ks[l][i][ctx[i] - 1] for i in range(n)])
            vn = np.stack([vs[l][i][ctx[i] - 1] for i in range(n)])
            out = torch.zeros((n, H, D), dtype=torch.float16, device="cuda")
            pool.append_decode(plan, l, torch.from_numpy(q).cuda(), torch.from_numpy(kn).cuda(),
                               torch.from_numpy(vn).cuda(), out, bt, 0.09)
            got = out.cpu().numpy()
            for i in range(n):
                c = int(ctx[i])
                ref = gqa_ref.ref_gqa_attention(q[i:i + 1], ks[l][i][:c], vs[l][i][:c], c - 1, 0.09)
                assert_attention_close(got[i:i + 1], ref, f"step {s} layer {l} query {i}")
    assert ffi.device_error(0) == (0, 0)
