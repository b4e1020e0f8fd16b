"""Layer pipeline on the B200 (forward_layer_cached, attention.hip:603-695) against
the pinned oracle (oracle/layer_ref.py, pinned to the reference's own numpy code by
tests/golden/layer_golden.npz).

Tolerances:
  projections   max-abs <= 2e-3 * max(1, max|ref|): the oracle multiplies fp16-rounded
                dequantized weights (the reference's numpy check, test_layer.py:233-235),
                the kernels the exact fp32 block scale times the quantized integers (the
                reference's HIP kernels, dequantize.hip:120-137)
  whole layer   max-abs <= 5e-3 (the reference's own layer check, test_layer.py:307) on
                its case; 5e-3 * max(1, max|ref|) on larger layers, whose outputs reach
                magnitudes where the fp16 spacing is 4e-3 and one rounding flip of the
                weights' fp16 form moves an output by a spacing or two
  host vs device entry point, repeated calls: bit-exact
"""

from __future__ import annotations

import math

import numpy as np
import pytest

import layer_ref as L
from conftest import HAS_GPU
from make_layer_golden import LAYER, OUT as LAYER_GOLDEN

pytestmark = pytest.mark.gpu

if HAS_GPU:
    import torch

    import kvcache_ffi as ffi
    import matmul_module

TYPES = [L.F16, L.Q4_0, L.Q8_0, L.Q4_K, L.Q6_K]


@pytest.fixture(autouse=True)
def _clean(cuda_device):
    yield
    matmul_module.kv_cache_free()
    code, info = ffi.device_error(0, clear=True)
    assert code == 0, f"device error word left set: {code} {info}"


def _maxerr(a, b):
    return float(np.max(np.abs(a.astype(np.float32) - b.astype(np.float32))))


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _linear_dev(x, raw, w_type, n, epi="store", raw2=None, res=None):
    m, k = x.shape
    dx, dw = _dev(x), _dev(raw)
    out = torch.zeros((m, n), dtype=torch.float16, device="cuda")
    st = ffi.torch_stream_ptr()
    if epi == "store":
        ffi.check(ffi.lib.kvc_linear(dx.data_ptr(), m, k, dw.data_ptr(), w_type, n, out.data_ptr(), st))
    elif epi == "swiglu":
        dw2 = _dev(raw2)
        ffi.check(ffi.lib.kvc_linear_swiglu(dx.data_ptr(), m, k, dw.data_ptr(), dw2.data_ptr(),
                                            w_type, n, out.data_ptr(), st))
    else:
        dr = _dev(res)
        ffi.check(ffi.lib.kvc_linear_residual(dx.data_ptr(), m, k, dw.data_ptr(), w_type, n,
                                              dr.data_ptr(), out.data_ptr(), st))
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("w_type", TYPES)
@pytest.mark.parametrize("m", [1, 5, 8, 13, 40])
def test_linear_matches_oracle(w_type, m):
    """Every weight type, single-token to prefill-sized m (partial token tiles)."""
    rng = np.random.default_rng(100 + w_type * 7 + m)
    n, k = 80, 768   # 5 row tiles; 3 super-blocks per row for the K types
    x = (rng.standard_normal((m, k), dtype=np.float32) * 0.5).astype(np.float16)
    raw = L.random_weight(rng, w_type, n, k)
    got = _linear_dev(x, raw, w_type, n)
    ref = L.linear(x, raw, w_type, n)
    tol = 2e-3 * max(1.0, float(np.abs(ref.astype(np.float32)).max()))
    assert _maxerr(got, ref) <= tol, (w_type, m, _maxerr(got, ref))


@pytest.mark.parametrize("w_type", TYPES)
@pytest.mark.parametrize("m", [1, 13, 40])
def test_linear_staged_multi_stage(w_type, m):
    """k = 4096: whole stages for every type (the bulk-copy ring path), several of
    them per CTA, partial token tiles."""
    rng = np.random.default_rng(300 + w_type * 3 + m)
    n, k = 48, 4096
    x = (rng.standard_normal((m, k), dtype=np.float32) * 0.5).astype(np.float16)
    raw = L.random_weight(rng, w_type, n, k)
    got = _linear_dev(x, raw, w_type, n)
    ref = L.linear(x, raw, w_type, n)
    tol = 2e-3 * max(1.0, float(np.abs(ref.astype(np.float32)).max()))
    assert _maxerr(got, ref) <= tol, (w_type, m, _maxerr(got, ref))


@pytest.mark.parametrize("w_type", [L.Q4_0, L.Q4_K, L.Q6_K])
def test_linear_large_grid(w_type):
    """Llama-3-8B row counts (the grid's row-tiles-per-CTA choices) at m = 1 and 3."""
    rng = np.random.default_rng(5 + w_type)
    for n, k in [(6144, 512), (14336, 256), (1024, 4096)]:
        raw = L.random_weight(rng, w_type, n, k)
        for m in (1, 3):
            x = (rng.standard_normal((m, k), dtype=np.float32) * 0.5).astype(np.float16)
            got = _linear_dev(x, raw, w_type, n)
            ref = L.linear(x, raw, w_type, n)
            tol = 2e-3 * max(1.0, float(np.abs(ref.astype(np.float32)).max()))
            assert _maxerr(got, ref) <= tol, (w_type, n, k, m)


@pytest.mark.parametrize("w_type", [L.F16, L.Q4_0, L.Q4_K, L.Q6_K])
@pytest.mark.parametrize("m", [1, 9])
def test_linear_epilogues(w_type, m):
    """SwiGLU of gate/up (both rounded to fp16 first) and the residual add."""
    rng = np.random.default_rng(200 + w_type + m)
    n, k = 96, 512
    x = (rng.standard_normal((m, k), dtype=np.float32) * 0.5).astype(np.float16)
    wg, wu = L.random_weight(rng, w_type, n, k), L.random_weight(rng, w_type, n, k)
    got = _linear_dev(x, wg, w_type, n, "swiglu", raw2=wu)
    ref = L.swiglu(L.linear(x, wg, w_type, n), L.linear(x, wu, w_type, n))
    assert _maxerr(got, ref) <= 2e-3 * max(1.0, float(np.abs(ref.astype(np.float32)).max()))
    res = (rng.standard_normal((m, n), dtype=np.float32)).astype(np.float16)
    got = _linear_dev(x, wg, w_type, n, "residual", res=res)
    ref = L.residual_add(res, L.linear(x, wg, w_type, n))
    assert _maxerr(got, ref) <= 2e-3 * max(1.0, float(np.abs(ref.astype(np.float32)).max()))


@pytest.mark.parametrize("w_type", [L.F16, L.Q4_0, L.Q8_0, L.Q4_K])
@pytest.mark.parametrize("m", [9, 20, 32])
def test_linear_batch_tokens_long_k(w_type, m):
    """9-32 tokens (the 32-token tiles a batched decode step uses) at the down
    projection's k = 14336, n = 208 (13 row tiles); store and residual epilogues."""
    rng = np.random.default_rng(400 + w_type + m)
    n, k = 208, 14336
    x = (rng.standard_normal((m, k), dtype=np.float32) * 0.5).astype(np.float16)
    raw = L.random_weight(rng, w_type, n, k)
    ref = L.linear(x, raw, w_type, n)
    got = _linear_dev(x, raw, w_type, n)
    tol = 2e-3 * max(1.0, float(np.abs(ref.astype(np.float32)).max()))
    assert _maxerr(got, ref) <= tol, (w_type, m, _maxerr(got, ref))
    res = (rng.standard_normal((m, n), dtype=np.float32)).astype(np.float16)
    got = _linear_dev(x, raw, w_type, n, "residual", res=res)
    ref = L.residual_add(res, ref)
    assert _maxerr(got, ref) <= 2e-3 * max(1.0, float(np.abs(ref.astype(np.float32)).max()))


def test_linear_rejects_bad_shapes():
    x = torch.zeros((1, 256), dtype=torch.float16, device="cuda")
    w = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    out = torch.zeros((1, 32), dtype=torch.float16, device="cuda")
    for args in [(x.data_ptr(), 1, 256, w.data_ptr(), 3, 32),      # unknown type
                 (x.data_ptr(), 1, 96, w.data_ptr(), L.Q4_K, 32),   # k not a super-block multiple
                 (x.data_ptr(), 1, 256, w.data_ptr(), L.Q4_0, 24),  # n not a multiple of 16
                 (x.data_ptr() + 2, 1, 256, w.data_ptr(), L.Q4_0, 32)]:  # misaligned x
        with pytest.raises(ValueError):
            ffi.check(ffi.lib.kvc_linear(*args, out.data_ptr(), None))


def test_rmsnorm_and_residual():
    rng = np.random.default_rng(10)
    for m, k in [(1, 4096), (16, 2048), (7, 1024)]:  # test_layer.py:118
        x = rng.standard_normal((m, k), dtype=np.float32).astype(np.float16)
        r = rng.standard_normal((m, k), dtype=np.float32).astype(np.float16)
        w = (1.0 + 0.1 * rng.standard_normal((k,), dtype=np.float32)).astype(np.float16)
        dx, dr, dw = _dev(x), _dev(r), _dev(w)
        out = torch.zeros_like(dx)
        h = torch.zeros_like(dx)
        ffi.check(ffi.lib.kvc_rmsnorm(dx.data_ptr(), None, None, dw.data_ptr(), out.data_ptr(),
                                      m, k, 1e-5, ffi.torch_stream_ptr()))
        torch.cuda.synchronize()
        assert _maxerr(out.cpu().numpy(), L.rmsnorm(x, w, 1e-5)) < 2e-3
        ffi.check(ffi.lib.kvc_rmsnorm(dx.data_ptr(), dr.data_ptr(), h.data_ptr(), dw.data_ptr(),
                                      out.data_ptr(), m, k, 1e-5, ffi.torch_stream_ptr()))
        torch.cuda.synchronize()
        hh = L.residual_add(x, r)
        assert np.array_equal(h.cpu().numpy(), hh)
        assert _maxerr(out.cpu().numpy(), L.rmsnorm(hh, w, 1e-5)) < 2e-3


def test_forward_layer_cached_matches_reference_golden():
    """The reference's layer check (test_layer.py:206-320): prefill of 4 tokens, then a
    decode step at position 4, mixed weight types; outputs and pool rows."""
    g = np.load(LAYER_GOLDEN)
    c = LAYER
    H, Hkv, D, hid, inter = c["H"], c["Hkv"], c["D"], c["hidden"], c["inter"]
    names = ("q", "k", "v", "o", "gate", "up", "down")
    ws = [g[f"layer_w_{n}"] for n in names]
    x = g["layer_x"]
    matmul_module.kv_cache_init(1, 16, Hkv, D)
    outs = []
    for lo, hi in ((0, 4), (4, 5)):
        out = np.zeros((hi - lo, hid), np.float16)
        matmul_module.forward_layer_cached(
            x[lo:hi], out, g["layer_attn_norm"], ws[0], c["types"]["q"], ws[1], c["types"]["k"],
            ws[2], c["types"]["v"], ws[3], c["types"]["o"], g["layer_ffn_norm"], ws[4],
            c["types"]["gate"], ws[5], c["types"]["up"], ws[6], c["types"]["down"], 0, hi - lo,
            lo, hid, inter, H, Hkv, D, c["eps"], c["base"], c["neox"], 1.0 / math.sqrt(D))
        outs.append(out)
    got = np.concatenate(outs)
    assert _maxerr(got, g["layer_out"]) <= 5e-3, _maxerr(got, g["layer_out"])
    k_pool, v_pool = matmul_module.kv_cache_gather(0, 0, 5)
    assert _maxerr(k_pool, g["layer_k_rot"]) <= 2e-3
    assert _maxerr(v_pool, g["layer_v"]) <= 2e-3


def _random_layer(rng, hid, inter, H, Hkv, D, types):
    qd, kd = H * D, Hkv * D
    shapes = {"q": (qd, hid), "k": (kd, hid), "v": (kd, hid), "o": (hid, qd),
              "gate": (inter, hid), "up": (inter, hid), "down": (hid, inter)}
    raws = {n: L.random_weight(rng, types[n], *shapes[n]) for n in shapes}
    an = (1.0 + 0.05 * rng.standard_normal(hid, dtype=np.float32)).astype(np.float16)
    fn = (1.0 + 0.05 * rng.standard_normal(hid, dtype=np.float32)).astype(np.float16)
    lw = L.LayerWeights(an, *[(raws[n], types[n]) for n in ("q", "k", "v", "o")], fn,
                        *[(raws[n], types[n]) for n in ("gate", "up", "down")])
    return lw, raws, an, fn


@pytest.mark.parametrize("neox", [False, True])
def test_forward_layer_device_matches_oracle_and_host(neox):
    """A Llama-shaped layer (GQA 4:1, Q4_K q/k/o/gate/up, Q6_K v/down as in Q4_K_M
    files) over two layers of the pool: prefill 37 tokens, then 3 decode steps; the
    device entry point equals the host one bit for bit."""
    rng = np.random.default_rng(77 + neox)
    hid, inter, H, Hkv, D = 512, 1024, 8, 2, 64
    types = {"q": L.Q4_K, "k": L.Q4_K, "v": L.Q6_K, "o": L.Q4_K, "gate": L.Q4_K, "up": L.Q4_K,
             "down": L.Q6_K}
    lw, raws, an, fn = _random_layer(rng, hid, inter, H, Hkv, D, types)
    n_layers, S = 2, 64
    kc = [np.zeros((S, Hkv, D), np.float16) for _ in range(n_layers)]
    vc = [np.zeros((S, Hkv, D), np.float16) for _ in range(n_layers)]
    kw = dict(num_heads=H, num_kv_heads=Hkv, head_dim=D, inter=inter, eps=1e-5,
              rope_base=500000.0, neox=neox, scale=1.0 / math.sqrt(D))
    steps = [(0, 37), (37, 38), (38, 39), (39, 40)]
    xs = (rng.standard_normal((40, hid), dtype=np.float32) * 0.5).astype(np.float16)
    names = ("q", "k", "v", "o", "gate", "up", "down")
    dw = {n: _dev(raws[n]) for n in names}
    dan, dfn = _dev(an), _dev(fn)
    matmul_module.kv_cache_init(n_layers, S, Hkv, D)
    st = ffi.torch_stream_ptr()
    for lo, hi in steps:
        x = xs[lo:hi]
        for layer in range(n_layers):
            ref = L.layer_forward(x, lw, kc[layer], vc[layer], lo, **kw)
            if layer == 0:  # host buffers
                got = np.zeros_like(x)
                matmul_module.forward_layer_cached(
                    x, got, an, raws["q"], types["q"], raws["k"], types["k"], raws["v"],
                    types["v"], raws["o"], types["o"], fn, raws["gate"], types["gate"],
                    raws["up"], types["up"], raws["down"], types["down"], layer, hi - lo, lo,
                    hid, inter, H, Hkv, D, 1e-5, 500000.0, neox, 1.0 / math.sqrt(D))
            else:  # device buffers
                dx = _dev(x)
                dout = torch.zeros_like(dx)
                ffi.check(ffi.lib.kvc_forward_layer_cached_device(
                    dx.data_ptr(), dout.data_ptr(), dan.data_ptr(), dw["q"].data_ptr(), types["q"],
                    dw["k"].data_ptr(), types["k"], dw["v"].data_ptr(), types["v"],
                    dw["o"].data_ptr(), types["o"], dfn.data_ptr(), dw["gate"].data_ptr(),
                    types["gate"], dw["up"].data_ptr(), types["up"], dw["down"].data_ptr(),
                    types["down"], layer, hi - lo, lo, hid, inter, H, Hkv, D, 1e-5, 500000.0,
                    int(neox), 1.0 / math.sqrt(D), st))
                torch.cuda.synchronize()
                got = dout.cpu().numpy()
                assert np.array_equal(got, host_out), "device and host entry points differ"
            tol = 5e-3 * max(1.0, float(np.abs(ref.astype(np.float32)).max()))
            assert _maxerr(got, ref) <= tol, (lo, layer, _maxerr(got, ref), tol)
            host_out = got
    for layer in range(n_layers):
        k_pool, v_pool = matmul_module.kv_cache_gather(layer, 0, 40)
        assert _maxerr(k_pool, kc[layer][:40]) <= 2e-3
        assert _maxerr(v_pool, vc[layer][:40]) <= 2e-3


def test_forward_layer_validation():
    """The reference's checks: pool state and positions (attention.hip:316-329),
    weight buffers (bindings.cpp:518-557)."""
    rng = np.random.default_rng(3)
    hid, inter, H, Hkv, D = 256, 512, 4, 2, 64
    types = {n: L.Q4_0 for n in ("q", "k", "v", "o", "gate", "up", "down")}
    lw, raws, an, fn = _random_layer(rng, hid, inter, H, Hkv, D, types)
    x = np.zeros((1, hid), np.float16)
    out = np.zeros_like(x)

    def call(layer=0, pos=0, wq=None, wq_type=L.Q4_0, hd=D):
        matmul_module.forward_layer_cached(
            x, out, an, raws["q"] if wq is None else wq, wq_type, raws["k"], L.Q4_0, raws["v"],
            L.Q4_0, raws["o"], L.Q4_0, fn, raws["gate"], L.Q4_0, raws["up"], L.Q4_0, raws["down"],
            L.Q4_0, layer, 1, pos, hid, inter, H, Hkv, hd, 1e-5, 10000.0, False, 0.125)

    with pytest.raises(RuntimeError, match="not initialized"):
        call()
    matmul_module.kv_cache_init(2, 8, Hkv, D)
    call()                      # fine
    with pytest.raises(IndexError):
        call(layer=2)
    with pytest.raises(IndexError):
        call(pos=8)
    with pytest.raises(ValueError, match="smaller than required"):
        call(wq=raws["q"][:-1])
    with pytest.raises(ValueError, match="unsupported"):
        call(wq_type=5)
    with pytest.raises(ValueError):
        call(hd=32)             # head_dim mismatch with the pool
