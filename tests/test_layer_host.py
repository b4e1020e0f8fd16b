"""forward_layer_cached argument checks that run before any native call
(check_fp16_contiguous / check_weight_buffer, bindings.cpp:20-38 and :518-557),
and the C ABI's weight size rule.  CPU only."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import kvcache_ffi as ffi
import layer_ref as L
import matmul_module


def _args(**over):
    hid, inter, H, Hkv, D = 256, 512, 4, 2, 64
    w = lambda t, n, k: np.zeros(L.weight_bytes(t, n, k), np.uint8)  # noqa: E731
    a = dict(x_in=np.zeros((1, hid), np.float16), x_out=np.zeros((1, hid), np.float16),
             attn_norm_w=np.ones(hid, np.float16), wq=w(2, H * D, hid), wq_type=2,
             wk=w(2, Hkv * D, hid), wk_type=2, wv=w(2, Hkv * D, hid), wv_type=2,
             wo=w(2, hid, H * D), wo_type=2, ffn_norm_w=np.ones(hid, np.float16),
             wgate=w(12, inter, hid), wgate_type=12, wup=w(12, inter, hid), wup_type=12,
             wdown=w(14, hid, inter), wdown_type=14, layer_idx=0, seq_len=1, pos_offset=0,
             hidden_size=hid, intermediate_size=inter, num_heads=H, num_kv_heads=Hkv,
             head_dim=D, rms_norm_eps=1e-5, rope_freq_base=10000.0, rope_neox=False,
             scale=0.125)
    a.update(over)
    return a


@pytest.mark.parametrize("over,msg", [
    (dict(x_in=np.zeros((1, 256), np.float32)), "x_in"),
    (dict(x_out=np.zeros((1, 128), np.float16)), "smaller"),
    (dict(attn_norm_w=np.ones(255, np.float16)), "smaller"),
    (dict(wq=np.zeros(10, np.uint8)), "wq weight buffer is smaller"),
    (dict(wk_type=3), "wk has unsupported ggml_type"),
    (dict(wgate=np.zeros((2, 4 * 512 * 144), np.uint8)[:, ::2]), "C-contiguous"),
    (dict(hidden_size=96, x_in=np.zeros((1, 96), np.float16), x_out=np.zeros((1, 96), np.float16),
          attn_norm_w=np.ones(96, np.float16), ffn_norm_w=np.ones(96, np.float16)),
     "K must be divisible by 256 for Q4_K"),
])
def test_shim_checks_before_native_call(over, msg):
    with pytest.raises(ValueError, match=msg):
        matmul_module.forward_layer_cached(**_args(**over))


def test_weight_bytes_abi():
    out = ctypes.c_size_t(0)
    ffi.check(ffi.lib.kvc_weight_bytes(ffi.WTYPE_Q4_K, 14336, 4096, ctypes.byref(out)))
    assert out.value == L.weight_bytes(L.Q4_K, 14336, 4096)
    ffi.check(ffi.lib.kvc_weight_bytes(ffi.WTYPE_F16, 8, 40, ctypes.byref(out)))
    assert out.value == 8 * 40 * 2
    with pytest.raises(ValueError):
        ffi.check(ffi.lib.kvc_weight_bytes(ffi.WTYPE_Q8_0, 8, 40, ctypes.byref(out)))
    with pytest.raises(ValueError):
        ffi.check(ffi.lib.kvc_weight_bytes(7, 8, 64, ctypes.byref(out)))
