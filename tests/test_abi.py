"""The C ABI: libkvcache.so loads and exports every symbol include/kvcache.h
declares; argument errors that need no GPU map to the reference's exception
classes (CPU only, no compute calls)."""

from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

import kvcache_ffi as ffi
from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "kvcache.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^KVC_API\s+(?:const\s+)?\w+\s*\*?\s*(kvc_\w+)\s*\(", text,
                                 flags=re.M)))


def test_header_declares_the_reference_entry_points():
    names = declared_symbols()
    for required in ("kvc_cache_init", "kvc_cache_free", "kvc_gqa_attention_cached",
                     "kvc_gqa_attention_cached_device", "kvc_gqa_attention",
                     "kvc_offload_attend", "kvc_decode", "kvc_append", "kvc_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", ffi.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in declared_symbols() if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    extra = sorted(n for n in exported if n.startswith("kvc_") and n not in declared_symbols())
    assert not extra, f"exported but not declared: {extra}"


def test_ffi_binds_every_declared_symbol():
    assert sorted(ffi.SIGNATURES) == declared_symbols()
    for name in declared_symbols():
        assert getattr(ffi.lib, name) is not None


def test_version_and_no_error_initially():
    assert ffi.lib.kvc_version() == 1


def test_invalid_arguments_map_to_reference_exceptions():
    # init_device_kv_cache_fp16 rejects non-positive dims with invalid_argument
    # (attention.hip:292-294) -> ValueError
    with pytest.raises(ValueError, match="positive"):
        ffi.check(ffi.lib.kvc_cache_init(0, 16, 2, 32))
    h = ctypes.c_void_p()
    with pytest.raises(ValueError, match="page_size"):
        ffi.check(ffi.lib.kvc_pool_create(1, 4, 10, 2, 64, ffi.DTYPE_F16, 0, ctypes.byref(h)))
    with pytest.raises(ValueError, match="head_dim"):
        ffi.check(ffi.lib.kvc_pool_create(1, 4, 16, 2, 300, ffi.DTYPE_F16, 0, ctypes.byref(h)))
    # gqa_attention checks (attention.hip:242-247) run before any device work
    with pytest.raises(ValueError, match="head_dim"):
        ffi.check(ffi.lib.kvc_gqa_attention(None, None, None, None, 1, 1, 4, 2, 512, 0, 0.0, 1))
    with pytest.raises(ValueError, match="divisible"):
        ffi.check(ffi.lib.kvc_gqa_attention(None, None, None, None, 1, 1, 5, 2, 64, 0, 0.0, 1))
    # the cached path without a pool: runtime_error (attention.hip:317-319)
    ffi.lib.kvc_cache_free()
    with pytest.raises(RuntimeError, match="not initialized"):
        ffi.check(ffi.lib.kvc_gqa_attention_cached(None, None, None, None, 0, 1, 0, 4, 2, 32,
                                                   0.0, 1))
    assert "not initialized" in ffi.last_error()


def test_status_code_mapping():
    with pytest.raises(IndexError):
        ffi.check(ffi.KVC_ERR_OUT_OF_RANGE)
    with pytest.raises(ffi.KVCacheDeviceError):
        ffi.check(ffi.KVC_ERR_DEVICE)
    with pytest.raises(TimeoutError):
        ffi.check(ffi.KVC_ERR_TIMEOUT)
    with pytest.raises(RuntimeError):
        ffi.check(ffi.KVC_ERR_CUDA)
    ffi.check(ffi.KVC_OK)


def test_split_length_model_on_the_baseline_shapes():
    """The plan's split length (host-only model, kvc_plan_split_tokens) for the
    benchmark shapes on a 148-SM B200: 512 for the ragged batch and the unsharded
    70B shape, one wave of equal units for long even contexts and their KV-head
    shards, and the 4K single sequence."""
    import ctypes

    import numpy as np

    import bench
    import kvcache_ffi as ffi

    def split(ctx, H, Hkv, ps=16, sms=148):
        c = np.ascontiguousarray(np.asarray(ctx, dtype=np.int32))
        out = ctypes.c_int(0)
        ffi.check(ffi.lib.kvc_plan_split_tokens(ffi.np_ptr(c), len(c), H, Hkv, ps, sms,
                                                ctypes.byref(out)))
        return out.value

    c3 = bench.cached_lengths(bench.CONFIGS["3"]) + 1
    assert split(c3, 32, 8) == 512
    assert split([32769] * 8, 64, 8) == 512
    assert split([32769] * 8, 32, 4) == 896     # 2-way KV-head shard: 1,184 units
    assert split([32769] * 8, 16, 2) == 448     # 4-way
    assert split([32769] * 8, 8, 1) == 224      # 8-way: 1,176 units
    assert split([4096], 32, 32) == 128         # config 2: 1,024 units (8 slabs each at least)
    assert split([4096], 32, 32, ps=32) % 32 == 0
    for bad in ((c3, 30, 8), (c3, 32, 0)):
        out = ctypes.c_int(0)
        c = np.ascontiguousarray(np.asarray(bad[0], dtype=np.int32))
        rc = ffi.lib.kvc_plan_split_tokens(ffi.np_ptr(c), len(c), bad[1], bad[2], 16, 148,
                                           ctypes.byref(out))
        assert rc == ffi.KVC_ERR_INVALID_ARG


def test_split_partition_counts_on_the_baseline_shapes():
    """The whole partition (kvc_plan_split_counts, host only) on a 148-SM B200: the
    split slots a plan of each benchmark shape holds (the figures the bench reports
    as "splits"), ragged batches left unrefined, and the tail refinement cutting
    full splits into quarters only for even multi-wave batches."""
    import ctypes

    import numpy as np

    import bench
    import kvcache_ffi as ffi

    def counts(ctx, H, Hkv, ps=16, sms=148):
        c = np.ascontiguousarray(np.asarray(ctx, dtype=np.int32))
        per = np.zeros(len(c), dtype=np.int32)
        C, tot = ctypes.c_int(0), ctypes.c_int(0)
        ffi.check(ffi.lib.kvc_plan_split_counts(ffi.np_ptr(c), len(c), H, Hkv, ps, sms,
                                                ctypes.byref(C), ffi.np_ptr(per),
                                                ctypes.byref(tot)))
        assert int(per.sum()) == tot.value
        return C.value, per, tot.value

    c3 = bench.cached_lengths(bench.CONFIGS["3"]) + 1
    C, per, tot = counts(c3, 32, 8)
    assert (C, tot) == (512, 286)
    assert np.array_equal(per, -(-c3 // 512))          # ragged: no quartered splits
    C, per, tot = counts([32769] * 8, 64, 8)           # config 4: 4,096 full units, 1,184 warps
    assert C == 512 and tot == 724
    extra = per - -(-32769 // 512)
    assert np.all(extra % 3 == 0) and int(extra.sum()) == 3 * 68   # 68 full splits quartered
    C, per, tot = counts([32769] * 8, 8, 1)             # its 8-way KV-head shard: one wave
    assert C == 224 and tot == 1176 and np.all(per == 147)
    c3s = counts(c3, 4, 1)                              # config 3, 8-way KV-head shard
    assert (c3s[0], c3s[2]) == (128, 1093)
    assert counts([4096], 32, 32)[::2] == (128, 32)     # config 2
    assert counts([0, 5], 8, 8)[1].tolist() == [1, 1]   # an empty context has one split
    C, tot = ctypes.c_int(0), ctypes.c_int(0)
    bad = np.ascontiguousarray(np.asarray([-1], dtype=np.int32))
    assert ffi.lib.kvc_plan_split_counts(ffi.np_ptr(bad), 1, 8, 8, 16, 148, ctypes.byref(C), None,
                                         ctypes.byref(tot)) == ffi.KVC_ERR_INVALID_ARG
