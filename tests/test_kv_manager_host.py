"""KVCacheManager host-side behaviour (CPU only), after the reference's CPU
suite (tests/test_cpu_only.py:388-483) and the guard checks of
tests/test_phase5_scale.py:219-237.  The gpu mode runs against a stub
``matmul_module`` exactly like the reference's CPU test does."""

from __future__ import annotations

import os
import tempfile
import types
import warnings

import numpy as np
import pytest

import kv_cache
from kv_cache import KVCacheManager


@pytest.fixture
def stub_module(monkeypatch):
    calls = []
    stub = types.SimpleNamespace(
        kv_cache_init=lambda *a: calls.append(("init", a)),
        kv_cache_init_ex=lambda *a, **k: calls.append(("init_ex", a)),
        kv_cache_free=lambda *a: calls.append(("free", a)),
        gqa_attention_cached=lambda *a: calls.append(("attend", a)),
    )
    monkeypatch.setattr(kv_cache, "matmul_module", stub)
    yield stub, calls
    KVCacheManager._active_gpu_instance = False


def test_mmap_files_unique_private_and_removed():
    """S-3: O_CREAT|O_EXCL files, bystander untouched, files gone after close."""
    with tempfile.TemporaryDirectory() as tmpdir:
        bystander = os.path.join(tmpdir, "kv_cache_k.mmap")
        with open(bystander, "wb") as f:
            f.write(b"important_user_data")
        with KVCacheManager(num_layers=2, max_seq_len=16, num_kv_heads=2, head_dim=8,
                            mmap_dir=tmpdir) as kv:
            assert kv.mode == "mmap" and kv.device_bytes == 0
            assert len(kv.mmap_files) == 2
            for p in kv.mmap_files:
                assert os.path.exists(p)
                assert os.path.abspath(p) != os.path.abspath(bystander)
                assert (os.stat(p).st_mode & 0o777) == 0o600
                assert os.path.getsize(p) == kv.nbytes // 2
            created = kv.mmap_files
        assert all(not os.path.exists(p) for p in created)
        with open(bystander, "rb") as f:
            assert f.read() == b"important_user_data"


def test_del_warns_instead_of_raising():
    """D-4: __del__ emits RuntimeWarning when close() fails."""
    kv = KVCacheManager(num_layers=1, max_seq_len=8, num_kv_heads=1, head_dim=8,
                        offload_to_cpu=True)

    def failing_close():
        raise RuntimeError("simulated driver cleanup error")

    kv.close = failing_close
    with warnings.catch_warnings(record=True) as caught:
        warnings.simplefilter("always", RuntimeWarning)
        kv.__del__()
        # the garbage collector's own finalization of `kv` warns the same way
        del kv
        import gc

        gc.collect()
    assert any(issubclass(w.category, RuntimeWarning) for w in caught)


def test_properties_and_cpu_mode_needs_no_gpu():
    kv = KVCacheManager(3, 20, 2, 16, offload_to_cpu=True)
    assert kv.mode == "cpu" and kv.nbytes == 2 * 3 * 20 * 2 * 16 * 2 and kv.device_bytes == 0
    assert kv._k_host.shape == (3, 20, 2, 16) and kv._k_host.dtype == np.float16
    assert kv._k_host.ctypes.data % 4096 == 0
    kv32 = KVCacheManager(3, 20, 2, 16, offload_to_cpu=True, dtype=np.float32)
    assert kv32.nbytes == 2 * kv.nbytes
    kv.close()
    kv32.close()
    with pytest.raises(RuntimeError, match="not allocated"):
        kv.attend(None, None, None, None, 0, 1, 0, 4, 0.1)


def test_dimension_and_size_checks():
    with pytest.raises(ValueError, match="positive"):
        KVCacheManager(0, 16, 2, 8, offload_to_cpu=True)
    with pytest.raises(ValueError, match="max_kv_bytes"):
        KVCacheManager(2, 1024, 8, 128, offload_to_cpu=True, max_kv_bytes=1024)


def test_gpu_singleton_guard_and_rollback(stub_module):
    stub, calls = stub_module
    kv = KVCacheManager(2, 32, 2, 16)
    assert kv.mode == "gpu" and kv.device_bytes == kv.nbytes
    assert calls[0] == ("init", (2, 32, 2, 16))
    with pytest.raises(RuntimeError, match="already active"):
        KVCacheManager(2, 32, 2, 16)
    kv.close()
    assert ("free", ()) in calls and not KVCacheManager._active_gpu_instance

    # failed init rolls back the guard and frees (kv_cache.py:153-161)
    def bad_init(*a):
        raise ValueError("KV cache dimensions must all be positive.")

    stub.kv_cache_init = bad_init
    with pytest.raises(ValueError):
        KVCacheManager(2, 32, 2, 16)
    assert not KVCacheManager._active_gpu_instance
    # a zero dimension is rejected in Python before the native call
    with pytest.raises(ValueError):
        KVCacheManager(num_layers=0, max_seq_len=64, num_kv_heads=4, head_dim=32)
    assert not KVCacheManager._active_gpu_instance


def test_record_step_and_seq_len_semantics(stub_module):
    stub, calls = stub_module
    with KVCacheManager(3, 16, 2, 8) as kv:
        kv.record_gpu_layer_step(0, 4, 0)
        assert kv.current_seq_len == 0          # only the last layer moves it
        kv.record_gpu_layer_step(2, 4, 0)
        assert kv.current_seq_len == 4
        with pytest.raises(ValueError, match="exceeds max_seq_len"):
            kv.record_gpu_layer_step(2, 1, 16)
        q = np.zeros((1, 4, 8), np.float16)
        kv.attend(q, q[:, :2], q[:, :2], q.copy(), layer_idx=1, q_len=1, start_pos=4,
                  num_heads=4, scale=0.3)
        assert kv.current_seq_len == 4
        kv.attend(q, q[:, :2], q[:, :2], q.copy(), layer_idx=2, q_len=1, start_pos=4,
                  num_heads=4, scale=0.3)
        assert kv.current_seq_len == 5
        args = [c for c in calls if c[0] == "attend"][0][1]
        assert args[4:] == (1, 1, 4, 4, 2, 8, 0.3, True)  # kv_cache.py:243-256 order
        with pytest.raises(ValueError, match="exceeds max_seq_len"):
            kv.attend(q, q, q, q, layer_idx=0, q_len=2, start_pos=15, num_heads=4, scale=0.3)
        kv.reset()
        assert kv.current_seq_len == 0
    with pytest.raises(RuntimeError, match="not allocated"):
        kv.record_gpu_layer_step(0, 1, 0)
