"""KVCacheManager — drop-in replacement of gfx1150-inference's src/kv_cache.py
for B200.

Public API, arguments, defaults, error classes and state semantics are those of
the reference class (src/kv_cache.py:46-313):

* three storage modes, chosen as in the reference (kv_cache.py:69, :169-173):
  ``gpu``  — the process-wide device pool behind ``matmul_module.kv_cache_init``
             (one active GPU-resident manager per process, kv_cache.py:137-161);
  ``cpu``  — host arrays (num_layers, max_seq_len, num_kv_heads, head_dim);
  ``mmap`` — the same arrays backed by two private files created with
             O_CREAT | O_EXCL | O_NOFOLLOW, mode 0600, removed on close
             (kv_cache.py:100-132);
* ``attend`` appends the new rows at (layer_idx, start_pos) and attends over
  [0, start_pos + q_len); ``current_seq_len`` moves only on the last layer
  (kv_cache.py:195-259); ``record_gpu_layer_step`` does the bounds check of the
  fused layer path (kv_cache.py:180-193);
* ``nbytes``, ``mode``, ``device_bytes``, ``mmap_files``, ``reset``, ``close``,
  ``__del__`` (warns instead of raising) and the context-manager protocol.

What changes underneath: in the cpu and mmap modes the host arrays are
page-locked (cudaHostRegister) the first time they are attended, and
``attend`` goes through the library's offload engine (kvc_offload_attend):
the host append is done in C, the layer's rows are streamed to the GPU on a
copy stream while the previous layer attends, and the next layer is
prefetched.  Outputs are bit-identical to the gpu mode's.  Nothing touches the
GPU before the first ``attend`` in those modes, as in the reference.

Extensions (keyword-only): ``dtype`` selects float16 (the reference's only
type) or float32 storage; ``offload_mirror_bytes`` lets the cpu/mmap modes keep
an HBM copy of as many layers as that many bytes of device memory hold (the
host arrays stay the source of truth; a mirrored layer uploads only its new
rows per attend; outputs unchanged).
"""

from __future__ import annotations

import ctypes
import mmap
import os
import sys
import threading
import warnings
from typing import List, Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
if _HERE not in sys.path:
    sys.path.append(_HERE)

try:
    import matmul_module
except ImportError as exc:  # same message shape as kv_cache.py:35-40
    raise ImportError(
        "Failed to import 'matmul_module' (libkvcache.so). Build it first with:\n"
        f"  python {os.path.join(_HERE, 'build_lib.py')}"
    ) from exc


DEFAULT_MAX_KV_BYTES = 32 * (1 << 30)  # kv_cache.py:43
_PAGE = mmap.PAGESIZE


def _aligned_empty(shape, dtype) -> np.ndarray:
    """np.empty whose data starts on a page boundary (cudaHostRegister-friendly)."""
    dtype = np.dtype(dtype)
    nbytes = int(np.prod(shape)) * dtype.itemsize
    raw = np.empty(nbytes + _PAGE, dtype=np.uint8)
    off = (-raw.ctypes.data) % _PAGE
    return raw[off:off + nbytes].view(dtype).reshape(shape)


class KVCacheManager:
    """
    Manages the GQA KV cache across all transformer layers with GPU-resident,
    CPU-offloaded, or NVMe `mmap`-backed storage.
    """

    _active_gpu_instance: bool = False
    _gpu_lock: threading.Lock = threading.Lock()

    def __init__(
        self,
        num_layers: int,
        max_seq_len: int,
        num_kv_heads: int,
        head_dim: int,
        offload_to_cpu: bool = False,
        mmap_dir: Optional[str] = None,
        max_kv_bytes: int = DEFAULT_MAX_KV_BYTES,
        *,
        dtype=np.float16,
        offload_mirror_bytes: int = 0,
    ):
        self.num_layers = int(num_layers)
        self.max_seq_len = int(max_seq_len)
        self.num_kv_heads = int(num_kv_heads)
        self.head_dim = int(head_dim)
        self.dtype = np.dtype(dtype)
        self.offload_to_cpu = bool(offload_to_cpu or mmap_dir is not None)
        self.mmap_dir = mmap_dir
        self.current_seq_len = 0
        self._allocated = False
        self._k_host: Optional[np.ndarray] = None
        self._v_host: Optional[np.ndarray] = None
        self._k_mm: Optional[mmap.mmap] = None
        self._v_mm: Optional[mmap.mmap] = None
        self._created_mmap_files: List[str] = []
        self._offload = None  # kvc_offload_t* (created on first attend)
        self.offload_mirror_bytes = int(offload_mirror_bytes)
        if self.offload_mirror_bytes < 0:
            raise ValueError("offload_mirror_bytes must be non-negative")

        if self.dtype not in (np.dtype(np.float16), np.dtype(np.float32)):
            raise ValueError(f"unsupported KV storage dtype {self.dtype}")
        if (
            self.num_layers <= 0
            or self.max_seq_len <= 0
            or self.num_kv_heads <= 0
            or self.head_dim <= 0
        ):
            raise ValueError(
                f"KV cache dimensions must all be positive "
                f"(got layers={self.num_layers}, max_seq_len={self.max_seq_len}, "
                f"kv_heads={self.num_kv_heads}, head_dim={self.head_dim})"
            )

        if self.nbytes > max_kv_bytes:
            raise ValueError(
                f"Requested KV cache size ({self.nbytes} bytes) exceeds max_kv_bytes "
                f"sanity limit ({max_kv_bytes} bytes)."
            )

        shape = (self.num_layers, self.max_seq_len, self.num_kv_heads, self.head_dim)
        per_buf_bytes = self.nbytes // 2

        if self.mmap_dir is not None:
            os.makedirs(self.mmap_dir, exist_ok=True)
            uid = f"{os.getpid()}_{id(self):x}"
            k_path = os.path.join(self.mmap_dir, f"kv_cache_k_{uid}.mmap")
            v_path = os.path.join(self.mmap_dir, f"kv_cache_v_{uid}.mmap")
            open_flags = os.O_CREAT | os.O_EXCL | os.O_RDWR | getattr(os, "O_NOFOLLOW", 0)
            try:
                k_fd = os.open(k_path, open_flags, 0o600)
                self._created_mmap_files.append(k_path)
                try:
                    os.ftruncate(k_fd, per_buf_bytes)
                    self._k_mm = mmap.mmap(k_fd, per_buf_bytes, access=mmap.ACCESS_WRITE)
                finally:
                    os.close(k_fd)

                v_fd = os.open(v_path, open_flags, 0o600)
                self._created_mmap_files.append(v_path)
                try:
                    os.ftruncate(v_fd, per_buf_bytes)
                    self._v_mm = mmap.mmap(v_fd, per_buf_bytes, access=mmap.ACCESS_WRITE)
                finally:
                    os.close(v_fd)

                self._k_host = np.frombuffer(self._k_mm, dtype=self.dtype).reshape(shape)
                self._v_host = np.frombuffer(self._v_mm, dtype=self.dtype).reshape(shape)
            except BaseException:
                self.close()
                raise
        elif self.offload_to_cpu:
            self._k_host = _aligned_empty(shape, self.dtype)
            self._v_host = _aligned_empty(shape, self.dtype)
        else:
            with KVCacheManager._gpu_lock:
                if KVCacheManager._active_gpu_instance:
                    raise RuntimeError(
                        "A GPU-resident KVCacheManager is already active in this process "
                        "(DeviceKVCachePool is a singleton). Close the existing instance first "
                        "or pass offload_to_cpu=True."
                    )
                KVCacheManager._active_gpu_instance = True
            try:
                if self.dtype == np.float16:
                    matmul_module.kv_cache_init(
                        self.num_layers, self.max_seq_len, self.num_kv_heads, self.head_dim
                    )
                else:
                    matmul_module.kv_cache_init_ex(
                        self.num_layers, self.max_seq_len, self.num_kv_heads, self.head_dim,
                        dtype=self.dtype,
                    )
                self._allocated = True
            except BaseException:
                with KVCacheManager._gpu_lock:
                    KVCacheManager._active_gpu_instance = False
                self._allocated = False
                try:
                    matmul_module.kv_cache_free()
                except Exception:
                    pass
                raise

    @property
    def nbytes(self) -> int:
        """Total logical bytes across K and V pools (kv_cache.py:164-166)."""
        return (2 * self.num_layers * self.max_seq_len * self.num_kv_heads * self.head_dim
                * self.dtype.itemsize)

    @property
    def mode(self) -> str:
        """Active KV cache storage backend ('gpu', 'cpu', or 'mmap')."""
        if self.mmap_dir is not None:
            return "mmap"
        return "cpu" if self.offload_to_cpu else "gpu"

    @property
    def device_bytes(self) -> int:
        """Bytes allocated in persistent GPU KV pool (0 when offloaded to CPU/mmap)."""
        return 0 if self.offload_to_cpu else self.nbytes

    def record_gpu_layer_step(self, layer_idx: int, q_len: int, start_pos: int) -> None:
        """Bounds check + ``current_seq_len`` update for the fused device layer path
        (kv_cache.py:180-193)."""
        total_kv_len = start_pos + q_len
        if total_kv_len > self.max_seq_len:
            raise ValueError(
                f"Sequence length {total_kv_len} exceeds max_seq_len {self.max_seq_len}"
            )
        if not self._allocated:
            raise RuntimeError("GPU KV cache pool is not allocated or has been closed.")
        if layer_idx == self.num_layers - 1:
            self.current_seq_len = total_kv_len

    # -- offload engine ---------------------------------------------------------
    def _offload_handle(self):
        if self._offload is None:
            import kvcache_ffi as ffi

            h = ctypes.c_void_p()
            ffi.check(ffi.lib.kvc_offload_create(
                ffi.np_ptr(self._k_host), ffi.np_ptr(self._v_host), self.num_layers,
                self.max_seq_len, self.num_kv_heads, self.head_dim,
                ffi.dtype_code_of(self.dtype), ffi.OFFLOAD_REGISTER, _current_device(),
                ctypes.byref(h)))
            self._offload = h
            if self.offload_mirror_bytes > 0:
                n = ctypes.c_int(0)
                ffi.check(ffi.lib.kvc_offload_set_mirror(h, self.offload_mirror_bytes,
                                                         ctypes.byref(n)))
        return self._offload

    def offload_stats(self) -> dict:
        """Host-link statistics of the cpu/mmap modes (bytes, copy-engine ms,
        prefetch hits, attend calls)."""
        if self._offload is None:
            return {"h2d_bytes": 0.0, "h2d_ms": 0.0, "prefetch_hits": 0, "attend_calls": 0,
                    "mirror_layers": 0, "mirror_bytes": 0.0}
        import kvcache_ffi as ffi

        b, ms = ctypes.c_double(), ctypes.c_double()
        hits, calls = ctypes.c_int64(), ctypes.c_int64()
        ffi.check(ffi.lib.kvc_offload_stats(self._offload, ctypes.byref(b), ctypes.byref(ms),
                                            ctypes.byref(hits), ctypes.byref(calls)))
        nl, mb = ctypes.c_int(), ctypes.c_double()
        ffi.check(ffi.lib.kvc_offload_mirror_stats(self._offload, ctypes.byref(nl),
                                                   ctypes.byref(mb)))
        return {"h2d_bytes": b.value, "h2d_ms": ms.value, "prefetch_hits": hits.value,
                "attend_calls": calls.value, "mirror_layers": nl.value, "mirror_bytes": mb.value}

    def attend(
        self,
        q_rot: np.ndarray,
        k_new: np.ndarray,
        v_new: np.ndarray,
        out: np.ndarray,
        layer_idx: int,
        q_len: int,
        start_pos: int,
        num_heads: int,
        scale: float,
        causal: bool = True,
    ) -> None:
        """
        Write `k_new` and `v_new` (`q_len` tokens) into the KV cache at
        `(layer_idx, start_pos)` and compute GQA online-softmax attention over
        `[0 .. start_pos + q_len)`.
        """
        total_kv_len = start_pos + q_len
        if total_kv_len > self.max_seq_len:
            raise ValueError(
                f"Sequence length {total_kv_len} exceeds max_seq_len {self.max_seq_len}"
            )

        if self.offload_to_cpu:
            if self._k_host is None or self._v_host is None:
                raise RuntimeError("CPU/mmap KV cache buffers are not allocated or have been closed.")
            import kvcache_ffi as ffi

            rows = (int(q_len), self.num_kv_heads, self.head_dim)
            # numpy slice-assignment semantics of kv_cache.py:224-225 (cast, broadcast)
            k_rows = np.ascontiguousarray(np.broadcast_to(np.asarray(k_new), rows), dtype=self.dtype)
            v_rows = np.ascontiguousarray(np.broadcast_to(np.asarray(v_new), rows), dtype=self.dtype)
            q_elems = int(q_len) * int(num_heads) * self.head_dim
            q = matmul_module._check_array(q_rot, "Q", q_elems, self.dtype)
            o = matmul_module._check_array(out, "Out", q_elems, self.dtype, require_writeable=True)
            if int(num_heads) <= 0 or int(num_heads) % self.num_kv_heads != 0:
                raise ValueError("num_heads must be divisible by num_kv_heads.")
            ffi.check(ffi.lib.kvc_offload_attend(
                self._offload_handle(), ffi.np_ptr(q), ffi.np_ptr(k_rows), ffi.np_ptr(v_rows),
                ffi.np_ptr(o), int(layer_idx), int(q_len), int(start_pos), int(num_heads),
                float(scale), int(bool(causal))))
        else:
            if not self._allocated:
                raise RuntimeError("GPU KV cache pool is not allocated or has been closed.")
            matmul_module.gqa_attention_cached(
                q_rot,
                k_new,
                v_new,
                out,
                layer_idx,
                q_len,
                start_pos,
                num_heads,
                self.num_kv_heads,
                self.head_dim,
                scale,
                causal,
            )

        if layer_idx == self.num_layers - 1:
            self.current_seq_len = total_kv_len

    @property
    def mmap_files(self) -> List[str]:
        """Paths of disk-backed mmap files created by this instance."""
        return list(self._created_mmap_files)

    def reset(self) -> None:
        """Reset logical sequence length to 0 without reallocating memory."""
        self.current_seq_len = 0

    def close(self) -> None:
        if getattr(self, "_allocated", False):
            try:
                matmul_module.kv_cache_free()
            finally:
                self._allocated = False
                with KVCacheManager._gpu_lock:
                    KVCacheManager._active_gpu_instance = False
        off = getattr(self, "_offload", None)
        if off is not None:
            self._offload = None
            import kvcache_ffi as ffi

            ffi.check(ffi.lib.kvc_offload_destroy(off))
        self._k_host = None
        self._v_host = None
        for attr in ("_k_mm", "_v_mm"):
            mm = getattr(self, attr, None)
            if mm is not None:
                try:
                    mm.close()
                finally:
                    setattr(self, attr, None)
        for p in getattr(self, "_created_mmap_files", []):
            try:
                if os.path.exists(p):
                    os.remove(p)
            except OSError:
                pass
        if hasattr(self, "_created_mmap_files"):
            self._created_mmap_files.clear()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception as exc:
            try:
                warnings.warn(
                    f"KVCacheManager.close() raised during finalization: {exc}",
                    RuntimeWarning,
                    stacklevel=2,
                )
            except Exception:
                pass

    def __enter__(self) -> "KVCacheManager":
        return self

    def __exit__(self, exc_type, exc_val, exc_tb) -> None:
        self.close()


def _current_device() -> int:
    dev = os.environ.get("KVC_DEVICE")
    if dev is not None:
        return int(dev)
    try:
        import torch

        if torch.cuda.is_available():
            return int(torch.cuda.current_device())
    except Exception:
        pass
    return 0
