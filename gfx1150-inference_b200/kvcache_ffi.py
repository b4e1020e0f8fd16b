"""ctypes binding of libkvcache.so (the C ABI in include/kvcache.h).

This is the only place Python touches the native library.  Status codes are
turned into the exception classes the reference's pybind11 module raises for
the same failures (pybind11 maps std::invalid_argument -> ValueError,
std::out_of_range -> IndexError, std::runtime_error -> RuntimeError;
src/python_bindings/bindings.cpp and src/kernels/attention.hip:15-23, :242-247,
:316-329).

There is no fallback: if the library cannot be loaded, importing this module
raises ImportError with the build command, the way the reference's
``import matmul_module`` fails when the HIP extension is missing
(src/kv_cache.py:26-40).
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("KVC_LIB_PATH", os.path.join(_HERE, "libkvcache.so"))

KVC_OK = 0
KVC_ERR_INVALID_ARG = 1
KVC_ERR_OUT_OF_RANGE = 2
KVC_ERR_RUNTIME = 3
KVC_ERR_CUDA = 4
KVC_ERR_DEVICE = 5
KVC_ERR_TIMEOUT = 6

DTYPE_F16 = 0
DTYPE_BF16 = 1
DTYPE_F32 = 2

PLAN_KV_STABLE = 1
PLAN_GRAPH = 2

OFFLOAD_PINNED = 1
OFFLOAD_REGISTER = 2

# kvc_test_inject_failure sites
FAULT_DEVICE_ALLOC = 1
FAULT_HOST_ALLOC = 2
FAULT_HOST_REGISTER = 3
FAULT_WAIT = 4

_NP_DTYPE = {DTYPE_F16: np.dtype(np.float16), DTYPE_F32: np.dtype(np.float32)}

_c_int = ctypes.c_int
_c_float = ctypes.c_float
_c_size = ctypes.c_size_t
_vp = ctypes.c_void_p
_i32p = ctypes.POINTER(ctypes.c_int32)

# forward_layer_cached's 30 arguments (bindings.cpp:562-587 order; rope_neox as int)
_LAYER_ARGS = ([_vp, _vp, _vp] + [_vp, _c_int] * 4 + [_vp] + [_vp, _c_int] * 3
               + [_c_int] * 8 + [_c_float, _c_float, _c_int, _c_float])

# GGML weight type ids (KVC_WTYPE_*)
WTYPE_F16, WTYPE_Q4_0, WTYPE_Q8_0, WTYPE_Q4_K, WTYPE_Q6_K = 1, 2, 8, 12, 14

# name -> (restype, argtypes); mirrors include/kvcache.h one to one.
SIGNATURES = {
    "kvc_version": (_c_int, []),
    "kvc_last_error": (ctypes.c_char_p, []),
    "kvc_device_error": (_c_int, [_c_int, _c_int, ctypes.POINTER(ctypes.c_uint32),
                                  ctypes.POINTER(ctypes.c_uint32)]),
    "kvc_device_sm_count": (_c_int, [_c_int, ctypes.POINTER(_c_int)]),
    "kvc_set_host_wait_limit": (_c_int, [ctypes.c_double]),
    "kvc_test_inject_failure": (_c_int, [_c_int, _c_int, _c_int]),
    "kvc_cache_init": (_c_int, [_c_int, _c_int, _c_int, _c_int]),
    "kvc_cache_init_ex": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int]),
    "kvc_cache_free": (_c_int, []),
    "kvc_cache_dtype": (_c_int, []),
    "kvc_gqa_attention_cached": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                                          _c_int, _c_int, _c_float, _c_int]),
    "kvc_gqa_attention_cached_device": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int,
                                                 _c_int, _c_int, _c_int, _c_float, _c_int, _vp]),
    "kvc_gqa_attention": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                                   _c_int, _c_float, _c_int]),
    "kvc_gqa_attention_ex": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                                      _c_int, _c_float, _c_int, _c_int]),
    "kvc_cache_gather": (_c_int, [_c_int, _c_int, _c_int, _vp, _vp]),
    "kvc_pool_create": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                 ctypes.POINTER(_vp)]),
    "kvc_pool_destroy": (_c_int, [_vp]),
    "kvc_pool_info": (_c_int, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                               ctypes.POINTER(_c_size), ctypes.POINTER(_c_size)]),
    "kvc_pool_fill_normal": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, ctypes.c_uint64,
                                      _c_float, _vp]),
    "kvc_append": (_c_int, [_vp, _c_int, _vp, _vp, _vp, _c_int, _vp, _vp, _c_int, _vp]),
    "kvc_plan_create": (_c_int, [ctypes.POINTER(_vp)]),
    "kvc_plan_destroy": (_c_int, [_vp]),
    "kvc_plan_decode": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _vp]),
    "kvc_plan_set_flags": (_c_int, [_vp, _c_int]),
    "kvc_plan_generation": (_c_int, [_vp, ctypes.POINTER(ctypes.c_uint64)]),
    "kvc_plan_split_tokens": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                                       ctypes.POINTER(_c_int)]),
    "kvc_plan_split_counts": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                                       ctypes.POINTER(_c_int), _vp, ctypes.POINTER(_c_int)]),
    "kvc_plan_info": (_c_int, [_vp, ctypes.POINTER(_c_int), ctypes.POINTER(_c_int),
                               ctypes.POINTER(_c_size)]),
    "kvc_decode": (_c_int, [_vp, _vp, _c_int, _vp, _vp, _vp, _c_int, _c_float, _vp]),
    "kvc_append_decode": (_c_int, [_vp, _vp, _c_int, _vp, _vp, _vp, _vp, _vp, _c_int, _c_float,
                                   _vp]),
    "kvc_decode_host": (_c_int, [_vp, _vp, _c_int, _vp, _vp, _vp, _vp, _vp, _c_int, _c_float,
                                 _vp]),
    "kvc_gather": (_c_int, [_vp, _c_int, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp]),
    "kvc_decode_noalloc": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _c_int,
                                    _vp, _c_int, _c_int, _vp, _vp, _c_float, _vp]),
    "kvc_host_alloc": (_c_int, [_c_size, ctypes.POINTER(_vp)]),
    "kvc_host_free": (_c_int, [_vp]),
    "kvc_offload_create": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                    _c_int, ctypes.POINTER(_vp)]),
    "kvc_offload_destroy": (_c_int, [_vp]),
    "kvc_offload_attend": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                                    _c_float, _c_int]),
    "kvc_offload_invalidate": (_c_int, [_vp]),
    "kvc_offload_stats": (_c_int, [_vp, ctypes.POINTER(ctypes.c_double),
                                   ctypes.POINTER(ctypes.c_double),
                                   ctypes.POINTER(ctypes.c_int64),
                                   ctypes.POINTER(ctypes.c_int64)]),
    "kvc_rope_host": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_float, _c_int]),
    "kvc_rope": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _vp, _c_int, _c_float, _c_int, _c_int,
                          _vp]),
    "kvc_append_decode_rope": (_c_int, [_vp, _vp, _c_int, _vp, _vp, _vp, _vp, _vp, _c_int,
                                        _c_float, _c_float, _c_int, _vp]),
    "kvc_offload_set_mirror": (_c_int, [_vp, _c_size, ctypes.POINTER(_c_int)]),
    "kvc_offload_mirror_stats": (_c_int, [_vp, ctypes.POINTER(_c_int),
                                          ctypes.POINTER(ctypes.c_double)]),
    "kvc_xchg_create": (_c_int, [_c_int, _c_int, _c_int, _c_size, _c_int, ctypes.POINTER(_vp)]),
    "kvc_xchg_handle": (_c_int, [_vp, _vp]),
    "kvc_xchg_connect": (_c_int, [_vp, _vp]),
    "kvc_xchg_connect_ptrs": (_c_int, [_vp, ctypes.POINTER(_vp)]),
    "kvc_xchg_base": (_c_int, [_vp, ctypes.POINTER(_vp)]),
    "kvc_xchg_slot": (_c_int, [_vp, _c_int, ctypes.POINTER(_vp)]),
    "kvc_xchg_set_wait_limit": (_c_int, [_vp, ctypes.c_double]),
    "kvc_xchg_destroy": (_c_int, [_vp]),
    "kvc_append_decode_xchg": (_c_int, [_vp, _vp, _c_int, _vp, _vp, _vp, _vp, _c_int, _c_int,
                                        _c_int, _vp, _c_int, _c_float, _vp]),
    "kvc_weight_bytes": (_c_int, [_c_int, _c_int, _c_int, ctypes.POINTER(_c_size)]),
    "kvc_linear": (_c_int, [_vp, _c_int, _c_int, _vp, _c_int, _c_int, _vp, _vp]),
    "kvc_linear_swiglu": (_c_int, [_vp, _c_int, _c_int, _vp, _vp, _c_int, _c_int, _vp, _vp]),
    "kvc_linear_residual": (_c_int, [_vp, _c_int, _c_int, _vp, _c_int, _c_int, _vp, _vp, _vp]),
    "kvc_rmsnorm": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_float, _vp]),
    "kvc_forward_layer_cached": (_c_int, _LAYER_ARGS),
    "kvc_forward_layer_cached_device": (_c_int, _LAYER_ARGS + [_vp]),
    "kvc_forward_layer_paged": (_c_int, [_vp, _vp, _c_int, _vp, _vp, _vp, _vp, _c_int, _vp, _c_int,
                                         _vp, _c_int, _vp, _c_int, _vp, _vp, _c_int, _vp, _c_int,
                                         _vp, _c_int, _vp, _c_int, _c_int, _c_int, _c_float,
                                         _c_float, _c_int, _c_float, _vp]),
}

XCHG_HANDLE_BYTES = 64


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libkvcache.so not found at {LIB_PATH}. Build it first with:\n"
            f"  python {os.path.join(_HERE, 'build_lib.py')}\n"
            "(nvcc for sm_100a is required; there is no CPU fallback)."
        )
    try:
        lib = ctypes.CDLL(LIB_PATH)
    except OSError as exc:  # pragma: no cover - depends on the machine
        raise ImportError(f"failed to load {LIB_PATH}: {exc}") from exc
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class KVCacheDeviceError(RuntimeError):
    """A kernel reported a bad block-table entry or gave up a bounded wait."""


def last_error() -> str:
    msg = lib.kvc_last_error()
    return msg.decode("utf-8", "replace") if msg else ""


def check(rc: int, what: str = "") -> None:
    """Raise the reference's exception class for a non-zero status."""
    if rc == KVC_OK:
        return
    msg = last_error() or what
    if rc == KVC_ERR_INVALID_ARG:
        raise ValueError(msg)
    if rc == KVC_ERR_OUT_OF_RANGE:
        raise IndexError(msg)
    if rc == KVC_ERR_DEVICE:
        raise KVCacheDeviceError(msg)
    if rc == KVC_ERR_TIMEOUT:
        raise TimeoutError(msg)
    raise RuntimeError(msg)


# ---- pointer helpers -----------------------------------------------------------------
def np_ptr(a: Optional[np.ndarray]) -> Optional[int]:
    if a is None:
        return None
    return a.__array_interface__["data"][0]


def torch_ptr(t) -> Optional[int]:
    if t is None:
        return None
    return int(t.data_ptr())


def torch_stream_ptr(stream=None) -> Optional[int]:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream) or None


def device_error(device: int = 0, clear: bool = True):
    code = ctypes.c_uint32(0)
    info = ctypes.c_uint32(0)
    check(lib.kvc_device_error(device, int(clear), ctypes.byref(code), ctypes.byref(info)))
    return int(code.value), int(info.value)


def set_host_wait_limit(seconds: float) -> None:
    """Limit of the library's host waits for its own GPU work (kvc_set_host_wait_limit)."""
    check(lib.kvc_set_host_wait_limit(float(seconds)))


def inject_failure(site: int, count: int = 1, skip: int = 0) -> None:
    """Test hook: the next ``count`` calls at ``site`` (FAULT_*) after ``skip``
    successful ones fail on the host (kvc_test_inject_failure); count 0 disarms."""
    check(lib.kvc_test_inject_failure(int(site), int(skip), int(count)))


def np_dtype_of(dtype_code: int) -> np.dtype:
    if dtype_code not in _NP_DTYPE:
        raise ValueError(f"no numpy dtype for KV storage dtype {dtype_code}")
    return _NP_DTYPE[dtype_code]


def dtype_code_of(dtype) -> int:
    """KV storage dtype code for a numpy or torch dtype."""
    name = str(dtype).replace("torch.", "")
    if name in ("float16", "<f2", "half"):
        return DTYPE_F16
    if name in ("bfloat16",):
        return DTYPE_BF16
    if name in ("float32", "<f4", "float"):
        return DTYPE_F32
    raise ValueError(f"unsupported KV storage dtype {dtype}")
