"""Batched decode over a paged KV pool (torch device buffers + libkvcache.so).

The reference keeps one sequence in an unpaged pool and "batches" with a
sequential Python loop (src/inference.py:435-447).  This module is the batched
form of the same path: many sequences share one pool of fixed-size pages,
addressed through int32 block tables, and one decode step per layer appends the
new K/V row of every sequence and attends over its whole cached context
(the per-token append of attention.hip:410-415 and the attention of
attention.hip:35-123, for a batch).

Buffers are torch CUDA tensors; work is enqueued on torch's current stream
unless a stream is given.  KV-head sharding across GPUs is a matter of
building each rank's pool with its own ``num_kv_heads`` slice (see
``shard_heads``).
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np
import torch

import kvcache_ffi as ffi

_TORCH_CODE = {torch.float16: ffi.DTYPE_F16, torch.bfloat16: ffi.DTYPE_BF16,
               torch.float32: ffi.DTYPE_F32}


def _sp(stream) -> Optional[int]:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream) or None


def _i32(t: torch.Tensor) -> int:
    if t.dtype != torch.int32 or not t.is_cuda or not t.is_contiguous():
        raise ValueError("block tables / rows / positions must be contiguous int32 CUDA tensors")
    return int(t.data_ptr())


def _dev(t: torch.Tensor, name: str, dtype: torch.dtype, numel: int) -> int:
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous {dtype} CUDA tensor")
    if t.numel() < numel:
        raise ValueError(f"{name} buffer is smaller than expected dimensions.")
    return int(t.data_ptr())


@dataclass
class PlanInfo:
    n_queries: int
    n_items: int
    n_ctas: int
    scratch_bytes: int


class DecodePlan:
    """Split-K work list for one batch of queries (see kvc_plan_decode)."""

    def __init__(self):
        h = ctypes.c_void_p()
        ffi.check(ffi.lib.kvc_plan_create(ctypes.byref(h)))
        self.handle = h
        self.n_queries = 0
        self.num_heads = 0
        self.ctx_lens: Optional[np.ndarray] = None
        self.flags = 0

    def _set_flag(self, flag: int, on: bool) -> None:
        flags = (self.flags | flag) if on else (self.flags & ~flag)
        ffi.check(ffi.lib.kvc_plan_set_flags(self.handle, flags))
        self.flags = flags

    def set_kv_stable(self, stable: bool = True) -> None:
        """Declare that block tables and KV pages are not written by the kernel
        launched right before each decode (lets the kernel start streaming KV
        early; see KVC_PLAN_KV_STABLE)."""
        self._set_flag(ffi.PLAN_KV_STABLE, stable)

    def set_graph_stable(self, on: bool = True) -> None:
        """Let decode launches of this plan be captured in a CUDA graph and replayed
        after rebuilds for grown contexts (KVC_PLAN_GRAPH); re-capture whenever
        ``generation`` changes.  Set before the first build."""
        self._set_flag(ffi.PLAN_GRAPH, on)

    @property
    def generation(self) -> int:
        """Layout generation: launches captured under another value are stale."""
        g = ctypes.c_uint64()
        ffi.check(ffi.lib.kvc_plan_generation(self.handle, ctypes.byref(g)))
        return g.value

    def info(self) -> PlanInfo:
        n_items, n_ctas = ctypes.c_int(), ctypes.c_int()
        scratch = ctypes.c_size_t()
        ffi.check(ffi.lib.kvc_plan_info(self.handle, ctypes.byref(n_items), ctypes.byref(n_ctas),
                                        ctypes.byref(scratch)))
        return PlanInfo(self.n_queries, n_items.value, n_ctas.value, scratch.value)

    def close(self):
        if self.handle is not None:
            ffi.check(ffi.lib.kvc_plan_destroy(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PagedKVCache:
    """Paged K/V pool for ``num_layers`` layers on one GPU."""

    def __init__(self, num_layers: int, num_pages: int, page_size: int, num_kv_heads: int,
                 head_dim: int, dtype: torch.dtype = torch.float16, device: int = 0):
        if dtype not in _TORCH_CODE:
            raise ValueError(f"unsupported KV storage dtype {dtype}")
        h = ctypes.c_void_p()
        ffi.check(ffi.lib.kvc_pool_create(num_layers, num_pages, page_size, num_kv_heads,
                                          head_dim, _TORCH_CODE[dtype], device, ctypes.byref(h)))
        self.handle = h
        self.num_layers = num_layers
        self.num_pages = num_pages
        self.page_size = page_size
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = device

    # -- synthetic contents ------------------------------------------------------
    def fill_normal(self, seed: int, stddev: float = 1.0, layers=None, pages=None, stream=None):
        l0, l1 = layers if layers is not None else (0, self.num_layers)
        p0, p1 = pages if pages is not None else (0, self.num_pages)
        ffi.check(ffi.lib.kvc_pool_fill_normal(self.handle, l0, l1, p0, p1, int(seed),
                                               float(stddev), _sp(stream)))

    def info(self):
        k, v = ctypes.c_void_p(), ctypes.c_void_p()
        lb, phb = ctypes.c_size_t(), ctypes.c_size_t()
        ffi.check(ffi.lib.kvc_pool_info(self.handle, ctypes.byref(k), ctypes.byref(v),
                                        ctypes.byref(lb), ctypes.byref(phb)))
        return {"k": k.value, "v": v.value, "bytes_per_layer": lb.value,
                "bytes_per_page_head": phb.value}

    # -- plan / append / decode ---------------------------------------------------
    def plan(self, ctx_lens: Sequence[int], num_heads: int, rows: Optional[Sequence[int]] = None,
             plan: Optional[DecodePlan] = None, stream=None) -> DecodePlan:
        """Plan attention for query i over positions [0, ctx_lens[i]) of block-table
        row rows[i] (default i)."""
        p = plan if plan is not None else DecodePlan()
        ctx = np.ascontiguousarray(np.asarray(ctx_lens, dtype=np.int32))
        r = None if rows is None else np.ascontiguousarray(np.asarray(rows, dtype=np.int32))
        ffi.check(ffi.lib.kvc_plan_decode(p.handle, self.handle, ffi.np_ptr(r), ffi.np_ptr(ctx),
                                          int(ctx.size), int(num_heads), _sp(stream)))
        p.n_queries = int(ctx.size)
        p.num_heads = int(num_heads)
        p.ctx_lens = ctx
        return p

    def append(self, layer: int, k_new: torch.Tensor, v_new: torch.Tensor,
               block_tables: torch.Tensor, positions: torch.Tensor,
               rows: Optional[torch.Tensor] = None, stream=None):
        n = int(positions.numel())
        row_elems = self.num_kv_heads * self.head_dim
        ffi.check(ffi.lib.kvc_append(
            self.handle, layer, _dev(k_new, "k_new", self.dtype, n * row_elems),
            _dev(v_new, "v_new", self.dtype, n * row_elems), _i32(block_tables),
            int(block_tables.shape[-1]), None if rows is None else _i32(rows), _i32(positions), n,
            _sp(stream)))

    def decode(self, plan: DecodePlan, layer: int, q: torch.Tensor, out: torch.Tensor,
               block_tables: torch.Tensor, scale: float, stream=None):
        n = plan.n_queries * plan.num_heads * self.head_dim
        ffi.check(ffi.lib.kvc_decode(
            self.handle, plan.handle, layer, _dev(q, "q", self.dtype, n),
            _dev(out, "out", self.dtype, n), _i32(block_tables), int(block_tables.shape[-1]),
            float(scale), _sp(stream)))

    def append_decode(self, plan: DecodePlan, layer: int, q: torch.Tensor, k_new: torch.Tensor,
                      v_new: torch.Tensor, out: torch.Tensor, block_tables: torch.Tensor,
                      scale: float, stream=None):
        n = plan.n_queries * plan.num_heads * self.head_dim
        nk = plan.n_queries * self.num_kv_heads * self.head_dim
        ffi.check(ffi.lib.kvc_append_decode(
            self.handle, plan.handle, layer, _dev(q, "q", self.dtype, n),
            _dev(k_new, "k_new", self.dtype, nk), _dev(v_new, "v_new", self.dtype, nk),
            _dev(out, "out", self.dtype, n), _i32(block_tables), int(block_tables.shape[-1]),
            float(scale), _sp(stream)))

    def append_decode_rope(self, plan: DecodePlan, layer: int, q: torch.Tensor,
                           k_new: torch.Tensor, v_new: torch.Tensor, out: torch.Tensor,
                           block_tables: torch.Tensor, scale: float, freq_base: float = 10000.0,
                           neox: bool = False, stream=None):
        """append_decode with q and k_new rotated (RoPE) at each query's position
        first (kvc_append_decode_rope); q and k_new are not modified."""
        n = plan.n_queries * plan.num_heads * self.head_dim
        nk = plan.n_queries * self.num_kv_heads * self.head_dim
        ffi.check(ffi.lib.kvc_append_decode_rope(
            self.handle, plan.handle, layer, _dev(q, "q", self.dtype, n),
            _dev(k_new, "k_new", self.dtype, nk), _dev(v_new, "v_new", self.dtype, nk),
            _dev(out, "out", self.dtype, n), _i32(block_tables), int(block_tables.shape[-1]),
            float(scale), float(freq_base), int(bool(neox)), _sp(stream)))

    def append_decode_xchg(self, plan: DecodePlan, layer: int, q: torch.Tensor,
                           k_new: Optional[torch.Tensor], v_new: Optional[torch.Tensor],
                           xchg_handle, slot: int, total_heads: int, head_offset: int,
                           block_tables: torch.Tensor, scale: float, stream=None):
        """append_decode with the outputs pushed into every rank's exchange slot
        (kvc_append_decode_xchg); see sharding.HeadExchange."""
        n = plan.n_queries * plan.num_heads * self.head_dim
        nk = plan.n_queries * self.num_kv_heads * self.head_dim
        kp = None if k_new is None else _dev(k_new, "k_new", self.dtype, nk)
        vp = None if v_new is None else _dev(v_new, "v_new", self.dtype, nk)
        ffi.check(ffi.lib.kvc_append_decode_xchg(
            self.handle, plan.handle, layer, _dev(q, "q", self.dtype, n), kp, vp, xchg_handle,
            int(slot), int(total_heads), int(head_offset), _i32(block_tables),
            int(block_tables.shape[-1]), float(scale), _sp(stream)))

    def decode_host(self, plan: DecodePlan, layer: int, h_q: torch.Tensor, h_k: torch.Tensor,
                    h_v: torch.Tensor, h_out: torch.Tensor, block_tables: torch.Tensor,
                    scale: float, stream=None):
        """Reference-facing call: host (ideally pinned) buffers in, host result out."""
        for name, t in (("q", h_q), ("k_new", h_k), ("v_new", h_v), ("out", h_out)):
            if t.is_cuda or not t.is_contiguous() or t.dtype != self.dtype:
                raise ValueError(f"{name} must be a contiguous {self.dtype} host tensor")
        ffi.check(ffi.lib.kvc_decode_host(
            self.handle, plan.handle, layer, int(h_q.data_ptr()), int(h_k.data_ptr()),
            int(h_v.data_ptr()), int(h_out.data_ptr()), _i32(block_tables),
            int(block_tables.shape[-1]), float(scale), _sp(stream)))

    def forward_layer(self, plan: DecodePlan, layer: int, x: torch.Tensor, out: torch.Tensor,
                      weights: "DeviceLayerWeights", block_tables: torch.Tensor,
                      eps: float = 1e-5, freq_base: float = 10000.0, neox: bool = False,
                      scale: Optional[float] = None, stream=None):
        """One transformer layer for the plan's queries (kvc_forward_layer_paged):
        x / out (n_queries, hidden) fp16, token i being query i's new token at
        position ctx_i - 1 of its block-table row.  out may be x."""
        n = plan.n_queries * weights.hidden
        sc = default_scale(self.head_dim) if scale is None else float(scale)
        if len(weights.w) != 7 or len(weights.types) != 7:
            raise ValueError("a layer has seven weights: q, k, v, o, gate, up, down")
        for t in weights.w:
            if not t.is_cuda or not t.is_contiguous():
                raise ValueError("weights must be contiguous CUDA tensors")
        w = [int(t.data_ptr()) for t in weights.w]
        ty = [int(t) for t in weights.types]
        ffi.check(ffi.lib.kvc_forward_layer_paged(
            self.handle, plan.handle, layer, _dev(x, "x", torch.float16, n),
            _dev(out, "out", torch.float16, n),
            _dev(weights.attn_norm, "attn_norm", torch.float16, weights.hidden), w[0], ty[0],
            w[1], ty[1], w[2], ty[2], w[3], ty[3],
            _dev(weights.ffn_norm, "ffn_norm", torch.float16, weights.hidden), w[4], ty[4],
            w[5], ty[5], w[6], ty[6], _i32(block_tables), int(block_tables.shape[-1]),
            weights.hidden, weights.intermediate, float(eps), float(freq_base), int(bool(neox)),
            sc, _sp(stream)))

    def gather(self, layer: int, block_tables: torch.Tensor, row: int, start: int, count: int,
               stream=None):
        k = torch.empty((count, self.num_kv_heads, self.head_dim), dtype=self.dtype,
                        device=f"cuda:{self.device}")
        v = torch.empty_like(k)
        ffi.check(ffi.lib.kvc_gather(self.handle, layer, _i32(block_tables),
                                     int(block_tables.shape[-1]), row, start, count,
                                     int(k.data_ptr()), int(v.data_ptr()), _sp(stream)))
        return k, v

    def close(self):
        if self.handle is not None:
            ffi.check(ffi.lib.kvc_pool_destroy(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class DeviceLayerWeights:
    """One transformer layer's weights resident on the GPU: the two RMSNorm
    weights ((hidden,) fp16) and the seven GGML-typed weights (raw block bytes,
    kvc_weight_bytes long) in the order q, k, v, o, gate, up, down, with their
    type ids (KVC_WTYPE_*), as forward_layer_cached takes them."""
    attn_norm: torch.Tensor
    ffn_norm: torch.Tensor
    w: Sequence[torch.Tensor]
    types: Sequence[int]
    hidden: int
    intermediate: int


class BatchDecoder:
    """The decode loop of generate_batch_ids (src/inference.py:435-447) on the
    paged pool: the reference decodes its prompts one after another, one
    forward_layer_cached call per (sequence, layer, token); here every sequence
    of the batch advances by one token per step, one kvc_forward_layer_paged
    call per layer for the whole batch.  Sequence i owns block-table row i;
    ``ctx_lens[i]`` counts its cached positions.  The embedding lookup, the
    final norm, the LM head and sampling stay with the caller."""

    def __init__(self, cache: PagedKVCache, layers: Sequence[DeviceLayerWeights],
                 block_tables: torch.Tensor, num_heads: int, ctx_lens: Sequence[int],
                 eps: float = 1e-5, freq_base: float = 10000.0, neox: bool = False,
                 scale: Optional[float] = None):
        if len(layers) != cache.num_layers:
            raise ValueError("one DeviceLayerWeights per pool layer is required")
        if block_tables.dim() != 2 or block_tables.shape[0] < len(ctx_lens):
            raise ValueError("block_tables needs one row per sequence")
        self.cache, self.layers, self.bt = cache, list(layers), block_tables
        self.num_heads = int(num_heads)
        self.ctx = np.asarray(ctx_lens, dtype=np.int64).copy()
        self.eps, self.freq_base, self.neox, self.scale = eps, freq_base, neox, scale
        self.plan = DecodePlan()
        self.capacity = int(block_tables.shape[1]) * cache.page_size

    def prefill(self, seq: int, x: torch.Tensor, stream=None) -> torch.Tensor:
        """Run tokens x (n, hidden) of sequence `seq` at positions ctx_lens[seq]..
        through every layer (causal over the cached prefix and the chunk itself);
        returns the last layer's output (n, hidden)."""
        n = int(x.shape[0])
        if n == 0:
            return x
        p0 = int(self.ctx[seq])
        if p0 + n > self.capacity:
            raise IndexError("prefill exceeds the sequence's block-table capacity")
        self.cache.plan(np.arange(p0 + 1, p0 + n + 1), self.num_heads, rows=[seq] * n,
                        plan=self.plan, stream=stream)
        y = self._layers(x, stream)
        self.ctx[seq] += n
        return y

    def step(self, x: torch.Tensor, stream=None) -> torch.Tensor:
        """One decode step: token i of x (batch, hidden) is sequence i's next token
        at position ctx_lens[i]; returns the last layer's output (batch, hidden)."""
        b = len(self.ctx)
        if int(x.shape[0]) != b:
            raise ValueError(f"x must hold one token per sequence ({b})")
        if int(self.ctx.max(initial=0)) + 1 > self.capacity:
            raise IndexError("a sequence would exceed its block-table capacity")
        self.cache.plan(self.ctx + 1, self.num_heads, plan=self.plan, stream=stream)
        y = self._layers(x, stream)
        self.ctx += 1
        return y

    def _layers(self, x: torch.Tensor, stream) -> torch.Tensor:
        cur = x.contiguous()
        bufs = (torch.empty_like(cur), torch.empty_like(cur))   # x itself is never written
        for layer, lw in enumerate(self.layers):
            nxt = bufs[layer % 2]
            self.cache.forward_layer(self.plan, layer, cur, nxt, lw, self.bt, self.eps,
                                     self.freq_base, self.neox, self.scale, stream)
            cur = nxt
        return cur

    def close(self):
        self.plan.close()


# -- layout helpers -------------------------------------------------------------------
def rope(x: torch.Tensor, out: torch.Tensor, positions: Optional[torch.Tensor] = None,
         pos_offset: int = 0, freq_base: float = 10000.0, neox: bool = False, stream=None):
    """Rotary position embedding of x (tokens, heads, D) into out on the GPU
    (kvc_rope); token t at positions[t] (int32 CUDA tensor) or pos_offset + t."""
    if x.dim() != 3:
        raise ValueError("x must be (tokens, heads, head_dim)")
    n, heads, d = x.shape
    dt = _TORCH_CODE.get(x.dtype)
    if dt is None:
        raise ValueError(f"unsupported dtype {x.dtype}")
    xp = _dev(x, "x", x.dtype, n * heads * d)
    op = _dev(out, "out", x.dtype, n * heads * d)
    pp = None if positions is None else _i32(positions)
    ffi.check(ffi.lib.kvc_rope(xp, op, n, heads, d, pp, int(pos_offset), float(freq_base),
                               int(bool(neox)), dt, _sp(stream)))
    return out


def pages_for(ctx_lens: Sequence[int], page_size: int) -> np.ndarray:
    return np.array([(int(c) + page_size - 1) // page_size for c in ctx_lens], dtype=np.int64)


def random_block_tables(ctx_lens: Sequence[int], page_size: int, seed: int):
    """Block tables for sequences of the given lengths over a pool with exactly
    the pages they need, assigned in a seeded random permutation (benchmark
    config 3: "paged fp16 pool of 16-token pages with a random page permutation").
    Returns (table (n, max_pages) int32 numpy, total pages)."""
    need = pages_for(ctx_lens, page_size)
    total = int(need.sum())
    perm = np.random.default_rng(seed).permutation(total).astype(np.int32)
    width = int(need.max()) if len(need) else 1
    table = np.full((len(need), max(1, width)), -1, dtype=np.int32)
    o = 0
    for i, n in enumerate(need):
        table[i, :n] = perm[o:o + n]
        o += int(n)
    # unused tail entries point at page 0 (never read: beyond every context)
    table[table < 0] = 0
    return table, total


def shard_heads(num_kv_heads: int, world: int, rank: int):
    """KV heads [h0, h1) owned by `rank` when heads are split across `world` GPUs."""
    from sharding import shard_heads as _shard

    return _shard(num_kv_heads, world, rank)


def default_scale(head_dim: int) -> float:
    """1/sqrt(head_dim), the scale every caller passes (src/layer.py:181)."""
    return 1.0 / math.sqrt(head_dim)
