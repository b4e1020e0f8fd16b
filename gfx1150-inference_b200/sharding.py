"""Multi-GPU decode: one process per GPU, sharded by sequence or by KV head.

The reference runs one model on one GPU (src/inference.py); its KV path has no
multi-device form.  On an 8-GPU B200 node the decode step shards two ways:

* by sequence (``shard_sequences``): each rank owns whole sequences, their
  pages and block tables.  Ranks never exchange data, so there is no
  collective on the data path and per-GPU work stays fixed as GPUs are added
  (weak scaling).
* by KV head (``shard_heads`` / ``HeadShardedDecode``): each rank holds KV
  heads [h0, h1) of every sequence and the q-heads that read them (GQA keeps
  a q-head's whole group on the KV head's rank, so attention needs no
  exchange).  The next layer's output projection needs every head, so the
  per-head outputs are exchanged once per layer (strong scaling: total work
  fixed, per-GPU KV shrinks with the number of GPUs).  Two transports:
  ``"p2p"`` (default on GPUs) — the decode's merge kernel stores every output
  row into all ranks' exchange slots over NVLink and a one-warp kernel waits for the
  ranks' epochs (``HeadExchange``, the C ABI's kvc_xchg_*); ``"nccl"`` — a
  separate ``all_gather_into_tensor`` after the decode, plus a strided copy
  back into head order (``gather_head_outputs``, also runs over gloo on CPU).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def shard_heads(num_kv_heads: int, world: int, rank: int) -> Tuple[int, int]:
    """KV heads [h0, h1) owned by ``rank`` when heads are split over ``world`` GPUs."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is not in a world of {world}")
    if num_kv_heads % world != 0:
        raise ValueError(f"{num_kv_heads} KV heads cannot be split evenly over {world} GPUs")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def q_heads_for(num_heads: int, num_kv_heads: int, kv_range: Tuple[int, int]) -> Tuple[int, int]:
    """q-heads [q0, q1) that read KV heads [h0, h1): q-head h reads KV head
    h // (num_heads / num_kv_heads) (the GQA grouping of attention.hip:54)."""
    if num_heads % num_kv_heads != 0:
        raise ValueError("num_heads must be a multiple of num_kv_heads")
    group = num_heads // num_kv_heads
    return kv_range[0] * group, kv_range[1] * group


def shard_sequences(num_seqs: int, world: int, rank: int) -> Tuple[int, int]:
    """Sequences [s0, s1) owned by ``rank``: contiguous, sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is not in a world of {world}")
    base, extra = divmod(num_seqs, world)
    s0 = rank * base + min(rank, extra)
    return s0, s0 + base + (1 if rank < extra else 0)


def gather_head_outputs(local_out: torch.Tensor, out: torch.Tensor,
                        stage: Optional[torch.Tensor] = None, group=None) -> torch.Tensor:
    """All-gather every rank's per-head outputs into ``out``.

    ``local_out`` is this rank's [B, Hq_local, D] slice (its q-heads, in order);
    ``out`` receives [B, world * Hq_local, D] with rank r's heads at
    [r * Hq_local, (r + 1) * Hq_local), the order of the unsharded result.  The
    collective gathers rank-major into ``stage`` ([world, B, Hq_local, D],
    allocated when not given) and one strided copy puts the heads in place.
    """
    world = dist.get_world_size(group)
    B, hl, D = local_out.shape
    if out.shape != (B, world * hl, D):
        raise ValueError(f"out has shape {tuple(out.shape)}, expected {(B, world * hl, D)}")
    if stage is None:
        stage = torch.empty((world, B, hl, D), dtype=local_out.dtype, device=local_out.device)
    dist.all_gather_into_tensor(stage.view(world * B, hl, D), local_out.contiguous(), group=group)
    out.view(B, world, hl, D).copy_(stage.transpose(0, 1))
    return out


class _DeviceArray:
    """Zero-copy ``__cuda_array_interface__`` wrapper of a library-owned buffer."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3,
                                         "strides": None}


class HeadExchange:
    """This rank's exchange buffer for the ``"p2p"`` transport (kvc_xchg_*).

    ``n_slots`` output slots of shape ``(num_queries, total_heads, head_dim)``;
    the other ranks' merge kernels write their heads into them over NVLink.
    Creating it is collective: the ranks swap CUDA IPC handles over ``group``.
    """

    def __init__(self, device: int, num_queries: int, total_heads: int, head_dim: int,
                 dtype: torch.dtype = torch.float16, n_slots: int = 2, group=None):
        import ctypes

        import kvcache_ffi as ffi

        self._ffi = ffi
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device
        self.shape = (num_queries, total_heads, head_dim)
        self.dtype = dtype
        self.n_slots = n_slots
        es = torch.empty((), dtype=dtype).element_size()
        h = ctypes.c_void_p()
        ffi.check(ffi.lib.kvc_xchg_create(device, self.rank, self.world,
                                          num_queries * total_heads * head_dim * es, n_slots,
                                          ctypes.byref(h)))
        self.handle = h
        try:
            raw = (ctypes.c_uint8 * ffi.XCHG_HANDLE_BYTES)()
            ffi.check(ffi.lib.kvc_xchg_handle(h, raw))
            dev = torch.device("cuda", device) if dist.get_backend(group) == "nccl" else "cpu"
            mine = torch.tensor(list(bytes(raw)), dtype=torch.uint8, device=dev)
            every = torch.empty(self.world * ffi.XCHG_HANDLE_BYTES, dtype=torch.uint8, device=dev)
            dist.all_gather_into_tensor(every, mine, group=group)
            blob = bytes(every.cpu().numpy().tobytes())
            ffi.check(ffi.lib.kvc_xchg_connect(h, blob))
            dist.barrier(group=group)  # every rank mapped before anyone writes
        except Exception:
            ffi.lib.kvc_xchg_destroy(h)
            self.handle = None
            raise
        self._views = []
        for i in range(n_slots):
            ptr = ctypes.c_void_p()
            ffi.check(ffi.lib.kvc_xchg_slot(h, i, ctypes.byref(ptr)))
            arr = _DeviceArray(ptr.value, self.shape, "<f2")
            self._views.append(torch.as_tensor(arr, device=torch.device("cuda", device))
                               .view(dtype))

    def slot(self, i: int) -> torch.Tensor:
        """Slot ``i`` as a (num_queries, total_heads, head_dim) tensor (no copy)."""
        return self._views[i]

    def set_wait_limit(self, seconds: float) -> None:
        self._ffi.check(self._ffi.lib.kvc_xchg_set_wait_limit(self.handle, float(seconds)))

    def close(self) -> None:
        """Collective: every rank stops writing before any buffer is freed."""
        if self.handle is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._views = []
        self._ffi.lib.kvc_xchg_destroy(self.handle)
        self.handle = None


class HeadShardedDecode:
    """Decode step of one layer with KV heads split across the process group.

    ``pool`` is this rank's ``paged.PagedKVCache`` built with the rank's
    ``num_kv_heads`` slice; ``plan`` was made with the rank's q-head count.
    ``append_decode`` takes this rank's q-heads and new K/V rows, runs the fused
    append + attention kernel and returns all heads of every sequence,
    (B, num_heads, D), on every rank.

    transport ``"p2p"``: outputs arrive in the exchange slots (one fused launch
    chain, no collective call); the returned tensor is slot ``call % n_slots``,
    valid until the same slot comes round again.  ``"nccl"``: all-gather + copy
    into ``out`` (or an internal buffer).
    """

    def __init__(self, pool, num_heads: int, num_kv_heads: int, group=None,
                 transport: str = "p2p", num_queries: Optional[int] = None, n_slots: int = 2):
        if transport not in ("p2p", "nccl"):
            raise ValueError(f"unknown transport {transport!r}")
        self.pool = pool
        self.group = group
        self.transport = transport
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.num_heads = num_heads
        self.kv_range = shard_heads(num_kv_heads, self.world, self.rank)
        self.q_range = q_heads_for(num_heads, num_kv_heads, self.kv_range)
        if pool.num_kv_heads != self.kv_range[1] - self.kv_range[0]:
            raise ValueError(f"pool holds {pool.num_kv_heads} KV heads, this rank owns "
                             f"{self.kv_range[1] - self.kv_range[0]}")
        self.exchange = None
        self._calls = 0
        if transport == "p2p":
            if num_queries is None:
                raise ValueError("the p2p transport needs num_queries to size its slots")
            self.exchange = HeadExchange(pool.device, num_queries, num_heads, pool.head_dim,
                                         pool.dtype, n_slots, group)
        self._local = None
        self._stage = None

    def _buffers(self, q: torch.Tensor):
        B, hl, D = q.shape
        if self._local is None or self._local.shape != q.shape or self._local.device != q.device:
            self._local = torch.empty_like(q)
            self._stage = torch.empty((self.world, B, hl, D), dtype=q.dtype, device=q.device)
        return self._local, self._stage

    def append_decode(self, plan, layer: int, q_local: torch.Tensor, k_new: torch.Tensor,
                      v_new: torch.Tensor, out: Optional[torch.Tensor], block_tables: torch.Tensor,
                      scale: float, stream=None, slot: Optional[int] = None) -> torch.Tensor:
        if self.transport == "p2p":
            x = self.exchange
            if slot is None:
                slot = self._calls % x.n_slots
            self._calls += 1
            self.pool.append_decode_xchg(plan, layer, q_local, k_new, v_new, x.handle, slot,
                                         self.num_heads, self.q_range[0], block_tables, scale,
                                         stream=stream)
            res = x.slot(slot)[: q_local.shape[0]]
            if out is None:
                return res
            if stream is None:
                return out.copy_(res)
            with torch.cuda.stream(stream):
                return out.copy_(res)
        local, stage = self._buffers(q_local)
        if out is None:
            out = torch.empty((q_local.shape[0], self.num_heads, q_local.shape[2]),
                              dtype=q_local.dtype, device=q_local.device)
        self.pool.append_decode(plan, layer, q_local, k_new, v_new, local, block_tables, scale,
                                stream=stream)
        if stream is None:
            return gather_head_outputs(local, out, stage, self.group)
        with torch.cuda.stream(stream):  # the collective queues behind the kernel
            return gather_head_outputs(local, out, stage, self.group)

    def close(self) -> None:
        if self.exchange is not None:
            self.exchange.close()
            self.exchange = None
