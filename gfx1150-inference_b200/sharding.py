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
  per-head outputs are all-gathered once per layer (strong scaling: total
  work fixed, per-GPU KV shrinks with the number of GPUs).

Only process-group plumbing lives here; the attention itself is the CUDA path
of ``paged.PagedKVCache``.  The helpers take plain tensors so the same code runs
over NCCL on GPUs and over gloo on CPU.
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


class HeadShardedDecode:
    """Decode step of one layer with KV heads split across the process group.

    ``pool`` is this rank's ``paged.PagedKVCache`` built with the rank's
    ``num_kv_heads`` slice; ``plan`` was made with the rank's q-head count.
    ``append_decode`` takes this rank's q-heads and new K/V rows, runs the fused
    append + attention kernel, and leaves all heads of every sequence in ``out``
    on every rank.
    """

    def __init__(self, pool, num_heads: int, num_kv_heads: int, group=None):
        self.pool = pool
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.kv_range = shard_heads(num_kv_heads, self.world, self.rank)
        self.q_range = q_heads_for(num_heads, num_kv_heads, self.kv_range)
        if pool.num_kv_heads != self.kv_range[1] - self.kv_range[0]:
            raise ValueError(f"pool holds {pool.num_kv_heads} KV heads, this rank owns "
                             f"{self.kv_range[1] - self.kv_range[0]}")
        self._local = None
        self._stage = None

    def _buffers(self, q: torch.Tensor):
        B, hl, D = q.shape
        if self._local is None or self._local.shape != q.shape or self._local.device != q.device:
            self._local = torch.empty_like(q)
            self._stage = torch.empty((self.world, B, hl, D), dtype=q.dtype, device=q.device)
        return self._local, self._stage

    def append_decode(self, plan, layer: int, q_local: torch.Tensor, k_new: torch.Tensor,
                      v_new: torch.Tensor, out: torch.Tensor, block_tables: torch.Tensor,
                      scale: float, stream=None) -> torch.Tensor:
        local, stage = self._buffers(q_local)
        self.pool.append_decode(plan, layer, q_local, k_new, v_new, local, block_tables, scale,
                                stream=stream)
        if stream is None:
            return gather_head_outputs(local, out, stage, self.group)
        with torch.cuda.stream(stream):  # the collective queues behind the kernel
            return gather_head_outputs(local, out, stage, self.group)
