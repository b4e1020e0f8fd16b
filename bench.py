"""Benchmark of the B200 KV-cache decode path (append + split-K GQA attention).

Default workload (N=1 and the scaling run): benchmark config 3, Llama-3-8B
geometry batched decode — 32 layers, 32 q-heads, 8 KV heads, head_dim 128,
32 sequences per GPU with cached lengths drawn U[1024, 8192] from a seed, one
appended token each, fp16 paged pool of 16-token pages in a random page
permutation, N(0,1) K/V/q.  A step is one decode step over all 32 layers:
per layer, append each sequence's new K/V row and attend over its whole
context.  Multi-GPU: one process per GPU, each with its own 32 sequences
(sequences are independent; no collective in the data path) -> weak scaling.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
                  [--config 3|2|4]

Prints one JSON line (rank 0).  ``value`` is the whole-job algorithmic HBM
throughput in GB/s (KV bytes read + appended rows written + q read + out
written, per step, summed over ranks, divided by the max-over-ranks device
time); ``e2e`` is the same metric through the reference-facing host-buffer
call (kvc_decode_host: H2D of q and the new rows, append, attend, D2H, wait —
per layer, like gqa_attention_cached).  ``--impl reference`` times the
reference algorithm's CPU restatement (oracle/gqa_online.c, OpenMP on all host
cores) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "gfx1150-inference_b200"))

METRIC = "decode-attn+append HBM GB/s (% of ~8 TB/s) and decode steps/s at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0

CONFIGS = {
    # name: layers, q-heads, kv-heads, head_dim, batch per GPU, ctx generator
    "3": dict(workload="llama3-8b-batched-decode", layers=32, H=32, Hkv=8, D=128, batch=32,
              lens=("uniform", 1024, 8192), seed=2024),
    "2": dict(workload="llama2-7b-decode-4k", layers=32, H=32, Hkv=32, D=128, batch=1,
              lens=("fixed", 4095), seed=2),
    "4": dict(workload="llama3-70b-long-context-decode", layers=80, H=64, Hkv=8, D=128, batch=8,
              lens=("fixed", 32768), seed=4),
    "5": dict(workload="llama3-70b-offload-kv-cpu", layers=80, H=64, Hkv=8, D=128, batch=1,
              lens=("fixed", 131072), seed=5),
}
PAGE = 16
ROPE_BASE = 500000.0  # Llama-3 rope_freq_base (only with --rope)


def cached_lengths(cfg):
    kind = cfg["lens"][0]
    if kind == "fixed":
        return np.full(cfg["batch"], cfg["lens"][1], dtype=np.int64)
    rng = np.random.default_rng(cfg["seed"])
    return rng.integers(cfg["lens"][1], cfg["lens"][2] + 1, size=cfg["batch"]).astype(np.int64)


def step_bytes(cfg, ctx):
    """Algorithmic bytes of one decode step (all layers), fp16."""
    es = 2
    L, H, Hkv, D = cfg["layers"], cfg["H"], cfg["Hkv"], cfg["D"]
    kv_read = int(ctx.sum()) * Hkv * D * es * 2 * L
    appended = len(ctx) * Hkv * D * es * 2 * L
    qo = len(ctx) * H * D * es * 2 * L
    return kv_read, appended, qo


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------------------------
# clocks sampling (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------------
class ClockSampler:
    """SM clock and clock-event reasons of one GPU, sampled every 20 ms by a
    thread while the timed region runs (read-only NVML queries; nvidia-smi
    polling when NVML is unavailable)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, gpu_index: int, interval_s: float = 0.02):
        self.gpu = gpu_index
        self.interval = interval_s
        self.samples = []   # (sm_mhz, reasons bitmask)
        self.sm_max = 0.0
        self._stop = threading.Event()
        self.thread = None
        self.proc = None

    def start(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            h = self._nvml_handle(pynvml)
            self.sm_max = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))

            def loop():
                while not self._stop.is_set():
                    try:
                        mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((float(mhz), int(rs)))
                    except Exception:
                        pass
                    self._stop.wait(self.interval)

            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
        except Exception:
            self._start_smi()

    def _nvml_handle(self, pynvml):
        """NVML handle of the CUDA device (matched by PCI address, since NVML
        numbers every GPU of the machine, not only the visible ones)."""
        try:
            import torch

            p = torch.cuda.get_device_properties(self.gpu)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.gpu)

    def _start_smi(self):
        fields = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                  "clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={fields}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        bits = [0x8, 0x40, 0x20, 0x4]

        def read():
            for line in self.proc.stdout:
                parts = [x.strip() for x in line.split(",")]
                try:
                    mask = sum(b for b, v in zip(bits, parts[2:6]) if v.lower() == "active")
                    self.samples.append((float(parts[0]), mask))
                    self.sm_max = max(self.sm_max, float(parts[1]))
                except (ValueError, IndexError):
                    continue

        self.thread = threading.Thread(target=read, daemon=True)
        self.thread.start()

    def stop(self):
        self._stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        if not self.samples:
            return None
        reasons = sorted(n for n, b in self.REASONS.items()
                         if any(m & b for _, m in self.samples))
        return {"sm_mhz": statistics.median(s for s, _ in self.samples),
                "sm_max_mhz": self.sm_max, "reasons": reasons, "samples": len(self.samples)}


# ---------------------------------------------------------------------------------
# CPU baseline: reference algorithm (C restatement, OpenMP) on a bounded sample
# ---------------------------------------------------------------------------------
class CpuWorkload:
    """One layer of the workload in host memory for the reference algorithm's
    C restatement (oracle/gqa_online.c, OpenMP over (sequence, q-head))."""

    def __init__(self, cfg, ctx, threads=None):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import build_oracle  # test infrastructure: the CPU baseline leg only

        self.lib = build_oracle.load()
        self.threads = threads or os.cpu_count() or 1
        self.H, self.Hkv, self.D = cfg["H"], cfg["Hkv"], cfg["D"]
        self.n = len(ctx)
        rng = np.random.default_rng(cfg["seed"] + 99)
        block = rng.standard_normal(1 << 22, dtype=np.float32).astype(np.float16)
        self.ks, self.vs = [], []
        for c in ctx:
            m = int(c) * self.Hkv * self.D
            self.ks.append(np.resize(block, m).reshape(int(c), self.Hkv, self.D))
            self.vs.append(np.resize(block[::-1], m).reshape(int(c), self.Hkv, self.D))
        self.q = rng.standard_normal((self.n, self.H, self.D), dtype=np.float32).astype(np.float16)
        self.out = np.empty_like(self.q)
        self.kp = (ctypes.c_void_p * self.n)(*[k.ctypes.data for k in self.ks])
        self.vp = (ctypes.c_void_p * self.n)(*[v.ctypes.data for v in self.vs])
        self.cp = (ctypes.c_int * self.n)(*[int(c) for c in ctx])
        self.scale = 1.0 / math.sqrt(self.D)
        self.layer_bytes = (int(ctx.sum()) * self.Hkv * self.D * 2 * 2
                            + self.n * self.H * self.D * 2 * 2)

    def run_layer(self) -> float:
        t0 = time.perf_counter()
        rc = self.lib.gqa_decode_batch_f16(self.n, self.q.ctypes.data, self.kp, self.vp, self.cp,
                                           self.out.ctypes.data, self.H, self.Hkv, self.D,
                                           self.scale, self.threads)
        if rc != 0:
            raise RuntimeError("CPU baseline rejected its arguments")
        return time.perf_counter() - t0


def blas_threads() -> int:
    """Threads numpy's BLAS may use (the numpy path's matrix-vector products)."""
    try:
        from threadpoolctl import threadpool_info

        n = [d.get("num_threads", 1) for d in threadpool_info() if d.get("user_api") == "blas"]
        return int(max(n)) if n else 1
    except Exception:
        return 1


def numpy_path_sample(w, min_seconds=5.0):
    """The reference's numpy path for this step: per sequence, the host append
    (KVCacheManager's slice assignment, src/kv_cache.py:222-225) and
    ref_gqa_attention (tests/test_layer.py:76-105) over its whole context, as
    oracle/gqa_ref.py restates them; sequences of one layer in turn until
    min_seconds.  Returns (GB/s, seconds, sequences timed)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import gqa_ref  # test infrastructure: the CPU baseline leg only

    nbytes, total, done = 0, 0.0, 0
    while total < min_seconds:
        i = done % w.n
        k, v = w.ks[i], w.vs[i]
        ctx = k.shape[0]
        t0 = time.perf_counter()
        k[ctx - 1] = w.q[i, :w.Hkv]  # the appended row (host append of the new token)
        v[ctx - 1] = w.q[i, :w.Hkv]
        gqa_ref.ref_gqa_attention(w.q[i:i + 1], k, v, start_pos=ctx - 1, scale=w.scale)
        total += time.perf_counter() - t0
        nbytes += ctx * w.Hkv * w.D * 2 * 2 + w.H * w.D * 2 * 2
        done += 1
    return nbytes / total / 1e9, total, done


def cpu_sample(cfg, ctx, min_seconds=10.0, max_reps=50):
    """Time one layer of the workload (all sequences) on the host cores, repeated
    until min_seconds.  Returns (GB/s, seconds per layer, threads, reps)."""
    w = CpuWorkload(cfg, ctx)
    w.run_layer()  # warm-up
    reps, total = 0, 0.0
    while reps < max_reps:
        total += w.run_layer()
        reps += 1
        if total >= min_seconds:
            break
    dt = total / reps
    return w.layer_bytes / dt / 1e9, dt, w.threads, reps


# ---------------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------------
class DecodeWorkload:
    """One benchmark configuration (2, 3 or 4) set up on this rank's GPU, and its
    decode step: per layer, append each sequence's new K/V row at its last
    position and attend over the whole context (one fused launch + split merge).

    shard "seq": this rank holds its own ``batch`` sequences, all KV heads (no
    collective).  shard "heads" with world > 1: KV heads [r*Hkv/N, (r+1)*Hkv/N)
    of every sequence and their q-heads; each layer's outputs are exchanged
    (``xchg`` "p2p": the merge kernel stores them into every rank's exchange slot
    over NVLink; "nccl": all-gather).  ``one_rank_of`` > 1 on one GPU: rank 0's
    shard of that split with its exchange connected to itself (profiling).
    ``grow_extra`` positions per sequence are paged in for growing decode loops.
    Contents: seeded N(0,1) pages, q and new rows."""

    def __init__(self, config="3", layers=0, rank=0, world=1, local_rank=0, shard="seq",
                 xchg="p2p", page_size=PAGE, grow_extra=0, rope=False, one_rank_of=0,
                 kv_stable=True, graph_plan=True):
        import torch

        import kvcache_ffi as ffi
        import paged

        self.torch, self.ffi = torch, ffi
        dev = torch.device("cuda", local_rank)
        self.dev, self.local_rank, self.rank, self.world = dev, local_rank, rank, world
        cfg = dict(CONFIGS[config])
        if layers:
            cfg["layers"] = layers  # profiling / test subset (the bench line names it)
        self.cfg, self.config = cfg, config
        L, H, Hkv, D, B = cfg["layers"], cfg["H"], cfg["Hkv"], cfg["D"], cfg["batch"]
        self.H_full, self.Hkv_full = H, Hkv
        self.shard = shard if world > 1 else "seq"
        self.xchg = xchg
        self.head_offset = 0
        if self.shard == "heads":
            h0, h1 = paged.shard_heads(Hkv, world, rank)
            self.head_offset = h0 * (H // Hkv)
            Hkv = h1 - h0
            H = H * Hkv // cfg["Hkv"]
        self.one_rank_of = one_rank_of if world == 1 else 0
        if self.one_rank_of > 1:
            h0, h1 = paged.shard_heads(Hkv, self.one_rank_of, 0)
            Hkv = h1 - h0
            H = H * Hkv // cfg["Hkv"]
        self.L, self.H, self.Hkv, self.D, self.B = L, H, Hkv, D, B
        self.page_size = page_size
        self.rope = rope
        cached = cached_lengths(cfg)
        self.ctx = cached + 1                           # context includes the appended token
        table, self.total_pages = paged.random_block_tables(self.ctx + grow_extra, page_size,
                                                            cfg["seed"] + 17 * rank)
        self.grow_extra = grow_extra
        self.pool = paged.PagedKVCache(L, self.total_pages, page_size, Hkv, D,
                                       dtype=torch.float16, device=local_rank)
        self.pool.fill_normal(seed=1000 + rank, stddev=1.0)
        self.bt = torch.from_numpy(table).to(dev)
        g = torch.Generator(device=dev)
        g.manual_seed(7 + rank)
        self.q = torch.randn((L, B, H, D), generator=g, device=dev, dtype=torch.float32).half()
        self.kn = torch.randn((L, B, Hkv, D), generator=g, device=dev, dtype=torch.float32).half()
        self.vn = torch.randn((L, B, Hkv, D), generator=g, device=dev, dtype=torch.float32).half()
        self.out = torch.empty_like(self.q)
        self.gathered = None
        self.hsd = None
        if self.shard == "heads":
            import sharding

            # every rank ends each layer with all heads of every sequence
            self.hsd = sharding.HeadShardedDecode(self.pool, self.H_full, self.Hkv_full,
                                                  transport=xchg, num_queries=B)
            if xchg == "nccl":
                self.gathered = torch.empty((L, B, self.H_full, D), dtype=torch.float16,
                                            device=dev)
        self.self_xchg = None
        if self.one_rank_of > 1:
            import ctypes

            self.self_xchg = ctypes.c_void_p()
            ffi.check(ffi.lib.kvc_xchg_create(local_rank, 0, 1, B * self.H_full * D * 2, 2,
                                              ctypes.byref(self.self_xchg)))
            base = ctypes.c_void_p()
            ffi.check(ffi.lib.kvc_xchg_base(self.self_xchg, ctypes.byref(base)))
            ffi.check(ffi.lib.kvc_xchg_connect_ptrs(self.self_xchg,
                                                    (ctypes.c_void_p * 1)(base.value)))
        self.scale = 1.0 / math.sqrt(D)
        self.stream = torch.cuda.current_stream()
        self.grown = 0
        # block tables are static and pages are written only by the decode kernels
        # themselves, so each launch may start streaming KV before the previous one ends;
        # graph-stable: the step's launches are captured once and replayed after each
        # rebuild of the plan for grown contexts (re-captured when its layout moves)
        self.plan = paged.DecodePlan()
        self.plan.set_kv_stable(kv_stable)
        self.plan.set_graph_stable(graph_plan)
        if graph_plan and grow_extra:
            # a serving loop reserves for the longest contexts it will reach: one build
            # at those sizes the plan's block and scratch, so the rebuilds of the
            # growing loop keep the captured launches' addresses
            self.pool.plan(self.ctx + grow_extra, H, plan=self.plan, stream=self.stream)
        self.pool.plan(self.ctx, H, plan=self.plan, stream=self.stream)
        self.step_graph = None
        self.step_graph_gen = -1
        self.captures = 0
        # The step loop calls the C ABI with its pointer arguments prepared once (the
        # tensors above never move), as a native caller would: the per-layer checks of
        # the Python wrappers would otherwise bound the loop on small shards.
        self.layer_ptrs = [(int(self.q[l].data_ptr()), int(self.kn[l].data_ptr()),
                            int(self.vn[l].data_ptr()), int(self.out[l].data_ptr()))
                           for l in range(L)]
        self.bt_args = (int(self.bt.data_ptr()), int(self.bt.shape[-1]))
        torch.cuda.synchronize()

    @property
    def p2p(self) -> bool:
        return (self.hsd is not None and self.xchg == "p2p") or self.self_xchg is not None

    def launches_per_step(self) -> int:
        return (3 if self.p2p or (self.rope and self.hsd is None) else 2) * self.L

    def current_ctx(self):
        return self.ctx + self.grown

    def restart_growth(self):
        """Contexts back to the configured lengths: the next growing step decodes
        position ctx again (the rows appended past it are never read)."""
        self.grown = 0

    def step(self, s=None, grow=False, events=None, results=None):
        """One decode step over all layers on stream ``s``.  grow: the contexts grow
        by one position first (a new plan on the host, then the layers).  results:
        a dict that receives layer -> a copy of that layer's (all-heads) output."""
        s = self.stream if s is None else s
        sp = int(s.cuda_stream) or None
        if grow:
            if self.grown >= self.grow_extra:
                raise RuntimeError("the workload was set up for fewer growing steps")
            self.grown += 1
            self.pool.plan(self.ctx + self.grown, self.H, plan=self.plan, stream=s)
        for l in range(self.L):
            if events is not None:
                events[l][0].record(s)
            res = self.out[l]
            if self.self_xchg is not None:
                self.pool.append_decode_xchg(self.plan, l, self.q[l], self.kn[l], self.vn[l],
                                             self.self_xchg, l & 1, self.H_full, 0, self.bt,
                                             self.scale, stream=s)
            elif self.hsd is None and self.rope:
                # rotate q and the new K row (RoPE at each sequence's position) first
                self.pool.append_decode_rope(self.plan, l, self.q[l], self.kn[l], self.vn[l],
                                             self.out[l], self.bt, self.scale, ROPE_BASE, False,
                                             stream=s)
            elif self.hsd is None:
                qp, kp, vp, op = self.layer_ptrs[l]
                rc = self.ffi.lib.kvc_append_decode(self.pool.handle, self.plan.handle, l, qp, kp,
                                                    vp, op, *self.bt_args, self.scale, sp)
                if rc:
                    self.ffi.check(rc)
            elif self.xchg == "p2p":
                # the merge kernel pushes this rank's heads into every rank's slot
                # (the same calls HeadShardedDecode.append_decode makes)
                hx = self.hsd.exchange
                slot = self.hsd._calls % hx.n_slots
                self.hsd._calls += 1
                qp, kp, vp, _ = self.layer_ptrs[l]
                rc = self.ffi.lib.kvc_append_decode_xchg(
                    self.pool.handle, self.plan.handle, l, qp, kp, vp, hx.handle, slot,
                    self.H_full, self.head_offset, *self.bt_args, self.scale, sp)
                if rc:
                    self.ffi.check(rc)
                if results is not None:
                    res = hx.slot(slot)[: self.B]
            else:
                # fused append + attention on this rank's heads; p2p: the merge kernel
                # pushes the heads to every rank (result in an exchange slot), nccl:
                # all-gather + copy into gathered[l]
                res = self.hsd.append_decode(
                    self.plan, l, self.q[l], self.kn[l], self.vn[l],
                    self.gathered[l] if self.xchg == "nccl" else None, self.bt, self.scale,
                    stream=s)
            if events is not None:
                events[l][1].record(s)
            if results is not None and self.self_xchg is None:
                with self.torch.cuda.stream(s):
                    results[l] = res.clone()

    def step_graphed(self):
        """One step of the growing decode loop as a serving loop runs it: the plan is
        rebuilt on the host for contexts one position longer, then the step's
        launches are replayed from a CUDA graph (captured again only when the
        plan's layout generation moved)."""
        torch = self.torch
        if self.grown >= self.grow_extra:
            raise RuntimeError("the workload was set up for fewer growing steps")
        self.grown += 1
        self.pool.plan(self.ctx + self.grown, self.H, plan=self.plan, stream=self.stream)
        gen = self.plan.generation
        if self.step_graph is None or gen != self.step_graph_gen:
            if self.step_graph is not None:
                self.step_graph.reset()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.step(s=torch.cuda.current_stream())
            self.step_graph, self.step_graph_gen = g, gen
            self.captures += 1
        self.step_graph.replay()

    def release_graph(self):
        if self.step_graph is not None:
            self.step_graph.reset()
            self.step_graph = None

    def step_bytes(self, ctx=None):
        """Algorithmic bytes of one step on this rank: (KV read, appended, q + out)."""
        return step_bytes(dict(self.cfg, H=self.H, Hkv=self.Hkv),
                          self.current_ctx() if ctx is None else ctx)

    def close(self):
        self.release_graph()
        if self.hsd is not None:
            self.hsd.close()  # collective: exchange buffers freed after every rank is done
            self.hsd = None
        if self.self_xchg is not None:
            self.torch.cuda.synchronize()
            self.ffi.lib.kvc_xchg_destroy(self.self_xchg)
            self.self_xchg = None
        self.plan.close()
        self.pool.close()


def _max_over_ranks(x, world, dev):
    if world == 1:
        return x
    import torch

    t = torch.tensor([x], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(x, world, dev):
    if world == 1:
        return x
    import torch

    t = torch.tensor([x], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.SUM)
    return float(t.item())


def timed_passes(wl, steps, passes, grow=False, graph=None, events=None, graphed=False):
    """``passes`` timed passes of exactly ``steps`` steps each, every pass
    bracketed by a barrier and a device synchronisation, timed with CUDA events
    on the launching stream.  grow: contexts grow by one position per step (the
    plan rebuilt every step), the step's launches replayed from a graph when
    ``graphed``.  Returns [(ms, bytes of the pass on this rank)]."""
    torch = wl.torch
    out = []
    for p in range(passes):
        parts = []
        if grow:
            # every pass decodes the same positions past the configured contexts, so
            # the workload does not drift from the config over many passes
            wl.restart_growth()
        if wl.world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(wl.stream)
        for i in range(steps):
            if graph is not None:
                graph.replay()
            elif grow and graphed:
                wl.step_graphed()
            else:
                wl.step(grow=grow, events=events[i] if events else None)
            if grow:
                parts.append(sum(wl.step_bytes()))
        t1.record(wl.stream)
        torch.cuda.synchronize()
        if wl.world > 1:
            torch.distributed.barrier()
        nbytes = sum(parts) if grow else steps * sum(wl.step_bytes())
        out.append((t0.elapsed_time(t1), nbytes))
    return out


def _check_device(wl, what):
    code, info = wl.ffi.device_error(wl.local_rank)
    if code:
        raise RuntimeError(f"device error {code} ({info}) {what}")


def _pass_figures(wl, passes_res):
    """The median pass by throughput: (ms of the pass, max over ranks; bytes of the
    pass summed over ranks; this rank's bytes of the pass)."""
    figs = []
    for ms, nb in passes_res:
        figs.append((_max_over_ranks(ms, wl.world, wl.dev),
                     _sum_over_ranks(float(nb), wl.world, wl.dev), float(nb)))
    figs.sort(key=lambda f: f[1] / f[0], reverse=True)
    return figs[len(figs) // 2]


def exchange_parity(wl, layers=None):
    """Head-sharded runs: run one step directly, keep the exchanged (all-heads)
    outputs of a few layers, and compare them with this rank's own heads decoded
    without the exchange (kvc_decode on the same pool and plan), all-gathered over
    NCCL.  True on every rank when each layer agrees within the fp16 bound."""
    torch = wl.torch
    import sharding

    layers = layers or sorted({0, wl.L // 2, wl.L - 1})
    got = {}
    wl.step(results=got)
    torch.cuda.synchronize()
    _check_device(wl, "in the exchange check")
    worst = 0.0
    for l in layers:
        loc = torch.empty_like(wl.q[l])
        wl.pool.decode(wl.plan, l, wl.q[l], loc, wl.bt, wl.scale)
        full = torch.empty((wl.B, wl.H_full, wl.D), dtype=loc.dtype, device=loc.device)
        sharding.gather_head_outputs(loc, full)
        ref = full.float()
        d = (got[l].float() - ref).abs().amax(dim=(1, 2))
        m = ref.abs().amax(dim=(1, 2)).clamp_min(1e-30)
        worst = max(worst, float((d / m).max().item()))
    worst = _max_over_ranks(worst, wl.world, wl.dev)
    return worst <= 2e-3, worst


def run_b200(args, rank, world, local_rank):
    import torch

    import kvcache_ffi as ffi

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    shard = args.shard or ("heads" if world > 1 or args.config == "4" else "seq")
    cfg0 = dict(CONFIGS[args.config])
    if args.layers:
        cfg0["layers"] = args.layers
    # upper bound of the timed passes (each pass >= its bytes at 7 TB/s per GPU), so
    # the growing loop's pages can be laid out before anything runs
    ctx0 = cached_lengths(cfg0) + 1
    t_min = (sum(step_bytes(cfg0, ctx0)) / max(1, world if shard == "heads" else 1)
             / max(1, args.one_rank_of if world == 1 else 1) / 7.0e12)
    max_passes = max(1, min(args.max_passes,
                            math.ceil(args.min_timed_s / max(1e-6, args.steps * t_min)) + 1))
    grow_steps = (max(args.warmup, args.steps) + 2) if not args.no_grow else 0
    wl = DecodeWorkload(args.config, layers=args.layers, rank=rank, world=world,
                        local_rank=local_rank, shard=shard, xchg=args.xchg,
                        page_size=args.page_size, grow_extra=grow_steps, rope=args.rope,
                        one_rank_of=args.one_rank_of)
    L = wl.L
    sampler = ClockSampler(local_rank) if not args.no_clocks else None

    # ---- fixed step: the same step replayed (one CUDA graph per step) ----
    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize()
    _check_device(wl, "during warm-up")
    graph = None
    if not args.no_graph and not args.launch_events:
        # The step's launches are recorded once into a CUDA graph and replayed: the
        # same kernels, without the host's per-launch cost between them.
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            wl.step(s=torch.cuda.current_stream())
        graph.replay()  # one untimed replay
        torch.cuda.synchronize()
        _check_device(wl, "in the captured step")
    evs = ([[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(L)]
            for _ in range(args.steps)] if args.launch_events else None)
    # calibrate: one pass, then as many passes as fill min_timed_s
    first = timed_passes(wl, args.steps, 1, graph=graph, events=evs)
    pass_ms = _max_over_ranks(first[0][0], world, dev)
    passes = max(1, min(max_passes, math.ceil(args.min_timed_s * 1e3 / max(pass_ms, 1e-3))))
    if sampler:
        sampler.start()
    fixed_res = timed_passes(wl, args.steps, passes, graph=graph, events=evs)
    fixed_clocks = sampler.stop() if sampler else None
    _check_device(wl, "during timing")
    if graph is not None:
        graph.reset()  # released before any collective teardown (it may hold NCCL calls)
        graph = None
    f_ms, f_bytes, f_local = _pass_figures(wl, fixed_res)
    fixed = {"value": round(f_bytes / (f_ms / 1e3) / 1e9, 1),
             "ms_per_step": round(f_ms / args.steps, 4), "passes": passes,
             "launch": ("one CUDA graph replay per step (the step's launches)"
                        if not args.no_graph and not args.launch_events
                        else "direct launches from the host loop")}
    dec_ms = ([evs[i][l][0].elapsed_time(evs[i][l][1]) for i in range(args.steps)
               for l in range(L)] if evs else None)
    kv_read = wl.step_bytes()[0]
    # roofline of the dominant kernel: this rank's bytes per decode launch (one layer)
    # over the launch's average duration in the headline measurement
    dec_bytes = f_local / (args.steps * L)
    dec_avg_ms = float(np.mean(dec_ms)) if dec_ms else f_ms / (args.steps * L)
    dec_from = ("per-launch CUDA events" if dec_ms else
                "CUDA events around the fixed-step timed passes / launches (launches overlap)")

    # ---- growing decode loop: contexts +1 per step, plan rebuilt every step ----
    grow = None
    clocks = fixed_clocks
    if not args.no_grow:
        graphed = not args.no_graph and not args.launch_events
        for _ in range(args.warmup):
            if graphed:
                wl.step_graphed()
            else:
                wl.step(grow=True)
        torch.cuda.synchronize()
        _check_device(wl, "during the growing loop's warm-up")
        captures0 = wl.captures
        sampler = ClockSampler(local_rank) if not args.no_clocks else None
        if sampler:
            sampler.start()
        grow_res = timed_passes(wl, args.steps, passes, grow=True, graphed=graphed)
        clocks = sampler.stop() if sampler else fixed_clocks
        _check_device(wl, "during the growing loop")
        wl.release_graph()  # before any collective teardown (it may hold NCCL calls)
        g_ms, g_bytes, g_local = _pass_figures(wl, grow_res)
        if not dec_ms:
            dec_bytes = g_local / (args.steps * L)
            dec_avg_ms = g_ms / (args.steps * L)
            dec_from = ("CUDA events around the growing loop's timed passes / launches "
                        "(launches overlap)")
        grow = {"value": round(g_bytes / (g_ms / 1e3) / 1e9, 1),
                "ms_per_step": round(g_ms / args.steps, 4), "passes": passes,
                "ctx_tokens_per_gpu_last": int(wl.current_ctx().sum()),
                "launch": ((f"the plan is rebuilt on the host every step inside the timed "
                            f"region, then the step's launches replay from a CUDA graph "
                            f"(graph-stable plan; {wl.captures - captures0} captures in the "
                            f"timed passes, when the plan's layout moved)")
                           if graphed else
                           "direct launches from the host loop; the plan is rebuilt on the "
                           "host every step inside the timed region")}

    # ---- exchange check (head-sharded runs) ----
    xparity = None
    if wl.hsd is not None:
        ok, worst = exchange_parity(wl)
        xparity = {"exchange_parity_ok": bool(ok), "worst_rel_err": worst,
                   "checked": "layers 0, L/2, L-1: exchanged all-heads outputs vs every "
                              "rank's own heads decoded without the exchange, all-gathered"}

    headline = grow if grow is not None else fixed
    value = headline["value"]
    ms_per_step = headline["ms_per_step"]
    # what the line reports about this rank's workload (before any variant replaces it)
    L, H, Hkv, D, B, cfg = wl.L, wl.H, wl.Hkv, wl.D, wl.B, wl.cfg
    info = wl.plan.info()
    launches = wl.launches_per_step() * args.steps * passes * (2 if grow is not None else 1)

    # ---- e2e: reference-facing host-buffer call, per layer, copies inside ----
    e2e = run_e2e(wl, args) if not args.no_e2e else None

    # ---- extra lines of the same run (N > 1): the other sharding / transport ----
    extra = {}
    if world > 1 and wl.hsd is not None and not args.no_variants:
        wl.close()
        wl = None
        torch.cuda.empty_cache()
        for name, kw in (("seq_sharded", dict(shard="seq")),
                         ("heads_nccl", dict(shard="heads", xchg="nccl"))):
            v = DecodeWorkload(args.config, layers=args.layers, rank=rank, world=world,
                               local_rank=local_rank, page_size=args.page_size,
                               **dict(dict(xchg=args.xchg), **kw))
            for _ in range(args.warmup):
                v.step()
            torch.cuda.synchronize()
            _check_device(v, f"during the {name} warm-up")
            g2 = None
            if not args.no_graph:
                g2 = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g2):
                    v.step(s=torch.cuda.current_stream())
                g2.replay()
                torch.cuda.synchronize()
            r = timed_passes(v, args.steps, max(1, passes // 2), graph=g2)
            if g2 is not None:
                g2.reset()
                g2 = None
            ms, nb, _ = _pass_figures(v, r)
            extra[name] = {"value": round(nb / (ms / 1e3) / 1e9, 1),
                           "ms_per_step": round(ms / args.steps, 4),
                           "scaling": "weak" if name == "seq_sharded" else "strong",
                           "what": ("each rank its own 32 sequences, no collective"
                                    if name == "seq_sharded" else
                                    "KV-head split, NCCL all-gather of head outputs per layer "
                                    "+ strided copy")}
            v.close()
            torch.cuda.empty_cache()

    if rank != 0:
        if wl is not None:
            wl.close()
        return None

    peak, peak_kind = load_peaks()
    achieved = dec_bytes / (dec_avg_ms / 1e3) / 1e9
    res = {
        "metric": METRIC,
        "value": value,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "steps_per_s": round(1e3 / ms_per_step, 2),
        "pct_of_peak": round(100.0 * value / (peak * world), 2),
        "higher_is_better": True,
        "scaling": "strong" if shard == "heads" and world > 1 else "weak",
        "vs_baseline": None,
        "dtype": "f16 storage, f32 accumulate",
        "data": "synthetic: seeded N(0,1) K/V/q, random page permutation",
        "config": {
            "workload": f"{cfg['workload']} (benchmark config {args.config})"
                        + (f" [profiling subset: {L} layers]" if args.layers else "")
                        + (f" [profiling: one rank's shard of a {args.one_rank_of}-way KV-head "
                           "split, exchange connected to itself]" if args.one_rank_of > 1 else ""),
            "layers": L, "q_heads": cfg["H"], "kv_heads": cfg["Hkv"], "head_dim": cfg["D"],
            "q_heads_per_gpu": H, "kv_heads_per_gpu": Hkv,
            "sequences_per_gpu": cfg["batch"],
            "global_batch": cfg["batch"] if shard == "heads" else cfg["batch"] * world,
            "cached_len": (f"U[{cfg['lens'][1]},{cfg['lens'][2]}] seed {cfg['seed']}"
                           if cfg["lens"][0] == "uniform" else int(cfg["lens"][1])),
            "ctx_tokens_per_gpu_start": int(ctx0.sum()), "page_size": args.page_size,
            "kv_bytes_read_per_step_per_gpu": kv_read,
            "l2": "inputs larger than L2 (pool >> 126 MB), no flush",
            "rope": bool(args.rope),
            "timed": (f"{passes} passes of exactly {args.steps} steps each, each pass between a "
                      "barrier and a device sync; value = the median pass (max over ranks)"),
            "headline": ("growing decode loop (contexts +1 per step, plan rebuilt every step "
                         "inside the timed region)" if grow is not None else
                         "fixed step replayed"),
            "parallelism": (f"KV-head-sharded x{world} ({Hkv} KV heads per GPU), "
                            + ("NCCL all-gather" if args.xchg == "nccl" else
                               "merge kernel pushes outputs to every rank over NVLink (p2p)")
                            + f", {B * H * D * 2} B of head outputs per GPU per layer"
                            if shard == "heads" and world > 1 else
                            f"one GPU running rank 0's shard of a {args.one_rank_of}-way KV-head "
                            "split (profiling)" if args.one_rank_of > 1 else
                            f"sequence-sharded x{world} (independent batches, no collective)"),
        },
        "fixed_step": fixed,
        "roofline": {
            "bound": "hbm",
            "kernel": "decode_persistent_kernel (append fused) + merge_splits_kernel",
            "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind,
            "unit": "GB/s", "frac": round(achieved / peak, 4),
            "bytes_per_launch": int(dec_bytes), "avg_launch_us": round(dec_avg_ms * 1e3, 2),
            "duration_from": dec_from,
            "traffic": (TRAFFIC_PER_LAUNCH.get(args.config)
                        if (not args.layers and world == 1 and args.page_size == PAGE
                            and args.one_rank_of <= 1) else None),
            "traffic_from": "ncu dram__bytes_read.sum + dram__bytes_write.sum, decode kernel",
        },
        # per layer: the decode kernel and its split merge (PDL); with the p2p head
        # exchange the merge also pushes the outputs and a one-warp kernel
        # publishes and waits for the peers' epochs
        "gpu_launches": launches,
        "plan": {"work_units_per_launch": info.n_ctas, "splits": info.n_items},
    }
    if grow is not None:
        res["grow"] = grow
    if xparity is not None:
        res.update(xparity)
    if extra:
        res["variants"] = extra
    if e2e:
        res["e2e"] = e2e
    if clocks:
        res["clocks"] = clocks
    if not args.no_cpu_baseline and world == 1:
        gbs, dt, thr, reps = cpu_sample(cfg, ctx0, min_seconds=args.cpu_seconds)
        res["cpu_baseline"] = {
            "value": round(gbs, 3), "unit": "GB/s", "cores": thr, "kind": "port",
            "sample": f"1 of {L} layers x {cfg['batch']} sequences, {reps} reps, "
                      f"{dt * 1e3:.1f} ms/layer; oracle/gqa_online.c (reference kernel's "
                      "algorithm, OpenMP)",
            "steps_per_s_extrapolated": round(1.0 / (dt * L), 4),
        }
    if wl is not None:
        wl.close()
    return res


def run_e2e(wl, args):
    """The same metric through the reference-facing host-buffer call: per layer,
    H2D of q and the new rows from pinned host memory, append, attend, D2H of the
    output and a wait (kvc_decode_host, launch_gqa_attention_cached_fp16's
    semantics).  Head-sharded: this rank's inputs in, fused decode + exchange,
    all heads out."""
    torch = wl.torch
    hq = wl.q.cpu().pin_memory()
    hk = wl.kn.cpu().pin_memory()
    hv = wl.vn.cpu().pin_memory()
    ho = torch.empty_like(hq).pin_memory()
    steps = max(1, min(args.steps, args.e2e_steps))
    sharded = wl.hsd is not None
    if sharded:
        hg = torch.empty((wl.L, wl.B, wl.H_full, wl.D), dtype=torch.float16).pin_memory()
        qd, kd, vd = (torch.empty_like(wl.q[0]), torch.empty_like(wl.kn[0]),
                      torch.empty_like(wl.vn[0]))
        od = torch.empty((wl.B, wl.H_full, wl.D), dtype=torch.float16, device=wl.dev)
    # the e2e step runs at the workload's current contexts (a fresh plan)
    wl.pool.plan(wl.current_ctx(), wl.H, plan=wl.plan, stream=wl.stream)
    s = wl.stream
    # the C-ABI call a host application makes per layer (kvc_decode_host), its
    # pointer arguments prepared once like a plugin binding would
    call = wl.ffi.lib.kvc_decode_host
    fixed = (wl.pool.handle, wl.plan.handle)
    per_layer = [(int(hq[l].data_ptr()), int(hk[l].data_ptr()), int(hv[l].data_ptr()),
                  int(ho[l].data_ptr())) for l in range(wl.L)]
    tail = (int(wl.bt.data_ptr()), int(wl.bt.shape[-1]), float(wl.scale),
            int(s.cuda_stream) or None)

    def e2e_step():
        for l in range(wl.L):
            if not sharded:
                rc = call(*fixed, l, *per_layer[l], *tail)
                if rc:
                    wl.ffi.check(rc)
                continue
            qd.copy_(hq[l], non_blocking=True)
            kd.copy_(hk[l], non_blocking=True)
            vd.copy_(hv[l], non_blocking=True)
            res = wl.hsd.append_decode(wl.plan, l, qd, kd, vd,
                                       od if wl.xchg == "nccl" else None, wl.bt, wl.scale,
                                       stream=s)
            hg[l].copy_(res, non_blocking=True)
            s.synchronize()

    for _ in range(min(2, args.warmup)):
        e2e_step()
    if wl.world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        e2e_step()
    e1.record(s)
    torch.cuda.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1) / steps, wl.world, wl.dev)
    job_bytes = _sum_over_ranks(float(sum(wl.step_bytes())), wl.world, wl.dev)
    h2d = wl.L * wl.B * (wl.H * wl.D + 2 * wl.Hkv * wl.D) * 2
    d2h = wl.L * wl.B * (wl.H_full if sharded else wl.H) * wl.D * 2
    return {"value": round(job_bytes / (ms / 1e3) / 1e9, 1), "unit": "GB/s",
            "ms_per_step": round(ms, 4), "steps": steps,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "call": ("kvc_decode_host through the C ABI (pinned host q/k_new/v_new/out, one "
                     "call per layer, each waits for its output)"
                     if not sharded else
                     "HeadShardedDecode.append_decode (pinned H2D of this rank's q/k/v, "
                     "fused decode + exchange, D2H of all heads, per layer, waits)")}


# ---------------------------------------------------------------------------------
# offload arm (benchmark config 5): KV in host memory, streamed per layer
# ---------------------------------------------------------------------------------
def run_offload(args, rank, world, local_rank):
    """--offload-kv-cpu decode steps the way the reference's KVCacheManager runs
    them in its cpu mode (src/kv_cache.py:133-135, :219-239): K and V live in two
    host arrays (layers, max_seq_len, Hkv, D); per layer the new row is written
    there, then ``matmul_module.gqa_attention`` gets the layer's views, which the
    drop-in serves from its streaming engine (the layer's rows are copied to the
    GPU on a copy stream while the previous layer attends).  Each call returns
    after its output is on the host, so host wall time is device-complete time."""
    import torch

    import matmul_module

    torch.cuda.set_device(local_rank)
    cfg = dict(CONFIGS[args.config])
    if args.layers:
        cfg["layers"] = args.layers
    L, H, Hkv, D = cfg["layers"], cfg["H"], cfg["Hkv"], cfg["D"]
    cached = int(cfg["lens"][1])
    S = cached + 1
    # every rank holds its own host copy of the KV history (replicas): refuse
    # before allocating when the node's RAM cannot hold all of them
    need = world * L * S * Hkv * D * 2 * 2
    ram = os.sysconf("SC_PAGE_SIZE") * os.sysconf("SC_PHYS_PAGES")
    if need > 0.8 * ram:
        raise SystemExit(f"offload replicas need {need / 1e9:.1f} GB of host RAM for {world} ranks; "
                         f"this node has {ram / 1e9:.1f} GB (run fewer ranks or --layers)")
    t0 = time.perf_counter()
    matmul_module.set_offload_mirror_bytes(int(args.mirror_gb * 1e9))
    k_host = np.empty((L, S, Hkv, D), dtype=np.float16)   # kv_cache.py:133-135
    v_host = np.empty((L, S, Hkv, D), dtype=np.float16)
    rng = np.random.default_rng(cfg["seed"])
    block = rng.standard_normal(1 << 23, dtype=np.float32).astype(np.float16)
    for arr, shift in ((k_host, 0), (v_host, 12345)):
        flat = arr.reshape(-1)
        step = block.size
        for o in range(0, flat.size, step):
            n = min(step, flat.size - o)
            flat[o:o + n] = np.roll(block, shift + o // step)[:n]
    setup_s = time.perf_counter() - t0
    q = rng.standard_normal((L, 1, H, D), dtype=np.float32).astype(np.float16)
    kn = rng.standard_normal((L, 1, Hkv, D), dtype=np.float32).astype(np.float16)
    vn = rng.standard_normal((L, 1, Hkv, D), dtype=np.float32).astype(np.float16)
    out = np.empty((1, H, D), dtype=np.float16)
    scale = 1.0 / math.sqrt(D)

    def step():
        for l in range(L):
            # KVCacheManager.attend, cpu mode: host append, then the layer's views
            k_host[l][cached:S] = kn[l]
            v_host[l][cached:S] = vn[l]
            matmul_module.gqa_attention(q[l], k_host[l], v_host[l], out, 1, S, H, Hkv, D,
                                        cached, scale, True)

    t1 = time.perf_counter()
    for _ in range(args.warmup):
        step()
    first = matmul_module.offload_stats(k_host)
    assert first["engines"] == 1, "the host arrays were not served by the streaming engine"
    warm_s = time.perf_counter() - t1
    torch.cuda.synchronize()
    ts = time.perf_counter()
    for _ in range(args.steps):
        step()
    elapsed = time.perf_counter() - ts
    st = matmul_module.offload_stats(k_host)
    del k_host, v_host  # releases the engine (and unregisters the host arrays)
    kv_bytes = L * S * Hkv * D * 2 * 2
    h2d = st["h2d_bytes"] - first["h2d_bytes"]
    h2d_ms = st["h2d_ms"] - first["h2d_ms"]
    if rank != 0:
        return None
    return {
        "metric": METRIC,
        "value": round(kv_bytes * args.steps / elapsed / 1e9, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(elapsed / args.steps * 1e3, 2),
        "steps_per_s": round(args.steps / elapsed, 4),
        "higher_is_better": True,
        "scaling": "replicas",
        "vs_baseline": None,
        "dtype": "f16 storage, f32 accumulate",
        "data": "synthetic: seeded N(0,1) K/V/q (host KV filled from a tiled random block)",
        "config": {"workload": f"{cfg['workload']} (benchmark config {args.config})"
                               + (f" [subset: {L} layers]" if args.layers else ""),
                   "layers": L, "q_heads": H, "kv_heads": Hkv, "head_dim": D, "batch": 1,
                   "cached_len": cached, "host_kv_gb": round(kv_bytes / 1e9, 2),
                   "timing": "host wall clock; every attend call waits for its output",
                   "call": "matmul_module.gqa_attention on the layer views of (layers, S, Hkv, D) "
                           "host arrays after the host append (KVCacheManager's cpu mode)"},
        "hbm_mirror": {"budget_gb": args.mirror_gb, "layers": st["mirror_layers"],
                       "uploaded_gb_per_step": round((st["mirror_bytes"] - first["mirror_bytes"])
                                                     / args.steps / 1e9, 6)},
        "host_link": {"h2d_gb_per_step": round(h2d / args.steps / 1e9, 3),
                      "h2d_gbs_wall": round(h2d / elapsed / 1e9, 2),
                      "h2d_gbs_copy_engine": round(h2d / (h2d_ms / 1e3) / 1e9, 2) if h2d_ms else None,
                      "prefetch_hits": st["prefetch_hits"] - first["prefetch_hits"],
                      "attend_calls": st["attend_calls"] - first["attend_calls"]},
        "setup_s": round(setup_s, 1),
        "warmup_s": round(warm_s, 1),
    }


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one
# decode_persistent_kernel launch of config 3, measured by
#   ncu --set full --clock-control none -k regex:"decode_persistent|merge_splits" -s 8 -c 2 \
#       -o prof python bench.py --layers 2 --steps 3 --warmup 3 --min-timed-s 0 --max-passes 1 \
#       --no-cpu-baseline --no-e2e --no-clocks
# (a 2-layer subset with the same per-launch shape); None for other workloads.
TRAFFIC_PER_LAUNCH = {
    "3": 566_637_824 + 5_116_416,
}


# ---------------------------------------------------------------------------------
# reference arm: the reference algorithm on the host cores
# ---------------------------------------------------------------------------------
# Weight types of a layer: (q, k, v, o, gate, up, down) GGML ids; q4_k_m is the
# usual Q4_K_M mix (Q6_K for v and down).
LAYER_TYPES = {"q4_0": (2,) * 7, "q8_0": (8,) * 7, "f16": (1,) * 7,
               "q4_k_m": (12, 12, 14, 12, 12, 12, 14)}


def layer_launches(types) -> int:
    """Kernel launches of one decode layer call: two RMSNorms, one projection launch
    per run of equal q/k/v types, RoPE, the fused append + decode and its split merge,
    the output projection, gate + up (one SwiGLU launch for equal types, else two
    projections and the SwiGLU kernel) and the down projection."""
    q, k, v, _, gate, up, _ = types
    qkv = 1 + (k != q) + (v != k)
    ffn = 1 if gate == up else 3
    return 7 + qkv + ffn


def run_layer(args, rank, world, local_rank):
    """Whole-layer decode (forward_layer_cached, the layer the KV path serves):
    Llama-3-8B geometry (hidden 4096, intermediate 14336, 32 q-heads, 8 KV heads,
    head_dim 128, 32 layers, each with its own weights of the chosen types), one
    sequence with 4,095 cached positions (prefilled untimed in 512-token chunks),
    then K timed decode steps of all 32 layers on device buffers.  value =
    tokens/s; the roofline counts weight bytes + KV bytes read + appended rows per
    layer against the measured HBM copy bandwidth; e2e = one layer through the
    reference's host-buffer call (activations and all weights copied per call)."""
    import torch

    import kvcache_ffi as ffi
    import matmul_module

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import layer_ref  # seeded random GGML blocks (input generator only)

    torch.cuda.set_device(local_rank)
    L, hid, inter, H, Hkv, D = (args.layers or 32), 4096, 14336, 32, 8, 128
    types = LAYER_TYPES[args.layer_step]
    shapes = [(H * D, hid), (Hkv * D, hid), (Hkv * D, hid), (hid, H * D), (inter, hid),
              (inter, hid), (hid, inter)]
    rng = np.random.default_rng(11)
    host_w = [layer_ref.random_weight(rng, t, n, k) for t, (n, k) in zip(types, shapes)]
    dev_w = [[torch.from_numpy(w).cuda() for w in host_w]]
    for _ in range(L - 1):   # distinct weights per layer (no L2 reuse across layers)
        dev_w.append([w.clone() for w in dev_w[0]])
    an = (1.0 + 0.05 * torch.randn(hid, device="cuda")).half()
    fn = (1.0 + 0.05 * torch.randn(hid, device="cuda")).half()
    ctx0 = 4095
    S = ctx0 + args.warmup + args.steps + 8
    matmul_module.kv_cache_init(L, S, Hkv, D)
    st = torch.cuda.current_stream().cuda_stream
    scale = 1.0 / math.sqrt(D)

    def layer(l, x, out, seq, pos):
        w = dev_w[l]
        ffi.check(ffi.lib.kvc_forward_layer_cached_device(
            x.data_ptr(), out.data_ptr(), an.data_ptr(), w[0].data_ptr(), types[0],
            w[1].data_ptr(), types[1], w[2].data_ptr(), types[2], w[3].data_ptr(), types[3],
            fn.data_ptr(), w[4].data_ptr(), types[4], w[5].data_ptr(), types[5], w[6].data_ptr(),
            types[6], l, seq, pos, hid, inter, H, Hkv, D, 1e-5, ROPE_BASE, 0, scale, st))

    xp = (torch.randn((512, hid), device="cuda") * 0.5).half()
    op = torch.empty_like(xp)
    for l in range(L):
        pos = 0
        while pos < ctx0:
            n = min(512, ctx0 - pos)
            layer(l, xp[:n], op[:n], n, pos)
            pos += n
    torch.cuda.synchronize()
    x = (torch.randn((1, hid), device="cuda") * 0.5).half()
    y = torch.empty_like(x)
    pos = ctx0

    def step(p):
        a, b = x, y
        for l in range(L):
            layer(l, a, b, 1, p)
            a, b = b, a

    for _ in range(args.warmup):
        step(pos)
        pos += 1
    torch.cuda.synchronize()
    sampler = ClockSampler(local_rank) if not args.no_clocks else None
    if sampler:
        sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pos_t0 = pos
    e0.record()
    for _ in range(args.steps):
        step(pos)
        pos += 1
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    code, info = ffi.device_error(local_rank)
    if code:
        raise RuntimeError(f"device error {code} ({info}) in the timed layer steps")
    ms = e0.elapsed_time(e1) / args.steps
    wbytes = sum(w.numel() for w in dev_w[0])
    kv_read = sum((p + 1) * Hkv * D * 2 * 2 for p in range(pos_t0, pos)) / args.steps
    act = (hid * 2 * 2 + (H + 2 * Hkv) * D * 2 * 2 + inter * 2 * 2) * 2   # activations, loosely
    layer_bytes = wbytes + kv_read + 2 * Hkv * D * 2 + act
    peak, peak_kind = load_peaks()
    us_layer = ms * 1e3 / L
    achieved = layer_bytes / (us_layer * 1e-6) / 1e9

    # e2e: the reference's host-buffer call on layer 0 (weights copied every call)
    e2e = None
    if not args.no_e2e:
        xh = x.cpu().numpy()
        yh = np.empty_like(xh)
        an_h, fn_h = an.cpu().numpy(), fn.cpu().numpy()

        def host_layer(p):
            matmul_module.forward_layer_cached(
                xh, yh, an_h, host_w[0], types[0], host_w[1], types[1], host_w[2], types[2],
                host_w[3], types[3], fn_h, host_w[4], types[4], host_w[5], types[5], host_w[6],
                types[6], 0, 1, p, hid, inter, H, Hkv, D, 1e-5, ROPE_BASE, False, scale)

        host_layer(pos)   # untimed
        t0 = time.perf_counter()
        n_e2e = max(1, args.e2e_steps)
        for i in range(n_e2e):
            host_layer(pos + 1 + i)
        dt = (time.perf_counter() - t0) / n_e2e
        e2e = {"value": round(1.0 / (dt * L), 2), "unit": "tokens/s", "us_per_layer": round(dt * 1e6, 1),
               "h2d_bytes_per_step": int((wbytes + 2 * hid * 2 + hid * 2) * L),
               "d2h_bytes_per_step": int(hid * 2 * L),
               "call": "matmul_module.forward_layer_cached per layer (host x, norms and all weights copied per call, like the reference)"}

    cpu = None
    if not args.no_cpu_baseline:
        # the oracle layer (numpy, fp32) on one layer at 512 cached positions: bounded sample
        lw = layer_ref.LayerWeights(an.cpu().numpy(), *[(host_w[i], types[i]) for i in range(4)],
                                    fn.cpu().numpy(), *[(host_w[i], types[i]) for i in range(4, 7)])
        kc = np.zeros((ctx0 + 2, Hkv, D), np.float16)
        vc = np.zeros_like(kc)
        t0 = time.perf_counter()
        layer_ref.layer_forward(x.cpu().numpy(), lw, kc, vc, ctx0, H, Hkv, D, inter, 1e-5, ROPE_BASE,
                                False, scale)
        dt = time.perf_counter() - t0
        cpu = {"value": round(1.0 / (dt * L), 4), "unit": "tokens/s", "cores": os.cpu_count(),
               "kind": "port", "sample": f"one layer, numpy oracle (dequantize + fp32 matmuls), {dt:.2f} s"}
    return {
        "metric": "forward_layer_cached decode tokens/s (Llama-3-8B geometry, batch 1, 4K context)",
        "value": round(1e3 / ms, 2), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "us_per_layer": round(us_layer, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16 activations, GGML weights, f32 accumulate",
        "data": "synthetic: seeded random GGML blocks, N(0,1) activations",
        "config": {"workload": f"llama3-8b-layer-decode-{args.layer_step}", "layers": L,
                   "hidden": hid, "intermediate": inter, "q_heads": H, "kv_heads": Hkv,
                   "head_dim": D, "weight_types": list(types), "cached_len": ctx0,
                   "weight_bytes_per_layer": int(wbytes),
                   "l2": "weights per layer differ; 32 layers of weights >> L2"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None,
                     "peak_kind": peak_kind, "bytes_per_layer": int(layer_bytes)},
        "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks,
        "gpu_launches": L * args.steps * layer_launches(types),
    }


def run_layer_batch(args, rank, world, local_rank):
    """Whole-model batched decode (paged.BatchDecoder over kvc_forward_layer_paged):
    benchmark config 3's batch (32 sequences, cached lengths U[1024, 8192] from seed
    2024, paged fp16 pool of 16-position pages in a random permutation, N(0,1) KV)
    through 32 Llama-3-8B layers, each with its own weights of the chosen types.  A
    step is one new token for every sequence through every layer, in a real decode
    loop: contexts grow by one per step and the plan is rebuilt on the host every
    step, inside the timed region.  value = tokens/s (batch / step time); the
    roofline counts weights + KV read + appended rows per step against the
    measured HBM copy bandwidth.  e2e = the same step with the new tokens'
    activations copied from page-locked host memory and the last layer's output
    copied back every step."""
    import torch

    import kvcache_ffi as ffi
    import paged

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import layer_ref  # seeded random GGML blocks (input generator) and the CPU baseline

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = CONFIGS["3"]
    L, hid, inter = (args.layers or cfg["layers"]), 4096, 14336
    H, Hkv, D, B = cfg["H"], cfg["Hkv"], cfg["D"], cfg["batch"]
    types = LAYER_TYPES[args.layer_step]
    shapes = [(H * D, hid), (Hkv * D, hid), (Hkv * D, hid), (hid, H * D), (inter, hid),
              (inter, hid), (hid, inter)]
    rng = np.random.default_rng(11)
    host_w = [layer_ref.random_weight(rng, t, n, k) for t, (n, k) in zip(types, shapes)]
    dev_w = [[torch.from_numpy(w).to(dev) for w in host_w]]
    for _ in range(L - 1):   # distinct weights per layer (no L2 reuse across layers)
        dev_w.append([w.clone() for w in dev_w[0]])
    an = (1.0 + 0.05 * torch.randn(hid, device=dev)).half()
    fn = (1.0 + 0.05 * torch.randn(hid, device=dev)).half()
    layers = [paged.DeviceLayerWeights(an, fn, w, types, hid, inter) for w in dev_w]
    cached = cached_lengths(cfg)
    extra = args.warmup + args.steps + max(1, args.e2e_steps) + 2
    table, total_pages = paged.random_block_tables(cached + extra, PAGE, cfg["seed"] + 17 * rank)
    pool = paged.PagedKVCache(L, total_pages, PAGE, Hkv, D, dtype=torch.float16, device=local_rank)
    pool.fill_normal(seed=1000 + rank, stddev=1.0)
    bt = torch.from_numpy(table).to(dev)
    dec = paged.BatchDecoder(pool, layers, bt, H, cached, 1e-5, ROPE_BASE)
    x = (torch.randn((B, hid), device=dev) * 0.5).half()
    for _ in range(args.warmup):
        dec.step(x)
    torch.cuda.synchronize()
    sampler = ClockSampler(local_rank) if not args.no_clocks else None
    if sampler:
        sampler.start()
    ctx_t0 = dec.ctx.copy()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        dec.step(x)
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    code, info = ffi.device_error(local_rank)
    if code:
        raise RuntimeError(f"device error {code} ({info}) in the timed batched steps")
    ms = e0.elapsed_time(e1) / args.steps
    wbytes = sum(w.numel() for w in dev_w[0])
    # positions attended per step: step j reads ctx_t0 + j + 1 positions per sequence
    kv_read = sum(int((ctx_t0 + j + 1).sum()) for j in range(args.steps)) / args.steps
    kv_read *= Hkv * D * 2 * 2 * L
    appended = B * Hkv * D * 2 * 2 * L
    step_b = wbytes * L + kv_read + appended
    peak, peak_kind = load_peaks()
    achieved = step_b / (ms * 1e-3) / 1e9

    e2e = None
    if not args.no_e2e:
        xh = x.cpu().pin_memory()
        yh = torch.empty_like(xh).pin_memory()
        n_e2e = max(1, args.e2e_steps)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            yh.copy_(dec.step(xh.to(dev, non_blocking=True)))
        torch.cuda.synchronize()
        dt = (time.perf_counter() - t0) / n_e2e
        e2e = {"value": round(B / dt, 2), "unit": "tokens/s", "ms_per_step": round(dt * 1e3, 3),
               "h2d_bytes_per_step": int(B * hid * 2), "d2h_bytes_per_step": int(B * hid * 2),
               "call": "paged.BatchDecoder.step per step: host activations in, host output out "
                       "(page-locked), plan rebuilt per step"}

    cpu = None
    if not args.no_cpu_baseline:
        # the numpy oracle layer for ONE token of one sequence at the batch's mean
        # context; the reference decodes the batch one sequence at a time, so a step
        # costs B x layers such calls
        ctx_m = int(cached.mean())
        lw = layer_ref.LayerWeights(an.cpu().numpy(), *[(host_w[i], types[i]) for i in range(4)],
                                    fn.cpu().numpy(), *[(host_w[i], types[i]) for i in range(4, 7)])
        kc = np.zeros((ctx_m + 1, Hkv, D), np.float16)
        vc = np.zeros_like(kc)
        t0 = time.perf_counter()
        layer_ref.layer_forward(x[:1].cpu().numpy(), lw, kc, vc, ctx_m, H, Hkv, D, inter, 1e-5,
                                ROPE_BASE, False, 1.0 / math.sqrt(D))
        dt = time.perf_counter() - t0
        cpu = {"value": round(1.0 / (dt * L), 4), "unit": "tokens/s", "cores": os.cpu_count(),
               "kind": "port",
               "sample": f"one layer of one sequence at {ctx_m} cached positions, numpy oracle "
                         f"(dequantize + fp32 matmuls), {dt:.2f} s; x {L} layers per token"}
    dec.close()
    return {
        "metric": "batched decode tokens/s through the whole layer (Llama-3-8B geometry, "
                  "config-3 batch: 32 ragged sequences)",
        "value": round(B * 1e3 / ms, 2), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "us_per_layer": round(ms * 1e3 / L, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 activations and KV, GGML weights, f32 accumulate",
        "data": "synthetic: seeded random GGML blocks, N(0,1) KV pool and activations",
        "config": {"workload": f"llama3-8b-batched-layer-decode-{args.layer_step}", "layers": L,
                   "hidden": hid, "intermediate": inter, "q_heads": H, "kv_heads": Hkv,
                   "head_dim": D, "sequences": B, "weight_types": list(types),
                   "cached_tokens_at_start": int(ctx_t0.sum()), "page_size": PAGE,
                   "weight_bytes_per_layer": int(wbytes),
                   "l2": "weights per layer differ; KV and weights per step >> L2"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None,
                     "peak_kind": peak_kind, "bytes_per_step": int(step_b)},
        "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks,
        "gpu_launches": L * args.steps * layer_launches(types),
    }


def run_reference(args, rank, world):
    if rank != 0:
        return None
    cfg = CONFIGS[args.config]
    ctx = cached_lengths(cfg) + 1
    w = CpuWorkload(cfg, ctx)
    threads = w.threads
    times = [w.run_layer() for _ in range(args.warmup + args.steps)][args.warmup:]
    dt = float(np.mean(times))
    gbs = w.layer_bytes / dt / 1e9
    np_gbs, np_s, np_n = numpy_path_sample(w)
    sample = (f"each step: 1 of {cfg['layers']} layers x {cfg['batch']} sequences of the "
              f"workload; oracle/gqa_online.c, the reference kernel's algorithm "
              f"(attention.hip:35-123), OpenMP")
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": round(gbs, 3),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3),
        "ms_per_step_note": ("one step = the timed sample (1 layer of the workload); the whole "
                             "32-layer step would take ms_per_full_step"),
        "ms_per_full_step": round(dt * cfg["layers"] * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16 storage, f32 accumulate",
        "data": "synthetic: seeded N(0,1) K/V/q",
        "config": {"workload": f"{cfg['workload']} (benchmark config {args.config})",
                   "layers": cfg["layers"], "q_heads": cfg["H"], "kv_heads": cfg["Hkv"],
                   "head_dim": cfg["D"], "global_batch": cfg["batch"],
                   "cached_len": (f"U[{cfg['lens'][1]},{cfg['lens'][2]}] seed {cfg['seed']}"
                                  if cfg["lens"][0] == "uniform" else int(cfg["lens"][1])),
                   "ctx_tokens_per_gpu_start": int(ctx.sum()),
                   "kv_bytes_read_per_step_per_gpu": int(sum(step_bytes(cfg, ctx)[:1])),
                   "timed": (f"{args.steps} samples after {args.warmup} warm-up samples, each "
                             f"one layer of the workload on {threads} host threads; value = "
                             f"bytes / mean sample time")},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "numpy_path": {"value": round(np_gbs, 4), "unit": "GB/s", "cores": blas_threads(),
                       "kind": "port",
                       "sample": (f"{np_n} sequences of one layer in turn, {np_s:.1f} s: host "
                                  f"append + ref_gqa_attention (the reference's numpy path, "
                                  f"tests/test_layer.py:76-105, as oracle/gqa_ref.py restates "
                                  f"it)")},
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="3")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--page-size", type=int, default=PAGE, help="positions per KV page (multiple of 16)")
    ap.add_argument("--rope", action="store_true",
                    help="rotate q and the new K rows (RoPE) inside the step (rope + append + attend)")
    ap.add_argument("--mirror-gb", type=float, default=0.0,
                    help="config 5: keep an HBM mirror of as many layers as this many GB hold")
    ap.add_argument("--one-rank-of", type=int, default=0,
                    help="profiling on one GPU: run rank 0's shard of an N-way KV-head split "
                         "with its head exchange connected to itself")
    ap.add_argument("--no-grow", action="store_true",
                    help="skip the growing decode loop (contexts +1 per step, plan rebuilt every "
                         "step); the headline is then the replayed fixed step")
    ap.add_argument("--min-timed-s", type=float, default=1.0,
                    help="repeat the timed pass of --steps steps until about this many seconds "
                         "are timed (value = the median pass)")
    ap.add_argument("--max-passes", type=int, default=40)
    ap.add_argument("--no-variants", action="store_true",
                    help="N > 1: skip the sequence-sharded and NCCL-transport lines")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch every kernel from the host loop instead of replaying a CUDA graph")
    ap.add_argument("--xchg", choices=["p2p", "nccl"], default="p2p",
                    help="head-sharded output exchange: fused peer stores or NCCL all-gather")
    ap.add_argument("--shard", choices=["seq", "heads"], default=None,
                    help="multi-GPU split: independent sequences per GPU (weak scaling, default for "
                         "config 3) or KV heads with a per-layer all-gather (strong, config 4)")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling only: run this many layers instead of the config's")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--layer-step", choices=sorted(LAYER_TYPES), default=None,
                    help="time the whole layer (forward_layer_cached) instead of the KV path")
    ap.add_argument("--layer-batch", action="store_true",
                    help="with --layer-step: config 3's 32-sequence batch through the whole "
                         "layer (paged.BatchDecoder) instead of one sequence")
    ap.add_argument("--launch-events", action="store_true",
                    help="diagnostics: record events around every launch (serialises launches)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        res = run_reference(args, rank, world)
    else:
        if world > 1:
            import datetime

            import torch

            torch.cuda.set_device(local_rank)
            torch.distributed.init_process_group(
                "nccl", timeout=datetime.timedelta(seconds=120),
                device_id=torch.device("cuda", local_rank))
        try:
            if args.layer_step and args.layer_batch:
                res = run_layer_batch(args, rank, world, local_rank) if rank == 0 else None
            elif args.layer_step:
                res = run_layer(args, rank, world, local_rank) if rank == 0 else None
            elif args.config == "5":
                res = run_offload(args, rank, world, local_rank)
            else:
                res = run_b200(args, rank, world, local_rank)
        finally:
            if world > 1:
                import torch

                torch.distributed.destroy_process_group()
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
