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
def run_b200(args, rank, world, local_rank):
    import torch

    import kvcache_ffi as ffi
    import paged

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = dict(CONFIGS[args.config])
    if args.layers:
        cfg["layers"] = args.layers  # profiling subset only (the bench line names it)
    L, H, Hkv, D, B = cfg["layers"], cfg["H"], cfg["Hkv"], cfg["D"], cfg["batch"]
    shard = args.shard or ("heads" if args.config == "4" else "seq")
    H_full = H
    if shard == "heads" and world > 1:
        # KV-head sharding: this rank owns KV heads [r*Hkv/n, (r+1)*Hkv/n) and their
        # q-heads; the per-head outputs are all-gathered after every layer.
        h0, h1 = paged.shard_heads(Hkv, world, rank)
        Hkv = h1 - h0
        H = H * Hkv // cfg["Hkv"]
    one_rank_of = args.one_rank_of if world == 1 else 0
    if one_rank_of > 1:
        # profiling mode: rank 0's shard of a one_rank_of-way KV-head split on this one
        # GPU, its head exchange connected to itself (same kernels and launches as a
        # real rank, no peers to wait for)
        h0, h1 = paged.shard_heads(Hkv, one_rank_of, 0)
        Hkv = h1 - h0
        H = H * Hkv // cfg["Hkv"]
    cached = cached_lengths(cfg)
    ctx = cached + 1                                  # context includes the appended token
    # --grow: every step appends one more position (a real decode loop), so pages
    # for the extra positions are allocated up front
    extra = (args.warmup + args.steps + 1) if args.grow else 0
    table, total_pages = paged.random_block_tables(ctx + extra, args.page_size,
                                                   cfg["seed"] + 17 * rank)
    pool = paged.PagedKVCache(L, total_pages, args.page_size, Hkv, D, dtype=torch.float16,
                              device=local_rank)
    pool.fill_normal(seed=1000 + rank, stddev=1.0)
    bt = torch.from_numpy(table).to(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    q = torch.randn((L, B, H, D), generator=g, device=dev, dtype=torch.float32).half()
    kn = torch.randn((L, B, Hkv, D), generator=g, device=dev, dtype=torch.float32).half()
    vn = torch.randn((L, B, Hkv, D), generator=g, device=dev, dtype=torch.float32).half()
    out = torch.empty_like(q)
    gathered = None
    if shard == "heads" and world > 1:
        import sharding

        # every rank ends each layer with all heads of every sequence
        gathered = torch.empty((L, B, H_full, D), dtype=torch.float16, device=dev)
        hsd = sharding.HeadShardedDecode(pool, H_full, cfg["Hkv"], transport=args.xchg,
                                         num_queries=B)
    self_xchg = None
    if one_rank_of > 1:
        self_xchg = ctypes.c_void_p()
        ffi.check(ffi.lib.kvc_xchg_create(local_rank, 0, 1, B * H_full * D * 2, 2,
                                          ctypes.byref(self_xchg)))
        base = ctypes.c_void_p()
        ffi.check(ffi.lib.kvc_xchg_base(self_xchg, ctypes.byref(base)))
        ffi.check(ffi.lib.kvc_xchg_connect_ptrs(self_xchg, (ctypes.c_void_p * 1)(base.value)))
    pos = torch.from_numpy((ctx - 1).astype(np.int32)).to(dev)
    rows = torch.arange(B, dtype=torch.int32, device=dev)
    scale = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream()
    plan = pool.plan(ctx, H, stream=stream)
    # block tables are static and pages are written only by the decode kernels
    # themselves, so each launch may start streaming KV before the previous one ends
    plan.set_kv_stable(True)
    torch.cuda.synchronize()

    grown = [0]  # steps taken so far (--grow)

    def step(events=None, s=None):
        # one fused launch per layer: append each sequence's new row + attend
        s = stream if s is None else s
        if args.grow:
            # the contexts grew by one since the last step: a new plan (host), then the layers
            pool.plan(ctx + grown[0], H, plan=plan, stream=s)
            grown[0] += 1
        for l in range(L):
            if events is not None:
                events[l][0].record(s)
            if self_xchg is not None:
                pool.append_decode_xchg(plan, l, q[l], kn[l], vn[l], self_xchg, l & 1, H_full, 0,
                                        bt, scale, stream=s)
            elif gathered is None and args.rope:
                # rotate q and the new K row (RoPE at each sequence's position) first
                pool.append_decode_rope(plan, l, q[l], kn[l], vn[l], out[l], bt, scale,
                                        ROPE_BASE, False, stream=s)
            elif gathered is None:
                pool.append_decode(plan, l, q[l], kn[l], vn[l], out[l], bt, scale, stream=s)
            else:
                # fused append + attention on this rank's heads; p2p: the merge kernel
                # pushes the heads to every rank (result in an exchange slot), nccl:
                # all-gather + copy into gathered[l]
                hsd.append_decode(plan, l, q[l], kn[l], vn[l],
                                  gathered[l] if args.xchg == "nccl" else None, bt, scale,
                                  stream=s)
            if events is not None:
                events[l][1].record(s)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    code, info = ffi.device_error(local_rank)
    if code:
        raise RuntimeError(f"device error {code} ({info}) during warm-up")
    graph = None
    if not args.no_graph and not args.launch_events and not args.grow:
        # The step's 2 x L launches are recorded once into a CUDA graph and replayed:
        # the same kernels, without the host's per-launch cost between them.
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step(s=torch.cuda.current_stream())
        graph.replay()  # one untimed replay
        torch.cuda.synchronize()
        code, info = ffi.device_error(local_rank)
        if code:
            raise RuntimeError(f"device error {code} ({info}) in the captured step")

    # Per-launch events would serialise consecutive launches (they overlap by
    # programmatic dependent launch), so they are only recorded on request.
    evs = ([[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(L)]
            for _ in range(args.steps)] if args.launch_events else None)
    sampler = ClockSampler(local_rank) if not args.no_clocks else None
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
    t_start = torch.cuda.Event(enable_timing=True)
    t_stop = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for s in range(args.steps):
        if graph is not None:
            graph.replay()
        else:
            step(evs[s] if evs else None)
    t_stop.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    if world > 1:
        torch.distributed.barrier()
    elapsed_ms = t_start.elapsed_time(t_stop)
    used_graph = graph is not None
    hsd_p2p = (gathered is not None and args.xchg == "p2p") or self_xchg is not None
    if graph is not None:
        graph.reset()  # released before any collective teardown (it may hold NCCL calls)
        graph = None
    dec_ms = ([evs[s][l][0].elapsed_time(evs[s][l][1]) for s in range(args.steps) for l in range(L)]
              if evs else None)
    code, info = ffi.device_error(local_rank)
    if code:
        raise RuntimeError(f"device error {code} ({info}) during timing")

    kv_read, appended, qo = step_bytes(dict(cfg, H=H, Hkv=Hkv), ctx)
    if args.grow:  # the timed steps ran at contexts ctx + warmup ... ctx + warmup + steps - 1
        parts = [step_bytes(dict(cfg, H=H, Hkv=Hkv), ctx + args.warmup + i)
                 for i in range(args.steps)]
        kv_read, appended, qo = (sum(p[0] for p in parts) // args.steps,
                                 sum(p[1] for p in parts) // args.steps,
                                 sum(p[2] for p in parts) // args.steps)
    rank_bytes = kv_read + appended + qo
    # aggregate: max time over ranks, sum of bytes
    if world > 1:
        t = torch.tensor([elapsed_ms, float(rank_bytes)], dtype=torch.float64, device=dev)
        tmax = t[:1].clone()
        torch.distributed.all_reduce(tmax, op=torch.distributed.ReduceOp.MAX)
        tsum = t[1:].clone()
        torch.distributed.all_reduce(tsum, op=torch.distributed.ReduceOp.SUM)
        elapsed_ms, job_bytes = float(tmax.item()), float(tsum.item())
    else:
        job_bytes = float(rank_bytes)
    ms_per_step = elapsed_ms / args.steps
    value = job_bytes / (ms_per_step / 1e3) / 1e9

    # ---- e2e: reference-facing host-buffer call, per layer, copies inside ----
    e2e = None
    if not args.no_e2e:
        hq = q.cpu().pin_memory()
        hk = kn.cpu().pin_memory()
        hv = vn.cpu().pin_memory()
        ho = torch.empty_like(hq).pin_memory()
        e2e_steps = max(1, min(args.steps, args.e2e_steps))

        if gathered is not None:
            hg = torch.empty(tuple(gathered.shape), dtype=torch.float16).pin_memory()
            qd, kd, vd = torch.empty_like(q[0]), torch.empty_like(kn[0]), torch.empty_like(vn[0])
            od = torch.empty_like(gathered[0])

        def e2e_step():
            for l in range(L):
                if gathered is None:
                    pool.decode_host(plan, l, hq[l], hk[l], hv[l], ho[l], bt, scale, stream=stream)
                    continue
                # sharded: rank inputs in, fused decode, all-gather, all heads out, wait
                qd.copy_(hq[l], non_blocking=True)
                kd.copy_(hk[l], non_blocking=True)
                vd.copy_(hv[l], non_blocking=True)
                res = hsd.append_decode(plan, l, qd, kd, vd,
                                        od if args.xchg == "nccl" else None, bt, scale,
                                        stream=stream)
                hg[l].copy_(res, non_blocking=True)
                stream.synchronize()

        for _ in range(min(2, args.warmup)):
            e2e_step()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / e2e_steps
        if world > 1:
            t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            e2e_ms = float(t.item())
        h2d = L * B * (H * D + 2 * Hkv * D) * 2
        d2h = L * B * (H_full if gathered is not None else H) * D * 2
        e2e = {"value": round(job_bytes / (e2e_ms / 1e3) / 1e9, 1), "unit": "GB/s",
               "ms_per_step": round(e2e_ms, 4), "steps": e2e_steps,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "call": ("kvc_decode_host (pinned host q/k_new/v_new/out, per layer, waits)"
                        if gathered is None else
                        "HeadShardedDecode.append_decode (pinned H2D of this rank's q/k/v, "
                        "fused decode, NCCL all-gather, D2H of all heads, per layer, waits)")}

    if gathered is not None:
        hsd.close()  # collective: the exchange buffers are freed after every rank is done
    if self_xchg is not None:
        torch.cuda.synchronize()
        ffi.lib.kvc_xchg_destroy(self_xchg)

    if rank != 0:
        return None

    peak, peak_kind = load_peaks()
    # average launch duration over the timed region (timed region / launches; with
    # --launch-events, the mean of per-launch event pairs instead)
    dec_avg_ms = float(np.mean(dec_ms)) if dec_ms else elapsed_ms / (args.steps * L)
    dec_bytes = (kv_read + appended + qo) / L           # per launch (one layer)
    achieved = dec_bytes / (dec_avg_ms / 1e3) / 1e9
    res = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "steps_per_s": round(1e3 / ms_per_step, 2),
        "pct_of_peak": round(100.0 * value / (peak * world), 2),
        "higher_is_better": True,
        "scaling": "strong" if gathered is not None else "weak",
        "vs_baseline": None,
        "dtype": "f16 storage, f32 accumulate",
        "data": "synthetic: seeded N(0,1) K/V/q, random page permutation",
        "config": {
            "workload": f"{cfg['workload']} (benchmark config {args.config})"
                        + (f" [profiling subset: {L} layers]" if args.layers else "")
                        + (f" [profiling: one rank's shard of a {one_rank_of}-way KV-head split, "
                           "exchange connected to itself]" if one_rank_of > 1 else ""),
            "layers": L, "q_heads": H, "kv_heads": Hkv, "head_dim": D,
            "sequences_per_gpu": B, "global_batch": B if gathered is not None else B * world,
            "cached_len": (f"U[{cfg['lens'][1]},{cfg['lens'][2]}] seed {cfg['seed']}"
                           if cfg["lens"][0] == "uniform" else int(cfg["lens"][1])),
            "ctx_tokens_per_gpu": int(ctx.sum()), "page_size": args.page_size,
            "pool_gb_per_gpu": round(2 * L * total_pages * Hkv * args.page_size * D * 2 / 1e9, 2),
            "kv_bytes_read_per_step_per_gpu": kv_read,
            "l2": "inputs larger than L2 (pool >> 126 MB), no flush",
            "rope": bool(args.rope),
            "grow": ("contexts grow by one position per step; the plan is rebuilt every step "
                     "inside the timed region" if args.grow else False),
            "launch": ("one CUDA graph replay per step (the step's 2 x layers kernel launches)"
                       if used_graph else "direct launches from the host loop"),
            "parallelism": (f"KV-head-sharded x{world} ({Hkv} KV heads per GPU), "
                            + ("NCCL all-gather" if args.xchg == "nccl" else
                               "merge kernel pushes outputs to every rank over NVLink (p2p)")
                            + f", {B * H * D * 2} B of head outputs per GPU per layer"
                            if gathered is not None else
                            f"sequence-sharded x{world} (independent batches, no collective)"),
        },
        "roofline": {
            "bound": "hbm",
            "kernel": "decode_persistent_kernel (append fused) + merge_splits_kernel",
            "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind,
            "unit": "GB/s", "frac": round(achieved / peak, 4),
            "bytes_per_launch": int(dec_bytes), "avg_launch_us": round(dec_avg_ms * 1e3, 2),
            "duration_from": ("per-launch CUDA events" if dec_ms else
                              "CUDA events around the timed region / launches (launches overlap)"),
            "traffic": (TRAFFIC_PER_LAUNCH.get(args.config)
                        if not args.layers and world == 1 and args.page_size == PAGE else None),
            "traffic_from": "ncu dram__bytes_read.sum + dram__bytes_write.sum, decode kernel",
        },
        # per layer: the decode kernel and its split merge (PDL); with the p2p head
        # exchange the merge also pushes the outputs and a one-warp kernel
        # publishes and waits for the peers' epochs
        "gpu_launches": (3 if hsd_p2p or (args.rope and gathered is None) else 2) * L * args.steps,
        "plan": {"ctas_per_launch": plan.info().n_ctas, "splits": plan.info().n_items},
    }
    if e2e:
        res["e2e"] = e2e
    if clocks:
        res["clocks"] = clocks
    if not args.no_cpu_baseline:
        gbs, dt, thr, reps = cpu_sample(cfg, ctx, min_seconds=args.cpu_seconds)
        res["cpu_baseline"] = {
            "value": round(gbs, 3), "unit": "GB/s", "cores": thr, "kind": "port",
            "sample": f"1 of {L} layers x {B} sequences, {reps} reps, {dt * 1e3:.1f} ms/layer; "
                      "oracle/gqa_online.c (reference kernel's algorithm, OpenMP)",
            "steps_per_s_extrapolated": round(1.0 / (dt * L), 4),
        }
    plan.close()
    pool.close()
    return res


# ---------------------------------------------------------------------------------
# offload arm (benchmark config 5): KV in host memory, streamed per layer
# ---------------------------------------------------------------------------------
def run_offload(args, rank, world, local_rank):
    """--offload-kv-cpu decode steps through the drop-in KVCacheManager: every
    layer's cached K/V is streamed from (registered) host memory to the GPU on a
    copy stream while the previous layer attends.  Each attend call returns
    after its output is on the host, so host wall time is device-complete time."""
    import torch

    from kv_cache import KVCacheManager

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
    kv = KVCacheManager(L, S, Hkv, D, offload_to_cpu=True, max_kv_bytes=1 << 50,
                        offload_mirror_bytes=int(args.mirror_gb * 1e9))
    rng = np.random.default_rng(cfg["seed"])
    block = rng.standard_normal(1 << 23, dtype=np.float32).astype(np.float16)
    for arr, shift in ((kv._k_host, 0), (kv._v_host, 12345)):
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
            kv.attend(q[l], kn[l], vn[l], out, layer_idx=l, q_len=1, start_pos=cached,
                      num_heads=H, scale=scale, causal=True)

    t1 = time.perf_counter()
    for _ in range(args.warmup):
        step()
    first = kv.offload_stats()
    warm_s = time.perf_counter() - t1
    torch.cuda.synchronize()
    ts = time.perf_counter()
    for _ in range(args.steps):
        step()
    elapsed = time.perf_counter() - ts
    st = kv.offload_stats()
    kv.close()
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
                   "timing": "host wall clock; every attend call waits for its output"},
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


# DRAM traffic per decode launch (dram__bytes_read.sum + dram__bytes_write.sum)
# from the committed ncu captures; None until captured for a workload.
# DRAM bytes (read + write) of one decode_persistent_kernel launch, from an ncu
# capture of the same per-launch shape (profiles/decode_persistent_kernel_*.md).
TRAFFIC_PER_LAUNCH = {
    "3": 566_632_960 + 7_981_824,
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
        "ms_per_step": round(dt * cfg["layers"] * 1e3, 3),
        "ms_per_step_note": "extrapolated from the 1-layer sample x layers",
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16 storage, f32 accumulate",
        "data": "synthetic: seeded N(0,1) K/V/q",
        "config": {"workload": f"{cfg['workload']} (benchmark config {args.config})",
                   "layers": cfg["layers"], "q_heads": cfg["H"], "kv_heads": cfg["Hkv"],
                   "head_dim": cfg["D"], "sequences": cfg["batch"],
                   "ctx_tokens": int(ctx.sum())},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
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
    ap.add_argument("--grow", action="store_true",
                    help="a real decode loop: contexts grow by one per step and the plan is "
                         "rebuilt each step (no CUDA graph)")
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
