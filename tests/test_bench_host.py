"""The benchmark's byte accounting and workload generators on the CPU: the
algorithmic bytes per step that every reported GB/s divides by must equal the
figures the benchmark configs define (KV bytes read = Σ positions · Hkv · D · 2 B ·
2 for K and V, per layer), and the seeded workloads must be reproducible."""

from __future__ import annotations

import numpy as np

import bench


def test_config_bytes_match_the_defined_figures():
    c2 = bench.CONFIGS["2"]
    kv, app, qo = bench.step_bytes(c2, bench.cached_lengths(c2) + 1)
    assert kv == 2_147_483_648                      # 32 · 4096 · 32 · 128 · 2 · 2
    assert app == 32 * 32 * 128 * 2 * 2              # one row per layer, K and V
    assert qo == 32 * 32 * 128 * 2 * 2               # q read and out written per layer
    c4 = bench.CONFIGS["4"]
    kv, _, _ = bench.step_bytes(c4, bench.cached_lengths(c4) + 1)
    assert kv == 85_901_967_360                      # 80 · 8 · 32769 · 8 · 128 · 2 · 2
    c5 = bench.CONFIGS["5"]
    kv, _, _ = bench.step_bytes(c5, bench.cached_lengths(c5) + 1)
    assert kv == 42_950_000_640                      # 80 · 131073 · 8 · 128 · 2 · 2


def test_config3_ragged_lengths_are_seeded():
    c3 = bench.CONFIGS["3"]
    a, b = bench.cached_lengths(c3), bench.cached_lengths(c3)
    assert np.array_equal(a, b) and a.shape == (32,)
    assert a.min() >= 1024 and a.max() <= 8192
    assert int(a.sum()) + 32 == 137_887              # context tokens per step, as reported
    kv, _, _ = bench.step_bytes(c3, a + 1)
    assert kv == 137_887 * 8 * 128 * 2 * 2 * 32


def test_layer_launch_counts():
    assert bench.layer_launches(bench.LAYER_TYPES["q4_0"]) == 9
    assert bench.layer_launches(bench.LAYER_TYPES["q4_k_m"]) == 10   # v is Q6_K
    assert bench.layer_launches((1, 8, 2, 1, 2, 8, 1)) == 7 + 3 + 3  # every run split


def test_reference_numpy_path_sample_counts_its_bytes():
    """The reference arm's numpy-path leg (host append + ref_gqa_attention per
    sequence) times whole sequences and divides the bytes they read."""
    cfg = {"H": 4, "Hkv": 2, "D": 16, "seed": 3}
    ctx = np.array([5, 9])
    w = bench.CpuWorkload(cfg, ctx, threads=1)
    gbs, secs, n = bench.numpy_path_sample(w, min_seconds=0.01)
    assert n >= 1 and secs > 0 and gbs > 0
    per_seq = [int(c) * 2 * 16 * 2 * 2 + 4 * 16 * 2 * 2 for c in ctx]
    expect = sum(per_seq[i % 2] for i in range(n))
    assert abs(gbs * secs * 1e9 - expect) <= 1e-6 * expect
