"""Host-side arithmetic of bench.py (no GPU): the reference's tail-work share, the roofline choice
and the strong-scaling shard of a fixed global set."""
from __future__ import annotations

import importlib.util
import os

import pytest

import grouped_gemm_gpu_kernel_b200 as gg
from grouped_gemm_gpu_kernel_b200 import workloads as W

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(REPO, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _probs(dims):
    return [gg.ProblemDesc(m, n, k, 1, 1, None, 1, max(1, k), max(1, n), max(1, n), max(1, n)) for m, n, k in dims]


def test_tail_work_share_follows_the_reference_definition(bench):
    # work = tiles x ceil(K / cta_k); the tail is the last max(1, n // 10) problems in launch order
    cfg = gg.KernelConfig(64, 64, 16)
    dims = [(128, 128, 64)] * 9 + [(64, 64, 16)]  # 9 x (4 tiles x 4 k-steps) + 1 x (1 x 1)
    prep = gg.prepare_problem_set(_probs(dims), cfg, gg.SortMode.kNone)
    assert bench.tail_work_share(prep, cfg.cta_k) == pytest.approx(1.0 / (9 * 16 + 1))
    prep = gg.prepare_problem_set(_probs(dims), cfg, gg.SortMode.kByTiles)  # small problem stays last
    assert bench.tail_work_share(prep, cfg.cta_k) == pytest.approx(1.0 / (9 * 16 + 1))
    dims2 = [(64, 64, 16)] + [(128, 128, 64)] * 9
    prep = gg.prepare_problem_set(_probs(dims2), cfg, gg.SortMode.kNone)
    assert bench.tail_work_share(prep, cfg.cta_k) == pytest.approx(16.0 / (9 * 16 + 1))
    assert bench.tail_work_share(gg.PreparedProblemSet(), 16) == 0.0
    # K = 0 problems own tiles but no K steps: no work in the tail when one comes last
    prep = gg.prepare_problem_set(_probs([(64, 64, 32), (64, 64, 0)]), cfg, gg.SortMode.kNone)
    assert bench.tail_work_share(prep, cfg.cta_k) == 0.0
    prep = gg.prepare_problem_set(_probs([(64, 64, 0), (64, 64, 32)]), cfg, gg.SortMode.kNone)
    assert bench.tail_work_share(prep, cfg.cta_k) == 1.0


def test_roofline_bound_follows_the_ridge_point(bench):
    peaks = {"hbm_gbs": 6000.0, "bf16_tflops": 1500.0, "source": "measured"}
    # 100 GFLOP over 1 GB: 100 FLOP/B < ridge 250 FLOP/B -> HBM-bound
    r = bench.roofline_of(100e9, 1e9, 0.5, peaks)
    assert r["bound"] == "hbm" and r["achieved"] == pytest.approx(2000.0) and r["frac"] == pytest.approx(2000 / 6000)
    # 1 TFLOP over 1 GB: above the ridge -> tensor-bound
    r = bench.roofline_of(1e12, 1e9, 1.0, peaks)
    assert r["bound"] == "tensor" and r["achieved"] == pytest.approx(1000.0) and r["frac"] == pytest.approx(1 / 1.5)
    # 8-bit inputs: twice the BF16 rate as the tensor peak
    r = bench.roofline_of(1e12, 1e9, 1.0, peaks, in_type=2)
    assert r["peak"] == pytest.approx(3000.0)


@pytest.mark.parametrize("name, world", [("skew", 2), ("skew", 8), ("moe", 4), ("mixed512", 3)])
def test_strong_shards_cover_the_global_set_once(bench, name, world):
    glob = W.make_shapes(name)
    cfg = gg.KernelConfig(*bench.DEFAULT_CTA[name])
    flops = 0.0
    weights = None
    for r in range(world):
        mine, w = bench.shard(glob, world, r, cfg)
        weights = w
        flops += mine.flops
        assert all(m > 0 and n > 0 for m, n, k in mine.dims)
    assert flops == pytest.approx(glob.flops, rel=1e-12)  # every output element exactly once
    assert len(weights) == world
    assert max(weights) / (sum(weights) / world) < 1.02  # tile-weighted split is balanced
