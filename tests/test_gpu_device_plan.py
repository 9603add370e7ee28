"""The grouped GEMM prepared on the device (gg_device_plan_*), through the C-ABI (needs a B200).

The problem descriptors and their count are copied to device memory; the plan's preparation
kernel orders them, scans the tiles and writes the records on the device (no TMA descriptors: the
zero-fill loader and masked stores serve every problem). Checks: the order and tile offsets equal
gg_prepare's for every sort mode; D equals, bit for bit, the executor's D (host preparation, TMA
where aligned) for the same config and mode; the edge cases against the FP64 oracle; a run captured
in a CUDA graph follows problems changed on the device; a bad problem set computes nothing and
raises GG_STATUS_BAD_PROBLEMS.
"""
from __future__ import annotations

import numpy as np
import pytest

import grouped_gemm_gpu_kernel_b200 as gg
from grouped_gemm_gpu_kernel_b200 import capi
from grouped_gemm_gpu_kernel_b200 import workloads as W

from test_gpu_parity import EDGE_CASES, _check_edge, _edge_problem, check_full, run_grouped

pytestmark = pytest.mark.gpu

CONFIGS = [gg.KernelConfig(128, 256, 64), gg.KernelConfig(128, 128, 64), gg.KernelConfig(64, 64, 16),
           gg.KernelConfig(128, 64, 64), gg.KernelConfig(128, 128, 64, use_tensor_cores=False)]
MODES = (gg.SortMode.kNone, gg.SortMode.kByK, gg.SortMode.kByTiles, gg.SortMode.kByTilesThenK)


def _cfg_id(c):
    return f"{'' if c.use_tensor_cores else 'simt'}{c.cta_m}x{c.cta_n}x{c.cta_k}"


def _on_device(problems, device):
    import torch

    raw = gg.DevicePlan.pack_problems(problems)
    buf = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(device)
    count = torch.tensor([len(problems)], dtype=torch.int32, device=device)
    return buf, count


def _run_plan(plan, problems, device, mode, stream=None):
    import torch

    buf, count = _on_device(problems, device)
    assert plan.run(buf, count, mode, stream) == 0
    torch.cuda.synchronize()
    bits, total = plan.status()
    return bits, total


@pytest.mark.parametrize("cfg", CONFIGS, ids=_cfg_id)
def test_device_plan_matches_host_preparation(cuda, cfg):
    """small16 (odd pitches: zero-fill loads), mixed512 (TMA), tiny4096, every sort mode: the
    device order and offsets are gg_prepare's, and D is the executor's bit for bit."""
    import torch

    for name, modes in (("small16", MODES), ("mixed512", (gg.SortMode.kByK, gg.SortMode.kByTiles)),
                        ("tiny4096", (gg.SortMode.kNone, gg.SortMode.kByTilesThenK))):
        ps = W.allocate(W.make_shapes(name), cuda)
        probs = ps.problems()
        plan = gg.DevicePlan(cfg, min(len(probs) + 3, capi.GG_DEVICE_PLAN_MAX_PROBLEMS))  # spare slots past the count
        for mode in modes:
            prep = gg.prepare_problem_set(probs, cfg, mode)
            ps.d.fill_(float("nan"))
            run_grouped(probs, cfg, mode)
            want = ps.d.clone()
            ps.d.fill_(float("nan"))
            bits, total = _run_plan(plan, probs, cuda, mode)
            assert bits == 0 and total == prep.total_tiles, (name, mode)
            order, offs = plan.prepared(len(probs))
            assert order == prep.sorted_to_original, (name, mode)
            assert offs == prep.tile_offsets, (name, mode)
            assert torch.equal(torch.isnan(ps.d), torch.isnan(want)), (name, mode)
            assert torch.equal(torch.nan_to_num(ps.d), torch.nan_to_num(want)), (name, mode)
        plan.close()
        del ps


@pytest.mark.parametrize("cfg", [gg.KernelConfig(128, 128, 64), gg.KernelConfig(128, 256, 64)], ids=_cfg_id)
def test_device_plan_edge_cases(cuda, cfg):
    cases = [(_edge_problem(cuda, seed=i, **kw)) for i, kw in enumerate(EDGE_CASES.values())]
    probs = [p for p, _ in cases]
    plan = gg.DevicePlan(cfg, 64)
    bits, _ = _run_plan(plan, probs, cuda, gg.SortMode.kByTiles)
    assert bits == 0
    for (p, bufs), name in zip(cases, EDGE_CASES):
        try:
            _check_edge(p, bufs)
        except AssertionError as e:
            raise AssertionError(f"edge case {name}: {e}") from e
    plan.close()


def test_device_plan_follows_problems_changed_on_device_in_a_cuda_graph(cuda):
    """One captured run replayed over a different problem set and count written on the device."""
    import torch

    cfg = gg.KernelConfig(128, 128, 64)
    ps1 = W.allocate(W.make_shapes("small16"), cuda, seed=21)
    ps2 = W.allocate(W.make_shapes("mixed512"), cuda, seed=22)
    p1, p2 = ps1.problems(), ps2.problems()[:100]
    plan = gg.DevicePlan(cfg, 128)
    buf = torch.zeros(128 * 72, dtype=torch.uint8, device=cuda)
    count = torch.zeros(1, dtype=torch.int32, device=cuda)
    raw1 = torch.frombuffer(bytearray(gg.DevicePlan.pack_problems(p1)), dtype=torch.uint8).to(cuda)
    raw2 = torch.frombuffer(bytearray(gg.DevicePlan.pack_problems(p2)), dtype=torch.uint8).to(cuda)
    s = torch.cuda.Stream()
    buf[:raw1.numel()].copy_(raw1)
    count.fill_(len(p1))
    torch.cuda.synchronize()
    assert plan.run(buf, count, gg.SortMode.kByTiles, s) == 0  # outside the capture first
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        assert plan.run(buf, count, gg.SortMode.kByTiles, torch.cuda.current_stream()) == 0
    ps1.d.fill_(float("nan"))
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    assert plan.status() == (0, gg.prepare_problem_set(p1, cfg, 2).total_tiles)
    assert check_full(ps1) <= 1.0
    # new problems and count, written on the device; replay the same graph
    buf[:raw2.numel()].copy_(raw2)
    count.fill_(len(p2))
    ps2.d.fill_(float("nan"))
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    assert plan.status() == (0, gg.prepare_problem_set(p2, cfg, 2).total_tiles)
    want = ps2.d.clone()
    ps2.d.fill_(float("nan"))
    run_grouped(p2, cfg, gg.SortMode.kByTiles)
    assert torch.equal(torch.nan_to_num(ps2.d), torch.nan_to_num(want))
    del g
    plan.close()


def test_device_plan_rejects_bad_problem_sets(cuda):
    import dataclasses

    import torch

    cfg = gg.KernelConfig(128, 128, 64)
    ps = W.allocate(W.make_shapes("small16"), cuda, seed=23)
    probs = ps.problems()
    plan = gg.DevicePlan(cfg, 16)
    bad_sets = [
        [dataclasses.replace(probs[0], m=-1)] + probs[1:],   # negative dims
        probs[:3] + [dataclasses.replace(probs[3], a=None)],  # null A
        [dataclasses.replace(probs[0], ldd=1)] + probs[1:],  # ldd < n
    ]
    for bad in bad_sets:
        ps.d.fill_(float("nan"))
        bits, total = _run_plan(plan, bad, cuda, gg.SortMode.kNone)
        assert bits & capi.GG_STATUS_BAD_PROBLEMS and total == 0
        assert torch.isnan(ps.d).all()  # nothing computed
    # a count above the plan's capacity
    buf, _ = _on_device(probs, cuda)
    count = torch.tensor([17], dtype=torch.int32, device=cuda)
    assert plan.run(buf, count, 0) == 0
    bits, total = plan.status()
    assert bits & capi.GG_STATUS_BAD_PROBLEMS and total == 0
    # an empty set runs nothing
    count.zero_()
    assert plan.run(buf, count, 0) == 0
    assert plan.status() == (0, 0)
    # and a good set afterwards is computed
    ps.d.fill_(float("nan"))
    assert _run_plan(plan, probs, cuda, gg.SortMode.kByK)[0] == 0
    assert check_full(ps) <= 1.0
    plan.close()
