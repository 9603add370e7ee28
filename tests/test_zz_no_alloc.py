"""The no-allocation entry point gg_run_grouped_gemm_noalloc (needs a B200).

Some callers cannot call cudaMalloc: their device memory belongs to a caching allocator or pool
that forbids side allocations, or they sit on a latency-critical path where an allocation and
the synchronisation of the matching free are not acceptable. gg_run_grouped_gemm_noalloc serves
them from a fixed device array inside the library (at most GG_NOALLOC_MAX_PROBLEMS problems).

These tests call it through the C-ABI and hold its output to the output of the allocating entry
point gg_run_grouped_gemm_once on the same inputs, on two calls in a row with different problem
sets (the shared array keeps the previous call's contents, which must not leak into the next),
using the accuracy metric of the other GPU tests. This file is collected last on purpose.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import grouped_gemm_gpu_kernel_b200 as gg
import oracle as O
from grouped_gemm_gpu_kernel_b200 import capi
from grouped_gemm_gpu_kernel_b200 import workloads as W

pytestmark = pytest.mark.gpu


def noalloc(problems, mode, cfg, stream=None) -> int:
    arr = (capi.GGProblem * max(1, len(problems)))()
    for i, p in enumerate(problems):
        arr[i] = p.to_c()
    c = cfg.to_c()
    return capi.load().gg_run_grouped_gemm_noalloc(arr, len(problems), int(mode), ctypes.byref(c), stream)


def worst_vs(ps, got, want):
    """max over problems of (|got-want| / max(|want|, sqrt(K)/3)) / tolerance(K), U[-1,1] inputs."""
    worst = 0.0
    for i, (m, n, k) in enumerate(ps.shapes.dims):
        if m <= 0 or n <= 0:
            continue
        sl = slice(ps.d_off[i], ps.d_off[i] + m * n)
        x, y = got[sl].astype(np.float64), want[sl].astype(np.float64)
        scale = np.maximum(np.abs(y), np.sqrt(max(k, 1)) / 3.0)
        worst = max(worst, float((np.abs(x - y) / scale).max()) / O.tolerance(k))
    return worst


@pytest.mark.parametrize("cfg", [gg.KernelConfig(128, 128, 64), gg.KernelConfig(64, 64, 16)],
                         ids=lambda c: f"{c.cta_m}x{c.cta_n}")
def test_noalloc_matches_allocating_entry_point_on_two_calls(cuda, cfg):
    import torch

    calls = [("small16", 11, gg.SortMode.kByTiles), ("mixed512", 12, gg.SortMode.kByK)]
    for name, seed, mode in calls:
        ps = W.allocate(W.make_shapes(name), cuda, seed=seed)
        probs = ps.problems()
        assert gg.run_grouped_gemm_once(probs, mode, cfg) == 0
        torch.cuda.synchronize()
        want = ps.d.cpu().numpy()
        ps.d.fill_(float("nan"))
        torch.cuda.synchronize()
        assert noalloc(probs, mode, cfg) == 0
        torch.cuda.synchronize()
        got = ps.d.cpu().numpy()
        assert worst_vs(ps, got, want) <= 1.0, name
        assert np.array_equal(np.isnan(got), np.isnan(want)), name  # same elements written
        assert np.array_equal(got, want, equal_nan=True), name       # same kernel, same tiles: same bits


def test_noalloc_on_a_stream_and_repeated(cuda):
    import torch

    ps = W.allocate(W.make_shapes("small16"), cuda, seed=13)
    cfg = gg.KernelConfig(128, 128, 64)
    probs = ps.problems()
    assert gg.run_grouped_gemm_once(probs, gg.SortMode.kNone, cfg) == 0
    torch.cuda.synchronize()
    want = ps.d.cpu().numpy()
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    for _ in range(3):
        ps.d.fill_(float("nan"))
        torch.cuda.synchronize()
        assert noalloc(probs, gg.SortMode.kNone, cfg, s.cuda_stream) == 0
        s.synchronize()
        # the alignment gaps between problems stay NaN in both, so compare with equal_nan
        assert np.array_equal(ps.d.cpu().numpy(), want, equal_nan=True)


def test_noalloc_rejects_more_problems_than_its_scratch_holds(cuda):
    import torch

    n = capi.GG_NOALLOC_MAX_PROBLEMS + 1
    d = torch.full((n,), float("nan"), device=cuda)
    a = torch.zeros(n, dtype=torch.float16, device=cuda)
    probs = [gg.ProblemDesc(1, 1, 1, a.data_ptr() + 2 * i, a.data_ptr() + 2 * i, None, d.data_ptr() + 4 * i, 1, 1, 1, 1)
             for i in range(n)]
    assert noalloc(probs, gg.SortMode.kNone, gg.KernelConfig(128, 128, 64)) == 2  # cudaErrorMemoryAllocation
    torch.cuda.synchronize()
    assert torch.isnan(d).all()  # nothing was launched
    # the largest set it takes is accepted
    assert noalloc(probs[:-1], gg.SortMode.kNone, gg.KernelConfig(128, 128, 64)) == 0
    torch.cuda.synchronize()
    assert (d[:-1] == 0).all() and torch.isnan(d[-1])


def test_noalloc_does_not_change_free_device_memory(cuda):
    import torch

    ps = W.allocate(W.make_shapes("small16"), cuda, seed=14)
    cfg = gg.KernelConfig(128, 128, 64)
    assert noalloc(ps.problems(), gg.SortMode.kByTiles, cfg) == 0  # first call on the device: set-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(5):
        assert noalloc(ps.problems(), gg.SortMode.kByTiles, cfg) == 0
        assert gg.noalloc_status() == 0  # the status query allocates nothing either
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_noalloc_status_word_reports_a_timeout_then_clears(cuda):
    """gg_noalloc_status reads the status word kept in the fixed array: a timeout recorded there
    (by the bounded-wait self-test, which runs the kernel's wait on a barrier nothing completes)
    reaches the query once and is cleared by it, and every call clears the word before it launches."""
    ps = W.allocate(W.make_shapes("small16"), cuda, seed=15)
    cfg = gg.KernelConfig(128, 128, 64)
    assert noalloc(ps.problems(), gg.SortMode.kNone, cfg) == 0
    assert gg.noalloc_status() == 0
    assert gg.selftest_wait_timeout_word(capi.GG_STATUS_WORD_NOALLOC, 5_000_000) == 0
    bits = gg.noalloc_status()
    assert bits & capi.GG_STATUS_TIMEOUT_MMA and not (bits & 0x100)
    assert gg.noalloc_status() == 0
    assert gg.selftest_wait_timeout_word(capi.GG_STATUS_WORD_NOALLOC, 5_000_000) == 0
    assert noalloc(ps.problems(), gg.SortMode.kNone, cfg) == 0
    assert gg.noalloc_status() == 0
