"""Parity of the sm_100a kernel with the oracle, through the C-ABI (needs a B200).

Accuracy bar: for every checked element
    |D - D_fp64| / max(|D_fp64|, scale)  <=  2e-3 * sqrt(max(K, 1) / 1024)
with scale = |alpha| * sqrt(sum_k (a_ik b_kj)^2) + |beta c_ij| from the FP64 oracle
(oracle.rel_err / oracle.tolerance). Small configurations are checked in full; the full-size
ones (mixed512, moe, skew) on sampled rows and columns. The reference test's own inputs are
also held to its own absolute tolerance of 2e-2 against its own host GEMM output
(reference tests/test_correctness.cu:357).
"""
from __future__ import annotations

import os
import subprocess
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import grouped_gemm_gpu_kernel_b200 as gg
import oracle as O
from grouped_gemm_gpu_kernel_b200 import capi
from grouped_gemm_gpu_kernel_b200 import workloads as W

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ALL_CONFIGS = gg.REFERENCE_CONFIGS + gg.NATIVE_CONFIGS
MODES = (gg.SortMode.kNone, gg.SortMode.kByK, gg.SortMode.kByTiles, gg.SortMode.kByTilesThenK)
# CTA-pair configs whose executors cut problems into pair blocks and one-CTA rows (tile classes)
TILE_CLASS_CONFIGS = (gg.KernelConfig(256, 256, 64, tile_classes=gg.TileClasses.kPairBlocks),
                      gg.KernelConfig(256, 128, 64, tile_classes=gg.TileClasses.kPairBlocks))


def _cfg_id(c):
    return f"{c.cta_m}x{c.cta_n}" + ("-classes" if c.tile_classes else "")


def _torch():
    import torch

    return torch


def run_grouped(problems, cfg, mode, stream=None, check_status=True):
    torch = _torch()
    prep = gg.prepare_problem_set(problems, cfg, mode)
    ex = gg.GroupedGemmExecutor()
    st = ex.build(prep, cfg)
    assert st == 0, f"build failed: {st}"
    st = ex.run(stream)
    assert st == 0, f"run failed: {st}"
    torch.cuda.synchronize()
    if check_status:
        assert ex.status() == 0, "a bounded wait timed out inside the kernel"
    return ex


class HostSlabs:
    """Host copies of a DeviceProblemSet's slabs, sliced per problem for the oracle."""

    def __init__(self, ps: W.DeviceProblemSet):
        torch = _torch()
        self.ps = ps
        self.a = ps.a.view(torch.int16).cpu().numpy().view(np.uint16)
        self.b = ps.b.view(torch.int16).cpu().numpy().view(np.uint16)
        self.c = ps.c.cpu().numpy() if ps.c is not None else None
        self.d = ps.d.cpu().numpy()

    def problem(self, i):
        m, n, k = self.ps.shapes.dims[i]
        a = self.a[self.ps.a_off[i]:self.ps.a_off[i] + max(m * k, 1)]
        b = self.b[self.ps.b_off[i]:self.ps.b_off[i] + max(k * n, 1)]
        c = self.c[self.ps.c_off[i]:self.ps.c_off[i] + max(m * n, 1)] if self.c is not None else None
        d = self.d[self.ps.d_off[i]:self.ps.d_off[i] + max(m * n, 0)]
        return a, b, c, d


def check_full(ps: W.DeviceProblemSet, threads: int = 8, fmt: int = 0) -> float:
    """Every element of every problem against the FP64 oracle; returns the worst error/tolerance.
    fmt: the A/B element type of the run (0 FP16, 1 BF16)."""
    hs = HostSlabs(ps)

    def one(i):
        m, n, k = ps.shapes.dims[i]
        if m <= 0 or n <= 0:
            return 0.0
        a, b, c, d = hs.problem(i)
        ref, scale = O.gemm_f64(m, n, k, a, max(1, k), b, max(1, n), c, max(1, n), ps.shapes.alpha[i], ps.shapes.beta[i],
                                fmt=fmt)
        return O.rel_err(d.reshape(m, n), ref, scale) / O.tolerance(k)

    with ThreadPoolExecutor(threads) as pool:
        worst = max(pool.map(one, range(len(ps.shapes.dims))), default=0.0)
    return worst


def check_sampled(ps: W.DeviceProblemSet, rows_per=4, cols_per=96, seed=0, threads=8, fmt=0) -> float:
    rng = np.random.default_rng(seed)
    jobs = []
    for i, (m, n, k) in enumerate(ps.shapes.dims):
        if m <= 0 or n <= 0:
            continue
        rows = np.unique(np.concatenate([[0, m - 1], rng.integers(0, m, size=rows_per)])).astype(np.int64)
        cols = np.unique(np.concatenate([[0, n - 1], rng.integers(0, n, size=cols_per)])).astype(np.int64)
        h = W.host_inputs(ps, i, rows, cols)
        jobs.append((i, len(rows), len(cols), k, h))

    def one(job):
        i, r, c, k, h = job
        ref, scale = O.gemm_f64(r, c, k, h["a"], max(1, k), h["b"], c, h["c"], c, ps.shapes.alpha[i], ps.shapes.beta[i],
                                fmt=fmt)
        return O.rel_err(h["d"], ref, scale) / O.tolerance(k)

    with ThreadPoolExecutor(threads) as pool:
        return max(pool.map(one, jobs), default=0.0)


# ---------------------------------------------------------------------------------------------
def test_bounded_wait_selftest_reports_timeout_and_context_survives(cuda):
    torch = _torch()
    st, bits = gg.selftest_wait_timeout(5_000_000)
    assert st == 0
    assert bits & capi.GG_STATUS_TIMEOUT_MMA and not (bits & 0x100)
    x = torch.ones(1024, device=cuda)
    assert float(x.sum()) == 1024.0


def test_baseline_status_word_reports_a_timeout_then_clears(cuda):
    """gg_baseline_status reads the per-device word of the per-problem baseline: the self-test's
    timeout recorded there reaches the query once, and the query clears it."""
    torch = _torch()
    ps = W.allocate(W.make_shapes("small16"), cuda)
    assert gg.run_baseline_per_problem(ps.problems(), gg.KernelConfig(128, 128, 64)) == 0
    assert gg.baseline_status() == 0
    assert gg.selftest_wait_timeout_word(capi.GG_STATUS_WORD_BASELINE, 5_000_000) == 0
    bits = gg.baseline_status()
    assert bits & capi.GG_STATUS_TIMEOUT_MMA and not (bits & 0x100)
    assert gg.baseline_status() == 0
    ps.d.fill_(float("nan"))
    assert gg.run_baseline_per_problem(ps.problems(), gg.KernelConfig(128, 128, 64)) == 0
    assert gg.baseline_status() == 0
    assert check_full(ps) <= 1.0
    assert gg.selftest_wait_timeout_word(7, 1_000_000) == capi.CUDA_ERROR_INVALID_VALUE
    assert float(torch.ones(8, device=cuda).sum()) == 8.0


def test_run_once_reads_its_status_word(cuda):
    """run_grouped_gemm_once synchronises and checks its kernel's status before it returns
    (a timeout would return cudaErrorLaunchTimeout); a normal call returns success."""
    ps = W.allocate(W.make_shapes("small16"), cuda)
    for cfg in (gg.KernelConfig(128, 128, 64), gg.KernelConfig(128, 128, 64, use_tensor_cores=False)):
        ps.d.fill_(float("nan"))
        assert gg.run_grouped_gemm_once(ps.problems(), gg.SortMode.kByK, cfg) == 0
        assert check_full(ps) <= 1.0


def test_occupancy_report(cuda):
    for cfg in ALL_CONFIGS:
        st, info = gg.query_occupancy(cfg)
        assert st == 0
        assert info.sm_count >= 100 and info.active_blocks_per_sm == 1 and info.threads_per_block == 384
        assert info.warps_per_block == 12 and info.using_tensor_cores
        assert 100_000 < info.dynamic_shared_bytes <= 232_448
        assert 0 < info.registers_per_thread <= 168 and info.registers_per_block == info.registers_per_thread * 384
        assert info.theoretical_occupancy == pytest.approx(12 / info.max_warps_per_sm)


def test_single_tile_tma_path(cuda):
    torch = _torch()
    g = torch.Generator(device=cuda).manual_seed(1)
    A = torch.empty(128, 64, dtype=torch.float16, device=cuda).uniform_(-1, 1, generator=g)
    B = torch.empty(64, 128, dtype=torch.float16, device=cuda).uniform_(-1, 1, generator=g)
    D = torch.full((128, 128), float("nan"), device=cuda)
    p = gg.problem_from_tensors(A, B, None, D)
    run_grouped([p], gg.KernelConfig(128, 128, 64), gg.SortMode.kNone)
    ref = A.double() @ B.double()
    assert torch.allclose(D.double(), ref, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("bn", [128, 256])
def test_single_tile_pair_path(cuda, bn):
    """One 256 x BN tile on a CTA pair (cta_group::2): both halves of A and B, both TMEMs."""
    torch = _torch()
    g = torch.Generator(device=cuda).manual_seed(2)
    A = torch.empty(256, 128, dtype=torch.float16, device=cuda).uniform_(-1, 1, generator=g)
    B = torch.empty(128, bn, dtype=torch.float16, device=cuda).uniform_(-1, 1, generator=g)
    D = torch.full((256, bn), float("nan"), device=cuda)
    p = gg.problem_from_tensors(A, B, None, D)
    ex = run_grouped([p], gg.KernelConfig(256, bn, 64), gg.SortMode.kNone)
    assert ex.grid_ctas() == 2 and ex.total_tiles() == 1
    ref = A.double() @ B.double()
    assert torch.allclose(D.double(), ref, rtol=1e-5, atol=1e-4)


def _fixture_problems(cuda):
    """The reference test's eight problems with its own inputs, on the device."""
    torch = _torch()
    from tests.test_oracle import ref_test_problems

    probs, keep, refs = [], [], []
    for p in ref_test_problems():
        a = torch.from_numpy(p["a"].view(np.int16).copy()).to(cuda).view(torch.float16)
        b = torch.from_numpy(p["b"].view(np.int16).copy()).to(cuda).view(torch.float16)
        c = torch.from_numpy(p["c"].copy()).to(cuda)
        d = torch.full((O.safe_elems(p["m"], p["ldd"]),), float("nan"), device=cuda)
        keep += [a, b, c, d]
        probs.append(gg.ProblemDesc(p["m"], p["n"], p["k"], a.data_ptr(), b.data_ptr(), c.data_ptr(), d.data_ptr(),
                                    p["lda"], p["ldb"], p["ldc"], p["ldd"], p["alpha"], p["beta"]))
        refs.append((p, d))
    return probs, keep, refs


def _check_fixture(refs):
    for p, d in refs:
        m, n, k = p["m"], p["n"], p["k"]
        if m <= 0 or n <= 0:
            continue
        got = d.cpu().numpy()[:m * n].reshape(m, n)
        want = p["ref"][:m * n].reshape(m, n)
        assert np.abs(got - want).max() <= 2e-2  # the reference test's own bar
        ref64, scale = O.gemm_f64(m, n, k, p["a"], p["lda"], p["b"], p["ldb"], p["c"], p["ldc"], p["alpha"], p["beta"])
        assert O.rel_err(got, ref64, scale) <= O.tolerance(k), (m, n, k)


@pytest.mark.parametrize("cfg", ALL_CONFIGS, ids=lambda c: f"{c.cta_m}x{c.cta_n}x{c.cta_k}")
def test_reference_test_set_all_modes_and_baseline(cuda, cfg):
    """The reference test's matrix (tests/test_correctness.cu:309-362) on every config."""
    torch = _torch()
    probs, keep, refs = _fixture_problems(cuda)
    for mode in MODES:
        for _, d in refs:
            d.fill_(float("nan"))
        assert gg.run_grouped_gemm_once(probs, mode, cfg) == 0
        torch.cuda.synchronize()
        _check_fixture(refs)
    for _, d in refs:
        d.fill_(float("nan"))
    assert gg.run_baseline_per_problem(probs, cfg) == 0
    torch.cuda.synchronize()
    _check_fixture(refs)
    assert gg.run_grouped_gemm_once([], gg.SortMode.kByTiles, cfg) == 0
    assert gg.run_baseline_per_problem([], cfg) == 0


@pytest.mark.parametrize("cfg", [gg.KernelConfig(128, 128, 64), gg.KernelConfig(64, 64, 16),
                                 gg.KernelConfig(128, 256, 64), gg.KernelConfig(256, 128, 64),
                                 gg.KernelConfig(256, 256, 64)], ids=lambda c: f"{c.cta_m}x{c.cta_n}")
def test_small16_full(cuda, cfg):
    ps = W.allocate(W.make_shapes("small16"), cuda)
    for mode in MODES:
        ps.d.fill_(float("nan"))
        run_grouped(ps.problems(), cfg, mode)
        assert check_full(ps) <= 1.0
    ps.d.fill_(float("nan"))
    assert gg.run_baseline_per_problem(ps.problems(), cfg) == 0
    _torch().cuda.synchronize()
    assert check_full(ps) <= 1.0


@pytest.mark.parametrize("cfg", [gg.KernelConfig(128, 128, 64), gg.KernelConfig(64, 64, 16),
                                 gg.KernelConfig(256, 128, 64)], ids=lambda c: f"{c.cta_m}x{c.cta_n}")
def test_tiny4096_full(cuda, cfg):
    ps = W.allocate(W.make_shapes("tiny4096"), cuda)
    run_grouped(ps.problems(), cfg, gg.SortMode.kByTiles)
    assert check_full(ps) <= 1.0


@pytest.mark.parametrize("cfg", [gg.KernelConfig(128, 128, 64), gg.KernelConfig(64, 64, 16), gg.KernelConfig(128, 64, 64),
                                 gg.KernelConfig(256, 128, 64), gg.KernelConfig(128, 128, 64, use_tensor_cores=False)],
                         ids=lambda c: f"{'' if c.use_tensor_cores else 'simt'}{c.cta_m}x{c.cta_n}")
def test_exhaustive_small_dims(cuda, cfg):
    """Every (m, n, k) in 1..17 (4913 problems, packed odd leading dimensions, beta != 0), one
    grouped launch, every element against the FP64 oracle; the gaps between problems' D untouched."""
    dims = [(m, n, k) for m in range(1, 18) for n in range(1, 18) for k in range(1, 18)]
    shapes = W.Shapes("exhaustive17", dims, [1.25] * len(dims), [-0.75] * len(dims), True)
    ps = W.allocate(shapes, cuda, seed=17)
    run_grouped(ps.problems(), cfg, gg.SortMode.kByTiles)
    assert check_full(ps) <= 1.0
    d = ps.d.cpu().numpy()
    written = np.zeros(d.size, bool)
    for i, (m, n, k) in enumerate(dims):
        written[ps.d_off[i]:ps.d_off[i] + m * n] = True
    assert np.isnan(d[~written]).all()


def test_mixed512_all_modes_sampled(cuda):
    ps = W.allocate(W.make_shapes("mixed512"), cuda)
    for mode in MODES:
        ps.d.fill_(float("nan"))
        run_grouped(ps.problems(), gg.KernelConfig(128, 128, 64), mode)
        assert check_sampled(ps, seed=int(mode)) <= 1.0
    for i, cfg in enumerate((gg.KernelConfig(128, 256, 64), gg.KernelConfig(256, 128, 64),
                             gg.KernelConfig(256, 256, 64))):
        ps.d.fill_(float("nan"))
        run_grouped(ps.problems(), cfg, gg.SortMode.kByTiles)
        assert check_sampled(ps, seed=7 + i) <= 1.0
    # canaries: the 256-byte alignment gaps between problems' D are never written
    d = ps.d.cpu().numpy()
    written = np.zeros(d.size, bool)
    for i, (m, n, k) in enumerate(ps.shapes.dims):
        written[ps.d_off[i]:ps.d_off[i] + m * n] = True
    assert np.isnan(d[~written]).all()
    assert np.isfinite(d[written]).all()


@pytest.mark.slow
@pytest.mark.parametrize("cfg", [gg.KernelConfig(128, 256, 64), gg.KernelConfig(256, 256, 64)],
                         ids=lambda c: f"{c.cta_m}x{c.cta_n}")
def test_moe_full_size_sampled(cuda, cfg):
    ps = W.allocate(W.make_shapes("moe"), cuda)
    run_grouped(ps.problems(), cfg, gg.SortMode.kByTiles)
    assert check_sampled(ps, rows_per=3, cols_per=64) <= 1.0
    del ps


@pytest.mark.slow
@pytest.mark.parametrize("cfg", [gg.KernelConfig(128, 256, 64), gg.KernelConfig(256, 256, 64)],
                         ids=lambda c: f"{c.cta_m}x{c.cta_n}")
def test_skew_full_size_sampled(cuda, cfg):
    ps = W.allocate(W.make_shapes("skew"), cuda)
    run_grouped(ps.problems(), cfg, gg.SortMode.kByTiles)
    assert check_sampled(ps, rows_per=6, cols_per=64) <= 1.0


@pytest.mark.parametrize("cfg", TILE_CLASS_CONFIGS, ids=_cfg_id)
def test_tile_classes_match_oracle(cuda, cfg):
    """Tile classes: every problem's whole 256-row blocks on CTA pairs, the rows left over on one-CTA
    tiles (two launches). small16 in full; mixed512 and the MoE layer sampled, with the gaps between
    problems' D untouched; the executor still reports the prepared set's 256-row tiling."""
    torch = _torch()
    ps = W.allocate(W.make_shapes("small16"), cuda)
    for mode in (gg.SortMode.kNone, gg.SortMode.kByTiles):
        ps.d.fill_(float("nan"))
        run_grouped(ps.problems(), cfg, mode)
        assert check_full(ps) <= 1.0
    ps = W.allocate(W.make_shapes("mixed512"), cuda)
    prep = gg.prepare_problem_set(ps.problems(), cfg, gg.SortMode.kByK)
    ex = run_grouped(ps.problems(), cfg, gg.SortMode.kByK)
    assert ex.total_tiles() == prep.total_tiles and ex.problem_count() == 512
    assert check_sampled(ps, seed=3) <= 1.0
    d = ps.d.cpu().numpy()
    written = np.zeros(d.size, bool)
    for i, (m, n, k) in enumerate(ps.shapes.dims):
        written[ps.d_off[i]:ps.d_off[i] + m * n] = True
    assert np.isnan(d[~written]).all() and np.isfinite(d[written]).all()
    # same results as the one-variant pair launch, within the accuracy bound
    ref = ps.d.clone()
    ps.d.fill_(float("nan"))
    run_grouped(ps.problems(), gg.KernelConfig(cfg.cta_m, cfg.cta_n, 64), gg.SortMode.kByK)
    worst = 0.0
    for i, (m, n, k) in enumerate(ps.shapes.dims):
        sl = slice(ps.d_off[i], ps.d_off[i] + m * n)
        x, y = ps.d[sl].double(), ref[sl].double()
        worst = max(worst, float(((x - y).abs() / torch.clamp(y.abs(), min=float(np.sqrt(k) / 3))).max()) / O.tolerance(k))
    assert worst <= 1.0
    del ps, ref
    if cfg.cta_n == 256:
        ps = W.allocate(W.make_shapes("moe"), cuda)
        run_grouped(ps.problems(), cfg, gg.SortMode.kByTiles)
        assert check_sampled(ps, rows_per=3, cols_per=64) <= 1.0
        del ps


@pytest.mark.parametrize("cfg", [gg.KernelConfig(128, 64, 64, tile_classes=gg.TileClasses.kSmallOnCudaCores),
                                 gg.KernelConfig(128, 256, 64, tile_classes=gg.TileClasses.kSmallOnCudaCores)],
                         ids=lambda c: f"{c.cta_m}x{c.cta_n}")
def test_small_problems_on_cuda_cores(cuda, cfg):
    """Tile class 'small on CUDA cores': problems with m, n, k <= 64, and problems of at most
    2^25 multiply-adds that TMA cannot load (odd pitches), on the CUDA-core kernel with 64 x 64
    tiles; the others (aligned, or odd and larger) on the tensor cores. tiny4096 (all small),
    small16 (odd pitches, mostly routed to the CUDA cores) and a set mixing every kind, every
    element against the FP64 oracle."""
    ps = W.allocate(W.make_shapes("tiny4096"), cuda)
    run_grouped(ps.problems(), cfg, gg.SortMode.kByTiles)
    assert check_full(ps) <= 1.0
    ps = W.allocate(W.make_shapes("small16"), cuda)
    run_grouped(ps.problems(), cfg, gg.SortMode.kByK)
    assert check_full(ps) <= 1.0
    rng = np.random.default_rng(8)
    dims = [(int(rng.integers(1, 65)), int(rng.integers(1, 65)), int(rng.integers(1, 65))) for _ in range(200)]
    dims += [(int(8 * rng.integers(8, 40)), int(8 * rng.integers(8, 40)), int(8 * rng.integers(1, 40)))
             for _ in range(40)]
    dims += [(int(2 * rng.integers(33, 160) + 1), int(2 * rng.integers(33, 160) + 1), int(2 * rng.integers(33, 160) + 1))
             for _ in range(20)]                      # odd pitches, mostly below the volume bound
    dims += [(333, 331, 337), (321, 513, 257)]        # odd pitches above it: tensor cores, zero-fill loader
    order = rng.permutation(len(dims))
    shapes = W.Shapes("mixed_small", [dims[i] for i in order], [1.5] * len(dims), [0.25] * len(dims), True)
    ps = W.allocate(shapes, cuda, seed=9)
    for mode in (gg.SortMode.kNone, gg.SortMode.kByTiles):
        ps.d.fill_(float("nan"))
        run_grouped(ps.problems(), cfg, mode)
        assert check_full(ps) <= 1.0


@pytest.mark.parametrize("fmt", [0, 1], ids=["fp16", "bf16"])
def test_small_class_realigns_large_odd_pitches(cuda, fmt):
    """Tile class 'small on CUDA cores', problems above 2^25 multiply-adds whose A or B TMA cannot
    load (packed odd pitches): each run copies those operands into 16-byte-aligned scratch and
    the tensor cores load the copies by TMA. The tensor cores compute the same MMAs in the same
    order as with the zero-fill loader (the class off), so D is bit-identical; and every element
    against the FP64 oracle. A only, B only and both misaligned."""
    torch = _torch()
    dims = [(321, 333, 345), (333, 320, 345), (333, 321, 344), (512, 264, 300), (300, 1000, 129)]
    assert all(m * n * k > capi.GG_SMALL_ZERO_FILL_VOLUME for m, n, k in dims)
    shapes = W.Shapes("odd_large", dims, [1.25] * len(dims), [0.5] * len(dims), True)
    ps = W.allocate(shapes, cuda, seed=11)
    if fmt == 1:
        ps = ps.to_bf16()
    outs = []
    for classes in (gg.TileClasses.kNone, gg.TileClasses.kSmallOnCudaCores):
        ps.d.fill_(float("nan"))
        run_grouped(ps.problems(), gg.KernelConfig(128, 256, 64, input_type=fmt, tile_classes=classes),
                    gg.SortMode.kByTiles)
        torch.cuda.synchronize()
        outs.append(ps.d.clone())
    # bit patterns (the NaN fill stays in the slab's padding between problems)
    assert torch.equal(outs[0].view(torch.int32), outs[1].view(torch.int32))
    assert check_full(ps, fmt=fmt) <= 1.0


def test_executor_launches_per_run(cuda):
    """gg_executor_launches: 1 without tile classes; with the small-problem class one launch per
    non-empty part plus the operand copy when a problem is realigned."""
    def launches(shapes, classes):
        ps = W.allocate(shapes, cuda, seed=3)
        cfg = gg.KernelConfig(128, 256, 64, tile_classes=classes)
        ex = gg.GroupedGemmExecutor()
        assert ex.build(gg.prepare_problem_set(ps.problems(), cfg, gg.SortMode.kByTiles), cfg) == 0
        n = ex.launches()
        ex.close()
        return n
    tiny = W.Shapes("t", [(5, 7, 9), (64, 64, 64)], [1.0] * 2, [0.0] * 2, True)
    both = W.Shapes("b", [(5, 7, 9), (256, 256, 256)], [1.0] * 2, [0.0] * 2, True)
    odd = W.Shapes("o", [(5, 7, 9), (321, 333, 345)], [1.0] * 2, [0.0] * 2, True)
    assert launches(tiny, gg.TileClasses.kNone) == 1
    assert launches(tiny, gg.TileClasses.kSmallOnCudaCores) == 1      # CUDA-core part only
    assert launches(both, gg.TileClasses.kSmallOnCudaCores) == 2      # tensor-core + CUDA-core parts
    assert launches(odd, gg.TileClasses.kSmallOnCudaCores) == 3       # + the operand copy


@pytest.mark.parametrize("cfg", [gg.KernelConfig(128, 256, 64), gg.KernelConfig(256, 256, 64),
                                 gg.KernelConfig(128, 64, 64, use_tensor_cores=False),
                                 gg.KernelConfig(128, 256, 64, tile_classes=gg.TileClasses.kSmallOnCudaCores),
                                 gg.KernelConfig(256, 256, 64, tile_classes=gg.TileClasses.kPairBlocks)],
                         ids=_cfg_id)
def test_runs_back_to_back_reset_their_own_counters(cuda, cfg):
    """An executor run is its kernel launches alone: the last CTA of each launch sets the tile
    counter back to zero. Five runs in a row on one stream, with no host work between them, each
    writing D from NaN: every run computes every tile (bit-identical D each time)."""
    torch = _torch()
    shapes = W.Shapes("mix", [(200, 300, 100), (7, 9, 11), (513, 129, 64), (64, 64, 64), (1, 1000, 33)],
                      [1.0] * 5, [0.5] * 5, True)
    ps = W.allocate(shapes, cuda, seed=5)
    ex = gg.GroupedGemmExecutor()
    assert ex.build(gg.prepare_problem_set(ps.problems(), cfg, gg.SortMode.kByTiles), cfg) == 0
    stream = torch.cuda.current_stream()
    outs = []
    for _ in range(5):
        ps.d.fill_(float("nan"))
        assert ex.run(stream) == 0
        outs.append(ps.d.clone())
    torch.cuda.synchronize()
    assert ex.status() == 0
    ex.close()
    for o in outs[1:]:
        assert torch.equal(o.view(torch.int32), outs[0].view(torch.int32))
    assert check_full(ps) <= 1.0


def test_determinism_bitwise(cuda):
    torch = _torch()
    ps = W.allocate(W.make_shapes("mixed512"), cuda)
    cfg = gg.KernelConfig(128, 128, 64)
    run_grouped(ps.problems(), cfg, gg.SortMode.kByTiles)
    first = ps.d.clone()
    ps.d.fill_(0.0)
    run_grouped(ps.problems(), cfg, gg.SortMode.kNone)
    assert torch.equal(first, ps.d)


def test_executor_run_captured_in_cuda_graph(cuda):
    """gg_executor_run (counter reset + launch) replays from a CUDA graph with the same result."""
    torch = _torch()
    ps = W.allocate(W.make_shapes("small16"), cuda)
    for cfg in (gg.KernelConfig(128, 256, 64), gg.KernelConfig(256, 128, 64)):
        ex = gg.GroupedGemmExecutor()
        assert ex.build(gg.prepare_problem_set(ps.problems(), cfg, gg.SortMode.kByK), cfg) == 0
        s = torch.cuda.Stream(cuda)
        torch.cuda.synchronize()
        assert ex.run(s) == 0
        torch.cuda.synchronize()
        eager = ps.d.clone()
        ps.d.fill_(float("nan"))
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(3):
                assert ex.run(torch.cuda.current_stream()) == 0
        g.replay()
        torch.cuda.synchronize()
        assert ex.status() == 0
        # alignment gaps between the problems' D blocks hold NaN canaries in both copies
        assert torch.equal(torch.nan_to_num(eager, nan=7.0), torch.nan_to_num(ps.d, nan=7.0))
        del g
        ex.close()


def _edge_problem(cuda, m, n, k, lda=None, ldb=None, ldc=None, ldd=None, alpha=1.0, beta=0.0, a_shift=0,
                  b_shift=0, c_mode="rand", seed=0):
    """One problem with its own buffers; shifts misalign the base pointers by 2-byte steps."""
    torch = _torch()
    lda = lda or max(1, k)
    ldb = ldb or max(1, n)
    ldc = ldc or max(1, n)
    ldd = ldd or max(1, n)
    g = torch.Generator(device=cuda).manual_seed(seed)
    A = torch.empty(O.safe_elems(m, lda) + 8, dtype=torch.float16, device=cuda).uniform_(-1, 1, generator=g)
    B = torch.empty(O.safe_elems(k, ldb) + 8, dtype=torch.float16, device=cuda).uniform_(-1, 1, generator=g)
    C = torch.empty(O.safe_elems(m, ldc), dtype=torch.float32, device=cuda).uniform_(-1, 1, generator=g)
    if c_mode == "nan":
        C.fill_(float("nan"))
    D = torch.full((O.safe_elems(m, ldd) + 64,), float("nan"), device=cuda)
    cptr = None if c_mode == "null" else C.data_ptr()
    p = gg.ProblemDesc(m, n, k, A.data_ptr() + 2 * a_shift, B.data_ptr() + 2 * b_shift, cptr, D.data_ptr(),
                       lda, ldb, ldc, ldd, alpha, beta)
    return p, (A, B, C, D, a_shift, b_shift, c_mode)


def _check_edge(p, bufs):
    A, B, C, D, a_shift, b_shift, c_mode = bufs
    m, n, k = p.m, p.n, p.k
    a = A.view(_torch().int16).cpu().numpy().view(np.uint16)[a_shift:]
    b = B.view(_torch().int16).cpu().numpy().view(np.uint16)[b_shift:]
    c = None if c_mode == "null" else C.cpu().numpy()
    d = D.cpu().numpy()
    if m <= 0 or n <= 0:
        assert np.isnan(d).all()
        return
    ref, scale = O.gemm_f64(m, n, k, a, p.lda, b, p.ldb, c, p.ldc, p.alpha, p.beta)
    got = np.stack([d[r * p.ldd:r * p.ldd + n] for r in range(m)])
    assert O.rel_err(got, ref, scale) <= O.tolerance(k), (m, n, k)
    # nothing outside the m x n window of D was written (row padding and the trailing guard)
    mask = np.ones(d.size, bool)
    for r in range(m):
        mask[r * p.ldd:r * p.ldd + n] = False
    assert np.isnan(d[mask]).all()


EDGE_CASES = {
    "k0_beta_c": dict(m=70, n=50, k=0, beta=0.75),
    "k0_beta0": dict(m=130, n=136, k=0, beta=0.0),
    "beta0_nan_c": dict(m=96, n=80, k=64, beta=0.0, c_mode="nan"),
    "null_c_beta": dict(m=40, n=72, k=24, beta=0.9, c_mode="null"),
    "alpha0": dict(m=33, n=65, k=17, alpha=0.0, beta=1.0),
    "one_by_one": dict(m=1, n=1, k=1),
    "k1_wide": dict(m=3, n=300, k=1),
    "k_not_mult_64": dict(m=128, n=128, k=1000),
    "deep_k": dict(m=130, n=264, k=4160),
    "padded_aligned_ld": dict(m=200, n=136, k=72, lda=80, ldb=144, ldc=140, ldd=144, beta=-1.0),
    "padded_odd_ld": dict(m=77, n=51, k=35, lda=41, ldb=53, ldc=55, ldd=57, beta=0.5),
    "misaligned_a": dict(m=128, n=128, k=128, a_shift=1),
    "misaligned_b": dict(m=100, n=256, k=192, b_shift=3),
    "lda_lt_8_mult": dict(m=64, n=64, k=64, lda=68),
    "n8": dict(m=300, n=8, k=96),
    "m_exact_tiles": dict(m=256, n=512, k=128, beta=0.25),
    "packed_small_misaligned": dict(m=50, n=40, k=37, a_shift=1, b_shift=3, beta=0.5),
    "packed_k64_misaligned": dict(m=70, n=200, k=64, a_shift=1, b_shift=1),
    # rows past whole 256-row blocks (tile classes put them on one-CTA tiles)
    "rows_513_odd_ld": dict(m=513, n=264, k=200, lda=203, ldc=266, ldd=265, beta=0.5),
    "rows_767_aligned": dict(m=767, n=256, k=128, beta=-0.5),
}


@pytest.mark.parametrize("cfg", [gg.KernelConfig(128, 128, 64), gg.KernelConfig(64, 128, 32),
                                 gg.KernelConfig(128, 64, 32), gg.KernelConfig(256, 128, 64),
                                 gg.KernelConfig(256, 256, 64)] + list(TILE_CLASS_CONFIGS), ids=_cfg_id)
def test_edge_cases(cuda, cfg):
    cases = [(_edge_problem(cuda, seed=i, **kw)) for i, kw in enumerate(EDGE_CASES.values())]
    probs = [p for p, _ in cases]
    run_grouped(probs, cfg, gg.SortMode.kByTiles)
    for (p, bufs), name in zip(cases, EDGE_CASES):
        try:
            _check_edge(p, bufs)
        except AssertionError as e:
            raise AssertionError(f"edge case {name}: {e}") from e


SIMT_CONFIGS = [gg.KernelConfig(64, 64, 16, use_tensor_cores=False), gg.KernelConfig(128, 64, 32, use_tensor_cores=False),
                gg.KernelConfig(128, 256, 64, use_tensor_cores=False), gg.KernelConfig(256, 128, 64, use_tensor_cores=False)]


@pytest.mark.parametrize("cfg", SIMT_CONFIGS, ids=lambda c: f"simt{c.cta_m}x{c.cta_n}")
def test_cuda_core_path_matches_oracle(cuda, cfg):
    """use_tensor_cores = false (the reference's SIMT path): reference test set in every sort mode
    and through the per-problem baseline, small16, tiny4096 and the edge cases, against FP64."""
    torch = _torch()
    probs, keep, refs = _fixture_problems(cuda)
    for mode in MODES:
        for _, d in refs:
            d.fill_(float("nan"))
        assert gg.run_grouped_gemm_once(probs, mode, cfg) == 0
        torch.cuda.synchronize()
        _check_fixture(refs)
    for _, d in refs:
        d.fill_(float("nan"))
    assert gg.run_baseline_per_problem(probs, cfg) == 0
    torch.cuda.synchronize()
    _check_fixture(refs)
    for wl in ("small16", "tiny4096"):
        ps = W.allocate(W.make_shapes(wl), cuda)
        run_grouped(ps.problems(), cfg, gg.SortMode.kByTiles)
        assert check_full(ps) <= 1.0
    cases = [(_edge_problem(cuda, seed=i, **kw)) for i, kw in enumerate(EDGE_CASES.values())]
    run_grouped([p for p, _ in cases], cfg, gg.SortMode.kByK)
    for (p, bufs), name in zip(cases, EDGE_CASES):
        try:
            _check_edge(p, bufs)
        except AssertionError as e:
            raise AssertionError(f"edge case {name}: {e}") from e


def test_cuda_core_path_mixed512_sampled_and_occupancy(cuda):
    cfg = gg.KernelConfig(128, 128, 64, use_tensor_cores=False)
    ps = W.allocate(W.make_shapes("mixed512"), cuda)
    run_grouped(ps.problems(), cfg, gg.SortMode.kByK)
    assert check_sampled(ps) <= 1.0
    st, info = gg.query_occupancy(cfg)
    assert st == 0 and not info.using_tensor_cores and info.threads_per_block == 256
    assert info.active_blocks_per_sm >= 1 and info.dynamic_shared_bytes == 0


BF16_CONFIGS = [gg.KernelConfig(128, 256, 64, input_type=1), gg.KernelConfig(128, 128, 64, input_type=1),
                gg.KernelConfig(256, 256, 64, input_type=1), gg.KernelConfig(64, 64, 16, input_type=1),
                gg.KernelConfig(128, 128, 64, use_tensor_cores=False, input_type=1)]


@pytest.mark.parametrize("cfg", BF16_CONFIGS,
                         ids=lambda c: f"{'' if c.use_tensor_cores else 'simt'}{c.cta_m}x{c.cta_n}")
def test_bf16_inputs_match_oracle(cuda, cfg):
    """input_type = 1 (BF16 A and B; an extension, the reference is FP16 only): small16 and
    tiny4096 in full (TMA-ineligible odd ld -> zero-fill loader), mixed512 sampled, and the
    per-problem baseline, against the FP64 oracle decoding BF16."""
    for wl in ("small16", "tiny4096"):
        ps = W.allocate(W.make_shapes(wl), cuda).to_bf16()
        run_grouped(ps.problems(), cfg, gg.SortMode.kByK)
        assert check_full(ps, fmt=1) <= 1.0
    ps = W.allocate(W.make_shapes("small16"), cuda).to_bf16()
    assert gg.run_baseline_per_problem(ps.problems(), cfg) == 0
    _torch().cuda.synchronize()
    assert check_full(ps, fmt=1) <= 1.0
    ps = W.allocate(W.make_shapes("mixed512"), cuda).to_bf16()
    run_grouped(ps.problems(), cfg, gg.SortMode.kByK)
    assert check_sampled(ps, fmt=1) <= 1.0


def test_bf16_and_fp16_reads_differ(cuda):
    """The same bits read as BF16 and as FP16 give different products: input_type reaches the MMA."""
    torch = _torch()
    ps = W.allocate(W.make_shapes("small16"), cuda).to_bf16()
    run_grouped(ps.problems(), gg.KernelConfig(128, 128, 64, input_type=1), gg.SortMode.kNone)
    as_bf16 = ps.d.clone()
    run_grouped(ps.problems(), gg.KernelConfig(128, 128, 64, input_type=0), gg.SortMode.kNone)
    finite = torch.isfinite(as_bf16) & torch.isfinite(ps.d)
    assert not torch.equal(as_bf16[finite], ps.d[finite])
    st, _ = gg.query_occupancy(gg.KernelConfig(128, 128, 64, input_type=4))
    assert st == 1  # an unknown input type is an invalid config


def test_zero_dim_problems_untouched(cuda):
    cases = [_edge_problem(cuda, m=0, n=64, k=16), _edge_problem(cuda, m=64, n=0, k=16),
             _edge_problem(cuda, m=64, n=64, k=16)]
    run_grouped([p for p, _ in cases], gg.KernelConfig(128, 128, 64), gg.SortMode.kNone)
    for p, bufs in cases:
        _check_edge(p, bufs)


def test_two_executors_two_streams(cuda):
    torch = _torch()
    ps1 = W.allocate(W.make_shapes("small16"), cuda, seed=1)
    ps2 = W.allocate(W.make_shapes("mixed512"), cuda, seed=2)
    cfg = gg.KernelConfig(128, 128, 64)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    torch.cuda.synchronize()  # inputs were written on the default stream
    e1, e2 = gg.GroupedGemmExecutor(), gg.GroupedGemmExecutor()
    assert e1.build(gg.prepare_problem_set(ps1.problems(), cfg, 2), cfg) == 0
    assert e2.build(gg.prepare_problem_set(ps2.problems(), cfg, 2), cfg) == 0
    for _ in range(3):
        assert e1.run(s1) == 0
        assert e2.run(s2) == 0
    torch.cuda.synchronize()
    assert e1.status() == 0 and e2.status() == 0
    assert check_full(ps1) <= 1.0
    assert check_sampled(ps2) <= 1.0


def test_executor_rebuild_and_reuse(cuda):
    ps1 = W.allocate(W.make_shapes("small16"), cuda, seed=3)
    ps2 = W.allocate(W.make_shapes("tiny4096"), cuda, seed=4)
    cfg = gg.KernelConfig(128, 128, 64)
    ex = gg.GroupedGemmExecutor()
    assert ex.build(gg.prepare_problem_set(ps1.problems(), cfg, 0), cfg) == 0
    assert ex.run() == 0 and ex.run() == 0
    assert ex.build(gg.prepare_problem_set(ps2.problems(), cfg, 3), cfg) == 0
    assert ex.problem_count() == 4096 and ex.total_tiles() == 4096
    assert 0 < ex.grid_ctas() <= ex.total_tiles()
    assert ex.run() == 0
    _torch().cuda.synchronize()
    assert ex.status() == 0
    assert check_full(ps1) <= 1.0 and check_full(ps2) <= 1.0


def test_persistent_ctas_override(cuda):
    ps = W.allocate(W.make_shapes("small16"), cuda, seed=5)
    for ctas in (1, 3, 1000):
        cfg = gg.KernelConfig(128, 128, 64, persistent_ctas=ctas)
        ps.d.fill_(float("nan"))
        ex = run_grouped(ps.problems(), cfg, gg.SortMode.kByK)
        assert ex.grid_ctas() == ctas
        assert check_full(ps) <= 1.0
    for ctas, want in ((1, 2), (3, 4), (6, 6)):  # pair configs round up to whole CTA pairs
        cfg = gg.KernelConfig(256, 128, 64, persistent_ctas=ctas)
        ps.d.fill_(float("nan"))
        ex = run_grouped(ps.problems(), cfg, gg.SortMode.kByK)
        assert ex.grid_ctas() == want
        assert check_full(ps) <= 1.0


# ---- the reference's own build, run on the same inputs ---------------------------------------
needs_ref = pytest.mark.skipif(not O.ref_available(), reason="reference build oracle/_ref absent")


@needs_ref
def test_golden_inputs_are_the_reference_generators(cuda):
    """The fixture's inputs equal what the reference test's own init_problem_buffers makes."""
    import ctypes

    fx = np.load(os.path.join(REPO, "tests", "golden", "ref_test_shapes.npz"))
    lib = O.load_ref()
    a, b, c, r = (np.zeros_like(fx[x]) for x in ("a", "b", "c", "ref"))
    al, be = np.zeros_like(fx["alpha"]), np.zeros_like(fx["beta"])
    shapes = np.ascontiguousarray(fx["shapes"].reshape(-1).astype(np.int32))
    P = ctypes.POINTER
    rc = lib.ref_test_inputs(shapes.ctypes.data_as(P(ctypes.c_int)), len(fx["shapes"]),
                             a.ctypes.data_as(P(ctypes.c_uint16)), b.ctypes.data_as(P(ctypes.c_uint16)),
                             c.ctypes.data_as(P(ctypes.c_float)), al.ctypes.data_as(P(ctypes.c_float)),
                             be.ctypes.data_as(P(ctypes.c_float)), r.ctypes.data_as(P(ctypes.c_float)))
    assert rc == 0
    for x, y in ((a, "a"), (b, "b"), (c, "c"), (r, "ref"), (al, "alpha"), (be, "beta")):
        assert np.array_equal(x, fx[y]), y


def _ref_problems(problems):
    arr = (O.RefProblem * max(1, len(problems)))()
    for i, p in enumerate(problems):
        arr[i] = O.RefProblem(p.m, p.n, p.k, p.a, p.b, p.c, p.d, p.lda, p.ldb, p.ldc, p.ldd, p.alpha, p.beta)
    return arr


def _rms(law, std):
    """Root mean square of a workload's value law: U[-1, 1] or N(0, std)."""
    return std if law == "normal" else 1.0 / np.sqrt(3.0)


@needs_ref
@pytest.mark.parametrize("name, cfg", [("small16", (128, 128, 64)), ("tiny4096", (128, 128, 64)),
                                       ("mixed512", (128, 128, 64)), ("moe", (128, 256, 64)),
                                       ("skew", (128, 256, 64))])
def test_agrees_with_reference_cuda_build(cuda, name, cfg):
    """The reference's own kernels (sm_100a build, 64x64x16 tiles, sort by tiles) and this kernel
    agree on the same inputs, every element of every problem: |ours - ref| / max(|ref|, s) within
    the accuracy bound, s = sqrt(K) * rms(a) * rms(b) (the typical size of one output)."""
    torch = _torch()
    shapes = W.make_shapes(name)
    ps = W.allocate(shapes, cuda)
    probs = ps.problems()
    lib = O.load_ref()
    assert lib.ref_run_grouped_once(_ref_problems(probs), len(probs), 2, 64, 64, 16, 1, None) == 0
    torch.cuda.synchronize()
    ref_d = ps.d.clone()
    ps.d.fill_(float("nan"))
    run_grouped(probs, gg.KernelConfig(*cfg), gg.SortMode.kByTiles)
    ab_rms = _rms(shapes.a_law, shapes.a_std) * _rms(shapes.b_law, shapes.b_std)
    worst = 0.0
    for i, (m, n, k) in enumerate(shapes.dims):
        if m <= 0 or n <= 0:
            continue
        sl = slice(ps.d_off[i], ps.d_off[i] + m * n)
        x, y = ps.d[sl].double(), ref_d[sl].double()
        scale = torch.clamp(y.abs(), min=float(np.sqrt(max(k, 1)) * ab_rms))
        worst = max(worst, float(((x - y).abs() / scale).max()) / O.tolerance(k))
        del x, y, scale
    assert worst <= 1.0
    if name in ("small16", "tiny4096"):
        ps.d.copy_(ref_d)
        assert check_full(ps) <= 1.0  # the reference itself meets the bar on these inputs
    del ref_d, ps


@needs_ref
def test_reference_test_program_passes_on_this_library(cuda):
    """The reference's own test program, compiled against this library's drop-in header."""
    exe = os.path.join(REPO, "oracle", "_ref", "ref_test_on_b200")
    if not os.path.exists(exe):
        pytest.skip("drop-in test program not built (make -C oracle dropin)")
    out = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "All correctness checks passed." in out.stdout
