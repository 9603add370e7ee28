"""Grouped GEMM with device-side preparation (gg_moe_plan_*) against the host-prepared executor.

The plan packs the problems' rows back to back in A/C/D and reads the row counts from device
memory. On the same inputs it runs the same kernel with the same tiles as an executor built from
per-problem pointers, so D must match bit for bit; rows past the last problem must stay
untouched; a graph-captured run must follow row counts changed on the device; bad row counts
must compute nothing and raise GG_STATUS_BAD_ROWS.
"""
import numpy as np
import pytest

import grouped_gemm_gpu_kernel_b200 as gg
import oracle as O
from grouped_gemm_gpu_kernel_b200 import capi

pytestmark = pytest.mark.gpu


def _setup(cuda, rows, n, k, capacity, lda=None, seed=0, beta=0.0):
    import torch

    g = torch.Generator(device=cuda).manual_seed(seed)
    lda = lda or k
    E = len(rows)
    A = torch.empty((capacity, lda), dtype=torch.float16, device=cuda).uniform_(-1, 1, generator=g)
    Bs = [torch.empty((k, n), dtype=torch.float16, device=cuda).uniform_(-1, 1, generator=g) for _ in range(E)]
    C = torch.empty((capacity, n), device=cuda).uniform_(-1, 1, generator=g) if beta != 0.0 else None
    D = torch.full((capacity, n), float("nan"), device=cuda)
    return A, Bs, C, D


def _plan(A, Bs, C, D, n, k, capacity, cfg, beta=0.0, alpha=1.0):
    return gg.MoePlan(len(Bs), n, k, capacity, A.data_ptr(), A.stride(0), [b.data_ptr() for b in Bs], n,
                      D.data_ptr(), n, C.data_ptr() if C is not None else None, n, alpha, beta, cfg)


def _executor_reference(A, Bs, C, rows, n, k, cfg, alpha=1.0, beta=0.0, bias=None, dtype=None):
    """D of the same problems through the host-prepared executor (per-problem pointers); bias:
    one device pointer (or None) per expert; dtype: D's torch dtype (default FP32)."""
    import torch

    D2 = torch.full((A.shape[0], n), float("nan"), device=A.device, dtype=dtype or torch.float32)
    probs, r0 = [], 0
    for e, r in enumerate(rows):
        a = A[r0:r0 + max(r, 0)]
        c = C[r0:r0 + max(r, 0)] if C is not None else None
        probs.append(gg.ProblemDesc(r, n, k, a.data_ptr() if r > 0 else A.data_ptr(), Bs[e].data_ptr(),
                                    c.data_ptr() if c is not None and r > 0 else None,
                                    D2[r0:].data_ptr(), A.stride(0), n, n, n, alpha, beta))
        r0 += r
    if bias is None:
        assert gg.run_grouped_gemm_once(probs, gg.SortMode.kNone, cfg) == 0
    else:
        ex = gg.GroupedGemmExecutor()
        assert ex.build(gg.prepare_problem_set(probs, cfg, gg.SortMode.kNone), cfg, bias=bias) == 0
        assert ex.run() == 0
        torch.cuda.synchronize()
        ex.close()
    torch.cuda.synchronize()
    return D2


CFGS = [gg.KernelConfig(128, 256, 64), gg.KernelConfig(128, 128, 64), gg.KernelConfig(256, 128, 64),
        gg.KernelConfig(128, 128, 64, use_tensor_cores=False)]


@pytest.mark.parametrize("cfg", CFGS, ids=lambda c: f"{'' if c.use_tensor_cores else 'simt'}{c.cta_m}x{c.cta_n}")
def test_plan_matches_executor_bitwise(cuda, cfg):
    import torch

    rows = [0, 5, 130, 1, 64, 257, 31, 100]
    n, k, capacity = 320, 200, 700
    A, Bs, C, D = _setup(cuda, rows, n, k, capacity)
    plan = _plan(A, Bs, C, D, n, k, capacity, cfg)
    rows_t = torch.tensor(rows, dtype=torch.int32, device=cuda)
    torch.cuda.synchronize()
    assert plan.run(rows_t) == 0
    bits, total = plan.status()
    assert bits == 0
    tiles_n = -(-n // cfg.cta_n)
    assert total == sum(-(-r // cfg.cta_m) * tiles_n for r in rows)
    ref = _executor_reference(A, Bs, C, rows, n, k, cfg)
    used = sum(rows)
    assert torch.equal(D[:used], ref[:used])
    assert torch.isnan(D[used:]).all()  # rows past the packed problems are never written
    # independent accuracy check of one expert against the FP64 oracle
    e, r0 = 5, sum(rows[:5])
    a = A[r0:r0 + rows[e]].cpu().numpy()
    b = Bs[e].cpu().numpy()
    ref64, scale = O.gemm_f64(rows[e], n, k, a, k, b, n, None, n, 1.0, 0.0)
    err = O.rel_err(D[r0:r0 + rows[e]].cpu().numpy().astype(np.float64), ref64, scale)
    assert err <= O.tolerance(k)
    plan.close()


def test_plan_follows_rows_changed_on_device_in_a_cuda_graph(cuda):
    import torch

    cfg = gg.KernelConfig(128, 256, 64)
    n, k, capacity = 256, 128, 1024
    first, second = [300, 0, 17, 200], [1, 450, 0, 129]
    A, Bs, C, D = _setup(cuda, first, n, k, capacity, beta=0.5)
    plan = _plan(A, Bs, C, D, n, k, capacity, cfg, beta=0.5, alpha=1.5)
    rows_t = torch.tensor(first, dtype=torch.int32, device=cuda)
    s = torch.cuda.Stream(cuda)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        assert plan.run(rows_t, torch.cuda.current_stream()) == 0
    for rows in (first, second):
        rows_t.copy_(torch.tensor(rows, dtype=torch.int32))
        D.fill_(float("nan"))
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        assert plan.status()[0] == 0
        ref = _executor_reference(A, Bs, C, rows, n, k, cfg, alpha=1.5, beta=0.5)
        used = sum(rows)
        assert torch.equal(D[:used], ref[:used])
        assert torch.isnan(D[used:]).all()
    del g
    plan.close()


@pytest.mark.parametrize("rows", [[10, -1, 5], [600, 300, 200]])
def test_plan_rejects_bad_rows_without_computing(cuda, rows):
    import torch

    cfg = gg.KernelConfig(128, 128, 64)
    n, k, capacity = 128, 64, 1000
    A, Bs, C, D = _setup(cuda, rows, n, k, capacity)
    plan = _plan(A, Bs, C, D, n, k, capacity, cfg)
    assert plan.run(torch.tensor(rows, dtype=torch.int32, device=cuda)) == 0
    bits, total = plan.status()
    assert bits & capi.GG_STATUS_BAD_ROWS and total == 0
    assert torch.isnan(D).all()
    assert plan.status()[0] == 0  # cleared by the read
    plan.close()


def test_plan_on_the_moe_workload_matches_executor(cuda):
    """BASELINE's MoE up-projection (64 experts, Zipf token split, N 14336, K 4096) through the plan."""
    import torch

    from grouped_gemm_gpu_kernel_b200 import workloads as W

    sh = W.make_shapes("moe")
    rows = [m for m, n, k in sh.dims]
    n, k = sh.dims[0][1], sh.dims[0][2]
    capacity = sum(rows)
    cfg = gg.KernelConfig(128, 256, 64)
    g = torch.Generator(device=cuda).manual_seed(3)
    A = torch.empty((capacity, k), dtype=torch.float16, device=cuda).normal_(0, 1, generator=g)
    Bs = [torch.empty((k, n), dtype=torch.float16, device=cuda).normal_(0, 0.02, generator=g) for _ in rows]
    D = torch.full((capacity, n), float("nan"), device=cuda)
    plan = _plan(A, Bs, None, D, n, k, capacity, cfg)
    assert plan.run(torch.tensor(rows, dtype=torch.int32, device=cuda)) == 0
    assert plan.status()[0] == 0
    ref = _executor_reference(A, Bs, None, rows, n, k, cfg)
    assert torch.equal(D, ref)
    plan.close()


def test_plan_with_more_experts_than_one_preparation_block(cuda):
    """1500 problems: the preparation kernel scans in chunks of 1024 and keeps expert order."""
    import torch

    rng = np.random.default_rng(5)
    rows = [int(x) for x in rng.integers(0, 40, size=1500)]
    n, k = 96, 72
    capacity = sum(rows) + 17
    cfg = gg.KernelConfig(128, 128, 64)
    A, Bs, C, D = _setup(cuda, rows, n, k, capacity, beta=0.25)
    plan = _plan(A, Bs, C, D, n, k, capacity, cfg, beta=0.25)
    assert plan.run(torch.tensor(rows, dtype=torch.int32, device=cuda)) == 0
    bits, total = plan.status()
    assert bits == 0 and total == sum(-(-r // 128) for r in rows)
    ref = _executor_reference(A, Bs, C, rows, n, k, cfg, beta=0.25)
    used = sum(rows)
    assert torch.equal(D[:used], ref[:used])
    assert torch.isnan(D[used:]).all()
    plan.close()


@pytest.mark.parametrize("out", [gg.OutputType.kF16, gg.OutputType.kBF16], ids=["F16", "BF16"])
@pytest.mark.parametrize("cfg", [gg.KernelConfig(128, 256, 64), gg.KernelConfig(256, 128, 64),
                                 gg.KernelConfig(128, 128, 64, use_tensor_cores=False)],
                         ids=["128x256", "256x128", "simt128x128"])
def test_plan_output_type_bias_activation(cuda, cfg, out):
    """16-bit packed C/D, per-expert bias (one expert without) and GELU: the plan matches the
    executor bit for bit, rows past the problems stay untouched, and one expert meets the oracle."""
    import torch

    dt = torch.float16 if out == gg.OutputType.kF16 else torch.bfloat16
    rows = [130, 0, 257, 31, 64, 7]
    n, k, capacity = 200, 96, 600
    A, Bs, C, _ = _setup(cuda, rows, n, k, capacity, beta=0.5, seed=4)
    C = C.to(dt)
    D = torch.full((capacity, n), float("nan"), device=cuda, dtype=dt)
    g = torch.Generator(device=cuda).manual_seed(9)
    biases = [None if e == 3 else torch.empty(n, device=cuda).uniform_(-1, 1, generator=g) for e in range(len(rows))]
    ptrs = [None if t is None else t.data_ptr() for t in biases]
    run_cfg = gg.KernelConfig(cfg.cta_m, cfg.cta_n, cfg.cta_k, use_tensor_cores=cfg.use_tensor_cores,
                              output_type=out, activation=gg.Activation.kGELU)
    plan = gg.MoePlan(len(rows), n, k, capacity, A.data_ptr(), k, [b.data_ptr() for b in Bs], n, D.data_ptr(), n,
                      C.data_ptr(), n, 1.25, 0.5, run_cfg, bias_ptrs=ptrs)
    assert plan.run(torch.tensor(rows, dtype=torch.int32, device=cuda)) == 0
    assert plan.status()[0] == 0
    ref = _executor_reference(A, Bs, C, rows, n, k, run_cfg, alpha=1.25, beta=0.5, bias=ptrs, dtype=dt)
    used = sum(rows)
    assert torch.equal(D[:used].float().nan_to_num(7.0), ref[:used].float().nan_to_num(7.0))
    assert not torch.isnan(D[:used].float()).any()
    assert torch.isnan(D[used:].float()).all()
    for e in (2, 3):
        r0 = sum(rows[:e])
        a = A[r0:r0 + rows[e]].cpu().numpy()
        c = C[r0:r0 + rows[e]].float().cpu().numpy()
        bias = None if biases[e] is None else biases[e].cpu().numpy()
        ref64, scale = O.gemm_f64(rows[e], n, k, a, k, Bs[e].cpu().numpy(), n, c, n, 1.25, 0.5, bias=bias,
                                  act=int(gg.Activation.kGELU))
        err = O.rel_err(D[r0:r0 + rows[e]].float().cpu().numpy(), ref64, scale, int(out))
        assert err <= O.tolerance(k)
    plan.close()
