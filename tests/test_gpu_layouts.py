"""Column-major (transposed) operands through the C-ABI against the FP64 oracle (needs a B200).

KernelConfig.a_layout / b_layout = Layout.kColMajor store A as its transpose (k x m, lda >= m) and
B as n x k (ldb >= k); the reference takes row-major operands only. The tensor cores read both
forms directly: a column-major A is an MN-major shared-memory operand, a column-major B a K-major
one (the instruction descriptor's major bits). Checked on the 1-CTA and CTA-pair kernels, a
reference tile shape and the CUDA-core kernel, with packed row pitches (odd sizes: the zero-fill
loader) and 16-byte-aligned ones (TMA), 16-bit and 8-bit inputs, and through the
mixture-of-experts plan with [n][k] expert weights. The oracle computes on the logical operands
(the test copies them out row-major); the accuracy bar is the north-star bound of
test_gpu_parity.py.
"""
from __future__ import annotations

import numpy as np
import pytest

import grouped_gemm_gpu_kernel_b200 as gg
import oracle as O
from grouped_gemm_gpu_kernel_b200 import workloads as W
from test_gpu_epilogue import aligned_shapes, check_problems, padding_untouched, run_set

pytestmark = pytest.mark.gpu

ROW, COL = gg.Layout.kRowMajor, gg.Layout.kColMajor
CONFIGS = [gg.KernelConfig(128, 256, 64), gg.KernelConfig(128, 128, 64), gg.KernelConfig(64, 128, 32),
           gg.KernelConfig(64, 64, 16), gg.KernelConfig(256, 256, 64), gg.KernelConfig(256, 128, 64),
           gg.KernelConfig(128, 128, 64, use_tensor_cores=False),
           gg.KernelConfig(256, 256, 64, tile_classes=gg.TileClasses.kPairBlocks)]
LAYOUTS = [(COL, ROW), (ROW, COL), (COL, COL)]


def _id(c):
    return f"{'' if c.use_tensor_cores else 'simt'}{c.cta_m}x{c.cta_n}x{c.cta_k}" + ("-classes" if c.tile_classes else "")


def _lid(l):
    return f"A{'col' if l[0] == COL else 'row'}-B{'col' if l[1] == COL else 'row'}"


@pytest.mark.parametrize("layout", LAYOUTS, ids=_lid)
@pytest.mark.parametrize("cfg", CONFIGS, ids=_id)
def test_column_major_operands_match_oracle(cuda, cfg, layout):
    a_l, b_l = layout
    run_cfg = gg.KernelConfig(cfg.cta_m, cfg.cta_n, cfg.cta_k, use_tensor_cores=cfg.use_tensor_cores,
                              a_layout=a_l, b_layout=b_l)
    for shapes, pad in ((W.make_shapes("small16", seed=5), 1), (aligned_shapes(), 8), (aligned_shapes(4), 1)):
        ps = W.allocate(shapes, seed=11).to_layout(a_l == COL, b_l == COL, pad)
        run_set(ps, run_cfg, None)
        worst = check_problems(ps)
        assert worst <= 1.0, f"{shapes.name} pad {pad}: error/tolerance {worst:.3f}"
        assert padding_untouched(ps)


@pytest.mark.parametrize("cfg, layout", [
    (gg.KernelConfig(128, 64, 64), (ROW, COL)),     # K-major B lifts the 128-column rule for 8-bit B
    (gg.KernelConfig(128, 128, 64), (COL, ROW)),
    (gg.KernelConfig(128, 256, 64), (COL, COL)),
    (gg.KernelConfig(256, 128, 64), (ROW, COL)),
], ids=["128x64-Bcol", "128x128-Acol", "128x256-AcolBcol", "pair256x128-Bcol"])
def test_column_major_fp8(cuda, cfg, layout):
    a_l, b_l = layout
    fmt = gg.InputType.kE4M3
    run_cfg = gg.KernelConfig(cfg.cta_m, cfg.cta_n, cfg.cta_k, input_type=fmt, a_layout=a_l, b_layout=b_l)
    for shapes in (W.make_shapes("small16", seed=5), aligned_shapes()):
        ps = W.allocate(shapes, seed=11).to_layout(a_l == COL, b_l == COL).to_fp8(fmt)
        run_set(ps, run_cfg, None)
        assert check_problems(ps) <= 1.0
        assert padding_untouched(ps)


def test_column_major_mixed512_sampled(cuda):
    """The benchmark set with [n][k] weights (B column-major), TMA path, 16-bit and FP8."""
    for fmt in (gg.InputType.kF16, gg.InputType.kE4M3):
        ps = W.allocate(W.make_shapes("mixed512"), seed=42).to_layout(False, True, 8)
        if fmt != gg.InputType.kF16:
            ps.to_fp8(fmt)
        run_set(ps, gg.KernelConfig(128, 256, 64, input_type=fmt, b_layout=COL), None)
        assert check_problems(ps, sample=True) <= 1.0


def test_layouts_match_row_major_bitwise(cuda):
    """The same values in any storage layout give the same D bit for bit on the tensor cores: the
    products and their accumulation order do not depend on the operand majors."""
    import torch

    outs = []
    for a_l, b_l in [(ROW, ROW)] + LAYOUTS:
        ps = W.allocate(aligned_shapes(), seed=11).to_layout(a_l == COL, b_l == COL, 8)
        run_set(ps, gg.KernelConfig(128, 128, 64, a_layout=a_l, b_layout=b_l), None)
        outs.append(ps.d.nan_to_num(7.0))
    for o in outs[1:]:
        assert torch.equal(outs[0], o)


def test_moe_plan_with_column_major_expert_weights(cuda):
    """Expert weights stored [n][k] (B column-major): the plan matches the executor bit for bit and
    one expert meets the oracle; a column-major A is refused (packed rows are rows of A)."""
    import torch

    rows = [130, 0, 257, 31, 64]
    n, k, cap = 192, 96, 600
    g = torch.Generator(device=cuda).manual_seed(2)
    A = torch.empty((cap, k), dtype=torch.float16, device=cuda).uniform_(-1, 1, generator=g)
    Bt = [torch.empty((n, k), dtype=torch.float16, device=cuda).uniform_(-1, 1, generator=g) for _ in rows]
    D = torch.full((cap, n), float("nan"), device=cuda)
    cfg = gg.KernelConfig(128, 256, 64, b_layout=COL)
    plan = gg.MoePlan(len(rows), n, k, cap, A.data_ptr(), k, [b.data_ptr() for b in Bt], k, D.data_ptr(), n,
                      config=cfg)
    assert plan.run(torch.tensor(rows, dtype=torch.int32, device=cuda)) == 0
    assert plan.status()[0] == 0
    D2 = torch.full_like(D, float("nan"))
    probs, r0 = [], 0
    for e, r in enumerate(rows):
        probs.append(gg.ProblemDesc(r, n, k, A[r0:].data_ptr(), Bt[e].data_ptr(), None, D2[r0:].data_ptr(), k, k,
                                    n, n))
        r0 += r
    assert gg.run_grouped_gemm_once(probs, gg.SortMode.kNone, cfg) == 0
    torch.cuda.synchronize()
    used = sum(rows)
    assert torch.equal(D[:used], D2[:used]) and torch.isnan(D[used:]).all()
    e, r0 = 2, sum(rows[:2])
    a = A[r0:r0 + rows[e]].cpu().numpy()
    b = Bt[e].t().contiguous().cpu().numpy()
    ref, scale = O.gemm_f64(rows[e], n, k, a, k, b, n, None, n, 1.0, 0.0)
    assert O.rel_err(D[r0:r0 + rows[e]].cpu().numpy(), ref, scale) <= O.tolerance(k)
    plan.close()
    with pytest.raises(ValueError):
        gg.MoePlan(len(rows), n, k, cap, A.data_ptr(), k, [b.data_ptr() for b in Bt], k, D.data_ptr(), n,
                   config=gg.KernelConfig(128, 256, 64, a_layout=COL))
