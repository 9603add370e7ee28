"""Parity of the epilogue extensions through the C-ABI against the FP64 oracle (needs a B200).

The extensions have no reference counterpart (the reference stores FP32 D = alpha*A*B + beta*C):
16-bit C and D (KernelConfig.output_type), a per-column FP32 bias (gg_executor_build_with_bias)
and a fused activation (KernelConfig.activation), D = act(alpha * A x B + beta * C + bias). They
are checked on the tcgen05 kernels (one CTA per tile, CTA pairs, a reference tile shape) and the
CUDA-core kernel, on packed leading dimensions that TMA cannot take (direct loads and stores) and
on 16-byte-aligned ones (TMA stores, vector C loads).

Accuracy bar, for every element: the north-star bound applied to the FP32 result before its one
rounding to the output type,
    max(|D - D_fp64| - u |D_fp64| - s, 0) / max(|D_fp64|, scale)  <=  2e-3 * sqrt(max(K, 1) / 1024)
with (u, s) the unit roundoff and subnormal half-spacing of the output type (FP32: 0, 0; FP16:
2^-11, 2^-25; BF16: 2^-8, 2^-134) and scale = L * (|alpha| sqrt(sum_k (a_ik b_kj)^2) + |beta c_ij|
+ |bias_j|), L = 1.13 for GELU (a bound of its slope), 1 otherwise (oracle.rel_err,
oracle.gemm_f64).
"""
from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import grouped_gemm_gpu_kernel_b200 as gg
import oracle as O
from grouped_gemm_gpu_kernel_b200 import workloads as W

pytestmark = pytest.mark.gpu

F32, F16, BF16 = gg.OutputType.kF32, gg.OutputType.kF16, gg.OutputType.kBF16
NONE, RELU, GELU = gg.Activation.kNone, gg.Activation.kReLU, gg.Activation.kGELU

CONFIGS = [gg.KernelConfig(128, 256, 64), gg.KernelConfig(128, 128, 64), gg.KernelConfig(256, 256, 64),
           gg.KernelConfig(64, 64, 16), gg.KernelConfig(128, 128, 64, use_tensor_cores=False),
           gg.KernelConfig(256, 128, 64, tile_classes=gg.TileClasses.kPairBlocks)]
# (output type, activation, bias vectors: None, "aligned" (16-byte, vector loads) or "unaligned")
CASES = [(F16, GELU, "unaligned"), (BF16, RELU, "aligned"), (F32, GELU, "aligned"), (F16, NONE, None),
         (BF16, NONE, "unaligned"), (F32, RELU, "unaligned")]


def _cfg_id(c):
    return f"{'' if c.use_tensor_cores else 'simt'}{c.cta_m}x{c.cta_n}x{c.cta_k}" + ("-classes" if c.tile_classes else "")


def _case_id(case):
    out, act, bias = case
    return f"{out.name[1:]}-{act.name[1:]}{'-bias-' + bias if bias else ''}"


def aligned_shapes(seed=3) -> W.Shapes:
    """24 problems whose N and K are multiples of 8 (so every D and C row starts 16-byte aligned
    and D goes out by TMA), M anything in [1, 300]; C read (beta 0.5), alpha 1.25."""
    rng = np.random.default_rng(seed)
    dims = [(int(rng.integers(1, 301)), int(8 * rng.integers(1, 41)), int(8 * rng.integers(1, 41)))
            for _ in range(24)]
    return W.Shapes("aligned24", dims, [1.25] * 24, [0.5] * 24, True)


def run_set(ps: W.DeviceProblemSet, cfg: gg.KernelConfig, bias_ptrs, mode=gg.SortMode.kByTiles):
    import torch

    problems = ps.problems()
    prep = gg.prepare_problem_set(problems, cfg, mode)
    sorted_bias = None if bias_ptrs is None else [bias_ptrs[o] for o in prep.sorted_to_original]
    ex = gg.GroupedGemmExecutor()
    assert ex.build(prep, cfg, bias=sorted_bias) == 0
    assert ex.run() == 0
    torch.cuda.synchronize()
    assert ex.status() == 0, "a bounded wait timed out inside the kernel"
    ex.close()


def check_full(ps: W.DeviceProblemSet, act: int, threads: int = 8) -> float:
    """Worst error / tolerance over every element of every problem."""
    import torch

    a = ps.a.view(torch.int16).cpu().numpy().view(np.uint16)
    b = ps.b.view(torch.int16).cpu().numpy().view(np.uint16)
    c = ps.c.float().cpu().numpy() if ps.c is not None else None
    d = ps.d.float().cpu().numpy()

    def one(i):
        m, n, k = ps.shapes.dims[i]
        if m <= 0 or n <= 0:
            return 0.0
        ai = a[ps.a_off[i]:ps.a_off[i] + max(m * k, 1)]
        bi = b[ps.b_off[i]:ps.b_off[i] + max(k * n, 1)]
        ci = c[ps.c_off[i]:ps.c_off[i] + m * n] if c is not None else None
        di = d[ps.d_off[i]:ps.d_off[i] + m * n]
        ref, scale = O.gemm_f64(m, n, k, ai, max(1, k), bi, max(1, n), ci, max(1, n), ps.shapes.alpha[i],
                                ps.shapes.beta[i], bias=ps.bias_host(i), act=act)
        return O.rel_err(di.reshape(m, n), ref, scale, ps.out_fmt) / O.tolerance(k)

    with ThreadPoolExecutor(threads) as pool:
        return max(pool.map(one, range(len(ps.shapes.dims))), default=0.0)


def check_sampled(ps: W.DeviceProblemSet, act: int, rows_per=4, cols_per=96, seed=0, threads=8) -> float:
    rng = np.random.default_rng(seed)
    jobs = []
    for i, (m, n, k) in enumerate(ps.shapes.dims):
        if m <= 0 or n <= 0:
            continue
        rows = np.unique(np.concatenate([[0, m - 1], rng.integers(0, m, size=rows_per)])).astype(np.int64)
        cols = np.unique(np.concatenate([[0, n - 1], rng.integers(0, n, size=cols_per)])).astype(np.int64)
        jobs.append((i, len(rows), len(cols), k, W.host_inputs(ps, i, rows, cols), ps.bias_host(i, cols)))

    def one(job):
        i, r, c, k, h, bias = job
        ref, scale = O.gemm_f64(r, c, k, h["a"], max(1, k), h["b"], c, h["c"], c, ps.shapes.alpha[i],
                                ps.shapes.beta[i], bias=bias, act=act)
        return O.rel_err(h["d"], ref, scale, ps.out_fmt) / O.tolerance(k)

    with ThreadPoolExecutor(threads) as pool:
        return max(pool.map(one, jobs), default=0.0)


def padding_untouched(ps: W.DeviceProblemSet) -> bool:
    """D elements between the problems' regions (the slab's alignment padding) are still NaN."""
    import torch

    used = torch.zeros(ps.d.numel(), dtype=torch.bool, device=ps.d.device)
    for i, (m, n, k) in enumerate(ps.shapes.dims):
        if m > 0 and n > 0:
            used[ps.d_off[i]:ps.d_off[i] + m * n] = True
    return bool(torch.isnan(ps.d.float()[~used]).all().item())


@pytest.mark.parametrize("case", CASES, ids=_case_id)
@pytest.mark.parametrize("cfg", CONFIGS, ids=_cfg_id)
def test_epilogue_extensions_match_oracle(cuda, cfg, case):
    out, act, with_bias = case
    run_cfg = gg.KernelConfig(cfg.cta_m, cfg.cta_n, cfg.cta_k, use_tensor_cores=cfg.use_tensor_cores,
                              output_type=out, activation=act)
    for shapes in (W.make_shapes("small16", seed=5), aligned_shapes(), W.make_shapes("tiny4096", seed=6)):
        ps = W.allocate(shapes, seed=11)
        if out != F32:
            ps.to_output(out)
        bias = ps.make_bias(aligned=with_bias == "aligned") if with_bias else None
        run_set(ps, run_cfg, bias)
        worst = check_full(ps, act)
        assert worst <= 1.0, f"{shapes.name}: error/tolerance {worst:.3f}"
        assert padding_untouched(ps), f"{shapes.name}: a store landed outside its problem's D"


@pytest.mark.parametrize("out", [F16, BF16], ids=["F16", "BF16"])
def test_epilogue_mixed512_sampled(cuda, out):
    """The full-size benchmark set: TMA D stores of 16-bit tiles, GELU and bias on most problems."""
    ps = W.allocate(W.make_shapes("mixed512"), seed=42)
    ps.to_output(out)
    bias = ps.make_bias(aligned=out == F16)
    run_set(ps, gg.KernelConfig(128, 256, 64, output_type=out, activation=GELU), bias)
    assert check_sampled(ps, GELU) <= 1.0
    assert padding_untouched(ps)


def test_f32_identity_epilogue_unchanged_by_extensions(cuda):
    """output_type F32, no activation, no bias: bit-identical to the build without bias table, and
    an all-zero bias changes nothing either."""
    import torch

    cfg = gg.KernelConfig(128, 128, 64)
    runs = []
    for zero_bias in (False, True):
        ps = W.allocate(aligned_shapes(), seed=11)
        bias = None
        if zero_bias:
            bias = ps.make_bias(without=0.0)
            ps.bias.zero_()
        run_set(ps, cfg, bias)
        runs.append(ps.d.clone())
    assert torch.equal(torch.nan_to_num(runs[0], nan=7.0), torch.nan_to_num(runs[1], nan=7.0))


def test_relu_output_is_nonnegative_and_gelu_differs(cuda):
    import torch

    outs = {}
    for act in (NONE, RELU, GELU):
        ps = W.allocate(aligned_shapes(), seed=11)
        ps.to_output(F16)
        run_set(ps, gg.KernelConfig(128, 128, 64, output_type=F16, activation=act), None)
        outs[act] = ps.d.float()
    valid = ~torch.isnan(outs[NONE])
    assert (outs[RELU][valid] >= 0).all()
    assert torch.equal(outs[RELU][valid], torch.clamp(outs[NONE][valid], min=0))
    assert not torch.equal(outs[GELU][valid], outs[RELU][valid])


# ---- 8-bit inputs (KernelConfig.input_type E4M3 / E5M2; kind::f8f6f4 on the tensor cores) -------
E4M3, E5M2 = gg.InputType.kE4M3, gg.InputType.kE5M2
FP8_CONFIGS = [gg.KernelConfig(128, 256, 64), gg.KernelConfig(128, 128, 64), gg.KernelConfig(64, 128, 32),
               gg.KernelConfig(256, 256, 64), gg.KernelConfig(128, 128, 64, use_tensor_cores=False)]


def check_problems(ps: W.DeviceProblemSet, act: int = 0, sample: bool = False, threads: int = 8) -> float:
    """Worst error / tolerance of every problem (all elements, or sampled rows and columns) against
    the oracle, for any input format (host_inputs copies the operands' raw bits)."""
    rng = np.random.default_rng(0)
    jobs = []
    for i, (m, n, k) in enumerate(ps.shapes.dims):
        if m <= 0 or n <= 0:
            continue
        rows = cols = None
        if sample:
            rows = np.unique(np.concatenate([[0, m - 1], rng.integers(0, m, size=4)])).astype(np.int64)
            cols = np.unique(np.concatenate([[0, n - 1], rng.integers(0, n, size=96)])).astype(np.int64)
        h = W.host_inputs(ps, i, rows, cols)
        jobs.append((i, m if rows is None else len(rows), n if cols is None else len(cols), k, h,
                     ps.bias_host(i, cols)))

    def one(job):
        i, r, c, k, h, bias = job
        ref, scale = O.gemm_f64(r, c, k, h["a"], max(1, k), h["b"], c, h["c"], c, ps.shapes.alpha[i],
                                ps.shapes.beta[i], fmt=ps.in_fmt, bias=bias, act=act)
        return O.rel_err(h["d"].reshape(r, c), ref, scale, ps.out_fmt) / O.tolerance(k)

    with ThreadPoolExecutor(threads) as pool:
        return max(pool.map(one, jobs), default=0.0)


@pytest.mark.parametrize("fmt", [E4M3, E5M2], ids=["E4M3", "E5M2"])
@pytest.mark.parametrize("cfg", FP8_CONFIGS, ids=_cfg_id)
def test_fp8_inputs_match_oracle(cuda, cfg, fmt):
    run_cfg = gg.KernelConfig(cfg.cta_m, cfg.cta_n, cfg.cta_k, use_tensor_cores=cfg.use_tensor_cores,
                              input_type=fmt)
    for shapes in (W.make_shapes("small16", seed=5), aligned_shapes(), W.make_shapes("tiny4096", seed=6)):
        ps = W.allocate(shapes, seed=11).to_fp8(fmt)
        run_set(ps, run_cfg, None)
        worst = check_problems(ps)
        assert worst <= 1.0, f"{shapes.name}: error/tolerance {worst:.3f}"
        assert padding_untouched(ps)


@pytest.mark.parametrize("fmt", [E4M3, E5M2], ids=["E4M3", "E5M2"])
def test_fp8_mixed512_sampled_with_epilogue(cuda, fmt):
    """The benchmark set with 8-bit A/B, FP16 D, bias and GELU: every extension at once."""
    ps = W.allocate(W.make_shapes("mixed512"), seed=42).to_fp8(fmt)
    ps.to_output(F16)
    bias = ps.make_bias(aligned=True)
    run_set(ps, gg.KernelConfig(128, 256, 64, input_type=fmt, output_type=F16, activation=GELU), bias)
    assert check_problems(ps, act=GELU, sample=True) <= 1.0
    assert padding_untouched(ps)


def test_fp8_and_fp16_decode_differ(cuda):
    """The same bytes read as E4M3 and as E5M2 give different products (the format field reaches
    the tensor cores), and each matches its own oracle."""
    import torch

    outs = []
    for fmt in (E4M3, E5M2):
        ps = W.allocate(aligned_shapes(), seed=11).to_fp8(E4M3)  # the same E4M3 bytes both times
        ps.in_fmt = int(fmt)
        run_set(ps, gg.KernelConfig(128, 128, 64, input_type=fmt), None)
        assert check_problems(ps) <= 1.0
        outs.append(ps.d.clone())
    valid = ~torch.isnan(outs[0])
    assert not torch.equal(outs[0][valid], outs[1][valid])


@pytest.mark.parametrize("cfg", [gg.KernelConfig(128, 256, 64), gg.KernelConfig(128, 128, 64),
                                 gg.KernelConfig(256, 256, 64)], ids=_cfg_id)
def test_fp8_packed_pitches_take_the_zero_fill_loader(cuda, cfg):
    """8-bit operands whose rows TMA cannot load (packed odd pitches: 1-, 2- and 4-byte aligned
    rows) go through the zero-fill loader on the tensor cores, in both storage layouts."""
    fmt = E4M3
    for a_col, b_col in ((False, False), (True, True)):
        run_cfg = gg.KernelConfig(cfg.cta_m, cfg.cta_n, cfg.cta_k, input_type=fmt, a_layout=int(a_col),
                                  b_layout=int(b_col))
        for shapes in (W.make_shapes("small16", seed=5), W.make_shapes("tiny4096", seed=6)):
            ps = W.allocate(shapes, seed=11).to_layout(a_col, b_col).to_fp8(fmt, pad=1)
            run_set(ps, run_cfg, None)
            worst = check_problems(ps)
            assert worst <= 1.0, f"{shapes.name} layouts {a_col, b_col}: error/tolerance {worst:.3f}"
            assert padding_untouched(ps)
