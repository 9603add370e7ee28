"""Host side of the B200 library through its C-ABI (CPU, no GPU needed).

Mirrors the reference's API contract (reference include/grouped_gemm/grouped_gemm.cuh and
src/grouped_gemm.cu:952-1329): preparation is bit-identical to the reference, configs and
problem sets are validated with the reference's error codes before any device work, and the
library exports every entry point its C header declares.
"""
from __future__ import annotations

import json
import os
import re
import shutil
import subprocess

import numpy as np
import pytest

import grouped_gemm_gpu_kernel_b200 as gg
import oracle as O
from grouped_gemm_gpu_kernel_b200 import capi

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "grouped_gemm_b200.h")
GOLDEN = os.path.join(REPO, "tests", "golden")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gg_[a-z_0-9]+)\s*\(", text)))


def dims_problems(dims, ptr=0x1000):
    return [gg.ProblemDesc(m, n, k, ptr, ptr, None, ptr, max(1, k), max(1, n), max(1, n), max(1, n)) for m, n, k in dims]


def test_library_exports_every_declared_symbol():
    lib = capi.load()
    declared = header_functions()
    assert set(declared) == set(capi.EXPORTED_SYMBOLS), "capi.EXPORTED_SYMBOLS out of date"
    for name in declared:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", capi.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (gg_\w+)", out))
    assert set(declared) <= exported
    # the static CUDA runtime stays private to the library
    assert not re.search(r" T cuda[A-Z]", out)
    assert lib.gg_abi_version() == 2


def test_cpp_api_exported():
    out = subprocess.run(["nm", "-DC", "--defined-only", capi.LIB_PATH], capture_output=True, text=True).stdout
    for sym in ["grouped_gemm::prepare_problem_set", "grouped_gemm::sort_mode_name", "grouped_gemm::query_occupancy",
                "grouped_gemm::GroupedGemmExecutor::build", "grouped_gemm::GroupedGemmExecutor::run",
                "grouped_gemm::run_grouped_gemm_once", "grouped_gemm::run_baseline_per_problem",
                "grouped_gemm::count_non_empty_problems"]:
        assert sym in out, sym


def test_sort_mode_names():
    g = json.load(open(os.path.join(GOLDEN, "prepare_golden.json")))
    for mode, name in g["sort_mode_name"].items():
        assert gg.sort_mode_name(int(mode)) == name


def test_prepare_bit_identical_to_reference_golden():
    g = json.load(open(os.path.join(GOLDEN, "prepare_golden.json")))
    n = 0
    for name, entry in g["sets"].items():
        probs = dims_problems(entry["dims"])
        for r in entry["results"]:
            cfg = gg.KernelConfig(*r["cta"])
            prep = gg.prepare_problem_set(probs, cfg, r["mode"])
            assert prep.sorted_to_original == r["sorted_to_original"], (name, r["cta"], r["mode"])
            assert prep.tile_offsets == r["tile_offsets"]
            assert prep.total_tiles == r["total_tiles"]
            assert [(p.m, p.n, p.k) for p in prep.sorted_problems] == [tuple(entry["dims"][i]) for i in r["sorted_to_original"]]
            assert gg.count_non_empty_problems(probs, cfg) == r["non_empty"]
            n += 1
    assert n >= 300


def test_prepare_matches_oracle_random_with_ties():
    rng = np.random.default_rng(5)
    for _ in range(200):
        P = int(rng.integers(0, 80))
        dims = [(int(rng.choice([0, 1, 63, 64, 65, 128, 200])), int(rng.choice([0, 1, 64, 127, 128, 256, 300])),
                 int(rng.choice([0, 16, 64, 96]))) for _ in range(P)]
        probs = dims_problems(dims)
        for cfg in gg.REFERENCE_CONFIGS + gg.NATIVE_CONFIGS:
            for mode in range(5):
                prep = gg.prepare_problem_set(probs, cfg, mode)
                perm, offs, total = O.prepare(dims, cfg.cta_m, cfg.cta_n, mode)
                assert prep.sorted_to_original == perm.tolist()
                assert prep.tile_offsets == offs.tolist()
                assert prep.total_tiles == total


def test_prepare_carries_problem_fields():
    probs = [gg.ProblemDesc(10, 20, 30, 0x100, 0x200, 0x300, 0x400, 31, 21, 22, 23, 0.5, -2.0),
             gg.ProblemDesc(100, 200, 64, 0x500, 0x600, None, 0x700, 64, 200, 200, 200, 1.0, 0.0)]
    prep = gg.prepare_problem_set(probs, gg.KernelConfig(), gg.SortMode.kByTiles)
    assert prep.sorted_to_original == [1, 0]
    assert prep.sorted_problems[1] == probs[0]
    assert prep.sorted_problems[0] == probs[1]


def test_tile_count_entry_point():
    lib = capi.load()
    import ctypes

    cfg = gg.KernelConfig(128, 128, 64).to_c()
    for m, n, want in [(0, 5, 0), (5, 0, 0), (1, 1, 1), (128, 128, 1), (129, 128, 2), (300, 257, 9)]:
        p = gg.ProblemDesc(m, n, 7, 1, 1, None, 1, 7, max(1, n), max(1, n), max(1, n)).to_c()
        assert lib.gg_tile_count(ctypes.byref(p), ctypes.byref(cfg)) == want


@pytest.mark.parametrize("cfg,ok", [
    (gg.KernelConfig(64, 64, 16), True), (gg.KernelConfig(128, 64, 32), True), (gg.KernelConfig(64, 128, 32), True),
    (gg.KernelConfig(128, 128, 64), True), (gg.KernelConfig(128, 256, 64), True), (gg.KernelConfig(128, 64, 64), True),
    (gg.KernelConfig(256, 128, 64), True), (gg.KernelConfig(256, 256, 64), True), (gg.KernelConfig(256, 64, 64), False),
    (gg.KernelConfig(64, 64, 16, threads=128), False), (gg.KernelConfig(32, 32, 16), False),
    (gg.KernelConfig(128, 128, 32), False), (gg.KernelConfig(256, 128, 32), False),
    # tile classes: CTA-pair configs on the tensor cores only
    (gg.KernelConfig(256, 256, 64, tile_classes=1), True), (gg.KernelConfig(256, 128, 64, tile_classes=1), True),
    (gg.KernelConfig(128, 256, 64, tile_classes=1), False),
    (gg.KernelConfig(256, 256, 64, tile_classes=1, use_tensor_cores=False), False),
    (gg.KernelConfig(256, 256, 64, tile_classes=3), False),
    # small problems on the CUDA cores: any tensor-core config
    (gg.KernelConfig(128, 64, 64, tile_classes=2), True), (gg.KernelConfig(64, 64, 16, tile_classes=2), True),
    (gg.KernelConfig(128, 64, 64, tile_classes=2, use_tensor_cores=False), False),
])
def test_build_config_validation(cfg, ok):
    """Unsupported configs fail with cudaErrorInvalidValue (reference src/grouped_gemm.cu:121-123)."""
    ex = gg.GroupedGemmExecutor()
    prep = gg.prepare_problem_set([], cfg, gg.SortMode.kNone)
    st = ex.build(prep, cfg)
    assert (st == 0) == ok
    if not ok:
        assert st == capi.CUDA_ERROR_INVALID_VALUE
    ex.close()


def test_build_rejects_inconsistent_prepared_sets():
    cfg = gg.KernelConfig(128, 128, 64)
    probs = dims_problems([(64, 64, 64), (10, 10, 10)])
    prep = gg.prepare_problem_set(probs, cfg, gg.SortMode.kNone)
    ex = gg.GroupedGemmExecutor()
    bad = gg.PreparedProblemSet(prep.sorted_problems, prep.sorted_to_original, prep.tile_offsets[:-1], prep.total_tiles)
    assert ex.build(bad, cfg) == capi.CUDA_ERROR_INVALID_VALUE  # offsets size (src:1147-1149)
    bad = gg.PreparedProblemSet(prep.sorted_problems, prep.sorted_to_original, prep.tile_offsets, prep.total_tiles + 1)
    assert ex.build(bad, cfg) == capi.CUDA_ERROR_INVALID_VALUE  # back != total (src:1150-1152)
    neg = dims_problems([(64, -1, 64)])
    p2 = gg.prepare_problem_set(neg, cfg, gg.SortMode.kNone)
    assert ex.build(p2, cfg) == capi.CUDA_ERROR_INVALID_VALUE  # negative dims (src:1169-1171)
    nul = [gg.ProblemDesc(64, 64, 64, None, 0x10, None, 0x10, 64, 64, 64, 64)]
    p3 = gg.prepare_problem_set(nul, cfg, gg.SortMode.kNone)
    assert ex.build(p3, cfg) == capi.CUDA_ERROR_INVALID_DEVICE_POINTER  # null a (src:1172-1174)
    nul = [gg.ProblemDesc(64, 64, 64, 0x10, 0x10, None, None, 64, 64, 64, 64)]
    assert ex.build(gg.prepare_problem_set(nul, cfg, 0), cfg) == capi.CUDA_ERROR_INVALID_DEVICE_POINTER
    ex.close()
    # a destroyed executor answers like the reference's moved-from one (src:1135-1137, 1242-1244)
    assert ex.build(prep, cfg) == capi.CUDA_ERROR_INVALID_DEVICE_POINTER
    assert ex.run() == capi.CUDA_ERROR_INVALID_DEVICE_POINTER


def test_empty_sets_are_successful_noops_without_a_device():
    cfg = gg.KernelConfig()
    assert gg.run_grouped_gemm_once([], gg.SortMode.kByTiles, cfg) == 0
    assert gg.run_baseline_per_problem([], cfg) == 0
    # only zero-tile problems: nothing is launched either
    zero = dims_problems([(0, 64, 16), (64, 0, 16)])
    assert gg.run_grouped_gemm_once(zero, gg.SortMode.kNone, cfg) == 0
    ex = gg.GroupedGemmExecutor()
    assert ex.build(gg.prepare_problem_set(zero, cfg, 0), cfg) == 0
    assert ex.problem_count() == 2 and ex.total_tiles() == 0 and ex.grid_ctas() == 0
    assert ex.run() == 0
    ex.close()


def test_baseline_rejects_null_pointers_before_device_work():
    cfg = gg.KernelConfig()
    nul = [gg.ProblemDesc(64, 64, 64, 0x10, None, None, 0x10, 64, 64, 64, 64)]
    assert gg.run_baseline_per_problem(nul, cfg) == capi.CUDA_ERROR_INVALID_DEVICE_POINTER
    assert gg.run_baseline_per_problem(nul, gg.KernelConfig(16, 16, 16)) == capi.CUDA_ERROR_INVALID_VALUE


def test_query_occupancy_without_device_reports_cuda_error():
    # like the reference (src/grouped_gemm.cu:1024-1035) the CUDA error is passed through
    import torch

    if torch.cuda.is_available():
        pytest.skip("has a device")
    st, _ = gg.query_occupancy(gg.KernelConfig())
    assert st != 0
    st, _ = gg.query_occupancy(gg.KernelConfig(1, 2, 3))
    assert st == capi.CUDA_ERROR_INVALID_VALUE


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_c_header_compiles_as_plain_c(tmp_path):
    src = tmp_path / "abi.c"
    src.write_text('#include "grouped_gemm_b200.h"\n#include <stdio.h>\n'
                   'int main(void){ gg_problem p = {0}; gg_config c = {128,128,64,256,0,1};\n'
                   ' printf("%d %s %d\\n", gg_abi_version(), gg_sort_mode_name(2), gg_tile_count(&p,&c));\n'
                   ' return gg_abi_version() == GG_ABI_VERSION ? 0 : 1; }\n')
    exe = tmp_path / "abi"
    lib_dir = os.path.dirname(capi.LIB_PATH)
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I" + os.path.join(REPO, "include"), str(src), "-o", str(exe),
                    "-L" + lib_dir, "-lgrouped_gemm_b200", "-Wl,-rpath," + lib_dir], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    assert out.split() == ["2", "sort_by_tiles", "0"]


@pytest.mark.skipif(shutil.which("nvcc") is None and not os.path.exists("/usr/local/cuda/bin/nvcc"), reason="no nvcc")
def test_cpp_dropin_header_compiles_and_links(tmp_path):
    """A program written against the reference's API compiles against this header and links."""
    src = tmp_path / "dropin.cu"
    src.write_text('#include "grouped_gemm/grouped_gemm.cuh"\n#include <cstdio>\n'
                   'int main(){ using namespace grouped_gemm;\n'
                   ' std::vector<ProblemDesc> ps(3); ps[0].m=64; ps[0].n=64; ps[0].k=64; ps[1].m=0; ps[1].n=5; ps[1].k=1;\n'
                   ' ps[2].m=130; ps[2].n=70; ps[2].k=9; KernelConfig cfg;\n'
                   ' PreparedProblemSet p = prepare_problem_set(ps, cfg, SortMode::kByTiles);\n'
                   ' GroupedGemmExecutor ex; GroupedGemmExecutor ex2(std::move(ex));\n'
                   ' std::printf("%s %d %d %zu\\n", sort_mode_name(SortMode::kByK), p.total_tiles, count_non_empty_problems(ps, cfg), p.tile_offsets.size());\n'
                   ' return ex.build(p, cfg) == cudaErrorInvalidDevicePointer ? 0 : 1; }\n')
    exe = tmp_path / "dropin"
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    lib_dir = os.path.dirname(capi.LIB_PATH)
    subprocess.run([nvcc, "-std=c++17", "-I" + os.path.join(REPO, "include"), str(src), "-o", str(exe),
                    "-L" + lib_dir, "-lgrouped_gemm_b200", "-Xlinker", "-rpath," + lib_dir], check=True,
                   capture_output=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    assert out.split() == ["sort_by_k", str(1 + 0 + 6), "2", "4"]


def test_copy_rects_argument_checks_without_a_launch():
    """gg_copy_rects rejects bad arguments before touching the GPU; count 0 is a no-op."""
    lib = capi.load()
    assert lib.gg_copy_rects(None, None, 0, 1, None) == 0
    assert lib.gg_copy_rects(None, None, -1, 1, None) == 1
    assert lib.gg_copy_rects(None, None, 3, 0, None) == 1


def test_moe_plan_create_rejects_bad_arguments_before_device_work():
    """gg_moe_plan_create validates everything on the host first (no GPU needed for these)."""
    import ctypes

    lib = capi.load()
    cfg = gg.KernelConfig(128, 256, 64).to_c()
    b = (ctypes.c_void_p * 2)(ctypes.c_void_p(4096), ctypes.c_void_p(8192))
    good = dict(a=4096, b=ctypes.cast(b, ctypes.POINTER(ctypes.c_void_p)), c=None, d=4096, experts=2, n=64, k=64,
                capacity_rows=100, lda=64, ldb=64, ldc=64, ldd=64, alpha=1.0, beta=0.0)
    h = ctypes.c_void_p()

    def create(**kw):
        args = dict(good)
        args.update(kw)
        prob = capi.GGMoeProblem(**args)
        return lib.gg_moe_plan_create(ctypes.byref(prob), ctypes.byref(cfg), ctypes.byref(h))

    assert lib.gg_moe_plan_create(None, ctypes.byref(cfg), ctypes.byref(h)) == 1
    assert create(experts=0) == 1
    assert create(a=None) == 1
    assert create(d=None) == 1
    assert create(lda=8) == 1
    assert create(capacity_rows=-1) == 1
    nullb = (ctypes.c_void_p * 2)(ctypes.c_void_p(4096), None)
    assert create(b=ctypes.cast(nullb, ctypes.POINTER(ctypes.c_void_p))) == 1
    bad_cfg = gg.KernelConfig(96, 96, 64).to_c()
    prob = capi.GGMoeProblem(**good)
    assert lib.gg_moe_plan_create(ctypes.byref(prob), ctypes.byref(bad_cfg), ctypes.byref(h)) == 1
    assert lib.gg_moe_plan_run(None, None, None) == 17


def test_input_type_is_validated_on_the_host():
    """input_type must be GG_INPUT_F16 (0), GG_INPUT_BF16 (1), GG_INPUT_E4M3 (2) or GG_INPUT_E5M2 (3);
    anything else is an invalid config."""
    for t, want in ((0, 0), (1, 0), (2, 0), (3, 0), (4, 1), (-1, 1)):
        cfg = gg.KernelConfig(128, 128, 64, input_type=t)
        ex = gg.GroupedGemmExecutor()
        prep = gg.prepare_problem_set([], cfg, 0)
        assert ex.build(prep, cfg) == want
        ex.close()


def test_output_type_and_activation_are_validated_on_the_host():
    """output_type must be GG_OUTPUT_F32/F16/BF16 (0..2) and activation GG_ACT_NONE/RELU/GELU
    (0..2); anything else is an invalid config (status 1), checked before any device work."""
    for out, act, want in ((0, 0, 0), (1, 2, 0), (2, 1, 0), (3, 0, 1), (-1, 0, 1), (0, 3, 1), (1, -1, 1)):
        cfg = gg.KernelConfig(128, 128, 64, output_type=out, activation=act)
        ex = gg.GroupedGemmExecutor()
        prep = gg.prepare_problem_set([], cfg, 0)
        assert ex.build(prep, cfg) == want
        assert ex.build(prep, cfg, bias=[]) == want
        ex.close()


def test_bias_table_length_must_match_the_problem_count():
    cfg = gg.KernelConfig(128, 128, 64)
    ex = gg.GroupedGemmExecutor()
    prep = gg.prepare_problem_set([], cfg, 0)
    assert ex.build(prep, cfg, bias=[None]) == gg.capi.CUDA_ERROR_INVALID_VALUE
    ex.close()


def test_fp8_inputs_need_128_column_b_tiles_on_the_tensor_cores():
    """8-bit B fills 128-column shared-memory chunks: tensor-core tiles whose per-CTA B width is not a
    multiple of 128 are an invalid config with E4M3 / E5M2 inputs; the CUDA-core path takes them."""
    ok = [(128, 256, 64), (128, 128, 64), (64, 128, 32), (256, 256, 64)]
    bad = [(64, 64, 16), (128, 64, 32), (128, 64, 64), (256, 128, 64)]
    for fmt in (2, 3):
        for shape, want in [(s, 0) for s in ok] + [(s, 1) for s in bad]:
            for tc in (True, False):
                cfg = gg.KernelConfig(*shape, use_tensor_cores=tc, input_type=fmt)
                ex = gg.GroupedGemmExecutor()
                assert ex.build(gg.prepare_problem_set([], cfg, 0), cfg) == (want if tc else 0), (shape, tc)
                ex.close()
    cfg = gg.KernelConfig(128, 128, 64, input_type=4)
    ex = gg.GroupedGemmExecutor()
    assert ex.build(gg.prepare_problem_set([], cfg, 0), cfg) == 1
    ex.close()


def test_layouts_are_validated_on_the_host():
    """a_layout / b_layout must be GG_LAYOUT_ROW_MAJOR (0) or GG_LAYOUT_COL_MAJOR (1); with 8-bit
    inputs on the tensor cores a column-major A needs 128-row tiles per CTA and a column-major B
    lifts the 128-column rule of a row-major B."""
    cases = [((128, 128, 64), 0, 0, 1, 0, 0), ((128, 128, 64), 0, 1, 1, 0, 0), ((128, 128, 64), 0, 2, 0, 0, 1),
             ((128, 128, 64), 0, 0, -1, 0, 1),
             ((128, 64, 64), 2, 0, 1, 0, 0), ((128, 64, 64), 2, 0, 0, 0, 1),     # 8-bit B: K-major lifts the rule
             ((64, 128, 32), 2, 1, 0, 0, 1), ((64, 128, 32), 2, 1, 0, 1, 1),     # 8-bit MN-major A needs 128 rows
             ((64, 128, 32), 2, 0, 0, 0, 0), ((256, 128, 64), 3, 1, 1, 0, 0)]
    for shape, in_t, a_l, b_l, simt, want in cases:
        cfg = gg.KernelConfig(*shape, input_type=in_t, a_layout=a_l, b_layout=b_l, use_tensor_cores=not simt)
        ex = gg.GroupedGemmExecutor()
        got = ex.build(gg.prepare_problem_set([], cfg, 0), cfg)
        ex.close()
        assert got == (0 if simt and a_l in (0, 1) and b_l in (0, 1) else want), (shape, in_t, a_l, b_l, simt)


def test_ipc_entry_points_check_arguments_before_device_work():
    """gg_ipc_export / gg_ipc_open / gg_ipc_close reject null arguments, and closing a pointer that
    gg_ipc_open did not return, with cudaErrorInvalidValue (1) and no CUDA call."""
    import ctypes

    lib = gg.capi.load()
    h = gg.capi.GGIpcHandle()
    assert lib.gg_ipc_export(None, ctypes.byref(h)) == 1
    assert lib.gg_ipc_export(ctypes.c_void_p(0x1000), None) == 1
    ptr = ctypes.c_void_p()
    assert lib.gg_ipc_open(None, ctypes.byref(ptr)) == 1
    assert lib.gg_ipc_open(ctypes.byref(h), None) == 1
    assert lib.gg_ipc_close(None) == 1
    assert lib.gg_ipc_close(ctypes.c_void_p(0x1000)) == 1
    assert ctypes.sizeof(gg.capi.GGIpcHandle) == 80


@pytest.mark.parametrize("cfg,max_problems", [
    (gg.KernelConfig(256, 256, 64), 16),                          # CTA pairs
    (gg.KernelConfig(128, 128, 64, a_layout=1), 16),              # column-major A
    (gg.KernelConfig(128, 128, 64, tile_classes=2), 16),          # tile classes
    (gg.KernelConfig(32, 32, 16), 16),                            # unsupported tile
    (gg.KernelConfig(128, 128, 64), 0),                           # no room
    (gg.KernelConfig(128, 128, 64), capi.GG_DEVICE_PLAN_MAX_PROBLEMS + 1),
])
def test_device_plan_rejects_configs_before_device_work(cfg, max_problems):
    with pytest.raises(ValueError, match="status 1"):
        gg.DevicePlan(cfg, max_problems)
