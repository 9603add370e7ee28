"""CPU oracle for the grouped GEMM path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs may
import this package, and only as the checker or the timed CPU baseline. The product library
(``grouped_gemm_gpu_kernel_b200``) never imports it and has no CPU fallback.

Two native libraries back it:

* ``oracle/liboracle.so`` -- ``gg_oracle.c``, the C restatement of the reference's host algorithm
  (reference ``src/grouped_gemm.cu:54-65,967-1022`` and ``tests/test_correctness.cu:85-102``) and
  the FP64 accuracy reference.
* ``oracle/_ref/libgg_ref.so`` -- the reference's own sources compiled unmodified (see
  ``oracle/Makefile``) plus ``ref_shim.cu``; used to pin the restatement and as the
  ``"reference"`` CPU baseline. Absent when the reference tree was not available at build time.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libgg_ref.so")

SORT_MODES = (0, 1, 2, 3)


class RefProblem(ctypes.Structure):
    """Layout of ``gg_problem`` / ``grouped_gemm::ProblemDesc`` (reference grouped_gemm.cuh:18-35)."""

    _fields_ = [
        ("m", ctypes.c_int), ("n", ctypes.c_int), ("k", ctypes.c_int),
        ("a", ctypes.c_void_p), ("b", ctypes.c_void_p), ("c", ctypes.c_void_p), ("d", ctypes.c_void_p),
        ("lda", ctypes.c_int), ("ldb", ctypes.c_int), ("ldc", ctypes.c_int), ("ldd", ctypes.c_int),
        ("alpha", ctypes.c_float), ("beta", ctypes.c_float),
    ]


_P = ctypes.POINTER
_i32p = _P(ctypes.c_int)
_u16p = _P(ctypes.c_uint16)
_f32p = _P(ctypes.c_float)
_f64p = _P(ctypes.c_double)

_oracle: Optional[ctypes.CDLL] = None
_ref: Optional[ctypes.CDLL] = None


def load_oracle() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_SO):
            raise FileNotFoundError(f"{ORACLE_SO} missing: run `make -C oracle oracle`")
        lib = ctypes.CDLL(ORACLE_SO)
        lib.oracle_tile_count.argtypes = [ctypes.c_int] * 4
        lib.oracle_tile_count.restype = ctypes.c_int
        lib.oracle_prepare.argtypes = [_i32p, _i32p, _i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int, _i32p, _i32p]
        lib.oracle_prepare.restype = ctypes.c_int
        lib.oracle_gemm_f64.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, _u16p, ctypes.c_int,
                                        _u16p, ctypes.c_int, _f32p, ctypes.c_int, ctypes.c_float,
                                        ctypes.c_float, _i32p, ctypes.c_int, _f64p, ctypes.c_int, _f64p]
        lib.oracle_gemm_f64.restype = None
        lib.oracle_gemm_f64_fmt.argtypes = lib.oracle_gemm_f64.argtypes + [ctypes.c_int]
        lib.oracle_gemm_f64_fmt.restype = None
        lib.oracle_gemm_f64_epilogue.argtypes = [
            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
            _f32p, ctypes.c_int, ctypes.c_float, ctypes.c_float, _i32p, ctypes.c_int, _f64p, ctypes.c_int, _f64p,
            ctypes.c_int, ctypes.POINTER(ctypes.c_float), ctypes.c_int]
        lib.oracle_gemm_f64_epilogue.restype = None
        lib.oracle_fp8_to_double.argtypes = [ctypes.c_uint8, ctypes.c_int]
        lib.oracle_fp8_to_double.restype = ctypes.c_double
        lib.oracle_bf16_to_double.argtypes = [ctypes.c_uint16]
        lib.oracle_bf16_to_double.restype = ctypes.c_double
        lib.oracle_gemm_f32_refloop.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, _u16p,
                                                ctypes.c_int, _u16p, ctypes.c_int, _f32p, ctypes.c_int,
                                                ctypes.c_float, ctypes.c_float, _f32p, ctypes.c_int]
        lib.oracle_gemm_f32_refloop.restype = None
        lib.oracle_half_to_double.argtypes = [ctypes.c_uint16]
        lib.oracle_half_to_double.restype = ctypes.c_double
        _oracle = lib
    return _oracle


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def load_ref() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError(f"{REF_SO} missing: run `make -C oracle ref` where the reference tree exists")
        lib = ctypes.CDLL(REF_SO)
        rp = _P(RefProblem)
        lib.ref_prepare.argtypes = [rp, ctypes.c_int] + [ctypes.c_int] * 4 + [_i32p, _i32p]
        lib.ref_prepare.restype = ctypes.c_int
        lib.ref_sort_mode_name.argtypes = [ctypes.c_int]
        lib.ref_sort_mode_name.restype = ctypes.c_char_p
        lib.ref_count_non_empty.argtypes = [rp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.ref_count_non_empty.restype = ctypes.c_int
        lib.ref_host_gemm_batch.argtypes = [rp, ctypes.c_int, _P(ctypes.c_void_p), _P(ctypes.c_void_p),
                                            _P(ctypes.c_void_p), _P(ctypes.c_void_p), ctypes.c_int]
        lib.ref_host_gemm_batch.restype = ctypes.c_double
        lib.ref_test_inputs.argtypes = [_i32p, ctypes.c_int, _u16p, _u16p, _f32p, _f32p, _f32p, _f32p]
        lib.ref_test_inputs.restype = ctypes.c_int
        lib.ref_test_inputs_host.argtypes = [_i32p, ctypes.c_int, ctypes.c_uint, _u16p, _u16p, _f32p, _f32p,
                                             _f32p, _f32p]
        lib.ref_test_inputs_host.restype = ctypes.c_int
        lib.ref_run_grouped_once.argtypes = [rp, ctypes.c_int] + [ctypes.c_int] * 5 + [ctypes.c_void_p]
        lib.ref_run_grouped_once.restype = ctypes.c_int
        lib.ref_run_baseline.argtypes = [rp, ctypes.c_int] + [ctypes.c_int] * 4 + [ctypes.c_void_p]
        lib.ref_run_baseline.restype = ctypes.c_int
        lib.ref_time_grouped.argtypes = [rp, ctypes.c_int] + [ctypes.c_int] * 7 + [
            ctypes.c_void_p, _f32p, _i32p, _i32p]
        lib.ref_time_grouped.restype = ctypes.c_int
        _ref = lib
    return _ref


def safe_elems(rows: int, cols: int) -> int:
    """Element count the reference allocates for a rows x cols matrix: at least one element
    (reference tests/test_correctness.cu:75-80)."""
    return 1 if rows <= 0 or cols <= 0 else int(rows) * int(cols)


def _ptr(arr: np.ndarray, ctype):
    return arr.ctypes.data_as(_P(ctype))


def problems_from_dims(dims: Sequence[Sequence[int]]) -> "ctypes.Array":
    """Pointer-free RefProblem array for host-only preparation calls."""
    arr = (RefProblem * max(1, len(dims)))()
    for i, (m, n, k) in enumerate(dims):
        arr[i].m, arr[i].n, arr[i].k = int(m), int(n), int(k)
        arr[i].lda, arr[i].ldb, arr[i].ldc, arr[i].ldd = max(1, int(k)), max(1, int(n)), max(1, int(n)), max(1, int(n))
        arr[i].alpha, arr[i].beta = 1.0, 0.0
    return arr


# ---- the C restatement -----------------------------------------------------------------------

def tile_count(m: int, n: int, cta_m: int, cta_n: int) -> int:
    return load_oracle().oracle_tile_count(m, n, cta_m, cta_n)


def prepare(dims: Sequence[Sequence[int]], cta_m: int, cta_n: int, mode: int):
    """(sorted_to_original, tile_offsets, total_tiles), restating reference src/grouped_gemm.cu:967-1022."""
    lib = load_oracle()
    d = np.asarray(dims, dtype=np.int32).reshape(-1, 3)
    count = d.shape[0]
    m, n, k = (np.ascontiguousarray(d[:, i]) for i in range(3))
    perm = np.zeros(max(1, count), dtype=np.int32)
    offs = np.zeros(count + 1, dtype=np.int32)
    total = lib.oracle_prepare(_ptr(m, ctypes.c_int), _ptr(n, ctypes.c_int), _ptr(k, ctypes.c_int), count,
                               cta_m, cta_n, mode, _ptr(perm, ctypes.c_int), _ptr(offs, ctypes.c_int))
    if total < 0:
        raise ValueError("oracle_prepare rejected its arguments")
    return perm[:count], offs, int(total)


def gemm_f64(m, n, k, a, lda, b, ldb, c, ldc, alpha, beta, rows=None, fmt=0, bias=None, act=0):
    """FP64 D (and the error scale) for one problem; `a`/`b` are bit arrays of FP16 (fmt 0) or
    BF16 (fmt 1) values (2 bytes each), or of E4M3 (fmt 2) or E5M2 (fmt 3) values (1 byte). `bias` (n float32 values, one per output column, or None)
    and `act` (0 none, 1 ReLU, 2 GELU tanh form) give the library's epilogue extensions:
    D = act(alpha * A x B + beta * C + bias).

    Returns (d, scale), each shaped (len(rows) or m, n).
    """
    lib = load_oracle()
    elem = np.uint8 if int(fmt) in (2, 3) else np.uint16
    a = np.ascontiguousarray(a).view(elem)
    b = np.ascontiguousarray(b).view(elem)
    nrows = m if rows is None else len(rows)
    d = np.zeros((max(nrows, 1), max(n, 1)), dtype=np.float64)
    s = np.zeros_like(d)
    if m <= 0 or n <= 0 or nrows == 0:
        return d[:nrows, :max(n, 0)], s[:nrows, :max(n, 0)]
    rows_arr = None if rows is None else np.ascontiguousarray(rows, dtype=np.int32)
    c_arr = None if c is None else np.ascontiguousarray(c, dtype=np.float32)
    bias_arr = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    if bias_arr is not None and bias_arr.size < n:
        raise ValueError("bias needs one value per output column")
    lib.oracle_gemm_f64_epilogue(m, n, k, a.ctypes.data, lda, b.ctypes.data, ldb,
                                 None if c_arr is None else _ptr(c_arr, ctypes.c_float), ldc,
                                 float(alpha), float(beta),
                                 None if rows_arr is None else _ptr(rows_arr, ctypes.c_int), nrows,
                                 _ptr(d, ctypes.c_double), n, _ptr(s, ctypes.c_double), int(fmt),
                                 None if bias_arr is None else _ptr(bias_arr, ctypes.c_float), int(act))
    return d, s


def gemm_f32_refloop(m, n, k, a, lda, b, ldb, c, ldc, alpha, beta, ldd):
    """FP32 natural-order host GEMM restating reference tests/test_correctness.cu:85-102."""
    lib = load_oracle()
    a = np.ascontiguousarray(a).view(np.uint16)
    b = np.ascontiguousarray(b).view(np.uint16)
    c = np.ascontiguousarray(c, dtype=np.float32)
    d = np.zeros(max(1, m * ldd), dtype=np.float32)
    lib.oracle_gemm_f32_refloop(m, n, k, _ptr(a, ctypes.c_uint16), lda, _ptr(b, ctypes.c_uint16), ldb,
                                _ptr(c, ctypes.c_float), ldc, float(alpha), float(beta),
                                _ptr(d, ctypes.c_float), ldd)
    return d


# ---- the reference's own host code (oracle/_ref) ----------------------------------------------

def ref_prepare(dims: Sequence[Sequence[int]], cta_m: int, cta_n: int, cta_k: int, mode: int):
    lib = load_ref()
    arr = problems_from_dims(dims)
    count = len(dims)
    perm = np.zeros(max(1, count), dtype=np.int32)
    offs = np.zeros(count + 1, dtype=np.int32)
    total = lib.ref_prepare(arr, count, cta_m, cta_n, cta_k, mode, _ptr(perm, ctypes.c_int), _ptr(offs, ctypes.c_int))
    return perm[:count], offs, int(total)


def ref_sort_mode_name(mode: int) -> str:
    return load_ref().ref_sort_mode_name(mode).decode()


def ref_count_non_empty(dims, cta_m, cta_n, cta_k) -> int:
    return load_ref().ref_count_non_empty(problems_from_dims(dims), len(dims), cta_m, cta_n, cta_k)


def ref_host_gemm(problems: Sequence[dict], threads: int = 1):
    """Run the reference's compute_reference over host problems.

    Each problem dict holds m, n, k, lda, ldb, ldc, ldd, alpha, beta and host arrays a (uint16),
    b (uint16), c (float32). Returns (list of float32 D arrays, seconds in compute_reference).
    """
    lib = load_ref()
    count = len(problems)
    arr = (RefProblem * max(1, count))()
    keep = []
    ap = (ctypes.c_void_p * max(1, count))()
    bp = (ctypes.c_void_p * max(1, count))()
    cp = (ctypes.c_void_p * max(1, count))()
    dp = (ctypes.c_void_p * max(1, count))()
    outs = []
    for i, p in enumerate(problems):
        a = np.ascontiguousarray(p["a"]).view(np.uint16)
        b = np.ascontiguousarray(p["b"]).view(np.uint16)
        c = np.ascontiguousarray(p["c"], dtype=np.float32)
        # the shim copies safe_matrix_elems(rows, ld) elements of each operand
        # (reference tests/test_correctness.cu:75-80), so every buffer must hold at least that many
        if a.size < safe_elems(p["m"], p["lda"]) or b.size < safe_elems(p["k"], p["ldb"]) or \
                c.size < safe_elems(p["m"], p["ldc"]):
            raise ValueError(f"problem {i}: host buffers smaller than the reference's allocation rule")
        d = np.zeros(safe_elems(p["m"], p["ldd"]), dtype=np.float32)
        keep += [a, b, c]
        outs.append(d)
        arr[i].m, arr[i].n, arr[i].k = p["m"], p["n"], p["k"]
        arr[i].lda, arr[i].ldb, arr[i].ldc, arr[i].ldd = p["lda"], p["ldb"], p["ldc"], p["ldd"]
        arr[i].alpha, arr[i].beta = p["alpha"], p["beta"]
        ap[i], bp[i], cp[i], dp[i] = a.ctypes.data, b.ctypes.data, c.ctypes.data, d.ctypes.data
    secs = lib.ref_host_gemm_batch(arr, count, ap, bp, cp, dp, threads)
    return outs, float(secs)


# ---- accuracy metric shared by every parity test ------------------------------------------------

def tolerance(k: int) -> float:
    """The accuracy bound: max relative error 2e-3 * sqrt(K/1024), K floored at 1."""
    return 2e-3 * float(np.sqrt(max(int(k), 1) / 1024.0))


# Rounding of D to a 16-bit output type (library output_type 1 = FP16, 2 = BF16): relative unit
# roundoff, and the absolute half-spacing of the format's subnormals.
OUTPUT_ROUNDING = {0: (0.0, 0.0), 1: (2.0 ** -11, 2.0 ** -25), 2: (2.0 ** -8, 2.0 ** -134)}


def rel_err(d, ref, scale, out_fmt: int = 0) -> float:
    """max |d - ref| / max(|ref|, scale), with scale = |alpha|*sqrt(sum (a*b)^2) + |beta*c|.

    The scale is the magnitude of a random-sign sum of the K products, so outputs that cancel to
    near zero are judged against the size of their terms rather than against ~0. For a 16-bit D
    (out_fmt 1 or 2) the final rounding to that format, u*|ref| + the subnormal half-spacing, is
    taken off the error first: the bound then applies to the FP32 result before its rounding.
    """
    d = np.asarray(d, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if d.size == 0:
        return 0.0
    u, floor = OUTPUT_ROUNDING[int(out_fmt)]
    denom = np.maximum(np.maximum(np.abs(ref), np.asarray(scale, dtype=np.float64)), 1e-30)
    err = np.maximum(np.abs(d - ref) - u * np.abs(ref) - floor, 0.0) / denom
    if not np.all(np.isfinite(d)):
        return float("inf")
    return float(err.max())
