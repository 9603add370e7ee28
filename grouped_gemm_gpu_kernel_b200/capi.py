"""ctypes binding of the C-ABI in include/grouped_gemm_b200.h (libgrouped_gemm_b200.so).

This is the boundary the Python tests and bench.py call through. Loading fails loudly when the
library is missing: there is no fallback implementation of the path.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libgrouped_gemm_b200.so")

# Every declaration of include/grouped_gemm_b200.h; tests check the library exports each one.
EXPORTED_SYMBOLS = (
    "gg_abi_version", "gg_sort_mode_name", "gg_tile_count", "gg_prepare", "gg_query_occupancy",
    "gg_executor_create", "gg_executor_destroy", "gg_executor_build", "gg_executor_build_with_bias",
    "gg_executor_run",
    "gg_executor_problem_count", "gg_executor_total_tiles", "gg_executor_grid_ctas", "gg_executor_launches",
    "gg_executor_status",
    "gg_run_grouped_gemm_once", "gg_run_baseline_per_problem", "gg_count_non_empty_problems",
    "gg_partition", "gg_selftest_wait_timeout", "gg_run_grouped_gemm_noalloc", "gg_copy_rects",
    "gg_baseline_status", "gg_noalloc_status", "gg_selftest_wait_timeout_word",
    "gg_moe_plan_create", "gg_moe_plan_run", "gg_moe_plan_status", "gg_moe_plan_destroy",
    "gg_ipc_export", "gg_ipc_open", "gg_ipc_close",
    "gg_device_plan_create", "gg_device_plan_run", "gg_device_plan_status", "gg_device_plan_prepared",
    "gg_device_plan_destroy",
)
GG_STATUS_BAD_ROWS = 0x100
GG_STATUS_BAD_PROBLEMS = 0x200
GG_DEVICE_PLAN_MAX_PROBLEMS = 4096
GG_INPUT_F16 = 0
GG_INPUT_BF16 = 1
GG_INPUT_E4M3 = 2
GG_INPUT_E5M2 = 3
GG_OUTPUT_F32 = 0
GG_OUTPUT_F16 = 1
GG_OUTPUT_BF16 = 2
GG_ACT_NONE = 0
GG_ACT_RELU = 1
GG_ACT_GELU = 2
GG_LAYOUT_ROW_MAJOR = 0
GG_LAYOUT_COL_MAJOR = 1
GG_TILE_CLASSES_NONE = 0
GG_TILE_CLASSES_PAIR_BLOCKS = 1
GG_TILE_CLASSES_SMALL_ON_CUDA_CORES = 2
GG_SMALL_PROBLEM_DIM = 64
GG_SMALL_ZERO_FILL_VOLUME = 1 << 25
GG_NOALLOC_MAX_PROBLEMS = 1024

GG_STATUS_TIMEOUT_PRODUCER = 0x1
GG_STATUS_TIMEOUT_MMA = 0x2
GG_STATUS_TIMEOUT_EPILOGUE = 0x4
GG_STATUS_TIMEOUT_SCHEDULER = 0x8
GG_STATUS_WORD_BASELINE = 0
GG_STATUS_WORD_NOALLOC = 1

CUDA_SUCCESS = 0
CUDA_ERROR_INVALID_VALUE = 1
CUDA_ERROR_INVALID_DEVICE_POINTER = 17
CUDA_ERROR_LAUNCH_TIMEOUT = 702


class GGProblem(ctypes.Structure):
    _fields_ = [
        ("m", ctypes.c_int), ("n", ctypes.c_int), ("k", ctypes.c_int),
        ("a", ctypes.c_void_p), ("b", ctypes.c_void_p), ("c", ctypes.c_void_p), ("d", ctypes.c_void_p),
        ("lda", ctypes.c_int), ("ldb", ctypes.c_int), ("ldc", ctypes.c_int), ("ldd", ctypes.c_int),
        ("alpha", ctypes.c_float), ("beta", ctypes.c_float),
    ]


class GGConfig(ctypes.Structure):
    _fields_ = [("cta_m", ctypes.c_int), ("cta_n", ctypes.c_int), ("cta_k", ctypes.c_int),
                ("threads", ctypes.c_int), ("persistent_ctas", ctypes.c_int), ("use_tensor_cores", ctypes.c_int),
                ("input_type", ctypes.c_int), ("output_type", ctypes.c_int), ("activation", ctypes.c_int),
                ("a_layout", ctypes.c_int), ("b_layout", ctypes.c_int), ("tile_classes", ctypes.c_int)]


class GGOccupancy(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int) for name in (
        "sm_count", "max_blocks_per_sm", "active_blocks_per_sm", "threads_per_block", "max_threads_per_sm",
        "warps_per_block", "max_warps_per_sm", "active_warps_per_sm", "max_registers_per_sm",
        "max_registers_per_block", "estimated_registers_per_thread", "estimated_registers_per_block",
        "registers_per_thread", "registers_per_block", "register_limited_blocks_per_sm", "static_shared_bytes",
        "dynamic_shared_bytes")] + [("theoretical_occupancy", ctypes.c_float), ("using_tensor_cores", ctypes.c_int)]


class GGShardPiece(ctypes.Structure):
    _fields_ = [("problem", ctypes.c_int), ("row0", ctypes.c_int), ("rows", ctypes.c_int),
                ("col0", ctypes.c_int), ("cols", ctypes.c_int)]


class GGRectCopy(ctypes.Structure):
    _fields_ = [("strided", ctypes.c_void_p), ("packed", ctypes.c_longlong), ("rows", ctypes.c_int),
                ("cols", ctypes.c_int), ("ld", ctypes.c_int), ("reserved", ctypes.c_int)]


class GGMoeProblem(ctypes.Structure):
    _fields_ = [("a", ctypes.c_void_p), ("b", ctypes.POINTER(ctypes.c_void_p)), ("c", ctypes.c_void_p),
                ("d", ctypes.c_void_p), ("experts", ctypes.c_int), ("n", ctypes.c_int), ("k", ctypes.c_int),
                ("capacity_rows", ctypes.c_int), ("lda", ctypes.c_int), ("ldb", ctypes.c_int), ("ldc", ctypes.c_int),
                ("ldd", ctypes.c_int), ("alpha", ctypes.c_float), ("beta", ctypes.c_float),
                ("bias", ctypes.POINTER(ctypes.c_void_p))]


class GGIpcHandle(ctypes.Structure):
    _fields_ = [("handle", ctypes.c_ubyte * 64), ("offset", ctypes.c_ulonglong), ("bytes", ctypes.c_ulonglong)]


_lib: Optional[ctypes.CDLL] = None


def load() -> ctypes.CDLL:
    """Load libgrouped_gemm_b200.so (raises when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing; build it with `python -m grouped_gemm_gpu_kernel_b200.build`")
    lib = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER
    pp, pc, i32p = P(GGProblem), P(GGConfig), P(ctypes.c_int)
    vp = ctypes.c_void_p
    sig = {
        "gg_abi_version": ([], ctypes.c_int),
        "gg_sort_mode_name": ([ctypes.c_int], ctypes.c_char_p),
        "gg_tile_count": ([pp, pc], ctypes.c_int),
        "gg_prepare": ([pp, ctypes.c_int, pc, ctypes.c_int, pp, i32p, i32p, i32p], ctypes.c_int),
        "gg_query_occupancy": ([pc, P(GGOccupancy)], ctypes.c_int),
        "gg_executor_create": ([P(vp)], ctypes.c_int),
        "gg_executor_destroy": ([vp], None),
        "gg_executor_build": ([vp, pp, ctypes.c_int, i32p, ctypes.c_int, ctypes.c_int, pc], ctypes.c_int),
        "gg_executor_build_with_bias": ([vp, pp, ctypes.c_int, i32p, ctypes.c_int, ctypes.c_int, pc, P(vp)],
                                        ctypes.c_int),
        "gg_executor_run": ([vp, vp], ctypes.c_int),
        "gg_executor_problem_count": ([vp], ctypes.c_int),
        "gg_executor_total_tiles": ([vp], ctypes.c_int),
        "gg_executor_grid_ctas": ([vp], ctypes.c_int),
        "gg_executor_launches": ([vp], ctypes.c_int),
        "gg_executor_status": ([vp, i32p], ctypes.c_int),
        "gg_run_grouped_gemm_once": ([pp, ctypes.c_int, ctypes.c_int, pc, vp], ctypes.c_int),
        "gg_run_baseline_per_problem": ([pp, ctypes.c_int, pc, vp], ctypes.c_int),
        "gg_count_non_empty_problems": ([pp, ctypes.c_int, pc], ctypes.c_int),
        "gg_partition": ([pp, ctypes.c_int, pc, ctypes.c_int, ctypes.c_int, P(GGShardPiece), ctypes.c_int, i32p,
                          P(ctypes.c_double)], ctypes.c_int),
        "gg_selftest_wait_timeout": ([ctypes.c_ulonglong, i32p], ctypes.c_int),
        "gg_run_grouped_gemm_noalloc": ([pp, ctypes.c_int, ctypes.c_int, pc, vp], ctypes.c_int),
        "gg_baseline_status": ([i32p], ctypes.c_int),
        "gg_noalloc_status": ([i32p], ctypes.c_int),
        "gg_selftest_wait_timeout_word": ([ctypes.c_int, ctypes.c_ulonglong], ctypes.c_int),
        "gg_copy_rects": ([vp, vp, ctypes.c_int, ctypes.c_int, vp], ctypes.c_int),
        "gg_moe_plan_create": ([P(GGMoeProblem), pc, P(vp)], ctypes.c_int),
        "gg_moe_plan_run": ([vp, vp, vp], ctypes.c_int),
        "gg_moe_plan_status": ([vp, i32p, i32p], ctypes.c_int),
        "gg_moe_plan_destroy": ([vp], None),
        "gg_ipc_export": ([vp, P(GGIpcHandle)], ctypes.c_int),
        "gg_ipc_open": ([P(GGIpcHandle), P(vp)], ctypes.c_int),
        "gg_ipc_close": ([vp], ctypes.c_int),
        "gg_device_plan_create": ([pc, ctypes.c_int, P(vp)], ctypes.c_int),
        "gg_device_plan_run": ([vp, vp, vp, ctypes.c_int, vp], ctypes.c_int),
        "gg_device_plan_status": ([vp, i32p, i32p], ctypes.c_int),
        "gg_device_plan_prepared": ([vp, i32p, i32p, ctypes.c_int], ctypes.c_int),
        "gg_device_plan_destroy": ([vp], None),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib
