"""B200 (sm_100a) grouped GEMM: Python mirror of the reference's C++ API.

The names, argument meanings and error behaviour follow the reference header
(reference include/grouped_gemm/grouped_gemm.cuh:9-132): functions that can fail return the
cudaError_t value as an int (0 = success), ``prepare_problem_set`` is pure host code, and device
buffers are passed as raw device pointers (ints). Every call goes through the C-ABI of
``libgrouped_gemm_b200.so`` (include/grouped_gemm_b200.h); nothing here computes a GEMM.

    import grouped_gemm_gpu_kernel_b200 as gg
    probs = [gg.problem_from_tensors(A, B, C, D, alpha=1.0, beta=0.0), ...]
    cfg = gg.KernelConfig(cta_m=128, cta_n=128, cta_k=64)
    prep = gg.prepare_problem_set(probs, cfg, gg.SortMode.kByTiles)
    ex = gg.GroupedGemmExecutor(); assert ex.build(prep, cfg) == 0; ex.run(stream)
"""
from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

from . import capi

__all__ = [
    "SortMode", "ProblemDesc", "KernelConfig", "PreparedProblemSet", "OccupancyInfo", "GroupedGemmExecutor",
    "prepare_problem_set", "sort_mode_name", "query_occupancy", "run_grouped_gemm_once",
    "run_baseline_per_problem", "count_non_empty_problems", "partition", "ShardPiece", "problem_from_tensors",
    "NATIVE_CONFIGS", "REFERENCE_CONFIGS", "PAIR_CONFIGS", "selftest_wait_timeout", "capi", "MoePlan",
    "selftest_wait_timeout_word", "baseline_status", "noalloc_status", "DevicePlan",
    "InputType", "OutputType", "Activation", "Layout", "TileClasses",
]


class SortMode(enum.IntEnum):
    kNone = 0
    kByK = 1
    kByTiles = 2
    kByTilesThenK = 3


class InputType(enum.IntEnum):
    """Element type of every A and B (GG_INPUT_*); the reference's is FP16."""
    kF16 = capi.GG_INPUT_F16
    kBF16 = capi.GG_INPUT_BF16
    kE4M3 = capi.GG_INPUT_E4M3   # 8-bit float, 4 exponent bits, no infinities
    kE5M2 = capi.GG_INPUT_E5M2   # 8-bit float, 5 exponent bits


class OutputType(enum.IntEnum):
    """Element type of every C and D (GG_OUTPUT_*); the reference's is FP32."""
    kF32 = capi.GG_OUTPUT_F32
    kF16 = capi.GG_OUTPUT_F16
    kBF16 = capi.GG_OUTPUT_BF16


class Layout(enum.IntEnum):
    """Storage of A or B (GG_LAYOUT_*): row-major (the reference's: A m x k, B k x n) or
    column-major (A stored k x m with lda >= m, B stored n x k with ldb >= k)."""
    kRowMajor = capi.GG_LAYOUT_ROW_MAJOR
    kColMajor = capi.GG_LAYOUT_COL_MAJOR


class TileClasses(enum.IntEnum):
    """How an executor tiles its problems (GG_TILE_CLASSES_*): one tile shape for every problem (the
    reference's); with a CTA-pair config, whole 256-row blocks on CTA pairs and the rows left over
    on one-CTA 128-row tiles, as two launches that may overlap; or, on the CUDA-core kernel with
    64 x 64 tiles, the problems with m, n, k all at most capi.GG_SMALL_PROBLEM_DIM and those of at
    most capi.GG_SMALL_ZERO_FILL_VOLUME multiply-adds whose A or B TMA cannot load, the rest on the
    tensor cores."""
    kNone = capi.GG_TILE_CLASSES_NONE
    kPairBlocks = capi.GG_TILE_CLASSES_PAIR_BLOCKS
    kSmallOnCudaCores = capi.GG_TILE_CLASSES_SMALL_ON_CUDA_CORES


class Activation(enum.IntEnum):
    """Applied to D after the bias (GG_ACT_*); GELU is the tanh form."""
    kNone = capi.GG_ACT_NONE
    kReLU = capi.GG_ACT_RELU
    kGELU = capi.GG_ACT_GELU


@dataclass
class ProblemDesc:
    """D = alpha * A x B + beta * C; A m x k FP16, B k x n FP16, C/D m x n FP32, all row-major."""

    m: int
    n: int
    k: int
    a: Optional[int]
    b: Optional[int]
    c: Optional[int]
    d: Optional[int]
    lda: int
    ldb: int
    ldc: int
    ldd: int
    alpha: float = 1.0
    beta: float = 0.0

    def to_c(self) -> capi.GGProblem:
        return capi.GGProblem(self.m, self.n, self.k, self.a or None, self.b or None, self.c or None, self.d or None,
                              self.lda, self.ldb, self.ldc, self.ldd, self.alpha, self.beta)

    @staticmethod
    def from_c(p: capi.GGProblem) -> "ProblemDesc":
        return ProblemDesc(p.m, p.n, p.k, p.a, p.b, p.c, p.d, p.lda, p.ldb, p.ldc, p.ldd, p.alpha, p.beta)


@dataclass
class KernelConfig:
    cta_m: int = 64
    cta_n: int = 64
    cta_k: int = 16
    threads: int = 256
    persistent_ctas: int = 0
    use_tensor_cores: bool = True
    input_type: int = 0   # InputType: FP16 A/B (the reference's type), BF16, E4M3 or E5M2
    output_type: int = 0  # OutputType: FP32 C/D (the reference's type), FP16 or BF16
    activation: int = 0   # Activation applied after the bias
    a_layout: int = 0     # Layout of every A (row-major: the reference's)
    b_layout: int = 0     # Layout of every B
    tile_classes: int = 0  # TileClasses: CTA-pair configs may cut problems into pair blocks + one-CTA rows

    def to_c(self) -> capi.GGConfig:
        return capi.GGConfig(self.cta_m, self.cta_n, self.cta_k, self.threads, self.persistent_ctas,
                             1 if self.use_tensor_cores else 0, int(self.input_type), int(self.output_type),
                             int(self.activation), int(self.a_layout), int(self.b_layout), int(self.tile_classes))


# The reference's three tile shapes (reference src/grouped_gemm.cu:67-81) and the sm_100a ones.
REFERENCE_CONFIGS = (KernelConfig(64, 64, 16), KernelConfig(128, 64, 32), KernelConfig(64, 128, 32))
NATIVE_CONFIGS = (KernelConfig(128, 128, 64), KernelConfig(128, 256, 64), KernelConfig(128, 64, 64),
                  KernelConfig(256, 128, 64), KernelConfig(256, 256, 64))
# Tiles computed by a cluster of two CTAs (tcgen05 cta_group::2).
PAIR_CONFIGS = (KernelConfig(256, 128, 64), KernelConfig(256, 256, 64))


@dataclass
class PreparedProblemSet:
    sorted_problems: List[ProblemDesc] = field(default_factory=list)
    sorted_to_original: List[int] = field(default_factory=list)
    tile_offsets: List[int] = field(default_factory=list)
    total_tiles: int = 0


@dataclass
class OccupancyInfo:
    sm_count: int = 0
    max_blocks_per_sm: int = 0
    active_blocks_per_sm: int = 0
    threads_per_block: int = 0
    max_threads_per_sm: int = 0
    warps_per_block: int = 0
    max_warps_per_sm: int = 0
    active_warps_per_sm: int = 0
    max_registers_per_sm: int = 0
    max_registers_per_block: int = 0
    estimated_registers_per_thread: int = 0
    estimated_registers_per_block: int = 0
    registers_per_thread: int = 0
    registers_per_block: int = 0
    register_limited_blocks_per_sm: int = 0
    static_shared_bytes: int = 0
    dynamic_shared_bytes: int = 0
    theoretical_occupancy: float = 0.0
    using_tensor_cores: bool = False


@dataclass
class ShardPiece:
    problem: int
    row0: int
    rows: int
    col0: int
    cols: int


def _problems_array(problems: Sequence[ProblemDesc]):
    arr = (capi.GGProblem * max(1, len(problems)))()
    for i, p in enumerate(problems):
        arr[i] = p.to_c()
    return arr


def _stream_ptr(stream) -> Optional[int]:
    """Accepts None (legacy default stream), an int handle or a torch.cuda.Stream."""
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream or None
    return getattr(stream, "cuda_stream", None) or None


def variant_is_pair(config: KernelConfig) -> bool:
    """True for the CTA-pair tile shapes (256 rows: a cluster of two CTAs per tile)."""
    return config.cta_m == 256


def sort_mode_name(sort_mode: int) -> str:
    return capi.load().gg_sort_mode_name(int(sort_mode)).decode()


def prepare_problem_set(problems: Sequence[ProblemDesc], config: KernelConfig, sort_mode: int) -> PreparedProblemSet:
    lib = capi.load()
    count = len(problems)
    src = _problems_array(problems)
    dst = (capi.GGProblem * max(1, count))()
    s2o = (ctypes.c_int * max(1, count))()
    offs = (ctypes.c_int * (count + 1))()
    total = ctypes.c_int(0)
    cfg = config.to_c()
    st = lib.gg_prepare(src, count, ctypes.byref(cfg), int(sort_mode), dst, s2o, offs, ctypes.byref(total))
    if st != 0:
        raise ValueError(f"gg_prepare failed with status {st}")
    return PreparedProblemSet([ProblemDesc.from_c(dst[i]) for i in range(count)], list(s2o)[:count], list(offs),
                              total.value)


def query_occupancy(config: KernelConfig, info: Optional[OccupancyInfo] = None):
    """Returns (status, OccupancyInfo)."""
    o = capi.GGOccupancy()
    cfg = config.to_c()
    st = capi.load().gg_query_occupancy(ctypes.byref(cfg), ctypes.byref(o))
    out = info if info is not None else OccupancyInfo()
    if st == 0:
        for name, _ in capi.GGOccupancy._fields_:
            val = getattr(o, name)
            setattr(out, name, bool(val) if name == "using_tensor_cores" else val)
    return st, out


class GroupedGemmExecutor:
    """Owns the device problem table of one prepared set (reference src/grouped_gemm.cu:1085-1277)."""

    def __init__(self):
        self._lib = capi.load()
        self._h = ctypes.c_void_p()
        st = self._lib.gg_executor_create(ctypes.byref(self._h))
        if st != 0:
            raise MemoryError(f"gg_executor_create failed with status {st}")

    def close(self):
        if self._h:
            self._lib.gg_executor_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def build(self, prepared: PreparedProblemSet, config: KernelConfig,
              bias: Optional[Sequence[Optional[int]]] = None) -> int:
        """bias (an extension; gg_executor_build_with_bias): one device pointer (or None) per sorted
        problem, each to n FP32 values added to every row of that problem's D."""
        if not self._h:
            return capi.CUDA_ERROR_INVALID_DEVICE_POINTER
        count = len(prepared.sorted_problems)
        arr = _problems_array(prepared.sorted_problems)
        offs = (ctypes.c_int * max(1, len(prepared.tile_offsets)))(*prepared.tile_offsets)
        cfg = config.to_c()
        if bias is None:
            return self._lib.gg_executor_build(self._h, arr, count, offs, len(prepared.tile_offsets),
                                               int(prepared.total_tiles), ctypes.byref(cfg))
        if len(bias) != count:
            return capi.CUDA_ERROR_INVALID_VALUE
        tbl = (ctypes.c_void_p * max(1, count))(*[ctypes.c_void_p(int(x) if x else None) for x in bias])
        return self._lib.gg_executor_build_with_bias(self._h, arr, count, offs, len(prepared.tile_offsets),
                                                     int(prepared.total_tiles), ctypes.byref(cfg), tbl)

    def run(self, stream=None) -> int:
        if not self._h:
            return capi.CUDA_ERROR_INVALID_DEVICE_POINTER
        return self._lib.gg_executor_run(self._h, _stream_ptr(stream))

    def status(self) -> int:
        """Synchronises and returns (then clears) the GG_STATUS_* bits raised by this executor."""
        out = ctypes.c_int(0)
        st = self._lib.gg_executor_status(self._h, ctypes.byref(out))
        if st != 0:
            raise RuntimeError(f"gg_executor_status failed with status {st}")
        return out.value

    def problem_count(self) -> int:
        return self._lib.gg_executor_problem_count(self._h)

    def total_tiles(self) -> int:
        return self._lib.gg_executor_total_tiles(self._h)

    def grid_ctas(self) -> int:
        return self._lib.gg_executor_grid_ctas(self._h)

    def launches(self) -> int:
        """Kernel launches of one run (1 without tile classes)."""
        return self._lib.gg_executor_launches(self._h)


def run_grouped_gemm_once(problems: Sequence[ProblemDesc], sort_mode: int, config: KernelConfig, stream=None) -> int:
    cfg = config.to_c()
    return capi.load().gg_run_grouped_gemm_once(_problems_array(problems), len(problems), int(sort_mode),
                                                ctypes.byref(cfg), _stream_ptr(stream))


def run_baseline_per_problem(problems: Sequence[ProblemDesc], config: KernelConfig, stream=None) -> int:
    cfg = config.to_c()
    return capi.load().gg_run_baseline_per_problem(_problems_array(problems), len(problems), ctypes.byref(cfg),
                                                   _stream_ptr(stream))


def count_non_empty_problems(problems: Sequence[ProblemDesc], config: KernelConfig) -> int:
    cfg = config.to_c()
    return capi.load().gg_count_non_empty_problems(_problems_array(problems), len(problems), ctypes.byref(cfg))


def partition(problems: Sequence[ProblemDesc], config: KernelConfig, world_size: int, rank: int):
    """Pieces of the problem set assigned to `rank` of `world_size` GPUs, and their weight."""
    lib = capi.load()
    arr = _problems_array(problems)
    cfg = config.to_c()
    n = ctypes.c_int(0)
    w = ctypes.c_double(0.0)
    st = lib.gg_partition(arr, len(problems), ctypes.byref(cfg), world_size, rank, None, 0, ctypes.byref(n), None)
    if st != 0:
        raise ValueError(f"gg_partition failed with status {st}")
    out = (capi.GGShardPiece * max(1, n.value))()
    st = lib.gg_partition(arr, len(problems), ctypes.byref(cfg), world_size, rank, out, n.value, ctypes.byref(n),
                          ctypes.byref(w))
    if st != 0:
        raise ValueError(f"gg_partition failed with status {st}")
    return [ShardPiece(o.problem, o.row0, o.rows, o.col0, o.cols) for o in out[:n.value]], w.value


class MoePlan:
    """Grouped GEMM whose per-problem row counts live on the device (gg_moe_plan_*).

    Problems share n and k; their rows are packed back to back in A (capacity_rows x k FP16),
    C and D (capacity_rows x n FP32, or the config's output type); expert e multiplies its rows by
    its own B[e] (k x n FP16) and, when bias_ptrs is given, adds its bias (n FP32 values, or None).
    `run(rows)` takes an int32 device tensor of `experts` row counts and enqueues the device-side
    preparation and the grouped kernel on the stream, with no host synchronisation.
    """

    def __init__(self, experts: int, n: int, k: int, capacity_rows: int, a: int, lda: int, b_ptrs: Sequence[int],
                 ldb: int, d: int, ldd: int, c: Optional[int] = None, ldc: Optional[int] = None,
                 alpha: float = 1.0, beta: float = 0.0, config: Optional[KernelConfig] = None,
                 bias_ptrs: Optional[Sequence[Optional[int]]] = None):
        self._lib = capi.load()
        self._h = None
        if len(b_ptrs) != experts or (bias_ptrs is not None and len(bias_ptrs) != experts):
            raise ValueError("one B pointer (and bias pointer) per expert")
        bs = (ctypes.c_void_p * max(1, experts))(*[ctypes.c_void_p(int(x) if x else None) for x in b_ptrs])
        bias_tbl = None
        if bias_ptrs is not None:
            bias_tbl = (ctypes.c_void_p * max(1, experts))(*[ctypes.c_void_p(int(x) if x else None)
                                                             for x in bias_ptrs])
        prob = capi.GGMoeProblem(a, ctypes.cast(bs, ctypes.POINTER(ctypes.c_void_p)), c, d, experts, n, k,
                                 capacity_rows, lda, ldb, ldc if ldc is not None else max(1, n), ldd, alpha, beta,
                                 ctypes.cast(bias_tbl, ctypes.POINTER(ctypes.c_void_p)) if bias_tbl else None)
        cfg = (config or KernelConfig(128, 256, 64)).to_c()
        h = ctypes.c_void_p()
        st = self._lib.gg_moe_plan_create(ctypes.byref(prob), ctypes.byref(cfg), ctypes.byref(h))
        if st != 0:
            raise ValueError(f"gg_moe_plan_create failed with status {st}")
        self._h = h
        self.experts = experts

    def run(self, rows, stream=None) -> int:
        """rows: int32 device tensor (or device pointer) of `experts` row counts."""
        ptr = rows if isinstance(rows, int) else rows.data_ptr()
        return self._lib.gg_moe_plan_run(self._h, ctypes.c_void_p(ptr), _stream_ptr(stream))

    def status(self):
        """Synchronises; returns (GG_STATUS_* bits, then cleared; tile count of the last run)."""
        st_bits, total = ctypes.c_int(0), ctypes.c_int(0)
        st = self._lib.gg_moe_plan_status(self._h, ctypes.byref(st_bits), ctypes.byref(total))
        if st != 0:
            raise RuntimeError(f"gg_moe_plan_status failed with status {st}")
        return st_bits.value, total.value

    def close(self):
        if self._h:
            self._lib.gg_moe_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DevicePlan:
    """Grouped GEMM whose problem descriptors and count live in device memory (gg_device_plan_*).

    `run(problems, count, sort_mode)` takes a device buffer holding an array of gg_problem records
    (see `pack_problems`) and a device int32 count, and enqueues the device-side preparation
    (validation, the sort mode's order, tile offsets, records, TMA descriptors) and the grouped
    kernel, with no host synchronisation. One-CTA tensor-core configs or the CUDA-core path,
    row-major A and B.
    """

    def __init__(self, config: KernelConfig, max_problems: int):
        self._lib = capi.load()
        self._h = None
        h = ctypes.c_void_p()
        cfg = config.to_c()
        st = self._lib.gg_device_plan_create(ctypes.byref(cfg), int(max_problems), ctypes.byref(h))
        if st != 0:
            raise ValueError(f"gg_device_plan_create failed with status {st}")
        self._h = h
        self.max_problems = int(max_problems)

    @staticmethod
    def pack_problems(problems: Sequence[ProblemDesc]) -> bytes:
        """The gg_problem records of `problems` as bytes (copy them to device memory for run)."""
        arr = _problems_array(problems)
        return ctypes.string_at(ctypes.addressof(arr), ctypes.sizeof(capi.GGProblem) * len(problems))

    def run(self, problems, count, sort_mode: int = 0, stream=None) -> int:
        """problems / count: device pointers (ints) or tensors (a uint8 tensor of packed records, an
        int32 tensor holding the count)."""
        pp = problems if isinstance(problems, int) else problems.data_ptr()
        cp = count if isinstance(count, int) else count.data_ptr()
        return self._lib.gg_device_plan_run(self._h, ctypes.c_void_p(pp), ctypes.c_void_p(cp), int(sort_mode),
                                            _stream_ptr(stream))

    def status(self):
        """Synchronises; returns (GG_STATUS_* bits, then cleared; tile count of the last run)."""
        bits, total = ctypes.c_int(0), ctypes.c_int(0)
        st = self._lib.gg_device_plan_status(self._h, ctypes.byref(bits), ctypes.byref(total))
        if st != 0:
            raise RuntimeError(f"gg_device_plan_status failed with status {st}")
        return bits.value, total.value

    def prepared(self, count: int):
        """Synchronises; (sorted_to_original, tile_offsets) of the last run's first `count` slots."""
        order = (ctypes.c_int * max(1, count))()
        offs = (ctypes.c_int * (count + 1))()
        st = self._lib.gg_device_plan_prepared(self._h, order, offs, int(count))
        if st != 0:
            raise RuntimeError(f"gg_device_plan_prepared failed with status {st}")
        return list(order)[:count], list(offs)

    def close(self):
        if self._h:
            self._lib.gg_device_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def selftest_wait_timeout(timeout_ns: int = 20_000_000):
    """(status, device bits) of the bounded-wait self-test (see gg_selftest_wait_timeout)."""
    out = ctypes.c_int(0)
    st = capi.load().gg_selftest_wait_timeout(int(timeout_ns), ctypes.byref(out))
    return st, out.value


def selftest_wait_timeout_word(word: int, timeout_ns: int = 20_000_000) -> int:
    """The bounded-wait self-test recording into the baseline's (capi.GG_STATUS_WORD_BASELINE) or
    the no-allocation entry point's (capi.GG_STATUS_WORD_NOALLOC) status word; returns the
    cudaError_t of the launch."""
    return capi.load().gg_selftest_wait_timeout_word(int(word), int(timeout_ns))


def baseline_status() -> int:
    """Synchronises; returns (then clears) the GG_STATUS_* bits raised by run_baseline_per_problem
    launches on the current device."""
    out = ctypes.c_int(0)
    st = capi.load().gg_baseline_status(ctypes.byref(out))
    if st != 0:
        raise RuntimeError(f"gg_baseline_status failed with status {st}")
    return out.value


def noalloc_status() -> int:
    """Synchronises; returns (then clears) the GG_STATUS_* bits of the last no-allocation call
    (gg_run_grouped_gemm_noalloc) on the current device."""
    out = ctypes.c_int(0)
    st = capi.load().gg_noalloc_status(ctypes.byref(out))
    if st != 0:
        raise RuntimeError(f"gg_noalloc_status failed with status {st}")
    return out.value


def problem_from_tensors(a, b, c, d, alpha: float = 1.0, beta: float = 0.0) -> ProblemDesc:
    """ProblemDesc over torch tensors: a (m, k) fp16, b (k, n) fp16, c (m, n) fp32 or None, d (m, n) fp32
    (bf16 a/b and fp16/bf16 c/d with the matching KernelConfig input_type / output_type).

    Rows may be padded (row stride >= columns) but columns must be contiguous.
    """
    m, k = a.shape
    k2, n = b.shape
    if k2 != k or tuple(d.shape) != (m, n):
        raise ValueError("shape mismatch")
    for t in (a, b, d) + ((c,) if c is not None else ()):
        if t.dim() == 2 and t.shape[1] > 1 and t.stride(1) != 1:
            raise ValueError("columns must be contiguous")
    return ProblemDesc(m, n, k, a.data_ptr(), b.data_ptr(), c.data_ptr() if c is not None else None, d.data_ptr(),
                       max(1, a.stride(0)), max(1, b.stride(0)), max(1, c.stride(0)) if c is not None else max(1, n),
                       max(1, d.stride(0)), float(alpha), float(beta))
