#!/usr/bin/env python3
"""Benchmark of the B200 grouped GEMM on the BASELINE workloads (default: mixed512, 1 GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload mixed512] [--impl reference]

One step = one executor run (tile-counter reset + one persistent kernel launch) over the rank's
problem set, inputs resident in HBM. Prints ONE JSON line on rank 0:

  value      aggregate TFLOP/s = 2*sum(MNK) of all ranks / max-over-ranks device time
  e2e        the same metric through the C-ABI with the inputs copied from pinned host memory
             and D copied back inside every timed step
  roofline   the kernel's algorithmic bytes (or FLOPs) per launch / its event-timed duration
             against the measured peak in MEASURED_PEAKS.json
  cpu_baseline  the reference's own host GEMM (compute_reference, built from its sources into
             oracle/_ref) on a bounded sample, one host thread, as the reference runs it
  ref_gpu    the reference's own CUDA kernels (built for sm_100a) on the same device buffers

Multi-GPU (torchrun, one process per GPU): weak scaling. The global problem set is N seeded
replicas of the workload (seeds 42..42+N-1); gg_partition cuts it into N tile-weighted shards
and each rank materialises and runs only its own. No collective touches the data path; NCCL is
used for the barrier and the max-over-ranks timing reduction only.

--impl reference times the reference's CPU implementation of the path (compute_reference) on
all host threads, on a bounded sample of the same workload per step (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

L2_BYTES = 126 << 20
METRIC = "aggregate TFLOP/s (2·ΣMNK/s) at 1/2/4/8 B200, % of dense FP16 peak"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}
DEFAULT_CTA = {"small16": (128, 128, 64), "mixed512": (128, 256, 64), "moe": (128, 256, 64),
               "tiny4096": (128, 64, 64), "skew": (128, 256, 64), "moe_reduced": (128, 256, 64)}
# sort mode per workload: by K for mixed512 (the fastest of the four there), by tiles elsewhere
# (the largest problems first, which shortens the persistent schedule's tail)
DEFAULT_SORT = {"small16": 2, "mixed512": 1, "moe": 2, "tiny4096": 2, "skew": 2, "moe_reduced": 2}
ROW_WORKLOADS = ("moe", "skew", "tiny4096", "small16")  # driver-timed beside the headline (N = 1)
# Tile classes (gg_config.tile_classes): the two large workloads with CTA-pair blocks + one-CTA rows
# (1), tiny4096 with its small problems on the CUDA-core kernel (2)
CLASS_ROWS = {"moe_pair_classes": ("moe", 1), "skew_pair_classes": ("skew", 1),
              "tiny4096_small_on_cuda_cores": ("tiny4096", 2), "small16_small_on_cuda_cores": ("small16", 2)}
STRONG_WORKLOADS = ("skew", "moe")  # one fixed global set split over the N ranks


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", default="mixed512",
                    choices=["small16", "mixed512", "moe", "tiny4096", "skew", "moe_reduced"],
                    help="moe_reduced (8 experts, 2048 tokens) exists for small profiling captures")
    ap.add_argument("--sort-mode", type=int, default=1, help="0 none, 1 by K, 2 by tiles, 3 by tiles then K")
    ap.add_argument("--cta", default=None, help="tile shape MxNxK (default per workload)")
    ap.add_argument("--no-extras", action="store_true", help="skip the sort-mode sweep and the reference GPU row")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="target CPU work of the cpu_baseline sample")
    ap.add_argument("--input-type", choices=["f16", "bf16", "e4m3", "e5m2"], default="f16",
                    help="A/B element type (bf16 and the 8-bit floats are extensions; the reference is FP16 "
                         "only); 8-bit runs pad the row pitches to 16 bytes")
    ap.add_argument("--output-type", choices=["f32", "f16", "bf16"], default="f32",
                    help="element type of C and D (f32: the reference's)")
    ap.add_argument("--activation", choices=["none", "relu", "gelu"], default="none",
                    help="activation fused into the epilogue")
    ap.add_argument("--bias", action="store_true", help="a per-column FP32 bias on every problem")
    ap.add_argument("--a-layout", choices=["row", "col"], default="row",
                    help="storage of every A (col: k x m, an extension; row pitches padded to 16 bytes)")
    ap.add_argument("--b-layout", choices=["row", "col"], default="row",
                    help="storage of every B (col: n x k, the [out][in] weight layout; pitches padded to 16 bytes)")
    ap.add_argument("--gather", action="store_true",
                    help="N>1: after the timed region, gather every rank's D to rank 0 over NCCL and fused into "
                         "the kernel, and time both (the default at N>1 for the reference's FP32 output)")
    ap.add_argument("--no-gather", action="store_true", help="N>1: skip the gather rows")
    ap.add_argument("--tile-classes", type=int, choices=[0, 1, 2], default=0,
                    help="gg_config.tile_classes of the headline executor: 0 one tile shape (the reference's), "
                         "1 CTA-pair blocks + one-CTA rows (pair --cta), 2 small problems on the CUDA cores")
    ap.add_argument("--cuda-cores", action="store_true",
                    help="headline executor on the CUDA-core kernel (the reference's use_tensor_cores = false)")
    ap.add_argument("--no-rows", action="store_true",
                    help="skip the per-workload rows (N=1) and the strong-scaling rows (every N)")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        d["source"] = "measured"
        return d
    return dict(FALLBACK_PEAKS)


def tail_work_share(prepared, cta_k):
    """The reference's tail-balance figure (reference bench/benchmark_grouped_gemm.cu:580-607): the
    work (tiles x ceil(K / cta_k)) of the last 10 % of the problems in launch order, over the total."""
    n = len(prepared.sorted_problems)
    if n == 0:
        return 0.0
    tail = max(1, n // 10)
    total = tail_w = 0.0
    for i, p in enumerate(prepared.sorted_problems):
        w = (prepared.tile_offsets[i + 1] - prepared.tile_offsets[i]) * (-(-max(p.k, 0) // cta_k))
        total += w
        if i >= n - tail:
            tail_w += w
    return tail_w / total if total > 0 else 0.0


def roofline_of(flops, alg_bytes, ms, peaks, in_type=0):
    """Roofline of one launch: HBM-bound below the ridge point, tensor-bound above it."""
    tensor_peak, tensor_src = peaks["bf16_tflops"], peaks["source"]
    if in_type >= 2:  # no FP8 measurement: twice the measured dense BF16 rate (the FP8:BF16 ratio of B200)
        tensor_peak, tensor_src = 2.0 * peaks["bf16_tflops"], "2 x " + peaks["source"] + " bf16"
    ridge = tensor_peak * 1e12 / (peaks["hbm_gbs"] * 1e9)
    if flops / max(alg_bytes, 1.0) < ridge:
        achieved = alg_bytes / (ms * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "traffic": None, "peak_source": peaks["source"],
                "algorithmic_bytes_per_launch": alg_bytes}
    achieved = flops / (ms * 1e-3) / 1e12
    return {"bound": "tensor", "achieved": achieved, "peak": tensor_peak, "unit": "TFLOP/s",
            "frac": achieved / tensor_peak, "traffic": None, "peak_source": tensor_src,
            "algorithmic_flops_per_launch": flops}


class StepTimer:
    """Device time of executor runs on one stream. Footprints below twice L2 flush L2 before every
    step (a write of a buffer larger than L2, then a read of a second one so no dirty line is left
    to be written back inside the step) and time each step alone; larger ones run back to back."""

    def __init__(self, dev, stream):
        self.dev, self.stream = dev, stream
        self._flush = self._flush_read = None

    def flush_buffers(self):
        import torch

        if self._flush is None:
            self._flush = torch.empty(4 * L2_BYTES, dtype=torch.uint8, device=self.dev)
            self._flush_read = torch.ones(2 * L2_BYTES // 4, dtype=torch.float32, device=self.dev)
        return self._flush, self._flush_read

    def ms(self, run, steps, flush):
        """Mean device ms per step of `steps` calls of run(stream); no host synchronisation inside."""
        import torch

        stream = self.stream
        if not flush:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(steps):
                run(stream)
            e1.record(stream)
            e1.synchronize()
            return e0.elapsed_time(e1) / steps
        fw, fr = self.flush_buffers()
        evs = []
        with torch.cuda.stream(stream):
            sink = torch.zeros((), device=self.dev)
            for _ in range(steps):
                fw.zero_()
                sink += fr.sum()
                a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a0.record(stream)
                run(stream)
                a1.record(stream)
                evs.append((a0, a1))
        evs[-1][1].synchronize()
        return sum(a.elapsed_time(b) for a, b in evs) / steps

    def median_of(self, run, steps, flush, repeats=5):
        """(median, min, max) over `repeats` repeats of `steps` steps."""
        xs = sorted(self.ms(run, steps, flush) for _ in range(repeats))
        return xs[len(xs) // 2], xs[0], xs[-1]


def link_peaks(dev, nbytes=256 << 20, reps=3):
    """Measured pinned-host <-> device copy rates (GB/s) of this process's GPU: each direction alone
    and both at once (full duplex, as the streamed end-to-end loop runs them), best of `reps`."""
    import torch

    h_in = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    h_out = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    d_in = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    d_out = torch.ones(nbytes, dtype=torch.uint8, device=dev)
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def timed(fn):
        best = None
        for _ in range(reps):
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s1)
            s2.wait_event(e0)
            fn()
            s1.wait_stream(s2)
            e1.record(s1)
            torch.cuda.synchronize()
            t = e0.elapsed_time(e1)
            best = t if best is None else min(best, t)
        return best

    def h2d():
        with torch.cuda.stream(s1):
            d_in.copy_(h_in, non_blocking=True)

    def d2h():
        with torch.cuda.stream(s2):
            h_out.copy_(d_out, non_blocking=True)

    t_in, t_out = timed(h2d), timed(d2h)
    t_both = timed(lambda: (h2d(), d2h()))
    return {"h2d_gbs": nbytes / (t_in * 1e-3) / 1e9, "d2h_gbs": nbytes / (t_out * 1e-3) / 1e9,
            "duplex_gbs_each_way": nbytes / (t_both * 1e-3) / 1e9, "bytes": nbytes,
            "how": "pinned host <-> HBM cudaMemcpyAsync of 256 MiB, CUDA events, best of 3; duplex = one copy "
                   "each way at once on two streams"}


# ---- clocks ------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons around the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu=timestamp,{self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None

    def mark(self, start: bool):
        if start:
            self.t0 = time.time()
        else:
            self.t1 = time.time()

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 10:
                    continue
                try:
                    ts = time.mktime(time.strptime(parts[0].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                    rows.append((ts, float(parts[2]), float(parts[3]), parts[5:]))
                except Exception:
                    continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        # timestamps have 1 s resolution: keep samples within the timed window +- 1 s
        inwin = [r for r in rows if self.t0 is not None and self.t0 - 1.0 <= r[0] <= (self.t1 or self.t0) + 1.0] or rows
        load = [r for r in inwin if r[1] > 0.5 * r[2]] or inwin
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in load:
            for nm, val in zip(names, r[3][1:]):
                if val.lower() in ("active", "yes"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(r[1] for r in load), "sm_max_mhz": max(r[2] for r in load),
                "samples": len(load), "reasons": sorted(reasons)}


# ---- workload sharding -------------------------------------------------------------------------
def shard(glob, world: int, rank: int, cfg):
    """This rank's gg_partition pieces of the global set `glob` (a Shapes), as a Shapes of
    independent problems, and every rank's partition weight."""
    import grouped_gemm_gpu_kernel_b200 as gg
    from grouped_gemm_gpu_kernel_b200 import workloads as W

    probs = [gg.ProblemDesc(m, n, k, 1, 1, None, 1, max(1, k), max(1, n), max(1, n), max(1, n)) for m, n, k in glob.dims]
    parts = [gg.partition(probs, cfg, world, r) for r in range(world)]
    pieces = parts[rank][0]
    dims = [(pc.rows, pc.cols, glob.dims[pc.problem][2]) for pc in pieces]
    out = W.Shapes(glob.name, dims, [glob.alpha[pc.problem] for pc in pieces], [glob.beta[pc.problem] for pc in pieces],
                   glob.has_c, glob.a_law, glob.a_std, glob.b_law, glob.b_std)
    return out, [w for _, w in parts]


def rank_shapes(workload: str, world: int, rank: int, cfg):
    """This rank's shard of the N-replica problem set (weak scaling), the global FLOPs and every
    rank's partition weight."""
    from grouped_gemm_gpu_kernel_b200 import workloads as W

    reps = [W.make_shapes(workload, seed=42 + r) for r in range(world)]
    if world == 1:
        return reps[0], reps[0].flops, [1.0]
    glob = W.Shapes(workload, [d for s in reps for d in s.dims], [a for s in reps for a in s.alpha],
                    [b for s in reps for b in s.beta], reps[0].has_c, reps[0].a_law, reps[0].a_std, reps[0].b_law,
                    reps[0].b_std)
    out, weights = shard(glob, world, rank, cfg)
    return out, float(sum(s.flops for s in reps)), weights


# ---- CPU baselines -----------------------------------------------------------------------------
def host_problem(m, n, k, alpha, beta, shapes, rng):
    def draw(count, law, std):
        if law == "normal":
            return rng.normal(0.0, std, size=max(count, 1)).astype(np.float16).view(np.uint16)
        return rng.uniform(-1.0, 1.0, size=max(count, 1)).astype(np.float16).view(np.uint16)

    return dict(m=m, n=n, k=k, lda=max(1, k), ldb=max(1, n), ldc=max(1, n), ldd=max(1, n), alpha=alpha, beta=beta,
                a=draw(m * k, shapes.a_law, shapes.a_std), b=draw(k * n, shapes.b_law, shapes.b_std),
                c=rng.uniform(-1, 1, size=max(m * n, 1)).astype(np.float32))


def cpu_sample(shapes, target_flops, seed=1234):
    """Problems of the workload, in order, until their FLOPs reach target_flops (at least one);
    a problem larger than the target is cut to a row band of the needed height."""
    rng = np.random.default_rng(seed)
    out, fl = [], 0.0
    for (m, n, k), al, be in zip(shapes.dims, shapes.alpha, shapes.beta):
        if m <= 0 or n <= 0:
            continue
        f = 2.0 * m * n * k
        if fl + f > target_flops and out:
            break
        if f > target_flops:
            m = max(1, int(target_flops / (2.0 * n * max(k, 1))))
            f = 2.0 * m * n * k
        out.append(host_problem(m, n, k, al, be, shapes, rng))
        fl += f
        if fl >= target_flops:
            break
    return out, fl


def time_cpu(problems, threads):
    """(seconds, kind): the reference's compute_reference when built, else the oracle's port."""
    import oracle as O

    if O.ref_available():
        _, secs = O.ref_host_gemm(problems, threads=threads)
        return secs, "reference"
    t0 = time.perf_counter()
    for p in problems:
        O.gemm_f32_refloop(p["m"], p["n"], p["k"], p["a"], p["lda"], p["b"], p["ldb"], p["c"], p["ldc"], p["alpha"],
                           p["beta"], p["ldd"])
    return time.perf_counter() - t0, "port"


def cpu_baseline(shapes, seconds_target):
    probe, pf = cpu_sample(shapes, 2e8)
    secs, kind = time_cpu(probe, 1)
    rate = pf / max(secs, 1e-6)
    sample, fl = cpu_sample(shapes, max(pf, rate * seconds_target))
    secs, kind = time_cpu(sample, 1)
    return {"value": fl / secs / 1e12, "unit": "TFLOP/s", "cores": 1, "kind": kind,
            "sample": f"first {len(sample)} problems of the workload in input order ({fl / 1e9:.2f} GFLOP, "
                      f"host-generated with the workload's value laws), FP32 host GEMM "
                      f"tests/test_correctness.cu:85-102, {secs:.1f} s single-thread"}


def run_reference_arm(args):
    from grouped_gemm_gpu_kernel_b200 import workloads as W

    shapes = W.make_shapes(args.workload)
    threads = os.cpu_count() or 1
    # size one step so that warmup + steps take about a minute in total
    probe, pf = cpu_sample(shapes, 2e8)
    secs, kind = time_cpu(probe, threads)
    rate = pf / max(secs, 1e-6)
    per_step = max(pf, rate * min(5.0, 60.0 / max(1, args.steps + args.warmup)))
    sample, fl = cpu_sample(shapes, per_step)
    for _ in range(args.warmup):
        time_cpu(sample, threads)
    times = []
    for _ in range(args.steps):
        s, kind = time_cpu(sample, threads)
        times.append(s)
    total = sum(times)
    value = fl * args.steps / total / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "sample_problems": len(sample), "sample_gflop": fl / 1e9,
                   "threads": threads},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": kind,
                         "sample": f"first {len(sample)} problems of {args.workload} ({fl / 1e9:.2f} GFLOP) per step, "
                                   f"reference compute_reference over problems on {threads} host threads"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- the B200 arm ------------------------------------------------------------------------------
def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            run_reference_arm(args)
        return

    import torch

    import grouped_gemm_gpu_kernel_b200 as gg
    from grouped_gemm_gpu_kernel_b200 import workloads as W

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    cta = tuple(int(x) for x in args.cta.split("x")) if args.cta else DEFAULT_CTA[args.workload]
    out_type = {"f32": 0, "f16": 1, "bf16": 2}[args.output_type]
    act = {"none": 0, "relu": 1, "gelu": 2}[args.activation]
    if args.gather and out_type != 0:
        raise SystemExit("--gather packs FP32 D only")
    in_type = {"f16": 0, "bf16": 1, "e4m3": 2, "e5m2": 3}[args.input_type]
    a_col, b_col = args.a_layout == "col", args.b_layout == "col"
    cfg = gg.KernelConfig(*cta, input_type=in_type, output_type=out_type, activation=act, a_layout=int(a_col),
                          b_layout=int(b_col), use_tensor_cores=not args.cuda_cores, tile_classes=args.tile_classes)
    plain = (out_type == 0 and act == 0 and not args.bias and args.input_type == "f16" and not (a_col or b_col)
             and args.tile_classes == 0 and not args.cuda_cores)
    shapes, global_flops, rank_weights = rank_shapes(args.workload, world, rank, cfg)

    def make_set():
        p = W.allocate(shapes, dev, seed=42 + rank, d_fill=0.0)
        if a_col or b_col:
            p.to_layout(a_col, b_col, 8)
        if in_type == 1:
            p.to_bf16()
        elif in_type >= 2:
            p.to_fp8(in_type)  # row pitches padded to 16 bytes (8-bit operands load by TMA only)
        if out_type:
            p.to_output(out_type)
        return p, (p.make_bias(without=0.0, aligned=True) if args.bias else None)

    def build(p_set, bias_ptrs, mode):
        prepared = gg.prepare_problem_set(p_set.problems(), cfg, mode)
        e = gg.GroupedGemmExecutor()
        sb = None if bias_ptrs is None else [bias_ptrs[o] for o in prepared.sorted_to_original]
        return e, e.build(prepared, cfg, bias=sb)

    ps, bias_ptrs = make_set()
    problems = ps.problems()
    tail_share = tail_work_share(gg.prepare_problem_set(problems, cfg, args.sort_mode), cta[2])
    prep_t0 = time.perf_counter()
    ex, st = build(ps, bias_ptrs, args.sort_mode)
    prep_ms = 1e3 * (time.perf_counter() - prep_t0)
    if st != 0:
        raise RuntimeError(f"executor build failed: {st}")
    stream = torch.cuda.Stream(dev)
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(max(args.warmup, 3)):
        assert ex.run(stream) == 0
    clocks = ClockSampler(local_rank)
    clocks.start()
    for _ in range(max(args.warmup, 3)):
        assert ex.run(stream) == 0
    alg_bytes = shapes.algorithmic_bytes(4 if out_type == 0 else 2, args.bias, 1 if in_type >= 2 else 2)
    # Inputs smaller than twice L2 would stay cache-resident from one step to the next: such
    # workloads flush L2 before every step and time each step alone (StepTimer); larger ones run
    # back to back.
    flush = alg_bytes < 2 * L2_BYTES
    timer = StepTimer(dev, stream)
    if flush:
        timer.flush_buffers()
    barrier()
    clocks.mark(True)
    local_ms = timer.ms(ex.run, args.steps, flush)
    barrier()
    clocks.mark(False)
    clock_info = clocks.stop()
    if ex.status() != 0:
        raise RuntimeError("a bounded wait timed out inside the kernel during the timed region")
    ms = max_over_ranks(local_ms)
    value = global_flops / (ms * 1e-3) / 1e12
    # A second protocol beside the K timed steps: the median of 5 repeats of max(50, K) steps each.
    rep_med, rep_min, rep_max = timer.median_of(ex.run, max(50, args.steps), flush)
    rep_med, rep_min, rep_max = max_over_ranks(rep_med), max_over_ranks(rep_min), max_over_ranks(rep_max)
    protocol = {"repeats": 5, "steps_per_repeat": max(50, args.steps), "median_ms": rep_med, "min_ms": rep_min,
                "max_ms": rep_max, "median_value": global_flops / (rep_med * 1e-3) / 1e12}

    peaks = load_peaks()
    local_flops = shapes.flops
    roof = roofline_of(local_flops, alg_bytes, local_ms, peaks, in_type)
    traffic_path = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(traffic_path) and world == 1:
        with open(traffic_path) as f:
            tr = json.load(f).get(f"{args.workload}/{cta[0]}x{cta[1]}x{cta[2]}")
        if tr:
            roof["traffic"] = tr["bytes_per_launch"]
            roof["traffic_source"] = tr["source"]

    # ---- e2e through the C-ABI with host buffers (pinned), copies inside the timed step ----
    e2e = None
    if args.e2e_steps > 0:
        h_a = torch.empty(ps.a.shape, dtype=ps.a.dtype, pin_memory=True)
        h_b = torch.empty(ps.b.shape, dtype=ps.b.dtype, pin_memory=True)
        h_a.copy_(ps.a)
        h_b.copy_(ps.b)
        reads_c = ps.c is not None and any(b != 0.0 for b in shapes.beta)
        h_c = None
        if reads_c:
            h_c = torch.empty(ps.c.shape, dtype=ps.c.dtype, pin_memory=True)
            h_c.copy_(ps.c)
        h_d = torch.empty(ps.d.shape, dtype=ps.d.dtype, pin_memory=True)
        h2d = (h_a.numel() * h_a.element_size() + h_b.numel() * h_b.element_size() +
               (h_c.numel() * h_c.element_size() if h_c is not None else 0))
        d2h = h_d.numel() * h_d.element_size()

        def e2e_step():
            with torch.cuda.stream(stream):
                ps.a.copy_(h_a, non_blocking=True)
                ps.b.copy_(h_b, non_blocking=True)
                if h_c is not None:
                    ps.c.copy_(h_c, non_blocking=True)
                assert ex.run(stream) == 0
                h_d.copy_(ps.d, non_blocking=True)

        e2e_step()
        barrier()
        e2 = torch.cuda.Event(enable_timing=True)
        e3 = torch.cuda.Event(enable_timing=True)
        e2.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        e3.record(stream)
        barrier()
        serial_ms = max_over_ranks(e2.elapsed_time(e3) / args.e2e_steps)

        # Streamed: two device buffer sets, copies in on one stream, the grouped GEMM on another,
        # copies out on a third, so step i+1's inputs cross PCIe while step i computes and step
        # i-1's D comes back. Every step still moves its own inputs in and its D out.
        ps_b, bias_b = make_set()  # A/B/C overwritten by the copies in
        ex_b, st_b = build(ps_b, bias_b, args.sort_mode)
        assert st_b == 0
        sets = [(ps, ex), (ps_b, ex_b)]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        in_done = [torch.cuda.Event() for _ in range(2)]
        comp_done = [torch.cuda.Event() for _ in range(2)]
        out_done = [torch.cuda.Event() for _ in range(2)]

        def streamed_step(i):
            p_i, ex_i = sets[i % 2]
            b = i % 2
            s_in.wait_event(out_done[b])  # the set's previous D has left (so its compute is done)
            with torch.cuda.stream(s_in):
                p_i.a.copy_(h_a, non_blocking=True)
                p_i.b.copy_(h_b, non_blocking=True)
                if h_c is not None:
                    p_i.c.copy_(h_c, non_blocking=True)
                in_done[b].record(s_in)
            stream.wait_event(in_done[b])
            assert ex_i.run(stream) == 0
            comp_done[b].record(stream)
            s_out.wait_event(comp_done[b])
            with torch.cuda.stream(s_out):
                h_d.copy_(p_i.d, non_blocking=True)
                out_done[b].record(s_out)

        for b in range(2):
            out_done[b].record(s_out)
        for i in range(2):
            streamed_step(i)
        barrier()
        e4 = torch.cuda.Event(enable_timing=True)
        e5 = torch.cuda.Event(enable_timing=True)
        e4.record(stream)
        s_in.wait_event(e4)
        s_out.wait_event(e4)
        for i in range(args.e2e_steps):
            streamed_step(i)
        stream.wait_event(out_done[(args.e2e_steps - 1) % 2])
        e5.record(stream)
        barrier()
        e2e_ms = max_over_ranks(e4.elapsed_time(e5) / args.e2e_steps)
        e2e = {"value": global_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
               "path": "pinned host A/B(/C) -> cudaMemcpyAsync -> gg_executor_run -> D back to pinned host, "
                       "streamed: copies in, grouped GEMM and copies out of consecutive steps overlap on three "
                       "streams with two device buffer sets",
               "serial_ms_per_step": serial_ms,
               "serial_value": global_flops / (serial_ms * 1e-3) / 1e12}
        ex_b.close()
        del ps_b

    extras = {}
    gather = world > 1 and not args.no_gather and (args.gather or plain)
    if gather:
        extras["gather"] = gather_row(args, cfg, ps, world, rank, dev, max_over_ranks, barrier)
    if not args.no_extras and world == 1:
        sweep = {}
        for mode in range(4):
            ex2, st2 = build(ps, bias_ptrs, mode)
            assert st2 == 0
            for _ in range(10):
                ex2.run(stream)
            torch.cuda.synchronize()
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record(stream)
            for _ in range(50):
                ex2.run(stream)
            a1.record(stream)
            torch.cuda.synchronize()
            t = a0.elapsed_time(a1) / 50
            sweep[gg.sort_mode_name(mode)] = {"ms": t, "tflops": local_flops / (t * 1e-3) / 1e12,
                                             "grid": ex2.grid_ctas(), "tiles": ex2.total_tiles()}
            ex2.close()
        extras["sort_modes"] = sweep
        extras["cuda_graph"] = graph_row(ex, stream, local_flops)
        if args.workload == "moe":
            extras["device_prep"] = moe_plan_row(ps, shapes, cfg, stream, local_flops, ms, bias_ptrs)
        elif plain and not gg.variant_is_pair(cfg):
            extras["device_prepared"] = device_plan_row(problems, cfg, args.sort_mode, stream, local_flops, ms)
        if plain:  # the reference's kernels: FP16 in, FP32 out, no fused bias or activation
            extras["ref_gpu"] = reference_gpu_row(problems, stream, local_flops)

    if not args.no_rows and plain:
        torch.cuda.synchronize()
        peaks_rows = load_peaks()
        if world == 1:
            extras["workloads"] = {name: workload_row(name, dev, stream, args.steps, peaks_rows)
                                   for name in ROW_WORKLOADS if name != args.workload}
            for row, (name, classes) in CLASS_ROWS.items():
                extras["workloads"][row] = workload_row(name, dev, stream, args.steps, peaks_rows, classes=classes)
        extras["strong"] = {name: strong_row(name, world, rank, dev, stream, args.steps, max_over_ranks, barrier)
                            for name in STRONG_WORKLOADS}

    if e2e is not None:
        # The link's own roofline, measured last (large pinned copies): every rank measures its
        # pinned copy rates at the same time (the ranks share the host), and the streamed loop is
        # bound by the slower direction at the duplex rate.
        barrier()
        lk = link_peaks(dev)
        lk["duplex_gbs_each_way"] = -max_over_ranks(-lk["duplex_gbs_each_way"])
        bound_ms = 1e3 * max(e2e["h2d_bytes_per_step"], e2e["d2h_bytes_per_step"]) / (lk["duplex_gbs_each_way"] * 1e9)
        lk.update({"bound_ms_per_step": bound_ms, "frac": bound_ms / e2e["ms_per_step"],
                   "bound": "max(h2d, d2h bytes per step) / the slowest rank's duplex copy rate"})
        e2e["link"] = lk

    cpu = None
    if rank == 0 and world == 1:
        cpu = cpu_baseline(shapes, args.cpu_seconds)

    if rank == 0:
        n_tiles = ex.total_tiles()
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": args.input_type, "data": "synthetic",
            "config": {"workload": args.workload, "problems_per_gpu": len(shapes.dims), "cta": "x".join(map(str, cta)),
                       "sort_mode": gg.sort_mode_name(args.sort_mode), "tiles": n_tiles, "grid_ctas": ex.grid_ctas(),
                       "global_gflop": global_flops / 1e9,
                       "l2": (f"inputs larger than L2 ({alg_bytes / 1e9:.2f} GB algorithmic footprint per GPU "
                              "> 2 x 126 MB), steps back to back, no flush") if not flush else
                             (f"footprint {alg_bytes / 1e6:.1f} MB < 2 x L2: L2 flushed ({4 * L2_BYTES >> 20} MB "
                              f"write, then a {2 * L2_BYTES >> 20} MB read so no dirty line is left) before every "
                              "step, each step timed alone"),
                       "accumulate": "f32", "output_type": args.output_type, "activation": args.activation,
                       "bias": bool(args.bias), "a_layout": args.a_layout, "b_layout": args.b_layout,
                       "tile_classes": args.tile_classes,
                       "path": "cuda_cores" if args.cuda_cores else "tensor_cores",
                       "prep_build_ms": prep_ms, "parallelism": f"dp{world} (tile-balanced shards)",
                       "tail_work_share": tail_share,
                       "rank_weight_max_over_mean": max(rank_weights) / (sum(rank_weights) / len(rank_weights))},
            "timing_protocol": protocol,
            "pct_dense_fp16_peak": 100.0 * value / (world * peaks["bf16_tflops"]),
            "peak_source": peaks["source"],
            "roofline": roof,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "clocks": clock_info,
            "gpu_launches": args.steps * ex.launches(),
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    ex.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def gather_row(args, cfg, ps, world, rank, dev, max_over_ranks, barrier):
    """Optional NCCL gather of every rank's D rectangles into rank 0's full D (not in `value`)."""
    import torch

    import grouped_gemm_gpu_kernel_b200 as gg
    from grouped_gemm_gpu_kernel_b200 import workloads as W
    from grouped_gemm_gpu_kernel_b200.gather import gather_pieces, piece_elems

    reps = [W.make_shapes(args.workload, seed=42 + r) for r in range(world)]
    dims = [d for s in reps for d in s.dims]
    probs = [gg.ProblemDesc(m, n, k, 1, 1, None, 1, max(1, k), max(1, n), max(1, n), max(1, n)) for m, n, k in dims]
    by_rank = [gg.partition(probs, cfg, world, r)[0] for r in range(world)]
    local = []
    for i, pc in enumerate(by_rank[rank]):
        d = ps.views(i)[3]
        local.append(d if d is not None else torch.empty((pc.rows, pc.cols), device=dev))
    root_d = None
    if rank == 0:
        sizes = [max(m, 0) * max(n, 0) for m, n, k in dims]
        slab = torch.empty(sum(sizes), dtype=torch.float32, device=dev)
        root_d, off = {}, 0
        for i, ((m, n, k), sz) in enumerate(zip(dims, sizes)):
            root_d[i] = slab[off:off + sz].view(max(m, 0), max(n, 0))
            off += sz
    gather_pieces(by_rank, local, root_d)  # warm-up: NCCL P2P connections
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    got = gather_pieces(by_rank, local, root_d)
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1))
    into_root = sum(piece_elems(by_rank[r]) for r in range(1, world)) * 4
    ok = True
    if rank == 0:
        pc0 = by_rank[0][0] if by_rank[0] else None
        if pc0 is not None and pc0.rows and pc0.cols:
            ok = bool(torch.equal(root_d[pc0.problem][pc0.row0:pc0.row0 + pc0.rows, pc0.col0:pc0.col0 + pc0.cols],
                                  local[0]))
    barrier()
    row = {"ms": ms, "bytes_into_root": into_root, "gbps_into_root": into_root / (ms * 1e-3) / 1e9,
           "received_on_root": got if rank == 0 else None, "root_piece_check": ok,
           "how": "after the timed region: one packed FP32 buffer per rank, NCCL send/recv to rank 0, "
                  "unpacked into the full D of every global problem"}
    row["fused"] = fused_gather_row(cfg, ps, by_rank, dims, world, rank, dev, max_over_ranks, barrier,
                                    slab if rank == 0 else None)
    return row


def fused_gather_row(cfg, ps, by_rank, dims, world, rank, dev, max_over_ranks, barrier, gathered, runs=5):
    """The same gather fused into the kernel: the root exports a D buffer (CUDA IPC), every other
    rank maps it and runs its pieces with D pointers into it, so the epilogue stores each tile into
    the root's memory over NVLink (plain stores) while later tiles compute. Timed per run as the max
    over ranks; the root then checks the buffer against the NCCL-gathered D bit for bit."""
    import dataclasses

    import torch
    import torch.distributed as dist

    import grouped_gemm_gpu_kernel_b200 as gg
    from grouped_gemm_gpu_kernel_b200.gather import close_buffer, export_buffer, fused_targets, open_buffer

    total = sum(max(m, 0) * max(n, 0) for m, n, k in dims)
    fbuf = torch.full((max(total, 1),), float("nan"), device=dev) if rank == 0 else None
    obj = [export_buffer(fbuf) if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    base = fbuf.data_ptr() if rank == 0 else open_buffer(obj[0])
    mine = by_rank[rank]
    probs = [dataclasses.replace(p, d=t[0], ldd=t[1]) for p, t in zip(ps.problems(), fused_targets(mine, dims, base))]
    ex = gg.GroupedGemmExecutor()
    st = ex.build(gg.prepare_problem_set(probs, cfg, gg.SortMode.kByK), cfg)
    if st != 0:
        raise RuntimeError(f"fused-gather executor build failed: {st}")
    stream = torch.cuda.Stream(dev)
    assert ex.run(stream) == 0
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(runs):
        ex.run(stream)
    e1.record(stream)
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / runs)
    status = ex.status()
    ex.close()
    barrier()  # every rank's stores into the root's buffer have completed
    same = bool(torch.equal(fbuf[:total], gathered[:total])) if rank == 0 else None
    if rank != 0:
        close_buffer(base)
    barrier()  # the root frees its buffer only after every mapping is closed
    into_root = 4 * sum(pc.rows * pc.cols for r in range(1, world) for pc in by_rank[r])
    return {"ms": ms, "status": status, "bitwise_equal_to_nccl_gather": same,
            "gbps_into_root": into_root / (ms * 1e-3) / 1e9,
            "how": "one grouped-kernel launch per rank whose D pointers lie in rank 0's buffer (CUDA IPC "
                   "mapping, peer access): compute and the NVLink transfer of D in the same kernel"}


def moe_plan_row(ps, shapes, cfg, stream, flops, executor_ms, bias_ptrs=None, runs=20):
    """The same MoE problems through gg_moe_plan: row counts read from device memory, device-side
    preparation kernel + grouped kernel per run (the workload's slabs are already row-packed)."""
    import torch

    import grouped_gemm_gpu_kernel_b200 as gg

    rows = [m for m, n, k in shapes.dims]
    n, k = shapes.dims[0][1], shapes.dims[0][2]
    packed = all(ps.a_off[i + 1] == ps.a_off[i] + rows[i] * k and ps.d_off[i + 1] == ps.d_off[i] + rows[i] * n
                 for i in range(len(rows) - 1))
    if not packed or any(d[1] != n or d[2] != k for d in shapes.dims):
        return {"unavailable": "problems do not share n, k or are not row-packed"}
    if ps.a_col:
        return {"unavailable": "the plan takes a row-major A"}
    ei = ps.a.element_size()
    lda = ps.lda[0] if ps.lda else k
    ldb = ps.ldb[0] if ps.ldb else n
    b_ptrs = [ps.b.data_ptr() + ei * off for off in ps.b_off]
    plan = gg.MoePlan(len(rows), n, k, sum(rows), ps.a.data_ptr() + ei * ps.a_off[0], lda, b_ptrs, ldb,
                      ps.d.data_ptr() + ps.d.element_size() * ps.d_off[0], n, None, n, 1.0, 0.0, cfg,
                      bias_ptrs=bias_ptrs)
    rows_t = torch.tensor(rows, dtype=torch.int32, device=ps.a.device)
    ref = ps.d.clone()
    torch.cuda.synchronize()
    for _ in range(3):
        plan.run(rows_t, stream)
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(runs):
        plan.run(rows_t, stream)
    a1.record(stream)
    torch.cuda.synchronize()
    t = a0.elapsed_time(a1) / runs
    bits, total = plan.status()
    same = bool(torch.equal(ps.d, ref))
    plan.close()
    return {"ms": t, "tflops": flops / (t * 1e-3) / 1e12, "executor_ms": executor_ms, "status": bits,
            "tiles": total, "bitwise_equal_to_executor": same,
            "how": "row counts in device memory; one-block prefix-scan kernel writes problem records and "
                   "tile offsets, the persistent kernel reads the tile count from the device"}


def workload_row(name, dev, stream, steps, peaks, repeats=5, classes=0):
    """One BASELINE workload on this GPU with its default tile and sort mode, or with tile classes
    (1: CTA-pair 256x256 blocks + one-CTA rows; 2: the default tile, small problems on the CUDA
    cores): the median of `repeats` repeats of max(steps, 10) executor runs, its roofline, its
    tail-work share."""
    import torch

    import grouped_gemm_gpu_kernel_b200 as gg
    from grouped_gemm_gpu_kernel_b200 import workloads as W

    shapes = W.make_shapes(name)
    cta, mode = ((256, 256, 64) if classes == 1 else DEFAULT_CTA[name]), DEFAULT_SORT[name]
    cfg = gg.KernelConfig(*cta, tile_classes=classes)
    ps = W.allocate(shapes, dev, seed=42, d_fill=0.0)
    prep = gg.prepare_problem_set(ps.problems(), cfg, mode)
    ex = gg.GroupedGemmExecutor()
    assert ex.build(prep, cfg) == 0
    alg = shapes.algorithmic_bytes()
    flush = alg < 2 * L2_BYTES
    timer = StepTimer(dev, stream)
    for _ in range(3):
        assert ex.run(stream) == 0
    med, lo, hi = timer.median_of(ex.run, max(steps, 10), flush, repeats)
    status = ex.status()
    roof = roofline_of(shapes.flops, alg, med, peaks)
    traffic_path = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(traffic_path) and not classes:
        with open(traffic_path) as f:
            tr = json.load(f).get(f"{name}/{cta[0]}x{cta[1]}x{cta[2]}")
        if tr:
            roof["traffic"], roof["traffic_source"] = tr["bytes_per_launch"], tr["source"]
    row = {"ms": med, "min_ms": lo, "max_ms": hi, "tflops": shapes.flops / (med * 1e-3) / 1e12,
           "cta": "x".join(map(str, cta)) + {0: "", 1: " pair blocks + one-CTA rows",
                                             2: " small problems on CUDA cores"}[classes],
           "sort_mode": gg.sort_mode_name(mode),
           "problems": len(shapes.dims),
           "tiles": ex.total_tiles(), "grid_ctas": ex.grid_ctas(), "gflop": shapes.flops / 1e9,
           "algorithmic_gb": alg / 1e9, "roofline": roof,
           "tail_work_share": tail_work_share(prep, cta[2]), "status": status,
           "timing": f"median of {repeats} repeats of {max(steps, 10)} steps; "
                     + ("L2 flushed before every step, each step timed alone" if flush else
                        "footprint larger than 2 x L2, steps back to back")}
    ex.close()
    del ps, prep
    torch.cuda.empty_cache()
    return row


def strong_row(name, world, rank, dev, stream, steps, max_over_ranks, barrier):
    """Strong scaling: ONE fixed global set (seed 42) split by gg_partition over the N ranks; each
    rank materialises and runs only its pieces. Time = max over ranks of the per-step device time;
    value = the global set's FLOPs / that time."""
    import torch

    import grouped_gemm_gpu_kernel_b200 as gg
    from grouped_gemm_gpu_kernel_b200 import workloads as W

    glob = W.make_shapes(name)
    cta, mode = DEFAULT_CTA[name], DEFAULT_SORT[name]
    cfg = gg.KernelConfig(*cta)
    mine, weights = shard(glob, world, rank, cfg) if world > 1 else (glob, [1.0])
    ps = W.allocate(mine, dev, seed=42 + rank, d_fill=0.0)
    ex = gg.GroupedGemmExecutor()
    assert ex.build(gg.prepare_problem_set(ps.problems(), cfg, mode), cfg) == 0
    timer = StepTimer(dev, stream)
    flush = mine.algorithmic_bytes() < 2 * L2_BYTES
    for _ in range(3):
        assert ex.run(stream) == 0
    barrier()
    local = timer.ms(ex.run, max(steps, 10), flush)
    barrier()
    ms = max_over_ranks(local)
    fastest = -max_over_ranks(-local)
    status = int(max_over_ranks(float(ex.status())))
    tiles = int(max_over_ranks(float(ex.total_tiles())))
    ex.close()
    del ps
    torch.cuda.empty_cache()
    return {"ms": ms, "tflops": glob.flops / (ms * 1e-3) / 1e12, "n_gpus": world, "fastest_rank_ms": fastest,
            "max_rank_tiles": tiles, "rank_weight_max_over_mean": max(weights) / (sum(weights) / len(weights)),
            "cta": "x".join(map(str, cta)), "sort_mode": gg.sort_mode_name(mode), "gflop": glob.flops / 1e9,
            "status": status,
            "how": f"the one {name} set (seed 42) cut by gg_partition into {world} tile-weighted shards, one per "
                   f"rank; {max(steps, 10)} steps timed on each rank, max over ranks"}


def device_plan_row(problems, cfg, mode, stream, flops, executor_ms, runs=20):
    """The same problem set prepared on the device (gg_device_plan): descriptors and count copied to
    device memory once; each run = the one-block preparation kernel (sort, tile scan, records) +
    the grouped kernel, with no host work. No TMA descriptors on this path (zero-fill loads)."""
    import torch

    import grouped_gemm_gpu_kernel_b200 as gg

    plan = gg.DevicePlan(cfg, len(problems))
    raw = torch.frombuffer(bytearray(gg.DevicePlan.pack_problems(problems)), dtype=torch.uint8).to(stream.device)
    count = torch.tensor([len(problems)], dtype=torch.int32, device=stream.device)
    for _ in range(3):
        assert plan.run(raw, count, mode, stream) == 0
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(runs):
        plan.run(raw, count, mode, stream)
    a1.record(stream)
    torch.cuda.synchronize()
    t = a0.elapsed_time(a1) / runs
    bits, total = plan.status()
    plan.close()
    return {"ms": t, "tflops": flops / (t * 1e-3) / 1e12, "executor_ms": executor_ms, "status": bits, "tiles": total,
            "how": "problem descriptors and count in device memory; one-block preparation kernel (validation, "
                   "sort, tile scan, records) + the grouped kernel per run; 16-byte cp.async stage fills "
                   "(no TMA descriptors)"}


def graph_row(ex, stream, flops, runs=20, replays=10):
    """The same executor runs captured in one CUDA graph (counter reset + launch per run)."""
    import torch

    try:
        g = torch.cuda.CUDAGraph()
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=stream):
            for _ in range(runs):
                ex.run(torch.cuda.current_stream())
        g.replay()
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(replays):
                g.replay()
        a1.record(stream)
        torch.cuda.synchronize()
        t = a0.elapsed_time(a1) / (runs * replays)
        st = ex.status()
        del g
        return {"ms": t, "tflops": flops / (t * 1e-3) / 1e12, "runs_per_graph": runs, "status": st}
    except Exception as e:  # capture is optional evidence; the timed line above does not use it
        return {"unavailable": f"{type(e).__name__}: {e}"[:200]}


def reference_gpu_row(problems, stream, flops):
    """The reference's own kernels (sm_100a build of its sources) on the same device buffers."""
    import ctypes

    import oracle as O

    if not O.ref_available():
        return {"unavailable": "oracle/_ref/libgg_ref.so not built"}
    lib = O.load_ref()
    arr = (O.RefProblem * max(1, len(problems)))()
    for i, p in enumerate(problems):
        arr[i] = O.RefProblem(p.m, p.n, p.k, p.a, p.b, p.c, p.d, p.lda, p.ldb, p.ldc, p.ldd, p.alpha, p.beta)
    rows = {}
    best = None
    for cm, cn, ck in ((64, 64, 16), (128, 64, 32), (64, 128, 32)):
        for mode in (0, 2):
            ms, tiles, grid = ctypes.c_float(0), ctypes.c_int(0), ctypes.c_int(0)
            st = lib.ref_time_grouped(arr, len(problems), mode, cm, cn, ck, 1, 3, 10, ctypes.c_void_p(stream.cuda_stream),
                                      ctypes.byref(ms), ctypes.byref(tiles), ctypes.byref(grid))
            key = f"{cm}x{cn}x{ck}/{'none' if mode == 0 else 'sort_by_tiles'}"
            if st != 0:
                rows[key] = {"error": st}
                continue
            tf = flops / (ms.value * 1e-3) / 1e12
            rows[key] = {"ms": ms.value, "tflops": tf}
            if best is None or tf > best[1]:
                best = (key, tf)
    return {"best": best[0] if best else None, "best_tflops": best[1] if best else None, "runs": rows}


if __name__ == "__main__":
    main()
