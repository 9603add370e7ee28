"""Regenerate the committed golden fixtures from the reference's own code.

Run in a container where the reference tree exists and ``make -C oracle ref`` has built
``oracle/_ref/libgg_ref.so`` (the reference's sources compiled unmodified plus ``ref_shim.cu``):

    python tests/golden/make_golden.py

Writes, next to this script:

* ``ref_test_shapes.npz`` -- the reference test's eight shapes (tests/test_correctness.cu:313-322)
  with its inputs (std::mt19937(20260328), U[-1,1], tests/test_correctness.cu:114-150) and the
  output of the reference's own host GEMM compute_reference (tests/test_correctness.cu:85-102).
* ``prepare_golden.json`` -- prepare_problem_set / sort_mode_name / count_non_empty_problems
  results of the reference (src/grouped_gemm.cu:952-1022,1319-1329) on fixed problem sets.
"""
from __future__ import annotations

import ctypes
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

import oracle  # noqa: E402

REF_TEST_SHAPES = [(64, 64, 64), (128, 64, 96), (45, 81, 37), (17, 23, 9), (192, 32, 64), (16, 256, 48),
                   (0, 64, 16), (64, 0, 16)]
REF_TEST_SEED = 20260328
CONFIGS = [(64, 64, 16), (128, 64, 32), (64, 128, 32), (128, 128, 64), (128, 256, 64), (128, 64, 64)]


def safe_elems(rows: int, cols: int) -> int:
    return 1 if rows <= 0 or cols <= 0 else rows * cols


def packed_sizes(shapes):
    sa = [safe_elems(m, max(1, k)) for m, n, k in shapes]
    sb = [safe_elems(k, max(1, n)) for m, n, k in shapes]
    sc = [safe_elems(m, max(1, n)) for m, n, k in shapes]
    return sa, sb, sc


def make_test_inputs(lib, shapes, seed):
    sa, sb, sc = packed_sizes(shapes)
    a = np.zeros(sum(sa), np.uint16)
    b = np.zeros(sum(sb), np.uint16)
    c = np.zeros(sum(sc), np.float32)
    ref = np.zeros(sum(sc), np.float32)
    alpha = np.zeros(len(shapes), np.float32)
    beta = np.zeros(len(shapes), np.float32)
    flat = np.asarray(shapes, np.int32).reshape(-1)
    P = ctypes.POINTER
    rc = lib.ref_test_inputs_host(flat.ctypes.data_as(P(ctypes.c_int)), len(shapes), seed,
                                  a.ctypes.data_as(P(ctypes.c_uint16)), b.ctypes.data_as(P(ctypes.c_uint16)),
                                  c.ctypes.data_as(P(ctypes.c_float)), alpha.ctypes.data_as(P(ctypes.c_float)),
                                  beta.ctypes.data_as(P(ctypes.c_float)), ref.ctypes.data_as(P(ctypes.c_float)))
    assert rc == 0
    return dict(shapes=np.asarray(shapes, np.int32), a=a, b=b, c=c, alpha=alpha, beta=beta, ref=ref,
                seed=np.int64(seed))


def problem_sets():
    rng = np.random.default_rng(7)
    sets = {
        "ref_test_shapes": REF_TEST_SHAPES,
        "host_kat": [(64, 64, 64), (128, 64, 96), (45, 81, 37), (17, 23, 9), (0, 64, 16), (192, 32, 64)],
        "empty": [],
        "all_empty_problems": [(0, 5, 5), (5, 0, 5), (0, 0, 0)],
        "k_zero": [(64, 64, 0), (1, 1, 0), (130, 70, 0)],
    }
    # ties on K, on area and on tile count, so stability is exercised
    for t in range(6):
        P = int(rng.integers(5, 40))
        dims = []
        for _ in range(P):
            m = int(rng.choice([0, 1, 17, 64, 65, 128, 129, 200, 256]))
            n = int(rng.choice([0, 1, 31, 64, 100, 128, 255, 256, 300]))
            k = int(rng.choice([0, 8, 16, 64, 96]))
            dims.append((m, n, k))
        sets[f"ties_{t}"] = dims
    # the small BASELINE configuration's shape law (seed 42, U{16..256})
    r42 = np.random.default_rng(42)
    sets["small16_like"] = [tuple(int(x) for x in r42.integers(16, 257, size=3)) for _ in range(16)]
    return sets


def main():
    lib = oracle.load_ref()
    fx = make_test_inputs(lib, REF_TEST_SHAPES, REF_TEST_SEED)
    np.savez_compressed(os.path.join(HERE, "ref_test_shapes.npz"), **fx)

    out = {"sort_mode_name": {str(m): oracle.ref_sort_mode_name(m) for m in range(-1, 6)}, "sets": {}}
    for name, dims in problem_sets().items():
        entry = {"dims": [list(d) for d in dims], "results": []}
        for cta_m, cta_n, cta_k in CONFIGS:
            for mode in (0, 1, 2, 3, 4):
                perm, offs, total = oracle.ref_prepare(dims, cta_m, cta_n, cta_k, mode)
                entry["results"].append({"cta": [cta_m, cta_n, cta_k], "mode": mode,
                                         "sorted_to_original": perm.tolist(), "tile_offsets": offs.tolist(),
                                         "total_tiles": total,
                                         "non_empty": oracle.ref_count_non_empty(dims, cta_m, cta_n, cta_k)})
        out["sets"][name] = entry
    with open(os.path.join(HERE, "prepare_golden.json"), "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
