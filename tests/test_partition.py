"""Multi-GPU split of the problem set (CPU; the data path has no collective to test on a GPU).

gg_partition cuts the tile-weighted problem sequence into world_size contiguous shares; each
rank materialises only its pieces. These tests check that the pieces of all ranks tile every
problem's output exactly once, that the shares are balanced to within one tile's weight, and that
independent ranks (gloo, world_size 2) compute consistent, disjoint shards.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

import grouped_gemm_gpu_kernel_b200 as gg
from grouped_gemm_gpu_kernel_b200 import workloads as W


def as_problems(dims):
    return [gg.ProblemDesc(m, n, k, 1, 1, None, 1, max(1, k), max(1, n), max(1, n), max(1, n)) for m, n, k in dims]


def tile_weight(k, cfg):
    epi = max(1.0, cfg.cta_m * cfg.cta_n * 4.0 / ((cfg.cta_m + cfg.cta_n) * 128.0))
    return (-(-k // 64) if k > 0 else 0) + epi


def check_cover(dims, cfg, world):
    owner = {}
    weights = []
    for r in range(world):
        pieces, w = gg.partition(as_problems(dims), cfg, world, r)
        weights.append(w)
        for pc in pieces:
            m, n, k = dims[pc.problem]
            assert 0 <= pc.row0 and pc.row0 + pc.rows <= m and pc.rows > 0
            assert 0 <= pc.col0 and pc.col0 + pc.cols <= n and pc.cols > 0
            # pieces are aligned to the tiling, so every output tile lies in exactly one piece
            assert pc.row0 % cfg.cta_m == 0 and pc.col0 % cfg.cta_n == 0
            assert (pc.row0 + pc.rows) % cfg.cta_m == 0 or pc.row0 + pc.rows == m
            assert (pc.col0 + pc.cols) % cfg.cta_n == 0 or pc.col0 + pc.cols == n
            for tr in range(pc.row0 // cfg.cta_m, -(-(pc.row0 + pc.rows) // cfg.cta_m)):
                for tc in range(pc.col0 // cfg.cta_n, -(-(pc.col0 + pc.cols) // cfg.cta_n)):
                    key = (pc.problem, tr, tc)
                    assert key not in owner, f"tile {key} assigned twice"
                    owner[key] = r
    total_tiles = 0
    for i, (m, n, k) in enumerate(dims):
        if m > 0 and n > 0:
            tm, tn = -(-m // cfg.cta_m), -(-n // cfg.cta_n)
            total_tiles += tm * tn
    assert len(owner) == total_tiles
    maxw = max((tile_weight(k, cfg) for m, n, k in dims if m > 0 and n > 0), default=0.0)
    mean = sum(weights) / world
    assert max(weights) - mean <= maxw + 1e-6
    return weights


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_skew_split_inside_the_large_problem(world):
    dims = [(8192, 8192, 8192)] + [(128, 128, 128)] * 1023
    cfg = gg.KernelConfig(128, 256, 64)
    w = check_cover(dims, cfg, world)
    assert max(w) / (sum(w) / world) < 1.01


@pytest.mark.parametrize("name", ["small16", "mixed512", "tiny4096", "moe"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_workload_splits(name, world):
    dims = W.make_shapes(name).dims
    cfg = gg.KernelConfig(128, 128, 64)
    check_cover(dims, cfg, world)


def test_degenerate_sets():
    cfg = gg.KernelConfig(128, 128, 64)
    check_cover([], cfg, 4)
    check_cover([(0, 5, 5), (5, 0, 5)], cfg, 3)
    check_cover([(1, 1, 1)], cfg, 8)  # more ranks than tiles: the others get nothing
    check_cover([(300, 70, 0)], cfg, 2)  # K = 0 still has epilogue work
    with pytest.raises(ValueError):
        gg.partition(as_problems([(1, 1, 1)]), cfg, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, dims, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = gg.KernelConfig(128, 128, 64)
        pieces, w = gg.partition(as_problems(dims), cfg, world, rank)
        mine = [(p.problem, p.row0, p.rows, p.col0, p.cols) for p in pieces]
        gathered = [None] * world
        dist.all_gather_object(gathered, (rank, mine, w))
        if rank == 0:
            q.put(gathered)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_compute_disjoint_consistent_shards():
    import torch.multiprocessing as mp

    dims = W.make_shapes("mixed512").dims + [(8192, 1024, 512)]
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, dims, q)) for r in range(world)]
    for p in procs:
        p.start()
    gathered = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    cover = np.zeros(len(dims), dtype=np.int64)
    for rank, pieces, w in gathered:
        for prob, r0, rows, c0, cols in pieces:
            cover[prob] += rows * cols
    assert np.array_equal(cover, [m * n for m, n, k in dims])
    ws = [w for _, _, w in gathered]
    assert abs(ws[0] - ws[1]) / sum(ws) < 0.01
