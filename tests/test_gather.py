"""The optional D gather (grouped_gemm_gpu_kernel_b200.gather) with gloo ranks on CPU.

Every rank fills its own D rectangles (from gg_partition) with a value that encodes
(problem, row, column); after gather_pieces the root must hold every element of every problem
exactly once, with the encoded value, and nothing else.
"""
import os
import socket

import pytest

import grouped_gemm_gpu_kernel_b200 as gg
from grouped_gemm_gpu_kernel_b200 import workloads as W

DIMS = W.make_shapes("small16").dims + [(300, 70, 40), (1, 1, 1), (0, 50, 20), (513, 257, 64)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _code(torch, prob, r0, rows, c0, cols):
    r = torch.arange(r0, r0 + rows, dtype=torch.float64).view(-1, 1)
    c = torch.arange(c0, c0 + cols, dtype=torch.float64).view(1, -1)
    return (prob * 1_000_000 + r * 1_000 + c).to(torch.float32)


def _rank_main(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from grouped_gemm_gpu_kernel_b200.gather import gather_pieces

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = gg.KernelConfig(64, 64, 16)
        probs = [gg.ProblemDesc(m, n, k, 1, 1, None, 1, max(1, k), max(1, n), max(1, n), max(1, n))
                 for m, n, k in DIMS]
        by_rank = [gg.partition(probs, cfg, world, r)[0] for r in range(world)]
        local = [_code(torch, pc.problem, pc.row0, pc.rows, pc.col0, pc.cols) for pc in by_rank[rank]]
        root_d = None
        if rank == 0:
            root_d = {i: torch.full((max(m, 0), max(n, 0)), float("nan")) for i, (m, n, k) in enumerate(DIMS)}
        got = gather_pieces(by_rank, local, root_d)
        if rank == 0:
            ok = True
            for i, (m, n, k) in enumerate(DIMS):
                if m > 0 and n > 0:
                    ok &= bool(torch.equal(root_d[i], _code(torch, i, 0, m, 0, n)))
            expect = sum(pc.rows * pc.cols for r in range(1, world) for pc in by_rank[r]) * 4
            q.put((ok, got, expect))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gather_pieces_assembles_every_d_on_the_root(world):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    ok, got, expect = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert ok
    assert got == expect and expect > 0


def test_piece_elems_counts_rectangles():
    from grouped_gemm_gpu_kernel_b200.gather import piece_elems

    assert piece_elems([gg.ShardPiece(0, 0, 3, 0, 4), gg.ShardPiece(1, 2, 0, 0, 9)]) == 12
    assert piece_elems([]) == 0


def test_fused_targets_cover_the_root_buffer_exactly_once():
    """The D pointers that the fused gather gives each rank's pieces tile the root's buffer: every
    element of every global problem is written by exactly one piece of one rank, and no piece
    reaches outside its problem's matrix."""
    import numpy as np

    from grouped_gemm_gpu_kernel_b200.gather import fused_targets, root_offsets

    cfg = gg.KernelConfig(128, 256, 64)
    probs = [gg.ProblemDesc(m, n, k, 1, 1, None, 1, max(1, k), max(1, n), max(1, n), max(1, n)) for m, n, k in DIMS]
    total = sum(max(m, 0) * max(n, 0) for m, n, k in DIMS)
    for world in (1, 2, 3, 8):
        hits = np.zeros(total, dtype=np.int64)
        for r in range(world):
            pieces = gg.partition(probs, cfg, world, r)[0]
            for pc, (ptr, ldd) in zip(pieces, fused_targets(pieces, DIMS, base=0, elem_bytes=4)):
                first = ptr // 4
                for i in range(pc.rows):
                    hits[first + i * ldd:first + i * ldd + pc.cols] += 1
        assert (hits == 1).all(), world
    assert root_offsets([(2, 3, 1), (0, 5, 1), (4, 1, 1)]) == [0, 6, 6]
    with pytest.raises(ValueError):
        fused_targets([gg.ShardPiece(0, 1, 2, 0, 3)], [(2, 3, 1)], base=0)
