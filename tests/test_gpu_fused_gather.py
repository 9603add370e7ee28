"""The gather of D fused into the grouped kernel, through CUDA IPC (needs a GPU).

Two processes on one GPU stand in for two ranks: the root allocates the full D buffer of a problem
set and exports it (gg_ipc_export); the other process maps it (gg_ipc_open) and runs its
gg_partition pieces with D pointers into it (gather.fused_targets), while the root runs its own
pieces into the same buffer locally. The buffer must then equal, bit for bit, D computed whole in
one process, with every padding element untouched. On one GPU the mapping is same-device memory;
with two GPUs visible the second process also runs on GPU 1, where the same pointers are peer
memory that the kernel writes with plain stores over NVLink. Processes are spawned, never forked.
"""
from __future__ import annotations

import numpy as np
import pytest

import grouped_gemm_gpu_kernel_b200 as gg
from grouped_gemm_gpu_kernel_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _shapes(name):
    if name == "aligned":
        rng = np.random.default_rng(3)
        dims = [(int(rng.integers(1, 301)), int(8 * rng.integers(1, 41)), int(8 * rng.integers(1, 41)))
                for _ in range(24)]
        return W.Shapes("aligned24", dims, [1.25] * 24, [0.5] * 24, True)
    return W.make_shapes(name, seed=5)


def _piece_problems(ps, pieces, targets):
    """Sub-problems of the global set for `pieces`, D at the given (pointer, ldd) targets."""
    probs = ps.problems()
    out = []
    for pc, (dptr, ldd) in zip(pieces, targets):
        p = probs[pc.problem]
        c = None if p.c is None else p.c + 4 * (pc.row0 * p.ldc + pc.col0)
        out.append(gg.ProblemDesc(pc.rows, pc.cols, p.k, p.a + 2 * pc.row0 * p.lda, p.b + 2 * pc.col0, c, dptr,
                                  p.lda, p.ldb, p.ldc, ldd, p.alpha, p.beta))
    return out


def _run(problems, cfg):
    import torch

    ex = gg.GroupedGemmExecutor()
    assert ex.build(gg.prepare_problem_set(problems, cfg, gg.SortMode.kByTiles), cfg) == 0
    assert ex.run() == 0
    torch.cuda.synchronize()
    assert ex.status() == 0
    ex.close()


def _pieces(dims, cfg, world, rank):
    probs = [gg.ProblemDesc(m, n, k, 1, 1, None, 1, max(1, k), max(1, n), max(1, n), max(1, n)) for m, n, k in dims]
    return gg.partition(probs, cfg, world, rank)[0]


def _worker(name, cta, q_in, q_out, device=0):
    """Rank 1: maps the root's buffer, writes its pieces into it, reports, unmaps."""
    import torch

    from grouped_gemm_gpu_kernel_b200.gather import close_buffer, fused_targets, open_buffer

    try:
        torch.cuda.set_device(device)
        cfg = gg.KernelConfig(*cta)
        shapes = _shapes(name)
        ps = W.allocate(shapes, seed=11)
        handle = q_in.get(timeout=120)
        base = open_buffer(handle)
        pieces = _pieces(shapes.dims, cfg, 2, 1)
        _run(_piece_problems(ps, pieces, fused_targets(pieces, shapes.dims, base)), cfg)
        torch.cuda.synchronize()
        close_buffer(base)
        q_out.put(("ok", len(pieces)))
    except Exception as e:  # reported to the test, which fails on it
        q_out.put(("error", repr(e)))


def _two_devices():
    import torch

    return torch.cuda.is_available() and torch.cuda.device_count() >= 2


@pytest.mark.parametrize("name, cta, peer", [
    ("aligned", (128, 256, 64), False), ("small16", (128, 128, 64), False),
    pytest.param("aligned", (128, 256, 64), True,
                 marks=pytest.mark.skipif(not _two_devices(), reason="needs two GPUs")),
    pytest.param("mixed512", (128, 256, 64), True,
                 marks=pytest.mark.skipif(not _two_devices(), reason="needs two GPUs")),
], ids=["aligned-1gpu", "small16-1gpu", "aligned-2gpu", "mixed512-2gpu"])
def test_fused_gather_through_ipc_matches_whole_run(cuda, name, cta, peer):
    """peer: the second process runs on GPU 1, so its kernel stores its tiles into GPU 0's memory
    over NVLink (plain stores; its D is marked as another device's, never a TMA store)."""
    import torch
    import torch.multiprocessing as mp

    from grouped_gemm_gpu_kernel_b200.gather import export_buffer, fused_targets, root_offsets

    cfg = gg.KernelConfig(*cta)
    shapes = _shapes(name)
    dims = shapes.dims
    total = sum(max(m, 0) * max(n, 0) for m, n, k in dims)
    # the root's buffer, with NaN canaries past the end
    buf = torch.full((total + 256,), float("nan"), device=cuda)
    ctx = mp.get_context("spawn")
    q_in, q_out = ctx.Queue(), ctx.Queue()
    proc = ctx.Process(target=_worker, args=(name, cta, q_in, q_out, 1 if peer else 0))
    proc.start()
    try:
        q_in.put(export_buffer(buf))
        ps = W.allocate(shapes, seed=11)
        mine = _pieces(dims, cfg, 2, 0)
        _run(_piece_problems(ps, mine, fused_targets(mine, dims, buf.data_ptr())), cfg)
        status, info = q_out.get(timeout=180)
        assert status == "ok", info
        assert info > 0  # the other rank had pieces
    finally:
        proc.join(timeout=120)
    assert proc.exitcode == 0
    # the whole set computed in this process, D packed in the same layout
    whole = torch.full_like(buf, float("nan"))
    all_pieces = _pieces(dims, cfg, 1, 0)
    _run(_piece_problems(ps, all_pieces, fused_targets(all_pieces, dims, whole.data_ptr())), cfg)
    assert torch.equal(buf[:total], whole[:total])
    assert not torch.isnan(buf[:total]).any()
    assert torch.isnan(buf[total:]).all()
    assert root_offsets(dims)[-1] + dims[-1][0] * dims[-1][1] == total
