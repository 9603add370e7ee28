"""Optional gather of D to one rank after a sharded grouped GEMM (multi-GPU only).

The problems of a grouped GEMM are independent, so a problem set split across ranks by
`partition` (gg_partition: tile-weighted rectangles of D) needs no collective while it computes.
When the caller wants every D on one rank afterwards, `gather_pieces` moves each rank's D
rectangles there: a non-root rank packs all its rectangles into one contiguous FP32 buffer and
sends it with one point-to-point send (NCCL over NVLink/NVSwitch for CUDA tensors, gloo for CPU
tensors); the root posts one matching receive per rank, all in flight together, and unpacks the
rectangles into its full D matrices. Packing and unpacking of CUDA tensors are one gg_copy_rects
launch each. The reference is single-GPU and has no counterpart.
"""
from __future__ import annotations

from typing import Dict, List, Sequence

__all__ = ["gather_pieces", "piece_elems", "copy_rects", "export_buffer", "open_buffer", "close_buffer",
           "root_offsets", "fused_targets"]


def copy_rects(packed, views, to_packed: bool) -> None:
    """Moves 2-D FP32 tensors `views` (row pitch any, columns contiguous) to or from the 1-D
    tensor `packed`, each view's rows x cols elements back to back in order. CUDA tensors take
    one gg_copy_rects launch on the current stream; CPU tensors are copied view by view."""
    import ctypes

    import torch

    if packed.device.type != "cuda":
        off = 0
        for v in views:
            cnt = v.numel()
            if cnt:
                dst = packed[off:off + cnt].view(v.shape)
                if to_packed:
                    dst.copy_(v)
                else:
                    v.copy_(dst)
            off += cnt
        return
    from . import capi

    recs, off = [], 0
    for v in views:
        rows, cols = v.shape
        if rows and cols:
            if v.stride(1) != 1 and cols > 1:
                raise ValueError("columns must be contiguous")
            recs.append((v.data_ptr(), off, rows, cols, max(v.stride(0), cols) if rows > 1 else cols, 0))
        off += rows * cols
    if not recs:
        return
    arr = (capi.GGRectCopy * len(recs))(*[capi.GGRectCopy(*r) for r in recs])
    host = torch.frombuffer(bytearray(ctypes.string_at(ctypes.addressof(arr), ctypes.sizeof(arr))), dtype=torch.uint8)
    dev_recs = host.to(packed.device, non_blocking=False)
    st = capi.load().gg_copy_rects(packed.data_ptr(), dev_recs.data_ptr(), len(recs), 1 if to_packed else 0,
                                   torch.cuda.current_stream(packed.device).cuda_stream)
    if st != 0:
        raise RuntimeError(f"gg_copy_rects failed with status {st}")
    # dev_recs was allocated on the stream the copy runs on, so the caching allocator reuses its
    # memory only for work ordered after the copy.


def piece_elems(pieces) -> int:
    """FP32 elements a rank sends for these pieces (rows x cols each)."""
    return sum(max(0, p.rows) * max(0, p.cols) for p in pieces)


def gather_pieces(pieces_by_rank: Sequence[Sequence], local_d: Sequence, root_d: Dict[int, object] | None,
                  group=None, root: int = 0) -> int:
    """Collects every rank's D rectangles into the root's D matrices; returns bytes received.

    pieces_by_rank[r] -- the ShardPiece list of rank r (problem, row0, rows, col0, cols), the same
                         on every rank (gg_partition is deterministic)
    local_d           -- on every rank, one 2-D FP32 tensor per piece of this rank (rows x cols,
                         rows may be padded), in the order of pieces_by_rank[rank]
    root_d            -- on the root, {problem index: full 2-D FP32 D tensor}; None elsewhere
    The call is collective over `group`: every rank must enter it.
    """
    import torch
    import torch.distributed as dist

    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    mine = pieces_by_rank[rank]
    if len(local_d) != len(mine):
        raise ValueError("local_d must hold one tensor per piece of this rank")
    for t, pc in zip(local_d, mine):
        if tuple(t.shape) != (pc.rows, pc.cols) or t.dtype != torch.float32:
            raise ValueError("each local D must be a rows x cols FP32 tensor")

    def root_views(pieces):
        return [root_d[pc.problem][pc.row0:pc.row0 + pc.rows, pc.col0:pc.col0 + pc.cols] for pc in pieces]

    if rank == root:
        if root_d is None:
            raise ValueError("the root needs its full D tensors")
        device = next(iter(root_d.values())).device if root_d else torch.device("cpu")
        own = torch.empty(piece_elems(mine), dtype=torch.float32, device=device)
        copy_rects(own, list(local_d), to_packed=True)
        copy_rects(own, root_views(mine), to_packed=False)
        bufs: List = []
        ops = []
        for r in range(world):
            if r == root:
                bufs.append(None)
                continue
            n = piece_elems(pieces_by_rank[r])
            buf = torch.empty(n, dtype=torch.float32, device=device)
            bufs.append(buf)
            if n:
                ops.append(dist.P2POp(dist.irecv, buf, r, group))
        for w in dist.batch_isend_irecv(ops) if ops else []:
            w.wait()
        received = 0
        for r in range(world):
            if r != root and bufs[r] is not None and bufs[r].numel():
                copy_rects(bufs[r], root_views(pieces_by_rank[r]), to_packed=False)
                received += bufs[r].numel() * 4
        return received
    n = piece_elems(mine)
    if n:
        device = local_d[0].device
        buf = torch.empty(n, dtype=torch.float32, device=device)
        copy_rects(buf, list(local_d), to_packed=True)
        for w in dist.batch_isend_irecv([dist.P2POp(dist.isend, buf, root, group)]):
            w.wait()
    return 0


# ---- the gather fused into the grouped kernel ---------------------------------------------------
# Instead of computing D locally and moving it afterwards, every rank builds its executor with D
# pointers inside the root's D buffer (mapped into the rank's process with CUDA IPC): the kernel's
# epilogue then stores each tile straight into the root's memory over NVLink, overlapped with the
# tiles still being computed, and no separate gather runs. A D on another GPU is written with the
# kernel's plain coalesced stores (never TMA).

def export_buffer(t) -> bytes:
    """CUDA IPC handle (gg_ipc_handle bytes) of device tensor t's memory, for open_buffer in
    another process of this node."""
    import ctypes

    from . import capi

    h = capi.GGIpcHandle()
    st = capi.load().gg_ipc_export(ctypes.c_void_p(t.data_ptr()), ctypes.byref(h))
    if st != 0:
        raise RuntimeError(f"gg_ipc_export failed with status {st}")
    return bytes(ctypes.string_at(ctypes.addressof(h), ctypes.sizeof(h)))


def open_buffer(handle: bytes) -> int:
    """Maps another process's exported buffer; returns the device pointer of its first byte."""
    import ctypes

    from . import capi

    h = capi.GGIpcHandle.from_buffer_copy(handle)
    ptr = ctypes.c_void_p()
    st = capi.load().gg_ipc_open(ctypes.byref(h), ctypes.byref(ptr))
    if st != 0:
        raise RuntimeError(f"gg_ipc_open failed with status {st}")
    return int(ptr.value)


def close_buffer(ptr: int) -> None:
    import ctypes

    from . import capi

    st = capi.load().gg_ipc_close(ctypes.c_void_p(ptr))
    if st != 0:
        raise RuntimeError(f"gg_ipc_close failed with status {st}")


def root_offsets(dims) -> List[int]:
    """Element offsets of the global problems' D matrices (m x n, row-major, packed) back to back
    in the root's buffer."""
    offs, off = [], 0
    for m, n, k in dims:
        offs.append(off)
        off += max(m, 0) * max(n, 0)
    return offs


def fused_targets(pieces, dims, base: int, elem_bytes: int = 4):
    """(d pointer, ldd) of each piece of a rank inside the root's D buffer at device address
    `base` (layout of root_offsets): the piece's first element is row row0, column col0 of its
    global problem, whose row pitch is that problem's n."""
    offs = root_offsets(dims)
    out = []
    for pc in pieces:
        m, n, k = dims[pc.problem]
        if not (0 <= pc.row0 and pc.row0 + pc.rows <= m and 0 <= pc.col0 and pc.col0 + pc.cols <= n):
            raise ValueError("piece outside its problem")
        out.append((base + elem_bytes * (offs[pc.problem] + pc.row0 * n + pc.col0), max(1, n)))
    return out
