"""gg_copy_rects on the GPU: pack strided FP32 rectangles into one buffer and back (through the
C-ABI via gather.copy_rects), compared element for element with torch slicing."""
import pytest

from grouped_gemm_gpu_kernel_b200.gather import copy_rects

pytestmark = pytest.mark.gpu


def test_pack_unpack_rectangles_match_slicing(cuda):
    import torch

    g = torch.Generator(device=cuda).manual_seed(7)
    mats = [torch.rand((r, c), generator=g, device=cuda) for r, c in [(300, 257), (1, 1), (64, 1000), (5, 3), (1025, 64)]]
    rects = [(0, 10, 290, 3, 250), (1, 0, 1, 0, 1), (2, 5, 40, 100, 900), (3, 0, 5, 0, 3), (4, 0, 1025, 0, 64),
             (0, 0, 0, 0, 7), (2, 63, 1, 999, 1)]
    views = [mats[i][r0:r0 + rows, c0:c0 + cols] for i, r0, rows, c0, cols in rects]
    total = sum(v.numel() for v in views)
    packed = torch.full((total,), float("nan"), device=cuda)
    copy_rects(packed, views, to_packed=True)
    torch.cuda.synchronize()
    expect = torch.cat([v.reshape(-1) for v in views])
    assert torch.equal(packed, expect)
    # unpack into zeroed copies of the matrices: exactly the rectangles come back
    outs = [torch.zeros_like(m) for m in mats]
    oviews = [outs[i][r0:r0 + rows, c0:c0 + cols] for i, r0, rows, c0, cols in rects]
    copy_rects(packed, oviews, to_packed=False)
    torch.cuda.synchronize()
    for i, m in enumerate(mats):
        mask = torch.zeros_like(m, dtype=torch.bool)
        for j, r0, rows, c0, cols in rects:
            if j == i:
                mask[r0:r0 + rows, c0:c0 + cols] = True
        assert torch.equal(outs[i][mask], m[mask])
        assert torch.count_nonzero(outs[i][~mask]) == 0
