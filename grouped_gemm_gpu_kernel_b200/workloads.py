"""Seeded synthetic problem sets with the shapes and value laws of the five benchmark configurations.

The reference measures on no public suite; these generators stand in for its inputs:

  small16   16 problems, M, N, K ~ U{16..256}; A, B FP16 ~ U[-1,1]; C FP32 ~ U[-1,1]; alpha 1, beta 0.5
  mixed512  512 problems, M, N, K log-uniform on [64, 1024] rounded to multiples of 8; U[-1,1];
            C ~ U[-1,1] (allocated, not read: beta 0); alpha 1
  moe       64 experts, M_i = tokens routed to expert i when 16384 tokens each draw an expert from a
            Zipf(s=1.1) law over 64 ranks (zero-token experts are kept), N 14336, K 4096;
            A ~ N(0,1), B ~ N(0,0.02) FP16; no C; alpha 1, beta 0
  tiny4096  4096 problems, M, N, K ~ U{1..64}; U[-1,1]; alpha 1.5, beta -0.5
  skew      one 8192^3 problem followed by 1023 problems of 128^3; U[-1,1]; no C; alpha 1, beta 0

Leading dimensions are packed (lda = K, ldb = ldc = ldd = N, as the reference test packs them,
reference tests/test_correctness.cu:128-131), so odd K or N give problems that TMA cannot load
and the kernel's zero-fill loader takes. Each operand of each problem starts on a 256-byte
boundary inside one slab per operand kind. Shapes come from numpy's PCG64 seeded by `seed`;
values from a CUDA torch generator seeded by `seed`.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

CONFIG_NAMES = ("small16", "mixed512", "moe", "tiny4096", "skew")
# A reduced MoE layer (8 experts, 2048 tokens, the same N and K) for profiling captures that must
# stay small; not one of the benchmark configurations.
PROFILE_NAMES = ("moe_reduced",)
ALIGN_BYTES = 256


@dataclass
class Shapes:
    name: str
    dims: List[Tuple[int, int, int]]
    alpha: List[float]
    beta: List[float]
    has_c: bool
    a_law: str = "uniform"   # "uniform": U[-1,1]; "normal": N(0, a_std)
    a_std: float = 1.0
    b_law: str = "uniform"
    b_std: float = 1.0

    @property
    def flops(self) -> float:
        return float(sum(2.0 * m * n * k for m, n, k in self.dims))

    def algorithmic_bytes(self, out_bytes: int = 4, bias: bool = False, in_bytes: int = 2) -> float:
        """A and B read once (in_bytes per element: 2 for FP16/BF16, 1 for FP8), D written once, C
        read when beta != 0 (out_bytes per C/D element: 4 for FP32, 2 for FP16/BF16), and, with
        `bias`, n FP32 bias values per problem."""
        tot = 0.0
        for (m, n, k), b in zip(self.dims, self.beta):
            if m <= 0 or n <= 0:
                continue
            tot += in_bytes * (m * k + k * n) + out_bytes * m * n
            if self.has_c and b != 0.0:
                tot += out_bytes * m * n
            if bias:
                tot += 4.0 * n
        return tot


def _log_uniform8(rng, size):
    x = np.exp(rng.uniform(np.log(64.0), np.log(1024.0), size=size))
    return np.clip(np.round(x / 8.0) * 8.0, 64, 1024).astype(np.int64)


def zipf_split(total_tokens: int, experts: int, s: float, rng) -> np.ndarray:
    """Token counts per expert: each token draws a rank with P(r) ~ r^-s, ranks map to experts
    through a seeded permutation; experts that draw no token keep M_i = 0."""
    p = np.arange(1, experts + 1, dtype=np.float64) ** (-s)
    p /= p.sum()
    ranks = rng.choice(experts, size=total_tokens, p=p)
    perm = rng.permutation(experts)
    return np.bincount(perm[ranks], minlength=experts).astype(np.int64)


def make_shapes(name: str, seed: int = 42) -> Shapes:
    rng = np.random.default_rng(seed)
    if name == "small16":
        d = rng.integers(16, 257, size=(16, 3))
        dims = [tuple(int(x) for x in r) for r in d]
        return Shapes(name, dims, [1.0] * 16, [0.5] * 16, True)
    if name == "mixed512":
        d = _log_uniform8(rng, (512, 3))
        dims = [tuple(int(x) for x in r) for r in d]
        return Shapes(name, dims, [1.0] * 512, [0.0] * 512, True)
    if name == "moe":
        counts = zipf_split(16384, 64, 1.1, rng)
        dims = [(int(c), 14336, 4096) for c in counts]
        return Shapes(name, dims, [1.0] * 64, [0.0] * 64, False, "normal", 1.0, "normal", 0.02)
    if name == "moe_reduced":
        counts = zipf_split(2048, 8, 1.1, rng)
        dims = [(int(c), 14336, 4096) for c in counts]
        return Shapes(name, dims, [1.0] * 8, [0.0] * 8, False, "normal", 1.0, "normal", 0.02)
    if name == "tiny4096":
        d = rng.integers(1, 65, size=(4096, 3))
        dims = [tuple(int(x) for x in r) for r in d]
        return Shapes(name, dims, [1.5] * 4096, [-0.5] * 4096, True)
    if name == "skew":
        dims = [(8192, 8192, 8192)] + [(128, 128, 128)] * 1023
        return Shapes(name, dims, [1.0] * 1024, [0.0] * 1024, False)
    raise ValueError(f"unknown workload {name!r}; expected one of {CONFIG_NAMES + PROFILE_NAMES}")


def _aligned(n_elems: int, elem_bytes: int) -> int:
    per = ALIGN_BYTES // elem_bytes
    return (max(n_elems, 1) + per - 1) // per * per


@dataclass
class DeviceProblemSet:
    """Device slabs + per-problem offsets (elements) for one workload."""

    shapes: Shapes
    a: "object"  # torch fp16 slab
    b: "object"
    c: Optional["object"]
    d: "object"  # torch fp32 slab
    a_off: List[int] = field(default_factory=list)
    b_off: List[int] = field(default_factory=list)
    c_off: List[int] = field(default_factory=list)
    d_off: List[int] = field(default_factory=list)
    out_fmt: int = 0                  # C / D element type: 0 FP32, 1 FP16, 2 BF16 (KernelConfig.output_type)
    in_fmt: int = 0                   # A / B element type: 0 FP16, 1 BF16, 2 E4M3, 3 E5M2 (KernelConfig.input_type)
    lda: Optional[List[int]] = None   # row pitches of A and B per problem (None: packed, k and n)
    ldb: Optional[List[int]] = None
    a_col: bool = False               # A stored column-major (k x m, lda >= m; KernelConfig.a_layout)
    b_col: bool = False               # B stored column-major (n x k, ldb >= k; KernelConfig.b_layout)
    bias: Optional["object"] = None   # FP32 slab of per-problem bias vectors (make_bias)
    bias_off: List[Optional[int]] = field(default_factory=list)  # element offset, None = no bias

    def problems(self):
        from . import ProblemDesc
        out = []
        eo = 4 if self.out_fmt == 0 else 2
        ei = self.a.element_size()
        ab, bb, db = self.a.data_ptr(), self.b.data_ptr(), self.d.data_ptr()
        cb = self.c.data_ptr() if self.c is not None else None
        for i, ((m, n, k), al, be) in enumerate(zip(self.shapes.dims, self.shapes.alpha, self.shapes.beta)):
            lda = self.lda[i] if self.lda else max(1, k)
            ldb = self.ldb[i] if self.ldb else max(1, n)
            out.append(ProblemDesc(m, n, k, ab + ei * self.a_off[i], bb + ei * self.b_off[i],
                                   (cb + eo * self.c_off[i]) if cb is not None else None, db + eo * self.d_off[i],
                                   lda, ldb, max(1, n), max(1, n), al, be))
        return out

    def _relayout(self, convert, out_dtype, a_col: bool, b_col: bool, pad: int) -> None:
        """New A and B slabs holding convert(logical operand) in the given storage layouts, each
        operand starting on a 256-byte boundary, row pitches padded to multiples of `pad`."""
        import torch

        def up(x):
            return (max(x, 1) + pad - 1) // pad * pad

        esz = torch.empty(0, dtype=out_dtype).element_size()
        lda = [up(m if a_col else k) for m, n, k in self.shapes.dims]
        ldb = [up(k if b_col else n) for m, n, k in self.shapes.dims]
        a_off, b_off, na, nb = [], [], 0, 0
        for (m, n, k), la, lb in zip(self.shapes.dims, lda, ldb):
            a_off.append(na)
            na += _aligned(max(k if a_col else m, 0) * la, esz)
            b_off.append(nb)
            nb += _aligned(max(n if b_col else k, 0) * lb, esz)
        a2 = torch.zeros(max(na, 1), dtype=out_dtype, device=self.a.device)
        b2 = torch.zeros(max(nb, 1), dtype=out_dtype, device=self.b.device)
        for i, (m, n, k) in enumerate(self.shapes.dims):
            A, B, _, _ = self.views(i)  # logical m x k and k x n
            if A is not None:
                if a_col:
                    a2[a_off[i]:a_off[i] + k * lda[i]].view(k, lda[i])[:, :m].copy_(convert(A.t()))
                else:
                    a2[a_off[i]:a_off[i] + m * lda[i]].view(m, lda[i])[:, :k].copy_(convert(A))
            if B is not None:
                if b_col:
                    b2[b_off[i]:b_off[i] + n * ldb[i]].view(n, ldb[i])[:, :k].copy_(convert(B.t()))
                else:
                    b2[b_off[i]:b_off[i] + k * ldb[i]].view(k, ldb[i])[:, :n].copy_(convert(B))
        self.a, self.b, self.a_off, self.b_off, self.lda, self.ldb = a2, b2, a_off, b_off, lda, ldb
        self.a_col, self.b_col = a_col, b_col

    def to_fp8(self, fmt: int, pad: int = 16) -> "DeviceProblemSet":
        """A and B re-encoded as 8-bit floats for runs with KernelConfig.input_type = fmt (2 E4M3,
        3 E5M2): each FP16 value rounded to the nearest 8-bit value by torch, one byte per element,
        in new uint8 slabs whose operands start on 256-byte boundaries, row pitches padded to
        multiples of `pad` elements (16: every row 16-byte aligned, so TMA loads them; 1: packed,
        odd pitches go through the zero-fill loader). The storage layouts are kept."""
        import torch

        dt = {2: torch.float8_e4m3fn, 3: torch.float8_e5m2}[int(fmt)]
        self._relayout(lambda t: t.to(dt).view(torch.uint8), torch.uint8, self.a_col, self.b_col, pad)
        self.in_fmt = int(fmt)
        return self

    def to_layout(self, a_col: bool, b_col: bool, pad: int = 1) -> "DeviceProblemSet":
        """A and/or B stored column-major (A as k x m, B as n x k: KernelConfig.a_layout / b_layout
        = 1) with the same values; row pitches padded to multiples of `pad` elements (1: packed,
        so odd sizes reach the zero-fill loader; 8: every 16-bit row 16-byte aligned, for TMA)."""
        self._relayout(lambda t: t, self.a.dtype, a_col, b_col, pad)
        return self

    def to_output(self, out_fmt: int) -> "DeviceProblemSet":
        """C and D in the 16-bit output type `out_fmt` (1 FP16, 2 BF16; KernelConfig.output_type):
        C becomes its FP32 values rounded to that type, D a NaN-filled buffer of that type, both at
        the same element offsets (which keeps every row start 16-byte aligned)."""
        import torch

        dt = {1: torch.float16, 2: torch.bfloat16}[int(out_fmt)]
        if self.c is not None:
            self.c = self.c.to(dt)
        self.d = torch.full(self.d.shape, float("nan"), dtype=dt, device=self.d.device)
        self.out_fmt = int(out_fmt)
        return self

    def make_bias(self, seed: int = 7, without: float = 0.25, aligned: bool = False) -> List[Optional[int]]:
        """One FP32 bias vector of n values ~ U[-1,1] per problem, a seeded fraction `without` of
        the problems having none; returns the device pointers in problem order (None: no bias).
        Each vector starts on a 256-byte boundary (`aligned`) or 4 bytes past one (no vector
        16-byte aligned: the kernel's unaligned bias path)."""
        import torch

        rng = np.random.default_rng(seed)
        offs: List[Optional[int]] = []
        total = 0
        for m, n, k in self.shapes.dims:
            if rng.random() < without:
                offs.append(None)
                continue
            offs.append(total + (0 if aligned else 1))
            total += _aligned(max(n, 0) + 1, 4)
        g = torch.Generator(device=self.a.device)
        g.manual_seed(seed)
        self.bias = torch.empty(max(total, 1), dtype=torch.float32, device=self.a.device).uniform_(-1.0, 1.0,
                                                                                                  generator=g)
        self.bias_off = offs
        base = self.bias.data_ptr()
        return [None if o is None else base + 4 * o for o in offs]

    def bias_host(self, i: int, cols: Optional[np.ndarray] = None) -> Optional[np.ndarray]:
        """Host copy (float32) of problem i's bias, or of its entries `cols`; None without bias."""
        if self.bias is None or self.bias_off[i] is None:
            return None
        n = self.shapes.dims[i][1]
        v = self.bias[self.bias_off[i]:self.bias_off[i] + n].cpu().numpy()
        return v if cols is None else v[np.asarray(cols)]

    def to_bf16(self) -> "DeviceProblemSet":
        """Re-encodes A and B in place as BF16 (each FP16 value rounded to the nearest BF16), for
        runs with KernelConfig.input_type = 1. The slabs keep their torch dtype (float16) and now
        hold BF16 bit patterns."""
        import torch

        for t in (self.a, self.b):
            v = t.float()
            t.view(torch.bfloat16).copy_(v)
        return self

    def views(self, i: int):
        """(A, B, C or None, D) torch views of problem i; A and B are the logical m x k and k x n
        operands whatever their storage layout."""
        m, n, k = self.shapes.dims[i]
        la = self.lda[i] if self.lda else k
        lb = self.ldb[i] if self.ldb else n
        A = B = None
        if m * k > 0:  # logical m x k (a transposed view of a column-major store)
            A = (self.a[self.a_off[i]:self.a_off[i] + k * la].view(k, la)[:, :m].t() if self.a_col else
                 self.a[self.a_off[i]:self.a_off[i] + m * la].view(m, la)[:, :k])
        if k * n > 0:  # logical k x n
            B = (self.b[self.b_off[i]:self.b_off[i] + n * lb].view(n, lb)[:, :k].t() if self.b_col else
                 self.b[self.b_off[i]:self.b_off[i] + k * lb].view(k, lb)[:, :n])
        C = None
        if self.c is not None and m * n > 0:
            C = self.c[self.c_off[i]:self.c_off[i] + m * n].view(m, n)
        D = self.d[self.d_off[i]:self.d_off[i] + m * n].view(m, n) if m * n > 0 else None
        return A, B, C, D


def allocate(shapes: Shapes, device="cuda", seed: int = 42, d_fill: float = float("nan")) -> DeviceProblemSet:
    """Device slabs for `shapes`, filled with the config's value laws (seeded on the device)."""
    import torch

    a_off, b_off, c_off, d_off = [], [], [], []
    na = nb = nc = nd = 0
    for m, n, k in shapes.dims:
        a_off.append(na)
        na += _aligned(max(m, 0) * max(k, 0), 2)
        b_off.append(nb)
        nb += _aligned(max(k, 0) * max(n, 0), 2)
        c_off.append(nc)
        nc += _aligned(max(m, 0) * max(n, 0), 4)
        d_off.append(nd)
        nd += _aligned(max(m, 0) * max(n, 0), 4)
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def fill16(count, law, std):
        t = torch.empty(count, dtype=torch.float16, device=device)
        if law == "normal":
            t.normal_(0.0, std, generator=g)
        else:
            t.uniform_(-1.0, 1.0, generator=g)
        return t

    a = fill16(na, shapes.a_law, shapes.a_std)
    b = fill16(nb, shapes.b_law, shapes.b_std)
    c = None
    if shapes.has_c:
        c = torch.empty(nc, dtype=torch.float32, device=device)
        c.uniform_(-1.0, 1.0, generator=g)
    d = torch.full((nd,), d_fill, dtype=torch.float32, device=device)
    return DeviceProblemSet(shapes, a, b, c, d, a_off, b_off, c_off, d_off)


def host_inputs(ps: DeviceProblemSet, i: int, rows: Optional[np.ndarray] = None,
                cols: Optional[np.ndarray] = None) -> Dict[str, object]:
    """Host copies (16-bit A/B bits as uint16, C and D widened to float32) of problem i for the
    CPU oracle.

    With `rows`/`cols` only those rows of A (and C) and those columns of B (and C) are copied,
    so a full-size problem can be checked on a sample."""
    import torch

    m, n, k = ps.shapes.dims[i]
    A, B, C, D = ps.views(i)
    if rows is not None:
        ridx = torch.as_tensor(rows, device=ps.a.device, dtype=torch.long)
        A = A.index_select(0, ridx) if A is not None else None
        C = C.index_select(0, ridx) if C is not None else None
        D = D.index_select(0, ridx) if D is not None else None
    if cols is not None:
        cidx = torch.as_tensor(cols, device=ps.a.device, dtype=torch.long)
        B = B.index_select(1, cidx) if B is not None else None
        C = C.index_select(1, cidx) if C is not None else None
        D = D.index_select(1, cidx) if D is not None else None
    out = {}
    def bits(t):  # the operand's raw bits: uint16 for 16-bit types, uint8 for 8-bit ones
        if t is None:
            return np.zeros(1, np.uint8 if ps.a.element_size() == 1 else np.uint16)
        t = t.contiguous()
        return t.cpu().numpy() if t.element_size() == 1 else t.view(torch.int16).cpu().numpy().view(np.uint16)

    out["a"] = bits(A)
    out["b"] = bits(B)
    out["c"] = C.contiguous().float().cpu().numpy() if C is not None else None
    out["d"] = D.contiguous().float().cpu().numpy() if D is not None else None
    return out
