"""The CPU oracle, pinned against the reference's own code (CPU, no GPU).

The oracle (oracle/gg_oracle.c) restates the reference's host algorithm; these tests hold it to
the committed golden fixtures (made by tests/golden/make_golden.py from the reference's sources
compiled unmodified) and, where oracle/_ref/libgg_ref.so exists, to the reference build itself.
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_prepare_golden():
    with open(os.path.join(GOLDEN, "prepare_golden.json")) as f:
        return json.load(f)


def ref_test_problems():
    """The reference test's problems (tests/test_correctness.cu:313-322) from the fixture."""
    fx = np.load(os.path.join(GOLDEN, "ref_test_shapes.npz"))
    out = []
    oa = ob = oc = 0
    for (m, n, k), al, be in zip(fx["shapes"].tolist(), fx["alpha"].tolist(), fx["beta"].tolist()):
        lda, ldb, ldc = max(1, k), max(1, n), max(1, n)
        # packed with the reference's allocation rule (tests/test_correctness.cu:75-80,136-140)
        na, nb, nc = O.safe_elems(m, lda), O.safe_elems(k, ldb), O.safe_elems(m, ldc)
        out.append(dict(m=m, n=n, k=k, lda=lda, ldb=ldb, ldc=ldc, ldd=ldc, alpha=al, beta=be,
                        a=fx["a"][oa:oa + na], b=fx["b"][ob:ob + nb], c=fx["c"][oc:oc + nc], ref=fx["ref"][oc:oc + nc]))
        oa += na
        ob += nb
        oc += nc
    assert oa == fx["a"].size and ob == fx["b"].size and oc == fx["c"].size
    return out


def test_fp16_decode_exhaustive():
    lib = O.load_oracle()
    bits = np.arange(65536, dtype=np.uint16)
    want = bits.view(np.float16).astype(np.float64)
    got = np.array([lib.oracle_half_to_double(int(b)) for b in bits[::97]])
    w = want[::97]
    finite = np.isfinite(w)
    assert np.array_equal(got[finite], w[finite])
    assert np.array_equal(np.isnan(got), np.isnan(w))
    assert np.array_equal(np.isinf(got), np.isinf(w))


def test_host_known_answers():
    # reference src/grouped_gemm.cu:967-1022 on the six shapes with 64x64 tiles
    dims = [(64, 64, 64), (128, 64, 96), (45, 81, 37), (17, 23, 9), (0, 64, 16), (192, 32, 64)]
    perm, offs, total = O.prepare(dims, 64, 64, 0)
    assert offs.tolist() == [0, 1, 3, 5, 6, 6, 9] and total == 9
    assert O.prepare(dims, 64, 64, 1)[0].tolist() == [1, 5, 0, 2, 4, 3]
    assert O.prepare(dims, 64, 64, 2)[0].tolist() == [5, 1, 2, 0, 3, 4]
    assert O.prepare(dims, 64, 64, 3)[0].tolist() == [5, 1, 2, 0, 3, 4]


def test_prepare_matches_golden():
    g = load_prepare_golden()
    checked = 0
    for name, entry in g["sets"].items():
        for r in entry["results"]:
            perm, offs, total = O.prepare(entry["dims"], r["cta"][0], r["cta"][1], r["mode"])
            assert perm.tolist() == r["sorted_to_original"], (name, r["cta"], r["mode"])
            assert offs.tolist() == r["tile_offsets"], (name, r["cta"], r["mode"])
            assert total == r["total_tiles"]
            checked += 1
    assert checked >= 300


def test_tile_count_matches_golden_non_empty():
    g = load_prepare_golden()
    for entry in g["sets"].values():
        for r in entry["results"]:
            ne = sum(1 for m, n, k in entry["dims"] if O.tile_count(m, n, r["cta"][0], r["cta"][1]) > 0)
            assert ne == r["non_empty"]


def test_f32_port_bit_exact_against_reference_fixture():
    """oracle_gemm_f32_refloop restates compute_reference: identical bits on the fixture."""
    for p in ref_test_problems():
        if p["m"] <= 0 or p["n"] <= 0:
            continue
        d = O.gemm_f32_refloop(p["m"], p["n"], p["k"], p["a"], p["lda"], p["b"], p["ldb"], p["c"], p["ldc"],
                               p["alpha"], p["beta"], p["ldd"])
        assert np.array_equal(d[:p["m"] * p["n"]], p["ref"][:p["m"] * p["n"]])


def test_f64_oracle_against_reference_fixture():
    """The FP64 oracle agrees with the reference's FP32 host GEMM far inside the accuracy bound."""
    for p in ref_test_problems():
        m, n, k = p["m"], p["n"], p["k"]
        if m <= 0 or n <= 0:
            continue
        d, s = O.gemm_f64(m, n, k, p["a"], p["lda"], p["b"], p["ldb"], p["c"], p["ldc"], p["alpha"], p["beta"])
        err = O.rel_err(p["ref"][:m * n].reshape(m, n), d, s)
        assert err < 1e-5 < O.tolerance(k), (m, n, k, err)


def test_f64_row_sampling_matches_full():
    rng = np.random.default_rng(3)
    m, n, k = 37, 29, 53
    a = rng.uniform(-1, 1, m * k).astype(np.float16).view(np.uint16)
    b = rng.uniform(-1, 1, k * n).astype(np.float16).view(np.uint16)
    c = rng.uniform(-1, 1, m * n).astype(np.float32)
    full, sf = O.gemm_f64(m, n, k, a, k, b, n, c, n, 1.25, -0.5)
    rows = np.array([0, 5, 36, 17], dtype=np.int32)
    part, sp = O.gemm_f64(m, n, k, a, k, b, n, c, n, 1.25, -0.5, rows=rows)
    assert np.array_equal(part, full[rows])
    assert np.array_equal(sp, sf[rows])
    ref = (a.view(np.float16).astype(np.float64).reshape(m, k) @ b.view(np.float16).astype(np.float64).reshape(k, n))
    assert np.allclose(full, 1.25 * ref - 0.5 * c.reshape(m, n).astype(np.float64), rtol=1e-12, atol=1e-12)


def test_f64_beta_zero_ignores_nan_c():
    """C is read only when c != NULL and beta != 0 (reference src/grouped_gemm.cu:475,616)."""
    a = np.ones(4, np.float16).view(np.uint16)
    b = np.ones(4, np.float16).view(np.uint16)
    c = np.full(4, np.nan, np.float32)
    d, _ = O.gemm_f64(2, 2, 2, a, 2, b, 2, c, 2, 1.0, 0.0)
    assert np.all(d == 2.0)
    d2, _ = O.gemm_f64(2, 2, 2, a, 2, b, 2, None, 2, 1.0, 0.7)
    assert np.all(d2 == 2.0)


def test_tolerance_formula():
    assert O.tolerance(1024) == pytest.approx(2e-3)
    assert O.tolerance(4096) == pytest.approx(4e-3)
    assert O.tolerance(0) == O.tolerance(1)


def test_planted_mistake_is_caught():
    """A deliberately wrong result (planted on the CPU) fails the metric the GPU tests use."""
    rng = np.random.default_rng(9)
    m, n, k = 16, 16, 64
    a = rng.uniform(-1, 1, m * k).astype(np.float16).view(np.uint16)
    b = rng.uniform(-1, 1, k * n).astype(np.float16).view(np.uint16)
    d, s = O.gemm_f64(m, n, k, a, k, b, n, None, n, 1.0, 0.0)
    bad = d.copy()
    bad[3, 7] += 0.05
    assert O.rel_err(d.astype(np.float32), d, s) < O.tolerance(k)
    assert O.rel_err(bad, d, s) > O.tolerance(k)


@pytest.mark.skipif(not O.ref_available(), reason="reference build oracle/_ref absent")
def test_oracle_prepare_matches_reference_build_random():
    rng = np.random.default_rng(11)
    cfgs = [(64, 64, 16), (128, 64, 32), (64, 128, 32), (128, 128, 64), (128, 256, 64)]
    for _ in range(150):
        P = int(rng.integers(0, 50))
        dims = [(int(rng.integers(0, 4)) * int(rng.integers(1, 90)), int(rng.integers(0, 4)) * int(rng.integers(1, 90)),
                 int(rng.choice([0, 16, 32, 48]))) for _ in range(P)]
        for cm, cn, ck in cfgs:
            for mode in range(5):
                a = O.prepare(dims, cm, cn, mode)
                b = O.ref_prepare(dims, cm, cn, ck, mode)
                assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1]) and a[2] == b[2]


@pytest.mark.skipif(not O.ref_available(), reason="reference build oracle/_ref absent")
def test_reference_host_gemm_matches_fixture():
    probs = [p for p in ref_test_problems()]
    outs, secs = O.ref_host_gemm(probs, threads=2)
    for p, d in zip(probs, outs):
        if p["m"] > 0 and p["n"] > 0:
            assert np.array_equal(d[:p["m"] * p["n"]], p["ref"][:p["m"] * p["n"]])
    assert secs >= 0.0


def test_bf16_decode_and_gemm_against_numpy():
    """oracle_gemm_f64 with BF16 inputs (fmt 1): exact decode (top half of a float32) and the same
    FP64 result numpy gets from the decoded values."""
    rng = np.random.default_rng(11)
    m, n, k = 7, 5, 13
    af = rng.uniform(-2, 2, size=(m, k)).astype(np.float32)
    bf = rng.uniform(-2, 2, size=(k, n)).astype(np.float32)
    a16 = (af.view(np.uint32) >> 16).astype(np.uint16)
    b16 = (bf.view(np.uint32) >> 16).astype(np.uint16)
    lib = O.load_oracle()
    for bits in (0x3F80, 0xC000, 0x0001, 0x7F7F, 0x8000):
        want = float(np.array([bits << 16], dtype=np.uint32).view(np.float32)[0])
        assert lib.oracle_bf16_to_double(bits) == want
    ad = (a16.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    bd = (b16.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    c = rng.uniform(-1, 1, size=(m, n)).astype(np.float32)
    d, _ = O.gemm_f64(m, n, k, a16, k, b16, n, c, n, 1.5, -0.5, fmt=1)
    assert np.allclose(d, 1.5 * ad @ bd - 0.5 * c.astype(np.float64), rtol=0, atol=1e-12)


def test_epilogue_bias_and_activations_against_numpy():
    """oracle_gemm_f64_epilogue: D = act(alpha*A*B + beta*C + bias) for ReLU and the tanh form of
    GELU, scale = L * (|alpha| sqrt(sum p^2) + |beta c| + |bias|) with L = 1.13 for GELU; and the
    16-bit output rounding allowance of rel_err."""
    rng = np.random.default_rng(12)
    m, n, k = 6, 9, 17
    a = rng.uniform(-1, 1, size=(m, k)).astype(np.float16)
    b = rng.uniform(-1, 1, size=(k, n)).astype(np.float16)
    c = rng.uniform(-1, 1, size=(m, n)).astype(np.float32)
    bias = rng.uniform(-1, 1, size=n).astype(np.float32)
    p = a.astype(np.float64)[:, :, None] * b.astype(np.float64)[None, :, :]
    z = 1.5 * p.sum(1) - 0.5 * c + bias
    base_scale = 1.5 * np.sqrt((p * p).sum(1)) + np.abs(0.5 * c) + np.abs(bias)
    gelu = 0.5 * z * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (z + 0.044715 * z ** 3)))
    for act, want, lip in ((0, z, 1.0), (1, np.maximum(z, 0.0), 1.0), (2, gelu, 1.13)):
        d, s = O.gemm_f64(m, n, k, a.view(np.uint16), k, b.view(np.uint16), n, c, n, 1.5, -0.5, bias=bias, act=act)
        assert np.allclose(d, want, rtol=0, atol=1e-12)
        assert np.allclose(s, lip * base_scale, rtol=1e-12, atol=0)
    # the selected-rows path indexes bias by output column
    d_rows, _ = O.gemm_f64(m, n, k, a.view(np.uint16), k, b.view(np.uint16), n, c, n, 1.5, -0.5, rows=[4, 1],
                           bias=bias, act=2)
    assert np.allclose(d_rows, gelu[[4, 1]], rtol=0, atol=1e-12)
    # rel_err: an FP16-rounded result is within its rounding allowance, an FP32 check is stricter
    d16 = gelu.astype(np.float16).astype(np.float64)
    s = np.full_like(gelu, 1e-9)
    assert O.rel_err(d16, gelu, s, out_fmt=1) == 0.0
    assert O.rel_err(d16, gelu, s, out_fmt=0) > 0.0
    u = gelu.astype(np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000  # round to nearest even BF16
    dbf = u.astype(np.uint32).view(np.float32).astype(np.float64)
    assert O.rel_err(dbf, gelu, s, out_fmt=2) == 0.0
    assert O.rel_err(dbf, gelu, s, out_fmt=1) > 0.0


def test_fp8_decode_and_gemm_against_torch():
    """E4M3 and E5M2 decode (every one of the 256 codes against torch's float8 types) and an FP8
    oracle GEMM against numpy on the decoded values."""
    import torch

    lib = O.load_oracle()
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8)
    for fmt, dt in ((2, torch.float8_e4m3fn), (3, torch.float8_e5m2)):
        want = codes.view(dt).to(torch.float64).numpy()
        got = np.array([lib.oracle_fp8_to_double(int(v), fmt) for v in range(256)])
        assert np.array_equal(np.isnan(got), np.isnan(want))
        ok = ~np.isnan(want)
        assert np.array_equal(got[ok], want[ok])
    rng = np.random.default_rng(13)
    m, n, k = 5, 6, 40
    for fmt, dt in ((2, torch.float8_e4m3fn), (3, torch.float8_e5m2)):
        a8 = torch.from_numpy(rng.uniform(-2, 2, size=(m, k)).astype(np.float32)).to(dt)
        b8 = torch.from_numpy(rng.uniform(-2, 2, size=(k, n)).astype(np.float32)).to(dt)
        ad, bd = a8.to(torch.float64).numpy(), b8.to(torch.float64).numpy()
        d, _ = O.gemm_f64(m, n, k, a8.view(torch.uint8).numpy(), k, b8.view(torch.uint8).numpy(), n, None, n, 0.5,
                          0.0, fmt=fmt)
        assert np.allclose(d, 0.5 * ad @ bd, rtol=0, atol=1e-12)
