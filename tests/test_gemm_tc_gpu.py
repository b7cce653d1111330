"""The tensor-core CQ GEMM (wc_cq_gemm_ex with WC_GEMM_TENSOR_CORES).

It multiplies in the rotated domain with fp16 operands (each scaled by an
exact power of two, per activation row and per matrix) and fp32
accumulation, so it is checked against the float64 product of the
reference's dequantisation (internal/cq/cq_test.go:70 dequant64) under the
bound this repository states for it (refmath.tc_bound, the header's
WC_GEMM_TENSOR_CORES): per element

    |y - y64| <= (2^-10 + (K + log2 G + 6) · 2^-24) · Σ_k |x̂_k| · |ŵ_k|
                 + 2^-37 · (G·max|x| · Σ_k |ŵ_k| + max|ŵ| · Σ_k |x̂_k|)

(x̂ = H·x per group, ŵ = cb[idx]·n/√G), and by the reference's own accept
for its lut kernel, cosine >= 0.99999 per row against the float64 product
(internal/cq/cq_test.go:196-254).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import refmath

pytestmark = pytest.mark.gpu

WC_GEMM_TENSOR_CORES = 1


def tc_gemm(wb, cuda, m, x):
    rows = x.shape[0]
    xd = cuda.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    yd = cuda.full((rows, m.Out()), float("nan"), dtype=cuda.float32, device="cuda")
    wb._lib.check(wb._lib.lib().wc_cq_gemm_ex(m.handle, ctypes.c_void_p(xd.data_ptr()),
                                              ctypes.c_void_p(yd.data_ptr()), rows, WC_GEMM_TENSOR_CORES, None))
    code = ctypes.c_int(-1)
    wb._lib.check(wb._lib.lib().wc_device_status(ctypes.byref(code)))
    assert code.value == 0, f"a bounded wait expired (code {code.value})"
    return yd.cpu().numpy()


# (rows, out, in, group, bits); from 1024 rows the persistent kernel runs
# (128 x 256 tiles, two TMEM accumulators): outputs narrower than one tile,
# not a multiple of 256, K not a multiple of 64, several tiles per CTA.
CASES = [(128, 128, 64, 32, 4), (300, 200, 512, 32, 4), (257, 96, 512, 128, 2), (129, 384, 512, 128, 2),
         (64, 1024, 512, 128, 2), (200, 512, 2048, 32, 4), (1000, 2048, 512, 32, 4), (130, 70, 200, 32, 2),
         (1024, 96, 512, 128, 2), (1500, 700, 200, 32, 2), (2500, 2048, 512, 32, 4), (1100, 512, 2048, 32, 4),
         (24000, 384, 512, 128, 2), (1030, 130, 512, 32, 4)]


@pytest.mark.parametrize("case", CASES, ids=[f"m{c[0]}_{c[1]}x{c[2]}g{c[3]}b{c[4]}" for c in CASES])
def test_tc_gemm_within_bound(wb, cuda, case):
    rows, out, in_, group, bits = case
    rng = np.random.default_rng(sum(case))
    p = wb.synth.random_packed(rng, out, in_, group, bits, "lloyd")
    m = wb.cq.New(p)
    x = rng.normal(size=(rows, in_)).astype(np.float32)
    got = tc_gemm(wb, cuda, m, x)
    assert np.all(np.isfinite(got))
    want, bound = refmath.tc_bound(p, x.astype(np.float64))
    assert np.all(np.abs(got - want) <= bound)
    # the rotated product is the reference's product: dequant64 · x
    assert np.allclose(want, x.astype(np.float64) @ refmath.dequant64(p).T, rtol=1e-9, atol=1e-9)
    assert _rows_cosine(got.astype(np.float64), want).min() >= TC_COSINE


def test_tc_gemm_views_and_reuse(wb, cuda):
    """Rows views build their own weight image; repeated calls agree."""
    rng = np.random.default_rng(11)
    p = wb.synth.random_packed(rng, 700, 512, 32, 4, "lloyd")
    m = wb.cq.New(p)
    x = rng.normal(size=(256, 512)).astype(np.float32)
    full = tc_gemm(wb, cuda, m, x)
    again = tc_gemm(wb, cuda, m, x)
    assert np.array_equal(full, again)
    for lo, hi in ((0, 128), (5, 300), (640, 700)):
        part = tc_gemm(wb, cuda, m.Rows(lo, hi), x)
        assert np.array_equal(part, full[:, lo:hi])


WC_GEMM_AUTO = 2


def tc_gemms(wb, cuda, ms, x, flags):
    rows = x.shape[0]
    lib = wb._lib.lib()
    xd = cuda.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    yds = [cuda.full((rows, m.Out()), float("nan"), dtype=cuda.float32, device="cuda") for m in ms]
    hs = (ctypes.c_void_p * len(ms))(*[m.handle.value for m in ms])
    ys = (ctypes.c_void_p * len(ms))(*[y.data_ptr() for y in yds])
    wb._lib.check(lib.wc_cq_gemms_ex(hs, len(ms), ctypes.c_void_p(xd.data_ptr()), ys, rows, flags, None))
    code = ctypes.c_int(-1)
    wb._lib.check(lib.wc_device_status(ctypes.byref(code)))
    assert code.value == 0, f"a bounded wait expired (code {code.value})"
    return [y.cpu().numpy() for y in yds]


@pytest.mark.parametrize("rows", [1, 96, 256, 1200])
def test_tc_gemms_grouped(wb, cuda, rows):
    """GEMMs on the tensor cores: Whistle's q/k/v/gate set (one rotation,
    one grouped launch), a second group size in the same call, and more
    matrices than one launch carries. Every output has the bits of its own
    wc_cq_gemm_ex call and stays within the fp16 bound."""
    rng = np.random.default_rng(40 + rows)
    in_ = 512
    ps = [wb.synth.random_packed(rng, o, in_, 128, 2, "lloyd") for o in (384, 96, 128, 512)]
    ps += [wb.synth.random_packed(rng, o, in_, 32, 4, "lloyd") for o in (200, 64)]
    ps += [wb.synth.random_packed(rng, 40 + 8 * k, in_, 128, 2, "lloyd") for k in range(14)]
    ms = [wb.cq.New(p) for p in ps]
    x = rng.normal(size=(rows, in_)).astype(np.float32)
    got = tc_gemms(wb, cuda, ms, x, WC_GEMM_TENSOR_CORES)
    for k, (p, m) in enumerate(zip(ps, ms)):
        single = tc_gemm(wb, cuda, m, x)
        assert np.array_equal(got[k].view(np.uint32), single.view(np.uint32)), k
        want, bound = refmath.tc_bound(p, x.astype(np.float64))
        assert np.all(np.abs(got[k] - want) <= bound), k


def auto_takes_tc(rows, outs):
    """WC_GEMM_AUTO's rule (include/whistle_b200.h): the tensor cores once
    rows x output rows reach 65,536, from 2 rows."""
    return rows >= 2 and rows * outs >= 65536


def test_auto_dispatch(wb, orc, cuda):
    """WC_GEMM_AUTO: the bit-exact lut kernels (the oracle's bits) below the
    crossover, the tensor cores (WC_GEMM_TENSOR_CORES's bits) past it."""
    rng = np.random.default_rng(77)
    ps = [wb.synth.random_packed(rng, o, 512, 128, 2, "lloyd") for o in (384, 96)]
    ps[1].Codebook = ps[0].Codebook
    ms = [wb.cq.New(p) for p in ps]
    for rows in (2, 8, 136, 137, 160):
        x = rng.normal(size=(rows, 512)).astype(np.float32)
        got = tc_gemms(wb, cuda, ms, x, WC_GEMM_AUTO)
        if not auto_takes_tc(rows, 384 + 96):
            for p, g in zip(ps, got):
                want = orc.gemm_lut(orc.OracleMatrix.of(p), x, rows)
                assert np.array_equal(g.view(np.uint32), want.view(np.uint32))
        else:
            tc = tc_gemms(wb, cuda, ms, x, WC_GEMM_TENSOR_CORES)
            for g, t in zip(got, tc):
                assert np.array_equal(g.view(np.uint32), t.view(np.uint32))


# BASELINE configs[2] at full size: 64 streams × 375 frames = 24,000 rows
# through the encoder's FFN up/down and fused QKV (4-bit, group 32), and
# Whistle's own q/k/v/gate set (2-bit, group 128) as one GEMMs call.
PREFILL = [("up", 2048, 512, 32, 4), ("down", 512, 2048, 32, 4), ("qkv", 1536, 512, 32, 4)]

# The reference's accept for its lut kernel (internal/cq/cq_test.go:196-254
# TestKernels: cosine >= 0.99999 against the float64 product), applied to
# every row of the tensor-core product.
TC_COSINE = 0.99999


def _rows_cosine(a, b):
    num = np.einsum("ij,ij->i", a, b)
    return num / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))


def _check_prefill(orc, p, x, got):
    want, bound = refmath.tc_bound(p, x.astype(np.float64))
    assert np.all(np.isfinite(got))
    assert np.all(np.abs(got - want) <= bound)
    cos = _rows_cosine(got.astype(np.float64), want)
    assert cos.min() >= TC_COSINE, f"worst row cosine {cos.min():.9f}"
    # Sampled rows against the oracle's lut product (the reference's own
    # kernel): the two differ by at most the tensor-core bound plus the lut
    # kernel's own distance to the float64 product.
    sample = np.arange(0, x.shape[0], x.shape[0] // 48)
    lut = orc.gemm_lut(orc.OracleMatrix.of(p), np.ascontiguousarray(x[sample]), len(sample))
    lut_err = np.abs(lut.astype(np.float64) - want[sample])
    assert np.all(np.abs(got[sample] - lut) <= bound[sample] + lut_err)
    assert _rows_cosine(got[sample].astype(np.float64), lut.astype(np.float64)).min() >= TC_COSINE


@pytest.mark.parametrize("case", PREFILL, ids=[c[0] for c in PREFILL])
def test_tc_gemm_configs2_full_size(wb, orc, cuda, case):
    _, out, in_, group, bits = case
    rng = np.random.default_rng(2000 + out + in_)
    p = wb.synth.random_packed(rng, out, in_, group, bits, "baseline")
    m = wb.cq.New(p)
    x = rng.normal(size=(24000, in_)).astype(np.float32)
    got = tc_gemm(wb, cuda, m, x)
    _check_prefill(orc, p, x, got)


def test_tc_gemms_configs2_whistle_qkvg(wb, orc, cuda):
    rng = np.random.default_rng(2100)
    ps = [wb.synth.random_packed(rng, o, 512, 128, 2, "lloyd") for o in (384, 96, 128, 512)]
    for q in ps[1:]:
        q.Codebook = ps[0].Codebook
    ms = [wb.cq.New(p) for p in ps]
    x = rng.normal(size=(24000, 512)).astype(np.float32)
    got = tc_gemms(wb, cuda, ms, x, WC_GEMM_TENSOR_CORES)
    for p, g in zip(ps, got):
        _check_prefill(orc, p, x, g)
