"""Pins the CPU oracle to the reference's own known answers and bounds.

The reference stores no output vectors for this path; its tests pin it with
literal cases, explicit float64 products and per-element error bounds. Each
test below restates one of them (file:line in the go-whistle module) and
runs it against the oracle, plus an independent numpy restatement of the
table arithmetic as a second check.
"""

from __future__ import annotations

import numpy as np
import pytest

import refmath

# internal/cq/cq_test.go:183 testShapes
TEST_SHAPES = [(1, 8, 8), (3, 16, 8), (4, 13, 8), (5, 40, 32), (7, 200, 128), (6, 384, 128), (9, 129, 128)]


def packed(orc, rng, out, in_, group, bits, codebook="reference"):
    import importlib

    synth = importlib.import_module("go-whistle_b200.synth")
    p = synth.random_packed(rng, out, in_, group, bits, codebook)
    return p, orc.OracleMatrix.of(p)


def test_fwht_matches_sylvester(orc):
    """cq_test.go:613 TestFWHT: fwht equals the explicit Sylvester product."""
    rng = np.random.default_rng(11)
    for n in (1, 2, 8, 128):
        x = (rng.integers(0, 17, n) - 8).astype(np.float32)
        want = (refmath.sylvester(n) @ x.astype(np.float64)).astype(np.float32)
        assert np.array_equal(orc.fwht(x), want), n
    # lut_amd64.s:20 fwhtAVX2 restated: the same bits as fwht (asm_test.go)
    import ctypes

    f = ctypes.POINTER(ctypes.c_float)
    for n in (8, 16, 32, 64, 128, 256, 1024):
        for trial in range(3):
            x = rng.normal(size=n).astype(np.float32) * np.float32(10.0 ** (trial - 1))
            y = x.copy()
            orc.lib().wo_fwht_avx2(y.ctypes.data_as(f), n)
            assert np.array_equal(y.view(np.uint32), orc.fwht(x).view(np.uint32)), n


def test_float16_known_answers(orc):
    """internal/cact/half_test.go:9 TestFloat16ToFloat32's table."""
    cases = {0x0000: 0.0, 0x3C00: 1.0, 0xBC00: -1.0, 0x3800: 0.5, 0x4000: 2.0, 0x7BFF: 65504.0,
             0x0400: 2.0 ** -14, 0x0001: 2.0 ** -24, 0x7C00: np.inf, 0xFC00: -np.inf, 0x0200: 2.0 ** -15}
    for h, want in cases.items():
        assert orc.f16_to_f32(h) == want, hex(h)
    assert np.signbit(orc.f16_to_f32(0x8000)) and orc.f16_to_f32(0x8000) == 0.0
    assert np.isnan(orc.f16_to_f32(0x7E00))
    # every finite code agrees with numpy's binary16
    for h in range(0, 0x10000, 7):
        f = np.array([h], np.uint16).view(np.float16).astype(np.float32)[0]
        g = orc.f16_to_f32(h)
        assert (np.isnan(f) and np.isnan(g)) or np.float32(g) == f, hex(h)


def test_quantize_row_known_answers(orc):
    """internal/needle/int8_test.go:16 TestQuantizeRow."""
    q, s = orc.quantize_row(np.array([127, 2.5, -2.5, 3.5, -0.5, 1.4999], np.float32))
    assert s == 1 and list(q) == [127, 2, -2, 4, 0, 1]  # ties to even
    q, s = orc.quantize_row(np.array([-6.35, 0.05, 3], np.float32))
    assert s == np.float32(6.35) / np.float32(127) and list(q) == [-127, 1, 60]
    q, s = orc.quantize_row(np.zeros(4, np.float32))
    assert s == 1 and list(q) == [0, 0, 0, 0]
    rng = np.random.default_rng(1)
    for n in (1, 7, 48, 64, 2048):
        for scale in (1e-6, 1.0, 1e4):
            x = (rng.normal(size=n) * scale).astype(np.float32)
            x[rng.integers(n)] *= 9
            q, s = orc.quantize_row(x)
            m = np.max(np.abs(x))
            assert s == np.float32(m) / np.float32(127)
            d = np.abs(x.astype(np.float64) - np.float64(s) * q.astype(np.float64))
            assert np.all(d <= np.float64(s) * 0.5000001) and q.min() >= -127


def numpy_tables(bits, x, cb, cb_max):
    """An independent numpy restatement of lut.go:239-282 (float32 ops, rint)."""
    x = np.asarray(x, np.float32)
    cb = np.asarray(cb, np.float32)
    if bits == 4:
        mx = np.max(np.abs(x)) if x.size else np.float32(0)
    else:
        mx = np.max(np.abs(x[0::2]) + np.abs(x[1::2]))
    m = np.float32(cb_max) * np.float32(mx)
    inv = np.float32(8191) / m if m > 0 else np.float32(0)
    c = np.arange(16)
    if bits == 4:
        a = x * inv
        e = cb[None, :] * a[:, None]
    else:
        a, b = x[0::2] * inv, x[1::2] * inv
        e = (cb[c & 3][None, :] * a[:, None]) + (cb[c >> 2][None, :] * b[:, None])
    return np.float32(m), np.rint(e.astype(np.float32)).astype(np.int32)


@pytest.mark.parametrize("bits", [2, 4])
def test_lut_tables(orc, bits):
    """asm_test.go:61 TestLUTTablesMatchGeneric's cases: groups 8..256, an
    all-zero group (M = 0) and heavy tails; planes and integers agree."""
    rng = np.random.default_rng(23)
    for n in (8, 16, 32, 64, 128, 256):
        for trial in range(4):
            cb = np.sort(rng.normal(size=1 << bits)).astype(np.float32)
            cb_max = np.float32(np.max(np.abs(cb)))
            x = rng.normal(size=n)
            if trial == 3:
                x = x ** 3
            x[rng.integers(0, 16, n) == 0] = 0
            x = x.astype(np.float32)
            if trial == 0:
                x[:] = 0
            m, planes = orc.lut_tables_planes(bits, x, cb, cb_max)
            m2, ints = orc.lut_tables_int(bits, x, cb, cb_max)
            # lut_amd64.s:127/184 lutTables2AVX2/lutTables4AVX2 restated: the same planes
            import ctypes

            planes2 = np.zeros_like(planes)
            m3 = orc.lib().wo_lut_tables_planes_avx2(bits, planes2.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
                                                     x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), n,
                                                     cb.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                                     float(cb_max))
            assert np.float32(m3) == m and np.array_equal(planes2, planes), (n, trial)
            mn, vn = numpy_tables(bits, x, cb, cb_max)
            assert m == m2 == mn
            assert np.array_equal(ints.astype(np.int32), vn)
            assert np.all(np.abs(vn) <= 8191)
            pl = planes.reshape(-1, 2, 16).astype(np.int32)
            assert pl.min() >= 0 and pl.max() <= 127
            assert np.array_equal(pl[:, 0] + 128 * (pl[:, 1] - 64), vn)
            if trial == 0:
                assert m == 0 and np.all(vn == 0)


def test_lut_lookup_blocked(orc):
    """asm_test.go:114 TestLUTLookupMatchesGeneric's shapes, including all
    planes at 127: the blocked lookup equals an integer-table restatement."""
    rng = np.random.default_rng(25)
    for gb in (1, 2, 3, 4, 8, 16, 32, 64, 256):
        for groups in (1, 2, 5):
            for blocks in (1, 2, 3):
                full = gb == 256 and groups == 1
                idx = rng.integers(0, 256, blocks * groups * gb * 32, dtype=np.uint8)
                tab = np.full(64 * groups * gb, 127, np.uint8) if full else \
                    rng.integers(0, 128, 64 * groups * gb, dtype=np.uint8)
                norm = rng.normal(size=blocks * groups * 32).astype(np.float32)
                steps = rng.normal(size=groups).astype(np.float32)
                y = np.zeros(blocks * 32, np.float32)
                import ctypes

                L = orc.lib()
                f = ctypes.POINTER(ctypes.c_float)
                u = ctypes.POINTER(ctypes.c_uint8)
                L.wo_lut_lookup_blocked(y.ctypes.data_as(f), idx.ctypes.data_as(u), tab.ctypes.data_as(u),
                                        norm.ctypes.data_as(f), steps.ctypes.data_as(f), blocks, groups, gb)
                t = tab.reshape(-1, 4, 16).astype(np.int64)  # per byte: lo(lo), hi(lo), lo(hi), hi(hi)
                v = t[:, 0, :][:, :, None] + t[:, 2, :][:, None, :] + 128 * (
                    t[:, 1, :][:, :, None] + t[:, 3, :][:, None, :] - 128)  # [byte][lo][hi]
                want = np.zeros(blocks * 32, np.float32)
                I = idx.reshape(blocks, groups * gb, 32)
                for b in range(blocks):
                    for g in range(groups):
                        js = np.arange(g * gb, (g + 1) * gb)
                        codes = I[b, js, :]
                        s = v[js[:, None], codes & 15, codes >> 4].sum(axis=0)
                        coef = norm.reshape(blocks, groups, 32)[b, g] * steps[g]
                        want[b * 32:(b + 1) * 32] = want[b * 32:(b + 1) * 32] + (s.astype(np.float32) * coef)
                assert np.array_equal(y, want), (gb, groups, blocks)
                # lut_amd64.s:236 lutLookupAVX2 restated: the same bits (asm_test.go)
                y2 = np.full(blocks * 32, np.nan, np.float32)
                L.wo_lut_lookup_blocked_avx2(y2.ctypes.data_as(f), idx.ctypes.data_as(u), tab.ctypes.data_as(u),
                                             norm.ctypes.data_as(f), steps.ctypes.data_as(f), blocks, groups, gb)
                assert np.array_equal(y2.view(np.uint32), y.view(np.uint32)), (gb, groups, blocks)


@pytest.mark.parametrize("shape", TEST_SHAPES)
@pytest.mark.parametrize("bits", [2, 4])
def test_kernels_within_reference_bounds(orc, shape, bits):
    """cq_test.go:196 TestKernels: lut, nibble4/nibble (Exact) and gather
    within rotatedBound (+ lutBound for lut) of the float64 product, and by
    cosine 0.999999 (0.99999 for lut)."""
    out, in_, group = shape
    rng = np.random.default_rng(1000 + out * 7 + bits)
    p, m = packed(orc, rng, out, in_, group, bits)
    w = refmath.dequant64(p)
    rows = 6
    x = rng.normal(size=rows * in_).astype(np.float32)
    for name, fn in (("lut", orc.gemm_lut), ("exact", orc.gemm_exact), ("gather", orc.gemm_gather)):
        got = fn(m, x, rows)
        for i in range(rows):
            xi = x[i * in_:(i + 1) * in_]
            bound = refmath.rotated_bound(p, xi)
            min_cos = 0.999999
            if name == "lut":
                bound = bound + refmath.lut_bound(p, xi)
                min_cos = 0.99999
            want = w @ xi.astype(np.float64)
            assert np.all(np.abs(got[i].astype(np.float64) - want) <= bound), name
            assert refmath.cosine(got[i], want) >= min_cos, name


def test_gemm_rows_independent(orc):
    """cq_test.go:260 TestGEMMRows: reversing the activations reverses the
    result bit for bit."""
    rng = np.random.default_rng(3)
    p, m = packed(orc, rng, 33, 256, 128, 2)
    x = rng.normal(size=(4, 256)).astype(np.float32)
    a = orc.gemm_lut(m, x, 4)
    b = orc.gemm_lut(m, x[::-1].copy(), 4)
    assert np.array_equal(a, b[::-1])


# parallel_test.go:29 parallelShapes
PARALLEL_SHAPES = [(384, 512, 128, 2, 375), (1024, 512, 128, 2, 101), (128, 2048, 128, 4, 375),
                   (8199, 512, 128, 4, 1), (8199, 512, 128, 4, 5), (4133, 300, 64, 2, 1), (1031, 200, 32, 4, 37)]


@pytest.mark.parametrize("sh", PARALLEL_SHAPES)
def test_workers_invariance(orc, sh):
    """parallel_test.go:45 TestGEMMWorkers: 1, 2, 5 and 16 threads give the
    bits of the unsplit reference."""
    out, in_, group, bits, rows = sh
    rng = np.random.default_rng(38)
    p, m = packed(orc, rng, out, in_, group, bits)
    x = rng.normal(size=rows * in_).astype(np.float32)
    want = orc.gemm_lut(m, x, rows, threads=1)
    for w in (2, 5, 16):
        assert np.array_equal(orc.gemm_lut(m, x, rows, threads=w), want), w


def test_gemms_matches_gemm(orc):
    """parallel_test.go:101 TestGEMMsMatchesGEMM: shared tables give each
    matrix's own GEMM bit for bit."""
    rng = np.random.default_rng(382)
    mats = [packed(orc, rng, o, 512, 128, 2)[1] for o in (384, 96, 128, 512)]
    cb = mats[0].cb
    for mm in mats[1:]:
        mm.cb[:] = cb  # one codebook per width, as whistle.cact has
    for rows in (1, 3, 8):
        x = rng.normal(size=rows * 512).astype(np.float32)
        got = orc.gemms_lut(mats, x, rows)
        for mm, g in zip(mats, got):
            assert np.array_equal(g, orc.gemm_lut(mm, x, rows))


@pytest.mark.parametrize("shape", TEST_SHAPES)
@pytest.mark.parametrize("bits", [2, 4])
def test_row(orc, shape, bits):
    """cq_test.go:335 TestRow: Row against the float64 dequantisation."""
    out, in_, group = shape
    rng = np.random.default_rng(5 + out)
    p, m = packed(orc, rng, out, in_, group, bits)
    w = refmath.dequant64(p)
    for r in range(out):
        assert refmath.cosine(orc.row(m, r), w[r]) >= 0.9999999


def test_attend_int8_matches_float(orc):
    """int8_test.go:212 TestAttendInt8MatchesFloat: GQA 8/2, qk 48, v 64,
    37 keys, causal and full, quantQ on and off: probabilities and outputs
    within 2e-6 of the float attention on the codes' values, probabilities
    summing to 1 within 1e-5."""
    heads, kvh, qk, vd, n, rows = 8, 2, 48, 64, 37, 3
    rng = np.random.default_rng(9)
    q = rng.normal(size=rows * heads * qk).astype(np.float32)
    k8, ks = orc.quantize_rows(rng.normal(size=n * kvh * qk).astype(np.float32), kvh * qk, qk)
    v8, vs = orc.quantize_rows(rng.normal(size=n * kvh * vd).astype(np.float32), kvh * vd, vd)
    kf = (k8.astype(np.float32) * np.repeat(ks, qk)).reshape(n, kvh, qk)
    vf = (v8.astype(np.float32) * np.repeat(vs, vd)).reshape(n, kvh, vd)
    scale = np.float32(np.sqrt(qk))
    for causal in (False, True):
        keys = (lambda i: n - rows + i + 1) if causal else (lambda i: n)
        for quant_q in (True, False):
            out, probs = orc.attend_int8(q, rows, heads, k8, ks, v8, vs, n, kvh, qk, vd, keys, scale, quant_q,
                                         want_probs=True)
            qq = q.copy()
            if quant_q:
                for c in range(rows * heads):
                    qc, sc = orc.quantize_row(q[c * qk:(c + 1) * qk])
                    qq[c * qk:(c + 1) * qk] = qc.astype(np.float32) * sc
            for i in range(rows):
                for h in range(heads):
                    kv = h // (heads // kvh)
                    nk = keys(i)
                    s = np.array([np.float32(np.dot(qq[(i * heads + h) * qk:(i * heads + h + 1) * qk].astype(
                        np.float64), kf[j, kv].astype(np.float64))) / scale for j in range(nk)], np.float32)
                    p = orc.softmax(s)
                    got = probs[(i * heads + h) * n:(i * heads + h) * n + nk]
                    assert np.max(np.abs(p - got)) <= 2e-6
                    assert abs(got.astype(np.float64).sum() - 1) <= 1e-5
                    want = (p.astype(np.float64)[:, None] * vf[:nk, kv].astype(np.float64)).sum(axis=0)
                    assert np.max(np.abs(out[(i * heads + h) * vd:(i * heads + h + 1) * vd] - want)) <= 2e-6


def test_int8_dots_extreme(orc):
    """int8_test.go:149: -128 · -128 is the largest product; dots are exact."""
    heads, kvh, qk, vd, n = 1, 1, 16, 16, 5
    rng = np.random.default_rng(7)
    k8 = rng.integers(-128, 128, n * qk, dtype=np.int8)
    k8[0] = -128
    ks = np.ones(n, np.float32)
    v8 = rng.integers(-128, 128, n * vd, dtype=np.int8)
    vs = np.ones(n, np.float32)
    q = np.full(qk, -1.0, np.float32)  # quantises to all -127
    out, probs = orc.attend_int8(q, 1, heads, k8, ks, v8, vs, n, kvh, qk, vd, lambda i: n, np.float32(1), True,
                                 want_probs=True)
    q8, sq = orc.quantize_row(q)
    dots = (k8.reshape(n, qk).astype(np.int64) * q8.astype(np.int64)).sum(axis=1)
    logits = np.array([np.float32(np.float32(d) * (sq * np.float32(1))) / np.float32(1) for d in dots], np.float32)
    assert np.array_equal(probs, orc.softmax(logits))
