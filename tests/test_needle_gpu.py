"""int8 quantiser and int8 KV-cache attention on the GPU through the C ABI,
against the oracle's restatement of the reference's generic path."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def bits_eq(a, b) -> bool:
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    if a.dtype == np.float32:
        a, b = a.view(np.uint32), np.ascontiguousarray(b, np.float32).view(np.uint32)
    return a.shape == b.shape and np.array_equal(a, b)


def dp(t):
    return ctypes.c_void_p(t.data_ptr())


def test_quantize_row_known_answers(wb, cuda):
    """int8_test.go:16 TestQuantizeRow's literal cases on the GPU."""
    q = np.zeros(6, np.int8)
    s = wb.needle.QuantizeRow(q, np.array([127, 2.5, -2.5, 3.5, -0.5, 1.4999], np.float32))
    assert s == 1 and list(q) == [127, 2, -2, 4, 0, 1]
    s = wb.needle.QuantizeRow(q[:3], np.array([-6.35, 0.05, 3], np.float32))
    assert s == np.float32(6.35) / np.float32(127) and list(q[:3]) == [-127, 1, 60]
    s = wb.needle.QuantizeRow(q[:4], np.zeros(4, np.float32))
    assert s == 1 and list(q[:4]) == [0, 0, 0, 0]


@pytest.mark.parametrize("width", [8, 17, 48, 64, 128, 2048])
def test_quantize_rows_bit_exact(wb, orc, cuda, width):
    rng = np.random.default_rng(width)
    for scale in (1e-6, 1.0, 1e4):
        cols = width * 3
        x = (rng.normal(size=5 * cols) * scale).astype(np.float32)
        x[rng.integers(x.size)] *= 9
        x[:width] = 0  # a zero chunk: scale 1
        r = wb.needle.QuantizeRows(x, cols, width)
        q, s = orc.quantize_rows(x, cols, width)
        assert bits_eq(r.Q, q) and bits_eq(r.S, s)
        # device form, as a KV-cache append at an offset
        xd = cuda.from_numpy(x).cuda()
        qd = cuda.zeros(x.size + 7, dtype=cuda.int8, device="cuda")
        sd = cuda.zeros(s.size + 3, dtype=cuda.float32, device="cuda")
        wb._lib.check(wb._lib.lib().wc_quantize_rows(dp(xd), 5, cols, width, ctypes.c_void_p(qd.data_ptr() + 7),
                                                     ctypes.c_void_p(sd.data_ptr() + 12), None))
        assert bits_eq(qd.cpu().numpy()[7:], q) and bits_eq(sd.cpu().numpy()[3:], s)


def kv(wb, orc, rng, n, kvh, width, quantized_from_float=True):
    if quantized_from_float:
        return orc.quantize_rows(rng.normal(size=n * kvh * width).astype(np.float32), kvh * width, width)
    return wb.synth.random_kv(rng, n, kvh, width)


# (heads, kv_heads, qk, vd, keys): Whistle self-attention (GQA 8/2, qk 48,
# v 64, 1..224 keys), cross-attention (8/8 over 375 frames), the benchmark's
# 8 x 64/64 heads, and odd widths the byte path takes.
GEOMS = [(8, 2, 48, 64, 1), (8, 2, 48, 64, 37), (8, 2, 48, 64, 224), (8, 8, 48, 64, 375), (8, 8, 64, 64, 160),
         (4, 1, 17, 9, 33), (2, 2, 16, 32, 5)]


@pytest.mark.parametrize("geom", GEOMS, ids=[f"h{g[0]}kv{g[1]}qk{g[2]}v{g[3]}n{g[4]}" for g in GEOMS])
@pytest.mark.parametrize("quant_q", [True, False])
def test_attend_bit_exact(wb, orc, cuda, geom, quant_q):
    heads, kvh, qk, vd, n = geom
    rng = np.random.default_rng(sum(geom) + quant_q)
    rows = 3 if n >= 3 else 1
    q = rng.normal(size=rows * heads * qk).astype(np.float32)
    k8, ks = kv(wb, orc, rng, n, kvh, qk, rng.random() < 0.5)
    v8, vs = kv(wb, orc, rng, n, kvh, vd, rng.random() < 0.5)
    scale = np.float32(np.sqrt(qk))
    # causal rows, a sink + window pair of spans, and the full key range
    spans = np.array([[0, min(2, n), max(min(2, n), n - 5 - i), n - rows + i + 1] for i in range(rows)], np.int32)
    spans[:, 2] = np.minimum(spans[:, 2], spans[:, 3])
    for sp in (spans, np.array([[0, 0, 0, n]] * rows, np.int32)):
        want, wprobs = orc.attend_int8_spans(q, rows, heads, k8, ks, v8, vs, n, kvh, qk, vd, sp, scale, quant_q,
                                             want_probs=True)
        D = lambda a: cuda.from_numpy(np.ascontiguousarray(a)).cuda()
        qd, k8d, ksd, v8d, vsd, spd = D(q), D(k8), D(ks), D(v8), D(vs), D(sp.reshape(-1))
        out = cuda.zeros(rows * heads * vd, dtype=cuda.float32, device="cuda")
        probs = cuda.zeros(rows * heads * n, dtype=cuda.float32, device="cuda")
        wb._lib.check(wb._lib.lib().wc_attend_int8(dp(qd), rows, heads, dp(k8d), dp(ksd), dp(v8d), dp(vsd), n, kvh,
                                                   qk, vd, dp(spd), float(scale), int(quant_q), dp(probs), dp(out),
                                                   None))
        got = out.cpu().numpy()
        assert bits_eq(got, want), np.max(np.abs(got - want))
        assert bits_eq(probs.cpu().numpy(), wprobs)


def test_attend_host_mirror_matches_float(wb, orc, cuda):
    """int8_test.go:212 TestAttendInt8MatchesFloat through the host mirror,
    and equal to the oracle bit for bit."""
    heads, kvh, qk, vd, n, rows = 8, 2, 48, 64, 37, 3
    rng = np.random.default_rng(9)
    q = rng.normal(size=rows * heads * qk).astype(np.float32)
    k = wb.needle.QuantizeRows(rng.normal(size=n * kvh * qk).astype(np.float32), kvh * qk, qk)
    v = wb.needle.QuantizeRows(rng.normal(size=n * kvh * vd).astype(np.float32), kvh * vd, vd)
    scale = np.float32(np.sqrt(qk))
    for causal in (False, True):
        keys = (lambda i: n - rows + i + 1) if causal else (lambda i: n)
        for quant_q in (True, False):
            probs = np.zeros(rows * heads * n, np.float32)
            got = wb.needle.AttendInt8(q, rows, heads, k, v, keys, scale, quant_q, probs)
            want, wprobs = orc.attend_int8(q, rows, heads, k.Q, k.S, v.Q, v.S, n, kvh, qk, vd, keys, scale, quant_q,
                                           want_probs=True)
            assert bits_eq(got, want) and bits_eq(probs, wprobs)
            for i in range(rows):
                for h in range(heads):
                    p = probs[(i * heads + h) * n:(i * heads + h) * n + keys(i)]
                    assert abs(p.astype(np.float64).sum() - 1) <= 1e-5


@pytest.mark.parametrize("geom", [(8, 2, 48, 64, 224), (8, 8, 48, 64, 375), (8, 8, 64, 64, 224)])
def test_attend_streams(wb, orc, cuda, geom):
    """The decode step of many streams, each against its own cache."""
    heads, kvh, qk, vd, cap = geom
    streams = 64
    rng = np.random.default_rng(cap)
    nk = rng.integers(1, cap + 1, streams).astype(np.int32)
    nk[0], nk[1] = cap, 1
    q = rng.normal(size=streams * heads * qk).astype(np.float32)
    k8, ks = wb.synth.random_kv(rng, streams * cap, kvh, qk)
    v8, vs = wb.synth.random_kv(rng, streams * cap, kvh, vd)
    scale = np.float32(np.sqrt(qk))
    want = orc.attend_streams(q, heads, k8, ks, v8, vs, cap, nk, kvh, qk, vd, scale, threads=8)
    D = lambda a: cuda.from_numpy(np.ascontiguousarray(a)).cuda()
    qd, k8d, ksd, v8d, vsd, nkd = D(q), D(k8), D(ks), D(v8), D(vs), D(nk)  # held until the kernel has run
    out = cuda.zeros(streams * heads * vd, dtype=cuda.float32, device="cuda")
    wb._lib.check(wb._lib.lib().wc_attend_int8_streams(streams, dp(qd), heads, dp(k8d), dp(ksd), dp(v8d), dp(vsd),
                                                       cap, dp(nkd), kvh, qk, vd, float(scale), 1, dp(out), None))
    assert bits_eq(out.cpu().numpy(), want)


WC_ATTEND_QUANT_Q, WC_ATTEND_ANY_ORDER = 1, 2
# The north star's tolerance for the float results of the attention: the
# any-order kernel (float sums reordered, FMA, expf) must stay within 1e-5
# relative of the reference's order; the integer work (query codes, int32
# logits) is exact either way.
ANY_ORDER_RTOL = 1e-5


@pytest.mark.parametrize("geom", GEOMS, ids=[f"h{g[0]}kv{g[1]}qk{g[2]}v{g[3]}n{g[4]}" for g in GEOMS])
@pytest.mark.parametrize("quant_q", [True, False])
def test_attend_any_order_within_tolerance(wb, orc, cuda, geom, quant_q):
    heads, kvh, qk, vd, n = geom
    rng = np.random.default_rng(7 * sum(geom) + quant_q)
    rows = 3 if n >= 3 else 1
    q = rng.normal(size=rows * heads * qk).astype(np.float32)
    k8, ks = kv(wb, orc, rng, n, kvh, qk)
    v8, vs = kv(wb, orc, rng, n, kvh, vd, False)
    scale = np.float32(np.sqrt(qk))
    spans = np.array([[0, min(2, n), max(min(2, n), n - 5 - i), n - rows + i + 1] for i in range(rows)], np.int32)
    spans[:, 2] = np.minimum(spans[:, 2], spans[:, 3])
    want, wprobs = orc.attend_int8_spans(q, rows, heads, k8, ks, v8, vs, n, kvh, qk, vd, spans, scale, quant_q,
                                         want_probs=True)
    D = lambda a: cuda.from_numpy(np.ascontiguousarray(a)).cuda()
    qd, k8d, ksd, v8d, vsd, spd = D(q), D(k8), D(ks), D(v8), D(vs), D(spans.reshape(-1))
    out = cuda.zeros(rows * heads * vd, dtype=cuda.float32, device="cuda")
    probs = cuda.zeros(rows * heads * n, dtype=cuda.float32, device="cuda")
    flags = WC_ATTEND_ANY_ORDER | (WC_ATTEND_QUANT_Q if quant_q else 0)
    wb._lib.check(wb._lib.lib().wc_attend_int8(dp(qd), rows, heads, dp(k8d), dp(ksd), dp(v8d), dp(vsd), n, kvh, qk,
                                               vd, dp(spd), float(scale), flags, dp(probs), dp(out), None))
    got = out.cpu().numpy().reshape(rows * heads, vd)
    want = want.reshape(rows * heads, vd)
    scale_row = np.maximum(np.abs(want).max(axis=1, keepdims=True), 1e-30)
    assert np.all(np.abs(got - want) <= ANY_ORDER_RTOL * scale_row)
    gp = probs.cpu().numpy()
    assert np.all(np.abs(gp - wprobs) <= ANY_ORDER_RTOL * np.maximum(np.abs(wprobs), 1e-3))


@pytest.mark.parametrize("geom", [(8, 2, 48, 64, 224), (8, 8, 48, 64, 375), (8, 8, 64, 64, 224)])
def test_attend_streams_any_order(wb, orc, cuda, geom):
    heads, kvh, qk, vd, cap = geom
    streams = 64
    rng = np.random.default_rng(cap + 1)
    nk = rng.integers(1, cap + 1, streams).astype(np.int32)
    nk[0], nk[1] = cap, 1
    q = rng.normal(size=streams * heads * qk).astype(np.float32)
    k8, ks = wb.synth.random_kv(rng, streams * cap, kvh, qk)
    v8, vs = wb.synth.random_kv(rng, streams * cap, kvh, vd)
    scale = np.float32(np.sqrt(qk))
    want = orc.attend_streams(q, heads, k8, ks, v8, vs, cap, nk, kvh, qk, vd, scale, threads=8)
    D = lambda a: cuda.from_numpy(np.ascontiguousarray(a)).cuda()
    qd, k8d, ksd, v8d, vsd, nkd = D(q), D(k8), D(ks), D(v8), D(vs), D(nk)
    out = cuda.zeros(streams * heads * vd, dtype=cuda.float32, device="cuda")
    wb._lib.check(wb._lib.lib().wc_attend_int8_streams(streams, dp(qd), heads, dp(k8d), dp(ksd), dp(v8d), dp(vsd),
                                                       cap, dp(nkd), kvh, qk, vd, float(scale),
                                                       WC_ATTEND_QUANT_Q | WC_ATTEND_ANY_ORDER, dp(out), None))
    got = out.cpu().numpy().reshape(-1, vd)
    want = want.reshape(-1, vd)
    scale_row = np.maximum(np.abs(want).max(axis=1, keepdims=True), 1e-30)
    assert np.all(np.abs(got - want) <= ANY_ORDER_RTOL * scale_row)
