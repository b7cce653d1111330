"""The bulk-copy attention kernel (one query row per stream over all of its
keys, cache rows staged in shared memory by cp.async.bulk), against the
oracle's restatement of AttendInt8Spans (internal/needle/int8.go:194-285):
bit for bit in the reference's order, within 1e-5 relative with
WC_ATTEND_ANY_ORDER. These calls (t = 1, no spans, no probabilities,
16-byte aligned rows) are the ones the kernel serves."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WC_ATTEND_QUANT_Q, WC_ATTEND_ANY_ORDER = 1, 2
ANY_ORDER_RTOL = 1e-5  # the any-order tolerance the other attention tests state

# (heads, kv_heads, qk, vd, cap): Whistle self (GQA 8/2) and cross (8/8 x 375)
# attention, the benchmark's 64/64 heads, one KV head for 8 query heads,
# wide heads (several 4-column groups per thread), and caps at, below and
# just above the 32-key chunk.
GEOMS = [(8, 2, 48, 64, 224), (8, 8, 48, 64, 375), (8, 8, 64, 64, 160), (8, 1, 16, 16, 33), (16, 16, 128, 128, 64),
         (32, 4, 64, 128, 100), (2, 2, 16, 32, 5), (8, 8, 48, 64, 32), (4, 2, 32, 48, 65)]


def dp(t):
    return ctypes.c_void_p(t.data_ptr())


def bits_eq(a, b) -> bool:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def oracle_streams(orc, q, heads, k8, ks, v8, vs, cap, nk, kvh, qk, vd, scale, quant_q):
    out = []
    for b, n in enumerate(nk):
        sl = slice(b * cap, b * cap + int(n))
        o, _ = orc.attend_int8_spans(q[b * heads * qk:(b + 1) * heads * qk], 1, heads,
                                     k8.reshape(-1, kvh * qk)[sl], ks.reshape(-1, kvh)[sl],
                                     v8.reshape(-1, kvh * vd)[sl], vs.reshape(-1, kvh)[sl], int(n), kvh, qk, vd,
                                     np.array([[0, 0, 0, int(n)]], np.int32), scale, quant_q)
        out.append(o)
    return np.concatenate(out)


@pytest.mark.parametrize("geom", GEOMS, ids=[f"h{g[0]}kv{g[1]}qk{g[2]}v{g[3]}c{g[4]}" for g in GEOMS])
@pytest.mark.parametrize("quant_q", [True, False], ids=["qq", "fq"])
@pytest.mark.parametrize("any_order", [False, True], ids=["exact", "any"])
def test_attend_streams_bulk(wb, orc, cuda, geom, quant_q, any_order):
    heads, kvh, qk, vd, cap = geom
    streams = 40
    rng = np.random.default_rng(sum(geom) * 4 + 2 * quant_q + any_order)
    nk = rng.integers(0, cap + 1, streams).astype(np.int32)
    nk[0], nk[1], nk[2], nk[3] = cap, 0, 1, min(32, cap)
    q = rng.normal(size=streams * heads * qk).astype(np.float32)
    k8, ks = wb.synth.random_kv(rng, streams * cap, kvh, qk)
    v8, vs = wb.synth.random_kv(rng, streams * cap, kvh, vd)
    scale = np.float32(np.sqrt(qk))
    want = oracle_streams(orc, q, heads, k8, ks, v8, vs, cap, nk, kvh, qk, vd, scale, quant_q)
    D = lambda a: cuda.from_numpy(np.ascontiguousarray(a)).cuda()
    qd, k8d, ksd, v8d, vsd, nkd = D(q), D(k8), D(ks), D(v8), D(vs), D(nk)
    out = cuda.full((streams * heads * vd,), float("nan"), dtype=cuda.float32, device="cuda")
    flags = (WC_ATTEND_QUANT_Q if quant_q else 0) | (WC_ATTEND_ANY_ORDER if any_order else 0)
    wb._lib.check(wb._lib.lib().wc_attend_int8_streams(streams, dp(qd), heads, dp(k8d), dp(ksd), dp(v8d), dp(vsd),
                                                       cap, dp(nkd), kvh, qk, vd, float(scale), flags, dp(out), None))
    code = ctypes.c_int(-1)
    wb._lib.check(wb._lib.lib().wc_device_status(ctypes.byref(code)))
    assert code.value == 0
    got = out.cpu().numpy()
    if not any_order:
        assert bits_eq(got, want), np.max(np.abs(got - want))
    else:
        g, w = got.reshape(-1, vd), want.reshape(-1, vd)
        scale_row = np.maximum(np.abs(w).max(axis=1, keepdims=True), 1e-30)
        assert np.all(np.abs(g - w) <= ANY_ORDER_RTOL * scale_row)
    # a stream without keys attends to nothing
    assert np.all(got.reshape(streams, -1)[1] == 0)


@pytest.mark.parametrize("any_order", [False, True], ids=["exact", "any"])
def test_attend_decode_row_bulk(wb, orc, cuda, any_order):
    """AttendInt8 with one query row over every key (no spans, no
    probabilities) takes the bulk kernel with a single stream."""
    heads, kvh, qk, vd, n = 8, 8, 48, 64, 375
    rng = np.random.default_rng(11 + any_order)
    q = rng.normal(size=heads * qk).astype(np.float32)
    k8, ks = wb.synth.random_kv(rng, n, kvh, qk)
    v8, vs = wb.synth.random_kv(rng, n, kvh, vd)
    scale = np.float32(np.sqrt(qk))
    want, _ = orc.attend_int8_spans(q, 1, heads, k8, ks, v8, vs, n, kvh, qk, vd, np.array([[0, 0, 0, n]], np.int32),
                                    scale, True)
    D = lambda a: cuda.from_numpy(np.ascontiguousarray(a)).cuda()
    qd, k8d, ksd, v8d, vsd = D(q), D(k8), D(ks), D(v8), D(vs)
    out = cuda.zeros(heads * vd, dtype=cuda.float32, device="cuda")
    flags = WC_ATTEND_QUANT_Q | (WC_ATTEND_ANY_ORDER if any_order else 0)
    wb._lib.check(wb._lib.lib().wc_attend_int8(dp(qd), 1, heads, dp(k8d), dp(ksd), dp(v8d), dp(vsd), n, kvh, qk, vd,
                                               None, float(scale), flags, None, dp(out), None))
    got = out.cpu().numpy()
    if not any_order:
        assert bits_eq(got, want)
    else:
        g, w = got.reshape(-1, vd), want.reshape(-1, vd)
        assert np.all(np.abs(g - w) <= ANY_ORDER_RTOL * np.maximum(np.abs(w).max(axis=1, keepdims=True), 1e-30))


def test_attend_streams_bulk_unaligned_falls_back(wb, orc, cuda):
    """Caches that do not start on a 16-byte boundary take the other
    kernels, with the same bits."""
    heads, kvh, qk, vd, cap, streams = 8, 2, 48, 64, 50, 8
    rng = np.random.default_rng(23)
    nk = rng.integers(1, cap + 1, streams).astype(np.int32)
    q = rng.normal(size=streams * heads * qk).astype(np.float32)
    k8, ks = wb.synth.random_kv(rng, streams * cap, kvh, qk)
    v8, vs = wb.synth.random_kv(rng, streams * cap, kvh, vd)
    scale = np.float32(np.sqrt(qk))
    want = oracle_streams(orc, q, heads, k8, ks, v8, vs, cap, nk, kvh, qk, vd, scale, True)
    D = lambda a: cuda.from_numpy(np.ascontiguousarray(a)).cuda()
    qd, ksd, vsd, nkd = D(q), D(ks), D(vs), D(nk)
    k8buf = cuda.zeros(k8.size + 4, dtype=cuda.int8, device="cuda")
    v8buf = cuda.zeros(v8.size + 4, dtype=cuda.int8, device="cuda")
    k8buf[4:] = cuda.from_numpy(k8.reshape(-1)).cuda()
    v8buf[4:] = cuda.from_numpy(v8.reshape(-1)).cuda()
    out = cuda.zeros(streams * heads * vd, dtype=cuda.float32, device="cuda")
    wb._lib.check(wb._lib.lib().wc_attend_int8_streams(
        streams, dp(qd), heads, ctypes.c_void_p(k8buf.data_ptr() + 4), dp(ksd), ctypes.c_void_p(v8buf.data_ptr() + 4),
        dp(vsd), cap, dp(nkd), kvh, qk, vd, float(scale), WC_ATTEND_QUANT_Q, dp(out), None))
    assert bits_eq(out.cpu().numpy(), want)
