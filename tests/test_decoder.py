"""The decoder head's scale and greedy argmax (internal/decoder/decoder.go:
508-523, greedy.go:182): the oracle against a direct restatement of the Go
loop on the CPU, then the CUDA kernel against the oracle bit for bit."""

from __future__ import annotations

import numpy as np
import pytest


def go_argmax(v) -> int:
    """greedy.go:182 argmax: best = 0, moved only on x > v[best]."""
    best = 0
    for i, x in enumerate(v):
        if x > v[best]:
            best = i
    return best


def same_floats(a, b) -> bool:
    """Bit for bit, except that any NaN matches any NaN (a product's NaN
    payload is the hardware's, not part of the arithmetic)."""
    a = np.ascontiguousarray(a, np.float32).reshape(-1)
    b = np.ascontiguousarray(b, np.float32).reshape(-1)
    na, nb = np.isnan(a), np.isnan(b)
    return a.shape == b.shape and np.array_equal(na, nb) and np.array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32))


def edge_rows(vocab: int) -> np.ndarray:
    """Rows the comparison semantics decide: ties, NaN first and later, both
    zeros, infinities, all NaN, a maximum in the last slot."""
    rng = np.random.default_rng(9)
    rows = []
    r = rng.normal(size=vocab).astype(np.float32)
    r[[3, vocab // 2, vocab - 1]] = 7.0
    rows.append(r)  # ties: the first wins
    r = rng.normal(size=vocab).astype(np.float32)
    r[0] = np.nan
    r[5] = 9.0
    rows.append(r)  # NaN at 0 keeps 0
    r = rng.normal(size=vocab).astype(np.float32)
    r[1::7] = np.nan
    rows.append(r)  # later NaNs never win
    r = np.full(vocab, -1.0, np.float32)
    r[2] = -0.0
    r[4] = 0.0
    rows.append(r)  # -0 then +0: a tie, -0 first
    r = np.full(vocab, -np.inf, np.float32)
    r[vocab - 1] = np.float32(-3.4e38)
    rows.append(r)  # -inf everywhere but the last
    rows.append(np.full(vocab, np.nan, np.float32))  # all NaN: 0
    r = np.full(vocab, -np.inf, np.float32)
    rows.append(r)  # all -inf: 0
    r = rng.normal(size=vocab).astype(np.float32)
    r[vocab - 1] = np.inf
    rows.append(r)
    return np.stack(rows)


@pytest.mark.parametrize("head", [1.0, 0.5, 1.0e-3])
def test_oracle_head_argmax_matches_go_loop(orc, head):
    y = edge_rows(300)
    logits, idx = orc.head_argmax(y, y.shape[0], y.shape[1], head)
    want_logits = y * np.float32(head) if head != 1.0 else y
    assert same_floats(logits, want_logits)
    assert [int(i) for i in idx] == [go_argmax(row) for row in want_logits]


def test_oracle_head_scale_ties(orc):
    """Scaling can round two different logits to one value: the argmax is
    taken after the scale, as the reference's loop sees it."""
    a = np.float32(1.0)
    b = np.nextafter(a, np.float32(2.0))
    y = np.array([[0.0, a, b, 0.5]], np.float32)
    head = np.float32(2.0**-149) * np.float32(2.0**23)  # coarse scale: a and b collapse
    logits, idx = orc.head_argmax(y, 1, 4, float(head))
    assert idx[0] == go_argmax(logits[0])


@pytest.mark.gpu
@pytest.mark.parametrize("vocab", [1, 7, 256, 300, 8199, 16384])
@pytest.mark.parametrize("head", [1.0, 0.25, 3.0])
def test_head_argmax_gpu(wb, orc, cuda, vocab, head):
    rng = np.random.default_rng(vocab)
    y = rng.normal(size=(64, vocab)).astype(np.float32)
    if vocab >= 8:
        y = np.concatenate([y, edge_rows(vocab)])
    rows = y.shape[0]
    want_logits, want_idx = orc.head_argmax(y, rows, vocab, head)
    yd = cuda.from_numpy(y.reshape(-1).copy()).cuda()
    out = cuda.empty(rows * vocab, dtype=cuda.float32, device="cuda")
    idx = wb.decoder.HeadArgmax(yd, rows, vocab, head, logits=out)
    assert np.array_equal(idx.cpu().numpy(), want_idx)
    assert same_floats(out.cpu().numpy(), want_logits)
    # in place, as decoder.logits scales its output slice
    idx2 = wb.decoder.HeadArgmax(yd, rows, vocab, head, logits=yd)
    assert np.array_equal(idx2.cpu().numpy(), want_idx)
    assert same_floats(yd.cpu().numpy(), want_logits)


@pytest.mark.gpu
def test_head_argmax_edges(wb, orc, cuda):
    """Many rows (past one grid's 65535), an empty vocabulary, bad arguments."""
    rng = np.random.default_rng(4)
    rows, vocab = 70000, 5
    y = rng.integers(-3, 4, size=(rows, vocab)).astype(np.float32)  # many ties
    _, want = orc.head_argmax(y, rows, vocab, 1.0)
    idx = wb.decoder.HeadArgmax(cuda.from_numpy(y.reshape(-1)).cuda(), rows, vocab)
    assert np.array_equal(idx.cpu().numpy(), want)
    empty = cuda.empty(0, dtype=cuda.float32, device="cuda")
    idx = cuda.full((3,), 7, dtype=cuda.int32, device="cuda")
    wb.decoder.HeadArgmax(empty, 3, 0, idx=idx)
    assert idx.cpu().tolist() == [0, 0, 0]
    with pytest.raises(wb.Panic):
        wb.decoder.HeadArgmax(empty, -1, 0)
    with pytest.raises(wb.Panic):
        wb.decoder.HeadArgmax(cuda.zeros(6, device="cuda"), 2, 4)


@pytest.mark.gpu
def test_greedy_step_head(wb, orc, cuda):
    """A greedy step's head: the CQ4 G32 embedding product of a few decode
    rows on the lut path (bit-exact), scaled, argmax — the oracle's
    gemm_lut and head_argmax give the same token ids."""
    rng = np.random.default_rng(77)
    vocab, d, rows, head = 1031, 512, 5, 0.125
    p = wb.synth.random_packed(rng, vocab, d, 32, 4, "lloyd")
    m = wb.cq.New(p)
    x = rng.normal(size=rows * d).astype(np.float32)
    y = cuda.empty(rows * vocab, dtype=cuda.float32, device="cuda")
    m.GEMM(y, cuda.from_numpy(x).cuda(), rows)
    idx = wb.decoder.HeadArgmax(y, rows, vocab, head, logits=y)
    want_y = orc.gemm_lut(orc.OracleMatrix.of(p), x, rows)
    want_logits, want_idx = orc.head_argmax(want_y, rows, vocab, head)
    assert np.array_equal(idx.cpu().numpy(), want_idx)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want_logits.reshape(-1).view(np.uint32))
