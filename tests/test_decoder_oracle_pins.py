"""The decoder step's CPU restatement (oracle/whistle_oracle.c) pinned to the
reference's own known answers for its pieces (CPU only):

- internal/needle/engram_test.go:16 TestNgramHashHandComputed (the hash
  values and the table seeds);
- internal/needle/rope_test.go:10 TestRopeHandComputed;
- internal/needle/norm_test.go:9 TestZCRMSNormTiny, :46 TestRMSUnitTiny;
- internal/needle/mhc_test.go:76 TestSinkhornStochastic (column sums),
  :152 TestSinkhornLargeLogits (the log-domain path), :181
  TestSinkhornUniform;
and the whole decoder's internal consistency: a sequence fed in one greedy
run equals the same tokens fed one Extend at a time, and states are
independent of each other.
"""

from __future__ import annotations

import importlib
import math

import numpy as np
import pytest


def test_ngram_hash_hand_computed(orc):
    cases = [(0, 1, [5], 0xCD55385D), (0, 2, [7, 42], 0x1ED6CE87), (3, 3, [1, 2, 3], 0x420599E6),
             (1, 2, [8198], 0x7922F0D0), (2, 3, [0, 0, 0], 0xEBB8DBEB), (0, 2, [], 0xBE346A8B),
             (0, 2, [9, 9, 7, 42], 0x1ED6CE87)]
    for col, order, hist, want in cases:
        assert orc.ngram_hash(col, order, hist) == want, (col, order, hist)
    # col 3's seed 0x9E3779B9 · 4 keeps its low 32 bits: the hash of order 0.
    assert orc.ngram_hash(3, 0, []) == (0x78DDE6E4 ^ (0x78DDE6E4 >> 15))


def test_rope_hand_computed(orc):
    theta = 1e5
    c, s = orc.rope_tables(4, 3, theta)
    f1 = 1 / math.sqrt(theta)
    for pos in range(3):
        assert np.max(np.abs(c[2 * pos:2 * pos + 2] - [math.cos(pos), math.cos(pos * f1)])) <= 1e-7
        assert np.max(np.abs(s[2 * pos:2 * pos + 2] - [math.sin(pos), math.sin(pos * f1)])) <= 1e-7
    x = orc.rope_apply(np.array([1, 2, 3, 4], np.float32), c[4:6], s[4:6])
    c0, s0, c1, s1 = math.cos(2), math.sin(2), math.cos(2 * f1), math.sin(2 * f1)
    want = [1 * c0 - 3 * s0, 2 * c1 - 4 * s1, 3 * c0 + 1 * s0, 4 * c1 + 2 * s1]
    assert np.max(np.abs(x - want)) <= 1e-6
    assert np.array_equal(orc.rope_apply(np.array([1, 2, 3, 4], np.float32), c[0:2], s[0:2]), [1, 2, 3, 4])


def test_zc_norm_tiny(orc):
    x = np.array([3, 4, 0, 0, 0, 0, -1, 2, 2], np.float32)
    got = orc.zc_norm(x, np.array([0, 1, -0.5], np.float32))
    want = []
    for r in range(3):
        row = x[3 * r:3 * r + 3].astype(np.float64)
        rms = math.sqrt((row ** 2).sum() / 3 + 1e-6)
        want += [row[0] / rms, 2 * row[1] / rms, 0.5 * row[2] / rms]
    assert np.max(np.abs(got - want)) <= 1e-6
    assert np.all(got[3:6] == 0)


def test_rms_unit_tiny(orc):
    got = orc.rms_unit(np.array([1, 1, 1, 1, 2, 0, 0, 0], np.float32), 4)
    one = 1 / math.sqrt(1 + 1e-6)
    want = np.array([one] * 4 + [2 / math.sqrt(1 + 1e-6), 0, 0, 0])
    assert np.max(np.abs(got - want)) <= 1e-7


def _ref_sinkhorn(k, n, iters):
    e = np.exp(k.astype(np.float64) - k.max()).reshape(n, n)
    for _ in range(iters):
        e /= e.sum(axis=1, keepdims=True)
        e /= e.sum(axis=0, keepdims=True)
    return e.reshape(-1)


@pytest.mark.parametrize("scale", [0.1, 1, 4])
def test_sinkhorn_stochastic(orc, scale):
    rng = np.random.default_rng(int(scale * 10))
    for trial in range(20):
        logits = rng.normal(0, scale, size=16).astype(np.float32)
        if trial % 2 == 1:
            logits[::5] += 4
        h = orc.sinkhorn(logits)
        cols = h.reshape(4, 4).astype(np.float64).sum(axis=0)
        assert np.all(np.abs(cols - 1) <= 4e-7)
        assert np.max(np.abs(h - _ref_sinkhorn(logits, 4, 20))) <= 1e-6


def test_sinkhorn_uniform_and_large(orc):
    assert np.all(orc.sinkhorn(np.full(16, 3.5, np.float32)) == 0.25)
    rng = np.random.default_rng(9)
    for scale in (1e3, 1e4, 1e30):
        h = orc.sinkhorn(rng.normal(0, scale, size=16).astype(np.float32))  # the log-domain path
        assert np.all(np.isfinite(h)) and np.all(h >= 0) and np.all(h <= 1)
        assert np.all(np.abs(h.reshape(4, 4).astype(np.float64).sum(axis=0) - 1) <= 4e-7)


@pytest.fixture(scope="module")
def small_decoder(orc):
    wb = importlib.import_module("go-whistle_b200")
    w = wb.synth.DecoderWeights(seed=4100, vocab=2048, layers=8, slots=512)
    return wb, w, orc.OracleDecoder(w)


def test_greedy_equals_step_by_step(small_decoder):
    """GreedyMemory's tokens are the argmax of Extend one token at a time
    (decoder.go:252 with t = 1 is all a greedy step is)."""
    wb, w, od = small_decoder
    S = wb.synth
    enc = S.encoder_output(np.random.default_rng(3), 1, 40)[0]
    st = od.state(40, 40)
    st.memory(enc)
    toks, lang, eos, _ = st.greedy(S.WHISTLE_BOS, [8 + i for i in range(7)], S.WHISTLE_EOS, 12)
    st2 = od.state(40, 40)
    st2.memory(enc)
    logits = st2.extend(S.WHISTLE_BOS)
    langs = [8 + i for i in range(7)]
    best = max(range(7), key=lambda i: (logits[langs[i]], -i))
    assert langs[best] == lang
    nxt, got = lang, []
    for _ in range(11):
        logits = st2.extend(nxt)
        nxt = int(np.argmax(logits))
        if nxt == S.WHISTLE_EOS:
            break
        got.append(nxt)
    assert got == list(toks)


def test_streams_are_independent(small_decoder):
    """The multi-stream CPU run equals one run per stream."""
    wb, w, od = small_decoder
    S = wb.synth
    enc = S.encoder_output(np.random.default_rng(4), 3, 24)
    langs = [8 + i for i in range(7)]
    tok, cnt, lang, eh = od.greedy_streams(enc, S.WHISTLE_BOS, langs, S.WHISTLE_EOS, 10, threads=3)
    for b in range(3):
        st = od.state(16, 24)
        st.memory(enc[b])
        t, l, e, _ = st.greedy(S.WHISTLE_BOS, langs, S.WHISTLE_EOS, 10)
        assert list(tok[b, :cnt[b]]) == list(t) and lang[b] == l and bool(eh[b]) == e
