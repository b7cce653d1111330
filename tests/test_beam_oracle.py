"""The CPU restatement of internal/search (oracle/beam.py), the checker of
the device beam search, against the reference's hand-computed tests:
options.go's Validate and penalty (options_test.go:11, :54), candidates
(options_test.go:83, the hook-free cases), the admission and stopping
rules of one step (options_test.go:161 TestStepRules) and the final pick
at the token limit (options_test.go:233 TestPickAtTokenLimit); and one
beam equals greedy decoding on the oracle decoder (search_test.go:13
TestOneBeamIsGreedy)."""

from __future__ import annotations

import math

import numpy as np
import pytest


@pytest.fixture(scope="module")
def bm():
    from oracle import beam

    return beam


def test_options_validate(bm):
    bm.Options().validate()
    mods = {"zero beams": dict(beams=0), "negative max": dict(max_tokens=-1), "unset norm": dict(norm=0),
            "unset length": dict(length=0), "unknown stop": dict(stop=bm.STOP_HF + 1), "unset admit": dict(admit=0),
            "unset lang": dict(lang=0), "NaN alpha": dict(alpha=math.nan), "infinite alpha": dict(alpha=math.inf),
            "unknown norm": dict(norm=bm.NORM_GNMT + 1), "unknown admit": dict(admit=bm.ADMIT_ABOVE_LIVE + 1)}
    for name, kw in mods.items():
        with pytest.raises(bm.OptionsError, match="search: invalid options"):
            bm.Options(**kw).validate()


@pytest.mark.parametrize("norm,alpha,l,want", [("NONE", 0, 7, 1), ("LEN", 0, 7, 7), ("LEN", 0, 0, 1),
                                               ("POW", 0.5, 9, 3), ("POW", 2, 3, 9), ("GNMT", 1, 7, 2),
                                               ("GNMT", 2, 1, 1)])
def test_penalty(bm, norm, alpha, l, want):
    o = bm.Options(norm=getattr(bm, "NORM_" + norm), alpha=alpha)
    assert abs(o.penalty(l) - want) <= 1e-12


def test_candidates(bm):
    lp = bm.log_softmax([1, 3, 2, 3, 0, 2.5])
    assert abs(sum(math.exp(v) for v in lp) - 1) <= 1e-12
    toks = lambda cs: [c.tok for c in cs]  # noqa: E731
    assert toks(bm.candidates(lp, 4)) == [1, 3, 5, 2]
    assert toks(bm.candidates(lp, 10)) == [1, 3, 5, 2, 0, 4]
    assert toks(bm.candidates(lp, 2, [0, 4, 2])) == [2, 0]


class Fixed:
    """options_test.go:138 fixed: the same candidates for every hypothesis
    with a given text length."""

    def __init__(self, table):
        self.table = table

    def expand(self, hs, n, allowed):
        return [self.table[h.text_len()][:n] for h in hs]


EOS = 1


def _c(bm, tok, lp):
    return bm.Cand(tok, lp, lp)


def _start(bm):
    return [bm.Hyp(seq=[2, 9], text=2)]


def test_step_rules(bm):
    """options_test.go:161: one step from one live hypothesis, 2 beams. In
    high, EOS ranks second (inside the top 2, above b); in low, third."""
    c = lambda t, lp: _c(bm, t, lp)  # noqa: E731
    high = Fixed({0: [c(10, -0.1), c(EOS, -0.5), c(11, -1), c(12, -2)]})
    low = Fixed({0: [c(10, -0.1), c(11, -0.3), c(EOS, -0.5), c(12, -2)]})
    cases = [("above-live, EOS second", high, bm.STOP_K, bm.ADMIT_ABOVE_LIVE, [10, 11], 1, False),
             ("top-k, EOS second", high, bm.STOP_K, bm.ADMIT_TOPK, [10, 11], 1, False),
             ("above-live, EOS third", low, bm.STOP_K, bm.ADMIT_ABOVE_LIVE, [10, 11], 0, False),
             ("top-k, EOS third", low, bm.STOP_K, bm.ADMIT_TOPK, [10, 11], 0, False),
             ("best, EOS second", high, bm.STOP_BEST, bm.ADMIT_ABOVE_LIVE, [10, 11], 1, False),
             ("all, EOS second", high, bm.STOP_ALL, bm.ADMIT_TOPK, [10], 1, False)]
    for name, ex, stop, admit, alive, finished, done in cases:
        s = bm.Beam(bm.Options(beams=2, stop=stop, admit=admit, norm=bm.NORM_NONE), EOS)
        nxt, d = s.step(ex, _start(bm))
        assert [h.seq[-1] for h in nxt] == alive and len(s.fin) == finished and d == done, name
    # StopBest ends once the finished score reaches the best live one.
    s = bm.Beam(bm.Options(beams=2, stop=bm.STOP_BEST, norm=bm.NORM_NONE), EOS)
    _, d = s.step(Fixed({0: [c(EOS, -0.05), c(10, -0.1), c(11, -1)]}), _start(bm))
    assert d
    # StopK ends at Beams finished hypotheses: two EOS from two parents.
    s = bm.Beam(bm.Options(beams=2, stop=bm.STOP_K, norm=bm.NORM_NONE), EOS)
    two = [bm.Hyp(seq=[2, 9, 10], text=2), bm.Hyp(seq=[2, 9, 11], text=2, adj=-0.2)]
    _, d = s.step(Fixed({1: [c(EOS, -0.1), c(12, -3)]}), two)
    assert d and len(s.fin) == 2


def test_pick_at_token_limit(bm):
    """options_test.go:233: at the token limit the best live hypotheses
    compete with the finished (up to Beams of them under StopK); a search
    StopK ended picks among the finished only."""
    o = bm.Options(beams=3, norm=bm.NORM_NONE)
    short = bm.Hyp(seq=[2, 9], text=2, adj=-5, sum=-5, eos=True)
    good = bm.Hyp(seq=[2, 9, 10], text=2, adj=-1, sum=-1)
    worse = bm.Hyp(seq=[2, 9, 11], text=2, adj=-2, sum=-2)
    third = bm.Hyp(seq=[2, 9, 12], text=2, adj=-0.5, sum=-0.5)
    s = bm.Beam(o, EOS)
    s.fin = [short]
    assert s.pick([good, worse], False) is good
    assert s.pick([worse, good, third], False) is third
    s.opt.beams = 2
    assert s.pick([worse, third], False) is third
    assert s.pick([good, worse], True) is short
    assert bm.Beam(bm.Options(beams=3, norm=bm.NORM_NONE), EOS).pick([worse, good], False) is good


def test_one_beam_is_greedy(wb, orc, bm):
    """search_test.go:13: with one beam the search is greedy decoding."""
    w = wb.synth.DecoderWeights(seed=4300, vocab=2048, layers=2, slots=256)
    od = orc.OracleDecoder(w)
    enc = wb.synth.encoder_output(np.random.default_rng(7), 2, 24)
    langs = [8 + i for i in range(7)]
    for b in range(2):
        st = od.state(12, 24)
        st.memory(enc[b])
        r = bm.search(st, wb.synth.WHISTLE_BOS, langs, wb.synth.WHISTLE_EOS, bm.Options(beams=1), 10)
        g = od.state(12, 24)
        g.memory(enc[b])
        tok, lang, eos, _ = g.greedy(wb.synth.WHISTLE_BOS, langs, wb.synth.WHISTLE_EOS, 10)
        assert r.lang == lang and r.eos == eos and r.tokens == [int(t) for t in tok]


def test_fork_is_independent(wb, orc):
    """decoder.go:223 Fork: the fork and the original extend independently
    and each gives what an unforked state fed the same tokens gives."""
    w = wb.synth.DecoderWeights(seed=4301, vocab=2048, layers=2, slots=256)
    od = orc.OracleDecoder(w)
    enc = wb.synth.encoder_output(np.random.default_rng(8), 1, 16)[0]
    a = od.state(8, 16)
    a.memory(enc)
    for t in (1, 9, 300):
        a.extend(t)
    f = a.fork()
    la, lf = a.extend(5), f.extend(6)
    ref = od.state(8, 16)
    ref.memory(enc)
    for t in (1, 9, 300):
        ref.extend(t)
    assert np.array_equal(lf, ref.extend(6))
    ref2 = od.state(8, 16)
    ref2.memory(enc)
    for t in (1, 9, 300):
        ref2.extend(t)
    assert np.array_equal(la, ref2.extend(5))
