"""The device beam search (wc_decoder_beam: beam.cu over decoder.cu's
streams, forks and candidate kernel) against the CPU restatement of
internal/search (oracle/beam.py) on the oracle decoder: for every stopping
rule, admission rule, length normalisation, length count and language
step, and EOS tokens the synthetic decoder does reach, each clip's best
hypothesis is the same (text tokens, language, EOS), its score and the
model log-probabilities agree to float64 rounding of nearly equal logits,
and one beam is the device's greedy decode (search_test.go:13)."""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CLIPS, FRAMES, MAX_TOK, BEAMS = 3, 48, 12, 5
# Logits agree with the oracle's within 1e-5 of the row's largest |logit|
# (tests/test_decoder_step_gpu.py); log p and the scores inherit that.
LP_ATOL = 1e-4


@pytest.fixture(scope="module")
def setup(wb, orc, cuda):
    w = wb.synth.DecoderWeights(seed=4200, vocab=16384)
    enc = wb.synth.encoder_output(np.random.default_rng(31), CLIPS, FRAMES)
    dec = wb.decoder.Decoder(w, max_streams=CLIPS * BEAMS, max_frames=FRAMES, max_positions=MAX_TOK + 1)
    return w, orc.OracleDecoder(w), enc, cuda.from_numpy(enc).cuda(), dec


def _option_sets(bm, D):
    return {
        "default": (bm.Options(), {}),
        "all gnmt seq langbeam": (
            bm.Options(stop=bm.STOP_ALL, admit=bm.ADMIT_TOPK, norm=bm.NORM_GNMT, alpha=0.6, length=bm.LEN_SEQ,
                       lang=bm.LANG_BEAM),
            dict(stop=D.WC_STOP_ALL, admit=D.WC_ADMIT_TOPK, norm=D.WC_NORM_GNMT, alpha=0.6, length=D.WC_LEN_SEQ,
                 lang_step=D.WC_LANG_BEAM)),
        "best pow text+eos": (
            bm.Options(stop=bm.STOP_BEST, norm=bm.NORM_POW, alpha=0.8, length=bm.LEN_TEXT_EOS),
            dict(stop=D.WC_STOP_BEST, norm=D.WC_NORM_POW, alpha=0.8, length=D.WC_LEN_TEXT_EOS)),
        "hf scored topk": (
            bm.Options(stop=bm.STOP_HF, admit=bm.ADMIT_TOPK, lang=bm.LANG_ARGMAX_SCORED),
            dict(stop=D.WC_STOP_HF, admit=D.WC_ADMIT_TOPK, lang_step=D.WC_LANG_ARGMAX_SCORED)),
        "forced language, none norm": (
            bm.Options(language=3, norm=bm.NORM_NONE, lang=bm.LANG_BEAM),
            dict(language=3, norm=D.WC_NORM_NONE, lang_step=D.WC_LANG_BEAM)),
    }


@pytest.mark.parametrize("eos", [2, 12487, 725])
def test_beam_matches_oracle(wb, cuda, setup, eos):
    from oracle import beam as bm

    w, od, enc, denc, dec = setup
    S_ = wb.synth
    D = wb.decoder
    for name, (oo, kw) in _option_sets(bm, D).items():
        oo.beams, oo.max_tokens = BEAMS, MAX_TOK
        dec.MemoryBeams(denc, BEAMS)
        tok, cnt, lang, eos_hit, score, lang_lp, lps = dec.Beam(S_.WHISTLE_BOS, S_.WHISTLE_LANGS, eos,
                                                               D.DefaultBeam(beams=BEAMS, max_tokens=MAX_TOK, **kw))
        for c in range(CLIPS):
            st = od.state(MAX_TOK + 1, FRAMES)
            st.memory(enc[c])
            r = bm.search(st, S_.WHISTLE_BOS, S_.WHISTLE_LANGS, eos, oo, MAX_TOK)
            where = (name, eos, c)
            assert int(lang[c]) == r.lang, where
            assert bool(eos_hit[c]) == r.eos, where
            assert int(cnt[c]) == len(r.tokens), where
            assert tok[c, :cnt[c]].tolist() == r.tokens, where
            assert np.all(tok[c, cnt[c]:] == -1), where
            assert abs(score[c] - r.score) <= LP_ATOL * max(1.0, abs(r.score)), where
            assert abs(lang_lp[c] - r.lang_lp) <= LP_ATOL, where
            assert np.allclose(lps[c, :len(r.logprobs)], r.logprobs, rtol=0, atol=LP_ATOL), where


def test_one_beam_is_greedy(wb, cuda, setup):
    """search_test.go:13: one beam (LangArgmax, Whisper's rules) is greedy."""
    w, od, enc, denc, dec = setup
    S_ = wb.synth
    dec.MemoryBeams(denc, 1)
    tok, cnt, lang, eos_hit, *_ = dec.Beam(S_.WHISTLE_BOS, S_.WHISTLE_LANGS, 725,
                                           wb.decoder.DefaultBeam(beams=1, max_tokens=MAX_TOK))
    dec.Memory(denc)
    gtok, gcnt, glang, geos = (t.cpu().numpy() for t in dec.GreedyMemory(S_.WHISTLE_BOS, S_.WHISTLE_LANGS, 725,
                                                                        MAX_TOK))
    assert np.array_equal(lang, glang) and np.array_equal(cnt, gcnt) and np.array_equal(eos_hit, geos.astype(bool))
    assert np.array_equal(tok, gtok)


def test_beam_errors(wb, cuda, setup):
    w, od, enc, denc, dec = setup
    S_ = wb.synth
    D = wb.decoder
    dec.MemoryBeams(denc, BEAMS)
    with pytest.raises(wb.Panic, match="search: invalid options: 0 beams"):
        dec.Beam(S_.WHISTLE_BOS, S_.WHISTLE_LANGS, 2, D.DefaultBeam(beams=0, max_tokens=4))
    with pytest.raises(wb.Panic, match="5 streams per clip, the options 4 beams"):
        dec.Beam(S_.WHISTLE_BOS, S_.WHISTLE_LANGS, 2, D.DefaultBeam(beams=4, max_tokens=4))
    with pytest.raises(wb.Panic, match="invalid options: norm 9"):
        dec.Beam(S_.WHISTLE_BOS, S_.WHISTLE_LANGS, 2, D.DefaultBeam(beams=BEAMS, max_tokens=4, norm=9))
    with pytest.raises(wb.Panic, match="unknown language 7 of 7"):
        dec.Beam(S_.WHISTLE_BOS, S_.WHISTLE_LANGS, 2, D.DefaultBeam(beams=BEAMS, max_tokens=4, language=7))
    with pytest.raises(wb.Panic, match="exceed"):
        dec.Beam(S_.WHISTLE_BOS, S_.WHISTLE_LANGS, 2, D.DefaultBeam(beams=BEAMS, max_tokens=MAX_TOK + 5))
    with pytest.raises(wb.Panic, match="clips x 4 beams"):
        dec.MemoryBeams(cuda.zeros((4, FRAMES, 512), dtype=cuda.float32, device="cuda"), 4)
