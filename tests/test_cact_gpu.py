"""A decoder loaded from a .cact file on the device: a synthetic
whistle.cact (Whistle's 681-record layout, vocabulary 8199) through
weights.load_decoder and decoder.Decoder.Load, its greedy tokens against
the CPU restatement's on the same loaded weights: identical token ids."""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def whistle(wb):
    w = wb.synth.DecoderWeights(seed=4500, vocab=8199)
    return wb.weights.write_whistle_cact(w, seed=5)


def test_loaded_decoder_greedy_matches_oracle(wb, orc, cuda, whistle, tmp_path):
    path = tmp_path / "whistle.cact"
    path.write_bytes(whistle)
    S, F, max_tok = 8, 96, 16
    S_ = wb.synth
    enc = S_.encoder_output(np.random.default_rng(21), S, F)
    dec = wb.decoder.Decoder.Load(str(path), max_streams=S, max_frames=F, max_positions=max_tok + 1)
    dec.Memory(cuda.from_numpy(enc).cuda())
    tok, cnt, lang, eos = (t.cpu().numpy() for t in dec.GreedyMemory(S_.WHISTLE_BOS, S_.WHISTLE_LANGS,
                                                                     S_.WHISTLE_EOS, max_tok))
    w = wb.weights.load_decoder(whistle)
    otok, ocnt, olang, oeos = orc.OracleDecoder(w).greedy_streams(enc, S_.WHISTLE_BOS, S_.WHISTLE_LANGS,
                                                                 S_.WHISTLE_EOS, max_tok, threads=8)
    assert np.array_equal(lang, olang)
    assert np.array_equal(cnt, ocnt)
    assert np.array_equal(eos, oeos)
    assert np.array_equal(tok, otok[:, :max_tok - 1])
    assert len({tuple(t) for t in otok}) > 1


def test_loaded_decoder_logits_match_oracle(wb, orc, cuda, whistle):
    """Extend on random tokens: every step's logits within 1e-5 of the
    row's largest |logit| and bit-exact on >= 99 % of values, as for the
    synthetic decoder built in memory (test_decoder_step_gpu.py)."""
    S, F, steps = 3, 40, 6
    w = wb.weights.load_decoder(whistle)
    od = orc.OracleDecoder(w)
    enc = wb.synth.encoder_output(np.random.default_rng(22), S, F)
    dec = wb.decoder.Decoder.Load(whistle, max_streams=S, max_frames=F, max_positions=steps + 1)
    dec.Memory(cuda.from_numpy(enc).cuda())
    states = []
    for b in range(S):
        st = od.state(steps + 1, F)
        st.memory(enc[b])
        states.append(st)
    rng = np.random.default_rng(6)
    logits = cuda.empty((S, w.vocab), dtype=cuda.float32, device="cuda")
    exact = total = 0
    for _ in range(steps):
        toks = rng.integers(0, w.vocab, size=S).astype(np.int32)
        dec.Extend(cuda.from_numpy(toks).cuda(), logits)
        got = logits.cpu().numpy()
        for b in range(S):
            want = states[b].extend(int(toks[b]))
            assert np.abs(got[b] - want).max() <= 1e-5 * np.abs(want).max()
            exact += int(np.sum(got[b].view(np.uint32) == want.view(np.uint32)))
            total += want.size
    assert exact >= 0.99 * total, f"{exact} of {total}"
