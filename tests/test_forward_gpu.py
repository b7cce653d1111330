"""The full synthetic forward on the device, whistle.Transcribe's greedy
path: 16 kHz audio through encoder.Encoder.Embed (front end, stem, the
8-layer stack; lut products, the attention's exact order) and
decoder.Decoder (Memory, GreedyMemory), against the CPU restatement's
whole chain (oracle/frontend.py, wo_enc_stack with the reference's float
attention, the decoder restatement): the same language and text tokens.

On these synthetic weights the decoder, fed the synthetic encoder's output,
emits one repeated token, so this test pins the chain's plumbing end to
end more than its numerics; those are pinned piece by piece (the encoder's
per-frame bounds in tests/test_encoder_gpu.py, the decoder's logits and
diverse greedy tokens on random memories in tests/test_decoder_step_gpu.py)."""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CLIPS, SAMPLES, MAX_TOK = 2, 80000, 16  # 5 s: 500 mel frames -> 63 encoder frames
LANGS = [8 + i for i in range(7)]


def test_audio_to_tokens_matches_oracle(wb, orc, cuda):
    from oracle import frontend as fe

    S_ = wb.synth
    dw = S_.DecoderWeights(seed=4600, vocab=2048, slots=256)
    ew = S_.EncoderWeights(seed=5600)
    audio = S_.audio(np.random.default_rng(35), CLIPS, SAMPLES)
    T = wb.encoder.Encoder.stem_frames(SAMPLES // 160)
    enc = wb.encoder.Encoder(ew, max_clips=CLIPS, max_frames=T)
    dec = wb.decoder.Decoder(dw, max_streams=CLIPS, max_frames=T, max_positions=MAX_TOK + 1)
    dec.Memory(enc.Embed(cuda.from_numpy(audio).cuda()))
    tok, cnt, lang, eos = (t.cpu().numpy() for t in dec.GreedyMemory(S_.WHISTLE_BOS, LANGS, S_.WHISTLE_EOS, MAX_TOK))
    xs = np.stack([fe.stem(fe.logmel(a, ew.mel_filters), ew, orc) for a in audio])
    memory = orc.OracleEncoder(ew).stack(xs, orc.ENC_ATTEND_FLOAT)
    otok, ocnt, olang, oeos = orc.OracleDecoder(dw).greedy_streams(memory, S_.WHISTLE_BOS, LANGS, S_.WHISTLE_EOS,
                                                                   MAX_TOK)
    assert np.array_equal(lang, olang)
    assert np.array_equal(cnt, ocnt) and np.array_equal(eos, oeos)
    assert np.array_equal(tok, otok[:, :MAX_TOK - 1])
