"""The CPU restatement of Whistle's encoder stack (oracle/whistle_oracle.c,
wo_enc_*), the checker of the device encoder: the reference's known
answers for the conv module's pieces (encoder_test.go:99 TestApplyAct's
SiLU, :138 TestGLUAndDepthwise's value·σ(gate) row and centred depthwise
conv), clips that do not see one another, and the stated bound between
the reference's float attention (attention.go:480 attendGEMM on the
fake-quantised q, k, v) and the int8 kernel's order (int8.go:208
AttendInt8Spans on the same codes) that the device runs bit for bit."""

from __future__ import annotations

import math

import numpy as np
import pytest

# The two attention forms differ by float rounding in the logits and the
# value sums; the lut products then round their tables on slightly
# different inputs. Over the 8 layers at 375 frames the outputs agree to
# cosine >= 0.99999 per frame (cq_test.go's accept for a lut product) and
# within 2e-3 of each frame's largest |value|.
FORM_COS = 0.99999
FORM_ATOL = 2e-3


@pytest.fixture(scope="module")
def enc(wb, orc):
    w = wb.synth.EncoderWeights(seed=5100, layers=8)
    return w, orc.OracleEncoder(w)


def test_silu_known_answers(orc):
    x = np.array([-2, -0.5, 0, 1, 3], np.float32)
    want = [float(v) / (1 + math.exp(-float(v))) for v in x]
    assert np.max(np.abs(orc.silu(x) - want)) <= 1e-6


def test_glu_and_depthwise_known_answers(orc):
    sig = lambda v: 1 / (1 + math.exp(-v))  # noqa: E731
    got = orc.enc_glu(np.array([1, -2, 0, 3], np.float32), 1, 2)
    assert np.max(np.abs(got - [1 * sig(0), -2 * sig(3)])) <= 1e-6
    # taps (1, 10, 100) weight frames i-1, i, i+1 (centred, zeros outside)
    got = orc.enc_depthwise(np.array([1, 2, 3, 4], np.float32), 4, 1, np.array([1, 10, 100], np.float32))
    assert got.tolist() == [10 + 200, 1 + 20 + 300, 2 + 30 + 400, 3 + 40]


def test_clips_are_independent(wb, orc):
    w = wb.synth.EncoderWeights(seed=5101, layers=2)
    oe = orc.OracleEncoder(w)
    x = wb.synth.stem_output(np.random.default_rng(3), 3, 24)
    both = oe.stack(x)
    for c in range(3):
        assert np.array_equal(both[c], oe.stack(x[c]))
    # threads change nothing
    assert np.array_equal(both, oe.stack(x, threads=3))


def test_attention_forms_within_stated_bound(wb, orc, enc):
    w, oe = enc
    x = wb.synth.stem_output(np.random.default_rng(5), 1, 375)
    a = oe.stack(x, orc.ENC_ATTEND_INT8)[0]
    b = oe.stack(x, orc.ENC_ATTEND_FLOAT)[0]
    assert np.isfinite(a).all() and np.isfinite(b).all()
    cos = (a * b).sum(-1) / np.linalg.norm(a, axis=-1) / np.linalg.norm(b, axis=-1)
    assert cos.min() >= FORM_COS, cos.min()
    rel = np.abs(a - b).max(-1) / np.abs(b).max(-1)
    assert rel.max() <= FORM_ATOL, rel.max()
    assert not np.array_equal(a, b)  # the forms do differ: the bound is not vacuous


def test_rope_tables_bound_frames(wb, orc):
    w = wb.synth.EncoderWeights(seed=5102, layers=1)
    w.rope_len = 16
    oe = orc.OracleEncoder(w)
    with pytest.raises(ValueError, match="exceed the RoPE tables"):
        oe.stack(wb.synth.stem_output(np.random.default_rng(0), 1, 17))


# ------------------------------------------------------------ front end, stem

def test_stem_frames_known_answers(wb, orc):
    """encoder_test.go:64 TestStemFrames (Best: stride 2 everywhere,
    symmetric padding) and the engine's ceil(floor(n/160)/8) rule on its
    measured lengths; the library's wc_encoder_stem_frames gives the same."""
    from oracle import frontend as fe

    assert fe.stem_frames(3000) == 375 and fe.stem_frames(80) == 10
    for n, want in {1280: 1, 1281: 1, 2560: 2, 16000: 13, 53040: 42, 160000: 125, 480000: 375}.items():
        assert fe.stem_frames(n // 160) == want, n
        assert wb.encoder.Encoder.stem_frames(n // 160) == want, n
    assert wb.encoder.Encoder.stem_frames(0) == 0


def test_frame_count_known_answers():
    """stft_test.go:54 TestFrameCount, centred framing: n // 160."""
    from oracle import frontend as fe

    for n, want in ((480000, 3000), (0, 0), (159, 0), (160, 1), (399, 2), (400, 2), (559, 3), (4321, 27),
                    (16000, 100)):
        assert fe.spectrum(np.zeros(n, np.float32)).shape[0] == want, n


def test_spectrum_is_the_windowed_dft(wb):
    """A tone at bin 32 puts its energy in bins 31-33 (the Hann main
    lobe), and the power equals numpy's float64 rfft of the windowed frame."""
    from oracle import frontend as fe

    n = 16000
    x = (0.5 * np.sin(2 * np.pi * 32 * np.arange(n) / 512)).astype(np.float32)
    s = fe.spectrum(x)
    mid = s[50]
    assert set(np.argsort(mid)[-3:]) == {31, 32, 33}
    pad = np.zeros(n + 512, np.float32)
    pad[256:256 + n] = x
    frame = (pad[50 * 160:50 * 160 + 512] * fe.window()).astype(np.float64)
    ref = np.abs(np.fft.rfft(frame)) ** 2
    assert np.allclose(mid, ref.astype(np.float32), rtol=1e-5, atol=1e-6 * ref.max())


def test_logmel_standardises_each_channel(wb):
    """mel.go:320 NormChannel: every channel has mean 0 and (n−1) deviation
    1 over time (to the 1e-5 in the divisor)."""
    from oracle import frontend as fe

    w = wb.synth.EncoderWeights(seed=5103, layers=1)
    m = fe.logmel(wb.synth.audio(np.random.default_rng(1), 1, 32000)[0], w.mel_filters).astype(np.float64)
    assert m.shape == (200, 80)
    assert np.abs(m.mean(0)).max() < 1e-5
    assert np.abs(m.std(0, ddof=1) - 1).max() < 1e-4
