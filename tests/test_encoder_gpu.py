"""The device encoder stack (wc_encoder_*, decoder.cu) against the CPU
restatement of internal/encoder's Stack (oracle/whistle_oracle.c) on a
synthetic Whistle-shaped encoder: 8 layers of width 512 in 4 mHC lanes,
macaron blocks (two HadamardMLPs, int8 self-attention with no mask and
RoPE, the conv module with CQ2 pw1/pw2 and a 9-tap depthwise conv).

- With the lut products and the attention's exact order, every frame of
  every clip is the oracle's with the int8 attention form bit for bit,
  but for the float64 sums of squares of the norms, which run as a tree
  on the device: such a sum can move a float32 result by one ulp when it
  lies within about 2^-44 of a rounding boundary, and later layers carry
  that on. So: bit for bit on nearly every frame, all within the
  attention-form bound below.
- With the attention in any order, and with the products on the tensor
  cores, the outputs stay within stated bounds of the reference's own
  float attention (attention.go:480 attendGEMM).
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# The bound between the two attention forms (tests/test_encoder_oracle.py):
# cosine per frame, and the largest difference over the frame's largest
# |value|.
FORM_COS, FORM_ATOL = 0.99999, 2e-3
# The tensor cores' fp16 operands (power-of-two scales, fp32 accumulate) in
# every product of every layer: measured min cosine 0.9999986 and largest
# difference 2.4e-3 of the frame's largest |value| on this case.
TC_COS, TC_ATOL = 0.99999, 1e-2


def _cmp(got, want):
    g, w = got.reshape(-1, got.shape[-1]), want.reshape(-1, want.shape[-1])
    cos = (g * w).sum(-1) / np.linalg.norm(g, axis=-1) / np.linalg.norm(w, axis=-1)
    rel = np.abs(g - w).max(-1) / np.abs(w).max(-1)
    same = np.all(g.view(np.uint32) == w.view(np.uint32), axis=-1)
    return cos.min(), rel.max(), same.mean()


@pytest.fixture(scope="module")
def setup(wb, orc, cuda):
    w = wb.synth.EncoderWeights(seed=5200, layers=8)
    return w, orc.OracleEncoder(w)


def _x(wb, cuda, clips, frames, seed):
    x = wb.synth.stem_output(np.random.default_rng(seed), clips, frames)
    return x, cuda.from_numpy(x).cuda()


@pytest.mark.parametrize("clips,frames", [(3, 40), (1, 375)])
def test_stack_matches_oracle(wb, orc, cuda, setup, clips, frames):
    w, oe = setup
    x, dx = _x(wb, cuda, clips, frames, 11 + frames)
    enc = wb.encoder.Encoder(w, max_clips=clips, max_frames=frames)
    got = enc.Stack(dx).cpu().numpy()
    want = oe.stack(x, orc.ENC_ATTEND_INT8)
    cos, rel, same = _cmp(got, want)
    assert np.isfinite(got).all()
    assert same >= 0.99, (same, cos, rel)
    assert cos >= FORM_COS and rel <= FORM_ATOL, (same, cos, rel)
    # the reference's float attention form is within the stated bound too
    cos2, rel2, _ = _cmp(got, oe.stack(x, orc.ENC_ATTEND_FLOAT))
    assert cos2 >= FORM_COS and rel2 <= FORM_ATOL, (cos2, rel2)


def test_stack_repeats_and_shrinks(wb, cuda, setup):
    w, _ = setup
    x, dx = _x(wb, cuda, 4, 32, 7)
    enc = wb.encoder.Encoder(w, max_clips=4, max_frames=32)
    a = enc.Stack(dx).cpu().numpy()
    b = enc.Stack(dx).cpu().numpy()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    # fewer clips and frames than the room: clip 1 alone, its first 20 frames
    one = enc.Stack(dx[1:2, :20].contiguous()).cpu().numpy()
    ref = wb.encoder.Encoder(w, max_clips=1, max_frames=20).Stack(dx[1:2, :20].contiguous()).cpu().numpy()
    assert np.array_equal(one.view(np.uint32), ref.view(np.uint32))


def test_any_order_within_bound(wb, orc, cuda, setup):
    w, oe = setup
    x, dx = _x(wb, cuda, 2, 96, 21)
    enc = wb.encoder.Encoder(w, max_clips=2, max_frames=96, flags=wb.encoder.WC_ENCODER_ANY_ORDER)
    got = enc.Stack(dx).cpu().numpy()
    cos, rel, _ = _cmp(got, oe.stack(x, orc.ENC_ATTEND_FLOAT))
    assert cos >= FORM_COS and rel <= FORM_ATOL, (cos, rel)


def test_tensor_cores_within_bound(wb, orc, cuda, setup):
    w, oe = setup
    x, dx = _x(wb, cuda, 2, 96, 22)
    flags = wb.encoder.WC_ENCODER_TENSOR_CORES | wb.encoder.WC_ENCODER_ANY_ORDER
    enc = wb.encoder.Encoder(w, max_clips=2, max_frames=96, flags=flags)
    got = enc.Stack(dx).cpu().numpy()
    cos, rel, _ = _cmp(got, oe.stack(x, orc.ENC_ATTEND_FLOAT))
    print(f"tensor cores against the reference form: min cos {cos:.7f}, max rel {rel:.2e}")
    assert cos >= TC_COS and rel <= TC_ATOL, (cos, rel)


def test_errors(wb, cuda, setup):
    w, _ = setup
    E = wb.encoder.Encoder
    with pytest.raises(wb.Panic, match="room for 300 clips of 375 frames"):
        E(w, max_clips=300, max_frames=375)
    w2 = wb.synth.EncoderWeights(seed=5201, layers=1)
    w2.dw_k = 8
    with pytest.raises(wb.Panic, match="depthwise kernel of 8 taps"):
        E(w2, max_clips=1, max_frames=8)
    enc = E(w, max_clips=2, max_frames=16)
    _, dx = _x(wb, cuda, 3, 16, 1)
    with pytest.raises(wb.Panic, match="3 clips of 16 frames exceed the room for 2 of 16"):
        enc.Stack(dx)
    w3 = wb.synth.EncoderWeights(seed=5202, layers=1)
    w3.rope_len = 8
    with pytest.raises(wb.Panic, match="RoPE tables for 8 positions, want 16"):
        E(w3, max_clips=1, max_frames=16).Stack(dx[:1])


# ------------------------------------------------------------ front end, stem
# frontend/mel.go:226 LogMel and encoder/stem.go:198 against the CPU
# restatement (oracle/frontend.py). LogMel: the device and the restatement
# both take a float64 DFT and float64 mel sums, in different orders; the
# float32 results agree to LOGMEL_ATOL (values are standardised, |x| < 10).
# Stem: the same float32 operations in the same order and the lut products;
# float64 exp in the SiLU may round the last bit differently.
LOGMEL_ATOL = 1e-5


def test_logmel_matches_oracle(wb, cuda, setup):
    from oracle import frontend as fe

    w, _ = setup
    a = wb.synth.audio(np.random.default_rng(31), 2, 48000 + 77)
    enc = wb.encoder.Encoder(w, max_clips=2, max_frames=40)
    got = enc.LogMel(cuda.from_numpy(a).cuda()).cpu().numpy()
    for c in range(2):
        want = fe.logmel(a[c], w.mel_filters)
        assert got[c].shape == want.shape == (300, 80)
        assert np.abs(got[c] - want).max() <= LOGMEL_ATOL, np.abs(got[c] - want).max()


@pytest.mark.parametrize("flags", [0, 1], ids=["lut", "tensor-cores"])
def test_stem_matches_oracle(wb, orc, cuda, setup, flags):
    from oracle import frontend as fe

    w, _ = setup
    a = wb.synth.audio(np.random.default_rng(32), 2, 40000)
    mel = np.stack([fe.logmel(x, w.mel_filters) for x in a])  # 250 frames -> 32 stem frames
    enc = wb.encoder.Encoder(w, max_clips=2, max_frames=32, flags=flags)
    got = enc.Stem(cuda.from_numpy(mel).cuda()).cpu().numpy()
    assert got.shape == (2, 32, 512)
    for c in range(2):
        want = fe.stem(mel[c], w, orc)
        if flags == 0:
            assert np.mean(got[c] == want) >= 0.99
            assert np.abs(got[c] - want).max() <= 1e-5 * np.abs(want).max()
        else:
            cos = (got[c] * want).sum(-1) / np.linalg.norm(got[c], axis=-1) / np.linalg.norm(want, axis=-1)
            assert cos.min() >= TC_COS, cos.min()


@pytest.mark.parametrize("flags", [0, 3], ids=["exact", "tensor-cores"])
def test_embed_matches_oracle(wb, orc, cuda, setup, flags):
    """encoder.go:108 Embed: LogMel, Stem and Stack on the device against
    the restatement's (the reference's float attention form)."""
    from oracle import frontend as fe

    w, oe = setup
    a = wb.synth.audio(np.random.default_rng(33), 2, 64000)  # 400 mel frames -> 50 stem frames
    enc = wb.encoder.Encoder(w, max_clips=2, max_frames=50, flags=flags)
    got = enc.Embed(cuda.from_numpy(a).cuda()).cpu().numpy()
    assert got.shape == (2, 50, 512)
    want = np.stack([oe.stack(fe.stem(fe.logmel(x, w.mel_filters), w, orc), orc.ENC_ATTEND_FLOAT) for x in a])
    cos, rel, _ = _cmp(got, want)
    bound = (FORM_COS, FORM_ATOL) if flags == 0 else (TC_COS, TC_ATOL)
    assert cos >= bound[0] and rel <= bound[1], (cos, rel)


def test_stem_errors(wb, cuda, setup):
    w0 = wb.synth.EncoderWeights(seed=5203, layers=1)
    w0.stem_w = None
    bare = wb.encoder.Encoder(w0, max_clips=1, max_frames=8)
    x = cuda.zeros(1, 1600, device="cuda")
    with pytest.raises(wb.Panic, match="built without the stem"):
        bare.LogMel(x)
    w, _ = setup
    enc = wb.encoder.Encoder(w, max_clips=1, max_frames=8)
    with pytest.raises(wb.Panic, match="exceed the room"):
        enc.Embed(cuda.zeros(1, 160 * 65, device="cuda"))  # 65 mel frames -> 9 stem frames > 8


def test_loaded_encoder_matches_oracle(wb, orc, cuda):
    """An encoder loaded from a synthetic whistle.cact (encoder.Encoder.Load):
    Embed against the CPU restatement on the same loaded weights."""
    from oracle import frontend as fe

    w = wb.synth.DecoderWeights(seed=4520, vocab=8199)
    e = wb.synth.EncoderWeights(seed=5520)
    e.hada_p1, e.hada_p2 = w.hada_p1, w.hada_p2
    data = wb.weights.write_whistle_cact(w, seed=4, enc=e)
    le = wb.weights.load_encoder(data)
    a = wb.synth.audio(np.random.default_rng(34), 2, 48000)  # 300 mel frames -> 38 stem frames
    got = wb.encoder.Encoder.Load(data, max_clips=2, max_frames=38).Embed(cuda.from_numpy(a).cuda()).cpu().numpy()
    oe = orc.OracleEncoder(le)
    want = np.stack([oe.stack(fe.stem(fe.logmel(x, le.mel_filters), le, orc), orc.ENC_ATTEND_FLOAT) for x in a])
    cos, rel, _ = _cmp(got, want)
    assert cos >= FORM_COS and rel <= FORM_ATOL, (cos, rel)
