"""CPU restatement of Whistle's log-mel front end and conv stem (Best()
hypothesis) — TEST INFRASTRUCTURE ONLY: the checker of wc_encoder_logmel,
wc_encoder_stem and wc_encoder_embed.

- frontend/stft.go:113 spectrum: frame f is the 512 samples centred on
  sample 160·f (zeros outside the clip), times the 400-sample symmetric
  Hann window at offset 56 (stft.go:60-85); the power |X_k|² of bins
  0 … 256. The reference takes it from algo-dsp's float32 FFT (a
  third-party module absent from the reference tree, pinned in its go.mod);
  here it is a float64 DFT of the float32 windowed samples, rounded to
  float32, as the device computes it. The two agree to the float32 FFT's
  rounding.
- mel.go:78 MelBank.apply (float64 sums), mel.go:302 softLog (ε = 10^-7.6 ×
  the clip's largest energy; log10 as Go's math.Log10, ln(x)·(1/ln 10)),
  mel.go:320 normalise with NormChannel ((x − mean) / (std + 1e-5), the
  n − 1 deviation), then float32.
- encoder/stem.go:198 forward: the 3×3 stride-2 convs with symmetric
  padding (the taps summed in (time, mel) order from 0, each float32
  product rounded before its add — algo-tensor's ops.Conv2D, third-party,
  fixes the reference's order), SiLU after the full conv and after each
  pointwise product, the channel-major flatten and stem.out; the CQ
  products are the lut restatement's (bit-exact with the reference's).
"""

from __future__ import annotations

import numpy as np

NFFT, HOP, BINS, MELS = 512, 160, 257, 80
WIN_LO = (NFFT - 400) // 2


def window() -> np.ndarray:
    """The 512-point frame window: the symmetric 400-point Hann at offset 56."""
    k = np.arange(400)
    w = np.zeros(NFFT, np.float32)
    w[WIN_LO:WIN_LO + 400] = (0.5 - 0.5 * np.cos(2.0 * np.pi * k / 399.0)).astype(np.float32)
    return w


def spectrum(x: np.ndarray) -> np.ndarray:
    """Power spectrum [n // 160][257] (float32) of one clip's samples."""
    x = np.asarray(x, np.float32)
    n = x.size
    F = n // HOP
    pad = np.zeros(n + NFFT, np.float32)
    pad[NFFT // 2:NFFT // 2 + n] = x
    idx = np.arange(F)[:, None] * HOP + np.arange(NFFT)[None, :]
    frames = (pad[idx] * window()[None, :]).astype(np.float32)  # float32 products
    j = np.arange(WIN_LO, WIN_LO + 400)
    k = np.arange(BINS)
    m = (k[:, None] * j[None, :]) % NFFT
    cs, sn = np.cos(2.0 * np.pi * m / NFFT), np.sin(2.0 * np.pi * m / NFFT)
    xw = frames[:, WIN_LO:WIN_LO + 400].astype(np.float64)
    re, im = xw @ cs.T, -(xw @ sn.T)
    return (re * re + im * im).astype(np.float32)


def logmel(x: np.ndarray, bank: np.ndarray) -> np.ndarray:
    """frontend/mel.go:226 LogMel on one clip: [n // 160][80] float32."""
    spec = spectrum(x).astype(np.float64)
    mel = spec @ np.asarray(bank, np.float32).astype(np.float64)
    if mel.size == 0:
        return mel.astype(np.float32)
    eps = 10.0 ** -7.6 * mel.max()
    if eps == 0:
        eps = 1e-10
    mel = np.log(mel + eps) * (1.0 / np.log(10.0))
    F = mel.shape[0]
    mean = mel.sum(0) / F
    sd = np.sqrt(((mel - mean) ** 2).sum(0) / (F - 1)) if F > 1 else np.zeros(MELS)
    return ((mel - mean) / (sd + 1e-5)).astype(np.float32)


def stem_frames(frames: int) -> int:
    """stem.go:166 length for three stride-2 stages of symmetric padding."""
    n = frames
    for _ in range(3):
        if n + 2 < 3:
            return 0
        n = (n - 1) // 2 + 1
    return n


def _silu(v: np.ndarray) -> np.ndarray:
    return (v * (1.0 / (1.0 + np.exp(-v.astype(np.float64)))).astype(np.float32)).astype(np.float32)


def _conv(x: np.ndarray, k: np.ndarray, depthwise: bool) -> np.ndarray:
    """A 3×3 stride-2 conv, padding 1: x [h][w][cin] -> [h'][w'][C]. Taps
    outside the clip add nothing (as on the device, which skips them)."""
    h, w = x.shape[0], x.shape[1]
    C = k.shape[1]
    ho, wo = (h - 1) // 2 + 1, (w - 1) // 2 + 1
    xp = np.zeros((h + 2, w + 2, x.shape[2]), np.float32)
    xp[1:h + 1, 1:w + 1] = x
    acc = np.zeros((ho, wo, C), np.float32)
    for kh in range(3):
        ih = 2 * np.arange(ho) - 1 + kh
        for kw in range(3):
            iw = 2 * np.arange(wo) - 1 + kw
            inside = ((ih >= 0) & (ih < h))[:, None] & ((iw >= 0) & (iw < w))[None, :]
            tap = xp[(ih + 1)[:, None], (iw + 1)[None, :]]  # [ho][wo][cin]
            prod = (tap * k[kh * 3 + kw][None, None, :]).astype(np.float32)
            acc = np.where(inside[:, :, None], (acc + prod).astype(np.float32), acc)
    return acc


def stem(mel: np.ndarray, w, orc) -> np.ndarray:
    """encoder/stem.go:198 forward on one clip's mel [frames][80]: [T][dim]."""
    C = w.stem_channels
    x = np.asarray(mel, np.float32)[:, :, None]
    x = _silu(_conv(x, w.stem_w, False))
    for dw, pw in ((w.stem_dw_1, w.stem_pw_1), (w.stem_dw_2, w.stem_pw_2)):
        x = _conv(x, dw, True)
        h, wd = x.shape[0], x.shape[1]
        y = orc.gemm_lut(orc.OracleMatrix.of(pw), x.reshape(-1, C), h * wd).reshape(h, wd, C)
        x = _silu(y)
    T, m = x.shape[0], x.shape[1]
    flat = np.ascontiguousarray(x.transpose(0, 2, 1)).reshape(T, C * m)
    return orc.gemm_lut(orc.OracleMatrix.of(w.stem_out), flat, T).reshape(T, -1)
