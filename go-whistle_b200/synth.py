"""Seeded synthetic inputs in the reference's formats (no corpora, no model
file exist in this image; these stand in for them with the shapes, sizes and
value distributions the benchmark configurations name).

- CQ tensors as cact.Packed holds them (internal/cact/packed.go:18-40): one
  sorted codebook per width, uniform index bytes (every code uniform), FP16
  norms with exponent uniform in 11..19 and a random mantissa (2^-4..2^4),
  as the reference's own tests draw them (internal/cq/cq_test.go:20-41).
- int8 KV caches: codes uniform in [-127, 127], scales uniform 0.01..0.05
  per (token, head); queries ~N(0, 1).
"""

from __future__ import annotations

import numpy as np

from .cq import Packed

# quantize.py's unit-variance Gaussian Lloyd-Max levels, as the reference's
# tests record them (internal/cact/cq_test.go:16-29); the whistle.cact
# codebooks are these over sqrt(group), rounded to float32.
LLOYD_MAX_UNIT = {
    2: [-1.5066708475715247, -0.45144060939344055, 0.4529474939511613, 1.5099326242547164],
    4: [-2.709990028558534, -2.0444556051349227, -1.5947570221842273, -1.233336191082712,
        -0.9222139662739897, -0.6395373737252813, -0.37266394934485414, -0.11445072030649898,
        0.14380628677643076, 0.4039889754802918, 0.6726933686864701, 0.9614053009735016,
        1.2755257831234952, 1.637058796059282, 2.0844263722579237, 2.7410141261982846],
}


def lloyd_max_codebook(bits: int, group: int) -> np.ndarray:
    """cact_test.go portCodebook: the stored whistle.cact levels."""
    return np.array([c / np.sqrt(group) for c in LLOYD_MAX_UNIT[bits]], np.float32)


def random_norms16(rng: np.random.Generator, n: int) -> np.ndarray:
    """FP16 norms 2^-4..2^4: exponent field 11..19, random mantissa."""
    exp = rng.integers(11, 20, size=n, dtype=np.uint16)
    man = rng.integers(0, 1024, size=n, dtype=np.uint16)
    return (exp << 10) | man


def random_packed(rng: np.random.Generator, out: int, in_: int, group: int, bits: int,
                  codebook: str = "baseline") -> Packed:
    """A random CQ tensor. codebook: "baseline" = sorted ~N(0, 0.02) (the
    benchmark configurations), "reference" = sorted ~N(0,1)/sqrt(G)
    (cq_test.go randomPacked), "lloyd" = the whistle.cact levels."""
    if codebook == "baseline":
        cb = np.sort(rng.normal(0.0, 0.02, size=1 << bits)).astype(np.float32)
    elif codebook == "reference":
        cb = np.sort(rng.normal(0.0, 1.0, size=1 << bits) / np.sqrt(group)).astype(np.float32)
    elif codebook == "lloyd":
        cb = lloyd_max_codebook(bits, group)
    else:
        raise ValueError(codebook)
    groups = (in_ + group - 1) // group
    row_bytes = groups * group * bits // 8
    index = rng.integers(0, 256, size=out * row_bytes, dtype=np.uint8)
    norms = random_norms16(rng, out * groups).astype("<u2").view(np.uint8)
    return Packed(Out=out, In=in_, Group=group, Bits=bits, Width=bits, Codebook=cb, Index=index, Norms=norms)


def algorithmic_bytes_gemv(out: int, in_: int, group: int, bits: int) -> int:
    """Bytes one batch-1 GEMV must move: packed index + FP16 norms + x + y +
    codebook, B = Out·RowBytes + 2·Out·Groups + 4·In + 4·Out + 4·2^bits."""
    groups = (in_ + group - 1) // group
    row_bytes = groups * group * bits // 8
    return out * row_bytes + 2 * out * groups + 4 * in_ + 4 * out + 4 * (1 << bits)


def random_kv(rng: np.random.Generator, rows: int, kv_heads: int, width: int):
    """An int8 cache: codes uniform in [-127, 127], scales U(0.01, 0.05)."""
    q = rng.integers(-127, 128, size=rows * kv_heads * width, dtype=np.int8)
    s = rng.uniform(0.01, 0.05, size=rows * kv_heads).astype(np.float32)
    return q, s


# ------------------------------------------------------------------ decoder
#
# Whistle's decoder as whistle.cact lays it out (internal/cact/testdata/
# whistle_names.txt): 8 layers of width 512 in 4 mHC lanes; self-attention
# 8 query heads / 2 KV heads of 48 (values 64) with 3 causal taps; a gated
# cross-attention of 8 heads (48 / 64); a HadamardMLP of 16 × 32 Kronecker
# factors with a rank-8 condition; engram sites at layers 3 and 7 with
# orders (2, 3) × 2 hashes = 4 tables of 18432 slots × 128; RoPE θ = 1e5.
# CQ tensors use one codebook per width (the .cact header's cb2/cb4), group
# 128: CQ4 for the embedding / head and the mHC φ, CQ2 for every other
# product. Values: CQ rows and float tensors ~N(0, 0.02) in scale, norm
# gains near 1 (scales ~N(0, 0.02)), as the benchmark configuration asks.

WHISTLE_LANGS = list(range(8192, 8199))  # "<|en|>" … "<|pl|>" (decoder.go:58)
WHISTLE_BOS, WHISTLE_EOS = 1, 2


def _cq_tensor(rng, out, in_, bits, group, cb, rms=0.02):
    """A CQ tensor whose rows have the given RMS: norms ≈ rms·√G (the
    codebook holds unit-variance levels over √G), spread ±25 %."""
    groups = (in_ + group - 1) // group
    row_bytes = groups * group * bits // 8
    index = rng.integers(0, 256, size=out * row_bytes, dtype=np.uint8)
    n = (rms * np.sqrt(group) * rng.uniform(0.8, 1.25, size=out * groups)).astype(np.float16)
    return Packed(Out=out, In=in_, Group=group, Bits=bits, Width=bits, Codebook=cb, Index=index,
                  Norms=n.view(np.uint16).astype("<u2").view(np.uint8))


class DecoderWeights:
    """A synthetic Whistle decoder: sizes as attributes, CQ tensors as
    Packed, float tensors as float32 arrays; per-layer tensors in
    ``layers[l]`` (dicts keyed by the .cact names without the prefix) and
    the engram sites in ``sites``."""

    def __init__(self, seed: int = 4000, vocab: int = 16384, layers: int = 8, slots: int = 18432):
        rng = np.random.default_rng(seed)
        self.seed = seed
        self.dim, self.lanes, self.n_layers, self.vocab = 512, 4, layers, vocab
        self.heads, self.kv_heads, self.qk, self.vd, self.taps = 8, 2, 48, 64, 3
        self.x_heads, self.x_qk, self.x_vd = 8, 48, 64
        self.na, self.nb, self.rank = 16, 32, 8
        self.orders = [2, 2, 3, 3]
        self.n_tables, self.slots, self.sub, self.etaps = 4, slots, 128, 4
        self.max_order = 3
        self.site_layers = [3, 7] if layers > 7 else [min(3, layers - 1)]
        self.rope_theta, self.rope_len = 1e5, 512
        G = 128
        self.cb2, self.cb4 = lloyd_max_codebook(2, G), lloyd_max_codebook(4, G)
        D, n = self.dim, self.lanes

        def vec(k, mean=0.0, sd=0.02):
            return (mean + rng.normal(0.0, sd, size=k)).astype(np.float32)

        # The tied embedding at a smaller scale than the other products, so
        # that the blocks, not the fed token alone, decide the next token.
        self.embedding = _cq_tensor(rng, vocab, D, 4, G, self.cb4, rms=0.005)
        self.final_norm = vec(D)
        self.hada_p1 = rng.permutation(self.na * self.nb).astype(np.int32)
        self.hada_p2 = rng.permutation(self.na * self.nb).astype(np.int32)
        # The stacked mHC heads (mhc_*: one row block per layer).
        self.phi_pre = _cq_tensor(rng, layers * n, n * D, 4, G, self.cb4)
        self.phi_post = _cq_tensor(rng, layers * n, n * D, 4, G, self.cb4)
        self.phi_res = _cq_tensor(rng, layers * n * n, n * D, 4, G, self.cb4)
        self.layers = []
        for _ in range(layers):
            L = {}
            for k in ("norm_in", "post_norm", "pre_hada", "q_norm", "k_norm"):
                L[k] = vec(self.qk if k in ("q_norm", "k_norm") else D)
            L["attn_gate"] = float(rng.normal(0.0, 0.5))
            qw, kw, vw = self.heads * self.qk, self.kv_heads * self.qk, self.kv_heads * self.vd
            for k, o in (("q_proj", qw), ("k_proj", kw), ("v_proj", vw), ("gate_proj", self.heads * self.vd),
                         ("out_proj", D)):
                L[k] = _cq_tensor(rng, o, D if k != "out_proj" else self.heads * self.vd, 2, G, self.cb2)
            for k, w in (("q_taps", qw), ("k_taps", kw), ("v_taps", vw)):
                t = rng.normal(0.0, 0.1, size=(self.taps, w)).astype(np.float32)
                t[0] += 1.0
                L[k] = t
            nn_ = self.na * self.nb
            for k in ("d1", "d2", "d3", "d4"):
                L[k] = vec(nn_, 1.0)
            L["b2"] = vec(nn_)
            for s in range(3):
                L[f"w{s + 1}a"] = rng.normal(0.0, 1.0 / np.sqrt(self.na), size=(self.na, self.na)).astype(np.float32)
                L[f"w{s + 1}b"] = rng.normal(0.0, 1.0 / np.sqrt(self.nb), size=(self.nb, self.nb)).astype(np.float32)
            L["cond_v"] = rng.normal(0.0, 0.02, size=(D, self.rank)).astype(np.float32)
            L["cond_u"] = rng.normal(0.0, 0.02, size=(self.rank, nn_)).astype(np.float32)
            # cross-attention (crossNN.*)
            for k in ("x_norm_in", "x_post_norm"):
                L[k] = vec(D)
            for k in ("x_q_norm", "x_k_norm"):
                L[k] = vec(self.x_qk)
            L["x_attn_gate"] = float(rng.normal(0.0, 0.5))
            xq, xv = self.x_heads * self.x_qk, self.x_heads * self.x_vd
            for k, o, i in (("x_q_proj", xq, D), ("x_k_proj", xq, D), ("x_v_proj", xv, D), ("x_gate_proj", xv, D),
                            ("x_out_proj", D, xv)):
                L[k] = _cq_tensor(rng, o, i, 2, G, self.cb2)
            # this layer's mHC scalars and biases (mhc_a_*, mhc_b_*)
            L["a_pre"], L["a_post"], L["a_res"] = (float(v) for v in 0.1 + rng.normal(0.0, 0.02, size=3))
            L["b_pre"], L["b_post"] = vec(n, 0.0, 0.1), vec(n, 0.0, 0.1)
            L["b_res"] = (2.0 * np.eye(n) + rng.normal(0.0, 0.1, size=(n, n))).astype(np.float32).reshape(-1)
            self.layers.append(L)
        self.sites = []
        for lay in self.site_layers:
            S = {"layer": lay,
                 "tables": _cq_tensor(rng, self.n_tables * slots, self.sub, 2, G, self.cb2),
                 "key_proj": _cq_tensor(rng, D, self.n_tables * self.sub, 2, G, self.cb2),
                 "value_proj": _cq_tensor(rng, D, self.n_tables * self.sub, 2, G, self.cb2)}
            t = rng.normal(0.0, 0.1, size=(self.etaps, D)).astype(np.float32)
            t[0] += 1.0
            S["taps"] = t
            self.sites.append(S)

    def phi_rows(self, name: str, l: int):
        """Layer l's row range of a stacked φ (mhc.go:94-96)."""
        n = self.lanes
        per = n * n if name == "phi_res" else n
        return l * per, (l + 1) * per


class EncoderWeights:
    """A synthetic Whistle encoder stack (encNN.*, enc.mhc_*, enc.final_norm;
    the shapes of the exported file's map): sizes as attributes, CQ tensors
    as Packed (2-bit projections, pw1 and pw2; 4-bit φ), float tensors as
    float32 arrays; per-layer tensors in ``layers[l]`` keyed by the .cact
    names without the prefix, the FFN1 HadamardMLP under ``hada_0.*`` and
    the FFN2 one under ``hada.*``."""

    def __init__(self, seed: int = 5000, layers: int = 8):
        rng = np.random.default_rng(seed)
        self.seed = seed
        self.dim, self.lanes, self.n_layers = 512, 4, layers
        self.heads, self.kv_heads, self.qk, self.vd = 8, 2, 48, 64
        self.na, self.nb, self.rank = 16, 32, 8
        self.dw_k = 9
        self.rope_theta, self.rope_len = 1e5, 1536
        G = 128
        self.cb2, self.cb4 = lloyd_max_codebook(2, G), lloyd_max_codebook(4, G)
        D, n = self.dim, self.lanes

        def vec(k, mean=0.0, sd=0.02):
            return (mean + rng.normal(0.0, sd, size=k)).astype(np.float32)

        def mlp(L, pre):
            nn_ = self.na * self.nb
            for k in ("d1", "d2", "d3", "d4"):
                L[pre + k] = vec(nn_, 1.0)
            L[pre + "b2"] = vec(nn_)
            for s in range(3):
                L[f"{pre}w{s + 1}a"] = rng.normal(0.0, 1.0 / np.sqrt(self.na), size=(self.na, self.na)).astype(
                    np.float32)
                L[f"{pre}w{s + 1}b"] = rng.normal(0.0, 1.0 / np.sqrt(self.nb), size=(self.nb, self.nb)).astype(
                    np.float32)
            L[pre + "cond_v"] = rng.normal(0.0, 0.02, size=(D, self.rank)).astype(np.float32)
            L[pre + "cond_u"] = rng.normal(0.0, 0.02, size=(self.rank, nn_)).astype(np.float32)

        self.final_norm = vec(D)
        self.hada_p1 = rng.permutation(self.na * self.nb).astype(np.int32)
        self.hada_p2 = rng.permutation(self.na * self.nb).astype(np.int32)
        self.phi_pre = _cq_tensor(rng, layers * n, n * D, 4, G, self.cb4)
        self.phi_post = _cq_tensor(rng, layers * n, n * D, 4, G, self.cb4)
        self.phi_res = _cq_tensor(rng, layers * n * n, n * D, 4, G, self.cb4)
        self.layers = []
        qw, kw, vw, ow = self.heads * self.qk, self.kv_heads * self.qk, self.kv_heads * self.vd, self.heads * self.vd
        for _ in range(layers):
            L = {}
            for k in ("pre_hada_0", "norm_in", "post_norm", "conv_norm", "conv_out_norm", "pre_hada"):
                L[k] = vec(D)
            for k in ("q_norm", "k_norm"):
                L[k] = vec(self.qk)
            L["attn_gate"] = float(rng.normal(0.0, 0.5))
            for k, o, i in (("q_proj", qw, D), ("k_proj", kw, D), ("v_proj", vw, D), ("gate_proj", ow, D),
                            ("out_proj", D, ow), ("pw1", 2 * D, D), ("pw2", D, D)):
                L[k] = _cq_tensor(rng, o, i, 2, G, self.cb2)
            dw = rng.normal(0.0, 0.1, size=(self.dw_k, D)).astype(np.float32)
            dw[self.dw_k // 2] += 1.0
            L["dw"] = dw
            mlp(L, "hada_0.")
            mlp(L, "hada.")
            L["a_pre"], L["a_post"], L["a_res"] = (float(v) for v in 0.1 + rng.normal(0.0, 0.02, size=3))
            L["b_pre"], L["b_post"] = vec(n, 0.0, 0.1), vec(n, 0.0, 0.1)
            L["b_res"] = (2.0 * np.eye(n) + rng.normal(0.0, 0.1, size=(n, n))).astype(np.float32).reshape(-1)
            self.layers.append(L)
        # The conv stem (stem.*: 3x3 kernels as (9, C), taps time-major;
        # CQ2 pointwise and output products) and the front end's mel bank.
        C = self.stem_channels = 128
        self.stem_w = rng.normal(0.0, 0.4, size=(9, C)).astype(np.float32)
        self.stem_dw_1 = rng.normal(0.0, 0.4, size=(9, C)).astype(np.float32)
        self.stem_dw_2 = rng.normal(0.0, 0.4, size=(9, C)).astype(np.float32)
        self.stem_pw_1 = _cq_tensor(rng, C, C, 2, G, self.cb2, rms=0.08)
        self.stem_pw_2 = _cq_tensor(rng, C, C, 2, G, self.cb2, rms=0.08)
        self.stem_out = _cq_tensor(rng, D, 10 * C, 2, G, self.cb2, rms=0.05)
        self.mel_filters = triangular_mel_bank()

    def phi_rows(self, name: str, l: int):
        """Layer l's row range of a stacked φ (mhc.go:94-96)."""
        n = self.lanes
        per = n * n if name == "phi_res" else n
        return l * per, (l + 1) * per


def triangular_mel_bank(bins: int = 257, mels: int = 80, rate: float = 16000.0) -> np.ndarray:
    """A synthetic (bins, mels) filterbank standing in for the exported
    audio.mel_filters: triangles evenly spaced on the HTK mel scale over
    0 .. rate/2, each channel's non-zero bins contiguous."""
    def mel(f):
        return 2595.0 * np.log10(1.0 + f / 700.0)

    def hz(m):
        return 700.0 * (10.0 ** (m / 2595.0) - 1.0)

    edges = hz(np.linspace(0.0, mel(rate / 2), mels + 2))
    f = np.arange(bins) * rate / (2 * (bins - 1))
    w = np.zeros((bins, mels), np.float32)
    for m in range(mels):
        lo, c, hi = edges[m], edges[m + 1], edges[m + 2]
        up = (f - lo) / (c - lo)
        down = (hi - f) / (hi - c)
        w[:, m] = np.maximum(0.0, np.minimum(up, down)) * (2.0 / (hi - lo))
    return w


def audio(rng: np.random.Generator, clips: int, samples: int) -> np.ndarray:
    """Synthetic 16 kHz clips [clips][samples]: a few tones with slow
    amplitude changes over noise, peak about 0.5."""
    t = np.arange(samples) / 16000.0
    out = np.zeros((clips, samples), np.float32)
    for c in range(clips):
        x = 0.02 * rng.normal(size=samples)
        for _ in range(4):
            f0, a = rng.uniform(80, 4000), rng.uniform(0.05, 0.15)
            x += a * np.sin(2 * np.pi * f0 * t + rng.uniform(0, 6.28)) * (1 + 0.5 * np.sin(2 * np.pi * 0.7 * t))
        out[c] = x.astype(np.float32)
    return out


def stem_output(rng: np.random.Generator, clips: int, frames: int = 375, dim: int = 512) -> np.ndarray:
    """Synthetic stem outputs [clips][frames][dim] (the encoder stack's
    input), ~N(0, 1)."""
    return rng.normal(0.0, 1.0, size=(clips, frames, dim)).astype(np.float32)


def encoder_output(rng: np.random.Generator, streams: int, frames: int = 375, dim: int = 512) -> np.ndarray:
    """Synthetic encoder outputs [streams][frames][dim] (the final-normed
    memory the decoder reads), ~N(0, 1)."""
    return rng.normal(0.0, 1.0, size=(streams, frames, dim)).astype(np.float32)
