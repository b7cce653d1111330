"""Weights by name over a .cact file (internal/weights), the decoder's
weight set loaded from it, and a synthetic whistle.cact writer.

``Open``/``Parse`` check every record against the name map and read the
geometry from the header and the 13-float audio manifest
(weights/cact.go:42-73, config.go:100-145). ``Source.Matrix`` serves a CQ
record packed, as the reference's Packer does (weights/cact.go Matrix), so
the device decoder builds on the stored bytes with no float copy.

``decoder_weights(src)`` assembles what ``decoder.Decoder`` (and the CPU
restatement) takes, by the names internal/decoder loads: ``embedding``,
``layerNN.*`` (needle.LoadBlock), ``crossNN.*`` (decoder/cross.go),
the stack's ``mhc_*`` (needle.LoadMHC), ``hada_p1/p2``, ``engramS.*`` at the
header's sites (needle.LoadEngram) and ``final_norm``
(decoder/decoder.go:89-113, 330-387).

``write_whistle_cact(w)`` lays a synthetic decoder out as whistle.cact:
all 681 records of the Whistle map in order, with the dtypes and shapes of
the exported file; the decoder records carry w's tensors, the audio
records (encoder, stem, mel filterbank, tokenizer) seeded random values of
their shapes.
"""

from __future__ import annotations

import math
from typing import Optional, Sequence, Union

import numpy as np

from . import cact
from .cq import Packed

MANIFEST_NAME = "audio.manifest"
MANIFEST_LEN = 13
ROPE_LEN = 512  # decoder.go:63 ropeLen


class WeightsError(ValueError):
    """A weight file that does not fit the name map or the model."""


class Config:
    """weights/config.go Config: the decoder geometry from the header, the
    encoder and front end from the audio manifest."""

    _MANIFEST = ("Text", "EncLayers", "EncLanes", "ConvKernel", "Stem", "StemStages", "Mels", "Rate", "FFT", "Win",
                 "Hop")

    def __init__(self, h: cact.Header, manifest: np.ndarray):
        self.Vocab, self.Dim, self.HadaN = h.Vocab, h.DModel, h.HadaN
        self.Heads, self.KVHeads, self.QKDim, self.VDim = h.NumHeads, h.NumKVHeads, h.QKHeadDim, h.VHeadDim
        self.DecLayers, self.Lanes, self.Taps = h.NumLayers, h.MHCLanes, h.QKVConvTaps
        self.Sites, self.Orders = h.Sites(), h.Orders()
        self.Slots, self.Tables = h.EngramSlots, h.NumEngramTables
        self.Rope, self.MaxTokens = float(h.RopeTheta), h.MaxSeqLen
        v = np.asarray(manifest, np.float32)
        if v.size != MANIFEST_LEN:
            raise WeightsError(f"weights: audio manifest has {v.size} values, want {MANIFEST_LEN}")
        if v[0] != 0xCAE:
            raise WeightsError(f"weights: audio manifest magic {v[0]:g}, want {0xCAE}")
        if v[1] != 1:
            raise WeightsError(f"weights: audio manifest version {v[1]:g}, want 1")
        for k, name in enumerate(self._MANIFEST):
            x = v[2 + k]
            if x < 0 or x != np.float32(int(x)):
                raise WeightsError(f"weights: audio manifest value {2 + k} = {x:g} is not a count")
            setattr(self, name, int(x))


class Source:
    """A .cact file seen through its name map (weights/cact.go Cact)."""

    def __init__(self, f: cact.File, names: Optional[Sequence[cact.Entry]] = None):
        entries = list(names) if names is not None else cact.whistle_names()
        if len(entries) != f.Len():
            raise WeightsError(f"weights: {len(entries)} names for {f.Len()} tensors")
        self._index = {}
        for i, e in enumerate(entries):
            if e.Name in self._index:
                raise WeightsError(f"weights: name {e.Name} appears twice")
            self._index[e.Name] = i
            rec = f.Record(i)
            blob = rec.DType == cact.RAW
            if blob != (e.Shape is None) or (not blob and tuple(rec.Dims()) != tuple(e.Shape)):
                raise WeightsError(f"weights: {e.Name}: record {i} is {cact.dtype_name(rec.DType)} "
                                   f"{cact._go_list(rec.Dims())}, the map says "
                                   f"{cact._go_list(e.Shape or ())}")
        self.file, self.entries = f, entries
        if MANIFEST_NAME not in self._index:
            raise WeightsError("weights: the name map has no audio.manifest")
        self._config = Config(f.Header(), f.FP32(self._index[MANIFEST_NAME]))

    def Config(self) -> Config:
        return self._config

    def _i(self, name: str) -> int:
        i = self._index.get(name)
        if i is None:
            raise WeightsError(f"weights: no tensor {name}")
        return i

    def Has(self, name: str) -> bool:
        return name in self._index

    def Shape(self, name: str) -> list[int]:
        return self.file.Record(self._i(name)).Dims()

    def Tensor(self, name: str) -> np.ndarray:
        """The record's float32 values (CQ records dequantised), shaped."""
        i = self._i(name)
        rec = self.file.Record(i)
        v = self.file.CQ(i) if rec.DType == cact.CQ else self.file.Float32(i)
        return v.reshape(rec.Dims()) if rec.Dims() else v

    def Matrix(self, name: str) -> Packed:
        """A CQ record in its stored form for cq.New (2- and 4-bit only,
        the widths the lut kernels take)."""
        i = self._i(name)
        rec = self.file.Record(i)
        if rec.DType != cact.CQ:
            raise WeightsError(f"weights: {name} is {cact.dtype_name(rec.DType)}, not CQ")
        if rec.Bits not in (2, 4):
            raise WeightsError(f"weights: {name} is {rec.Bits}-bit CQ; the kernels take 2 and 4 bits")
        return self.file.CQPacked(i)

    def Raw(self, name: str) -> bytes:
        return self.file.Raw(self._i(name))


def Parse(data: bytes, names: Optional[Sequence[cact.Entry]] = None) -> Source:
    return Source(cact.Parse(data), names)


def Open(path: str, names: Optional[Sequence[cact.Entry]] = None) -> Source:
    return Source(cact.Open(path), names)


class DecoderTensors:
    """The decoder's weight set as ``decoder.Decoder`` takes it (the
    attributes of synth.DecoderWeights), loaded from a Source."""

    def phi_rows(self, name: str, l: int):
        """Layer l's row range of a stacked φ (mhc.go:94-96)."""
        per = self.lanes * self.lanes if name == "phi_res" else self.lanes
        return l * per, (l + 1) * per


def _perm(src: Source, name: str, n: int) -> np.ndarray:
    """hadamard.go:143 perm: a permutation of n stored as float32."""
    v = src.Tensor(name).reshape(-1)
    if v.size != n:
        raise WeightsError(f"weights: {name} has {v.size} values, want {n}")
    seen = np.zeros(n, bool)
    out = np.empty(n, np.int32)
    for i, f in enumerate(v):
        k = int(f)
        if np.float32(k) != f or k < 0 or k >= n or seen[k]:
            raise WeightsError(f"weights: {name} is not a permutation of {n} (entry {i} = {f:g})")
        seen[k] = True
        out[i] = k
    return out


def decoder_weights(src: Source) -> DecoderTensors:
    """The decoder's tensors by the names internal/decoder loads, geometry
    from the header (decoder.go:89-113, 330-387)."""
    cfg = src.Config()
    w = DecoderTensors()
    w.embedding = src.Matrix("embedding")
    w.vocab, w.dim = w.embedding.Out, w.embedding.In
    if cfg.Vocab and cfg.Vocab != w.vocab:
        raise WeightsError(f"weights: embedding has {w.vocab} rows, the header {cfg.Vocab}")
    w.lanes, w.n_layers = cfg.Lanes, cfg.DecLayers
    w.heads, w.kv_heads, w.qk, w.vd, w.taps = cfg.Heads, cfg.KVHeads, cfg.QKDim, cfg.VDim, cfg.Taps
    w.rope_theta, w.rope_len = cfg.Rope, ROPE_LEN
    w.final_norm = src.Tensor("final_norm").astype(np.float32)
    w.hada_p1 = _perm(src, "hada_p1", cfg.HadaN)
    w.hada_p2 = _perm(src, "hada_p2", cfg.HadaN)
    a = {k: src.Tensor("mhc_a_" + k) for k in ("pre", "post", "res")}
    b = {k: src.Tensor("mhc_b_" + k) for k in ("pre", "post", "res")}
    w.phi_pre, w.phi_post, w.phi_res = (src.Matrix("mhc_phi_" + k) for k in ("pre", "post", "res"))
    w.layers = []
    for l in range(cfg.DecLayers):
        p, x = f"layer{l:02d}.", f"cross{l:02d}."
        L = {}
        for k in ("norm_in", "post_norm", "pre_hada", "q_norm", "k_norm", "q_taps", "k_taps", "v_taps", "d1", "d2",
                  "b2", "d3", "d4", "w1a", "w1b", "w2a", "w2b", "w3a", "w3b", "cond_v", "cond_u"):
            L[k] = src.Tensor(p + k).astype(np.float32)
        L["attn_gate"] = float(src.Tensor(p + "attn_gate").reshape(-1)[0])
        for k in ("q_proj", "k_proj", "v_proj", "gate_proj", "out_proj"):
            L[k] = src.Matrix(p + k)
            L["x_" + k] = src.Matrix(x + k)
        for k in ("norm_in", "post_norm", "q_norm", "k_norm"):
            L["x_" + k] = src.Tensor(x + k).astype(np.float32)
        L["x_attn_gate"] = float(src.Tensor(x + "attn_gate").reshape(-1)[0])
        L["a_pre"], L["a_post"], L["a_res"] = (float(a[k][l]) for k in ("pre", "post", "res"))
        L["b_pre"], L["b_post"] = b["pre"][l].astype(np.float32), b["post"][l].astype(np.float32)
        L["b_res"] = b["res"][l].astype(np.float32).reshape(-1)
        w.layers.append(L)
    L0 = w.layers[0]
    w.x_qk = int(L0["x_q_norm"].size)
    w.x_heads = L0["x_q_proj"].Out // w.x_qk
    w.x_vd = L0["x_v_proj"].Out // w.x_heads
    w.na, w.nb = int(L0["w1a"].shape[0]), int(L0["w1b"].shape[0])
    w.rank = int(L0["cond_v"].shape[1])
    orders, tables = cfg.Orders, cfg.Tables
    if not orders or tables <= 0 or tables % len(orders) or min(orders) < 1:
        raise WeightsError(f"weights: {tables} engram tables for orders {orders}")
    w.orders = [o for o in orders for _ in range(tables // len(orders))]  # engram.go:80-86
    w.n_tables, w.max_order = tables, max(orders)
    w.site_layers = list(cfg.Sites)
    w.sites = []
    for s, layer in enumerate(cfg.Sites):
        p = f"engram{s}."
        S = {"layer": int(layer), "tables": src.Matrix(p + "tables"), "key_proj": src.Matrix(p + "key_proj"),
             "value_proj": src.Matrix(p + "value_proj"), "taps": src.Tensor(p + "taps").astype(np.float32)}
        if S["tables"].Out % tables:
            raise WeightsError(f"weights: {p}tables has {S['tables'].Out} rows, not a multiple of {tables} tables")
        w.sites.append(S)
    if w.sites:
        w.slots = w.sites[0]["tables"].Out // tables
        w.sub = w.sites[0]["tables"].In
        w.etaps = int(w.sites[0]["taps"].shape[0])
    else:
        w.slots, w.sub, w.etaps = cfg.Slots, 0, 0
    w.cb2 = np.asarray(L0["q_proj"].Codebook, np.float32)
    w.cb4 = np.asarray(w.embedding.Codebook, np.float32)
    return w


class EncoderTensors:
    """The encoder's weight set as ``encoder.Encoder`` takes it (the
    attributes of synth.EncoderWeights), loaded from a Source."""

    def phi_rows(self, name: str, l: int):
        """Layer l's row range of a stacked φ (mhc.go:94-96)."""
        per = self.lanes * self.lanes if name == "phi_res" else self.lanes
        return l * per, (l + 1) * per


ENC_ROPE_LEN = 4096  # RoPE positions the device tables hold (encoder.go:276 rope builds them per call)
_ENC_FLOATS = ("pre_hada_0", "norm_in", "post_norm", "conv_norm", "conv_out_norm", "pre_hada", "q_norm", "k_norm",
               "dw")
_ENC_MLP = ("d1", "d2", "b2", "d3", "d4", "w1a", "w1b", "w2a", "w2b", "w3a", "w3b", "cond_v", "cond_u")
_ENC_CQ = ("q_proj", "k_proj", "v_proj", "gate_proj", "out_proj", "pw1", "pw2")


def encoder_weights(src: Source) -> EncoderTensors:
    """The encoder's tensors by the names internal/encoder loads
    (encoder.go:50 LoadInt8, block.go:42 loadBlock, mhc.go LoadMHC with the
    "enc." prefix, stem.go:43 loadStem, frontend/mel.go:67 LoadMelBank),
    the layer and lane counts from the audio manifest, the widths from the
    shapes (Best(): RoPE θ = 1e5, the shared Hadamard permutations)."""
    cfg = src.Config()
    w = EncoderTensors()
    w.n_layers, w.lanes = cfg.EncLayers, cfg.EncLanes
    w.final_norm = src.Tensor("enc.final_norm").astype(np.float32)
    w.dim = int(w.final_norm.size)
    w.hada_p1 = _perm(src, "hada_p1", cfg.HadaN)
    w.hada_p2 = _perm(src, "hada_p2", cfg.HadaN)
    a = {k: src.Tensor("enc.mhc_a_" + k) for k in ("pre", "post", "res")}
    b = {k: src.Tensor("enc.mhc_b_" + k) for k in ("pre", "post", "res")}
    w.phi_pre, w.phi_post, w.phi_res = (src.Matrix("enc.mhc_phi_" + k) for k in ("pre", "post", "res"))
    w.layers = []
    for l in range(cfg.EncLayers):
        p = f"enc{l:02d}."
        L = {k: src.Tensor(p + k).astype(np.float32) for k in _ENC_FLOATS}
        for m in ("hada_0.", "hada."):
            for k in _ENC_MLP:
                L[m + k] = src.Tensor(p + m + k).astype(np.float32)
        L["attn_gate"] = float(src.Tensor(p + "attn_gate").reshape(-1)[0])
        for k in _ENC_CQ:
            L[k] = src.Matrix(p + k)
        L["a_pre"], L["a_post"], L["a_res"] = (float(a[k][l]) for k in ("pre", "post", "res"))
        L["b_pre"], L["b_post"] = b["pre"][l].astype(np.float32), b["post"][l].astype(np.float32)
        L["b_res"] = b["res"][l].astype(np.float32).reshape(-1)
        w.layers.append(L)
    L0 = w.layers[0]
    w.qk = int(L0["q_norm"].size)
    w.heads, w.kv_heads = L0["q_proj"].Out // w.qk, L0["k_proj"].Out // w.qk
    w.vd = L0["v_proj"].Out // w.kv_heads
    w.dw_k = int(L0["dw"].shape[0])
    w.na, w.nb = int(L0["hada.w1a"].shape[0]), int(L0["hada.w1b"].shape[0])
    w.rank = int(L0["hada.cond_v"].shape[1])
    w.rope_theta, w.rope_len = 1e5, ENC_ROPE_LEN
    w.stem_w, w.stem_dw_1, w.stem_dw_2 = (src.Tensor("stem." + k).astype(np.float32) for k in ("w", "dw_1", "dw_2"))
    w.stem_pw_1, w.stem_pw_2, w.stem_out = (src.Matrix("stem." + k) for k in ("pw_1", "pw_2", "out"))
    w.stem_channels = int(w.stem_w.shape[1])
    w.mel_filters = src.Tensor("audio.mel_filters").astype(np.float32)
    w.cb2 = np.asarray(L0["q_proj"].Codebook, np.float32)
    w.cb4 = np.asarray(w.phi_pre.Codebook, np.float32)
    return w


# ---- a synthetic whistle.cact -------------------------------------------

# The audio manifest of a Whistle export: magic, version, then text vocab,
# encoder layers and lanes, conv kernel, stem width and stages, mels,
# sample rate, FFT, window and hop (weights/config.go:67 manifestFields).
WHISTLE_MANIFEST = [0xCAE, 1, 8192, 8, 4, 9, 128, 3, 80, 16000, 512, 400, 160]


def lloyd_max_unit(bits: int, iters: int = 2000) -> np.ndarray:
    """The unit-Gaussian Lloyd-Max levels for 2**bits cells (Lloyd's
    algorithm: each level the conditional mean of its cell, each boundary
    the midpoint of its neighbours), float64."""
    n = 1 << bits
    levels = np.linspace(-2.0, 2.0, n)
    sq2 = math.sqrt(2.0)

    def pdf(t):
        return math.exp(-0.5 * t * t) / math.sqrt(2 * math.pi)

    def cdf(t):
        return 0.5 * (1 + math.erf(t / sq2))

    for _ in range(iters):
        edges = [-math.inf] + [(levels[i] + levels[i + 1]) / 2 for i in range(n - 1)] + [math.inf]
        new = []
        for i in range(n):
            lo, hi = edges[i], edges[i + 1]
            mass = cdf(hi) - cdf(lo)
            new.append(((pdf(lo) if lo > -math.inf else 0.0) - (pdf(hi) if hi < math.inf else 0.0)) / mass)
        levels = np.array(new)
    return levels


def whistle_header(w, max_seq: int = 320) -> cact.Header:
    """The header of a Whistle-geometry file for decoder weights w."""
    orders = sorted(set(w.orders))
    return cact.Header(KVBits=8, Vocab=w.vocab, DModel=w.dim, NumHeads=w.heads, NumKVHeads=w.kv_heads,
                       NumLayers=len(w.layers), QKHeadDim=w.qk, VHeadDim=w.vd, MaxSeqLen=max_seq,
                       HadaN=w.na * w.nb, MHCLanes=w.lanes, QKVConvTaps=w.taps, EngramSlots=w.slots,
                       EngramSubDim=w.sub, NumEngramTables=w.n_tables, EngramConvTaps=w.etaps,
                       EngramConvDilation=max(orders), NumEngramOrders=len(orders),
                       EngramOrders=tuple(orders) + (0,) * (4 - len(orders)),
                       NumEngramSites=len(w.sites),
                       EngramSites=tuple(s["layer"] for s in w.sites) + (0,) * (16 - len(w.sites)),
                       RopeTheta=float(w.rope_theta))


def write_whistle_cact(w, path: Optional[str] = None, seed: int = 0, enc=None) -> bytes:
    """A whistle.cact holding decoder weights w (synth.DecoderWeights of
    Whistle's shapes: vocab 8199, 8 layers, 18,432 engram slots) and, with
    enc (synth.EncoderWeights of Whistle's shapes, the same hada_p1/hada_p2:
    the file holds one pair), the encoder's, the stem's and the mel bank's;
    without enc those audio tensors are seeded random. Returns the bytes and
    writes them to path if given. The file's CQ group is w's (one group for
    the whole file, as _pack_cact writes), its codebook w's 2- and 4-bit
    levels and the 3-bit Lloyd-Max levels over sqrt(group)."""
    from .synth import _cq_tensor

    group = int(w.embedding.Group)
    rng = np.random.default_rng(seed)
    cb3 = (lloyd_max_unit(3) / math.sqrt(group)).astype(np.float32)
    codebook = np.concatenate([np.asarray(w.cb2, np.float32), cb3, np.asarray(w.cb4, np.float32)])
    entries = cact.whistle_names()
    layers = w.layers

    def dec_value(name):
        """w's tensor for a decoder record, or None for an audio record."""
        if name == "embedding":
            return w.embedding
        if name == "final_norm":
            return w.final_norm
        if name in ("hada_p1", "hada_p2"):
            return np.asarray(getattr(w, name), np.float32)
        if name.startswith("mhc_"):
            k = name[4:]
            if k.startswith("phi_"):
                return getattr(w, k)
            if k.startswith("a_"):
                return np.array([L[k] for L in layers], np.float32)
            vals = np.stack([np.asarray(L[k], np.float32) for L in layers])
            return vals.reshape(len(layers), w.lanes, w.lanes) if k == "b_res" else vals
        if name.startswith("layer") or name.startswith("cross"):
            l, k = int(name[5:7]), name.split(".", 1)[1]
            key = ("x_" + k) if name.startswith("cross") else k
            v = layers[l][key]
            return np.array([v], np.float32) if np.isscalar(v) else v
        if name.startswith("engram"):
            s, k = int(name[6]), name.split(".", 1)[1]
            return w.sites[s][k]
        return None

    if enc is not None and not (np.array_equal(enc.hada_p1, w.hada_p1) and np.array_equal(enc.hada_p2, w.hada_p2)):
        raise WeightsError("weights: the encoder's hada_p1/hada_p2 differ from the decoder's (a file holds one pair)")

    def enc_value(name):
        """enc's tensor for an encoder, stem or mel-bank record, else None."""
        if enc is None:
            return None
        if name == "enc.final_norm":
            return enc.final_norm
        if name.startswith("enc.mhc_"):
            k = name[8:]
            if k.startswith("phi_"):
                return getattr(enc, k)
            if k.startswith("a_"):
                return np.array([L[k] for L in enc.layers], np.float32)
            vals = np.stack([np.asarray(L[k], np.float32) for L in enc.layers])
            return vals.reshape(len(enc.layers), enc.lanes, enc.lanes) if k == "b_res" else vals
        if name.startswith("enc") and name[3:5].isdigit():
            v = enc.layers[int(name[3:5])][name.split(".", 1)[1]]
            return np.array([v], np.float32) if np.isscalar(v) else v
        if name.startswith("stem."):
            return getattr(enc, "stem_" + name[5:])
        if name == "audio.mel_filters":
            return enc.mel_filters
        return None

    tensors = []
    for e in entries:
        dtype, bits = cact.whistle_storage(e.Name)
        v = dec_value(e.Name)
        if v is None:
            v = enc_value(e.Name)
        if dtype == cact.RAW:
            tensors.append(cact.raw_tensor(np.uint32(w.vocab).tobytes() + b"synthetic tokenizer"))
            continue
        if e.Name == MANIFEST_NAME:
            v = np.array(WHISTLE_MANIFEST, np.float32)
        if v is None:  # an audio record: seeded values of its shape
            if dtype == cact.CQ:
                cb = w.cb4 if bits == 4 else w.cb2
                v = _cq_tensor(rng, e.Shape[0], e.Shape[1], bits, group, cb)
            elif e.Name == "audio.mel_filters":
                v = np.abs(rng.normal(0.0, 0.01, size=e.Shape)).astype(np.float32)
            else:
                v = rng.normal(0.0, 0.05, size=e.Shape).astype(np.float32)
        if dtype == cact.CQ:
            if not isinstance(v, Packed) or (v.Out, v.In) != tuple(e.Shape) or v.Bits != bits:
                raise WeightsError(f"weights: {e.Name}: want a {bits}-bit CQ {e.Shape}")
            if v.Group != group:
                raise WeightsError(f"weights: {e.Name}: CQ group {v.Group}, the file's is {group}")
            tensors.append(cact.cq_tensor(v))
            continue
        v = np.asarray(v, np.float32)
        if v.size != int(np.prod(e.Shape)):
            raise WeightsError(f"weights: {e.Name}: {v.size} values for shape {e.Shape}")
        v = v.reshape(e.Shape)
        tensors.append(cact.fp32_tensor(v) if dtype == cact.FP32 else cact.fp16_tensor(v))
    data = cact.encode(whistle_header(w), codebook, tensors)
    if path is not None:
        with open(path, "wb") as fh:
            fh.write(data)
    return data


def load_decoder(path_or_data: Union[str, bytes], names: Optional[Sequence[cact.Entry]] = None) -> DecoderTensors:
    """The decoder's weight set from a .cact file (a path or its bytes)."""
    src = Parse(path_or_data, names) if isinstance(path_or_data, (bytes, bytearray)) else Open(path_or_data, names)
    return decoder_weights(src)


def load_encoder(path_or_data: Union[str, bytes], names: Optional[Sequence[cact.Entry]] = None) -> EncoderTensors:
    """The encoder's weight set from a .cact file (a path or its bytes)."""
    src = Parse(path_or_data, names) if isinstance(path_or_data, (bytes, bytearray)) else Open(path_or_data, names)
    return encoder_weights(src)
