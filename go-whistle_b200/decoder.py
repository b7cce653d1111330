"""The decoder head's scale and greedy choice on the B200 library:
``logits`` (internal/decoder/decoder.go:508-523, the head scale) and
``argmax`` (internal/decoder/greedy.go:182) for rows of vocabulary logits in
device memory, so a greedy decode step brings back one token id per stream.
"""

from __future__ import annotations

import ctypes

from ._lib import Panic, WC_ERR_INVALID, check, lib

__all__ = ["HeadArgmax", "Decoder"]


def HeadArgmax(y, rows: int, vocab: int, head: float = 1.0, logits=None, idx=None):
    """idx[r] = argmax over row r of y·head (y·head only when head != 1; the
    first index of the largest value, a NaN at 0 gives 0). y, logits (None,
    or y itself for the reference's in-place scale) and idx are CUDA tensors
    (float32 [rows·vocab], int32 [rows]); returns idx."""
    import torch

    if rows < 0 or vocab < 0 or y.numel() != rows * vocab:
        raise Panic(WC_ERR_INVALID, f"decoder: head of {rows} rows of {vocab} logits on {y.numel()} values")
    for t in (y, logits):
        if t is not None and (not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous()):
            raise Panic(WC_ERR_INVALID, "decoder: logits must be contiguous float32 CUDA tensors")
    if idx is None:
        idx = torch.empty(rows, dtype=torch.int32, device=y.device)
    if logits is not None and logits.numel() != rows * vocab:
        raise Panic(WC_ERR_INVALID, f"decoder: {logits.numel()} logits for {rows} rows of {vocab}")
    if idx.numel() != rows or idx.dtype != torch.int32 or not idx.is_cuda:
        raise Panic(WC_ERR_INVALID, "decoder: idx must be an int32 CUDA tensor of one entry per row")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    check(lib().wc_head_argmax(ctypes.c_void_p(y.data_ptr()), rows, vocab, float(head),
                               ctypes.c_void_p(logits.data_ptr()) if logits is not None else None,
                               ctypes.c_void_p(idx.data_ptr()), stream))
    return idx


# ------------------------------------------------------------------ Decoder
#
# internal/decoder's Decoder (decoder.go:25) on the device: Load builds it
# from a weight set, Memory projects the encoder output (decoder.go:157),
# Extend feeds one token per stream (decoder.go:252), GreedyMemory runs
# greedy.go:40 for every stream without leaving the device.

_f32p = ctypes.c_void_p


class _Layer(ctypes.Structure):
    """wc_decoder_layer (include/whistle_b200.h)."""
    _fields_ = ([(k, _f32p) for k in ("norm_in", "post_norm", "pre_hada")] + [("attn_gate", ctypes.c_float)]
                + [(k, ctypes.c_void_p) for k in ("q_proj", "k_proj", "v_proj", "gate_proj", "out_proj")]
                + [(k, _f32p) for k in ("q_taps", "k_taps", "v_taps", "q_norm", "k_norm", "d1", "d2", "b2", "d3",
                                        "d4", "w1a", "w1b", "w2a", "w2b", "w3a", "w3b", "cond_v", "cond_u",
                                        "x_norm_in", "x_post_norm", "x_q_norm", "x_k_norm")]
                + [("x_attn_gate", ctypes.c_float)]
                + [(k, ctypes.c_void_p) for k in ("x_q_proj", "x_k_proj", "x_v_proj", "x_gate_proj", "x_out_proj")]
                + [(k, ctypes.c_float) for k in ("a_pre", "a_post", "a_res")]
                + [(k, _f32p) for k in ("b_pre", "b_post", "b_res")]
                + [(k, ctypes.c_void_p) for k in ("phi_pre", "phi_post", "phi_res")])


class _Site(ctypes.Structure):
    _fields_ = [("tables", ctypes.c_void_p), ("key_proj", ctypes.c_void_p), ("value_proj", ctypes.c_void_p),
                ("taps", _f32p), ("layer", ctypes.c_int)]


class _Desc(ctypes.Structure):
    _fields_ = ([(k, ctypes.c_int) for k in ("dim", "lanes", "layers", "vocab", "heads", "kv_heads", "qk", "vd",
                                             "taps", "x_heads", "x_qk", "x_vd", "na", "nb", "rank", "n_sites",
                                             "n_tables", "slots", "sub", "etaps")]
                + [("orders", ctypes.c_void_p), ("hada_p1", ctypes.c_void_p), ("hada_p2", ctypes.c_void_p),
                   ("rope_theta", ctypes.c_double), ("rope_len", ctypes.c_int), ("embedding", ctypes.c_void_p),
                   ("final_norm", _f32p), ("layer", ctypes.POINTER(_Layer)), ("site", ctypes.POINTER(_Site))])


WC_DECODER_TENSOR_CORES = 1
WC_DECODER_NO_GRAPH = 2


class BeamOptions(ctypes.Structure):
    """search/options.go:105 Options as wc_beam_options (no Adjust hook)."""

    _fields_ = [("beams", ctypes.c_int), ("max_tokens", ctypes.c_int), ("language", ctypes.c_int),
                ("norm", ctypes.c_int), ("alpha", ctypes.c_double), ("length", ctypes.c_int), ("stop", ctypes.c_int),
                ("admit", ctypes.c_int), ("lang_step", ctypes.c_int)]


def DefaultBeam(**kw) -> BeamOptions:
    """options.go:143 Default, with any field overridden by keyword."""
    o = BeamOptions()
    lib().wc_beam_default(ctypes.addressof(o))
    for k, v in kw.items():
        setattr(o, k, v)
    return o


WC_NORM_NONE, WC_NORM_LEN, WC_NORM_POW, WC_NORM_GNMT = 1, 2, 3, 4
WC_LEN_TEXT, WC_LEN_TEXT_EOS, WC_LEN_SEQ = 1, 2, 3
WC_STOP_ALL, WC_STOP_BEST, WC_STOP_K, WC_STOP_HF = 1, 2, 3, 4
WC_ADMIT_TOPK, WC_ADMIT_ABOVE_LIVE = 1, 2
WC_LANG_ARGMAX, WC_LANG_ARGMAX_SCORED, WC_LANG_BEAM = 1, 2, 3


class Decoder:
    """Whistle's decoder (decoder.go:25) with int8 numerics on the GPU, for
    up to ``max_streams`` independent streams.

    ``w`` is a weight set with the attributes of ``synth.DecoderWeights``
    (CQ tensors as ``cq.Packed``, float tensors as arrays); the CQ tensors
    are uploaded once here (cq.New), the float tensors copied by the
    library. flags: ``WC_DECODER_TENSOR_CORES``, ``WC_DECODER_NO_GRAPH``.
    """

    def __init__(self, w, max_streams: int, max_frames: int = 375, max_positions: int = 80, flags: int = 0):
        import numpy as np

        from . import cq

        self.w, self.flags = w, flags
        self.max_positions = min(max_positions, int(w.rope_len))
        self._keep = []

        def f(a):
            a = np.ascontiguousarray(a, np.float32).reshape(-1)
            self._keep.append(a)
            return a.ctypes.data

        def m(p):
            mat = cq.New(p)
            self._keep.append(mat)
            return mat.handle.value

        def rows(p, lo, hi):
            mat = cq.New(p) if id(p) not in self._stacked else self._stacked[id(p)]
            self._stacked[id(p)] = mat
            v = mat.Rows(lo, hi)
            self._keep.append(v)
            return v.handle.value

        self._stacked = {}
        L = (_Layer * len(w.layers))()
        for l, src in enumerate(w.layers):
            d = L[l]
            for k in ("norm_in", "post_norm", "pre_hada", "q_taps", "k_taps", "v_taps", "q_norm", "k_norm", "d1",
                      "d2", "b2", "d3", "d4", "w1a", "w1b", "w2a", "w2b", "w3a", "w3b", "cond_v", "cond_u",
                      "x_norm_in", "x_post_norm", "x_q_norm", "x_k_norm", "b_pre", "b_post", "b_res"):
                setattr(d, k, f(src[k]))
            for k in ("attn_gate", "x_attn_gate", "a_pre", "a_post", "a_res"):
                setattr(d, k, float(src[k]))
            for k in ("q_proj", "k_proj", "v_proj", "gate_proj", "out_proj", "x_q_proj", "x_k_proj", "x_v_proj",
                      "x_gate_proj", "x_out_proj"):
                setattr(d, k, m(src[k]))
            for k in ("phi_pre", "phi_post", "phi_res"):
                lo, hi = w.phi_rows(k, l)
                setattr(d, k, rows(getattr(w, k), lo, hi))
        S = (_Site * max(1, len(w.sites)))()
        for i, src in enumerate(w.sites):
            S[i].tables, S[i].key_proj, S[i].value_proj = (m(src[k]) for k in ("tables", "key_proj", "value_proj"))
            S[i].taps = f(src["taps"])
            S[i].layer = src["layer"]
        orders = np.ascontiguousarray(w.orders, np.int32)
        p1, p2 = np.ascontiguousarray(w.hada_p1, np.int32), np.ascontiguousarray(w.hada_p2, np.int32)
        self._keep += [orders, p1, p2, L, S]
        desc = _Desc(w.dim, w.lanes, len(w.layers), w.vocab, w.heads, w.kv_heads, w.qk, w.vd, w.taps, w.x_heads,
                     w.x_qk, w.x_vd, w.na, w.nb, w.rank, len(w.sites), w.n_tables, w.slots, w.sub, w.etaps)
        desc.orders, desc.hada_p1, desc.hada_p2 = orders.ctypes.data, p1.ctypes.data, p2.ctypes.data
        desc.rope_theta, desc.rope_len = float(w.rope_theta), int(w.rope_len)
        desc.embedding = m(w.embedding)
        desc.final_norm = f(w.final_norm)
        desc.layer, desc.site = L, S
        h = ctypes.c_void_p()
        check(lib().wc_decoder_create(ctypes.byref(desc), max_streams, max_frames, max_positions, flags,
                                      ctypes.byref(h)))
        self.handle = h
        self.streams = 0

    @classmethod
    def Load(cls, path_or_data, max_streams: int, max_frames: int = 375, max_positions: int = 80, flags: int = 0):
        """decoder.LoadInt8 over a .cact file (a path or its bytes): the
        decoder's tensors by name (weights.decoder_weights), CQ records
        uploaded as stored."""
        from . import weights

        return cls(weights.load_decoder(path_or_data), max_streams, max_frames, max_positions, flags)

    def __del__(self):
        if getattr(self, "handle", None) and self.handle.value:
            lib().wc_decoder_destroy(self.handle)
            self.handle = None

    @staticmethod
    def _stream():
        import torch

        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def Memory(self, enc):
        """decoder.go:157 Memory + NewState for every stream: enc is a CUDA
        float32 tensor [streams, frames, dim]."""
        streams, frames = enc.shape[0], enc.shape[1]
        check(lib().wc_decoder_memory(self.handle, ctypes.c_void_p(enc.data_ptr()), streams, frames, self._stream()))
        self.streams = streams

    def MemoryBeams(self, enc, beams: int):
        """Memory for a beam search: enc is a CUDA float32 tensor [clips,
        frames, dim]; the decoder then runs clips × beams streams whose
        beams share their clip's cross memory."""
        clips, frames = enc.shape[0], enc.shape[1]
        check(lib().wc_decoder_memory_beams(self.handle, ctypes.c_void_p(enc.data_ptr()), clips, frames, beams,
                                            self._stream()))
        self.streams, self.beams = clips * beams, beams

    def Beam(self, bos: int, langs, eos: int, opts: "BeamOptions" = None):
        """search/beam.go:73 Beam for every clip of the last MemoryBeams:
        host numpy arrays (tokens [clips, max_tokens − 1] padded with −1,
        counts, lang, eos_hit, score, lang_logprob, logprobs [clips,
        max_tokens])."""
        import numpy as np

        o = opts if opts is not None else DefaultBeam(beams=self.beams)
        clips = self.streams // max(1, o.beams)
        max_tok = o.max_tokens if o.max_tokens > 0 else self.positions_left()
        out_w = max(1, max_tok - 1)
        lg = np.ascontiguousarray(langs, np.int32)
        tokens = np.zeros((clips, out_w), np.int32)
        counts, lang, eos_hit = (np.zeros(clips, np.int32) for _ in range(3))
        score, lang_lp = np.zeros(clips, np.float64), np.zeros(clips, np.float64)
        logprobs = np.zeros((clips, max_tok), np.float64)
        check(lib().wc_decoder_beam(self.handle, ctypes.addressof(o), int(bos), lg.ctypes.data, lg.size, int(eos),
                                    tokens.ctypes.data, counts.ctypes.data, lang.ctypes.data, eos_hit.ctypes.data,
                                    score.ctypes.data, lang_lp.ctypes.data, logprobs.ctypes.data, self._stream()))
        return tokens, counts, lang, eos_hit.astype(bool), score, lang_lp, logprobs

    def positions_left(self) -> int:
        return self.max_positions - self.Len()

    def memory_of(self, l: int):
        """Layer l's device memory pointers (k8, ks, v8, vs)."""
        ps = [ctypes.c_void_p() for _ in range(4)]
        check(lib().wc_decoder_memory_of(self.handle, l, *[ctypes.byref(p) for p in ps]))
        return [p.value for p in ps]

    def Extend(self, tokens, logits=None, next_=None):
        """decoder.go:252 Extend with one token per stream (CUDA int32
        [streams]); logits (CUDA float32 [streams, vocab]) and next_ (CUDA
        int32 [streams], the argmax) are filled when given."""
        check(lib().wc_decoder_extend(self.handle, ctypes.c_void_p(tokens.data_ptr()),
                                      ctypes.c_void_p(logits.data_ptr()) if logits is not None else None,
                                      ctypes.c_void_p(next_.data_ptr()) if next_ is not None else None,
                                      self._stream()))

    def Len(self) -> int:
        return lib().wc_decoder_len(self.handle)

    def GreedyMemory(self, bos: int, langs, eos: int, max_tokens: int):
        """greedy.go:40 GreedyMemory for every stream, on the device: returns
        CUDA tensors (tokens [streams, max_tokens − 1] padded with −1,
        counts, lang, eos_hit)."""
        import numpy as np
        import torch

        S = self.streams
        out_w = max(1, max_tokens - 1)
        dev = torch.device("cuda")
        tokens = torch.empty((S, out_w), dtype=torch.int32, device=dev)
        counts, lang, eos_hit = (torch.empty(S, dtype=torch.int32, device=dev) for _ in range(3))
        lg = np.ascontiguousarray(langs, np.int32)
        check(lib().wc_decoder_greedy(self.handle, int(bos), lg.ctypes.data, lg.size, int(eos), int(max_tokens),
                                      ctypes.c_void_p(tokens.data_ptr()), ctypes.c_void_p(counts.data_ptr()),
                                      ctypes.c_void_p(lang.data_ptr()), ctypes.c_void_p(eos_hit.data_ptr()),
                                      self._stream()))
        return tokens, counts, lang, eos_hit
