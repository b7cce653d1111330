"""Whistle's encoder stack on the B200 library (wc_encoder_*):
internal/encoder's Stack (encoder.go:167) with the Best() hypothesis
(hypothesis.go:284) and the engine's int8 numerics (whistle/model.go:85
WithInt8), for many clips at once with every intermediate in device memory.
Its input is the stem's output (encoder.go:132 Stem); the log-mel front end
and the conv stem run before it.
"""

from __future__ import annotations

import ctypes

from ._lib import check, lib

__all__ = ["Encoder", "WC_ENCODER_TENSOR_CORES", "WC_ENCODER_ANY_ORDER"]

WC_ENCODER_TENSOR_CORES = 1
WC_ENCODER_ANY_ORDER = 2

_p = ctypes.c_void_p
_MLP_KEYS = ("d1", "d2", "b2", "d3", "d4", "w1a", "w1b", "w2a", "w2b", "w3a", "w3b", "cond_v", "cond_u")


class _Mlp(ctypes.Structure):
    """wc_hadamard_mlp (include/whistle_b200.h)."""
    _fields_ = [(k, _p) for k in _MLP_KEYS]


class _Layer(ctypes.Structure):
    """wc_encoder_layer."""
    _fields_ = ([(k, _p) for k in ("pre_hada_0", "norm_in", "post_norm", "conv_norm", "conv_out_norm", "pre_hada")]
                + [("attn_gate", ctypes.c_float)]
                + [(k, _p) for k in ("q_proj", "k_proj", "v_proj", "gate_proj", "out_proj", "pw1", "pw2", "q_norm",
                                     "k_norm", "dw")]
                + [("hada_0", _Mlp), ("hada", _Mlp)]
                + [(k, ctypes.c_float) for k in ("a_pre", "a_post", "a_res")]
                + [(k, _p) for k in ("b_pre", "b_post", "b_res", "phi_pre", "phi_post", "phi_res")])


class _Desc(ctypes.Structure):
    """wc_encoder_desc."""
    _fields_ = ([(k, ctypes.c_int) for k in ("dim", "lanes", "layers", "heads", "kv_heads", "qk", "vd", "dw_kernel",
                                             "na", "nb", "rank")]
                + [("hada_p1", _p), ("hada_p2", _p), ("rope_theta", ctypes.c_double), ("rope_len", ctypes.c_int),
                   ("final_norm", _p), ("layer", ctypes.POINTER(_Layer))]
                + [(k, _p) for k in ("stem_w", "stem_dw_1", "stem_dw_2", "stem_pw_1", "stem_pw_2", "stem_out")]
                + [("stem_channels", ctypes.c_int), ("mel_filters", _p)])


class Encoder:
    """Whistle's encoder stack (encoder.go:24 Encoder's blocks, mHC layers
    and final norm) with int8 numerics on the GPU, for up to ``max_clips``
    clips of up to ``max_frames`` frames.

    ``w`` is a weight set with the attributes of ``synth.EncoderWeights``
    (CQ tensors as ``cq.Packed``, float tensors as arrays; the FFN1
    HadamardMLP under ``hada_0.*``, FFN2's under ``hada.*``). flags:
    ``WC_ENCODER_TENSOR_CORES`` (products on the tensor cores, within the
    fp16 bound) and ``WC_ENCODER_ANY_ORDER`` (attention within 1e-5).
    Without them every product is the bit-exact lut path and the attention
    the int8 kernel's exact order.
    """

    def __init__(self, w, max_clips: int, max_frames: int = 375, flags: int = 0):
        import numpy as np

        from . import cq

        self.w, self.flags = w, flags
        self.max_clips, self.max_frames = max_clips, max_frames
        self._keep = []

        def f(a):
            a = np.ascontiguousarray(a, np.float32).reshape(-1)
            self._keep.append(a)
            return a.ctypes.data

        def m(p):
            mat = cq.New(p)
            self._keep.append(mat)
            return mat.handle.value

        stacked = {}

        def rows(p, lo, hi):
            mat = stacked.get(id(p)) or cq.New(p)
            stacked[id(p)] = mat
            v = mat.Rows(lo, hi)
            self._keep += [mat, v]
            return v.handle.value

        L = (_Layer * len(w.layers))()
        for l, src in enumerate(w.layers):
            d = L[l]
            for k in ("pre_hada_0", "norm_in", "post_norm", "conv_norm", "conv_out_norm", "pre_hada", "q_norm",
                      "k_norm", "dw", "b_pre", "b_post", "b_res"):
                setattr(d, k, f(src[k]))
            for k in ("attn_gate", "a_pre", "a_post", "a_res"):
                setattr(d, k, float(src[k]))
            for k in ("q_proj", "k_proj", "v_proj", "gate_proj", "out_proj", "pw1", "pw2"):
                setattr(d, k, m(src[k]))
            for mlp, pre in ((d.hada_0, "hada_0."), (d.hada, "hada.")):
                for k in _MLP_KEYS:
                    setattr(mlp, k, f(src[pre + k]))
            for k in ("phi_pre", "phi_post", "phi_res"):
                lo, hi = w.phi_rows(k, l)
                setattr(d, k, rows(getattr(w, k), lo, hi))
        p1, p2 = np.ascontiguousarray(w.hada_p1, np.int32), np.ascontiguousarray(w.hada_p2, np.int32)
        self._keep += [p1, p2, L]
        desc = _Desc(w.dim, w.lanes, len(w.layers), w.heads, w.kv_heads, w.qk, w.vd, w.dw_k, w.na, w.nb, w.rank)
        desc.hada_p1, desc.hada_p2 = p1.ctypes.data, p2.ctypes.data
        desc.rope_theta, desc.rope_len = float(w.rope_theta), int(w.rope_len)
        desc.final_norm = f(w.final_norm)
        desc.layer = L
        if getattr(w, "stem_w", None) is not None:
            desc.stem_w, desc.stem_dw_1, desc.stem_dw_2 = f(w.stem_w), f(w.stem_dw_1), f(w.stem_dw_2)
            desc.stem_pw_1, desc.stem_pw_2, desc.stem_out = m(w.stem_pw_1), m(w.stem_pw_2), m(w.stem_out)
            desc.stem_channels = int(w.stem_channels)
            desc.mel_filters = f(w.mel_filters)
        h = ctypes.c_void_p()
        check(lib().wc_encoder_create(ctypes.byref(desc), max_clips, max_frames, flags, ctypes.byref(h)))
        self.handle = h

    @classmethod
    def Load(cls, path_or_data, max_clips: int, max_frames: int = 375, flags: int = 0):
        """encoder.LoadInt8 over a .cact file (a path or its bytes): the
        encoder's, the stem's and the mel bank's tensors by name
        (weights.encoder_weights), CQ records uploaded as stored."""
        from . import weights

        return cls(weights.load_encoder(path_or_data), max_clips, max_frames, flags)

    def __del__(self):
        if getattr(self, "handle", None) and self.handle.value:
            lib().wc_encoder_destroy(self.handle)
            self.handle = None

    def Stack(self, x, out=None):
        """encoder.go:167 Stack on a CUDA tensor x [clips][frames][dim] (or
        [frames][dim]) of stem outputs; returns (or fills) out, same shape."""
        import torch

        if not (isinstance(x, torch.Tensor) and x.is_cuda and x.dtype == torch.float32):
            raise TypeError("encoder: x must be a float32 CUDA tensor")
        x = x.contiguous()
        x3 = x.reshape(-1, x.shape[-2], x.shape[-1])
        if out is None:
            out = torch.empty_like(x)
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        check(lib().wc_encoder_stack(self.handle, ctypes.c_void_p(x3.data_ptr()), x3.shape[0], x3.shape[1],
                                     ctypes.c_void_p(out.data_ptr()), st))
        return out

    @staticmethod
    def stem_frames(frames: int) -> int:
        """stem.go:166 length: the stem's output frames for `frames` mel frames."""
        return lib().wc_encoder_stem_frames(int(frames))

    def LogMel(self, samples, out=None):
        """frontend/mel.go:226 LogMel on a CUDA tensor samples [clips][n] (16 kHz):
        [clips][n // 160][80] float32."""
        import torch

        s2 = samples.contiguous().reshape(-1, samples.shape[-1])
        F = s2.shape[1] // 160
        if out is None:
            out = torch.empty(s2.shape[0], F, 80, device=samples.device, dtype=torch.float32)
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        check(lib().wc_encoder_logmel(self.handle, ctypes.c_void_p(s2.data_ptr()), s2.shape[0], s2.shape[1],
                                      ctypes.c_void_p(out.data_ptr()), st))
        return out

    def Stem(self, mel, out=None):
        """encoder.go:132 Stem on a CUDA tensor mel [clips][frames][80]:
        [clips][stem_frames(frames)][dim]."""
        import torch

        m3 = mel.contiguous().reshape(-1, mel.shape[-2], mel.shape[-1])
        T = self.stem_frames(m3.shape[1])
        if out is None:
            out = torch.empty(m3.shape[0], T, self.w.dim, device=mel.device, dtype=torch.float32)
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        check(lib().wc_encoder_stem(self.handle, ctypes.c_void_p(m3.data_ptr()), m3.shape[0], m3.shape[1],
                                    ctypes.c_void_p(out.data_ptr()), st))
        return out

    def Embed(self, samples, out=None):
        """encoder.go:108 Embed: LogMel, Stem and Stack on samples [clips][n]."""
        import torch

        s2 = samples.contiguous().reshape(-1, samples.shape[-1])
        T = self.stem_frames(s2.shape[1] // 160)
        if out is None:
            out = torch.empty(s2.shape[0], T, self.w.dim, device=samples.device, dtype=torch.float32)
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        check(lib().wc_encoder_embed(self.handle, ctypes.c_void_p(s2.data_ptr()), s2.shape[0], s2.shape[1],
                                     ctypes.c_void_p(out.data_ptr()), st))
        return out
