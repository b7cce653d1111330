"""CPU oracle for go-whistle's quantized hot path — TEST INFRASTRUCTURE ONLY.

This package is the checker that the CUDA library is compared against and the
timed CPU baseline of ``bench.py``. Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference``) may use
it; the product (``go-whistle_b200``) never imports it.

The C sources (``cq_oracle.c``, ``lut_avx2.c``, ``needle_oracle.c``, ``decoder_oracle.c``,
``whistle_oracle.c``) restate the reference's Go
routines operation for operation; each names the file:line it follows. The
reference (a Go module) cannot be built in this image (no Go toolchain, and
its third-party modules are not vendored), so there is no ``oracle/_ref``.
Parity is pinned against the reference's own known-answer tests and error
bounds (``tests/test_oracle_pins.py``); the reference stores no golden output
vectors for this path.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_i8p = ctypes.POINTER(ctypes.c_int8)
_i16p = ctypes.POINTER(ctypes.c_int16)
_i32p = ctypes.POINTER(ctypes.c_int32)


class Packed(ctypes.Structure):
    """``wo_packed``: cact.Packed (internal/cact/packed.go:18-40) as C sees it."""

    _fields_ = [
        ("out", ctypes.c_int),
        ("in_", ctypes.c_int),
        ("group", ctypes.c_int),
        ("bits", ctypes.c_int),
        ("index", _u8p),
        ("norms16", _u16p),
        ("cb", _f32p),
    ]


def build(force: bool = False) -> Path:
    """Compiles liboracle.so with the Makefile beside it (gcc, no GPU)."""
    srcs = [HERE / n for n in ("cq_oracle.c", "lut_avx2.c", "needle_oracle.c", "decoder_oracle.c", "whistle_oracle.c",
                                "oracle.h", "par.h", "Makefile")]
    if force or not LIB_PATH.exists() or any(s.stat().st_mtime > LIB_PATH.stat().st_mtime for s in srcs):
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.wo_f16_to_f32.restype = ctypes.c_float
        L.wo_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.wo_fwht.argtypes = [_f32p, ctypes.c_int]
        L.wo_lut_step_of.restype = ctypes.c_float
        L.wo_lut_step_of.argtypes = [ctypes.c_int]
        for name, tp in (("wo_lut_tables_planes", _u8p), ("wo_lut_tables_int", _i16p)):
            fn = getattr(L, name)
            fn.restype = ctypes.c_float
            fn.argtypes = [ctypes.c_int, tp, _f32p, ctypes.c_int, _f32p, ctypes.c_float]
        L.wo_lut_lookup_blocked.argtypes = [_f32p, _u8p, _u8p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.wo_lut_lookup_blocked_avx2.argtypes = L.wo_lut_lookup_blocked.argtypes
        L.wo_fwht_avx2.argtypes = [_f32p, ctypes.c_int]
        L.wo_lut_tables_planes_avx2.restype = ctypes.c_float
        L.wo_lut_tables_planes_avx2.argtypes = [ctypes.c_int, _u8p, _f32p, ctypes.c_int, _f32p, ctypes.c_float]
        pp = ctypes.POINTER(Packed)
        L.wo_cq_gemm_lut.restype = ctypes.c_int
        L.wo_cq_gemm_lut.argtypes = [pp, _f32p, ctypes.c_int, _f32p]
        L.wo_cq_gemm_lut_mt.restype = ctypes.c_int
        L.wo_cq_gemm_lut_mt.argtypes = [pp, _f32p, ctypes.c_int, _f32p, ctypes.c_int]
        L.wo_cq_gemms_lut.restype = ctypes.c_int
        L.wo_cq_gemms_lut.argtypes = [pp, ctypes.c_int, _f32p, ctypes.c_int, ctypes.POINTER(_f32p)]
        L.wo_cq_gemm_exact.argtypes = [pp, _f32p, ctypes.c_int, _f32p]
        L.wo_cq_gemm_gather.argtypes = [pp, _f32p, ctypes.c_int, _f32p]
        L.wo_cq_row.argtypes = [pp, ctypes.c_int, _f32p]
        L.wo_lut_prepare.restype = ctypes.c_void_p
        L.wo_lut_prepare.argtypes = [pp]
        L.wo_lut_gemm_prepared.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, _f32p, ctypes.c_int]
        L.wo_lut_release.argtypes = [ctypes.c_void_p]
        L.wo_max_threads.restype = ctypes.c_int
        L.wo_quantize_row.restype = ctypes.c_float
        L.wo_quantize_row.argtypes = [_i8p, _f32p, ctypes.c_int]
        L.wo_quantize_rows.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _i8p, _f32p]
        L.wo_softmax.argtypes = [_f32p, ctypes.c_int]
        args = [_f32p, ctypes.c_int, ctypes.c_int, _i8p, _f32p, _i8p, _f32p, ctypes.c_int, ctypes.c_int,
                ctypes.c_int, ctypes.c_int, _i32p, ctypes.c_float, ctypes.c_int, _f32p, _f32p]
        L.wo_attend_int8_spans.argtypes = args
        L.wo_attend_int8_spans_mt.argtypes = args + [ctypes.c_int]
        L.wo_attend_int8_streams_mt.argtypes = [ctypes.c_int, _f32p, ctypes.c_int, _i8p, _f32p, _i8p, _f32p,
                                                ctypes.c_int, _i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                ctypes.c_float, _f32p, ctypes.c_int]
        L.wo_head_argmax.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float, _f32p, _i32p]
        _lib = L
    return _lib


def _ptr(a: np.ndarray, tp):
    return a.ctypes.data_as(tp)


def _c(a, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


class OracleMatrix:
    """A packed CQ matrix held for the oracle (keeps its arrays alive)."""

    def __init__(self, index, norms16, cb, out, in_, group, bits):
        self.index = _c(index, np.uint8).reshape(-1)
        self.norms16 = _c(norms16, np.uint16).reshape(-1)
        self.cb = _c(cb, np.float32).reshape(-1)
        self.out, self.in_, self.group, self.bits = int(out), int(in_), int(group), int(bits)
        self.s = Packed(self.out, self.in_, self.group, self.bits, _ptr(self.index, _u8p),
                        _ptr(self.norms16, _u16p), _ptr(self.cb, _f32p))

    @classmethod
    def of(cls, m) -> "OracleMatrix":
        """From any object with index, norms16, codebook, out, in_, group, bits."""
        return cls(m.index, m.norms16, m.codebook, m.out, m.in_, m.group, m.bits)


def f16_to_f32(h: int) -> float:
    return lib().wo_f16_to_f32(int(h))


def fwht(x: np.ndarray) -> np.ndarray:
    y = _c(x, np.float32).copy()
    lib().wo_fwht(_ptr(y, _f32p), y.size)
    return y


def lut_step_of(group: int) -> float:
    return lib().wo_lut_step_of(group)


def lut_tables_planes(bits, x, cb, cb_max):
    x, cb = _c(x, np.float32), _c(cb, np.float32)
    tab = np.zeros(32 * (x.size if bits == 4 else x.size // 2), np.uint8)
    m = lib().wo_lut_tables_planes(bits, _ptr(tab, _u8p), _ptr(x, _f32p), x.size, _ptr(cb, _f32p), cb_max)
    return np.float32(m), tab


def lut_tables_int(bits, x, cb, cb_max):
    x, cb = _c(x, np.float32), _c(cb, np.float32)
    tab = np.zeros(16 * (x.size if bits == 4 else x.size // 2), np.int16)
    m = lib().wo_lut_tables_int(bits, _ptr(tab, _i16p), _ptr(x, _f32p), x.size, _ptr(cb, _f32p), cb_max)
    return np.float32(m), tab.reshape(-1, 16)


def gemm_lut(m: OracleMatrix, x: np.ndarray, rows: int, threads: int = 1) -> np.ndarray:
    x = _c(x, np.float32)
    y = np.zeros(rows * m.out, np.float32)
    rc = lib().wo_cq_gemm_lut_mt(ctypes.byref(m.s), _ptr(x, _f32p), rows, _ptr(y, _f32p), threads)
    if rc != 0:
        raise ValueError("oracle: group index bytes exceed lutMaxGroupBytes")
    return y.reshape(rows, m.out)


def gemms_lut(ms, x: np.ndarray, rows: int):
    x = _c(x, np.float32)
    arr = (Packed * len(ms))(*[m.s for m in ms])
    ys = [np.zeros(rows * m.out, np.float32) for m in ms]
    yp = (_f32p * len(ms))(*[_ptr(y, _f32p) for y in ys])
    rc = lib().wo_cq_gemms_lut(arr, len(ms), _ptr(x, _f32p), rows, yp)
    if rc != 0:
        raise ValueError("oracle: group index bytes exceed lutMaxGroupBytes")
    return [y.reshape(rows, m.out) for y, m in zip(ys, ms)]


def gemm_exact(m: OracleMatrix, x: np.ndarray, rows: int) -> np.ndarray:
    x = _c(x, np.float32)
    y = np.zeros(rows * m.out, np.float32)
    lib().wo_cq_gemm_exact(ctypes.byref(m.s), _ptr(x, _f32p), rows, _ptr(y, _f32p))
    return y.reshape(rows, m.out)


def gemm_gather(m: OracleMatrix, x: np.ndarray, rows: int) -> np.ndarray:
    x = _c(x, np.float32)
    y = np.zeros(rows * m.out, np.float32)
    lib().wo_cq_gemm_gather(ctypes.byref(m.s), _ptr(x, _f32p), rows, _ptr(y, _f32p))
    return y.reshape(rows, m.out)


def row(m: OracleMatrix, r: int) -> np.ndarray:
    y = np.zeros(m.in_, np.float32)
    lib().wo_cq_row(ctypes.byref(m.s), r, _ptr(y, _f32p))
    return y


class PreparedLUT:
    """A matrix prepared once (the 32-row repack) for timed CPU products."""

    def __init__(self, m: OracleMatrix):
        self.m = m
        self.h = lib().wo_lut_prepare(ctypes.byref(m.s))
        if not self.h:
            raise ValueError("oracle: group index bytes exceed lutMaxGroupBytes")

    def gemm(self, x: np.ndarray, rows: int, y: np.ndarray, threads: int) -> None:
        lib().wo_lut_gemm_prepared(self.h, _ptr(x, _f32p), rows, _ptr(y, _f32p), threads)

    def __del__(self):
        if getattr(self, "h", None):
            lib().wo_lut_release(self.h)
            self.h = None


def max_threads() -> int:
    return lib().wo_max_threads()


def quantize_row(x: np.ndarray):
    x = _c(x, np.float32)
    q = np.zeros(x.size, np.int8)
    s = lib().wo_quantize_row(_ptr(q, _i8p), _ptr(x, _f32p), x.size)
    return q, np.float32(s)


def quantize_rows(x: np.ndarray, cols: int, width: int):
    x = _c(x, np.float32).reshape(-1)
    rows = x.size // cols
    q = np.zeros(x.size, np.int8)
    s = np.zeros(x.size // width, np.float32)
    lib().wo_quantize_rows(_ptr(x, _f32p), rows, cols, width, _ptr(q, _i8p), _ptr(s, _f32p))
    return q, s


def softmax(s: np.ndarray) -> np.ndarray:
    s = _c(s, np.float32).copy()
    lib().wo_softmax(_ptr(s, _f32p), s.size)
    return s


def attend_int8_spans(q, t, heads, k8, ks, v8, vs, nkeys, kv_heads, qk, vd, spans, scale, quant_q,
                      want_probs=False, threads=1):
    q = _c(q, np.float32)
    k8, v8 = _c(k8, np.int8), _c(v8, np.int8)
    ks, vs = _c(ks, np.float32), _c(vs, np.float32)
    sp = _c(spans, np.int32).reshape(-1)
    out = np.zeros(t * heads * vd, np.float32)
    probs = np.zeros(t * heads * nkeys, np.float32) if want_probs else None
    lib().wo_attend_int8_spans_mt(_ptr(q, _f32p), t, heads, _ptr(k8, _i8p), _ptr(ks, _f32p), _ptr(v8, _i8p),
                                  _ptr(vs, _f32p), nkeys, kv_heads, qk, vd, _ptr(sp, _i32p), scale,
                                  1 if quant_q else 0, _ptr(probs, _f32p) if probs is not None else None,
                                  _ptr(out, _f32p), threads)
    return out, probs


def attend_int8(q, t, heads, k8, ks, v8, vs, nkeys, kv_heads, qk, vd, keys, scale, quant_q, want_probs=False):
    """AttendInt8 (int8.go:194): row i sees keys [0, keys(i))."""
    spans = np.array([[0, 0, 0, keys(i)] for i in range(t)], np.int32)
    return attend_int8_spans(q, t, heads, k8, ks, v8, vs, nkeys, kv_heads, qk, vd, spans, scale, quant_q,
                             want_probs)


def attend_streams(q, heads, k8, ks, v8, vs, cap, nkeys, kv_heads, qk, vd, scale, threads):
    """Decode-step attention of many streams (one query row each)."""
    streams = len(nkeys)
    nk = _c(nkeys, np.int32)
    q, k8, v8, ks, vs = _c(q, np.float32), _c(k8, np.int8), _c(v8, np.int8), _c(ks, np.float32), _c(vs, np.float32)
    out = np.zeros(streams * heads * vd, np.float32)
    lib().wo_attend_int8_streams_mt(streams, _ptr(q, _f32p), heads, _ptr(k8, _i8p), _ptr(ks, _f32p),
                                    _ptr(v8, _i8p), _ptr(vs, _f32p), cap, _ptr(nk, _i32p), kv_heads, qk, vd, scale,
                                    _ptr(out, _f32p), threads)
    return out



def head_argmax(y: np.ndarray, rows: int, vocab: int, head: float = 1.0):
    """decoder.go:508 logits' head scale and greedy.go:182 argmax per row:
    (logits [rows, vocab], idx [rows])."""
    yy = _c(y, np.float32).reshape(-1)
    assert yy.size == rows * vocab
    logits = np.empty(rows * vocab, np.float32)
    idx = np.empty(rows, np.int32)
    lib().wo_head_argmax(_ptr(yy, _f32p), rows, vocab, float(head), _ptr(logits, _f32p), _ptr(idx, _i32p))
    return logits.reshape(rows, vocab), idx


# ---------------------------------------------------------------- decoder
#
# whistle_oracle.c: Whistle's decoder step (internal/decoder, Best(), int8
# numerics) on the CPU, over a synthetic weight set (any object with the
# attributes of go-whistle_b200's synth.DecoderWeights).

_i32 = ctypes.c_int


class _DecLayer(ctypes.Structure):
    _fields_ = ([(k, _f32p) for k in ("norm_in", "post_norm", "pre_hada")] + [("attn_gate", ctypes.c_float)]
                + [(k, Packed) for k in ("q_proj", "k_proj", "v_proj", "gate_proj", "out_proj")]
                + [(k, _f32p) for k in ("q_taps", "k_taps", "v_taps", "q_norm", "k_norm", "d1", "d2", "b2", "d3",
                                        "d4")]
                + [("hada_w", (_f32p * 2) * 3), ("cond_v", _f32p), ("cond_u", _f32p)]
                + [(k, _f32p) for k in ("x_norm_in", "x_post_norm", "x_q_norm", "x_k_norm")]
                + [("x_attn_gate", ctypes.c_float)]
                + [(k, Packed) for k in ("x_q_proj", "x_k_proj", "x_v_proj", "x_gate_proj", "x_out_proj")]
                + [(k, ctypes.c_float) for k in ("a_pre", "a_post", "a_res")]
                + [(k, _f32p) for k in ("b_pre", "b_post", "b_res")]
                + [(k, Packed) for k in ("phi_pre", "phi_post", "phi_res")])


class _EngramSite(ctypes.Structure):
    _fields_ = [("tables", Packed), ("key_proj", Packed), ("value_proj", Packed), ("taps", _f32p), ("layer", _i32)]


class _Decoder(ctypes.Structure):
    _fields_ = ([(k, _i32) for k in ("dim", "lanes", "layers", "vocab", "heads", "kv_heads", "qk", "vd", "taps",
                                     "x_heads", "x_qk", "x_vd", "na", "nb", "rank", "n_sites", "n_tables", "slots",
                                     "sub", "etaps", "max_order")]
                + [("orders", _i32p), ("hada_p1", _i32p), ("hada_p2", _i32p), ("rope_cos", _f32p),
                   ("rope_sin", _f32p), ("rope_len", _i32), ("embedding", Packed), ("final_norm", _f32p),
                   ("layer", ctypes.POINTER(_DecLayer)), ("site", ctypes.POINTER(_EngramSite))])


def _dec_lib():
    L = lib()
    if not getattr(L, "_dec_ready", False):
        dp, sp = ctypes.POINTER(_Decoder), ctypes.c_void_p
        L.wo_rope_tables.argtypes = [_i32, _i32, ctypes.c_double, _f32p, _f32p]
        L.wo_sinkhorn.argtypes = [_f32p, _i32]
        L.wo_dec_new.restype = sp
        L.wo_dec_new.argtypes = [dp, _i32, _i32]
        L.wo_dec_fork.restype = sp
        L.wo_dec_fork.argtypes = [dp, sp]
        L.wo_dec_free.argtypes = [sp]
        L.wo_dec_memory.argtypes = [dp, sp, _f32p, _i32]
        L.wo_dec_memory_of.argtypes = [dp, sp, _i32, ctypes.POINTER(_i8p), ctypes.POINTER(_f32p),
                                       ctypes.POINTER(_i8p), ctypes.POINTER(_f32p)]
        L.wo_dec_extend.restype = _i32
        L.wo_dec_extend.argtypes = [dp, sp, _i32, _f32p]
        L.wo_dec_greedy.restype = _i32
        L.wo_dec_greedy.argtypes = [dp, sp, _i32, _i32p, _i32, _i32, _i32, _i32p, _i32p, _i32p, _f32p]
        L.wo_ngram_hash.restype = ctypes.c_uint32
        L.wo_ngram_hash.argtypes = [_i32, _i32, _i32p, _i32]
        L.wo_zc_norm.argtypes = [_f32p, _f32p, _i32, _i32, _f32p]
        L.wo_rms_unit.argtypes = [_f32p, _f32p, _i32, _i32]
        L.wo_rope_apply.argtypes = [_f32p, _i32, _f32p, _f32p]
        L.wo_sinkhorn_iters.argtypes = [_f32p, _i32, _i32]
        L.wo_dec_states_mt.restype = sp
        L.wo_dec_states_mt.argtypes = [dp, _i32, _f32p, _i32, _i32, _i32]
        L.wo_dec_states_free.argtypes = [sp, _i32]
        L.wo_dec_greedy_states_mt.argtypes = [dp, sp, _i32, _i32, _i32p, _i32, _i32, _i32, _i32p, _i32p, _i32p,
                                              _i32p, _i32]
        L.wo_dec_greedy_streams_mt.argtypes = [dp, _i32, _f32p, _i32, _i32, _i32p, _i32, _i32, _i32, _i32p, _i32p,
                                               _i32p, _i32p, _i32]
        L._dec_ready = True
    return L


def rope_tables(head_dim: int, length: int, theta: float):
    """rope.go:20 NewRope's cos and sin tables [length][head_dim/2]."""
    c = np.zeros(length * (head_dim // 2), np.float32)
    s = np.zeros_like(c)
    _dec_lib().wo_rope_tables(head_dim, length, float(theta), _ptr(c, _f32p), _ptr(s, _f32p))
    return c, s


def sinkhorn(k: np.ndarray, iters: int = 20) -> np.ndarray:
    """mhc.go:300 sinkhorn on an n×n matrix of logits."""
    k = _c(k, np.float32).copy()
    n = int(round(np.sqrt(k.size)))
    _dec_lib().wo_sinkhorn_iters(_ptr(k.reshape(-1), _f32p), n, iters)
    return k


def ngram_hash(c: int, order: int, hist) -> int:
    """engram.go:141 ngramHash."""
    h = _c(hist if len(hist) else [0], np.int32)
    return int(_dec_lib().wo_ngram_hash(c, order, _ptr(h, _i32p), len(hist)))


def zc_norm(x: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """norm.go:60 ZCRMSNorm.Apply on rows of len(scale)."""
    x, sc = _c(x, np.float32).reshape(-1), _c(scale, np.float32)
    out = np.zeros_like(x)
    _dec_lib().wo_zc_norm(_ptr(out, _f32p), _ptr(x, _f32p), x.size // sc.size, sc.size, _ptr(sc, _f32p))
    return out


def rms_unit(x: np.ndarray, dim: int) -> np.ndarray:
    """norm.go:82 RMSUnit."""
    x = _c(x, np.float32).reshape(-1)
    out = np.zeros_like(x)
    _dec_lib().wo_rms_unit(_ptr(out, _f32p), _ptr(x, _f32p), x.size // dim, dim)
    return out


def rope_apply(x: np.ndarray, cos_row: np.ndarray, sin_row: np.ndarray) -> np.ndarray:
    """rope.go:73 apply at one position (its table rows)."""
    x = _c(x, np.float32).copy()
    c, s = _c(cos_row, np.float32), _c(sin_row, np.float32)
    _dec_lib().wo_rope_apply(_ptr(x, _f32p), x.size // 2, _ptr(c, _f32p), _ptr(s, _f32p))
    return x


class OracleDecoder:
    """The CPU restatement of Whistle's decoder over weights ``w``."""

    def __init__(self, w):
        self._keep = []

        def arr(a, dt=np.float32):
            a = _c(a, dt).reshape(-1)
            self._keep.append(a)
            return a

        def f(a):
            return _ptr(arr(a), _f32p)

        def pk(p, lo=None, hi=None):
            m = OracleMatrix.of(p)
            self._keep.append(m)
            if lo is None:
                return m.s
            return lib().wo_rows_py(m, lo, hi) if False else _rows(m, lo, hi)

        def _rows(m, lo, hi):
            groups = (m.in_ + m.group - 1) // m.group
            rb = groups * m.group * m.bits // 8
            return Packed(hi - lo, m.in_, m.group, m.bits, _ptr(m.index[lo * rb:], _u8p),
                          _ptr(m.norms16[lo * groups:], _u16p), _ptr(m.cb, _f32p))

        self.w = w
        n = len(w.layers)
        layers = (_DecLayer * n)()
        for l, L in enumerate(w.layers):
            d = layers[l]
            for k in ("norm_in", "post_norm", "pre_hada", "q_taps", "k_taps", "v_taps", "q_norm", "k_norm", "d1",
                      "d2", "b2", "d3", "d4", "cond_v", "cond_u", "x_norm_in", "x_post_norm", "x_q_norm",
                      "x_k_norm", "b_pre", "b_post", "b_res"):
                setattr(d, k, f(L[k]))
            for k in ("attn_gate", "x_attn_gate", "a_pre", "a_post", "a_res"):
                setattr(d, k, float(L[k]))
            for k in ("q_proj", "k_proj", "v_proj", "gate_proj", "out_proj", "x_q_proj", "x_k_proj", "x_v_proj",
                      "x_gate_proj", "x_out_proj"):
                setattr(d, k, pk(L[k]))
            for s in range(3):
                d.hada_w[s][0] = f(L[f"w{s + 1}a"])
                d.hada_w[s][1] = f(L[f"w{s + 1}b"])
            for k in ("phi_pre", "phi_post", "phi_res"):
                lo, hi = w.phi_rows(k, l)
                setattr(d, k, pk(getattr(w, k), lo, hi))
        sites = (_EngramSite * max(1, len(w.sites)))()
        for i, S in enumerate(w.sites):
            sites[i].tables, sites[i].key_proj, sites[i].value_proj = (pk(S[k]) for k in ("tables", "key_proj",
                                                                                          "value_proj"))
            sites[i].taps = f(S["taps"])
            sites[i].layer = S["layer"]
        self._layers, self._sites = layers, sites
        self.rope_cos, self.rope_sin = rope_tables(w.qk, w.rope_len, w.rope_theta)
        D = _Decoder(w.dim, w.lanes, n, w.vocab, w.heads, w.kv_heads, w.qk, w.vd, w.taps, w.x_heads, w.x_qk,
                     w.x_vd, w.na, w.nb, w.rank, len(w.sites), w.n_tables, w.slots, w.sub, w.etaps, w.max_order)
        D.orders = _ptr(arr(w.orders, np.int32), _i32p)
        D.hada_p1 = _ptr(arr(w.hada_p1, np.int32), _i32p)
        D.hada_p2 = _ptr(arr(w.hada_p2, np.int32), _i32p)
        D.rope_cos, D.rope_sin = _ptr(self.rope_cos, _f32p), _ptr(self.rope_sin, _f32p)
        D.rope_len = w.rope_len
        D.embedding = pk(w.embedding)
        D.final_norm = f(w.final_norm)
        D.layer = layers
        D.site = sites
        self.d = D

    def state(self, cap: int, frames: int) -> "OracleState":
        return OracleState(self, cap, frames)

    def greedy_streams(self, enc: np.ndarray, bos: int, langs, eos: int, max_tok: int, threads: int = 1):
        """GreedyMemory for every stream of enc [streams][frames][dim]:
        (tokens [streams][max_tok] (−1 past each count), counts, langs, eos)."""
        enc = _c(enc, np.float32)
        streams, frames = enc.shape[0], enc.shape[1]
        lg = _c(langs, np.int32)
        tok = np.full((streams, max_tok), -1, np.int32)
        cnt, lang, eh = (np.zeros(streams, np.int32) for _ in range(3))
        _dec_lib().wo_dec_greedy_streams_mt(ctypes.byref(self.d), streams, _ptr(enc, _f32p), frames, bos,
                                            _ptr(lg, _i32p), lg.size, eos, max_tok, _ptr(tok, _i32p),
                                            _ptr(cnt, _i32p), _ptr(lang, _i32p), _ptr(eh, _i32p), threads)
        for b in range(streams):
            tok[b, cnt[b]:] = -1
        return tok, cnt, lang, eh


def timed_greedy(dec: "OracleDecoder", enc: np.ndarray, bos: int, langs, eos: int, max_tok: int, threads: int):
    """The CPU baseline of the decoder: every stream's memory on threads
    (untimed), then their greedy decodes on threads, timed by the wall
    clock. Returns (seconds, tokens [streams][max_tok], counts, langs, eos)."""
    import time

    L = _dec_lib()
    enc = _c(enc, np.float32)
    streams, frames = enc.shape[0], enc.shape[1]
    st = L.wo_dec_states_mt(ctypes.byref(dec.d), streams, _ptr(enc, _f32p), frames, max_tok + 1, threads)
    lg = _c(langs, np.int32)
    tok = np.full((streams, max_tok), -1, np.int32)
    cnt, lang, eh = (np.zeros(streams, np.int32) for _ in range(3))
    t0 = time.perf_counter()
    L.wo_dec_greedy_states_mt(ctypes.byref(dec.d), st, streams, bos, _ptr(lg, _i32p), lg.size, eos, max_tok,
                              _ptr(tok, _i32p), _ptr(cnt, _i32p), _ptr(lang, _i32p), _ptr(eh, _i32p), threads)
    secs = time.perf_counter() - t0
    L.wo_dec_states_free(st, streams)
    return secs, tok, cnt, lang, eh


class OracleState:
    """One sequence (decoder.go:173 State) with its memory."""

    def __init__(self, dec: OracleDecoder, cap: int, frames: int):
        self.dec, self.frames = dec, frames
        self.h = _dec_lib().wo_dec_new(ctypes.byref(dec.d), cap, frames)

    def memory(self, enc: np.ndarray) -> None:
        enc = _c(enc, np.float32)
        self._enc = enc
        _dec_lib().wo_dec_memory(ctypes.byref(self.dec.d), self.h, _ptr(enc, _f32p), enc.shape[0])

    def memory_of(self, l: int):
        """Layer l's int8 memory (k8, ks, v8, vs) as numpy copies."""
        w = self.dec.w
        k8, ks, v8, vs = _i8p(), _f32p(), _i8p(), _f32p()
        _dec_lib().wo_dec_memory_of(ctypes.byref(self.dec.d), self.h, l, ctypes.byref(k8), ctypes.byref(ks),
                                    ctypes.byref(v8), ctypes.byref(vs))
        F = self.frames
        return (np.ctypeslib.as_array(k8, (F * w.x_heads * w.x_qk,)).copy(),
                np.ctypeslib.as_array(ks, (F * w.x_heads,)).copy(),
                np.ctypeslib.as_array(v8, (F * w.x_heads * w.x_vd,)).copy(),
                np.ctypeslib.as_array(vs, (F * w.x_heads,)).copy())

    def fork(self) -> "OracleState":
        """decoder.go:223 State.Fork: an independent copy."""
        f = OracleState.__new__(OracleState)
        f.dec, f.frames = self.dec, self.frames
        f.h = _dec_lib().wo_dec_fork(ctypes.byref(self.dec.d), self.h)
        return f

    def extend(self, tok: int) -> np.ndarray:
        logits = np.zeros(self.dec.w.vocab, np.float32)
        if _dec_lib().wo_dec_extend(ctypes.byref(self.dec.d), self.h, int(tok), _ptr(logits, _f32p)) != 0:
            raise ValueError(f"oracle: token {tok} out of range or cache full")
        return logits

    def greedy(self, bos: int, langs, eos: int, max_tok: int):
        lg = _c(langs, np.int32)
        tok = np.zeros(max_tok, np.int32)
        lang, eh = ctypes.c_int(0), ctypes.c_int(0)
        margins = np.zeros(max_tok, np.float32)
        n = _dec_lib().wo_dec_greedy(ctypes.byref(self.dec.d), self.h, bos, _ptr(lg, _i32p), lg.size, eos, max_tok,
                                     _ptr(tok, _i32p), ctypes.byref(lang), ctypes.byref(eh), _ptr(margins, _f32p))
        if n < 0:
            raise ValueError("oracle: greedy decode failed")
        return tok[:n], lang.value, bool(eh.value), margins

    def __del__(self):
        if getattr(self, "h", None):
            _dec_lib().wo_dec_free(self.h)
            self.h = None


# ---------------------------------------------------------------- encoder
# internal/encoder's Stack (Best() hypothesis, needle.Int8{Act, KV}) over a
# synthetic weight set (go-whistle_b200's synth.EncoderWeights).

ENC_ATTEND_FLOAT, ENC_ATTEND_INT8 = 0, 1


class _EncLayer(ctypes.Structure):
    _fields_ = [("b", _DecLayer), ("hada0", _DecLayer), ("conv_norm", _f32p), ("conv_out_norm", _f32p),
                ("pw1", Packed), ("pw2", Packed), ("dw", _f32p)]


class _Encoder(ctypes.Structure):
    _fields_ = [("d", _Decoder), ("dw_k", _i32), ("layer", ctypes.POINTER(_EncLayer))]


def _enc_lib():
    L = lib()
    if not getattr(L, "_enc_ready", False):
        ep = ctypes.POINTER(_Encoder)
        L.wo_enc_stack.restype = _i32
        L.wo_enc_stack.argtypes = [ep, _f32p, _i32, _i32, _i32, _f32p]
        L.wo_enc_stack_mt.restype = _i32
        L.wo_enc_stack_mt.argtypes = [ep, _f32p, _i32, _i32, _i32, _f32p, _i32]
        L.wo_enc_glu.argtypes = [_f32p, _i32, _i32, _f32p]
        L.wo_enc_depthwise.argtypes = [_f32p, _i32, _i32, _f32p, _i32, _f32p]
        L.wo_silu.argtypes = [_f32p, _i32]
        L._enc_ready = True
    return L


def enc_glu(p: np.ndarray, t: int, half: int) -> np.ndarray:
    p = _c(p, np.float32)
    out = np.zeros(t * half, np.float32)
    _enc_lib().wo_enc_glu(_ptr(p, _f32p), t, half, _ptr(out, _f32p))
    return out


def enc_depthwise(x: np.ndarray, t: int, h: int, dw: np.ndarray) -> np.ndarray:
    x, dw = _c(x, np.float32), _c(dw, np.float32)
    out = np.zeros(t * h, np.float32)
    _enc_lib().wo_enc_depthwise(_ptr(x, _f32p), t, h, _ptr(dw, _f32p), dw.size // h, _ptr(out, _f32p))
    return out


def silu(x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32).copy()
    _enc_lib().wo_silu(_ptr(x, _f32p), x.size)
    return x


class OracleEncoder:
    """The CPU restatement of Whistle's encoder stack over weights ``w``."""

    def __init__(self, w):
        self._keep = []

        def arr(a, dt=np.float32):
            a = _c(a, dt).reshape(-1)
            self._keep.append(a)
            return a

        def f(a):
            return _ptr(arr(a), _f32p)

        def pk(p, lo=None, hi=None):
            m = OracleMatrix.of(p)
            self._keep.append(m)
            if lo is None:
                return m.s
            groups = (m.in_ + m.group - 1) // m.group
            rb = groups * m.group * m.bits // 8
            return Packed(hi - lo, m.in_, m.group, m.bits, _ptr(m.index[lo * rb:], _u8p),
                          _ptr(m.norms16[lo * groups:], _u16p), _ptr(m.cb, _f32p))

        def mlp(d, L, pre, norm):
            for k in ("d1", "d2", "b2", "d3", "d4", "cond_v", "cond_u"):
                setattr(d, k, f(L[pre + k]))
            for s in range(3):
                d.hada_w[s][0] = f(L[f"{pre}w{s + 1}a"])
                d.hada_w[s][1] = f(L[f"{pre}w{s + 1}b"])
            d.pre_hada = f(L[norm])

        self.w = w
        n = len(w.layers)
        layers = (_EncLayer * n)()
        for l, L in enumerate(w.layers):
            e = layers[l]
            b = e.b
            b.norm_in, b.post_norm = f(L["norm_in"]), f(L["post_norm"])
            b.q_norm, b.k_norm = f(L["q_norm"]), f(L["k_norm"])
            b.attn_gate = float(L["attn_gate"])
            for k in ("q_proj", "k_proj", "v_proj", "gate_proj", "out_proj"):
                setattr(b, k, pk(L[k]))
            mlp(b, L, "hada.", "pre_hada")
            mlp(e.hada0, L, "hada_0.", "pre_hada_0")
            for k in ("a_pre", "a_post", "a_res"):
                setattr(b, k, float(L[k]))
            for k in ("b_pre", "b_post", "b_res"):
                setattr(b, k, f(L[k]))
            for k in ("phi_pre", "phi_post", "phi_res"):
                lo, hi = w.phi_rows(k, l)
                setattr(b, k, pk(getattr(w, k), lo, hi))
            e.conv_norm, e.conv_out_norm = f(L["conv_norm"]), f(L["conv_out_norm"])
            e.pw1, e.pw2 = pk(L["pw1"]), pk(L["pw2"])
            e.dw = f(L["dw"])
        self._layers = layers
        self.rope_cos, self.rope_sin = rope_tables(w.qk, w.rope_len, w.rope_theta)
        D = _Decoder()
        D.dim, D.lanes, D.layers, D.heads, D.kv_heads, D.qk, D.vd = (w.dim, w.lanes, n, w.heads, w.kv_heads, w.qk,
                                                                      w.vd)
        D.na, D.nb, D.rank = w.na, w.nb, w.rank
        D.hada_p1 = _ptr(arr(w.hada_p1, np.int32), _i32p)
        D.hada_p2 = _ptr(arr(w.hada_p2, np.int32), _i32p)
        D.rope_cos, D.rope_sin = _ptr(self.rope_cos, _f32p), _ptr(self.rope_sin, _f32p)
        D.rope_len = w.rope_len
        D.final_norm = f(w.final_norm)
        self.e = _Encoder(D, w.dw_k, layers)

    def stack(self, x: np.ndarray, form: int = ENC_ATTEND_INT8, threads: int = 1) -> np.ndarray:
        """encoder.go:167 Stack on x [clips][t][dim] (or [t][dim])."""
        x = _c(x, np.float32)
        shape = x.shape
        x3 = x.reshape(-1, shape[-2], shape[-1])
        clips, t = x3.shape[0], x3.shape[1]
        out = np.zeros_like(x3)
        L = _enc_lib()
        if threads > 1:
            rc = L.wo_enc_stack_mt(ctypes.byref(self.e), _ptr(x3, _f32p), clips, t, form, _ptr(out, _f32p), threads)
        else:
            rc = L.wo_enc_stack(ctypes.byref(self.e), _ptr(x3, _f32p), clips, t, form, _ptr(out, _f32p))
        if rc != 0:
            raise ValueError(f"oracle: {t} frames exceed the RoPE tables ({self.w.rope_len})")
        return out.reshape(shape)
