"""CPU oracle for go-whistle's quantized hot path — TEST INFRASTRUCTURE ONLY.

This package is the checker that the CUDA library is compared against and the
timed CPU baseline of ``bench.py``. Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference``) may use
it; the product (``go-whistle_b200``) never imports it.

The C sources (``cq_oracle.c``, ``lut_avx2.c``, ``needle_oracle.c``, ``decoder_oracle.c``) restate the reference's Go
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
    srcs = [HERE / n for n in ("cq_oracle.c", "lut_avx2.c", "needle_oracle.c", "decoder_oracle.c", "oracle.h", "par.h",
                                "Makefile")]
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
