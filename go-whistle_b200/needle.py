"""The host side of internal/needle's int8 numerics on the B200 library:
``QuantizeRow``, ``QuantizeRows``, ``Int8Rows``, ``AttendInt8``,
``AttendInt8Spans`` (internal/needle/int8.go), with the reference's names,
argument meaning and panics. The arithmetic runs on the GPU through the C
ABI; host (numpy) arguments are copied to the device and back.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Callable

import numpy as np

from . import _lib
from ._lib import Panic, check, lib

__all__ = ["QuantizeRow", "QuantizeRows", "NewInt8Rows", "Int8Rows", "AttendInt8", "AttendInt8Spans", "Span"]


def _hp(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def _dp(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def QuantizeRow(q: np.ndarray, x) -> np.float32:
    """int8.go:36 QuantizeRow: q (int8, len(x)) gets the codes, returns s."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    if q.dtype != np.int8 or q.size < x.size:
        raise Panic(_lib.WC_ERR_INVALID, f"needle: QuantizeRow into {q.size} codes of {x.size} values")
    qq = np.zeros(x.size, np.int8)
    s = np.zeros(1, np.float32)
    if x.size:
        check(lib().wc_quantize_rows_host(_hp(x), x.size, x.size, x.size, _hp(qq), _hp(s)))
    else:
        s[0] = 1.0
    q[: x.size] = qq
    return s[0]


@dataclass
class Int8Rows:
    """int8.go:99 Int8Rows: rows of Cols int8 codes, a float32 scale per
    chunk of Width codes."""

    Cols: int
    Width: int
    Q: np.ndarray = field(default_factory=lambda: np.zeros(0, np.int8))
    S: np.ndarray = field(default_factory=lambda: np.zeros(0, np.float32))

    def Len(self) -> int:  # int8.go:144
        return 0 if self.Cols == 0 else self.Q.size // self.Cols

    def Append(self, x) -> "Int8Rows":  # int8.go:125
        x = np.ascontiguousarray(x, np.float32).reshape(-1)
        if x.size % self.Cols != 0:
            raise Panic(_lib.WC_ERR_INVALID, f"needle: {x.size} values are not rows of {self.Cols}")
        q = np.zeros(x.size, np.int8)
        s = np.zeros(x.size // self.Width, np.float32)
        if x.size:
            check(lib().wc_quantize_rows_host(_hp(x), x.size, self.Cols, self.Width, _hp(q), _hp(s)))
        return Int8Rows(self.Cols, self.Width, np.concatenate([self.Q, q]), np.concatenate([self.S, s]))

    def Floats(self) -> np.ndarray:  # int8.go:163
        return (self.Q.astype(np.float32) * np.repeat(self.S, self.Width)).astype(np.float32)

    def Bytes(self) -> int:  # int8.go:174
        return self.Q.size + 4 * self.S.size


def NewInt8Rows(cols: int, width: int) -> Int8Rows:  # int8.go:107
    if width <= 0 or cols % width != 0:
        raise Panic(_lib.WC_ERR_INVALID, f"needle: int8 rows of {cols} in chunks of {width}")
    return Int8Rows(cols, width)


def QuantizeRows(x, cols: int, width: int) -> Int8Rows:  # int8.go:116
    return NewInt8Rows(cols, width).Append(x)


@dataclass
class Span:
    """needle.Span: key rows [Lo, Hi)."""

    Lo: int = 0
    Hi: int = 0

    def Len(self) -> int:
        return self.Hi - self.Lo


def AttendInt8Spans(q, t: int, heads: int, k: Int8Rows, v: Int8Rows, spans: Callable[[int], tuple],
                    scale: float, quantQ: bool, probs: np.ndarray | None) -> np.ndarray:
    """int8.go:208 AttendInt8Spans on the GPU. spans(i) returns two Spans."""
    import torch

    qk, vd = k.Width, v.Width
    kv_heads = k.Cols // qk
    n = k.Len()
    sp = np.zeros((max(t, 1), 4), np.int32)
    for i in range(t):
        a, b = spans(i)
        sp[i] = (a.Lo, a.Hi, b.Lo, b.Hi)
    dev = torch.device("cuda")
    qd = torch.from_numpy(np.ascontiguousarray(q, np.float32).reshape(-1)).to(dev)
    k8 = torch.from_numpy(k.Q.reshape(-1) if k.Q.size else np.zeros(1, np.int8)).to(dev)
    ks = torch.from_numpy(k.S.reshape(-1) if k.S.size else np.zeros(1, np.float32)).to(dev)
    v8 = torch.from_numpy(v.Q.reshape(-1) if v.Q.size else np.zeros(1, np.int8)).to(dev)
    vs = torch.from_numpy(v.S.reshape(-1) if v.S.size else np.zeros(1, np.float32)).to(dev)
    spd = torch.from_numpy(sp.reshape(-1)).to(dev)
    out = torch.zeros(t * heads * vd, dtype=torch.float32, device=dev)
    pd = torch.zeros(max(t * heads * n, 1), dtype=torch.float32, device=dev) if probs is not None else None
    check(lib().wc_attend_int8(_dp(qd), t, heads, _dp(k8), _dp(ks), _dp(v8), _dp(vs), n, kv_heads, qk, vd, _dp(spd),
                               float(scale), 1 if quantQ else 0, _dp(pd) if pd is not None else None, _dp(out),
                               _stream()))
    torch.cuda.current_stream().synchronize()
    if probs is not None:
        got = pd.cpu().numpy()[: t * heads * n]
        mask = np.zeros(t * heads * n, bool)
        for i in range(t):
            a, b = spans(i)
            for h in range(heads):
                base = (i * heads + h) * n
                mask[base + a.Lo: base + a.Hi] = True
                mask[base + b.Lo: base + b.Hi] = True
        probs[: t * heads * n][mask] = got[mask]
    return out.cpu().numpy()


def AttendInt8(q, t: int, heads: int, k: Int8Rows, v: Int8Rows, keys: Callable[[int], int], scale: float,
               quantQ: bool, probs: np.ndarray | None) -> np.ndarray:
    """int8.go:194 AttendInt8: row i sees the first keys(i) rows."""
    return AttendInt8Spans(q, t, heads, k, v, lambda i: (Span(), Span(0, keys(i))), scale, quantQ, probs)
