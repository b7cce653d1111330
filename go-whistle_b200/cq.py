"""The host side of internal/cq on the B200 library: ``Matrix``, ``New``,
``GEMM``, ``GEMMs``.

This mirrors the reference's Go API (internal/cq/matrix.go, kernel.go) name
for name, with the same argument meaning and error behaviour: ``New`` raises
``CQError`` with the reference's error text where Go returns an error, and
misuse raises ``Panic`` with its panic text. Every product runs on the GPU
through the C ABI (include/whistle_b200.h); nothing here computes.

Arrays may be numpy arrays (host memory: the call copies in and out and
synchronises, like the reference's Go slices) or torch CUDA tensors (device
memory: the call enqueues on torch's current stream and returns).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

from . import _lib
from ._lib import CQError, Panic, check, lib

__all__ = ["Packed", "Matrix", "New", "NewGather", "GEMMs", "CQError", "Panic"]


@dataclass
class Packed:
    """cact.Packed (internal/cact/packed.go:18-29): a CQ tensor as stored.

    Index holds Out rows of RowBytes() bytes of LSB-first indices; Norms holds
    Out*Groups() little-endian FP16 values as bytes; Codebook the levels.
    """

    Out: int
    In: int
    Group: int
    Bits: int
    Width: int
    Codebook: np.ndarray
    Index: np.ndarray
    Norms: np.ndarray = field(repr=False)

    def Groups(self) -> int:  # packed.go:32
        return (self.In + self.Group - 1) // self.Group

    def RowBytes(self) -> int:  # packed.go:35
        return self.Groups() * self.Group * self.Width // 8

    def Norm(self, r: int, g: int) -> float:  # packed.go:38
        n = np.frombuffer(np.ascontiguousarray(self.Norms, np.uint8).tobytes(), "<f2")
        return float(n[r * self.Groups() + g])

    # Accessors under the names the oracle uses.
    @property
    def out(self) -> int:
        return self.Out

    @property
    def in_(self) -> int:
        return self.In

    @property
    def group(self) -> int:
        return self.Group

    @property
    def bits(self) -> int:
        return self.Bits

    @property
    def index(self) -> np.ndarray:
        return np.ascontiguousarray(self.Index, np.uint8)

    @property
    def norms16(self) -> np.ndarray:
        return np.frombuffer(np.ascontiguousarray(self.Norms, np.uint8).tobytes(), "<u2").copy()

    @property
    def codebook(self) -> np.ndarray:
        return np.ascontiguousarray(self.Codebook, np.float32)


def _is_device(a) -> bool:
    return hasattr(a, "is_cuda") and bool(a.is_cuda)


def _stream():
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _dptr(t, dtype_name: str):
    if str(t.dtype) != dtype_name:
        raise Panic(_lib.WC_ERR_INVALID, f"cq: {dtype_name} tensor wanted, got {t.dtype}")
    if not t.is_contiguous():
        raise Panic(_lib.WC_ERR_INVALID, "cq: tensor is not contiguous")
    return ctypes.c_void_p(t.data_ptr())


def _hptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def _host_f32(a, writable=False) -> np.ndarray:
    if a is None:
        return np.zeros(0, np.float32)
    if not isinstance(a, np.ndarray) or a.dtype != np.float32 or not a.flags["C_CONTIGUOUS"]:
        if writable:
            raise Panic(_lib.WC_ERR_INVALID, "cq: dst must be a C-contiguous float32 numpy array")
        a = np.ascontiguousarray(a, np.float32)
    return a


class Matrix:
    """internal/cq/matrix.go:25 Matrix: a 2- or 4-bit CQ matrix [out, in],
    resident on the GPU that was current when it was made. Safe for
    concurrent use."""

    __slots__ = ("_h", "_root")

    def __init__(self, handle: ctypes.c_void_p, root=None):
        self._h = handle
        self._root = root  # keeps a parent alive while views exist (storage is shared either way)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                lib().wc_cq_destroy(h)
            except Exception:
                pass
            self._h = None

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def Out(self) -> int:  # matrix.go:99
        return lib().wc_cq_out(self._h)

    def In(self) -> int:  # matrix.go:102
        return lib().wc_cq_in(self._h)

    def Bits(self) -> int:  # matrix.go:105
        return lib().wc_cq_bits(self._h)

    def Prepare(self) -> None:  # matrix.go:111: the device copy is made by New
        return None

    def Bytes(self) -> int:  # matrix.go:121 (device bytes)
        return int(lib().wc_cq_bytes(self._h))

    def Rows(self, lo: int, hi: int) -> "Matrix":  # matrix.go:133
        v = ctypes.c_void_p()
        check(lib().wc_cq_rows(self._h, lo, hi, ctypes.byref(v)))
        return Matrix(v, self)

    def Exact(self) -> "Matrix":  # matrix.go:152
        v = ctypes.c_void_p()
        check(lib().wc_cq_exact(self._h, ctypes.byref(v)))
        return Matrix(v, self)

    def Row(self, dst, r: int) -> None:  # matrix.go:161
        if _is_device(dst):
            if dst.numel() != self.In():
                raise Panic(_lib.WC_ERR_INVALID, f"cq: Row(len {dst.numel()}, {r}) of [{self.Out()}, {self.In()}]")
            check(lib().wc_cq_row(self._h, r, _dptr(dst, "torch.float32"), _stream()))
            return
        d = _host_f32(dst, writable=True)
        check(lib().wc_cq_row_host(self._h, r, _hptr(d), d.size))

    def GEMV(self, dst, x) -> None:  # kernel.go:78
        self.GEMM(dst, x, 1)

    def GEMM(self, dst, x, rows: int) -> None:  # kernel.go:85
        if _is_device(x) or _is_device(dst):
            if not (_is_device(x) and _is_device(dst)):
                raise Panic(_lib.WC_ERR_INVALID, "cq: GEMM mixes host and device arrays")
            out, in_ = self.Out(), self.In()
            if rows < 0 or x.numel() != rows * in_ or dst.numel() != rows * out:
                raise Panic(_lib.WC_ERR_INVALID,
                            f"cq: GEMM(len {dst.numel()}, len {x.numel()}, {rows} rows) on [{out}, {in_}]")
            check(lib().wc_cq_gemm(self._h, _dptr(x, "torch.float32"), _dptr(dst, "torch.float32"), rows,
                                   _stream()))
            return
        d = _host_f32(dst, writable=True)
        xx = _host_f32(x)
        check(lib().wc_cq_gemm_host(self._h, _hptr(xx), xx.size, _hptr(d), d.size, rows))


def New(p: Packed) -> Matrix:
    """internal/cq/matrix.go:46 New: validates p and copies it to the GPU."""
    index = np.ascontiguousarray(p.Index, np.uint8).reshape(-1)
    norms = np.ascontiguousarray(p.Norms, np.uint8).reshape(-1)
    cb = np.ascontiguousarray(p.Codebook, np.float32).reshape(-1)
    h = ctypes.c_void_p()
    check(lib().wc_cq_create(_hptr(index), index.size, _hptr(norms), norms.size, _hptr(cb), cb.size, p.Out, p.In,
                             p.Group, p.Bits, p.Width, ctypes.byref(h)))
    return Matrix(h)


# matrix.go:60 NewGather defers the reference's CPU-side blocked copy; the
# device copy here has no such second layout, so it is New.
NewGather = New


def GEMMs(ms: Sequence[Matrix], dsts: Sequence, x, rows: int) -> None:
    """internal/cq/kernel.go:134 GEMMs: dsts[k] = x · ms[k]ᵀ, tables shared."""
    if len(ms) != len(dsts):
        raise Panic(_lib.WC_ERR_INVALID, f"cq: GEMMs of {len(ms)} matrices into {len(dsts)} outputs")
    n = len(ms)
    hs = (ctypes.c_void_p * max(n, 1))(*[m.handle for m in ms])
    if _is_device(x):
        for k, m in enumerate(ms):
            if rows < 0 or x.numel() != rows * m.In() or dsts[k].numel() != rows * m.Out():
                raise Panic(_lib.WC_ERR_INVALID, f"cq: GEMMs(len {dsts[k].numel()}, len {x.numel()}, {rows} rows) "
                                                 f"on [{m.Out()}, {m.In()}]")
        ys = (ctypes.c_void_p * max(n, 1))(*[_dptr(d, "torch.float32").value for d in dsts])
        check(lib().wc_cq_gemms(hs, n, _dptr(x, "torch.float32"), ys, rows, _stream()))
        return
    xx = _host_f32(x)
    ds = [_host_f32(d, writable=True) for d in dsts]
    ys = (ctypes.c_void_p * max(n, 1))(*[d.ctypes.data for d in ds])
    lens = (ctypes.c_size_t * max(n, 1))(*[d.size for d in ds])
    check(lib().wc_cq_gemms_host(hs, n, _hptr(xx), xx.size, ys, lens, rows))
