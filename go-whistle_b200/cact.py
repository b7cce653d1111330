"""The .cact deployment container (internal/cact): parse, read and write.

A .cact file is a fixed little-endian header with the model geometry
(format.go:52-84), a 28-float codebook (2-, 3- and 4-bit levels, already
scaled by 1/sqrt(group)), a directory of 44-byte records (format.go:125-135)
and each record's blob at the next 64-byte boundary, in directory order.
Tensors are positional; ``whistle_names()`` maps Whistle's 681 records to
names and shapes (names.go:272).

This module mirrors the reference's reader API name for name (``Parse``,
``Open``, ``File.Header/Len/Record/Codebook/FP32/FP16/Float32/Raw/CQ/
CQPacked``) with its validation and error texts (cact.go:36-202), adds the
writer a synthetic file needs (the layout cact_test.go encodeTestFile and
export.py _pack_cact describe), and hands CQ tensors to the device as
``cq.Packed`` without dequantising them (packed.go:45).
"""

from __future__ import annotations

import dataclasses
import math
import struct
from typing import Optional, Sequence

import numpy as np

from .cq import Packed

TAG = 0x05E12A84
ALIGN = 64
HEADER_SIZE = 196  # "<48If"
RECORD_SIZE = 44   # "<BBHIIIIQQII"
CODEBOOK_LEN = 28  # cb2[4] | cb3[8] | cb4[16]
MAX_DIMS = 4
TERNARY_RECORD_BITS = 5  # trits stored as 2-bit crumbs (cq.go:11)

FP16, FP32, CQ, RAW = 1, 2, 3, 4
_DTYPE_NAMES = {FP16: "FP16", FP32: "FP32", CQ: "CQ", RAW: "RAW"}
_MAX_INT64 = (1 << 63) - 1

_HEADER_FMT = struct.Struct("<48If")
_RECORD_FMT = struct.Struct("<BBHIIIIQQII")
assert _HEADER_FMT.size == HEADER_SIZE and _RECORD_FMT.size == RECORD_SIZE


class CactError(ValueError):
    """A .cact file or call the reader rejects (the reference's error)."""


class DTypeError(CactError):
    """A reader called on a tensor of another dtype (cact.go:14 ErrDType)."""


def dtype_name(d: int) -> str:
    """format.go:33 DType.String."""
    return _DTYPE_NAMES.get(d, f"dtype {d}")


def _go_list(vals) -> str:
    return "[" + " ".join(str(int(v)) for v in vals) + "]"


@dataclasses.dataclass
class Header:
    """format.go:52 Header, field for field in file order."""

    Tag: int = TAG
    NumTensors: int = 0
    CodebookLen: int = CODEBOOK_LEN
    KVWindow: int = 0
    KVBits: int = 0
    Vocab: int = 0
    OutVocab: int = 0
    DModel: int = 0
    NumHeads: int = 0
    NumKVHeads: int = 0
    NumLayers: int = 0
    QKHeadDim: int = 0
    VHeadDim: int = 0
    MaxSeqLen: int = 0
    HadaN: int = 0
    MHCLanes: int = 0
    SlidingWindow: int = 0
    GlobalMaskLo: int = 0
    GlobalMaskHi: int = 0
    QKVConvTaps: int = 0
    EngramSlots: int = 0
    EngramSubDim: int = 0
    NumEngramTables: int = 0
    EngramConvTaps: int = 0
    EngramConvDilation: int = 0
    EngramSeedHeads: int = 0
    NumEngramOrders: int = 0
    EngramOrders: tuple = (0, 0, 0, 0)
    NumEngramSites: int = 0
    EngramSites: tuple = (0,) * 16
    RopeTheta: float = 0.0

    _SCALARS = ("Tag", "NumTensors", "CodebookLen", "KVWindow", "KVBits", "Vocab", "OutVocab", "DModel", "NumHeads",
                "NumKVHeads", "NumLayers", "QKHeadDim", "VHeadDim", "MaxSeqLen", "HadaN", "MHCLanes",
                "SlidingWindow", "GlobalMaskLo", "GlobalMaskHi", "QKVConvTaps", "EngramSlots", "EngramSubDim",
                "NumEngramTables", "EngramConvTaps", "EngramConvDilation", "EngramSeedHeads", "NumEngramOrders")

    def pack(self) -> bytes:
        vals = [int(getattr(self, k)) for k in self._SCALARS]
        vals += [int(v) for v in self.EngramOrders] + [int(self.NumEngramSites)] + [int(v) for v in self.EngramSites]
        return _HEADER_FMT.pack(*vals, float(self.RopeTheta))

    @classmethod
    def unpack(cls, data: bytes) -> "Header":
        v = _HEADER_FMT.unpack(data[:HEADER_SIZE])
        h = cls(**dict(zip(cls._SCALARS, v[:27])))
        h.EngramOrders = tuple(v[27:31])
        h.NumEngramSites = v[31]
        h.EngramSites = tuple(v[32:48])
        h.RopeTheta = v[48]
        return h

    def GlobalLayers(self) -> list[int]:
        """format.go:87: the full-attention layers of the 64-bit mask."""
        mask = (self.GlobalMaskHi << 32) | self.GlobalMaskLo
        return [i for i in range(min(self.NumLayers, 64)) if mask >> i & 1]

    def Orders(self) -> list[int]:
        """format.go:103 (Parse guarantees NumEngramOrders <= 4)."""
        return [int(v) for v in self.EngramOrders[:self.NumEngramOrders]]

    def Sites(self) -> list[int]:
        """format.go:109 (Parse guarantees NumEngramSites <= 16)."""
        return [int(v) for v in self.EngramSites[:self.NumEngramSites]]


@dataclasses.dataclass
class Record:
    """format.go:125 Record: one 44-byte directory entry."""

    DType: int = 0
    NDim: int = 0
    Pad: int = 0
    Shape: tuple = (0, 0, 0, 0)
    Offset: int = 0
    NBytes: int = 0
    Group: int = 0
    Bits: int = 0

    def pack(self) -> bytes:
        return _RECORD_FMT.pack(self.DType, self.NDim, self.Pad, *self.Shape, self.Offset, self.NBytes, self.Group,
                                self.Bits)

    @classmethod
    def unpack(cls, data: bytes) -> "Record":
        v = _RECORD_FMT.unpack(data)
        return cls(v[0], v[1], v[2], tuple(v[3:7]), v[7], v[8], v[9], v[10])

    def Dims(self) -> list[int]:
        return [int(d) for d in self.Shape[:min(self.NDim, MAX_DIMS)]]

    def Numel(self) -> int:
        n = 1
        for d in self.Dims():
            n *= d
        return n


def _blob_size(r: Record) -> int:
    """cact.go:152 blobSize: the bytes the dtype and shape imply, or -1 for
    RAW, whose length is free."""
    if r.DType in (FP16, FP32):
        numel = 1
        for d in r.Shape[:r.NDim]:
            numel *= int(d)
        n = numel * (2 if r.DType == FP16 else 4)
        if n > _MAX_INT64:
            raise CactError("blob size overflows")
        return n
    if r.DType == RAW:
        if r.NDim != 0:
            raise CactError(f"RAW needs ndim 0, got {r.NDim}")
        return -1
    if r.DType == CQ:
        return _cq_blob_size(r)
    raise CactError(f"unknown {dtype_name(r.DType)}")


def _cq_blob_size(r: Record) -> int:
    """cact.go:180 cqBlobSize (export.py _packed_row_bytes): per row the
    packed indices of the group-padded input, then one FP16 norm a group."""
    if r.NDim != 2:
        raise CactError(f"CQ needs ndim 2, got {r.NDim}")
    if r.Group == 0 or r.Group % 8 != 0:
        raise CactError(f"CQ group {r.Group} is not a positive multiple of 8")
    if r.Bits < 1 or r.Bits > 5:
        raise CactError(f"CQ bits {r.Bits} not in 1..5")
    out, in_, group = int(r.Shape[0]), int(r.Shape[1]), int(r.Group)
    groups = (in_ + group - 1) // group
    idx_bits = 2 if r.Bits == TERNARY_RECORD_BITS else int(r.Bits)
    n = out * (groups * group * idx_bits // 8 + groups * 2)
    if n > _MAX_INT64:
        raise CactError("blob size overflows")
    return n


def _check_record(r: Record, prev_end: int, size: int) -> None:
    """cact.go:116 checkRecord: the entry against the file size and the end
    of the previous blob (blobs lie in directory order)."""
    if r.Pad != 0:
        raise CactError(f"non-zero pad {r.Pad}")
    if r.NDim > MAX_DIMS:
        raise CactError(f"ndim {r.NDim} > {MAX_DIMS}")
    if any(r.Shape[k] != 0 for k in range(r.NDim, MAX_DIMS)):
        raise CactError(f"shape {_go_list(r.Shape)} has a dimension past ndim {r.NDim}")
    want = _blob_size(r)
    if r.Offset % ALIGN != 0:
        raise CactError(f"offset {r.Offset} is not {ALIGN}-byte aligned")
    if r.Offset < prev_end:
        raise CactError(f"blob at {r.Offset} overlaps the directory or the previous blob (ends at {prev_end})")
    if r.Offset > size or r.NBytes > size - r.Offset:
        raise CactError(f"blob [{r.Offset}, +{r.NBytes}) runs past EOF ({size} bytes)")
    if want >= 0 and want != r.NBytes:
        raise CactError(f"nbytes {r.NBytes}, want {want} for shape {_go_list(r.Dims())}")


def _check_header(h: Header) -> None:
    """cact.go:99 checkHeader."""
    if h.Tag != TAG:
        raise CactError(f"cact: bad tag 0x{h.Tag:08x}, want 0x{TAG:08x}")
    if h.CodebookLen != CODEBOOK_LEN:
        raise CactError(f"cact: codebook length {h.CodebookLen}, want {CODEBOOK_LEN}")
    if h.NumEngramOrders > 4:
        raise CactError(f"cact: {h.NumEngramOrders} engram orders, the header holds 4")
    if h.NumEngramSites > 16:
        raise CactError(f"cact: {h.NumEngramSites} engram sites, the header holds 16")


def float16_to_float32(bits) -> np.ndarray:
    """half.go float16ToFloat32: IEEE binary16 widened exactly (subnormals,
    infinities and NaN payloads included)."""
    return np.asarray(bits, np.uint16).view(np.float16).astype(np.float32)


def unpack_lsb(packed: np.ndarray, width: int, count: int) -> np.ndarray:
    """cq.go:128 unpackLSB over rows: index k of a row occupies bits
    [k·width, (k+1)·width) of its LSB-first bitstream. packed is
    [rows][count·width/8] bytes; returns [rows][count] uint8."""
    packed = np.asarray(packed, np.uint8)
    rows = packed.shape[0]
    bits = np.unpackbits(packed.reshape(rows, -1), axis=1, bitorder="little")[:, :count * width]
    bits = bits.reshape(rows, count, width).astype(np.uint8)
    weights = (1 << np.arange(width, dtype=np.uint8)).astype(np.uint8)
    return (bits * weights).sum(axis=2).astype(np.uint8)


def pack_lsb(idx: np.ndarray, width: int) -> np.ndarray:
    """The inverse of unpack_lsb: [rows][count] indices to LSB-first bytes
    (count·width a multiple of 8)."""
    idx = np.asarray(idx, np.uint8)
    rows, count = idx.shape
    bits = ((idx[:, :, None] >> np.arange(width, dtype=np.uint8)) & 1).astype(np.uint8).reshape(rows, count * width)
    return np.packbits(bits, axis=1, bitorder="little")


def _crumbs_to_trits(idx: np.ndarray, row0: int = 0) -> np.ndarray:
    """cq.go:150 crumbsToTrits: crumbs 3, 0, 1 are the trits 0, 1, 2."""
    bad = np.argwhere(idx == 2)
    if bad.size:
        r, k = bad[0]
        raise CactError(f"row {row0 + r}: ternary crumb 2 at column {k} is not 0, 1 or 3")
    out = idx.copy()
    out[idx == 3] = 0
    out[idx == 0] = 1
    out[idx == 1] = 2
    return out


def fwht_rows(x: np.ndarray) -> np.ndarray:
    """cq.go:169 fwht along the last axis, in float32, stage by stage
    (h = 1, 2, 4, …), each butterfly (a, b) -> (a + b, a - b)."""
    x = np.array(x, np.float32, copy=True)
    n = x.shape[-1]
    h = 1
    while h < n:
        v = x.reshape(x.shape[:-1] + (n // (2 * h), 2, h))
        a, b = v[..., 0, :].copy(), v[..., 1, :].copy()
        v[..., 0, :] = a + b
        v[..., 1, :] = a - b
        h *= 2
    return x


class File:
    """cact.go:17 File: a parsed container; the readers check only the
    index and the dtype (Parse validated the directory)."""

    def __init__(self, data: bytes, header: Header, codebook: np.ndarray, records: list[Record]):
        self._data, self._header, self._codebook, self._records = data, header, codebook, records

    def Header(self) -> Header:
        return dataclasses.replace(self._header)

    def Len(self) -> int:
        return len(self._records)

    def Record(self, i: int) -> Record:
        if i < 0 or i >= len(self._records):
            raise CactError(f"cact: tensor {i} out of range [0, {len(self._records)})")
        return dataclasses.replace(self._records[i])

    def Codebook(self, width: int) -> np.ndarray:
        """cact.go:229: a copy of the stored levels for 2, 3 or 4 bits."""
        span = {2: (0, 4), 3: (4, 12), 4: (12, 28)}.get(width)
        if span is None:
            raise CactError(f"cact: no stored codebook for {width}-bit CQ")
        return self._codebook[span[0]:span[1]].copy()

    def _blob(self, i: int, want: int) -> memoryview:
        rec = self.Record(i)
        if rec.DType != want:
            raise DTypeError(f"cact: tensor {i} is {dtype_name(rec.DType)}, not {dtype_name(want)}: wrong dtype")
        return memoryview(self._data)[rec.Offset:rec.Offset + rec.NBytes]

    def FP32(self, i: int) -> np.ndarray:
        return np.frombuffer(self._blob(i, FP32), "<f4").astype(np.float32)

    def FP16(self, i: int) -> np.ndarray:
        return float16_to_float32(np.frombuffer(self._blob(i, FP16), "<u2"))

    def Float32(self, i: int) -> np.ndarray:
        return self.FP16(i) if self.Record(i).DType == FP16 else self.FP32(i)

    def Raw(self, i: int) -> bytes:
        return bytes(self._blob(i, RAW))

    def _levels(self, rec: Record) -> np.ndarray:
        """cq.go:44 cqLevels: the stored codebook for 2-4 bits; the analytic
        1-bit (±sqrt(2/pi)) and ternary (±1.2240064, 0) levels over sqrt(group)."""
        if rec.Bits == 1:
            c = math.sqrt(2 / math.pi)
            unit = [-c, c]
        elif rec.Bits == TERNARY_RECORD_BITS:
            unit = [-1.2240064, 0.0, 1.2240064]
        else:
            return self.Codebook(int(rec.Bits))
        return np.array([u / math.sqrt(rec.Group) for u in unit], np.float32)

    def CQ(self, i: int) -> np.ndarray:
        """cq.go:21 CQ: the dequantised [out][in] float32 matrix, per group
        H·(cb[idx]·norm/sqrt(group)) with the ±1 Sylvester H, padding
        columns dropped (cq.go:68 dequantCQ)."""
        blob = self._blob(i, CQ)
        rec = self._records[i]
        try:
            cb = self._levels(rec)
            return _dequant(rec, np.frombuffer(blob, np.uint8), cb)
        except CactError as e:
            raise CactError(f"cact: tensor {i}: {e}") from None

    def CQPacked(self, i: int) -> Packed:
        """packed.go:45 CQPacked: the stored form (index bitstream, FP16
        norms) and the codebook CQ would use, ready for cq.New."""
        blob = self._blob(i, CQ)
        rec = self._records[i]
        if rec.Group & (rec.Group - 1):
            raise CactError(f"cact: tensor {i}: CQ group {rec.Group} is not a power of two")
        try:
            cb = self._levels(rec)
        except CactError as e:
            raise CactError(f"cact: tensor {i}: {e}") from None
        out, in_, group = int(rec.Shape[0]), int(rec.Shape[1]), int(rec.Group)
        width = 2 if rec.Bits == TERNARY_RECORD_BITS else int(rec.Bits)
        groups = (in_ + group - 1) // group
        n = out * groups * group * width // 8
        raw = np.frombuffer(blob, np.uint8)
        return Packed(Out=out, In=in_, Group=group, Bits=int(rec.Bits), Width=width, Codebook=cb,
                      Index=raw[:n], Norms=raw[n:])


def _dequant(rec: Record, blob: np.ndarray, cb: np.ndarray) -> np.ndarray:
    out, in_, group = int(rec.Shape[0]), int(rec.Shape[1]), int(rec.Group)
    if group & (group - 1):
        raise CactError(f"CQ group {group} is not a power of two")
    groups = (in_ + group - 1) // group
    in_pad = groups * group
    width = 2 if rec.Bits == TERNARY_RECORD_BITS else int(rec.Bits)
    row_bytes = in_pad * width // 8
    idx = unpack_lsb(blob[:out * row_bytes].reshape(out, row_bytes), width, in_pad)
    if rec.Bits == TERNARY_RECORD_BITS:
        idx = _crumbs_to_trits(idx)
    norms = float16_to_float32(blob[out * row_bytes:].view("<u2")).reshape(out, groups)
    s = norms * np.float32(1.0 / math.sqrt(group))  # float32 products, as the reference's
    vals = cb[idx].reshape(out, groups, group) * s[:, :, None]
    w = fwht_rows(vals).reshape(out, in_pad)
    return np.ascontiguousarray(w[:, :in_])


def Parse(data: bytes) -> File:
    """cact.go:36 Parse: validates and indexes data (the File keeps it)."""
    data = bytes(data)
    size = len(data)
    if size < HEADER_SIZE:
        raise CactError(f"cact: {size} bytes is shorter than the {HEADER_SIZE}-byte header")
    h = Header.unpack(data)
    _check_header(h)
    dir_start = HEADER_SIZE + 4 * CODEBOOK_LEN
    dir_end = dir_start + h.NumTensors * RECORD_SIZE
    if dir_end > size:
        raise CactError(f"cact: directory of {h.NumTensors} records ends at {dir_end}, past EOF ({size} bytes)")
    codebook = np.frombuffer(data, "<f4", CODEBOOK_LEN, HEADER_SIZE).astype(np.float32)
    records = []
    prev_end = dir_end
    for i in range(h.NumTensors):
        at = dir_start + i * RECORD_SIZE
        r = Record.unpack(data[at:at + RECORD_SIZE])
        try:
            _check_record(r, prev_end, size)
        except CactError as e:
            raise CactError(f"cact: tensor {i} ({dtype_name(r.DType)}): {e}") from None
        records.append(r)
        prev_end = r.Offset + r.NBytes
    return File(data, h, codebook, records)


def Open(path: str) -> File:
    """cact.go:26 Open."""
    try:
        with open(path, "rb") as fh:
            data = fh.read()
    except OSError as e:
        raise CactError(f"cact: {e}") from None
    return Parse(data)


# ---- writing -----------------------------------------------------------


@dataclasses.dataclass
class Tensor:
    """One record to write: its dtype, logical shape, blob and CQ fields."""

    dtype: int
    shape: Sequence[int]
    blob: bytes
    group: int = 0
    bits: int = 0


def fp16_tensor(a) -> Tensor:
    a = np.asarray(a, np.float32)
    return Tensor(FP16, a.shape, a.astype("<f2").tobytes())


def fp32_tensor(a) -> Tensor:
    a = np.asarray(a, np.float32)
    return Tensor(FP32, a.shape, a.astype("<f4").tobytes())


def cq_tensor(p: Packed) -> Tensor:
    """A CQ record from a cq.Packed: its index bitstream, then its norms."""
    bits = int(p.Bits)
    blob = np.ascontiguousarray(p.Index, np.uint8).tobytes() + np.ascontiguousarray(p.Norms, np.uint8).tobytes()
    return Tensor(CQ, (int(p.Out), int(p.In)), blob, int(p.Group), bits)


def raw_tensor(b: bytes) -> Tensor:
    return Tensor(RAW, (), bytes(b))


def encode(header: Header, codebook, tensors: Sequence[Tensor]) -> bytes:
    """A .cact file laid out as export.py _pack_cact writes one: header,
    codebook, directory, then each blob at the next 64-byte boundary with
    zero padding between. header.NumTensors and CodebookLen are set here."""
    cb = np.asarray(codebook, np.float32).reshape(-1)
    h = dataclasses.replace(header, NumTensors=len(tensors), CodebookLen=cb.size)
    pos = HEADER_SIZE + 4 * cb.size + RECORD_SIZE * len(tensors)
    recs = []
    for t in tensors:
        pos = (pos + ALIGN - 1) & ~(ALIGN - 1)
        shape = tuple(int(d) for d in t.shape)
        if len(shape) > MAX_DIMS:
            raise CactError(f"cact: shape {shape} has more than {MAX_DIMS} dimensions")
        recs.append(Record(t.dtype, len(shape), 0, shape + (0,) * (MAX_DIMS - len(shape)), pos, len(t.blob),
                           t.group, t.bits))
        pos += len(t.blob)
    out = bytearray(h.pack())
    out += cb.astype("<f4").tobytes()
    for r in recs:
        out += r.pack()
    for r, t in zip(recs, tensors):
        out += bytes(r.Offset - len(out))
        out += t.blob
    return bytes(out)


# ---- Whistle's tensor map ---------------------------------------------

DERIVED, RESHAPE, TRANSPOSE, LANE_MAJOR = 0, 1, 2, 3
_TRANSFORM_NAMES = {DERIVED: "derived", RESHAPE: "reshape", TRANSPOSE: "transpose", LANE_MAJOR: "lane-major"}


def transform_name(t: int) -> str:
    """names.go:30 Transform.String."""
    return _TRANSFORM_NAMES.get(t, f"transform {t}")


@dataclasses.dataclass(frozen=True)
class Entry:
    """names.go:46 Entry: a record's name, its safetensors source (layer
    slice, transform) and its .cact shape (None for the RAW tokenizer)."""

    Name: str
    Source: str
    Layer: int
    Transform: int
    Shape: Optional[tuple]


# Whistle's geometry (names.go:55-73).
W_LAYERS, W_DIM, W_Q, W_KV, W_V, W_HEAD, W_LANES = 8, 512, 384, 96, 128, 48, 4
W_VOCAB, W_TAPS, W_KERNEL, W_STEM, W_SLOTS, W_TABLES, W_SUB = 8199, 3, 9, 128, 18432, 4, 128
W_ENGRAMS, W_BINS, W_MELS, W_RANK = 2, 257, 80, 8


def whistle_names() -> list[Entry]:
    """names.go:272 WhistleNames: entry i names record i of whistle.cact.
    The decoder first (embedding, 8 × 27 block tensors, the stack's mHC,
    the Hadamard permutations, two engram sites, the final norm), the audio
    manifest, 8 × 10 cross-attention tensors, pe_gate, then the encoder
    (8 × 43 block tensors, its mHC and final norm), the conv stem, the mel
    filterbank and the tokenizer: 681 records."""
    D = W_DIM

    def vec(suf, path, n):
        return (suf, path, RESHAPE, (n,))

    def mat(suf, path, r, c):
        return (suf, path, RESHAPE, (r, c))

    def kern(suf, path, out):  # a Flax (dim, out) kernel stored (out, dim)
        return (suf, path, TRANSPOSE, (out, D))

    def hada(suf, path):
        ps = [vec(suf + d, path + d, D) for d in ("d1", "d2", "b2", "d3", "d4")]
        for w in ("w1", "w2", "w3"):
            ps += [mat(suf + w + "a", path + w + "a", 16, 16), mat(suf + w + "b", path + w + "b", 32, 32)]
        return ps + [mat(suf + "cond_v", path + "cond_v", D, W_RANK), mat(suf + "cond_u", path + "cond_u", W_RANK, D)]

    qkv = [kern("q_proj", "self_attn/q_proj/kernel", W_Q), kern("k_proj", "self_attn/k_proj/kernel", W_KV),
           kern("v_proj", "self_attn/v_proj/kernel", W_V)]
    gate_out = [kern("gate_proj", "self_attn/gate_proj/kernel", D), kern("out_proj", "self_attn/out_proj/kernel", D)]
    dec_block = ([vec("norm_in", "ZCRMSNorm_0/scale", D)] + qkv +
                 [mat("q_taps", "self_attn/q_taps", W_TAPS, W_Q), mat("k_taps", "self_attn/k_taps", W_TAPS, W_KV),
                  mat("v_taps", "self_attn/v_taps", W_TAPS, W_V), vec("q_norm", "self_attn/q_norm/scale", W_HEAD),
                  vec("k_norm", "self_attn/k_norm/scale", W_HEAD)] + gate_out +
                 [vec("post_norm", "post_attn_norm/scale", D), vec("attn_gate", "attn_gate", 1),
                  vec("pre_hada", "pre_hada_norm/scale", D)] + hada("", "hadamard_mlp/"))
    cross_block = [vec("norm_in", "cross_norm/scale", D), kern("q_proj", "cross_attn/q_proj/kernel", W_Q),
                   kern("k_proj", "cross_attn/k_proj/kernel", W_Q), kern("v_proj", "cross_attn/v_proj/kernel", D),
                   kern("gate_proj", "cross_attn/gate_proj/kernel", D),
                   kern("out_proj", "cross_attn/out_proj/kernel", D), vec("q_norm", "cross_attn/q_norm/scale", W_HEAD),
                   vec("k_norm", "cross_attn/k_norm/scale", W_HEAD), vec("post_norm", "post_cross_norm/scale", D),
                   vec("attn_gate", "cross_gate", 1)]
    enc_block = ([vec("pre_hada_0", "pre_hada_norm_0/scale", D), vec("norm_in", "ZCRMSNorm_0/scale", D),
                  vec("post_norm", "post_attn_norm/scale", D), vec("conv_norm", "conv_norm/scale", D),
                  vec("conv_out_norm", "conv_out_norm/scale", D), vec("pre_hada", "pre_hada_norm/scale", D)] +
                 qkv + gate_out +
                 [vec("q_norm", "self_attn/q_norm/scale", W_HEAD), vec("k_norm", "self_attn/k_norm/scale", W_HEAD),
                  vec("attn_gate", "attn_gate", 1), kern("pw1", "pw1/kernel", 2 * D), kern("pw2", "pw2/kernel", D),
                  mat("dw", "dw", W_KERNEL, D)] + hada("hada_0.", "hadamard_mlp_0/") + hada("hada.", "hadamard_mlp/"))

    def layered(fmt, prefix, parts):
        return [Entry(fmt % l + suf, prefix + path, l, tr, shape) for l in range(W_LAYERS)
                for suf, path, tr, shape in parts]

    def mhc(name, path):
        l, n, nc = W_LAYERS, W_LANES, W_LANES * D
        return [Entry(name + "mhc_a_pre", path + "mhc_a_pre", -1, RESHAPE, (l,)),
                Entry(name + "mhc_a_post", path + "mhc_a_post", -1, RESHAPE, (l,)),
                Entry(name + "mhc_a_res", path + "mhc_a_res", -1, RESHAPE, (l,)),
                Entry(name + "mhc_b_pre", path + "mhc_b_pre", -1, RESHAPE, (l, n)),
                Entry(name + "mhc_b_post", path + "mhc_b_post", -1, RESHAPE, (l, n)),
                Entry(name + "mhc_b_res", path + "mhc_b_res", -1, RESHAPE, (l, n, n)),
                Entry(name + "mhc_phi_pre", path + "mhc_phi_pre", -1, LANE_MAJOR, (l * n, nc)),
                Entry(name + "mhc_phi_post", path + "mhc_phi_post", -1, LANE_MAJOR, (l * n, nc)),
                Entry(name + "mhc_phi_res", path + "mhc_phi_res", -1, LANE_MAJOR, (l * n * n, nc))]

    def engram(s):
        name, path = f"engram{s}.", f"engrams_{s}/"
        return [Entry(name + "tables", path + "embedding", -1, RESHAPE, (W_TABLES * W_SLOTS, W_SUB)),
                Entry(name + "key_proj", path + "key_proj/kernel", -1, TRANSPOSE, (D, D)),
                Entry(name + "value_proj", path + "value_proj/kernel", -1, TRANSPOSE, (D, D)),
                Entry(name + "taps", path + "taps", -1, RESHAPE, (W_TABLES, D))]

    es = [Entry("embedding", "embedding/embedding", -1, RESHAPE, (W_VOCAB, D))]
    es += layered("layer%02d.", "stack/layers/block/", dec_block)
    es += mhc("", "stack/")
    es += [Entry("hada_p1", "", -1, DERIVED, (D,)), Entry("hada_p2", "", -1, DERIVED, (D,))]
    for s in range(W_ENGRAMS):
        es += engram(s)
    es += [Entry("final_norm", "stack/final_norm/scale", -1, RESHAPE, (D,)),
           Entry("audio.manifest", "", -1, DERIVED, (13,))]
    es += layered("cross%02d.", "stack/layers/block/", cross_block)
    es += [Entry("pe_gate", "pe_gate", -1, RESHAPE, (1,))]
    es += layered("enc%02d.", "encoder/layers/block/", enc_block)
    es += mhc("enc.", "encoder/")
    es += [Entry("enc.final_norm", "encoder/final_norm/scale", -1, RESHAPE, (D,))]
    es += [Entry("stem.w", "stem/w", -1, RESHAPE, (9, W_STEM)),
           Entry("stem.dw_1", "stem/dw_1", -1, RESHAPE, (9, W_STEM)),
           Entry("stem.pw_1", "stem/pw_1/kernel", -1, TRANSPOSE, (W_STEM, W_STEM)),
           Entry("stem.dw_2", "stem/dw_2", -1, RESHAPE, (9, W_STEM)),
           Entry("stem.pw_2", "stem/pw_2/kernel", -1, TRANSPOSE, (W_STEM, W_STEM)),
           Entry("stem.out", "stem/out/kernel", -1, TRANSPOSE, (D, 10 * W_STEM))]
    es += [Entry("audio.mel_filters", "", -1, DERIVED, (W_BINS, W_MELS)), Entry("tokenizer", "", -1, DERIVED, None)]
    return es


# The CQ-coded records of whistle.cact: the 4-bit token embedding and mHC
# heads, 2-bit projections, engram tables and stem kernels. Everything else
# is FP16 but the four derived FP32 records and the RAW tokenizer.
_CQ2_SUFFIXES = ("q_proj", "k_proj", "v_proj", "gate_proj", "out_proj", "pw1", "pw2", "tables", "key_proj",
                 "value_proj")
_FP32_NAMES = ("hada_p1", "hada_p2", "audio.manifest", "audio.mel_filters")


def whistle_storage(name: str) -> tuple[int, int]:
    """(dtype, CQ bits) of a whistle.cact record by name."""
    if name == "tokenizer":
        return RAW, 0
    if name in _FP32_NAMES:
        return FP32, 0
    if name == "embedding" or ".mhc_phi_" in "." + name:
        return CQ, 4
    last = name.rsplit(".", 1)[-1]
    if last in _CQ2_SUFFIXES or name in ("stem.pw_1", "stem.pw_2", "stem.out"):
        return CQ, 2
    return FP16, 0
