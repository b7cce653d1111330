"""The .cact container (go-whistle_b200/cact.py) against internal/cact's
tests: the layout constants, the header and directory checks with their
error texts (cact_test.go TestParse_*), the readers, the LSB-first unpack,
the FWHT and hand-computed CQ dequantisations (cq_test.go), the packed
form (packed_test.go), the Whistle tensor map against the reference's
golden testdata/whistle_names.txt, and a synthetic whistle.cact whose
record census is the exported file's (whistle_test.go:97-101)."""

from __future__ import annotations

import math
import struct
from collections import Counter
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden" / "whistle_names.txt"

# Record field offsets (format.go:125 Record, "<BBHIIIIQQII").
R_DTYPE, R_NDIM, R_PAD, R_SHAPE, R_OFFSET, R_NBYTES, R_GROUP, R_BITS = 0, 1, 2, 4, 20, 28, 36, 40


@pytest.fixture(scope="module")
def ct(wb):
    return wb.cact


def small_header(ct):
    return ct.Header(KVBits=8, Vocab=16, DModel=8, NumHeads=2, NumKVHeads=1, NumLayers=3, QKHeadDim=4, VHeadDim=4,
                     MaxSeqLen=32, HadaN=8, MHCLanes=4, GlobalMaskLo=0b101, QKVConvTaps=3, EngramSlots=64,
                     EngramSubDim=2, NumEngramTables=4, EngramConvTaps=4, EngramConvDilation=3, NumEngramOrders=2,
                     EngramOrders=(2, 3, 0, 0), NumEngramSites=1, EngramSites=(1,) + (0,) * 15, RopeTheta=10000.0)


def small_codebook():
    return np.arange(28, dtype=np.float32) - 14


def small_tensors(ct):
    """Every dtype: FP32 (2, 3), FP16 (3), an FP16 scalar, CQ2 (2, 200) of
    group 128 (padded to 256), ternary CQ (1, 128) and RAW."""
    f16 = np.array([0x3C00, 0xC000, 0x3800], "<u2").tobytes()
    return [ct.Tensor(ct.FP32, (2, 3), np.array([1, 2, 3, 4, 5, -6], "<f4").tobytes()),
            ct.Tensor(ct.FP16, (3,), f16),
            ct.Tensor(ct.FP16, (), np.array([0x4400], "<u2").tobytes()),
            ct.Tensor(ct.CQ, (2, 200), bytes(2 * 256 * 2 // 8 + 2 * 2 * 2), 128, 2),
            ct.Tensor(ct.CQ, (1, 128), bytes(128 * 2 // 8 + 2), 128, 5),
            ct.Tensor(ct.RAW, (), b"tokenizer")]


def small_file(ct):
    return ct.encode(small_header(ct), small_codebook(), small_tensors(ct))


def rec_at(ct, i):
    return ct.HEADER_SIZE + 4 * ct.CODEBOOK_LEN + ct.RECORD_SIZE * i


def test_layout_sizes(ct):
    assert len(ct.Header().pack()) == ct.HEADER_SIZE == 196
    assert len(ct.Record().pack()) == ct.RECORD_SIZE == 44


def test_parse_header(ct):
    f = ct.Parse(small_file(ct))
    want = small_header(ct)
    want.NumTensors, want.CodebookLen = 6, 28
    assert f.Header() == want
    assert f.Len() == 6
    assert f.Header().GlobalLayers() == [0, 2]
    assert f.Header().Orders() == [2, 3]
    assert f.Header().Sites() == [1]
    h = ct.Header(NumLayers=40, GlobalMaskLo=1 << 31, GlobalMaskHi=1 << 3)
    assert h.GlobalLayers() == [31, 35]


def test_codebook(ct):
    f = ct.Parse(small_file(ct))
    cb = small_codebook()
    for bits, lo, hi in ((2, 0, 4), (3, 4, 12), (4, 12, 28)):
        got = f.Codebook(bits)
        assert np.array_equal(got, cb[lo:hi])
        got[0] = 99  # a copy, not the file's own
        assert f.Codebook(bits)[0] == cb[lo]
    for bits in (1, 5, 0):
        with pytest.raises(ct.CactError, match=f"no stored codebook for {bits}-bit CQ"):
            f.Codebook(bits)


def test_records(ct):
    f = ct.Parse(small_file(ct))
    r = f.Record(3)
    assert (r.DType, r.Dims(), r.Group, r.Bits) == (ct.CQ, [2, 200], 128, 2)
    assert r.Offset % ct.ALIGN == 0 and r.Numel() == 400
    s = f.Record(2)
    assert s.Dims() == [] and s.Numel() == 1
    for i in (-1, 6):
        with pytest.raises(ct.CactError, match="out of range"):
            f.Record(i)


def test_readers(ct):
    f = ct.Parse(small_file(ct))
    assert f.FP32(0).tolist() == [1, 2, 3, 4, 5, -6]
    assert f.FP16(1).tolist() == [1, -2, 0.5]
    assert f.FP16(2).tolist() == [4]
    assert f.Float32(0).tolist() == [1, 2, 3, 4, 5, -6] and f.Float32(1).tolist() == [1, -2, 0.5]
    assert f.Raw(5) == b"tokenizer"
    wrong = {"FP32(FP16)": lambda: f.FP32(1), "FP16(FP32)": lambda: f.FP16(0), "Float32(CQ)": lambda: f.Float32(3),
             "Float32(RAW)": lambda: f.Float32(5), "Raw(FP32)": lambda: f.Raw(0)}
    for name, call in wrong.items():
        with pytest.raises(ct.DTypeError, match="wrong dtype"):
            call()
    with pytest.raises(ct.CactError, match="out of range"):
        f.FP32(99)


def _put32(b, at, v):
    b[at:at + 4] = struct.pack("<I", v)


def _put64(b, at, v):
    b[at:at + 8] = struct.pack("<Q", v)


def _off(b, i, ct):
    return struct.unpack_from("<Q", b, rec_at(ct, i) + R_OFFSET)[0]


# cact_test.go:322 TestParse_Errors: a mutation of the small file and a word
# the error must mention.
def _error_cases(ct):
    R = lambda i: rec_at(ct, i)  # noqa: E731

    def raw_ndim(b):
        b[R(5) + R_NDIM] = 1
        _put32(b, R(5) + R_SHAPE, 9)

    def cq_ndim(b):
        b[R(3) + R_NDIM] = 3
        _put32(b, R(3) + R_SHAPE + 8, 1)

    def overflow(b):
        b[R(0) + R_NDIM] = 4
        for k in range(4):
            _put32(b, R(0) + R_SHAPE + 4 * k, 0xFFFFFFFF)

    return [
        ("short header", lambda b: b.__delitem__(slice(ct.HEADER_SIZE - 1, None)), "header"),
        ("bad tag", lambda b: _put32(b, 0, 0xDEADBEEF), "tag"),
        ("codebook length", lambda b: _put32(b, 8, 27), "codebook"),
        ("too many orders", lambda b: _put32(b, 4 * 26, 5), "orders"),
        ("too many sites", lambda b: _put32(b, 4 * 31, 17), "sites"),
        ("directory past EOF", lambda b: _put32(b, 4, 1000), "directory"),
        ("directory size wraps uint32", lambda b: _put32(b, 4, 97612894), "directory"),
        ("unknown dtype", lambda b: b.__setitem__(R(0) + R_DTYPE, 9), "dtype 9"),
        ("ndim > 4", lambda b: b.__setitem__(R(0) + R_NDIM, 5), "ndim"),
        ("dim past ndim", lambda b: _put32(b, R(1) + R_SHAPE + 4, 7), "past ndim"),
        ("pad", lambda b: b.__setitem__(R(0) + R_PAD, 1), "pad"),
        ("misaligned", lambda b: _put64(b, R(0) + R_OFFSET, _off(b, 0, ct) + 4), "aligned"),
        ("inside directory", lambda b: _put64(b, R(0) + R_OFFSET, 0), "overlaps"),
        ("overlap", lambda b: _put64(b, R(1) + R_OFFSET, _off(b, 0, ct)), "overlaps"),
        ("blob past EOF", lambda b: b.__delitem__(slice(len(b) - 1, None)), "past EOF"),
        ("FP32 nbytes", lambda b: _put32(b, R(0) + R_SHAPE, 3), "nbytes"),
        ("FP16 nbytes", lambda b: _put64(b, R(1) + R_NBYTES, 4), "nbytes"),
        ("RAW ndim", raw_ndim, "RAW"),
        ("CQ ndim", cq_ndim, "CQ"),
        ("CQ group 0", lambda b: _put32(b, R(3) + R_GROUP, 0), "group"),
        ("CQ group not /8", lambda b: _put32(b, R(3) + R_GROUP, 100), "group"),
        ("CQ bits 6", lambda b: _put32(b, R(3) + R_BITS, 6), "bits"),
        ("CQ nbytes", lambda b: _put32(b, R(3) + R_BITS, 4), "nbytes"),
        ("numel overflow", overflow, "overflow"),
    ]


def test_parse_errors(ct):
    for name, mutate, want in _error_cases(ct):
        b = bytearray(small_file(ct))
        mutate(b)
        with pytest.raises(ct.CactError) as e:
            ct.Parse(bytes(b))
        assert want in str(e.value), (name, str(e.value))
        assert str(e.value).startswith("cact: "), name


def test_parse_error_texts(ct):
    """The reference's messages word for word (cact.go:99-149)."""
    b = bytearray(small_file(ct))
    _put32(b, 0, 0xDEADBEEF)
    with pytest.raises(ct.CactError, match=r"^cact: bad tag 0xdeadbeef, want 0x05e12a84$"):
        ct.Parse(bytes(b))
    b = bytearray(small_file(ct))
    _put32(b, rec_at(ct, 1) + R_SHAPE + 4, 7)
    with pytest.raises(ct.CactError, match=r"^cact: tensor 1 \(FP16\): shape \[3 7 0 0\] has a dimension past ndim 1$"):
        ct.Parse(bytes(b))
    b = bytearray(small_file(ct))
    _put32(b, rec_at(ct, 3) + R_BITS, 4)
    with pytest.raises(ct.CactError, match=r"^cact: tensor 3 \(CQ\): nbytes 136, want 264 for shape \[2 200\]$"):
        ct.Parse(bytes(b))


def test_parse_empty_and_missing(ct, tmp_path):
    f = ct.Parse(ct.encode(small_header(ct), small_codebook(), []))
    assert f.Len() == 0
    with pytest.raises(ct.CactError):
        ct.Open(str(tmp_path / "nope.cact"))


def test_dtype_and_transform_names(ct):
    for d, want in {ct.FP16: "FP16", ct.FP32: "FP32", ct.CQ: "CQ", ct.RAW: "RAW", 7: "dtype 7"}.items():
        assert ct.dtype_name(d) == want
    for t, want in {ct.DERIVED: "derived", ct.RESHAPE: "reshape", ct.TRANSPOSE: "transpose",
                    ct.LANE_MAJOR: "lane-major", 9: "transform 9"}.items():
        assert ct.transform_name(t) == want


# cq_test.go:298 TestUnpackLSB.
UNPACK = [(1, [0xA5], [1, 0, 1, 0, 0, 1, 0, 1]),
          (2, [0xE4, 0x1B], [0, 1, 2, 3, 3, 2, 1, 0]),
          (3, [0x88, 0xC6, 0xFA], [0, 1, 2, 3, 4, 5, 6, 7]),
          (3, [0xFF, 0xFF, 0xFF, 0x40, 0x00, 0x00], [7] * 8 + [0, 0, 1, 0, 0, 0, 0, 0]),
          (4, [0x21, 0x43, 0x65, 0xF7], [1, 2, 3, 4, 5, 6, 7, 15])]


@pytest.mark.parametrize("width,packed,want", UNPACK)
def test_unpack_lsb(ct, width, packed, want):
    got = ct.unpack_lsb(np.array([packed], np.uint8), width, len(want))
    assert got[0].tolist() == want
    assert ct.pack_lsb(np.array([want], np.uint8), width)[0].tolist() == packed


def test_unpack_round_trip(ct):
    rng = np.random.default_rng(12)
    for width in (1, 2, 3, 4):
        idx = rng.integers(0, 1 << width, size=(5, 24), dtype=np.uint8)
        assert np.array_equal(ct.unpack_lsb(ct.pack_lsb(idx, width), width, 24), idx)


def sylvester(n):
    h = np.ones((1, 1))
    while h.shape[0] < n:
        h = np.block([[h, h], [h, -h]])
    return h


def test_fwht(ct):
    rng = np.random.default_rng(3)
    for n in (1, 2, 8, 128):
        x = rng.integers(-8, 9, size=(3, n)).astype(np.float32)  # small integers: every sum exact
        assert np.array_equal(ct.fwht_rows(x), x.astype(np.float64) @ sylvester(n))


def _cq_file(ct, width, blob, out=1, in_=8, group=8):
    from importlib import import_module

    cb = np.concatenate([import_module("go-whistle_b200").weights.lloyd_max_unit(b) / math.sqrt(group)
                         for b in (2, 3, 4)]).astype(np.float32)
    return ct.Parse(ct.encode(small_header(ct), cb, [ct.Tensor(ct.CQ, (out, in_), bytes(blob), group, width)])), cb


def test_cq_hand(ct):
    """cq_test.go:383 TestCQ_Hand: group 8, where H/sqrt(8) maps a constant
    group onto column 0 and a one-hot onto a ± row of Sylvester's H."""
    half, one = 0x3800, 0x3C00
    h8 = sylvester(8)
    tern = np.float32(1.2240064 / math.sqrt(8))
    binl = float(np.float32(math.sqrt(2 / math.pi) / math.sqrt(8)))

    def row(r, level):
        return float(level) * h8[r] / math.sqrt(8)

    f, cb = _cq_file(ct, 2, [0xFF, 0xFF, half & 0xFF, half >> 8])
    want = np.zeros(8)
    want[0] = 8 * float(cb[3]) * 0.5 / math.sqrt(8)
    assert np.allclose(f.CQ(0)[0], want, rtol=1e-6, atol=1e-6)
    for blob, r, sign in (([0x01, 0x00], 0, 1), ([0x0C, 0x00], 1, -1), ([0x10, 0x00], 2, 1), ([0x00, 0x04], 5, 1)):
        f, _ = _cq_file(ct, 5, blob + [one & 0xFF, one >> 8])
        assert np.allclose(f.CQ(0)[0], row(r, sign * tern), rtol=1e-6, atol=1e-6), r
    f, _ = _cq_file(ct, 1, [0x01, one & 0xFF, one >> 8])
    want = np.full(8, 2 * binl / math.sqrt(8))
    want[0] -= binl * math.sqrt(8)
    assert np.allclose(f.CQ(0)[0], want, rtol=1e-6, atol=1e-6)


def test_cq_bad_crumb(ct):
    f, _ = _cq_file(ct, 5, [0x02, 0x00, 0x00, 0x3C])
    with pytest.raises(ct.CactError, match="tensor 0: row 0: ternary crumb 2 at column 0 is not 0, 1 or 3"):
        f.CQ(0)


@pytest.mark.parametrize("out,in_,group", [(1, 8, 8), (3, 16, 8), (4, 13, 8), (2, 40, 32), (2, 200, 128),
                                           (3, 384, 128), (5, 129, 128)])
@pytest.mark.parametrize("width", [1, 2, 3, 4, 5])
def test_cq_matrix_reference(ct, out, in_, group, width):
    """cq_test.go:470: random indices and norms against the float64
    arithmetic (cb[idx]·norm) @ H/sqrt(group), cut to [out][in], within the
    float32 rounding bound."""
    rng = np.random.default_rng(out * 1000 + in_ + width)
    groups = (in_ + group - 1) // group
    w_bits = 2 if width == 5 else width
    levels = 3 if width == 5 else 1 << width
    idx = rng.integers(0, levels, size=(out, groups * group)).astype(np.uint8)
    stored = idx.copy()
    if width == 5:  # trits 0, 1, 2 are stored as crumbs 3, 0, 1
        stored = np.array([3, 0, 1], np.uint8)[idx]
    norms = rng.uniform(0.25, 2.0, size=(out, groups)).astype(np.float16)
    blob = ct.pack_lsb(stored, w_bits).tobytes() + norms.astype("<f2").tobytes()
    f, cb = _cq_file(ct, width, blob, out, in_, group)
    levels_used = f._levels(f.Record(0)).astype(np.float64)
    w = (levels_used[idx].reshape(out, groups, group) * norms.astype(np.float64)[:, :, None])
    want = (w @ sylvester(group) / math.sqrt(group)).reshape(out, -1)[:, :in_]
    got = f.CQ(0)
    gamma = (2 + math.log2(group)) * 2.0 ** -24 * 2
    bound = gamma * (np.abs(w).reshape(out, groups, group).sum(axis=2, keepdims=True) / math.sqrt(group))
    bound = np.broadcast_to(bound, (out, groups, group)).reshape(out, -1)[:, :in_]
    assert np.all(np.abs(got - want) <= bound + 1e-30)


def test_cq_packed(ct):
    """packed.go:45 CQPacked: the stored bytes and the codebook CQ uses."""
    rng = np.random.default_rng(9)
    idx = rng.integers(0, 4, size=(2, 256)).astype(np.uint8)
    norms = rng.uniform(0.5, 1.5, size=(2, 2)).astype(np.float16)
    blob = ct.pack_lsb(idx, 2).tobytes() + norms.astype("<f2").tobytes()
    f, cb = _cq_file(ct, 2, blob, 2, 200, 128)
    p = f.CQPacked(0)
    assert (p.Out, p.In, p.Group, p.Bits, p.Width) == (2, 200, 128, 2, 2)
    assert np.array_equal(p.Codebook, cb[:4])
    assert bytes(p.Index) == blob[:128] and bytes(p.Norms) == blob[128:]
    f, _ = _cq_file(ct, 2, bytes(2 * (48 * 2 // 8 + 2 * 2)), 2, 48, 24)
    with pytest.raises(ct.CactError, match="tensor 0: CQ group 24 is not a power of two"):
        f.CQPacked(0)


def _golden_entries():
    rows = []
    for ln in GOLDEN.read_text().splitlines():
        if not ln.strip() or ln.startswith("#"):
            continue
        i, name, shape, tr, src = ln.split()
        dims = tuple(int(d) for d in shape[1:-1].split(",") if d)
        rows.append((int(i), name, dims, tr, src))
    return rows


def test_whistle_names_golden(ct):
    """names.go:272 WhistleNames against the reference's golden
    testdata/whistle_names.txt: every index, name, shape, transform and
    source[layer]."""
    names = ct.whistle_names()
    golden = _golden_entries()
    assert len(names) == len(golden) == 681
    for e, (i, name, dims, tr, src) in zip(names, golden):
        assert e.Name == name, i
        assert (e.Shape or ()) == dims, name
        assert ct.transform_name(e.Transform) == tr, name
        want_src = "-" if e.Transform == ct.DERIVED else e.Source + (f"[{e.Layer}]" if e.Layer >= 0 else "")
        assert want_src == src, name


@pytest.fixture(scope="module")
def whistle_file(wb):
    w = wb.synth.DecoderWeights(seed=4400, vocab=8199)
    return w, wb.weights.write_whistle_cact(w, seed=3)


def test_synthetic_whistle_layout(ct, whistle_file):
    """A synthetic whistle.cact has the exported file's layout: the record
    census of whistle_test.go:97-101, the CQ4 embedding right after the
    directory, FP32 derived records, the manifest, no bytes past the last
    blob, group 128 throughout."""
    _, data = whistle_file
    f = ct.Parse(data)
    assert f.Len() == 681
    hist = Counter()
    for i in range(f.Len()):
        r = f.Record(i)
        hist[(ct.dtype_name(r.DType), r.Bits, r.NDim)] += 1
        if r.DType == ct.CQ:
            assert r.Group == 128, i
    assert hist == {("FP16", 0, 1): 289, ("FP16", 0, 2): 233, ("FP16", 0, 3): 2, ("FP32", 0, 1): 3,
                    ("FP32", 0, 2): 1, ("CQ", 2, 2): 145, ("CQ", 4, 2): 7, ("RAW", 0, 0): 1}
    first = f.Record(0)
    assert (first.DType, first.Bits, first.Dims()) == (ct.CQ, 4, [8199, 512])
    assert first.Offset == ct.HEADER_SIZE + 4 * ct.CODEBOOK_LEN + 681 * ct.RECORD_SIZE
    for i, dims in {226: [512], 227: [512], 237: [13], 679: [257, 80]}.items():
        r = f.Record(i)
        assert r.DType == ct.FP32 and r.Dims() == dims, i
    last = f.Record(680)
    assert last.Offset + last.NBytes == len(data)
    h = f.Header()
    assert (h.Vocab, h.DModel, h.NumHeads, h.NumKVHeads, h.NumLayers, h.QKHeadDim, h.VHeadDim, h.MHCLanes,
            h.QKVConvTaps, h.EngramSlots, h.EngramSubDim, h.NumEngramTables, h.EngramConvTaps,
            h.EngramConvDilation) == (8199, 512, 8, 2, 8, 48, 64, 4, 3, 18432, 128, 4, 4, 3)
    assert h.Orders() == [2, 3] and h.Sites() == [3, 7] and h.RopeTheta == 100000.0


def test_decoder_weights_round_trip(wb, whistle_file):
    """Loading the synthetic file gives back w: every CQ tensor byte for
    byte, every float tensor as its FP16 rounding, the geometry."""
    w, data = whistle_file
    src = wb.weights.Parse(data)
    got = wb.weights.decoder_weights(src)

    def same_cq(a, b):
        return ((a.Out, a.In, a.Group, a.Bits) == (b.Out, b.In, b.Group, b.Bits) and
                np.array_equal(np.asarray(a.Index, np.uint8), np.asarray(b.Index, np.uint8)) and
                np.array_equal(np.asarray(a.Norms, np.uint8), np.asarray(b.Norms, np.uint8)) and
                np.array_equal(np.asarray(a.Codebook, np.float32), np.asarray(b.Codebook, np.float32)))

    def f16(a):
        return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)

    for k in ("vocab", "dim", "lanes", "heads", "kv_heads", "qk", "vd", "taps", "x_heads", "x_qk", "x_vd", "na",
              "nb", "rank", "n_tables", "slots", "sub", "etaps", "max_order", "rope_len"):
        assert getattr(got, k) == getattr(w, k), k
    assert got.orders == w.orders and got.site_layers == w.site_layers and got.rope_theta == w.rope_theta
    assert same_cq(got.embedding, w.embedding)
    for k in ("phi_pre", "phi_post", "phi_res"):
        assert same_cq(getattr(got, k), getattr(w, k)), k
    assert np.array_equal(got.hada_p1, w.hada_p1) and np.array_equal(got.hada_p2, w.hada_p2)
    assert np.array_equal(got.final_norm, f16(w.final_norm))
    for l, (A, B) in enumerate(zip(got.layers, w.layers)):
        for k, v in B.items():
            if isinstance(v, float):
                assert A[k] == float(np.float16(v)), (l, k)
            elif hasattr(v, "Index"):
                assert same_cq(A[k], v), (l, k)
            else:
                assert np.array_equal(np.asarray(A[k]).reshape(-1), f16(v).reshape(-1)), (l, k)
    for A, B in zip(got.sites, w.sites):
        assert A["layer"] == B["layer"]
        for k in ("tables", "key_proj", "value_proj"):
            assert same_cq(A[k], B[k]), k
        assert np.array_equal(A["taps"], f16(B["taps"]))


def test_source_checks(wb, ct, whistle_file):
    _, data = whistle_file
    names = ct.whistle_names()
    with pytest.raises(wb.weights.WeightsError, match="680 names for 681 tensors"):
        wb.weights.Parse(data, names[:-1])
    bad = list(names)
    bad[1] = ct.Entry(bad[1].Name, bad[1].Source, 0, ct.RESHAPE, (511,))
    with pytest.raises(wb.weights.WeightsError, match=r"layer00.norm_in: record 1 is FP16 \[512\], the map says \[511\]"):
        wb.weights.Parse(data, bad)
    src = wb.weights.Parse(data)
    with pytest.raises(wb.weights.WeightsError, match="no tensor nope"):
        src.Tensor("nope")
    with pytest.raises(wb.weights.WeightsError, match="not CQ"):
        src.Matrix("final_norm")
    assert src.Shape("engram0.tables") == [73728, 128]
    cfg = src.Config()
    assert (cfg.Text, cfg.EncLayers, cfg.Mels, cfg.Rate, cfg.Hop) == (8192, 8, 80, 16000, 160)
    # A manifest with another magic is refused.
    f = ct.Parse(data)
    b = bytearray(data)
    b[f.Record(237).Offset:f.Record(237).Offset + 4] = np.float32(1234).tobytes()
    with pytest.raises(wb.weights.WeightsError, match="audio manifest magic 1234, want 3246"):
        wb.weights.Parse(bytes(b))


def test_dequantised_embedding_matches_rows(wb, ct, whistle_file):
    """File.CQ on the embedding against the float64 formula on a sample of
    rows: the stored bytes through H/sqrt(group)."""
    w, data = whistle_file
    f = ct.Parse(data)
    emb = f.CQ(0)
    p = w.embedding
    rows = [0, 1, 4097, 8198]
    idx = ct.unpack_lsb(np.asarray(p.Index, np.uint8).reshape(p.Out, -1)[rows], 4, 512)
    nrm = np.asarray(p.Norms, np.uint8).view("<f2").reshape(p.Out, -1)[rows].astype(np.float64)
    cb = np.asarray(p.Codebook, np.float64)
    want = ((cb[idx].reshape(4, 4, 128) * nrm[:, :, None]) @ sylvester(128) / math.sqrt(128)).reshape(4, -1)
    assert np.allclose(emb[rows], want, rtol=0, atol=1e-6 * np.abs(want).max())
