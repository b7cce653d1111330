"""CQ products on the GPU through the C ABI, bit for bit against the oracle's
restatement of the reference's lut and Exact kernels."""

from __future__ import annotations

import ctypes
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# internal/cq/cq_test.go:183 testShapes, Whistle's shapes (parallel_test.go:29)
# and the benchmark configurations' shapes: (out, in, group).
SHAPES = [(1, 8, 8), (3, 16, 8), (4, 13, 8), (5, 40, 32), (7, 200, 128), (6, 384, 128), (9, 129, 128),
          (33, 256, 128), (384, 512, 128), (96, 512, 128), (4133, 300, 64), (1031, 200, 32),
          (2048, 512, 32), (512, 512, 32), (512, 2048, 32), (128, 2048, 128)]


def bits_eq(a, b) -> bool:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def make(wb, orc, seed, out, in_, group, bits, codebook="reference"):
    rng = np.random.default_rng(seed)
    p = wb.synth.random_packed(rng, out, in_, group, bits, codebook)
    return rng, p, wb.cq.New(p), orc.OracleMatrix.of(p)


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{o}x{i}g{g}" for o, i, g in SHAPES])
@pytest.mark.parametrize("bits", [2, 4])
def test_gemm_lut_bit_exact(wb, orc, cuda, shape, bits):
    out, in_, group = shape
    rng, p, m, om = make(wb, orc, 100 + out + in_ + bits, out, in_, group, bits)
    for rows in (1, 3, 6):
        x = rng.normal(size=rows * in_).astype(np.float32)
        want = orc.gemm_lut(om, x, rows).reshape(-1)
        got = np.zeros(rows * out, np.float32)
        m.GEMM(got, x, rows)
        assert bits_eq(got, want), rows
        xd = cuda.from_numpy(x).cuda()
        yd = cuda.empty(rows * out, dtype=cuda.float32, device="cuda")
        m.GEMM(yd, xd, rows)
        assert bits_eq(yd.cpu().numpy(), want), rows


@pytest.mark.parametrize("bits", [2, 4])
def test_gemm_many_activations(wb, orc, cuda, bits):
    """A prefill-sized batch (375 frames) and a batch past one grid's 65535
    activations."""
    rng, p, m, om = make(wb, orc, 7, 384, 512, 128, bits, "lloyd")
    x = rng.normal(size=375 * 512).astype(np.float32)
    got = np.zeros(375 * 384, np.float32)
    m.GEMM(got, x, 375)
    assert bits_eq(got, orc.gemm_lut(om, x, 375, threads=8).reshape(-1))
    rng, p, m, om = make(wb, orc, 8, 5, 32, 32, bits)
    rows = 70000
    x = rng.normal(size=rows * 32).astype(np.float32)
    got = np.zeros(rows * 5, np.float32)
    m.GEMM(got, x, rows)
    assert bits_eq(got, orc.gemm_lut(om, x, rows, threads=8).reshape(-1))


@pytest.mark.parametrize("bits", [2, 4])
def test_rows_views(wb, orc, cuda, bits):
    """cq_test.go:335 TestRow (views part) and asm_test.go:171: views that
    start and end inside a block equal the full product's rows."""
    for out, in_, group in ((70, 384, 128), (45, 2048, 128), (33, 40, 8)):
        rng, p, m, om = make(wb, orc, out, out, in_, group, bits)
        x = rng.normal(size=3 * in_).astype(np.float32)
        full = orc.gemm_lut(om, x, 3)
        for lo, hi in ((0, out), (5, out - 7), (out // 3, out - out // 5), (out - 1, out)):
            v = m.Rows(lo, hi)
            assert v.Out() == hi - lo and v.In() == in_ and v.Bits() == bits
            got = np.zeros(3 * (hi - lo), np.float32)
            v.GEMM(got, x, 3)
            assert bits_eq(got.reshape(3, -1), full[:, lo:hi]), (lo, hi)
            vv = v.Rows(1, hi - lo) if hi - lo > 1 else v
            got2 = np.zeros(3 * vv.Out(), np.float32)
            vv.GEMM(got2, x, 3)
            off = 1 if hi - lo > 1 else 0
            assert bits_eq(got2.reshape(3, -1), full[:, lo + off:hi])


def test_gemms_shared_and_mixed(wb, orc, cuda):
    """parallel_test.go:101 TestGEMMsMatchesGEMM: q/k/v/gate sharing tables,
    a matrix with another codebook, an Exact view and an empty view."""
    rng = np.random.default_rng(382)
    ps = [wb.synth.random_packed(rng, o, 512, 128, 2, "lloyd") for o in (384, 96, 128, 512)]
    other = wb.synth.random_packed(rng, 64, 512, 128, 2, "reference")
    ms = [wb.cq.New(p) for p in ps] + [wb.cq.New(other)]
    ms.append(ms[0].Exact().Rows(3, 40))
    ms.append(ms[1].Rows(5, 5))
    oms = [orc.OracleMatrix.of(p) for p in ps] + [orc.OracleMatrix.of(other)]
    for rows in (1, 3, 8):
        x = rng.normal(size=rows * 512).astype(np.float32)
        dsts = [np.zeros(rows * m.Out(), np.float32) for m in ms]
        wb.cq.GEMMs(ms, dsts, x, rows)
        for k, om in enumerate(oms):
            assert bits_eq(dsts[k], orc.gemm_lut(om, x, rows).reshape(-1)), k
        assert bits_eq(dsts[5].reshape(rows, -1), orc.gemm_exact(oms[0], x, rows)[:, 3:40])
        assert dsts[6].size == 0
        # device form: one launch for the shared set
        xd = cuda.from_numpy(x).cuda()
        yds = [cuda.empty(rows * m.Out(), dtype=cuda.float32, device="cuda") for m in ms]
        wb.cq.GEMMs(ms, yds, xd, rows)
        for k in range(len(ms)):
            assert bits_eq(yds[k].cpu().numpy(), dsts[k]), k


@pytest.mark.parametrize("bits", [2, 4])
def test_exact_bit_exact(wb, orc, cuda, bits):
    """cq_test.go:516 TestExact: an Exact view runs the nibble4/nibble float
    kernels, the reference's purego bits."""
    for out, in_, group in ((70, 384, 128), (5, 40, 32), (4, 13, 8), (31, 512, 32)):
        rng, p, m, om = make(wb, orc, 19 + out, out, in_, group, bits)
        e = m.Exact()
        for rows in (1, 3, 4, 5, 6, 9):
            x = rng.normal(size=rows * in_).astype(np.float32)
            got = np.zeros(rows * out, np.float32)
            e.GEMM(got, x, rows)
            assert bits_eq(got, orc.gemm_exact(om, x, rows).reshape(-1)), (out, rows)
        v = e.Rows(1, out)
        x = rng.normal(size=5 * in_).astype(np.float32)
        got = np.zeros(5 * (out - 1), np.float32)
        v.GEMM(got, x, 5)
        assert bits_eq(got.reshape(5, -1), orc.gemm_exact(om, x, 5)[:, 1:])


@pytest.mark.parametrize("bits", [2, 4])
def test_row_bit_exact(wb, orc, cuda, bits):
    """matrix.go:161 Row equals cact.CQ's dequantisation bit for bit."""
    for out, in_, group in ((7, 200, 128), (9, 129, 128), (4, 13, 8), (64, 512, 32)):
        rng, p, m, om = make(wb, orc, 5 + out, out, in_, group, bits)
        for r in range(out):
            got = np.zeros(in_, np.float32)
            m.Row(got, r)
            assert bits_eq(got, orc.row(om, r)), r
        v = m.Rows(1, out)
        got = np.zeros(in_, np.float32)
        v.Row(got, 0)
        assert bits_eq(got, orc.row(om, 1))
        # batched gather with an out-of-range row
        import ctypes

        rows = np.array([0, out - 1, out, 2 % out], np.int32)
        rd = cuda.from_numpy(rows).cuda()
        dst = cuda.full((4, in_), 7.0, dtype=cuda.float32, device="cuda")
        bad = cuda.zeros(1, dtype=cuda.int32, device="cuda")
        wb._lib.check(wb._lib.lib().wc_cq_row_gather(m.handle, ctypes.c_void_p(rd.data_ptr()), 4,
                                                     ctypes.c_void_p(dst.data_ptr()),
                                                     ctypes.c_void_p(bad.data_ptr()), None))
        d = dst.cpu().numpy()
        assert bits_eq(d[0], orc.row(om, 0)) and bits_eq(d[1], orc.row(om, out - 1))
        assert np.all(d[2] == 0) and bits_eq(d[3], orc.row(om, 2 % out)) and int(bad.item()) == 1


def test_no_rows(wb, orc, cuda):
    """cq_test.go:304 TestGEMMNoRows: Out 0 and empty views are no-ops."""
    rng = np.random.default_rng(5)
    empty = wb.cq.New(wb.synth.random_packed(rng, 0, 256, 128, 2))
    m = wb.cq.New(wb.synth.random_packed(rng, 64, 256, 128, 4))
    x = rng.normal(size=2 * 256).astype(np.float32)
    for v in (empty, m.Rows(32, 32), m.Rows(5, 5)):
        v.GEMM(np.zeros(0, np.float32), x, 2)
        v.GEMV(np.zeros(0, np.float32), x[:256])
        v.Exact().GEMM(np.zeros(0, np.float32), x, 2)
    m.GEMM(np.zeros(0, np.float32), np.zeros(0, np.float32), 0)


def test_gemm_panics(wb, cuda):
    """cq_test.go:587 TestGEMMPanics, with the reference's panic texts."""
    m = wb.cq.New(wb.synth.random_packed(np.random.default_rng(9), 4, 128, 128, 4))
    cases = {
        "short x": lambda: m.GEMV(np.zeros(4, np.float32), np.zeros(127, np.float32)),
        "short dst": lambda: m.GEMV(np.zeros(3, np.float32), np.zeros(128, np.float32)),
        "rows": lambda: m.GEMM(np.zeros(8, np.float32), np.zeros(128, np.float32), 2),
        "row": lambda: m.Row(np.zeros(128, np.float32), 4),
        "view": lambda: m.Rows(3, 5),
    }
    for name, f in cases.items():
        with pytest.raises(wb.Panic):
            f()
    with pytest.raises(wb.Panic, match=r"^cq: GEMM\(len 4, len 127, 1 rows\) on \[4, 128\]$"):
        m.GEMV(np.zeros(4, np.float32), np.zeros(127, np.float32))
    with pytest.raises(wb.Panic, match=r"^cq: Rows\(3, 5\) of 4 rows$"):
        m.Rows(3, 5)


def test_concurrent(wb, orc, cuda):
    """cq_test.go:393 TestGEMMConcurrent: threads on their own streams, views
    of one matrix, every result the serial one's bits."""
    rng, p, m, om = make(wb, orc, 15, 70, 384, 128, 4)
    x = rng.normal(size=3 * 384).astype(np.float32)
    views = [(0, 70), (5, 40), (33, 70), (64, 66)]
    full = orc.gemm_lut(om, x, 3)
    errors = []

    def work(g):
        s = cuda.cuda.Stream()
        with cuda.cuda.stream(s):
            xd = cuda.from_numpy(x).cuda()
            for n in range(20):
                lo, hi = views[(g + n) % len(views)]
                yd = cuda.empty(3 * (hi - lo), dtype=cuda.float32, device="cuda")
                m.Rows(lo, hi).GEMM(yd, xd, 3)
                s.synchronize()
                if not bits_eq(yd.cpu().numpy().reshape(3, -1), full[:, lo:hi]):
                    errors.append((g, n))

    ts = [threading.Thread(target=work, args=(g,)) for g in range(8)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errors


def test_bytes(wb, cuda):
    rng = np.random.default_rng(1)
    p = wb.synth.random_packed(rng, 70, 384, 128, 2)
    m = wb.cq.New(p)
    assert m.Bytes() == p.Index.size + p.Norms.size + 4 * 4


# Products large enough (>= 2 MB of index bytes per activation) for the
# streaming kernel: every group width it takes (gb 8, 16, 32, 64), one and
# several table passes (rows of 256 and 1024 index bytes), and GEMMs over
# views that start inside a 32-row tile.
STREAM_CASES = [(16384, 512, 32, 4), (8199, 512, 128, 4), (16384, 512, 32, 2), (8192, 2048, 32, 4),
                (8192, 2048, 32, 2), (20000, 512, 128, 2), (4096, 2048, 128, 4), (16384, 512, 16, 4),
                (16384, 512, 64, 2)]


@pytest.mark.parametrize("case", STREAM_CASES, ids=[f"{o}x{i}g{g}b{b}" for o, i, g, b in STREAM_CASES])
def test_stream_kernel_bit_exact(wb, orc, cuda, case):
    out, in_, group, bits = case
    rng, p, m, om = make(wb, orc, out + in_ + group + bits, out, in_, group, bits, "lloyd")
    x = rng.normal(size=in_).astype(np.float32)
    x[group:2 * group] = 0.0  # a group whose bound M is 0 (lut.go:219: 8191/M taken as 0)
    want = orc.gemm_lut(om, x, 1, threads=8).reshape(-1)
    xd = cuda.from_numpy(x).cuda()
    yd = cuda.full((out,), float("nan"), dtype=cuda.float32, device="cuda")
    m.GEMV(yd, xd)
    assert bits_eq(yd.cpu().numpy(), want)
    # GEMMs over views of the same matrix, unaligned starts, > 1 launch of views
    bounds = [(0, 1000), (5, 1200), (33, 2500), (1000, 1001), (out - 700, out)]
    views = [m.Rows(lo, hi) for lo, hi in bounds] * 3
    yds = [cuda.full((v.Out(),), float("nan"), dtype=cuda.float32, device="cuda") for v in views]
    wb.cq.GEMMs(views, yds, xd, 1)
    for (lo, hi), y in zip(bounds * 3, yds):
        assert bits_eq(y.cpu().numpy(), want[lo:hi]), (lo, hi)


def test_stream_many_matrices(wb, orc, cuda):
    """More matrices than one launch carries, each its own weights."""
    rng = np.random.default_rng(77)
    ps = [wb.synth.random_packed(rng, 96, 512, 32, 4, "lloyd") for _ in range(600)]
    for p in ps[1:]:
        p.Codebook = ps[0].Codebook
    ms = [wb.cq.New(p) for p in ps]
    x = rng.normal(size=512).astype(np.float32)
    xd = cuda.from_numpy(x).cuda()
    yds = [cuda.empty(96, dtype=cuda.float32, device="cuda") for _ in ms]
    wb.cq.GEMMs(ms, yds, xd, 1)
    for p, y in zip(ps[::37], yds[::37]):
        want = orc.gemm_lut(orc.OracleMatrix.of(p), x, 1).reshape(-1)
        assert bits_eq(y.cpu().numpy(), want)


@pytest.mark.parametrize("rows,view_rows", [(1, 16384), (3, 4096)])
def test_gemms_host_chunked(wb, orc, cuda, rows, view_rows):
    """GEMMs on host slices with outputs large enough to split into chunks
    (3 and 4 MiB: the kernels of one chunk overlap the copy of the previous
    one), outputs in one contiguous host array and in separate arrays: bit
    for bit the device call's and the oracle's."""
    rng = np.random.default_rng(90 + rows)
    n = 64
    base = wb.synth.random_packed(rng, n * view_rows, 512, 32, 2, "lloyd")
    big = wb.cq.New(base)
    views = [big.Rows(k * view_rows, (k + 1) * view_rows) for k in range(n)]
    x = rng.normal(size=rows * 512).astype(np.float32)
    flat = np.full((n, rows * view_rows), np.nan, np.float32)
    wb.cq.GEMMs(views, [flat[k] for k in range(n)], x, rows)
    sep = [np.full(rows * view_rows, np.nan, np.float32) for _ in range(n)]
    wb.cq.GEMMs(views, sep, x, rows)
    xd = cuda.from_numpy(x).cuda()
    yds = [cuda.empty(rows * view_rows, dtype=cuda.float32, device="cuda") for _ in views]
    wb.cq.GEMMs(views, yds, xd, rows)
    for k in range(n):
        dev = yds[k].cpu().numpy()
        assert bits_eq(flat[k], dev) and bits_eq(sep[k], dev), k
    want = orc.gemm_lut(orc.OracleMatrix.of(base), x, rows, threads=8).reshape(rows, n, view_rows)
    for k in (0, 17, n - 1):
        assert bits_eq(flat[k].reshape(rows, view_rows), want[:, k])


@pytest.mark.parametrize("in_,bits,rows,view_rows", [(512, 4, 1, 384), (2048, 4, 1, 96), (512, 2, 1, 16),
                                                     (1024, 4, 3, 96)])
def test_gemms_host_direct(wb, orc, cuda, in_, bits, rows, view_rows):
    """GEMMs and GEMM on host slices in page-locked memory: the kernels store
    the results there directly (the streaming kernel with one table pass,
    and with four, its partial sums kept on the device; the small-product
    kernels; several activations). Bit for bit the pageable-memory call's,
    the device call's and the oracle's; a list mixing page-locked and
    pageable outputs also matches."""
    rng = np.random.default_rng(700 + in_ + bits + rows)
    n = 64
    base = wb.synth.random_packed(rng, n * view_rows, in_, 32, bits, "lloyd")
    big = wb.cq.New(base)
    views = [big.Rows(k * view_rows, (k + 1) * view_rows) for k in range(n)]
    x = rng.normal(size=rows * in_).astype(np.float32)
    pinned = cuda.full((n, rows * view_rows), float("nan"), dtype=cuda.float32).pin_memory().numpy()
    wb.cq.GEMMs(views, [pinned[k] for k in range(n)], x, rows)
    sep = [cuda.full((rows * view_rows,), float("nan"), dtype=cuda.float32).pin_memory().numpy() for _ in range(n)]
    wb.cq.GEMMs(views, sep, x, rows)
    pageable = np.full((n, rows * view_rows), np.nan, np.float32)
    wb.cq.GEMMs(views, [pageable[k] for k in range(n)], x, rows)
    mixed = [sep[k] if k % 2 else pageable[k] for k in range(n)]
    for a in mixed:
        a[:] = np.nan
    wb.cq.GEMMs(views, mixed, x, rows)
    yds = [cuda.empty(rows * view_rows, dtype=cuda.float32, device="cuda") for _ in views]
    wb.cq.GEMMs(views, yds, cuda.from_numpy(x).cuda(), rows)
    for k in range(n):
        dev = yds[k].cpu().numpy()
        assert bits_eq(pinned[k], dev) and bits_eq(sep[k], dev) and bits_eq(pageable[k], dev), k
        assert bits_eq(mixed[k], dev), k
    one = cuda.full((rows * view_rows,), float("nan"), dtype=cuda.float32).pin_memory().numpy()
    views[5].GEMM(one, x, rows)
    assert bits_eq(one, yds[5].cpu().numpy())
    want = orc.gemm_lut(orc.OracleMatrix.of(base), x, rows, threads=8).reshape(rows, n, view_rows)
    for k in (0, 17, n - 1):
        assert bits_eq(pinned[k].reshape(rows, view_rows), want[:, k])


def test_gemms_host_direct_mixed(wb, orc, cuda):
    """Page-locked host outputs for a list that mixes shared-table matrices,
    another codebook, an Exact view and an empty view (kernel.go:134's
    GEMMs cases): every kernel stores into host memory directly, the empty
    output stays untouched; bit for bit the oracle's."""
    rng = np.random.default_rng(383)
    ps = [wb.synth.random_packed(rng, o, 512, 128, 2, "lloyd") for o in (384, 96, 128, 512)]
    other = wb.synth.random_packed(rng, 64, 512, 128, 2, "reference")
    ms = [wb.cq.New(p) for p in ps] + [wb.cq.New(other)]
    ms.append(ms[0].Exact().Rows(3, 40))
    ms.append(ms[1].Rows(5, 5))
    oms = [orc.OracleMatrix.of(p) for p in ps] + [orc.OracleMatrix.of(other)]
    for rows in (1, 3):
        x = rng.normal(size=rows * 512).astype(np.float32)
        total = sum(rows * m.Out() for m in ms)
        flat = cuda.full((total,), float("nan"), dtype=cuda.float32).pin_memory().numpy()
        dsts, off = [], 0
        for m in ms:
            dsts.append(flat[off:off + rows * m.Out()])
            off += rows * m.Out()
        wb.cq.GEMMs(ms, dsts, x, rows)
        for k, om in enumerate(oms):
            assert bits_eq(dsts[k], orc.gemm_lut(om, x, rows).reshape(-1)), k
        assert bits_eq(dsts[5].reshape(rows, -1), orc.gemm_exact(oms[0], x, rows)[:, 3:40])
        assert dsts[6].size == 0


def test_gemms_host_large_pinned(wb, cuda):
    """Host GEMMs whose page-locked outputs exceed the direct-store limit
    (34 MB): the products go to device memory in chunks and come back by
    copies; bit for bit the device call's."""
    rng = np.random.default_rng(808)
    n, view_rows, rows = 64, 96, 1400
    big = wb.cq.New(wb.synth.random_packed(rng, n * view_rows, 512, 32, 4, "lloyd"))
    views = [big.Rows(k * view_rows, (k + 1) * view_rows) for k in range(n)]
    x = rng.normal(size=rows * 512).astype(np.float32)
    pinned = cuda.full((n, rows * view_rows), float("nan"), dtype=cuda.float32).pin_memory().numpy()
    assert pinned.nbytes > 32 << 20
    wb.cq.GEMMs(views, [pinned[k] for k in range(n)], x, rows)
    yds = [cuda.empty(rows * view_rows, dtype=cuda.float32, device="cuda") for _ in views]
    wb.cq.GEMMs(views, yds, cuda.from_numpy(x).cuda(), rows)
    for k in range(n):
        assert bits_eq(pinned[k], yds[k].cpu().numpy()), k


def test_stream_runs(wb, orc, cuda):
    """GEMMs calls the streaming kernel carries as strided runs: a stack of
    views with a constant row step and contiguous outputs, one matrix
    repeated into evenly spaced outputs with gaps, steps that change (new
    runs), and more distinct runs than one launch holds. Bit for bit the
    oracle's products."""
    rng = np.random.default_rng(123)
    base = wb.synth.random_packed(rng, 64 * 160, 512, 32, 4, "lloyd")
    big = wb.cq.New(base)
    want = orc.gemm_lut(orc.OracleMatrix.of(base), (x := rng.normal(size=512).astype(np.float32)), 1, threads=8)
    want = want.reshape(-1)
    xd = cuda.from_numpy(x).cuda()
    lib = wb._lib.lib()

    def gemms(views, out_ptrs):
        hs = (ctypes.c_void_p * len(views))(*[v.handle.value for v in views])
        ys = (ctypes.c_void_p * len(views))(*out_ptrs)
        wb._lib.check(lib.wc_cq_gemms(hs, len(views), ctypes.c_void_p(xd.data_ptr()), ys, 1, None))
        cuda.cuda.synchronize()

    # a stack: 64 views of 160 rows, outputs back to back (one run)
    views = [big.Rows(160 * k, 160 * (k + 1)) for k in range(64)]
    y = cuda.full((64 * 160,), float("nan"), dtype=cuda.float32, device="cuda")
    gemms(views, [y.data_ptr() + 4 * 160 * k for k in range(64)])
    assert bits_eq(y.cpu().numpy(), want)
    # one view repeated 60 times into outputs 200 floats apart (row step 0)
    y2 = cuda.full((60 * 200,), float("nan"), dtype=cuda.float32, device="cuda")
    v = views[5]
    gemms([v] * 60, [y2.data_ptr() + 4 * 200 * k for k in range(60)])
    got = y2.cpu().numpy().reshape(60, 200)
    for k in range(60):
        assert bits_eq(got[k, :160], want[800:960]) and np.all(np.isnan(got[k, 160:]))
    # steps that change: rows 0, 160, 320 then 960, 1280, ...; outputs packed
    # (each call streams at least 2 MB of index, so the streaming kernel runs)
    idx = [0, 1, 2, 6, 8, 10, 12, 13, 63, 62, 61] * 6
    y3 = cuda.full((len(idx) * 160,), float("nan"), dtype=cuda.float32, device="cuda")
    gemms([views[i] for i in idx], [y3.data_ptr() + 4 * 160 * j for j in range(len(idx))])
    got = y3.cpu().numpy().reshape(len(idx), 160)
    for j, i in enumerate(idx):
        assert bits_eq(got[j], want[160 * i:160 * (i + 1)])
    # 300 matrices in random order into randomly placed outputs: about one
    # run each, more than one launch holds
    order = rng.integers(0, 64, 300)
    place = rng.permutation(300)
    y4 = cuda.full((300 * 160,), float("nan"), dtype=cuda.float32, device="cuda")
    gemms([views[i] for i in order], [y4.data_ptr() + 4 * 160 * int(place[j]) for j in range(300)])
    got = y4.cpu().numpy().reshape(300, 160)
    for j, i in enumerate(order):
        assert bits_eq(got[place[j]], want[160 * i:160 * (i + 1)])


# Many activations against small matrices (Whistle's decode GEMMs at
# batched streams, its prefill and the cross-memory projection): the
# streaming kernel over (activation, tile) items from 5 activations and 128
# rows, the per-activation kernel (cq_lut_acts.cu) for fewer rows of group
# 128 (the mHC φ).
ACTS_CASES = [(8, (384, 96, 128, 512), 512, 2), (37, (512,), 512, 2), (256, (384, 512), 512, 2), (5, (96, 40), 512, 2),
              (9, (4, 4, 16), 2048, 4), (300, (24,), 2048, 4), (12, (16384,), 512, 4), (200, (1000, 7), 512, 4),
              (64, (1, 3, 130, 511), 1024, 2)]


@pytest.mark.parametrize("case", ACTS_CASES, ids=[f"r{c[0]}_{'+'.join(map(str, c[1]))}x{c[2]}b{c[3]}"
                                                  for c in ACTS_CASES])
def test_acts_kernel_bit_exact(wb, orc, cuda, case):
    rows, outs, in_, bits = case
    rng = np.random.default_rng(rows + in_ + bits + len(outs))
    ps = [wb.synth.random_packed(rng, o, in_, 128, bits, "lloyd") for o in outs]
    for q in ps[1:]:
        q.Codebook = ps[0].Codebook
    ms = [wb.cq.New(p) for p in ps]
    x = (rng.normal(size=rows * in_) * rng.choice([1e-3, 1.0, 30.0], size=rows * in_)).astype(np.float32)
    x[:in_] = 0.0  # an all-zero activation: M = 0 in every group
    xd = cuda.from_numpy(x).cuda()
    yds = [cuda.full((rows * m.Out(),), float("nan"), dtype=cuda.float32, device="cuda") for m in ms]
    wb.cq.GEMMs(ms, yds, xd, rows)
    wants = orc.gemms_lut([orc.OracleMatrix.of(p) for p in ps], x, rows)
    for k in range(len(ms)):
        assert bits_eq(yds[k].cpu().numpy(), wants[k].reshape(-1)), k
