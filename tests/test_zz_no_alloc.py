"""wc_cq_gemm_tc_noalloc: the tensor-core GEMM for callers that must not
allocate GPU memory while they run (a real-time transcription loop that
cannot afford a cudaMalloc stall in a decode step, or a serving process whose
GPU memory is reserved once at start-up). It runs the same kernels as
wc_cq_gemm_ex with WC_GEMM_TENSOR_CORES, on a fixed scratch array inside the
library instead of an allocated buffer.

This file is collected last (its name sorts last) so that a run that stops
at the first failure has already run every other test; it also passes on
its own in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import refmath

pytestmark = pytest.mark.gpu

WC_GEMM_TENSOR_CORES = 1
WC_ERR_INVALID = 1


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


# (out, in, group, bits, row counts of the calls in a row). A smaller call
# after a larger one finds the larger one's rotated rows in the array; from
# 1024 rows both entry points run the persistent kernel.
@pytest.mark.parametrize("shape", [(512, 512, 32, 4, (1000, 200)), (1120, 512, 128, 2, (1000, 200)),
                                   (300, 2048, 32, 4, (1000, 200)), (512, 512, 32, 4, (4096, 1500))])
def test_no_alloc_matches_allocating_entry_point(wb, cuda, shape):
    out, in_, group, bits, calls = shape
    lib = wb._lib.lib()
    rng = np.random.default_rng(out + in_)
    p = wb.synth.random_packed(rng, out, in_, group, bits, "lloyd")
    m = wb.cq.New(p)
    # Load time: the weight image is built here (this call may allocate).
    wb._lib.check(lib.wc_cq_prepare_tc(m.handle))
    err = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    # Two calls in a row with different inputs: the second must not see the
    # first's scratch contents.
    for rows in calls:
        x = cuda.randn(rows, in_, device="cuda", dtype=cuda.float32)
        want = cuda.empty(rows, out, device="cuda", dtype=cuda.float32)
        got = cuda.full((rows, out), float("nan"), device="cuda", dtype=cuda.float32)
        wb._lib.check(lib.wc_cq_gemm_ex(m.handle, _ptr(x), _ptr(want), rows, WC_GEMM_TENSOR_CORES, None))
        wb._lib.check(lib.wc_cq_gemm_tc_noalloc(m.handle, _ptr(x), _ptr(got), rows, _ptr(err), None))
        cuda.cuda.synchronize()
        assert int(err.item()) == 0
        g, w = got.cpu().numpy(), want.cpu().numpy()
        # Same kernels on the same inputs: the same bits, and so within the
        # tensor-core bound of the float64 product.
        assert np.array_equal(g.view(np.uint32), w.view(np.uint32))
        ref, bound = refmath.tc_bound(p, x.cpu().numpy().astype(np.float64))
        assert np.all(np.abs(g - ref) <= bound)


def test_no_alloc_limits(wb, cuda):
    lib = wb._lib.lib()
    rng = np.random.default_rng(5)
    p = wb.synth.random_packed(rng, 128, 2048, 32, 4, "lloyd")
    m = wb.cq.New(p)
    x = cuda.zeros(5000, 2048, device="cuda", dtype=cuda.float32)
    y = cuda.full((5000, 128), 7.0, device="cuda", dtype=cuda.float32)
    # Not prepared: refused, nothing allocated on its behalf.
    assert lib.wc_cq_gemm_tc_noalloc(m.handle, _ptr(x), _ptr(y), 16, None, None) == WC_ERR_INVALID
    assert "wc_cq_prepare_tc" in wb._lib.last_error()
    wb._lib.check(lib.wc_cq_prepare_tc(m.handle))
    # 5000 rows of 2048 columns exceed the 16 MiB array (4096 rows at most).
    assert lib.wc_cq_gemm_tc_noalloc(m.handle, _ptr(x), _ptr(y), 5000, None, None) == WC_ERR_INVALID
    assert "4096 rows" in wb._lib.last_error()
    assert bool((y == 7.0).all())
    # At the limit it runs.
    wb._lib.check(lib.wc_cq_gemm_tc_noalloc(m.handle, _ptr(x), _ptr(y), 4096, None, None))
    cuda.cuda.synchronize()
    assert bool((y[:4096] == 0.0).all()) and bool((y[4096:] == 7.0).all())


def test_no_alloc_allocates_nothing(wb, cuda):
    """Device memory stays where it was across repeated calls (after the
    one-time look-up of the array's address), both in torch's view and in
    the driver's free-memory count."""
    lib = wb._lib.lib()
    rng = np.random.default_rng(9)
    p = wb.synth.random_packed(rng, 1024, 512, 32, 4, "lloyd")
    m = wb.cq.New(p)
    wb._lib.check(lib.wc_cq_prepare_tc(m.handle))
    x = cuda.randn(2048, 512, device="cuda", dtype=cuda.float32)
    y = cuda.empty(2048, 1024, device="cuda", dtype=cuda.float32)
    # Warm-up: module load, the address look-up, kernel attributes.
    wb._lib.check(lib.wc_cq_gemm_tc_noalloc(m.handle, _ptr(x), _ptr(y), 2048, None, None))
    cuda.cuda.synchronize()
    free0, _ = cuda.cuda.mem_get_info()
    alloc0 = cuda.cuda.memory_allocated()
    for rows in (2048, 100, 1024, 7):
        wb._lib.check(lib.wc_cq_gemm_tc_noalloc(m.handle, _ptr(x), _ptr(y), rows, None, None))
    cuda.cuda.synchronize()
    free1, _ = cuda.cuda.mem_get_info()
    assert free1 == free0, f"free device memory moved by {free0 - free1} bytes"
    assert cuda.cuda.memory_allocated() == alloc0
    code = ctypes.c_int(-1)
    wb._lib.check(lib.wc_device_status(ctypes.byref(code)))
    assert code.value == 0
