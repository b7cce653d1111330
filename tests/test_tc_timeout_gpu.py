"""The tensor-core GEMM's bounded waits, run out on purpose without a fault.

wc_testing_gemm_tc_stall launches the kernel with a producer that issues no
copies at all, so nothing is ever in flight: the MMA issuer's wait for the
first chunk and the epilogue's wait for the accumulator run out after a
short bound, the kernel records its code on the device error word, frees
its TMEM and returns. The test reads the code through wc_device_status, then
checks that the next normal call on the same matrix (whose TMEM allocation
would never succeed had the stalled CTAs kept theirs) runs clean and gives
the same bits as before the stall.
"""

from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WC_GEMM_TENSOR_CORES = 1

# Codes the kernels record (cq_gemm_tc.cu): 2 the MMA issuer's wait for a
# chunk, 3 the epilogue's wait for the accumulator; 14 and 15 the same two
# in the persistent kernel (from 1,024 rows).
STALL_CODES = {300: {2, 3}, 1024: {14, 15}}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _status(wb):
    code = ctypes.c_int(-1)
    wb._lib.check(wb._lib.lib().wc_device_status(ctypes.byref(code)))
    return code.value


@pytest.mark.parametrize("rows", sorted(STALL_CODES))
def test_stalled_producer_times_out_and_recovers(wb, cuda, rows):
    lib = wb._lib.lib()
    rng = np.random.default_rng(rows)
    p = wb.synth.random_packed(rng, 512, 512, 32, 4, "lloyd")
    m = wb.cq.New(p)
    x = cuda.randn(rows, 512, device="cuda", dtype=cuda.float32)
    want = cuda.empty(rows, 512, device="cuda", dtype=cuda.float32)
    got = cuda.full((rows, 512), float("nan"), device="cuda", dtype=cuda.float32)
    wb._lib.check(lib.wc_cq_gemm_ex(m.handle, _ptr(x), _ptr(want), rows, WC_GEMM_TENSOR_CORES, None))
    assert _status(wb) == 0

    scratch = cuda.empty(rows, 512, device="cuda", dtype=cuda.float32)
    t0 = time.perf_counter()
    wb._lib.check(lib.wc_testing_gemm_tc_stall(m.handle, _ptr(x), _ptr(scratch), rows, None))
    code = _status(wb)  # synchronises: the stalled kernel has returned
    took = time.perf_counter() - t0
    assert code in STALL_CODES[rows], code
    assert took < 30.0, took
    # The error word is cleared by the read.
    assert _status(wb) == 0

    # The next normal call: TMEM was freed, the barriers start afresh.
    wb._lib.check(lib.wc_cq_gemm_ex(m.handle, _ptr(x), _ptr(got), rows, WC_GEMM_TENSOR_CORES, None))
    assert _status(wb) == 0
    assert np.array_equal(got.cpu().numpy().view(np.uint32), want.cpu().numpy().view(np.uint32))


def test_stall_entry_point_checks_its_arguments(wb, cuda):
    lib = wb._lib.lib()
    p = wb.synth.random_packed(np.random.default_rng(1), 128, 512, 32, 4, "lloyd")
    m = wb.cq.New(p)
    x = cuda.zeros(4, 512, device="cuda", dtype=cuda.float32)
    with pytest.raises(wb.Panic, match="nil matrix"):
        wb._lib.check(lib.wc_testing_gemm_tc_stall(None, _ptr(x), _ptr(x), 4, None))
    with pytest.raises(wb.Panic, match="empty product"):
        wb._lib.check(lib.wc_testing_gemm_tc_stall(m.handle, _ptr(x), _ptr(x), 0, None))
