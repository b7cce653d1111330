/* whistle_b200_testing.h — test-only entry points of libwhistle_b200.so.
 *
 * Not part of the drop-in boundary: nothing in the reference binds these.
 * They exist so that the error paths of the device kernels can be exercised
 * without a GPU fault.
 */
#ifndef WHISTLE_B200_TESTING_H
#define WHISTLE_B200_TESTING_H

#include "whistle_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* One tensor-core GEMM (as wc_cq_gemm_ex with WC_GEMM_TENSOR_CORES; the
 * persistent kernel from 1,024 rows) whose producer issues no copies: the
 * MMA and epilogue waits run out after a short bound with nothing in
 * flight, the kernel records a nonzero code on the device error word, frees
 * its TMEM and returns. y is left undefined. wc_device_status reads (and
 * clears) the code; the next call runs normally. */
wc_status wc_testing_gemm_tc_stall(const wc_cq *m, const float *x, float *y, int rows, wc_stream stream);

#ifdef __cplusplus
}
#endif

#endif
