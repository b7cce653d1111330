// common.cuh — shared definitions of the whistle_b200 CUDA library (sm_100a).
//
// The device-side CQ matrix layout and the constants of the reference's lut
// kernel (internal/cq/lut.go:31-39), plus error plumbing for the C ABI.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <cstdarg>
#include <cstdio>

#include <string>

#include "../../include/whistle_b200.h"

namespace wb {

// internal/cq/lut.go:33 lutQ: table entries are integers in [-lutQ, lutQ].
constexpr int kLutQ = 8191;
// internal/cq/lut.go:38 lutMaxGroupBytes: the reference's lut kernel takes
// groups of at most 256 index bytes (its uint16 plane sums); larger groups
// run its nibble4 kernel, and so they do here (the Exact kernels).
constexpr int kLutMaxGroupBytes = 256;

// A CQ matrix (or a Rows view) as the kernels see it.
//
// HBM layout, chosen for coalesced 16-byte loads by lanes that each own one
// row of one group:
//   idx[(g * ld + r) * gb + j]  index byte j of group g of layout row r
//   nrm[g * ld + r]             FP16 norm of (r, g)
// i.e. group-major: all rows' bytes of group 0, then group 1, ... A view
// [lo, hi) keeps ld and adds lo to row0, so it shares the parent's storage
// without a copy (matrix.go:133 Rows).
struct CqView {
    const uint8_t *idx;
    const __half *nrm;
    int out;   // rows of this view
    int row0;  // first layout row of the view
    int ld;    // rows of the layout (the root matrix's Out)
};

// The parameters every matrix sharing one activation's tables has in
// common (lut.go:206 sharesTables): input width, group, index width and
// codebook.
struct CqShape {
    int in, group, bits, groups, gb, row_bytes, pad;
    float cb[16];
    float cb_max;    // max |cb| (matrix.go:87-89)
    float lut_step;  // lutStepOf(group) (lut.go:213)
    float inv_sqrt;  // invSqrt(group) (kernel.go:375)
};

}  // namespace wb

// Error plumbing shared by the C-ABI translation units.
namespace wb {
wc_status set_error(wc_status st, const std::string &msg);
wc_status cuda_error(cudaError_t e, const char *what);
// Counts one kernel launch (wc_launch_count).
void count_launch();
// The current device's error word of the kernels' bounded waits.
int *err_word();
// GEMMs on device memory (api.cu): lut, or tensor cores with the rotated
// image in tc_buf (at least tc_a_bytes of the rows and widths).
wc_status gemms_device(const wc_cq *const *ms, int n, const float *x, float *const *ys, int rows, bool tc,
                       void *tc_buf, size_t tc_bytes, cudaStream_t st);
// A matrix's shape and device view, for the library's own kernels.
bool cq_internal(const wc_cq *h, CqShape *s, CqView *v);
// printf-style formatting of an error message.
inline std::string fmt(const char *f, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, f);
    vsnprintf(buf, sizeof buf, f, ap);
    va_end(ap);
    return buf;
}
// wc_attend_int8_streams with kv_group streams reading each K/V block
// (stream b reads block b / kv_group): the beams of one clip share its
// cross-attention memory.
wc_status attend_streams_grouped(int streams, const float *q, int heads, const int8_t *k8, const float *ks,
                                 const int8_t *v8, const float *vs, int cap, const int32_t *nkeys, int kv_heads,
                                 int qk, int vd, float scale, int flags, float *out, int kv_group, cudaStream_t st);
}  // namespace wb

#define WB_CUDA(call)                                            \
    do {                                                         \
        cudaError_t e_ = (call);                                 \
        if (e_ != cudaSuccess) return ::wb::cuda_error(e_, #call); \
    } while (0)
