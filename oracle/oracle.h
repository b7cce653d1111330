/*
 * oracle.h — CPU restatement of go-whistle's quantized hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker the CUDA kernels are
 * compared against, and the timed CPU baseline in bench.py. The product path
 * (libwhistle_b200.so) never links, loads or calls it.
 *
 * Every function restates one routine of the reference (a Go module with no
 * C, C++ or CUDA of its own) with the same float32 operations in the same
 * order. Compile with -ffp-contract=off and without -ffast-math: the
 * reference's lut path protects each rounding with an explicit float32()
 * conversion, and the amd64 Go compiler never fuses a multiply into an add,
 * so no FMA may appear here either.
 *
 * Parity is pinned by the reference's own known-answer tests and bounds
 * (tests/test_oracle_pins.py): TestFWHT's explicit Sylvester product,
 * TestQuantizeRow's literal cases, TestFloat16ToFloat32's table, and
 * TestKernels' float64 dequantisation with rotatedBound + lutBound. The
 * reference publishes no stored output vectors for this path.
 */
#ifndef WHISTLE_ORACLE_H
#define WHISTLE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* internal/cact/half.go:8 float16ToFloat32 */
float wo_f16_to_f32(uint16_t h);

/* internal/cq/kernel.go:384 fwht: in-place ±1 Sylvester FWHT, n a power of two */
void wo_fwht(float *x, int n);

/* internal/cq/lut.go:213 lutStepOf */
float wo_lut_step_of(int group);

/* internal/cq/lut.go:239,263 lutTables2Generic / lutTables4Generic: the byte
 * planes as the reference stores them (32 bytes per nibble table: 16 lo, then
 * 16 hi). n = len(x) = the group size. Returns the group bound M. */
float wo_lut_tables_planes(int bits, uint8_t *tab, const float *x, int n, const float *cb, float cb_max);

/* The same tables as signed integers v (tab[q*16 + c]), lo + 128*(hi-64). */
float wo_lut_tables_int(int bits, int16_t *tab, const float *x, int n, const float *cb, float cb_max);

/* internal/cq/lut.go:289 lutLookupGeneric on the reference's 32-row blocked
 * layout (lut.go:51-54): y[b*32+i] for `blocks` blocks. */
void wo_lut_lookup_blocked(float *y, const uint8_t *idx, const uint8_t *tab, const float *norm,
                           const float *steps, int blocks, int groups, int gb);

/* internal/cq/lut_amd64.s:236 lutLookupAVX2, restated with AVX2 intrinsics:
 * the same products as wo_lut_lookup_blocked, bit for bit (asm_test.go). */
void wo_lut_lookup_blocked_avx2(float *y, const uint8_t *idx, const uint8_t *tab, const float *norm,
                                const float *steps, int blocks, int groups, int gb);

/* lut_amd64.s:20 fwhtAVX2 (n a power of two >= 8) and :127/:184
 * lutTables2AVX2 / lutTables4AVX2 (n a multiple of 8), restated: the same
 * bits as wo_fwht and wo_lut_tables_planes. */
void wo_fwht_avx2(float *x, int n);
float wo_lut_tables_planes_avx2(int bits, uint8_t *tab, const float *x, int n, const float *cb, float cb_max);

/*
 * A CQ matrix as cact.Packed holds it (internal/cact/packed.go:18-40): index
 * = out rows of row_bytes LSB-first bytes, norms16 = [out][groups] FP16,
 * cb = 2^bits float32 levels.
 */
typedef struct {
    int out, in, group, bits;
    const uint8_t *index;
    const uint16_t *norms16;
    const float *cb;
} wo_packed;

/* The lut kernel's GEMM (internal/cq/lut.go:102-204 with the generic
 * routines, i.e. asm_test.go:189 lutGEMMGeneric): x is [rows][in],
 * y is [rows][out]. Returns 0, or -1 if a group's index bytes exceed
 * lutMaxGroupBytes. */
int wo_cq_gemm_lut(const wo_packed *p, const float *x, int rows, float *y);

/* The same with the reference's work split on `threads` OS threads
 * (lut.go:93-124): the timed CPU baseline. Same bits as wo_cq_gemm_lut. */
int wo_cq_gemm_lut_mt(const wo_packed *p, const float *x, int rows, float *y, int threads);

/* GEMMs (internal/cq/kernel.go:134): n matrices sharing one x, tables built
 * once per activation. ys[k] is [rows][p[k].out]. */
int wo_cq_gemms_lut(const wo_packed *ps, int n, const float *x, int rows, float **ys);

/* The Exact path (internal/cq/kernel.go:162-373, matrix.go:152): nibble4 on
 * activations in blocks of four, nibble on the leftover ones, as gemm's
 * split (kernel.go:117-129) gives for any worker count. */
void wo_cq_gemm_exact(const wo_packed *p, const float *x, int rows, float *y);

/* internal/cq/kernel.go:220 gather: the float reference kernel. */
void wo_cq_gemm_gather(const wo_packed *p, const float *x, int rows, float *y);

/* internal/cq/matrix.go:161 Row: row r dequantised as cact.CQ does it. */
void wo_cq_row(const wo_packed *p, int r, float *dst);

/* internal/needle/int8.go:36 QuantizeRow; returns the scale. */
float wo_quantize_row(int8_t *q, const float *x, int n);

/* internal/needle/int8.go:115 QuantizeRows: rows*cols values in chunks of width. */
void wo_quantize_rows(const float *x, int rows, int cols, int width, int8_t *q, float *s);

/* internal/needle/exp.go:238 expSubSumGeneric + load.go:127 softmaxInPlace. */
void wo_softmax(float *s, int n);

/*
 * internal/needle/int8.go:208 AttendInt8Spans. q is [t][heads][qk]; k8 is
 * [nkeys][kv_heads*qk] with ks [nkeys][kv_heads]; v8 is [nkeys][kv_heads*vd]
 * with vs [nkeys][kv_heads]; spans is [t][4] = lo0, hi0, lo1, hi1 (two
 * ascending disjoint key ranges per query row). out is [t][heads][vd];
 * probs, if not NULL, is [t][heads][nkeys] and only written at span keys.
 */
void wo_attend_int8_spans(const float *q, int t, int heads, const int8_t *k8, const float *ks,
                          const int8_t *v8, const float *vs, int nkeys, int kv_heads, int qk, int vd,
                          const int32_t *spans, float scale, int quant_q, float *probs, float *out);

/* The same on `threads` OS threads, one (row, head) per task: the CPU
 * baseline of the attention. Same bits. */
void wo_attend_int8_spans_mt(const float *q, int t, int heads, const int8_t *k8, const float *ks,
                             const int8_t *v8, const float *vs, int nkeys, int kv_heads, int qk, int vd,
                             const int32_t *spans, float scale, int quant_q, float *probs, float *out,
                             int threads);

/* internal/decoder/decoder.go:508-523 logits' head scale (logits = y·head
 * when head != 1, else y) and greedy.go:182 argmax per row of vocab values. */
void wo_head_argmax(const float *y, int rows, int vocab, float head, float *logits, int32_t *idx);

#ifdef __cplusplus
}
#endif
#endif
