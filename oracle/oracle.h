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

/* ------------------------------------------------------------------
 * Whistle's decoder step (whistle_oracle.c): internal/decoder with the
 * Best() hypothesis (decoder/hypothesis.go:199) and needle.Int8{Act, KV}.
 */

/* Rows [lo, hi) of p sharing its storage (matrix.go:133 Rows). */
wo_packed wo_rows(const wo_packed *p, int lo, int hi);

/* internal/needle/rope.go:20 NewRope's tables [len][head_dim/2]. */
void wo_rope_tables(int head_dim, int len, double theta, float *cos_t, float *sin_t);

/* internal/needle/mhc.go:300 sinkhorn (20 iterations) on an n×n matrix. */
void wo_sinkhorn(float *k, int n);

/* The decoder step's pieces, for the reference's known-answer tests:
 * engram.go:141 ngramHash over hist[0..len) (hist[len-1] the current
 * token), norm.go:60 ZCRMSNorm.Apply (scale, not gain), norm.go:82 RMSUnit,
 * rope.go:73 apply with one position's tables, mhc.go:300 sinkhorn with a
 * chosen iteration count. */
uint32_t wo_ngram_hash(int c, int order, const int *hist, int len);
void wo_zc_norm(float *dst, const float *x, int rows, int d, const float *scale);
void wo_rms_unit(float *dst, const float *x, int rows, int d);
void wo_rope_apply(float *x, int half, const float *cs, const float *sn);
void wo_sinkhorn_iters(float *k, int n, int iters);

/* One decoder layer's weights: needle.Block (block.go:21), its Attention
 * (attention.go:38), HadamardMLP (hadamard.go:28), the layer's cross
 * (decoder/cross.go:26) and its mHC heads (mhc.go:30). Norm vectors are the
 * stored scales (gain = 1 + scale); gates are the raw parameters. */
typedef struct {
    const float *norm_in, *post_norm, *pre_hada; /* [dim] */
    float attn_gate;
    wo_packed q_proj, k_proj, v_proj, gate_proj, out_proj;
    const float *q_taps, *k_taps, *v_taps; /* [taps][width] */
    const float *q_norm, *k_norm;          /* [qk] */
    const float *d1, *d2, *b2, *d3, *d4;   /* [na·nb] */
    const float *hada_w[3][2];             /* stage s: a [na][na], b [nb][nb] */
    const float *cond_v;                   /* [dim][rank] */
    const float *cond_u;                   /* [rank][na·nb] */
    const float *x_norm_in, *x_post_norm, *x_q_norm, *x_k_norm;
    float x_attn_gate;
    wo_packed x_q_proj, x_k_proj, x_v_proj, x_gate_proj, x_out_proj;
    float a_pre, a_post, a_res;
    const float *b_pre, *b_post; /* [lanes] */
    const float *b_res;          /* [lanes·lanes] */
    wo_packed phi_pre, phi_post, phi_res; /* this layer's rows of the stacked φ */
} wo_dec_layer;

/* One engram site (needle/engram.go:35 Engram) and its decoder layer. */
typedef struct {
    wo_packed tables;                /* [n_tables·slots][sub] */
    wo_packed key_proj, value_proj;  /* [dim][n_tables·sub] */
    const float *taps;               /* [etaps][dim] */
    int layer;
} wo_engram_site;

typedef struct {
    int dim, lanes, layers, vocab;
    int heads, kv_heads, qk, vd, taps; /* self-attention */
    int x_heads, x_qk, x_vd;           /* cross-attention */
    int na, nb, rank;                  /* HadamardMLP */
    int n_sites, n_tables, slots, sub, etaps, max_order;
    const int *orders;                 /* [n_tables]: the n-gram order of table c */
    const int *hada_p1, *hada_p2;      /* [na·nb] */
    const float *rope_cos, *rope_sin;  /* [rope_len][qk/2] */
    int rope_len;
    wo_packed embedding;               /* [vocab][dim], also the tied head */
    const float *final_norm;           /* [dim] */
    const wo_dec_layer *layer;         /* [layers] */
    const wo_engram_site *site;        /* [n_sites] */
} wo_decoder;

typedef struct wo_dec_state wo_dec_state;

/* A sequence with room for cap positions and a memory of frames rows. */
wo_dec_state *wo_dec_new(const wo_decoder *d, int cap, int frames);
void wo_dec_free(wo_dec_state *s);
int wo_dec_len(const wo_dec_state *s);
/* decoder.go:223 State.Fork: an independent copy of s. */
wo_dec_state *wo_dec_fork(const wo_decoder *d, const wo_dec_state *s);

/* decoder.go:157 Memory for enc [frames][dim] (cross.go:181 project per
 * layer); starts the sequence afresh (decoder.go:194 NewState). */
void wo_dec_memory(const wo_decoder *d, wo_dec_state *s, const float *enc, int frames);

/* Layer l's int8 memory: k8 [frames][x_heads·x_qk], ks [frames][x_heads],
 * v8 [frames][x_heads·x_vd], vs. */
void wo_dec_memory_of(const wo_decoder *d, const wo_dec_state *s, int l, const int8_t **k8, const float **ks,
                      const int8_t **v8, const float **vs);

/* decoder.go:252 Extend with one token; logits [vocab]. -1 on a bad token
 * or a full cache. */
int wo_dec_extend(const wo_decoder *d, wo_dec_state *s, int tok, float *logits);

/* greedy.go:40 GreedyMemory with the language detected among langs. */
int wo_dec_greedy(const wo_decoder *d, wo_dec_state *s, int bos, const int *langs, int nlangs, int eos,
                  int max_tok, int *tokens, int *lang, int *eos_hit, float *margins);

/* GreedyMemory for many streams (enc [streams][frames][dim]) on threads. */
void wo_dec_greedy_streams_mt(const wo_decoder *d, int streams, const float *enc, int frames, int bos,
                              const int *langs, int nlangs, int eos, int max_tok, int *tokens, int *counts,
                              int *lang, int *eos_hit, int threads);

/* The same in two phases (the timed CPU baseline): every stream's memory
 * on threads (states with room for cap positions), then their greedy
 * decodes on threads. */
wo_dec_state **wo_dec_states_mt(const wo_decoder *d, int streams, const float *enc, int frames, int cap, int threads);
void wo_dec_states_free(wo_dec_state **st, int streams);
void wo_dec_greedy_states_mt(const wo_decoder *d, wo_dec_state **st, int streams, int bos, const int *langs,
                             int nlangs, int eos, int max_tok, int *tokens, int *counts, int *lang, int *eos_hit,
                             int threads);

/* ------------------------------------------------------------------
 * Whistle's encoder stack (whistle_oracle.c): internal/encoder's Stack
 * (encoder.go:167) with the Best() hypothesis (hypothesis.go:284: macaron
 * blocks, FFN scale 1/2, GLU value·σ(gate), SiLU after conv_out_norm,
 * centred depthwise conv, mHC lanes, RoPE θ = 1e5, final norm) and
 * needle.Int8{Act, KV} (whistle/model.go:85).
 *
 * One encoder layer (block.go:17). `b` holds the fields a decoder layer
 * shares with it: norm_in, post_norm, pre_hada (FFN2's norm), attn_gate,
 * q/k/v/gate/out_proj, q_norm, k_norm, the FFN2 HadamardMLP (hada.*: d1 …
 * cond_u), the mHC scalars, biases and φ rows; its taps and cross fields
 * are unused. hada0 holds the FFN1 HadamardMLP (hada_0.*) in the same
 * fields, with pre_hada_0 as its pre_hada. */
typedef struct {
    wo_dec_layer b, hada0;
    const float *conv_norm, *conv_out_norm; /* [dim] */
    wo_packed pw1, pw2;                     /* [2·dim][dim], [dim][dim] */
    const float *dw;                        /* [dw_k][dim] */
} wo_enc_layer;

/* `d` holds the sizes (dim, lanes, heads, kv_heads, qk, vd, na, nb, rank),
 * hada_p1/2, the RoPE tables (θ = 1e5) and final_norm; the rest unused. */
typedef struct {
    wo_decoder d;
    int dw_k;
    const wo_enc_layer *layer; /* [d.layers] */
} wo_encoder;

/* Attention forms of wo_enc_stack. */
enum {
    WO_ENC_ATTEND_FLOAT = 0, /* attention.go:480 attendGEMM on the fake-quantised q, k, v (the reference) */
    WO_ENC_ATTEND_INT8 = 1,  /* int8.go:208 AttendInt8Spans on their int8 codes (the device's exact order) */
};

/* encoder.go:167 Stack on `clips` clips of t rows of dim values each
 * (the stem's output, [clips][t][dim]): out [clips][t][dim]. Returns -1 if
 * t exceeds the RoPE tables, else 0. */
int wo_enc_stack(const wo_encoder *e, const float *x, int clips, int t, int form, float *out);
/* The same with one clip per task on `threads` OS threads. Same bits. */
int wo_enc_stack_mt(const wo_encoder *e, const float *x, int clips, int t, int form, float *out, int threads);

/* The block's row-wise pieces alone (the known-answer pins): block.go:257
 * gated (GLUValueGate) on t rows of 2·half values; block.go:290 depthwise
 * (DWCentred) on t rows of h channels with taps dw [k][h]; stem.go:367
 * applyAct (ActSiLU) on n values in place. */
void wo_enc_glu(const float *p, int t, int half, float *out);
void wo_enc_depthwise(const float *x, int t, int h, const float *dw, int k, float *out);
void wo_silu(float *x, int n);

#ifdef __cplusplus
}
#endif
#endif
