/*
 * needle_oracle.c — CPU restatement of internal/needle's int8 numerics: the
 * per-head int8 quantiser and the int8 KV-cache attention. TEST
 * INFRASTRUCTURE ONLY: the checker for tests/ and the CPU baseline of
 * bench.py, never part of the product.
 *
 * The attention follows the reference's generic (purego) routines: exact
 * int32 dots (int8kernel.go:46 dotsI8Generic), the float64 exp rounded to
 * float32 and summed in key order (exp.go:238 expSubSumGeneric), and the
 * key-by-key axpy with each product rounded before the add
 * (int8kernel.go:60 axpysI8Generic). exp() here is libm's; the reference's
 * is Go's math.Exp. Both are within one float64 ulp, so their float32
 * roundings differ only when e^x lies within about 2^-29 (relative) of a
 * float32 rounding boundary.
 */
#include "oracle.h"

#include <math.h>
#include "par.h"
#include <stdlib.h>
#include <string.h>

/* internal/needle/int8.go:36 QuantizeRow. */
float wo_quantize_row(int8_t *q, const float *x, int n) {
    float m = 0.0f;
    for (int i = 0; i < n; i++) {
        float a = fabsf(x[i]);
        if (a > m) m = a;
    }
    float s = 1.0f;
    if (m > 0.0f) s = m / 127.0f;
    for (int i = 0; i < n; i++) {
        double r = nearbyint((double)(x[i] / s));
        if (r < -128.0) r = -128.0;
        if (r > 127.0) r = 127.0;
        q[i] = (int8_t)r;
    }
    return s;
}

/* internal/needle/int8.go:115 QuantizeRows / :125 Append. */
void wo_quantize_rows(const float *x, int rows, int cols, int width, int8_t *q, float *s) {
    int chunks = rows * (cols / width);
    for (int c = 0; c < chunks; c++) s[c] = wo_quantize_row(q + (size_t)c * width, x + (size_t)c * width, width);
}

/* internal/needle/load.go:127 softmaxInPlace with exp.go:238 expSubSumGeneric. */
void wo_softmax(float *s, int n) {
    float m = -INFINITY;
    for (int i = 0; i < n; i++)
        if (s[i] > m) m = s[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        float d = s[i] - m;
        float e = (float)exp((double)d);
        s[i] = e;
        sum += e;
    }
    for (int i = 0; i < n; i++) s[i] /= sum;
}

/* One (row i, head h) of internal/needle/int8.go:208 AttendInt8Spans. w and
 * q8/dots are scratch of nkeys and qk. */
static void attend_one(const float *q, int i, int h, int heads, const int8_t *k8, const float *ks, const int8_t *v8,
                       const float *vs, int nkeys, int kv_heads, int qk, int vd, const int32_t *sp, float scale,
                       int quant_q, float *probs, float *out, float *w, int8_t *q8) {
    int kcols = kv_heads * qk, vcols = kv_heads * vd;
    int kv = h / (heads / kv_heads);
    const float *qi = q + ((size_t)i * heads + h) * qk;
    int len0 = sp[1] - sp[0], len1 = sp[3] - sp[2];
    int lens[2] = {len0, len1}, los[2] = {sp[0], sp[2]};
    float sq = 0.0f;
    if (quant_q) sq = wo_quantize_row(q8, qi, qk);

    int o = 0;
    for (int p = 0; p < 2; p++) {
        float *sj = w + o;
        int lo = los[p];
        for (int j = 0; j < lens[p]; j++) {
            const int8_t *row = k8 + (size_t)(lo + j) * kcols + (size_t)kv * qk;
            float sk = ks[(size_t)(lo + j) * kv_heads + kv];
            if (quant_q) {
                /* int8.go:278 int8Logits: float32(dot) * (sq * sk) / scale */
                int32_t dot = 0;
                for (int c = 0; c < qk; c++) dot += (int32_t)q8[c] * (int32_t)row[c];
                float f = (float)dot;
                float ss = sq * sk;
                float t = f * ss;
                sj[j] = t / scale;
            } else {
                /* int8.go:289 dotsF32I8, then sj * sk / scale (int8.go:245-247) */
                float s = 0.0f;
                for (int c = 0; c < qk; c++) {
                    float t = qi[c] * (float)row[c];
                    s += t;
                }
                float t = s * sk;
                sj[j] = t / scale;
            }
        }
        o += lens[p];
    }

    wo_softmax(w, len0 + len1);

    float *oh = out + ((size_t)i * heads + h) * vd;
    o = 0;
    for (int p = 0; p < 2; p++) {
        float *sj = w + o;
        int lo = los[p];
        if (probs) memcpy(probs + ((size_t)i * heads + h) * nkeys + lo, sj, (size_t)lens[p] * sizeof(float));
        for (int j = 0; j < lens[p]; j++) sj[j] *= vs[(size_t)(lo + j) * kv_heads + kv];
        /* int8kernel.go:60 axpysI8Generic */
        for (int j = 0; j < lens[p]; j++) {
            const int8_t *row = v8 + (size_t)(lo + j) * vcols + (size_t)kv * vd;
            for (int d = 0; d < vd; d++) {
                float t = sj[j] * (float)row[d];
                oh[d] += t;
            }
        }
        o += lens[p];
    }
}

typedef struct {
    const float *q;
    int t, heads;
    const int8_t *k8;
    const float *ks;
    const int8_t *v8;
    const float *vs;
    int nkeys, kv_heads, qk, vd;
    const int32_t *spans;
    float scale;
    int quant_q;
    float *probs, *out;
} spans_job;

/* Task = (head, row) in int8.go:218-221's order: heads outer, rows inner. */
static void spans_task(int task, void *arg) {
    const spans_job *j = arg;
    int h = task / j->t, i = task % j->t;
    float *w = malloc((size_t)(j->nkeys > 0 ? j->nkeys : 1) * sizeof(float));
    int8_t *q8 = malloc((size_t)j->qk);
    attend_one(j->q, i, h, j->heads, j->k8, j->ks, j->v8, j->vs, j->nkeys, j->kv_heads, j->qk, j->vd,
               j->spans + 4 * (size_t)i, j->scale, j->quant_q, j->probs, j->out, w, q8);
    free(w);
    free(q8);
}

void wo_attend_int8_spans(const float *q, int t, int heads, const int8_t *k8, const float *ks, const int8_t *v8,
                          const float *vs, int nkeys, int kv_heads, int qk, int vd, const int32_t *spans, float scale,
                          int quant_q, float *probs, float *out) {
    wo_attend_int8_spans_mt(q, t, heads, k8, ks, v8, vs, nkeys, kv_heads, qk, vd, spans, scale, quant_q, probs, out,
                            1);
}

void wo_attend_int8_spans_mt(const float *q, int t, int heads, const int8_t *k8, const float *ks, const int8_t *v8,
                             const float *vs, int nkeys, int kv_heads, int qk, int vd, const int32_t *spans,
                             float scale, int quant_q, float *probs, float *out, int threads) {
    memset(out, 0, (size_t)t * heads * vd * sizeof(float));
    spans_job job = {q, t, heads, k8, ks, v8, vs, nkeys, kv_heads, qk, vd, spans, scale, quant_q, probs, out};
    int tasks = t * heads;
    wo_parallel_for(tasks, threads < 1 ? 1 : threads, spans_task, &job);
}

/*
 * Many independent streams, each its own AttendInt8Spans call with one query
 * row (a decode step): the CPU baseline of the batched attention, one
 * stream per task. Stream b's arrays start at b times the given strides.
 */
typedef struct {
    const float *q;
    int heads;
    const int8_t *k8;
    const float *ks;
    const int8_t *v8;
    const float *vs;
    int cap;
    const int32_t *nkeys;
    int kv_heads, qk, vd;
    float scale;
    float *out;
} streams_job;

static void stream_task(int b, void *arg) {
    const streams_job *j = arg;
    float *w = malloc((size_t)(j->cap > 0 ? j->cap : 1) * sizeof(float));
    int8_t *q8 = malloc((size_t)j->qk);
    int32_t sp[4] = {0, 0, 0, j->nkeys[b]};
    float *ob = j->out + (size_t)b * j->heads * j->vd;
    memset(ob, 0, (size_t)j->heads * j->vd * sizeof(float));
    for (int h = 0; h < j->heads; h++)
        attend_one(j->q + (size_t)b * j->heads * j->qk, 0, h, j->heads, j->k8 + (size_t)b * j->cap * j->kv_heads * j->qk,
                   j->ks + (size_t)b * j->cap * j->kv_heads, j->v8 + (size_t)b * j->cap * j->kv_heads * j->vd,
                   j->vs + (size_t)b * j->cap * j->kv_heads, j->nkeys[b], j->kv_heads, j->qk, j->vd, sp, j->scale, 1,
                   NULL, ob, w, q8);
    free(w);
    free(q8);
}

void wo_attend_int8_streams_mt(int streams, const float *q, int heads, const int8_t *k8, const float *ks,
                               const int8_t *v8, const float *vs, int cap, const int32_t *nkeys, int kv_heads, int qk,
                               int vd, float scale, float *out, int threads) {
    streams_job job = {q, heads, k8, ks, v8, vs, cap, nkeys, kv_heads, qk, vd, scale, out};
    wo_parallel_for(streams, threads < 1 ? 1 : threads, stream_task, &job);
}
