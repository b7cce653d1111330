/*
 * whistle_oracle.c — CPU restatement of Whistle's decoder step with the
 * engine's int8 numerics (internal/decoder + internal/needle, Best()
 * hypothesis, needle.Int8{Act, KV}). TEST INFRASTRUCTURE ONLY: the checker
 * of the device decoder in tests/ and the CPU baseline of bench.py; the
 * product never links it.
 *
 * Every routine names the reference function it restates. The CQ products
 * are the lut kernel's (cq_oracle.c: bit-exact with the reference's), the
 * int8 attention needle_oracle.c's. float32 operations are separate IEEE
 * roundings (-ffp-contract=off), as the reference's amd64 build computes
 * them. Three routines come from the third-party module algo-tensor v0.4.0
 * (absent from the reference tree): tensor.Axpy (y[i] += a·x[i]),
 * tensor.DotProduct (Σ a[i]·b[i]) and tensor.MatMulTransB
 * (dst[i][j] = Σ_k a[i][k]·b[j][k]). They are restated here in index
 * order with every product rounded before its add; the reference pins them
 * only through fixtures that need the absent float32 weights, so at those
 * three routines this restatement is unpinned. exp/log/sqrt/pow/sin/cos
 * are libm's (the reference: Go's math package); every one is within one
 * float64 ulp of the exact value, so their float32 roundings agree except
 * within about 2^-29 (relative) of a float32 rounding boundary.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"
#include "par.h"

/* internal/needle/norm.go:9 normEps, as the float32 it becomes. */
static const float kNormEps = 1e-6f;

/* norm.go:104 meanSquare: four float64 partial sums, rounded to float32. */
static float mean_square(const float *row, int n) {
    double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    int i = 0;
    for (; i + 3 < n; i += 4) {
        s0 += (double)row[i] * (double)row[i];
        s1 += (double)row[i + 1] * (double)row[i + 1];
        s2 += (double)row[i + 2] * (double)row[i + 2];
        s3 += (double)row[i + 3] * (double)row[i + 3];
    }
    for (; i < n; i++) s0 += (double)row[i] * (double)row[i];
    return (float)((s0 + s1 + s2 + s3) / (double)n);
}

/* norm.go:60 ZCRMSNorm.Apply on rows of d values; gain = 1 + scale
 * (norm.go:22 NewZCRMSNorm), applied as (g·x)/rms. dst may be x. */
static void zc_norm(float *dst, const float *x, int rows, int d, const float *scale) {
    for (int r = 0; r < rows; r++) {
        const float *row = x + (size_t)r * d;
        float *out = dst + (size_t)r * d;
        float ms = mean_square(row, d) + kNormEps;
        float rms = (float)sqrt((double)ms); /* norm.go:99 rowRMS */
        for (int c = 0; c < d; c++) {
            float g = 1.0f + scale[c];
            float t = g * row[c];
            out[c] = t / rms;
        }
    }
}

/* norm.go:82 RMSUnit. */
static void rms_unit(float *dst, const float *x, int rows, int d) {
    for (int r = 0; r < rows; r++) {
        const float *row = x + (size_t)r * d;
        float *out = dst + (size_t)r * d;
        float ms = mean_square(row, d) + kNormEps;
        float inv = (float)(1.0 / sqrt((double)ms));
        for (int c = 0; c < d; c++) out[c] = row[c] * inv;
    }
}

/* internal/needle/load.go:132 sigmoid (and decoder/cross.go:327). */
static float sigmoid(float x) { return (float)(1.0 / (1.0 + exp(-(double)x))); }

/* int8.go:62 fakeQuant: QuantizeRow per chunk of width, then float32(q)·s. */
static void fake_quant(float *dst, const float *x, int n, int width) {
    int8_t *q = malloc((size_t)width);
    for (int c = 0; c < n / width; c++) {
        float s = wo_quantize_row(q, x + (size_t)c * width, width);
        for (int i = 0; i < width; i++) dst[(size_t)c * width + i] = (float)q[i] * s;
    }
    free(q);
}

/* algo-tensor tensor.Axpy: y[i] += a·x[i] (product rounded, then the add). */
static void axpy(float *y, float a, const float *x, int n) {
    for (int i = 0; i < n; i++) {
        float t = a * x[i];
        y[i] += t;
    }
}

/* algo-tensor tensor.DotProduct: Σ a[i]·b[i] in index order. */
static float dot(const float *a, const float *b, int n) {
    float s = 0.0f;
    for (int i = 0; i < n; i++) {
        float t = a[i] * b[i];
        s += t;
    }
    return s;
}

/* algo-tensor tensor.MatMulTransB(dst, ldd, a, b, m, n, k):
 * dst[i·ldd + j] = Σ_l a[i·k + l]·b[j·k + l]. */
static void matmul_tb(float *dst, int ldd, const float *a, const float *b, int m, int n, int k) {
    for (int i = 0; i < m; i++)
        for (int j = 0; j < n; j++) dst[(size_t)i * ldd + j] = dot(a + (size_t)i * k, b + (size_t)j * k, k);
}

/* Rows [lo, hi) of a packed matrix, sharing its storage (matrix.go:133 Rows). */
wo_packed wo_rows(const wo_packed *p, int lo, int hi) {
    int groups = (p->in + p->group - 1) / p->group;
    int row_bytes = groups * p->group * p->bits / 8;
    wo_packed v = *p;
    v.out = hi - lo;
    v.index = p->index + (size_t)lo * row_bytes;
    v.norms16 = p->norms16 + (size_t)lo * groups;
    return v;
}

/* internal/needle/rope.go:20 NewRope: the float32 steps of the tables. */
void wo_rope_tables(int head_dim, int len, double theta, float *cos_t, float *sin_t) {
    int half = head_dim / 2;
    float *freqs = malloc((size_t)half * sizeof(float));
    for (int i = 0; i < half; i++) {
        float e = (float)(2 * i) / (float)head_dim;
        freqs[i] = 1.0f / (float)pow(theta, (double)e);
    }
    for (int t = 0; t < len; t++)
        for (int i = 0; i < half; i++) {
            double angle = (double)((float)t * freqs[i]);
            cos_t[(size_t)t * half + i] = (float)cos(angle);
            sin_t[(size_t)t * half + i] = (float)sin(angle);
        }
    free(freqs);
}

/* rope.go:73 apply: [x1·cos − x2·sin, x2·cos + x1·sin]. */
static void rope_apply(float *x, int half, const float *cs, const float *sn) {
    for (int i = 0; i < half; i++) {
        float a = x[i], b = x[half + i];
        float ac = a * cs[i], bs = b * sn[i], bc = b * cs[i], as = a * sn[i];
        x[i] = ac - bs;
        x[half + i] = bc + as;
    }
}

/* mhc.go:316 sinkhornExp; false if the logits are out of range. */
static int sinkhorn_exp(float *k, int n, int iters) {
    float lo = k[0], hi = k[0];
    for (int i = 1; i < n * n; i++) {
        if (k[i] < lo) lo = k[i];
        if (k[i] > hi) hi = k[i];
    }
    double spread = (double)hi - (double)lo;
    if (isinf(spread) || isnan(spread) || spread + 2.0 * iters * log((double)n) > 700.0) return 0;
    double e[64];
    for (int i = 0; i < n * n; i++) e[i] = exp((double)k[i] - (double)hi);
    for (int it = 0; it < iters; it++) {
        for (int r = 0; r < n; r++) {
            double s = 0;
            for (int c = 0; c < n; c++) s += e[r * n + c];
            for (int c = 0; c < n; c++) e[r * n + c] /= s;
        }
        for (int c = 0; c < n; c++) {
            double s = 0;
            for (int r = 0; r < n; r++) s += e[r * n + c];
            for (int r = 0; r < n; r++) e[r * n + c] /= s;
        }
    }
    for (int i = 0; i < n * n; i++) k[i] = (float)e[i];
    return 1;
}

/* mhc.go:403 logSumExp over n values at stride. */
static float log_sum_exp(const float *k, int off, int stride, int n) {
    float m = -INFINITY;
    for (int i = 0; i < n; i++)
        if (k[off + i * stride] > m) m = k[off + i * stride];
    if (isinf(m)) m = 0.0f;
    float s = 0.0f;
    for (int i = 0; i < n; i++) {
        float d = k[off + i * stride] - m;
        s += (float)exp((double)d);
    }
    return m + (float)log((double)s);
}

/* mhc.go:374 sinkhornLog. */
static void sinkhorn_log(float *k, int n, int iters) {
    for (int it = 0; it < iters; it++) {
        for (int r = 0; r < n; r++) {
            float l = log_sum_exp(k, r * n, 1, n);
            for (int c = 0; c < n; c++) k[r * n + c] -= l;
        }
        for (int c = 0; c < n; c++) {
            float l = log_sum_exp(k, c, n, n);
            for (int r = 0; r < n; r++) k[r * n + c] -= l;
        }
    }
    for (int i = 0; i < n * n; i++) k[i] = (float)exp((double)k[i]);
}

/* mhc.go:300 sinkhorn (20 iterations: mhcSinkhornIters, mhc.go:13). */
static void sinkhorn(float *k, int n) {
    if (n * n > 64) return;
    if (!sinkhorn_exp(k, n, 20)) sinkhorn_log(k, n, 20);
}

void wo_sinkhorn(float *k, int n) { sinkhorn(k, n); }

/* GEMMs of the products that read x (one row): needle.ApplyShared
 * (linear.go:102) -> cq.GEMMs, the lut kernel's bits. */
static void gemms1(const wo_packed *ms, int n, const float *x, float **ys) { wo_cq_gemms_lut(ms, n, x, 1, ys); }
static void gemm1(const wo_packed *m, const float *x, float *y) { wo_cq_gemm_lut(m, x, 1, y); }

/* One decoding sequence's state (decoder.go:173 State): the self-attention
 * caches with their tap history (cache.go:14 KVCache), the engram caches
 * (cache.go:143 EngramCache) and the cross-attention memory
 * (cross.go:163 memory) of every layer. */
struct wo_dec_state {
    int n, cap, frames;
    int8_t *k8, *v8; /* [layers][cap][kvh·qk], [layers][cap][kvh·vd] */
    float *ks, *vs;  /* [layers][cap][kvh] */
    float *qh, *kh, *vh; /* [layers][taps−1][width] raw rows, oldest first */
    int nh;              /* rows of tap history held (the same for every layer) */
    int *etoks;          /* [sites][max_order−1] */
    int ntoks;
    float *evraw; /* [sites][(etaps−1)·dilation][dim] */
    int nvraw;
    int8_t *xk8, *xv8; /* [layers][frames][x_heads·x_qk], [..][x_heads·x_vd] */
    float *xks, *xvs;  /* [layers][frames][x_heads] */
};

wo_dec_state *wo_dec_new(const wo_decoder *d, int cap, int frames) {
    wo_dec_state *s = calloc(1, sizeof *s);
    s->cap = cap;
    s->frames = frames;
    int L = d->layers, kw = d->kv_heads * d->qk, vw = d->kv_heads * d->vd;
    s->k8 = calloc((size_t)L * cap * kw, 1);
    s->v8 = calloc((size_t)L * cap * vw, 1);
    s->ks = calloc((size_t)L * cap * d->kv_heads, sizeof(float));
    s->vs = calloc((size_t)L * cap * d->kv_heads, sizeof(float));
    int th = d->taps > 1 ? d->taps - 1 : 1;
    s->qh = calloc((size_t)L * th * d->heads * d->qk, sizeof(float));
    s->kh = calloc((size_t)L * th * kw, sizeof(float));
    s->vh = calloc((size_t)L * th * vw, sizeof(float));
    int sites = d->n_sites > 0 ? d->n_sites : 1;
    s->etoks = calloc((size_t)sites * (d->max_order > 1 ? d->max_order - 1 : 1), sizeof(int));
    int vr = (d->etaps > 1 ? d->etaps - 1 : 1) * d->max_order;
    s->evraw = calloc((size_t)sites * vr * d->dim, sizeof(float));
    int xkw = d->x_heads * d->x_qk, xvw = d->x_heads * d->x_vd;
    s->xk8 = calloc((size_t)L * frames * xkw, 1);
    s->xv8 = calloc((size_t)L * frames * xvw, 1);
    s->xks = calloc((size_t)L * frames * d->x_heads, sizeof(float));
    s->xvs = calloc((size_t)L * frames * d->x_heads, sizeof(float));
    return s;
}

void wo_dec_free(wo_dec_state *s) {
    if (!s) return;
    free(s->k8), free(s->v8), free(s->ks), free(s->vs), free(s->qh), free(s->kh), free(s->vh);
    free(s->etoks), free(s->evraw), free(s->xk8), free(s->xv8), free(s->xks), free(s->xvs);
    free(s);
}

int wo_dec_len(const wo_dec_state *s) { return s->n; }

/* decoder.go:223 State.Fork: a state with s's positions that extends
 * independently of s. The reference shares the rows so far and copies on
 * the next append; here the copy is made at once. */
wo_dec_state *wo_dec_fork(const wo_decoder *d, const wo_dec_state *s) {
    wo_dec_state *f = wo_dec_new(d, s->cap, s->frames);
    int L = d->layers, kw = d->kv_heads * d->qk, vw = d->kv_heads * d->vd;
    size_t cap = (size_t)s->cap, fr = (size_t)s->frames;
    memcpy(f->k8, s->k8, (size_t)L * cap * kw);
    memcpy(f->v8, s->v8, (size_t)L * cap * vw);
    memcpy(f->ks, s->ks, (size_t)L * cap * d->kv_heads * sizeof(float));
    memcpy(f->vs, s->vs, (size_t)L * cap * d->kv_heads * sizeof(float));
    int th = d->taps > 1 ? d->taps - 1 : 1;
    memcpy(f->qh, s->qh, (size_t)L * th * d->heads * d->qk * sizeof(float));
    memcpy(f->kh, s->kh, (size_t)L * th * kw * sizeof(float));
    memcpy(f->vh, s->vh, (size_t)L * th * vw * sizeof(float));
    int sites = d->n_sites > 0 ? d->n_sites : 1;
    memcpy(f->etoks, s->etoks, (size_t)sites * (d->max_order > 1 ? d->max_order - 1 : 1) * sizeof(int));
    int vr = (d->etaps > 1 ? d->etaps - 1 : 1) * d->max_order;
    memcpy(f->evraw, s->evraw, (size_t)sites * vr * d->dim * sizeof(float));
    int xkw = d->x_heads * d->x_qk, xvw = d->x_heads * d->x_vd;
    memcpy(f->xk8, s->xk8, (size_t)L * fr * xkw);
    memcpy(f->xv8, s->xv8, (size_t)L * fr * xvw);
    memcpy(f->xks, s->xks, (size_t)L * fr * d->x_heads * sizeof(float));
    memcpy(f->xvs, s->xvs, (size_t)L * fr * d->x_heads * sizeof(float));
    f->n = s->n, f->nh = s->nh, f->ntoks = s->ntoks, f->nvraw = s->nvraw;
    return f;
}

/* The int8 memory of layer l (for the tests): k8 [frames][x_heads·x_qk],
 * ks [frames][x_heads], v8, vs. */
void wo_dec_memory_of(const wo_decoder *d, const wo_dec_state *s, int l, const int8_t **k8, const float **ks,
                      const int8_t **v8, const float **vs) {
    size_t f = (size_t)s->frames;
    *k8 = s->xk8 + (size_t)l * f * d->x_heads * d->x_qk;
    *v8 = s->xv8 + (size_t)l * f * d->x_heads * d->x_vd;
    *ks = s->xks + (size_t)l * f * d->x_heads;
    *vs = s->xvs + (size_t)l * f * d->x_heads;
}

/* decoder.go:157 Memory -> cross.go:181 project for every layer (no RoPE:
 * CrossRopeNone; QKNormZC; Int8.KV): k, v = ApplyShared(k_proj, v_proj)
 * over the frames, the k norm per head, QuantizeRows per head. Resets the
 * sequence (NewState). */
void wo_dec_memory(const wo_decoder *d, wo_dec_state *s, const float *enc, int frames) {
    int kw = d->x_heads * d->x_qk, vw = d->x_heads * d->x_vd;
    float *k = malloc((size_t)frames * kw * sizeof(float)), *v = malloc((size_t)frames * vw * sizeof(float));
    for (int l = 0; l < d->layers; l++) {
        const wo_dec_layer *L = &d->layer[l];
        wo_packed ms[2] = {L->x_k_proj, L->x_v_proj};
        float *ys[2] = {k, v};
        wo_cq_gemms_lut(ms, 2, enc, frames, ys);
        zc_norm(k, k, frames * d->x_heads, d->x_qk, L->x_k_norm);
        size_t f = (size_t)frames;
        wo_quantize_rows(k, frames, kw, d->x_qk, s->xk8 + (size_t)l * f * kw, s->xks + (size_t)l * f * d->x_heads);
        wo_quantize_rows(v, frames, vw, d->x_vd, s->xv8 + (size_t)l * f * vw, s->xvs + (size_t)l * f * d->x_heads);
    }
    free(k), free(v);
    s->frames = frames;
    s->n = 0;
    s->nh = 0;
    s->ntoks = 0;
    s->nvraw = 0;
}

/* engram.go:141 ngramHash of table c over the history hist[0..len). */
static uint32_t ngram_hash(int c, int order, const int *hist, int len) {
    uint32_t acc = 0x9E3779B9u * (uint32_t)(c + 1);
    for (int j = 0; j < order; j++) {
        uint32_t tok = j < len ? (uint32_t)hist[len - 1 - j] : 0u;
        acc = (acc ^ tok) * 0x01000193u;
    }
    return acc ^ (acc >> 15);
}

/* cache.go:166 Engram.Extend for one token: keys k and values v [dim] of
 * site i, and the site's cache advanced (tokens and raw values). The
 * history is updated by the caller once every site has read it. */
static void engram_extend(const wo_decoder *d, wo_dec_state *s, int i, int tok, float *k, float *v) {
    const wo_engram_site *e = &d->site[i];
    int nt = d->n_tables, w = nt * d->sub, keep_t = d->max_order - 1;
    int hist[16];
    int h = s->ntoks;
    for (int j = 0; j < h; j++) hist[j] = s->etoks[(size_t)i * keep_t + j];
    hist[h] = tok;
    float *emb = calloc((size_t)w, sizeof(float));
    int pos = s->n;
    int from = h + 1 - d->max_order > 0 ? h + 1 - d->max_order : 0;
    for (int c = 0; c < nt; c++) {
        int order = d->orders[c];
        if (pos + 1 < order) continue; /* fetched · ngram_ok */
        uint32_t idx = ngram_hash(c, order, hist + from, h + 1 - from) % (uint32_t)d->slots;
        wo_cq_row(&e->tables, c * d->slots + (int)idx, emb + (size_t)c * d->sub);
    }
    float *vraw = malloc((size_t)d->dim * sizeof(float));
    wo_packed ms[2] = {e->key_proj, e->value_proj};
    float *ys[2] = {k, vraw};
    gemms1(ms, 2, emb, ys);
    /* attention.go:588 applyTaps with dilation max_order, last row only:
     * all = the cached raw rows (oldest first), then vraw. */
    int rh = s->nvraw, dil = d->max_order, vr = (d->etaps - 1) * dil;
    float *all = malloc((size_t)(rh + 1) * d->dim * sizeof(float));
    memcpy(all, s->evraw + (size_t)i * vr * d->dim, (size_t)rh * d->dim * sizeof(float));
    memcpy(all + (size_t)rh * d->dim, vraw, (size_t)d->dim * sizeof(float));
    for (int c = 0; c < d->dim; c++) v[c] = 0.0f;
    for (int j = 0; j < d->etaps; j++) {
        int src = rh - dil * j;
        if (src < 0) break;
        const float *tap = e->taps + (size_t)j * d->dim;
        for (int c = 0; c < d->dim; c++) {
            float t = tap[c] * all[(size_t)src * d->dim + c];
            v[c] += t;
        }
    }
    int keep = rh + 1 < vr ? rh + 1 : vr;
    memcpy(s->evraw + (size_t)i * vr * d->dim, all + (size_t)(rh + 1 - keep) * d->dim,
           (size_t)keep * d->dim * sizeof(float));
    free(all), free(vraw), free(emb);
}

/* attention.go:588 applyTaps (dilation 1) for the newest row of t raw rows
 * held as history hist (h rows, oldest first) plus z: out = Σ_j taps[j] ·
 * row(newest − j), j ascending, from 0. */
static void taps_last(float *out, const float *hist, int h, const float *z, const float *taps, int ntaps,
                      int width) {
    for (int c = 0; c < width; c++) out[c] = 0.0f;
    for (int j = 0; j < ntaps; j++) {
        if (j > h) break;
        const float *src = j == 0 ? z : hist + (size_t)(h - j) * width;
        const float *tap = taps + (size_t)j * width;
        for (int c = 0; c < width; c++) {
            float t = tap[c] * src[c];
            out[c] += t;
        }
    }
}

/* cache.go:185 extendTaps' history: keep the last taps − 1 raw rows. */
static void push_hist(float *hist, int h, const float *z, int keep, int width) {
    if (keep <= 0) return;
    if (h < keep) {
        memcpy(hist + (size_t)h * width, z, (size_t)width * sizeof(float));
        return;
    }
    memmove(hist, hist + width, (size_t)(keep - 1) * width * sizeof(float));
    memcpy(hist + (size_t)(keep - 1) * width, z, (size_t)width * sizeof(float));
}

/* hadamard.go:300 kronApply + :281 mix for stage st (a permutation after
 * stages 0 and 1). */
static void hada_mix(const wo_decoder *d, const wo_dec_layer *L, float *dst, const float *z, int st) {
    int na = d->na, nb = d->nb, n = na * nb;
    const float *a = L->hada_w[st][0], *b = L->hada_w[st][1];
    float *aT = malloc((size_t)na * na * sizeof(float)), *bT = malloc((size_t)nb * nb * sizeof(float));
    for (int i = 0; i < na; i++)
        for (int j = 0; j < na; j++) aT[j * na + i] = a[i * na + j];
    for (int i = 0; i < nb; i++)
        for (int j = 0; j < nb; j++) bT[j * nb + i] = b[i * nb + j];
    float *yT = malloc((size_t)n * sizeof(float)), *k = malloc((size_t)n * sizeof(float));
    matmul_tb(yT, na, bT, z, nb, na, nb);
    float *out = st == 2 ? dst : k;
    matmul_tb(out, nb, aT, yT, na, nb, na);
    if (st < 2) {
        const int *p = st == 0 ? d->hada_p1 : d->hada_p2;
        for (int i = 0; i < n; i++) dst[i] = k[p[i]];
    }
    free(aT), free(bT), free(yT), free(k);
}

/* hadamard.go:196 HadamardMLP.forward -> :211 rows for one row (dim = n). */
static void hadamard_mlp(const wo_decoder *d, const wo_dec_layer *L, const float *x, float *out) {
    int n = d->na * d->nb, dim = d->dim, rank = d->rank;
    float *logits = malloc((size_t)rank * sizeof(float));
    /* linear(logits, x, 1, condVT, rank, dim): condVT[r][c] = cond_v[c][r] */
    for (int r = 0; r < rank; r++) {
        float s = 0.0f;
        for (int c = 0; c < dim; c++) {
            float t = x[c] * L->cond_v[(size_t)c * rank + r];
            s += t;
        }
        logits[r] = s;
    }
    wo_softmax(logits, rank);
    float *cond = calloc((size_t)n, sizeof(float)), *z = malloc((size_t)n * sizeof(float));
    for (int r = 0; r < rank; r++) axpy(cond, logits[r], L->cond_u + (size_t)r * n, n);
    for (int c = 0; c < n; c++) cond[c] += 1.0f;
    for (int c = 0; c < dim; c++) z[c] = L->d1[c] * x[c];
    for (int c = dim; c < n; c++) z[c] = 0.0f;
    hada_mix(d, L, out, z, 0);
    for (int c = 0; c < n; c++) {
        float t = L->d2[c] * cond[c];
        float u = t * out[c];
        float a = u + L->b2[c];
        float sg = sigmoid(a);
        z[c] = a * sg;
    }
    hada_mix(d, L, out, z, 1);
    for (int c = 0; c < n; c++) z[c] = L->d3[c] * out[c];
    hada_mix(d, L, out, z, 2);
    for (int c = 0; c < n; c++) out[c] *= L->d4[c];
    free(logits), free(cond), free(z);
}

/* cache.go:78 Attention.Extend for one row u at position s->n of layer l,
 * with int8 KV (cache.go:120 extendInt8) and quantised queries: returns
 * the attention output y [dim]. */
static void self_attention(const wo_decoder *d, wo_dec_state *s, int l, const float *x, float *y) {
    const wo_dec_layer *L = &d->layer[l];
    int H = d->heads, KV = d->kv_heads, qk = d->qk, vd = d->vd;
    int qw = H * qk, kw = KV * qk, vw = KV * vd, ow = H * vd;
    float *q = malloc((size_t)qw * sizeof(float)), *k = malloc((size_t)kw * sizeof(float));
    float *v = malloc((size_t)vw * sizeof(float)), *gate = malloc((size_t)ow * sizeof(float));
    wo_packed ms[4] = {L->q_proj, L->k_proj, L->v_proj, L->gate_proj};
    float *ys[4] = {q, k, v, gate};
    gemms1(ms, 4, x, ys); /* attention.go:277 projections */
    int th = d->taps - 1, h = s->nh;
    float *qt = malloc((size_t)qw * sizeof(float)), *kt = malloc((size_t)kw * sizeof(float));
    float *vt = malloc((size_t)vw * sizeof(float));
    if (d->taps > 0) { /* cache.go:185 extendTaps */
        float *qh = s->qh + (size_t)l * th * qw, *kh = s->kh + (size_t)l * th * kw, *vh = s->vh + (size_t)l * th * vw;
        taps_last(qt, qh, h, q, L->q_taps, d->taps, qw);
        taps_last(kt, kh, h, k, L->k_taps, d->taps, kw);
        taps_last(vt, vh, h, v, L->v_taps, d->taps, vw);
        push_hist(qh, h, q, th, qw);
        push_hist(kh, h, k, th, kw);
        push_hist(vh, h, v, th, vw);
    } else {
        memcpy(qt, q, (size_t)qw * sizeof(float));
        memcpy(kt, k, (size_t)kw * sizeof(float));
        memcpy(vt, v, (size_t)vw * sizeof(float));
    }
    /* attention.go:300 normRotate at position s->n */
    zc_norm(qt, qt, H, qk, L->q_norm);
    zc_norm(kt, kt, KV, qk, L->k_norm);
    int half = qk / 2, pos = s->n;
    const float *cs = d->rope_cos + (size_t)pos * half, *sn = d->rope_sin + (size_t)pos * half;
    for (int hd = 0; hd < H; hd++) rope_apply(qt + (size_t)hd * qk, half, cs, sn);
    for (int hd = 0; hd < KV; hd++) rope_apply(kt + (size_t)hd * qk, half, cs, sn);
    /* cache.go:125 Int8Rows.Append of the new key and value row */
    size_t cap = (size_t)s->cap;
    int8_t *k8 = s->k8 + (size_t)l * cap * kw, *v8 = s->v8 + (size_t)l * cap * vw;
    float *ks = s->ks + (size_t)l * cap * KV, *vs = s->vs + (size_t)l * cap * KV;
    wo_quantize_rows(kt, 1, kw, qk, k8 + (size_t)pos * kw, ks + (size_t)pos * KV);
    wo_quantize_rows(vt, 1, vw, vd, v8 + (size_t)pos * vw, vs + (size_t)pos * KV);
    /* cache.go:129 AttendInt8Spans over keys 0 .. pos (attention.go:424 keySpans, causal) */
    int32_t sp[4] = {0, 0, 0, pos + 1};
    float *att = malloc((size_t)ow * sizeof(float));
    float scale = (float)sqrt((double)qk); /* attention.go:407 attendScale */
    wo_attend_int8_spans(qt, 1, H, k8, ks, v8, vs, pos + 1, KV, qk, vd, sp, scale, 1, NULL, att);
    /* attention.go:243 output: σ(gate) ⊙ out, then out_proj */
    for (int i = 0; i < ow; i++) {
        gate[i] = sigmoid(gate[i]);
        att[i] *= gate[i];
    }
    gemm1(&L->out_proj, att, y);
    free(q), free(k), free(v), free(gate), free(qt), free(kt), free(vt), free(att);
}

/* cross.go:209 branch (Best(): QKNormZC, GateSigmoid, ResSigmoid, no RoPE)
 * against the int8 memory (cross.go:273 attend, needle.AttendInt8 with
 * quantised queries), added to h. */
static void cross_branch(const wo_decoder *d, const wo_dec_state *s, int l, float *h) {
    const wo_dec_layer *L = &d->layer[l];
    int H = d->x_heads, qk = d->x_qk, vd = d->x_vd, dim = d->dim;
    float *x = malloc((size_t)dim * sizeof(float)), *q = malloc((size_t)H * qk * sizeof(float));
    float *gate = malloc((size_t)H * vd * sizeof(float)), *out = malloc((size_t)H * vd * sizeof(float));
    float *y = malloc((size_t)dim * sizeof(float));
    zc_norm(x, h, 1, dim, L->x_norm_in);
    gemm1(&L->x_q_proj, x, q);
    zc_norm(q, q, H, qk, L->x_q_norm);
    const int8_t *k8, *v8;
    const float *ks, *vs;
    wo_dec_memory_of(d, s, l, &k8, &ks, &v8, &vs);
    int32_t sp[4] = {0, 0, 0, s->frames};
    float scale = (float)sqrt((double)qk);
    wo_attend_int8_spans(q, 1, H, k8, ks, v8, vs, s->frames, H, qk, vd, sp, scale, 1, NULL, out);
    gemm1(&L->x_gate_proj, x, gate);
    for (int i = 0; i < H * vd; i++) {
        gate[i] = sigmoid(gate[i]);
        out[i] *= gate[i];
    }
    gemm1(&L->x_out_proj, out, y);
    zc_norm(y, y, 1, dim, L->x_post_norm);
    float resid = sigmoid(L->x_attn_gate); /* cross.go:148 setResidual */
    for (int i = 0; i < dim; i++) y[i] = resid * y[i];
    for (int i = 0; i < dim; i++) h[i] += y[i];
    free(x), free(q), free(gate), free(out), free(y);
}

/* decoder.go:446 layer l: mhc.go:182 MHC.forward around block.go:117
 * Block.Extend with the cross-attention at AfterAttn (CrossAfterAttn). */
static void layer_step(const wo_decoder *d, wo_dec_state *s, int l, float *stream, const float *ek,
                       const float *ev) {
    const wo_dec_layer *L = &d->layer[l];
    int n = d->lanes, c = d->dim, nC = n * c;
    /* mhc.go:193 nx = RMSUnit(stream); :241 logits (φ with int8 input) */
    float *nx = malloc((size_t)nC * sizeof(float));
    rms_unit(nx, stream, 1, nC);
    fake_quant(nx, nx, nC, nC); /* linear.go:108 ApplyShared's shared quantised copy */
    float pre[16], post[16], res[64];
    wo_packed ms[3] = {L->phi_pre, L->phi_post, L->phi_res};
    float *ys[3] = {pre, post, res};
    gemms1(ms, 3, nx, ys);
    for (int k = 0; k < n; k++) {
        float t = L->a_pre * pre[k];
        pre[k] = t + L->b_pre[k] + (k == l % n ? 4.0f : -4.0f); /* laneOffsets: pre_off */
        float t2 = L->a_post * post[k];
        post[k] = t2 + L->b_post[k] + (k == l % n ? 0.0f : -4.0f); /* post_off */
    }
    for (int k = 0; k < n * n; k++) {
        float t = L->a_res * res[k];
        res[k] = t + L->b_res[k];
    }
    float *u = calloc((size_t)c, sizeof(float));
    for (int k = 0; k < n; k++) {
        pre[k] = sigmoid(pre[k]);
        axpy(u, pre[k], stream + (size_t)k * c, c);
        post[k] = 2.0f * sigmoid(post[k]);
    }
    sinkhorn(res, n);
    /* block.go:148 run */
    float *hb = malloc((size_t)c * sizeof(float));
    memcpy(hb, u, (size_t)c * sizeof(float));
    if (ek) { /* block.go:231 applyEngram */
        float *ux = malloc((size_t)c * sizeof(float)), *uk = malloc((size_t)c * sizeof(float));
        float scale = (float)sqrt((double)c);
        rms_unit(ux, hb, 1, c);
        rms_unit(uk, ek, 1, c);
        float dp = dot(ux, uk, c);
        float a = sigmoid(dp / scale);
        for (int i = 0; i < c; i++) {
            float t = a * ev[i];
            hb[i] += t;
        }
        free(ux), free(uk);
    }
    float *nrm = malloc((size_t)c * sizeof(float)), *a = malloc((size_t)c * sizeof(float));
    zc_norm(nrm, hb, 1, c, L->norm_in);
    self_attention(d, s, l, nrm, a);
    zc_norm(a, a, 1, c, L->post_norm);
    float g = sigmoid(L->attn_gate); /* block.go:60 */
    for (int i = 0; i < c; i++) {
        float t = g * a[i];
        hb[i] += t;
    }
    cross_branch(d, s, l, hb);
    float *p = malloc((size_t)c * sizeof(float)), *m = malloc((size_t)c * sizeof(float));
    zc_norm(p, hb, 1, c, L->pre_hada);
    hadamard_mlp(d, L, p, m);
    for (int i = 0; i < c; i++) m[i] += hb[i];
    /* mhc.go:229 y = block(u) − u; :270 mix */
    float *y = malloc((size_t)c * sizeof(float)), *out = calloc((size_t)nC, sizeof(float));
    for (int i = 0; i < c; i++) y[i] = m[i] - u[i];
    for (int aa = 0; aa < n; aa++) {
        float *o = out + (size_t)aa * c;
        for (int b = 0; b < n; b++) axpy(o, res[aa * n + b], stream + (size_t)b * c, c);
        float hp = post[aa];
        for (int k = 0; k < c; k++) {
            float t = hp * y[k];
            o[k] += t;
        }
    }
    memcpy(stream, out, (size_t)nC * sizeof(float));
    free(nx), free(u), free(hb), free(nrm), free(a), free(p), free(m), free(y), free(out);
}

/* decoder.go:252 Extend for one token: the logits [vocab] of the next
 * token (decoder.go:508 logits: lane mean, final norm, the tied head).
 * Returns -1 for a token out of range or a full cache, else 0. */
int wo_dec_extend(const wo_decoder *d, wo_dec_state *s, int tok, float *logits) {
    if (tok < 0 || tok >= d->vocab || s->n >= s->cap || s->n >= d->rope_len) return -1;
    int c = d->dim, n = d->lanes;
    float *x = malloc((size_t)c * sizeof(float));
    wo_cq_row(&d->embedding, tok, x);
    float scale = (float)sqrt((double)c); /* ScaleSqrtDim */
    for (int i = 0; i < c; i++) x[i] = x[i] * scale;
    int sites = d->n_sites;
    float *ek = malloc((size_t)(sites > 0 ? sites : 1) * c * sizeof(float));
    float *ev = malloc((size_t)(sites > 0 ? sites : 1) * c * sizeof(float));
    for (int i = 0; i < sites; i++) engram_extend(d, s, i, tok, ek + (size_t)i * c, ev + (size_t)i * c);
    /* the engram caches' token history and raw-value count, once for all sites */
    if (sites > 0) {
        int keep_t = d->max_order - 1, h = s->ntoks;
        for (int i = 0; i < sites; i++) {
            int *t = s->etoks + (size_t)i * keep_t;
            if (keep_t <= 0) continue;
            if (h < keep_t) {
                t[h] = tok;
            } else {
                memmove(t, t + 1, (size_t)(keep_t - 1) * sizeof(int));
                t[keep_t - 1] = tok;
            }
        }
        if (h < keep_t) s->ntoks = h + 1;
        int vr = (d->etaps - 1) * d->max_order;
        if (s->nvraw < vr) s->nvraw++;
    }
    float *stream = malloc((size_t)n * c * sizeof(float));
    for (int k = 0; k < n; k++) memcpy(stream + (size_t)k * c, x, (size_t)c * sizeof(float)); /* ExpandLanes */
    for (int l = 0; l < d->layers; l++) {
        int site = -1;
        for (int i = 0; i < sites; i++)
            if (d->site[i].layer == l) site = i;
        layer_step(d, s, l, stream, site >= 0 ? ek + (size_t)site * c : NULL,
                   site >= 0 ? ev + (size_t)site * c : NULL);
    }
    if (s->nh < d->taps - 1) s->nh++;
    s->n++;
    /* mhc.go:140 CollapseLanes */
    float *mean = calloc((size_t)c, sizeof(float));
    for (int k = 0; k < n; k++)
        for (int i = 0; i < c; i++) mean[i] += stream[(size_t)k * c + i];
    for (int i = 0; i < c; i++) mean[i] /= (float)n;
    zc_norm(mean, mean, 1, c, d->final_norm); /* FinalNormOn */
    gemm1(&d->embedding, mean, logits);       /* HeadTied: head = 1 */
    free(x), free(ek), free(ev), free(stream), free(mean);
    return 0;
}

/* greedy.go:182 argmax. */
static int argmax(const float *v, int n) {
    int best = 0;
    for (int i = 0; i < n; i++)
        if (v[i] > v[best]) best = i;
    return best;
}

/* The gap between the largest logit and the next one (the greedy choice's
 * margin). */
static float top2_margin(const float *v, int n) {
    int b = argmax(v, n);
    float second = -INFINITY;
    for (int i = 0; i < n; i++)
        if (i != b && v[i] > second) second = v[i];
    return v[b] - second;
}

/* greedy.go:40 GreedyMemory on the state's memory with the language
 * detected (greedy.go:81 language over langs, the first on ties): the
 * prompt [bos], the language token, then argmax tokens until eos or
 * max_tok − 1 steps. tokens [max_tok] receives the text tokens (without
 * the language token and eos); returns their count, *lang the language
 * token, *eos_hit whether decoding stopped at eos. margins (or NULL)
 * [max_tok] receives each step's top-2 gap (step 0: the language step
 * among the language tokens). Returns -1 on an error. */
int wo_dec_greedy(const wo_decoder *d, wo_dec_state *s, int bos, const int *langs, int nlangs, int eos,
                  int max_tok, int *tokens, int *lang, int *eos_hit, float *margins) {
    float *logits = malloc((size_t)d->vocab * sizeof(float));
    int count = 0;
    *eos_hit = 0;
    if (wo_dec_extend(d, s, bos, logits) != 0) {
        free(logits);
        return -1;
    }
    int best = 0;
    for (int i = 1; i < nlangs; i++)
        if (logits[langs[i]] > logits[langs[best]]) best = i;
    if (margins) {
        float second = -INFINITY;
        for (int i = 0; i < nlangs; i++)
            if (i != best && logits[langs[i]] > second) second = logits[langs[i]];
        margins[0] = nlangs > 1 ? logits[langs[best]] - second : INFINITY;
    }
    int next = langs[best];
    *lang = next;
    for (int step = 0; step < max_tok - 1; step++) {
        if (wo_dec_extend(d, s, next, logits) != 0) {
            free(logits);
            return -1;
        }
        next = argmax(logits, d->vocab);
        if (margins) margins[step + 1] = top2_margin(logits, d->vocab);
        if (next == eos) {
            *eos_hit = 1;
            break;
        }
        tokens[count++] = next;
    }
    free(logits);
    return count;
}

/* Many independent streams, each its own GreedyMemory on its own memory
 * (enc [streams][frames][dim]), one stream per task on `threads` OS
 * threads: the CPU baseline of the device decoder. tokens [streams][max_tok],
 * counts/langs/eos [streams]. */
typedef struct {
    const wo_decoder *d;
    const float *enc;
    int frames, bos, nlangs, eos, max_tok;
    const int *langs;
    int *tokens, *counts, *lang, *eos_hit;
} greedy_job;

static void greedy_task(int b, void *arg) {
    const greedy_job *j = arg;
    wo_dec_state *s = wo_dec_new(j->d, j->max_tok + 1, j->frames);
    wo_dec_memory(j->d, s, j->enc + (size_t)b * j->frames * j->d->dim, j->frames);
    j->counts[b] = wo_dec_greedy(j->d, s, j->bos, j->langs, j->nlangs, j->eos, j->max_tok,
                                 j->tokens + (size_t)b * j->max_tok, &j->lang[b], &j->eos_hit[b], NULL);
    wo_dec_free(s);
}

void wo_dec_greedy_streams_mt(const wo_decoder *d, int streams, const float *enc, int frames, int bos,
                              const int *langs, int nlangs, int eos, int max_tok, int *tokens, int *counts,
                              int *lang, int *eos_hit, int threads) {
    greedy_job job = {d, enc, frames, bos, nlangs, eos, max_tok, langs, tokens, counts, lang, eos_hit};
    wo_parallel_for(streams, threads < 1 ? 1 : threads, greedy_task, &job);
}

/* The pieces alone, for the known-answer pins (tests/test_oracle_pins.py). */
uint32_t wo_ngram_hash(int c, int order, const int *hist, int len) { return ngram_hash(c, order, hist, len); }
void wo_zc_norm(float *dst, const float *x, int rows, int d, const float *scale) { zc_norm(dst, x, rows, d, scale); }
void wo_rms_unit(float *dst, const float *x, int rows, int d) { rms_unit(dst, x, rows, d); }
void wo_rope_apply(float *x, int half, const float *cs, const float *sn) { rope_apply(x, half, cs, sn); }
void wo_sinkhorn_iters(float *k, int n, int iters) {
    if (!sinkhorn_exp(k, n, iters)) sinkhorn_log(k, n, iters);
}

/* The CPU baseline in two phases, so that the decode rate excludes the
 * memory projection (the reference's decode rate starts after the first
 * text token; whistle/strategy.go:33 clock): the memories of many streams
 * on threads, then their greedy decodes on threads. */
typedef struct {
    const wo_decoder *d;
    wo_dec_state **st;
    const float *enc;
    int frames, cap;
} states_job;

static void states_task(int b, void *arg) {
    const states_job *j = arg;
    j->st[b] = wo_dec_new(j->d, j->cap, j->frames);
    wo_dec_memory(j->d, j->st[b], j->enc + (size_t)b * j->frames * j->d->dim, j->frames);
}

wo_dec_state **wo_dec_states_mt(const wo_decoder *d, int streams, const float *enc, int frames, int cap, int threads) {
    wo_dec_state **st = calloc((size_t)(streams > 0 ? streams : 1), sizeof *st);
    states_job job = {d, st, enc, frames, cap};
    wo_parallel_for(streams, threads < 1 ? 1 : threads, states_task, &job);
    return st;
}

void wo_dec_states_free(wo_dec_state **st, int streams) {
    if (!st) return;
    for (int b = 0; b < streams; b++) wo_dec_free(st[b]);
    free(st);
}

typedef struct {
    const wo_decoder *d;
    wo_dec_state **st;
    int bos, nlangs, eos, max_tok;
    const int *langs;
    int *tokens, *counts, *lang, *eos_hit;
} greedy_states_job;

static void greedy_states_task(int b, void *arg) {
    const greedy_states_job *j = arg;
    j->counts[b] = wo_dec_greedy(j->d, j->st[b], j->bos, j->langs, j->nlangs, j->eos, j->max_tok,
                                 j->tokens + (size_t)b * j->max_tok, &j->lang[b], &j->eos_hit[b], NULL);
}

void wo_dec_greedy_states_mt(const wo_decoder *d, wo_dec_state **st, int streams, int bos, const int *langs,
                             int nlangs, int eos, int max_tok, int *tokens, int *counts, int *lang, int *eos_hit,
                             int threads) {
    greedy_states_job job = {d, st, bos, nlangs, eos, max_tok, langs, tokens, counts, lang, eos_hit};
    wo_parallel_for(streams, threads < 1 ? 1 : threads, greedy_states_task, &job);
}

/* ------------------------------------------------------------------ encoder */

/* internal/encoder/stem.go:367 applyAct, ActSiLU: v·σ(v) (stem.go:393
 * sigmoid in float64). */
void wo_silu(float *x, int n) {
    for (int i = 0; i < n; i++) x[i] = x[i] * sigmoid(x[i]);
}

/* block.go:257 gated, GLUValueGate: o[k] = a[k]·σ(g[k]) with a, g the two
 * halves of a row of pw1's output. */
void wo_enc_glu(const float *p, int t, int half, float *out) {
    for (int i = 0; i < t; i++) {
        const float *a = p + (size_t)i * 2 * half, *g = a + half;
        for (int k = 0; k < half; k++) out[(size_t)i * half + k] = a[k] * sigmoid(g[k]);
    }
}

/* block.go:290 depthwise, DWCentred: out[i][c] = Σ_j dw[j][c]·x[i − pad + j][c]
 * over the frames inside the clip, j ascending, from 0, pad = (k − 1)/2. */
void wo_enc_depthwise(const float *x, int t, int h, const float *dw, int k, float *out) {
    int pad = (k - 1) / 2;
    memset(out, 0, (size_t)t * h * sizeof(float));
    for (int i = 0; i < t; i++)
        for (int j = 0; j < k; j++) {
            int src = i - pad + j;
            if (src < 0 || src >= t) continue;
            for (int c = 0; c < h; c++) {
                float tt = dw[(size_t)j * h + c] * x[(size_t)src * h + c];
                out[(size_t)i * h + c] += tt;
            }
        }
}

/* block.go:172 ffn: x += 1/2 · mlp(norm(x)) per row (FFNHalf; the product
 * is exact). */
static void enc_ffn(const wo_decoder *d, const wo_dec_layer *H, const float *norm, float *x, int t) {
    int c = d->dim;
    float *n = malloc((size_t)c * sizeof(float)), *m = malloc((size_t)c * sizeof(float));
    for (int i = 0; i < t; i++) {
        float *row = x + (size_t)i * c;
        zc_norm(n, row, 1, c, norm);
        hadamard_mlp(d, H, n, m);
        for (int k = 0; k < c; k++) {
            float tt = 0.5f * m[k];
            row[k] += tt;
        }
    }
    free(n), free(m);
}

/* attention.go:226 forward with MaskNone and RoPE at positions 0 … t − 1
 * over the t rows x of one clip, with Int8{Act, KV}: the projections
 * (:262, one shared input), the per-head q/k norms and RoPE (:300
 * normRotate), quantQKV (:342), attend (:360) and output (:242). form
 * WO_ENC_ATTEND_FLOAT restates attendGEMM (:480): logits Σ q̃·k̃ over the
 * fake-quantised values in index order, ÷ √qk, softmaxInPlace, then
 * Σ_j p_j·ṽ_j in key order; WO_ENC_ATTEND_INT8 runs AttendInt8Spans on the
 * same int8 codes (integer logits, the device kernel's exact order). */
static void enc_attention(const wo_encoder *e, const wo_dec_layer *L, const float *x, int t, int form, float *y) {
    const wo_decoder *d = &e->d;
    int H = d->heads, KV = d->kv_heads, qk = d->qk, vd = d->vd;
    int qw = H * qk, kw = KV * qk, vw = KV * vd, ow = H * vd, half = qk / 2;
    float *q = malloc((size_t)t * qw * sizeof(float)), *k = malloc((size_t)t * kw * sizeof(float));
    float *v = malloc((size_t)t * vw * sizeof(float)), *gate = malloc((size_t)t * ow * sizeof(float));
    float *att = calloc((size_t)t * ow, sizeof(float));
    wo_packed ms[4] = {L->q_proj, L->k_proj, L->v_proj, L->gate_proj};
    float *ys[4] = {q, k, v, gate};
    wo_cq_gemms_lut(ms, 4, x, t, ys);
    zc_norm(q, q, t * H, qk, L->q_norm);
    zc_norm(k, k, t * KV, qk, L->k_norm);
    for (int i = 0; i < t; i++) {
        const float *cs = d->rope_cos + (size_t)i * half, *sn = d->rope_sin + (size_t)i * half;
        for (int h = 0; h < H; h++) rope_apply(q + ((size_t)i * H + h) * qk, half, cs, sn);
        for (int h = 0; h < KV; h++) rope_apply(k + ((size_t)i * KV + h) * qk, half, cs, sn);
    }
    float scale = (float)sqrt((double)qk); /* attention.go:407 attendScale */
    if (form == WO_ENC_ATTEND_FLOAT) {
        fake_quant(q, q, t * qw, qk);
        fake_quant(k, k, t * kw, qk);
        fake_quant(v, v, t * vw, vd);
        float *row = malloc((size_t)t * sizeof(float));
        for (int h = 0; h < H; h++) {
            int kv = h / (H / KV); /* attention.go:191 kvHead */
            for (int i = 0; i < t; i++) {
                const float *qi = q + (size_t)i * qw + (size_t)h * qk;
                for (int j = 0; j < t; j++) row[j] = dot(qi, k + (size_t)j * kw + (size_t)kv * qk, qk);
                for (int j = 0; j < t; j++) row[j] /= scale; /* attention.go:587 softmaxSpans */
                wo_softmax(row, t);
                float *o = att + (size_t)i * ow + (size_t)h * vd;
                for (int dd = 0; dd < vd; dd++) {
                    float s = 0.0f;
                    for (int j = 0; j < t; j++) {
                        float tt = row[j] * v[(size_t)j * vw + (size_t)kv * vd + dd];
                        s += tt;
                    }
                    o[dd] = s;
                }
            }
        }
        free(row);
    } else {
        int8_t *k8 = malloc((size_t)t * kw), *v8 = malloc((size_t)t * vw);
        float *ks = malloc((size_t)t * KV * sizeof(float)), *vs = malloc((size_t)t * KV * sizeof(float));
        int32_t *sp = malloc((size_t)t * 4 * sizeof(int32_t));
        wo_quantize_rows(k, t, kw, qk, k8, ks);
        wo_quantize_rows(v, t, vw, vd, v8, vs);
        for (int i = 0; i < t; i++) sp[4 * i] = sp[4 * i + 1] = sp[4 * i + 2] = 0, sp[4 * i + 3] = t;
        wo_attend_int8_spans(q, t, H, k8, ks, v8, vs, t, KV, qk, vd, sp, scale, 1, NULL, att);
        free(k8), free(v8), free(ks), free(vs), free(sp);
    }
    for (size_t i = 0; i < (size_t)t * ow; i++) {
        gate[i] = sigmoid(gate[i]);
        att[i] *= gate[i];
    }
    wo_cq_gemm_lut(&L->out_proj, att, t, y);
    free(q), free(k), free(v), free(gate), free(att);
}

/* block.go:224 conv: x += pw2(SiLU(conv_out_norm(depthwise(glu(pw1(
 * conv_norm(x))))))) (NormBeforeAct). */
static void enc_conv(const wo_encoder *e, const wo_enc_layer *EL, float *x, int t) {
    int c = e->d.dim;
    float *n = malloc((size_t)t * c * sizeof(float)), *p = malloc((size_t)t * 2 * c * sizeof(float));
    float *g = malloc((size_t)t * c * sizeof(float)), *dw = malloc((size_t)t * c * sizeof(float));
    zc_norm(n, x, t, c, EL->conv_norm);
    wo_cq_gemm_lut(&EL->pw1, n, t, p);
    wo_enc_glu(p, t, c, g);
    wo_enc_depthwise(g, t, c, EL->dw, e->dw_k, dw);
    zc_norm(dw, dw, t, c, EL->conv_out_norm);
    wo_silu(dw, t * c);
    wo_cq_gemm_lut(&EL->pw2, dw, t, n);
    for (size_t i = 0; i < (size_t)t * c; i++) x[i] += n[i];
    free(n), free(p), free(g), free(dw);
}

/* mhc.go:182 MHC.forward of encoder layer l around block.go:148 forward
 * (FFN1, attention, conv module, FFN2: OrderMacaron) on t rows. */
static void enc_layer(const wo_encoder *e, int l, float *stream, int t, int form) {
    const wo_decoder *d = &e->d;
    const wo_enc_layer *EL = &e->layer[l];
    const wo_dec_layer *L = &EL->b;
    int n = d->lanes, c = d->dim, nC = n * c;
    float *nx = malloc((size_t)t * nC * sizeof(float));
    rms_unit(nx, stream, t, nC);
    fake_quant(nx, nx, t * nC, nC); /* linear.go:108 ApplyShared's quantised copy */
    float *pre = malloc((size_t)t * n * sizeof(float)), *post = malloc((size_t)t * n * sizeof(float));
    float *res = malloc((size_t)t * n * n * sizeof(float));
    wo_packed ms[3] = {L->phi_pre, L->phi_post, L->phi_res};
    float *ys[3] = {pre, post, res};
    wo_cq_gemms_lut(ms, 3, nx, t, ys);
    float *u = calloc((size_t)t * c, sizeof(float));
    for (int i = 0; i < t; i++) { /* mhc.go:241 logits, :205-221 */
        float *pr = pre + (size_t)i * n, *po = post + (size_t)i * n, *rs = res + (size_t)i * n * n;
        for (int k = 0; k < n; k++) {
            float tt = L->a_pre * pr[k];
            pr[k] = tt + L->b_pre[k] + (k == l % n ? 4.0f : -4.0f);
            float t2 = L->a_post * po[k];
            po[k] = t2 + L->b_post[k] + (k == l % n ? 0.0f : -4.0f);
        }
        for (int k = 0; k < n * n; k++) {
            float tt = L->a_res * rs[k];
            rs[k] = tt + L->b_res[k];
        }
        for (int k = 0; k < n; k++) {
            pr[k] = sigmoid(pr[k]);
            axpy(u + (size_t)i * c, pr[k], stream + ((size_t)i * n + k) * c, c);
            po[k] = 2.0f * sigmoid(po[k]);
        }
        sinkhorn(rs, n);
    }
    /* block.go:148 forward */
    float *xb = malloc((size_t)t * c * sizeof(float)), *nrm = malloc((size_t)t * c * sizeof(float));
    float *a = malloc((size_t)t * c * sizeof(float));
    memcpy(xb, u, (size_t)t * c * sizeof(float));
    enc_ffn(d, &EL->hada0, EL->hada0.pre_hada, xb, t);
    zc_norm(nrm, xb, t, c, L->norm_in); /* block.go:193 attend */
    enc_attention(e, L, nrm, t, form, a);
    zc_norm(a, a, t, c, L->post_norm);
    float g = sigmoid(L->attn_gate); /* block.go:91 */
    for (size_t i = 0; i < (size_t)t * c; i++) {
        float tt = g * a[i];
        xb[i] += tt;
    }
    enc_conv(e, EL, xb, t);
    enc_ffn(d, L, L->pre_hada, xb, t);
    /* mhc.go:229 y = block(u) − u; :270 mix */
    float *out = calloc((size_t)t * nC, sizeof(float));
    for (int i = 0; i < t; i++) {
        float *y = xb + (size_t)i * c;
        const float *ui = u + (size_t)i * c, *st = stream + (size_t)i * nC, *rs = res + (size_t)i * n * n;
        for (int k = 0; k < c; k++) y[k] = y[k] - ui[k];
        for (int aa = 0; aa < n; aa++) {
            float *o = out + (size_t)i * nC + (size_t)aa * c;
            for (int b = 0; b < n; b++) axpy(o, rs[aa * n + b], st + (size_t)b * c, c);
            float hp = post[(size_t)i * n + aa];
            for (int k = 0; k < c; k++) {
                float tt = hp * y[k];
                o[k] += tt;
            }
        }
    }
    memcpy(stream, out, (size_t)t * nC * sizeof(float));
    free(nx), free(pre), free(post), free(res), free(u), free(xb), free(nrm), free(a), free(out);
}

/* encoder.go:167 Stack for one clip: mhc.go:131 ExpandLanes, the layers,
 * mhc.go:140 CollapseLanes (Σ over the lanes, then ÷ lanes) and the final
 * norm (OutFinalNorm). */
static int enc_stack_clip(const wo_encoder *e, const float *x, int t, int form, float *out) {
    const wo_decoder *d = &e->d;
    if (t > d->rope_len) return -1;
    int n = d->lanes, c = d->dim, nC = n * c;
    float *stream = malloc((size_t)t * nC * sizeof(float)), *m = calloc((size_t)t * c, sizeof(float));
    for (int i = 0; i < t; i++)
        for (int k = 0; k < n; k++) memcpy(stream + (size_t)i * nC + (size_t)k * c, x + (size_t)i * c, c * sizeof(float));
    for (int l = 0; l < d->layers; l++) enc_layer(e, l, stream, t, form);
    for (int i = 0; i < t; i++) {
        float *o = m + (size_t)i * c;
        for (int k = 0; k < n; k++)
            for (int j = 0; j < c; j++) o[j] += stream[(size_t)i * nC + (size_t)k * c + j];
        for (int j = 0; j < c; j++) o[j] /= (float)n;
    }
    zc_norm(out, m, t, c, d->final_norm);
    free(stream), free(m);
    return 0;
}

int wo_enc_stack(const wo_encoder *e, const float *x, int clips, int t, int form, float *out) {
    size_t per = (size_t)t * e->d.dim;
    for (int b = 0; b < clips; b++)
        if (enc_stack_clip(e, x + b * per, t, form, out + b * per) != 0) return -1;
    return 0;
}

typedef struct {
    const wo_encoder *e;
    const float *x;
    float *out;
    int t, form;
    atomic_int bad;
} enc_job;

static void enc_task(int b, void *arg) {
    enc_job *j = arg;
    size_t per = (size_t)j->t * j->e->d.dim;
    if (enc_stack_clip(j->e, j->x + b * per, j->t, j->form, j->out + b * per) != 0) atomic_store(&j->bad, 1);
}

int wo_enc_stack_mt(const wo_encoder *e, const float *x, int clips, int t, int form, float *out, int threads) {
    enc_job job = {e, x, out, t, form, 0};
    wo_parallel_for(clips, threads < 1 ? 1 : threads, enc_task, &job);
    return atomic_load(&job.bad) ? -1 : 0;
}
