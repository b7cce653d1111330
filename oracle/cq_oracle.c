/*
 * cq_oracle.c — CPU restatement of internal/cq (the CQ LUT GEMV/GEMM) and of
 * the cact pieces it reads. TEST INFRASTRUCTURE ONLY: used by tests/ as the
 * checker and by bench.py as the timed CPU baseline, never by the product.
 *
 * Each function names the reference routine it follows (file:line in the
 * go-whistle module). The float32 operations and their order are the
 * reference's; see oracle.h for the compile flags that keep them so.
 */
#include "oracle.h"

#include <math.h>
#include "par.h"
#include <stdlib.h>
#include <string.h>

enum {
    LUT_ROWS = 32,              /* lut.go:32 lutRows */
    LUT_Q = 8191,               /* lut.go:33 lutQ */
    LUT_BIAS = 64,              /* lut.go:34 lutBias */
    LUT_MAX_GROUP_BYTES = 256,  /* lut.go:38 lutMaxGroupBytes */
    LUT_PIECE_BYTES = 1 << 18,  /* lut.go:93 lutPieceBytes */
};

/* internal/cact/half.go:8 float16ToFloat32: exact widening, subnormals
 * normalised, inf/NaN keep their fraction bits. */
float wo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) & 1u;
    uint32_t exp = (uint32_t)(h >> 10) & 0x1fu;
    uint32_t frac = (uint32_t)h & 0x3ffu;
    uint32_t bits;

    if (exp == 0) {
        if (frac == 0) {
            bits = sign << 31;
        } else {
            uint32_t exp32 = 113;
            while ((frac & 0x400u) == 0) {
                frac <<= 1;
                exp32--;
            }
            frac &= 0x3ffu;
            bits = (sign << 31) | (exp32 << 23) | (frac << 13);
        }
    } else if (exp == 0x1f) {
        bits = (sign << 31) | 0x7f800000u | (frac << 13);
    } else {
        bits = (sign << 31) | ((exp + 112u) << 23) | (frac << 13);
    }

    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* internal/cq/kernel.go:384 fwht (the same stages as cact/cq.go fwht). */
void wo_fwht(float *x, int n) {
    for (int h = 1; h < n; h *= 2) {
        for (int i = 0; i < n; i += 2 * h) {
            for (int j = i; j < i + h; j++) {
                float a = x[j], b = x[j + h];
                x[j] = a + b;
                x[j + h] = a - b;
            }
        }
    }
}

/* internal/cq/kernel.go:375 invSqrt: float32(1 / math.Sqrt(float64(G))). */
static float inv_sqrt(int group) { return (float)(1.0 / sqrt((double)group)); }

/* internal/cq/lut.go:213 lutStepOf: float32(1 / (lutQ * math.Sqrt(G))). */
float wo_lut_step_of(int group) { return (float)(1.0 / ((double)LUT_Q * sqrt((double)group))); }

/* internal/cq/lut.go:219 lutInv. */
static float lut_inv(float m) { return m > 0.0f ? (float)LUT_Q / m : 0.0f; }

/* internal/cq/lut.go:229 lutPut: math.RoundToEven(float64(e)) under the
 * default round-to-nearest-even mode, split into the two byte planes. */
static int32_t lut_round(float e) { return (int32_t)nearbyint((double)e); }

static void lut_put(uint8_t *t, int16_t *it, int c, float e) {
    int32_t v = lut_round(e);
    if (t) {
        t[c] = (uint8_t)(v & 127);
        t[16 + c] = (uint8_t)((v >> 7) + LUT_BIAS);
    }
    if (it) it[c] = (int16_t)v;
}

/* internal/cq/lut.go:239 lutTables2Generic and :263 lutTables4Generic. The
 * planes go to tab (32 bytes per nibble table), the integers to itab (16 per
 * table); either may be NULL. */
static float lut_tables(int bits, uint8_t *tab, int16_t *itab, const float *x, int n, const float *cb,
                        float cb_max) {
    float mx = 0.0f;

    if (bits == 2) {
        for (int q = 0; q < n; q += 2) {
            float v = fabsf(x[q]) + fabsf(x[q + 1]);
            if (v > mx) mx = v;
        }
        float m = cb_max * mx;
        float inv = lut_inv(m);
        for (int q = 0; q < n / 2; q++) {
            float a = x[2 * q] * inv, b = x[2 * q + 1] * inv;
            for (int c = 0; c < 16; c++) {
                float lo = cb[c & 3] * a;
                float hi = cb[c >> 2] * b;
                lut_put(tab ? tab + 32 * q : NULL, itab ? itab + 16 * q : NULL, c, lo + hi);
            }
        }
        return m;
    }

    for (int q = 0; q < n; q++) {
        float v = fabsf(x[q]);
        if (v > mx) mx = v;
    }
    float m = cb_max * mx;
    float inv = lut_inv(m);
    for (int q = 0; q < n; q++) {
        float a = x[q] * inv;
        for (int c = 0; c < 16; c++) lut_put(tab ? tab + 32 * q : NULL, itab ? itab + 16 * q : NULL, c, cb[c] * a);
    }
    return m;
}

float wo_lut_tables_planes(int bits, uint8_t *tab, const float *x, int n, const float *cb, float cb_max) {
    return lut_tables(bits, tab, NULL, x, n, cb, cb_max);
}

float wo_lut_tables_int(int bits, int16_t *tab, const float *x, int n, const float *cb, float cb_max) {
    return lut_tables(bits, NULL, tab, x, n, cb, cb_max);
}

/* internal/cq/lut.go:289 lutLookupGeneric. */
void wo_lut_lookup_blocked(float *y, const uint8_t *idx, const uint8_t *tab, const float *norm,
                           const float *steps, int blocks, int groups, int gb) {
    int32_t bias = 128 * LUT_BIAS * 2 * gb;
    int row_bytes = groups * gb;

    for (int b = 0; b < blocks; b++) {
        float *yb = y + (size_t)b * LUT_ROWS;
        for (int i = 0; i < LUT_ROWS; i++) yb[i] = 0.0f;

        for (int g = 0; g < groups; g++) {
            float step = steps[g];
            for (int i = 0; i < LUT_ROWS; i++) {
                int32_t lo = 0, hi = 0;
                for (int j = g * gb; j < (g + 1) * gb; j++) {
                    uint8_t v = idx[((size_t)b * row_bytes + j) * LUT_ROWS + i];
                    const uint8_t *t = tab + 64 * (size_t)j;
                    lo += (int32_t)t[v & 15] + (int32_t)t[32 + (v >> 4)];
                    hi += (int32_t)t[16 + (v & 15)] + (int32_t)t[48 + (v >> 4)];
                }
                float coef = norm[((size_t)b * groups + g) * LUT_ROWS + i] * step;
                float term = (float)(hi * 128 + lo - bias) * coef;
                yb[i] = yb[i] + term;
            }
        }
    }
}

/* ---- the lut kernel on a prepared matrix (matrix.go:60-96, lut.go:58-80) ---- */

typedef struct {
    int out, in, group, bits, groups, gb, row_bytes, blocks;
    float cb[16];
    float cb_max, lut_step;
    uint8_t *idx;  /* lut.go:51 idx[(b·rowBytes + j)·lutRows + i] */
    float *norm;   /* lut.go:53 norm[(b·groups + g)·lutRows + i] */
} lut_matrix;

static int lut_prepare(lut_matrix *m, const wo_packed *p) {
    memset(m, 0, sizeof *m);
    m->out = p->out;
    m->in = p->in;
    m->group = p->group;
    m->bits = p->bits;
    m->groups = (p->in + p->group - 1) / p->group;
    m->gb = p->group * p->bits / 8;
    m->row_bytes = m->groups * m->gb;
    m->blocks = (p->out + LUT_ROWS - 1) / LUT_ROWS;
    if (m->gb > LUT_MAX_GROUP_BYTES) return -1;

    for (int c = 0; c < (1 << p->bits); c++) {
        m->cb[c] = p->cb[c];
        float a = fabsf(p->cb[c]);
        if (a > m->cb_max) m->cb_max = a;
    }
    m->lut_step = wo_lut_step_of(p->group);

    size_t nb = (size_t)(m->blocks > 0 ? m->blocks : 1);
    m->idx = calloc(nb * m->row_bytes * LUT_ROWS, 1);
    m->norm = calloc(nb * m->groups * LUT_ROWS, sizeof(float));
    for (int r = 0; r < p->out; r++) {
        int b = r / LUT_ROWS, i = r % LUT_ROWS;
        for (int j = 0; j < m->row_bytes; j++)
            m->idx[((size_t)b * m->row_bytes + j) * LUT_ROWS + i] = p->index[(size_t)r * m->row_bytes + j];
        for (int g = 0; g < m->groups; g++)
            m->norm[((size_t)b * m->groups + g) * LUT_ROWS + i] = wo_f16_to_f32(p->norms16[(size_t)r * m->groups + g]);
    }
    return 0;
}

static void lut_release(lut_matrix *m) {
    free(m->idx);
    free(m->norm);
    m->idx = NULL;
    m->norm = NULL;
}

/* internal/cq/lut.go:160 lutTables: rotate one activation (FWHT, no 1/√G)
 * and build its byte-plane tables and group steps. */
static void lut_tables_act(const lut_matrix *m, const float *x, float *xh, uint8_t *tab, float *steps) {
    int pad = m->groups * m->group;
    int tab_bytes = 64 * m->gb;
    memcpy(xh, x, (size_t)m->in * sizeof(float));
    for (int k = m->in; k < pad; k++) xh[k] = 0.0f;
    for (int g = 0; g < m->groups; g++) {
        float *xg = xh + (size_t)g * m->group;
        float mm;
#ifdef __AVX2__
        /* lut_amd64.go:13 fwhtF32, :22 lutTables2, :35 lutTables4: the AVX2
         * kernels for groups of 8 and more, as the reference dispatches. */
        if (m->group >= 8) {
            wo_fwht_avx2(xg, m->group);
            mm = wo_lut_tables_planes_avx2(m->bits, tab + (size_t)g * tab_bytes, xg, m->group, m->cb, m->cb_max);
        } else
#endif
        {
            wo_fwht(xg, m->group);
            mm = lut_tables(m->bits, tab + (size_t)g * tab_bytes, NULL, xg, m->group, m->cb, m->cb_max);
        }
        steps[g] = mm * m->lut_step;
    }
}

/* lut.go:182 lutApply over blocks [b_lo, b_hi) into y (rows of the matrix). */
static void lut_apply(const lut_matrix *m, const uint8_t *tab, const float *steps, float *ybuf, float *y, int b_lo,
                      int b_hi) {
    int ib = m->row_bytes * LUT_ROWS, nbk = m->groups * LUT_ROWS;
    /* lut_amd64.go:46 lutLookup: the AVX2 kernel where the host has it, as
     * the reference dispatches (the same bits as the generic kernel). */
#ifdef __AVX2__
    wo_lut_lookup_blocked_avx2(ybuf, m->idx + (size_t)b_lo * ib, tab, m->norm + (size_t)b_lo * nbk, steps,
                               b_hi - b_lo, m->groups, m->gb);
#else
    wo_lut_lookup_blocked(ybuf, m->idx + (size_t)b_lo * ib, tab, m->norm + (size_t)b_lo * nbk, steps, b_hi - b_lo,
                          m->groups, m->gb);
#endif
    int r0 = b_lo * LUT_ROWS, r1 = b_hi * LUT_ROWS;
    if (r1 > m->out) r1 = m->out;
    if (r1 > r0) memcpy(y + r0, ybuf, (size_t)(r1 - r0) * sizeof(float));
}

/* A static split of [0, n) into at most `workers` pieces of at least `grain`
 * items: the products do not depend on it (TestGEMMWorkers). */
static int pieces_of(int n, int grain, int workers) {
    if (grain < 1) grain = 1;
    int p = (n + grain - 1) / grain;
    if (p > workers) p = workers;
    return p < 1 ? 1 : p;
}

/* One piece of activations [lo, hi) through every matrix (lut.go:110-115). */
typedef struct {
    const lut_matrix *ms;
    int n;
    const float *x;
    int rows;
    float **ys;
    int np, pad, nbmax;
} act_job;

static void act_piece(int piece, void *arg) {
    const act_job *j = arg;
    const lut_matrix *m0 = &j->ms[0];
    int lo = (int)((long)j->rows * piece / j->np), hi = (int)((long)j->rows * (piece + 1) / j->np);
    float *xh = malloc((size_t)j->pad * sizeof(float));
    uint8_t *tab = malloc((size_t)64 * m0->row_bytes);
    float *steps = malloc((size_t)m0->groups * sizeof(float));
    float *ybuf = malloc((size_t)j->nbmax * LUT_ROWS * sizeof(float));
    for (int i = lo; i < hi; i++) {
        lut_tables_act(m0, j->x + (size_t)i * m0->in, xh, tab, steps);
        for (int k = 0; k < j->n; k++)
            lut_apply(&j->ms[k], tab, steps, ybuf, j->ys[k] + (size_t)i * j->ms[k].out, 0, j->ms[k].blocks);
    }
    free(xh);
    free(tab);
    free(steps);
    free(ybuf);
}

/* One piece of blocks of a single activation's product (lut.go:190-194). */
typedef struct {
    const lut_matrix *m;
    const uint8_t *tab;
    const float *steps;
    float *y;
    int np;
} block_job;

static void block_piece(int piece, void *arg) {
    const block_job *j = arg;
    int lo = (int)((long)j->m->blocks * piece / j->np), hi = (int)((long)j->m->blocks * (piece + 1) / j->np);
    float *ybuf = malloc((size_t)(hi - lo + 1) * LUT_ROWS * sizeof(float));
    lut_apply(j->m, j->tab, j->steps, ybuf, j->y, lo, hi);
    free(ybuf);
}

/* internal/cq/lut.go:102 gemmLUT with lut.go:129 lutRun, on `threads`
 * threads. ms share their tables (kernel.go:134 GEMMs, lut.go:206). */
static void lut_gemm_shared(const lut_matrix *ms, int n, const float *x, int rows, float **ys, int threads) {
    const lut_matrix *m0 = &ms[0];
    long per = 0;
    int nbmax = 1;
    for (int k = 0; k < n; k++) {
        per += (long)ms[k].out * ms[k].row_bytes;
        if (ms[k].blocks > nbmax) nbmax = ms[k].blocks;
    }
    if (per == 0) per = 1;
    int pad = m0->groups * m0->group;

    if (rows > 1 && (rows >= threads || per < 2L * LUT_PIECE_BYTES)) {
        int grain = (int)((LUT_PIECE_BYTES + per - 1) / per);
        int np = pieces_of(rows, grain, threads);
act_job job = {ms, n, x, rows, ys, np, pad, nbmax};
        wo_parallel_for(np, threads, act_piece, &job);
        return;
    }

    float *xh = malloc((size_t)pad * sizeof(float));
    uint8_t *tab = malloc((size_t)64 * m0->row_bytes);
    float *steps = malloc((size_t)m0->groups * sizeof(float));
    int split = per >= 2L * LUT_PIECE_BYTES;
    for (int i = 0; i < rows; i++) {
        lut_tables_act(m0, x + (size_t)i * m0->in, xh, tab, steps);
        for (int k = 0; k < n; k++) {
            const lut_matrix *m = &ms[k];
            float *y = ys[k] + (size_t)i * m->out;
            if (!split || m->blocks == 0) {
                float *ybuf = malloc((size_t)(m->blocks > 0 ? m->blocks : 1) * LUT_ROWS * sizeof(float));
                lut_apply(m, tab, steps, ybuf, y, 0, m->blocks);
                free(ybuf);
                continue;
            }
            int ib = m->row_bytes * LUT_ROWS;
            int grain = (LUT_PIECE_BYTES + ib - 1) / ib;
            int np = pieces_of(m->blocks, grain, threads);
block_job job = {m, tab, steps, y, np};
            wo_parallel_for(np, threads, block_piece, &job);
        }
    }
    free(xh);
    free(tab);
    free(steps);
}

/* lut_apply writes whole blocks; y must hold the rows of full blocks only up
 * to out, which lut_apply's memcpy respects. */

int wo_cq_gemm_lut(const wo_packed *p, const float *x, int rows, float *y) {
    return wo_cq_gemm_lut_mt(p, x, rows, y, 1);
}

int wo_cq_gemm_lut_mt(const wo_packed *p, const float *x, int rows, float *y, int threads) {
    if (rows == 0 || p->out == 0) return 0; /* kernel.go:110 */
    lut_matrix m;
    if (lut_prepare(&m, p) != 0) {
        lut_release(&m);
        return -1;
    }
    lut_gemm_shared(&m, 1, x, rows, &y, threads < 1 ? 1 : threads);
    lut_release(&m);
    return 0;
}

int wo_cq_gemms_lut(const wo_packed *ps, int n, const float *x, int rows, float **ys) {
    if (rows == 0 || n == 0) return 0;
    lut_matrix *ms = calloc((size_t)n, sizeof *ms);
    int rc = 0;
    for (int k = 0; k < n; k++)
        if (lut_prepare(&ms[k], &ps[k]) != 0) rc = -1;
    if (rc == 0) lut_gemm_shared(ms, n, x, rows, ys, 1);
    for (int k = 0; k < n; k++) lut_release(&ms[k]);
    free(ms);
    return rc;
}

/* A prepared matrix for the timed CPU baseline: Prepare once, multiply many. */
void *wo_lut_prepare(const wo_packed *p) {
    lut_matrix *m = malloc(sizeof *m);
    if (lut_prepare(m, p) != 0) {
        lut_release(m);
        free(m);
        return NULL;
    }
    return m;
}

void wo_lut_gemm_prepared(void *h, const float *x, int rows, float *y, int threads) {
    lut_matrix *m = h;
    if (rows == 0 || m->out == 0) return;
    lut_gemm_shared(m, 1, x, rows, &y, threads < 1 ? 1 : threads);
}

void wo_lut_release(void *h) {
    lut_release(h);
    free(h);
}

int wo_max_threads(void) { return wo_cpu_count(); }

/* ---- the Exact path: rotate, nibble, nibble4, gather (kernel.go:162-373) ---- */

/* matrix.go:185 at: index k of a packed row, LSB first. */
static uint8_t at(const uint8_t *row, int k, int width) {
    int bit = k * width;
    return (uint8_t)((row[bit / 8] >> (bit % 8)) & ((1 << width) - 1));
}

typedef struct {
    int out, in, group, bits, groups, gb, row_bytes, pad;
    const uint8_t *index;
    const float *cb;
    float *norms; /* widened, [out][groups] (matrix.go:81-85) */
} flat_matrix;

static void flat_prepare(flat_matrix *m, const wo_packed *p) {
    m->out = p->out;
    m->in = p->in;
    m->group = p->group;
    m->bits = p->bits;
    m->groups = (p->in + p->group - 1) / p->group;
    m->gb = p->group * p->bits / 8;
    m->row_bytes = m->groups * m->gb;
    m->pad = m->groups * m->group;
    m->index = p->index;
    m->cb = p->cb;
    m->norms = malloc((size_t)(p->out > 0 ? p->out : 1) * m->groups * sizeof(float));
    for (size_t i = 0; i < (size_t)p->out * m->groups; i++) m->norms[i] = wo_f16_to_f32(p->norms16[i]);
}

/* kernel.go:392 rotate: zero-pad, FWHT per group, times invSqrt(G). */
static void rotate(const flat_matrix *m, float *xh, const float *x) {
    memcpy(xh, x, (size_t)m->in * sizeof(float));
    for (int k = m->in; k < m->pad; k++) xh[k] = 0.0f;
    float scale = inv_sqrt(m->group);
    for (int g = 0; g < m->groups; g++) {
        float *xg = xh + (size_t)g * m->group;
        wo_fwht(xg, m->group);
        for (int k = 0; k < m->group; k++) xg[k] *= scale;
    }
}

/* kernel.go:431 nibbleTables: nib[q][code], 2*rowBytes tables. */
static void nibble_tables(const flat_matrix *m, float (*nib)[16], const float *xh) {
    if (m->bits == 4) {
        for (int q = 0; q < m->pad; q++)
            for (int c = 0; c < 16; c++) nib[q][c] = m->cb[c] * xh[q];
        return;
    }
    for (int q = 0; q < 2 * m->row_bytes; q++) {
        float a = xh[2 * q], b = xh[2 * q + 1];
        for (int hi = 0; hi < 4; hi++) {
            float hb = m->cb[hi] * b;
            for (int lo = 0; lo < 4; lo++) {
                float la = m->cb[lo] * a;
                nib[q][hi << 2 | lo] = la + hb;
            }
        }
    }
}

/* kernel.go:460 lookupNibble: eight accumulators per group, then a pairwise
 * sum times the norm. */
static void lookup_nibble(const flat_matrix *m, float *y, float (*nib)[16]) {
    int gb = m->gb;
    for (int r = 0; r < m->out; r++) {
        const uint8_t *row = m->index + (size_t)r * m->row_bytes;
        const float *norms = m->norms + (size_t)r * m->groups;
        float acc = 0.0f;
        for (int g = 0; g < m->groups; g++) {
            const uint8_t *rg = row + (size_t)g * gb;
            float (*tg)[16] = nib + (size_t)2 * g * gb;
            float a0 = 0, a1 = 0, a2 = 0, a3 = 0, a4 = 0, a5 = 0, a6 = 0, a7 = 0;
            int j = 0;
            for (; j + 8 <= gb; j += 8) {
                uint64_t w = 0;
                for (int b = 0; b < 8; b++) w |= (uint64_t)rg[j + b] << (8 * b);
                float (*t)[16] = tg + 2 * j;
                a0 += t[0][w & 15] + t[8][(w >> 32) & 15];
                a1 += t[1][(w >> 4) & 15] + t[9][(w >> 36) & 15];
                a2 += t[2][(w >> 8) & 15] + t[10][(w >> 40) & 15];
                a3 += t[3][(w >> 12) & 15] + t[11][(w >> 44) & 15];
                a4 += t[4][(w >> 16) & 15] + t[12][(w >> 48) & 15];
                a5 += t[5][(w >> 20) & 15] + t[13][(w >> 52) & 15];
                a6 += t[6][(w >> 24) & 15] + t[14][(w >> 56) & 15];
                a7 += t[7][(w >> 28) & 15] + t[15][w >> 60];
            }
            for (; j < gb; j++) a0 += tg[2 * j][rg[j] & 15] + tg[2 * j + 1][rg[j] >> 4];
            float sum = ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7));
            acc += sum * norms[g];
        }
        y[r] = acc;
    }
}

/* kernel.go:519 lookupNibble4 for one of the four activations: the lo and
 * the hi nibbles' entries each summed byte after byte, then (a + b) * n. */
static void lookup_nibble4_one(const flat_matrix *m, float *y, float (*nib)[16]) {
    int gb = m->gb;
    for (int r = 0; r < m->out; r++) {
        const uint8_t *row = m->index + (size_t)r * m->row_bytes;
        const float *norms = m->norms + (size_t)r * m->groups;
        float c = 0.0f;
        for (int g = 0; g < m->groups; g++) {
            const uint8_t *rg = row + (size_t)g * gb;
            float (*tg)[16] = nib + (size_t)2 * g * gb;
            float a = 0.0f, b = 0.0f;
            for (int j = 0; j < gb; j++) {
                a += tg[2 * j][rg[j] & 15];
                b += tg[2 * j + 1][rg[j] >> 4];
            }
            float s = a + b;
            c += s * norms[g];
        }
        y[r] = c;
    }
}

/* kernel.go:220 gather. */
static void gather(const flat_matrix *m, float *y, const float *xh) {
    for (int r = 0; r < m->out; r++) {
        const uint8_t *row = m->index + (size_t)r * m->row_bytes;
        float acc = 0.0f;
        for (int g = 0; g < m->groups; g++) {
            float dot = 0.0f;
            for (int k = 0; k < m->group; k++) {
                float t = m->cb[at(row, g * m->group + k, m->bits)] * xh[g * m->group + k];
                dot += t;
            }
            float t = dot * m->norms[(size_t)r * m->groups + g];
            acc += t;
        }
        y[r] = acc;
    }
}

void wo_cq_gemm_exact(const wo_packed *p, const float *x, int rows, float *y) {
    if (rows == 0 || p->out == 0) return;
    flat_matrix m;
    flat_prepare(&m, p);
    float *xh = malloc((size_t)m.pad * sizeof(float));
    float (*nib)[16] = malloc((size_t)2 * m.row_bytes * sizeof *nib);
    int four = rows - rows % 4; /* kernel.go:359-372: nibble4 on whole blocks of four */
    for (int i = 0; i < rows; i++) {
        rotate(&m, xh, x + (size_t)i * m.in);
        nibble_tables(&m, nib, xh);
        if (i < four)
            lookup_nibble4_one(&m, y + (size_t)i * m.out, nib);
        else
            lookup_nibble(&m, y + (size_t)i * m.out, nib);
    }
    free(nib);
    free(xh);
    free(m.norms);
}

void wo_cq_gemm_gather(const wo_packed *p, const float *x, int rows, float *y) {
    if (rows == 0 || p->out == 0) return;
    flat_matrix m;
    flat_prepare(&m, p);
    float *xh = malloc((size_t)m.pad * sizeof(float));
    for (int i = 0; i < rows; i++) {
        rotate(&m, xh, x + (size_t)i * m.in);
        gather(&m, y + (size_t)i * m.out, xh);
    }
    free(xh);
    free(m.norms);
}

/* matrix.go:161 Row. */
void wo_cq_row(const wo_packed *p, int r, float *dst) {
    int groups = (p->in + p->group - 1) / p->group;
    int row_bytes = groups * p->group * p->bits / 8;
    const uint8_t *row = p->index + (size_t)r * row_bytes;
    float scale = inv_sqrt(p->group);
    float *buf = malloc((size_t)p->group * sizeof(float));
    for (int g = 0; g < groups; g++) {
        float s = wo_f16_to_f32(p->norms16[(size_t)r * groups + g]) * scale;
        for (int k = 0; k < p->group; k++) buf[k] = p->cb[at(row, g * p->group + k, p->bits)] * s;
        wo_fwht(buf, p->group);
        int col = g * p->group;
        int end = col + p->group < p->in ? col + p->group : p->in;
        memcpy(dst + col, buf, (size_t)(end - col) * sizeof(float));
    }
    free(buf);
}
