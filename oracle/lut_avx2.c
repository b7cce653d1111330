/*
 * lut_avx2.c — the reference's amd64 lookup kernel restated with AVX2
 * intrinsics (TEST INFRASTRUCTURE ONLY: the CPU baseline's inner loop).
 *
 * internal/cq/lut_amd64.s:236 lutLookupAVX2, which the reference runs on any
 * amd64 host with AVX2 (lut_amd64.go:9) and whose products equal
 * lutLookupGeneric's bit for bit (asm_test.go): per 32-row block and index
 * byte, one 32-byte load holds that byte of all 32 rows; the low and high
 * nibbles index the lo and hi planes of the byte's two tables with byte
 * shuffles (tables broadcast to both 128-bit lanes); each plane's two
 * lookups add in a byte and widen into uint16 sums per row; at the end of a
 * group 128·Σhi + Σlo − bias becomes float32 and is added to y times
 * norm · step. Same float32 operations, same order, as the generic kernel.
 */
#include <immintrin.h>
#include <stdint.h>

#include "oracle.h"

/* Rows 0-7 and 16-23 (s0 = Σlo, s1 = Σhi of those rows as uint16, in-lane
 * order) or 8-15 and 24-31: y[r] += float32(128·Σhi + Σlo − bias) ·
 * (norm[r] · step) for the eight rows of each half. */
static inline void group_rows(float *y, const float *norm, __m256i slo, __m256i shi, __m256i bias, __m256 step) {
    const __m256i zero = _mm256_setzero_si256();
    __m256i lo_a = _mm256_unpacklo_epi16(slo, zero), lo_b = _mm256_unpackhi_epi16(slo, zero);
    __m256i hi_a = _mm256_unpacklo_epi16(shi, zero), hi_b = _mm256_unpackhi_epi16(shi, zero);
    __m256i a = _mm256_sub_epi32(_mm256_add_epi32(lo_a, _mm256_slli_epi32(hi_a, 7)), bias);
    __m256i b = _mm256_sub_epi32(_mm256_add_epi32(lo_b, _mm256_slli_epi32(hi_b, 7)), bias);
    __m256 f0 = _mm256_cvtepi32_ps(_mm256_permute2x128_si256(a, b, 0x20)); /* first eight rows */
    __m256 f1 = _mm256_cvtepi32_ps(_mm256_permute2x128_si256(a, b, 0x31)); /* rows + 16 */
    __m256 c0 = _mm256_mul_ps(_mm256_loadu_ps(norm), step);
    __m256 c1 = _mm256_mul_ps(_mm256_loadu_ps(norm + 16), step);
    _mm256_storeu_ps(y, _mm256_add_ps(_mm256_loadu_ps(y), _mm256_mul_ps(f0, c0)));
    _mm256_storeu_ps(y + 16, _mm256_add_ps(_mm256_loadu_ps(y + 16), _mm256_mul_ps(f1, c1)));
}

void wo_lut_lookup_blocked_avx2(float *y, const uint8_t *idx, const uint8_t *tab, const float *norm,
                                const float *steps, int blocks, int groups, int gb) {
    const __m256i bias = _mm256_set1_epi32(gb << 14); /* 128 · lutBias · 2·gb */
    const __m256i m0f = _mm256_set1_epi8(0x0f);
    const __m256i zero = _mm256_setzero_si256();
    for (int b = 0; b < blocks; b++, y += 32) {
        for (int i = 0; i < 32; i += 8) _mm256_storeu_ps(y + i, _mm256_setzero_ps());
        const uint8_t *t = tab;
        for (int g = 0; g < groups; g++, norm += 32) {
            __m256i slo0 = zero, slo1 = zero, shi0 = zero, shi1 = zero;
            for (int k = 0; k < gb; k++, idx += 32, t += 64) {
                const __m256i v = _mm256_loadu_si256((const __m256i *)idx);
                const __m256i lo = _mm256_and_si256(v, m0f);
                const __m256i hi = _mm256_and_si256(_mm256_srli_epi16(v, 4), m0f);
                const __m256i t0lo = _mm256_broadcastsi128_si256(_mm_loadu_si128((const __m128i *)t));
                const __m256i t0hi = _mm256_broadcastsi128_si256(_mm_loadu_si128((const __m128i *)(t + 16)));
                const __m256i t1lo = _mm256_broadcastsi128_si256(_mm_loadu_si128((const __m128i *)(t + 32)));
                const __m256i t1hi = _mm256_broadcastsi128_si256(_mm_loadu_si128((const __m128i *)(t + 48)));
                const __m256i pl = _mm256_add_epi8(_mm256_shuffle_epi8(t0lo, lo), _mm256_shuffle_epi8(t1lo, hi));
                const __m256i ph = _mm256_add_epi8(_mm256_shuffle_epi8(t0hi, lo), _mm256_shuffle_epi8(t1hi, hi));
                slo0 = _mm256_add_epi16(slo0, _mm256_unpacklo_epi8(pl, zero));
                slo1 = _mm256_add_epi16(slo1, _mm256_unpackhi_epi8(pl, zero));
                shi0 = _mm256_add_epi16(shi0, _mm256_unpacklo_epi8(ph, zero));
                shi1 = _mm256_add_epi16(shi1, _mm256_unpackhi_epi8(ph, zero));
            }
            const __m256 step = _mm256_set1_ps(steps[g]);
            group_rows(y, norm, slo0, shi0, bias, step);         /* rows 0-7, 16-23 */
            group_rows(y + 8, norm + 8, slo1, shi1, bias, step); /* rows 8-15, 24-31 */
        }
    }
}

/* internal/cq/lut_amd64.s:20 fwhtAVX2 (n a power of two >= 8): h = 1, 2, 4
 * within each 8 floats by permutes (the sum in the lower element of a pair,
 * lower − upper in the upper one), then one pass per h = 8 ... n/2: the
 * butterflies of wo_fwht, stage by stage. */
void wo_fwht_avx2(float *x, int n) {
    for (int i = 0; i < n; i += 8) {
        __m256 v = _mm256_loadu_ps(x + i);
        __m256 p = _mm256_permute_ps(v, 0xB1);
        v = _mm256_blend_ps(_mm256_add_ps(v, p), _mm256_sub_ps(p, v), 0xAA);
        p = _mm256_permute_ps(v, 0x4E);
        v = _mm256_blend_ps(_mm256_add_ps(v, p), _mm256_sub_ps(p, v), 0xCC);
        p = _mm256_permute2f128_ps(v, v, 0x01);
        v = _mm256_blend_ps(_mm256_add_ps(v, p), _mm256_sub_ps(p, v), 0xF0);
        _mm256_storeu_ps(x + i, v);
    }
    for (int h = 8; h < n; h *= 2)
        for (int i = 0; i < n; i += 2 * h)
            for (int j = i; j < i + h; j += 8) {
                const __m256 a = _mm256_loadu_ps(x + j), b = _mm256_loadu_ps(x + j + h);
                _mm256_storeu_ps(x + j, _mm256_add_ps(a, b));
                _mm256_storeu_ps(x + j + h, _mm256_sub_ps(a, b));
            }
}

/* lut_amd64.s:103 lutQuantStore: the 16 entries lo (codes 0-7) and hi
 * (8-15) rounded to nearest even, as lo plane v & 127 and hi plane
 * (v >> 7) + lutBias, 32 bytes at t. */
static inline void quant_store(uint8_t *t, __m256 v0, __m256 v1) {
    __m256i w = _mm256_packs_epi32(_mm256_cvtps_epi32(v0), _mm256_cvtps_epi32(v1));
    w = _mm256_permute4x64_epi64(w, 0xD8); /* codes 0-15 in order */
    const __m256i hi = _mm256_add_epi16(_mm256_srai_epi16(w, 7), _mm256_set1_epi16(64));
    const __m256i lo = _mm256_and_si256(w, _mm256_set1_epi16(127));
    const __m256i b = _mm256_permute4x64_epi64(_mm256_packus_epi16(lo, hi), 0xD8);
    _mm256_storeu_si256((__m256i *)t, b);
}

/* The largest element of v (all >= 0, no NaN). */
static inline float hmax(__m256 v) {
    __m128 m = _mm_max_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
    m = _mm_max_ps(m, _mm_permute_ps(m, 0x4E));
    m = _mm_max_ps(m, _mm_permute_ps(m, 0xB1));
    return _mm_cvtss_f32(m);
}

/* internal/cq/lut_amd64.s:127 lutTables2AVX2 and :184 lutTables4AVX2 for one
 * group x[:n] (n a multiple of 8): the byte planes of wo_lut_tables_planes,
 * bit for bit; returns M. */
float wo_lut_tables_planes_avx2(int bits, uint8_t *tab, const float *x, int n, const float *cb, float cb_max) {
    const __m256 absmask = _mm256_castsi256_ps(_mm256_set1_epi32(0x7fffffff));
    __m256 mx = _mm256_setzero_ps();
    for (int i = 0; i < n; i += 8) {
        __m256 a = _mm256_and_ps(_mm256_loadu_ps(x + i), absmask);
        if (bits == 2) a = _mm256_hadd_ps(a, a); /* |x[2q]| + |x[2q+1]| */
        mx = _mm256_max_ps(mx, a);
    }
    const float m = cb_max * hmax(mx);
    const float inv = m > 0.0f ? 8191.0f / m : 0.0f; /* lut.go:219 lutInv */
    if (bits == 2) {
        /* cb[c & 3] for codes 0-7 and 8-15; cb[c >> 2] likewise */
        const __m256 clo = _mm256_setr_ps(cb[0], cb[1], cb[2], cb[3], cb[0], cb[1], cb[2], cb[3]);
        const __m256 chi0 = _mm256_setr_ps(cb[0], cb[0], cb[0], cb[0], cb[1], cb[1], cb[1], cb[1]);
        const __m256 chi1 = _mm256_setr_ps(cb[2], cb[2], cb[2], cb[2], cb[3], cb[3], cb[3], cb[3]);
        for (int q = 0; q < n / 2; q++) {
            const __m256 a = _mm256_set1_ps(x[2 * q] * inv), b = _mm256_set1_ps(x[2 * q + 1] * inv);
            const __m256 la = _mm256_mul_ps(clo, a);
            quant_store(tab + 32 * q, _mm256_add_ps(la, _mm256_mul_ps(chi0, b)),
                        _mm256_add_ps(la, _mm256_mul_ps(chi1, b)));
        }
    } else {
        const __m256 c0 = _mm256_loadu_ps(cb), c1 = _mm256_loadu_ps(cb + 8);
        for (int q = 0; q < n; q++) {
            const __m256 a = _mm256_set1_ps(x[q] * inv);
            quant_store(tab + 32 * q, _mm256_mul_ps(c0, a), _mm256_mul_ps(c1, a));
        }
    }
    return m;
}
