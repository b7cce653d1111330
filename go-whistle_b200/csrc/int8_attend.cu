// int8_attend.cu — the int8 KV-cache attention and the per-head int8
// quantiser of internal/needle (int8.go) on sm_100a.
//
// Quantiser (int8.go:36 QuantizeRow): s = max|x|/127 (1 for a zero chunk),
// q = clamp(rint_even(x/s), -128, 127), with IEEE division: one warp per
// chunk, the max by shuffles (order-free), bit-exact.
//
// Attention (int8.go:208 AttendInt8Spans), per (stream, query row, head):
//   q8, sq = QuantizeRow(q_h)                        (quant_q)
//   s_j = float32(dot_i32(q8, k8_j)) · (sq · sk_j) / scale
//   p = softmax(s): max, e_j = float32(exp(float64(s_j − max))), Σ e_j in key
//       order, e_j / Σ
//   out[d] = Σ_j float32((p_j · sv_j) · float32(v8_j[d])), key after key
// The logits stay in shared memory, so K and V each stream from HBM once.
// Every reduction whose order the reference fixes (the float sums over keys)
// runs in that order; the order-free ones (max, integer dots) run in
// parallel. The result equals the reference's generic path bit for bit,
// exp aside: CUDA's double exp and Go's math.Exp are both within one
// float64 ulp, so their float32 roundings can differ only within about
// 2^-29 (relative) of a float32 rounding boundary.
#include "common.cuh"
#include "needle_kernels.cuh"

namespace wb {

namespace {

constexpr int kAttThreads = 128;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// QuantizeRow of n values by one warp; q may alias nothing. Returns s.
__device__ float quantize_chunk_warp(const float *__restrict__ x, int n, int8_t *__restrict__ q, int lane) {
    float m = 0.0f;
    for (int i = lane; i < n; i += 32) m = fmaxf(m, fabsf(x[i]));
    m = warp_max(m);
    float s = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
    for (int i = lane; i < n; i += 32) {
        int r = __float2int_rn(__fdiv_rn(x[i], s));
        r = r < -128 ? -128 : (r > 127 ? 127 : r);
        q[i] = (int8_t)r;
    }
    return s;
}

__global__ void quantize_rows_kernel(const float *__restrict__ x, int chunks, int width, int8_t *__restrict__ q,
                                     float *__restrict__ s) {
    const int lane = threadIdx.x & 31;
    const int c = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (c >= chunks) return;
    float sc = quantize_chunk_warp(x + (size_t)c * width, width, q + (size_t)c * width, lane);
    if (lane == 0) s[c] = sc;
}

__global__ void __launch_bounds__(kAttThreads) attend_int8_kernel(const __grid_constant__ AttendParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int h = blockIdx.x, i = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int qk = p.qk, vd = p.vd, kvh = p.kv_heads;
    const int kv = h / (p.heads / kvh);
    const int kcols = kvh * qk, vcols = kvh * vd;

    // This stream's cache and key count.
    int nkeys = p.nkeys;
    if (p.nkeys_dev) nkeys = min(p.nkeys_dev[b], p.cap);
    const size_t blk = kv_block(p, b);
    const int8_t *k8 = p.k8 + blk * p.cap * kcols;
    const float *ks = p.ks + blk * p.cap * kvh;
    const int8_t *v8 = p.v8 + blk * p.cap * vcols;
    const float *vs = p.vs + blk * p.cap * kvh;

    int lo0, hi0, lo1, hi1;
    if (p.spans) {
        const int32_t *sp = p.spans + 4 * (size_t)i;
        lo0 = min(max(sp[0], 0), nkeys);
        hi0 = min(max(sp[1], lo0), nkeys);
        lo1 = min(max(sp[2], 0), nkeys);
        hi1 = min(max(sp[3], lo1), nkeys);
    } else {
        lo0 = hi0 = lo1 = 0;
        hi1 = nkeys;
    }
    const int len0 = hi0 - lo0, n = len0 + (hi1 - lo1);

    float *lg = reinterpret_cast<float *>(smem);  // [n] logits, then weights
    float *red = lg + p.max_keys;                 // [kAttThreads/32 + 2]
    float *qf = red + (kAttThreads / 32 + 2);     // [qk] float query
    int8_t *q8 = reinterpret_cast<int8_t *>(qf + qk);

    const float *qh = p.q + (((size_t)b * p.t + i) * p.heads + h) * qk;
    for (int c = tid; c < qk; c += kAttThreads) qf[c] = qh[c];
    __syncthreads();
    if (p.quant_q && warp == 0) {
        float sq = quantize_chunk_warp(qf, qk, q8, lane);
        if (lane == 0) red[kAttThreads / 32] = sq;
    }
    __syncthreads();
    const float sq = red[kAttThreads / 32];

    // Logits (int8.go:278 int8Logits, or :289 dotsF32I8 without quant_q).
    for (int jj = tid; jj < n; jj += kAttThreads) {
        int j = jj < len0 ? lo0 + jj : lo1 + (jj - len0);
        const int8_t *kr = k8 + (size_t)j * kcols + (size_t)kv * qk;
        float sk = ks[(size_t)j * kvh + kv];
        float logit;
        if (p.quant_q) {
            int32_t dot = 0;
            if (p.k_aligned4) {
                const int *kw = reinterpret_cast<const int *>(kr);
                const int *qw = reinterpret_cast<const int *>(q8);
                for (int c = 0; c < qk / 4; c++) dot = __dp4a(qw[c], __ldg(kw + c), dot);
            } else {
                for (int c = 0; c < qk; c++) dot += (int32_t)q8[c] * (int32_t)kr[c];
            }
            logit = __fdiv_rn(__fmul_rn(__int2float_rn(dot), __fmul_rn(sq, sk)), p.scale);
        } else {
            float sacc = 0.0f;
            for (int c = 0; c < qk; c++) sacc = __fadd_rn(sacc, __fmul_rn(qf[c], (float)kr[c]));
            logit = __fdiv_rn(__fmul_rn(sacc, sk), p.scale);
        }
        lg[jj] = logit;
    }
    __syncthreads();

    // Softmax (load.go:127 softmaxInPlace + exp.go:238 expSubSumGeneric).
    float m = -INFINITY;
    for (int jj = tid; jj < n; jj += kAttThreads) m = fmaxf(m, lg[jj]);
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
    for (int w = 1; w < kAttThreads / 32; w++) m = fmaxf(m, red[w]);
    for (int jj = tid; jj < n; jj += kAttThreads) lg[jj] = (float)exp((double)__fsub_rn(lg[jj], m));
    __syncthreads();
    if (tid == 0) {
        float sum = 0.0f;
        for (int jj = 0; jj < n; jj++) sum = __fadd_rn(sum, lg[jj]);
        red[kAttThreads / 32 + 1] = sum;
    }
    __syncthreads();
    const float sum = red[kAttThreads / 32 + 1];
    float *probs = p.probs ? p.probs + (((size_t)b * p.t + i) * p.heads + h) * (size_t)p.nkeys : nullptr;
    for (int jj = tid; jj < n; jj += kAttThreads) {
        int j = jj < len0 ? lo0 + jj : lo1 + (jj - len0);
        float pr = __fdiv_rn(lg[jj], sum);
        if (probs) probs[j] = pr;
        lg[jj] = __fmul_rn(pr, vs[(size_t)j * kvh + kv]);
    }
    __syncthreads();

    // out[d] += float32(w_j · float32(v8_j[d])), key after key (int8kernel.go:60).
    float *out = p.out + (((size_t)b * p.t + i) * p.heads + h) * vd;
    for (int d = tid; d < vd; d += kAttThreads) {
        float acc = 0.0f;
        for (int jj = 0; jj < n; jj++) {
            int j = jj < len0 ? lo0 + jj : lo1 + (jj - len0);
            float c = (float)v8[(size_t)j * vcols + (size_t)kv * vd + d];
            acc = __fadd_rn(acc, __fmul_rn(lg[jj], c));
        }
        out[d] = acc;
    }
}

// ---- v2: one CTA per (stream, query row, group of KV heads) -------------
//
// The KV heads [kg·kvpc, (kg+1)·kvpc) and all their query heads (GQA) share
// one pass over K and V. V's span rows are copied into shared memory with
// cp.async while the logits are computed from 16-byte key loads; the
// softmax's ordered sum runs one thread per head; the ordered output chain
// out[h][d] = Σ_j w_j·v_j[d] runs one thread per (head, d) from shared
// memory. Same operations in the same order as attend_int8_kernel.
constexpr int kAtt2Threads = 128;

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem_src) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <int QKV>  // qk / 16
__global__ void __launch_bounds__(kAtt2Threads, 6) attend_int8_v2_kernel(const __grid_constant__ AttendParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int kg = blockIdx.x, i = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int qk = 16 * QKV;
    const int vd = p.vd, kvh = p.kv_heads, gs = p.heads / kvh;
    const int kvpc = p.kv_per_cta, HB = kvpc * gs;  // query heads of this CTA
    const int kv0 = kg * kvpc, h0 = kv0 * gs;
    const int kcols = kvh * qk, vcols = kvh * vd;

    int nkeys = p.nkeys;
    if (p.nkeys_dev) nkeys = min(p.nkeys_dev[b], p.cap);
    const size_t blk = kv_block(p, b);
    const int8_t *k8 = p.k8 + blk * p.cap * kcols;
    const float *ks = p.ks + blk * p.cap * kvh;
    const int8_t *v8 = p.v8 + blk * p.cap * vcols;
    const float *vs = p.vs + blk * p.cap * kvh;

    int lo0, hi0, lo1, hi1;
    if (p.spans) {
        const int32_t *sp = p.spans + 4 * (size_t)i;
        lo0 = min(max(sp[0], 0), nkeys);
        hi0 = min(max(sp[1], lo0), nkeys);
        lo1 = min(max(sp[2], 0), nkeys);
        hi1 = min(max(sp[3], lo1), nkeys);
    } else {
        lo0 = hi0 = lo1 = 0;
        hi1 = nkeys;
    }
    const int len0 = hi0 - lo0, n = len0 + (hi1 - lo1);
    const int nmax = p.max_keys;
    const int lstride = (nmax + 3) & ~3;  // logit rows 16-byte aligned

    // Shared memory: V rows [kvpc][nmax][vd], logits/weights [HB][lstride],
    // float queries [HB][qk], int8 queries [HB][qk], scales and sums [2·HB].
    int8_t *Vs = reinterpret_cast<int8_t *>(smem);
    float *lg = reinterpret_cast<float *>(smem + (size_t)kvpc * nmax * vd);
    float *qf = lg + (size_t)HB * lstride;
    float *red = qf + HB * qk;  // [HB] sq, [HB] sums
    int8_t *q8 = reinterpret_cast<int8_t *>(red + 2 * HB);

    // 0. V's span rows for this CTA's KV heads, in span order: thread
    //    (row r0 + k·rstep, 16-byte chunk ch) copies asynchronously.
    {
        const int vchunks = vd / 16;
        const int ch = tid % vchunks, r0 = tid / vchunks, rstep = kAtt2Threads / vchunks;
        if (r0 < rstep) {
            for (int c = 0; c < kvpc; c++) {
                const int8_t *src = v8 + (size_t)(kv0 + c) * vd + 16 * ch;
                int8_t *dst = Vs + (size_t)c * nmax * vd + 16 * ch;
                for (int jj = r0; jj < n; jj += rstep) {
                    const int j = jj < len0 ? lo0 + jj : lo1 + (jj - len0);
                    cp_async16(dst + (size_t)jj * vd, src + (size_t)j * vcols);
                }
            }
        }
    }

    // 1. Queries (QuantizeRow per head, int8.go:36).
    for (int e = tid; e < HB * qk; e += kAtt2Threads) {
        const int hl = e / qk, c = e % qk;
        qf[e] = p.q[(((size_t)b * p.t + i) * p.heads + h0 + hl) * qk + c];
    }
    __syncthreads();
    if (p.quant_q) {
        for (int hl = warp; hl < HB; hl += kAtt2Threads / 32) {
            float sq = quantize_chunk_warp(qf + hl * qk, qk, q8 + hl * qk, lane);
            if (lane == 0) red[hl] = sq;
        }
    }
    __syncthreads();

    // 2. Logits: one thread per key, every query head of the CTA.
    for (int jj = tid; jj < n; jj += kAtt2Threads) {
        const int j = jj < len0 ? lo0 + jj : lo1 + (jj - len0);
        for (int c = 0; c < kvpc; c++) {
            const int kv = kv0 + c;
            const uint4 *kr = reinterpret_cast<const uint4 *>(k8 + (size_t)j * kcols + (size_t)kv * qk);
            const float sk = ks[(size_t)j * kvh + kv];
            uint32_t kw[4 * QKV];
#pragma unroll
            for (int v = 0; v < QKV; v++) {
                uint4 w = __ldg(kr + v);
                kw[4 * v] = w.x;
                kw[4 * v + 1] = w.y;
                kw[4 * v + 2] = w.z;
                kw[4 * v + 3] = w.w;
            }
            for (int r = 0; r < gs; r++) {
                const int hl = c * gs + r;
                float logit;
                if (p.quant_q) {
                    const int *qw = reinterpret_cast<const int *>(q8 + hl * qk);
                    int32_t dot = 0;
#pragma unroll
                    for (int w = 0; w < qk / 4; w++) dot = __dp4a(qw[w], (int)kw[w], dot);
                    logit = __fdiv_rn(__fmul_rn(__int2float_rn(dot), __fmul_rn(red[hl], sk)), p.scale);
                } else {
                    const float *qh = qf + hl * qk;
                    float sacc = 0.0f;
#pragma unroll
                    for (int cc = 0; cc < qk; cc++) {
                        const int8_t kb = (int8_t)((kw[cc >> 2] >> (8 * (cc & 3))) & 0xffu);
                        sacc = __fadd_rn(sacc, __fmul_rn(qh[cc], (float)kb));
                    }
                    logit = __fdiv_rn(__fmul_rn(sacc, sk), p.scale);
                }
                lg[(size_t)hl * lstride + jj] = logit;
            }
        }
    }
    __syncthreads();

    // 3. Softmax per head (load.go:127, exp.go:238): max, exp in float64, the
    //    sum in key order by one thread per head, then p and p·sv.
    for (int hl = warp; hl < HB; hl += kAtt2Threads / 32) {
        float m = -INFINITY;
        const float *l = lg + (size_t)hl * lstride;
        for (int jj = lane; jj < n; jj += 32) m = fmaxf(m, l[jj]);
        m = warp_max(m);
        if (lane == 0) red[HB + hl] = m;
    }
    __syncthreads();
    for (int hl = 0; hl < HB; hl++) {
        float *l = lg + (size_t)hl * lstride;
        const float m = red[HB + hl];
        for (int jj = tid; jj < n; jj += kAtt2Threads) l[jj] = (float)exp((double)__fsub_rn(l[jj], m));
    }
    __syncthreads();
    if (tid < HB) {
        const float *l = lg + (size_t)tid * lstride;
        float sum = 0.0f;
        for (int jj = 0; jj < n; jj++) sum = __fadd_rn(sum, l[jj]);
        red[HB + tid] = sum;
    }
    __syncthreads();
    for (int hl = 0; hl < HB; hl++) {
        float *l = lg + (size_t)hl * lstride;
        const float sum = red[HB + hl];
        const int kv = kv0 + hl / gs;
        float *prow = p.probs ? p.probs + (((size_t)b * p.t + i) * p.heads + h0 + hl) * (size_t)p.nkeys : nullptr;
        for (int jj = tid; jj < n; jj += kAtt2Threads) {
            const int j = jj < len0 ? lo0 + jj : lo1 + (jj - len0);
            const float pr = __fdiv_rn(l[jj], sum);
            if (prow) prow[j] = pr;
            l[jj] = __fmul_rn(pr, vs[(size_t)j * kvh + kv]);
        }
    }
    cp_async_wait_all();
    __syncthreads();

    // 4. out[h][d] += float32(w_j · float32(v8_j[d])), key after key.
    for (int e = tid; e < HB * vd; e += kAtt2Threads) {
        const int hl = e / vd, d = e % vd;
        const float *w = lg + (size_t)hl * lstride;
        const int8_t *vcol = Vs + (size_t)(hl / gs) * nmax * vd + d;
        float acc = 0.0f;
        int jj = 0;
        for (; jj + 4 <= n; jj += 4) {
            const float4 w4 = *reinterpret_cast<const float4 *>(w + jj);
            const float c0 = (float)vcol[(size_t)jj * vd], c1 = (float)vcol[(size_t)(jj + 1) * vd];
            const float c2 = (float)vcol[(size_t)(jj + 2) * vd], c3 = (float)vcol[(size_t)(jj + 3) * vd];
            acc = __fadd_rn(acc, __fmul_rn(w4.x, c0));
            acc = __fadd_rn(acc, __fmul_rn(w4.y, c1));
            acc = __fadd_rn(acc, __fmul_rn(w4.z, c2));
            acc = __fadd_rn(acc, __fmul_rn(w4.w, c3));
        }
        for (; jj < n; jj++) acc = __fadd_rn(acc, __fmul_rn(w[jj], (float)vcol[(size_t)jj * vd]));
        p.out[(((size_t)b * p.t + i) * p.heads + h0 + hl) * vd + d] = acc;
    }
}

// ---- any-order kernel (WC_ATTEND_ANY_ORDER) ------------------------------
//
// The same quantities with the float sums in any order: block-wide max and
// sum reductions, expf, and the output accumulated with FMAs by warps that
// each take every 8th key, then added across warps. Integer work (the query
// codes and the int32 logits) stays exact; the float results agree with the
// exact order to a few ulps (within 1e-5 relative).
constexpr int kAttFThreads = 256;
constexpr int kAttFWarps = kAttFThreads / 32;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <int QKV, int GS>  // qk / 16; query heads per KV head
__global__ void __launch_bounds__(kAttFThreads) attend_int8_any_kernel(const __grid_constant__ AttendParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int kg = blockIdx.x, i = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int qk = 16 * QKV;
    constexpr int gs = GS;
    const int vd = p.vd, kvh = p.kv_heads;
    const int kvpc = p.kv_per_cta, HB = kvpc * gs;
    const int kv0 = kg * kvpc, h0 = kv0 * gs;
    const int kcols = kvh * qk, vcols = kvh * vd;

    int nkeys = p.nkeys;
    if (p.nkeys_dev) nkeys = min(p.nkeys_dev[b], p.cap);
    const size_t blk = kv_block(p, b);
    const int8_t *k8 = p.k8 + blk * p.cap * kcols;
    const float *ks = p.ks + blk * p.cap * kvh;
    const int8_t *v8 = p.v8 + blk * p.cap * vcols;
    const float *vs = p.vs + blk * p.cap * kvh;

    int lo0, hi0, lo1, hi1;
    if (p.spans) {
        const int32_t *sp = p.spans + 4 * (size_t)i;
        lo0 = min(max(sp[0], 0), nkeys);
        hi0 = min(max(sp[1], lo0), nkeys);
        lo1 = min(max(sp[2], 0), nkeys);
        hi1 = min(max(sp[3], lo1), nkeys);
    } else {
        lo0 = hi0 = lo1 = 0;
        hi1 = nkeys;
    }
    const int len0 = hi0 - lo0, n = len0 + (hi1 - lo1);
    const int lstride = (p.max_keys + 3) & ~3;

    // Shared memory: weights [HB][lstride], partial outputs [warps][HB·vd],
    // float queries [HB][qk], reductions [warps][HB] x 2, scales [HB],
    // int8 queries [HB][qk].
    float *lg = reinterpret_cast<float *>(smem);
    float *part = lg + (size_t)HB * lstride;
    float *qf = part + (size_t)kAttFWarps * HB * vd;
    float *wred = qf + HB * qk;            // [warps][HB]
    float *hred = wred + kAttFWarps * HB;  // [HB] max, [HB] sum, [HB] sq
    int8_t *q8 = reinterpret_cast<int8_t *>(hred + 3 * HB);

    // L2 prefetch of this CTA's V slices (one row per thread), consumed
    // after the softmax.
    if (p.v_prefetch) {  // the host checked 16-byte alignment of every row slice
        for (int jj = tid; jj < n; jj += kAttFThreads) {
            const int j = jj < len0 ? lo0 + jj : lo1 + (jj - len0);
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(v8 + (size_t)j * vcols + (size_t)kv0 * vd),
                         "r"((uint32_t)(kvpc * vd))
                         : "memory");
        }
    }

    for (int e = tid; e < HB * qk; e += kAttFThreads)
        qf[e] = p.q[(((size_t)b * p.t + i) * p.heads + h0 + e / qk) * qk + e % qk];
    __syncthreads();
    if (p.quant_q) {
        for (int hl = warp; hl < HB; hl += kAttFWarps) {
            float sq = quantize_chunk_warp(qf + hl * qk, qk, q8 + hl * qk, lane);
            if (lane == 0) hred[2 * HB + hl] = sq;
        }
    }
    __syncthreads();

    // Logits, one thread per key.
    for (int jj = tid; jj < n; jj += kAttFThreads) {
        const int j = jj < len0 ? lo0 + jj : lo1 + (jj - len0);
        for (int c = 0; c < kvpc; c++) {
            const int kv = kv0 + c;
            const uint4 *kr = reinterpret_cast<const uint4 *>(k8 + (size_t)j * kcols + (size_t)kv * qk);
            const float sk = ks[(size_t)j * kvh + kv];
            uint32_t kw[4 * QKV];
#pragma unroll
            for (int v = 0; v < QKV; v++) {
                uint4 w = __ldg(kr + v);
                kw[4 * v] = w.x;
                kw[4 * v + 1] = w.y;
                kw[4 * v + 2] = w.z;
                kw[4 * v + 3] = w.w;
            }
#pragma unroll
            for (int r = 0; r < gs; r++) {
                const int hl = c * gs + r;
                float logit;
                if (p.quant_q) {
                    const int *qw = reinterpret_cast<const int *>(q8 + hl * qk);
                    int32_t dot = 0;
#pragma unroll
                    for (int w = 0; w < qk / 4; w++) dot = __dp4a(qw[w], (int)kw[w], dot);
                    logit = __fdiv_rn(__fmul_rn(__int2float_rn(dot), __fmul_rn(hred[2 * HB + hl], sk)), p.scale);
                } else {
                    const float *qh = qf + hl * qk;
                    float sacc = 0.0f;
#pragma unroll
                    for (int cc = 0; cc < qk; cc++)
                        sacc = fmaf(qh[cc], (float)(int8_t)((kw[cc >> 2] >> (8 * (cc & 3))) & 0xffu), sacc);
                    logit = sacc * sk / p.scale;
                }
                lg[(size_t)hl * lstride + jj] = logit;
            }
        }
    }
    __syncthreads();
    // Per-head max and sum, one pass each over the head's logits.
    for (int hl = 0; hl < HB; hl++) {
        const float *l = lg + (size_t)hl * lstride;
        float m = -INFINITY;
        for (int jj = tid; jj < n; jj += kAttFThreads) m = fmaxf(m, l[jj]);
        m = warp_max(m);
        if (lane == 0) wred[warp * HB + hl] = m;
    }
    __syncthreads();
    if (tid < HB) {
        float m = -INFINITY;
        for (int w = 0; w < kAttFWarps; w++) m = fmaxf(m, wred[w * HB + tid]);
        hred[tid] = m;
    }
    __syncthreads();
    for (int hl = 0; hl < HB; hl++) {
        float *l = lg + (size_t)hl * lstride;
        const float m = hred[hl];
        float sm = 0.0f;
        for (int jj = tid; jj < n; jj += kAttFThreads) {
            const float e = expf(l[jj] - m);
            l[jj] = e;
            sm += e;
        }
        sm = warp_sum(sm);
        if (lane == 0) wred[warp * HB + hl] = sm;
    }
    __syncthreads();
    if (tid < HB) {
        float sm = 0.0f;
        for (int w = 0; w < kAttFWarps; w++) sm += wred[w * HB + tid];
        hred[HB + tid] = sm;
    }
    __syncthreads();
    for (int hl = 0; hl < HB; hl++) {
        float *l = lg + (size_t)hl * lstride;
        const float inv = 1.0f / hred[HB + hl];
        const int kv = kv0 + hl / gs;
        float *prow = p.probs ? p.probs + (((size_t)b * p.t + i) * p.heads + h0 + hl) * (size_t)p.nkeys : nullptr;
        for (int jj = tid; jj < n; jj += kAttFThreads) {
            const int j = jj < len0 ? lo0 + jj : lo1 + (jj - len0);
            const float pr = l[jj] * inv;
            if (prow) prow[j] = pr;
            l[jj] = pr * vs[(size_t)j * kvh + kv];
        }
    }
    __syncthreads();

    // Output: each key row of the CTA's V slice is rbw lanes x 4 bytes; a
    // warp covers 32/rbw keys per step and the warps take keys round-robin.
    // Lane word lw holds d = 4·(lw mod (vd/4)) .. +3 of KV head lw / (vd/4).
    const int rbw = kvpc * vd / 4, kps = 32 / rbw;
    const int lw = lane % rbw, ksub = lane / rbw;
    const int c = (4 * lw) / vd, d0 = (4 * lw) % vd;
    float acc[GS][4];
#pragma unroll
    for (int r = 0; r < GS; r++)
#pragma unroll
        for (int q = 0; q < 4; q++) acc[r][q] = 0.0f;
    const float *wrow = lg + (size_t)(c * gs) * lstride;
    const uint32_t *vbase = reinterpret_cast<const uint32_t *>(v8 + (size_t)kv0 * vd) + lw;
    const int kstep = kAttFWarps * kps;
    constexpr int UNR = 8;  // V words in flight per lane
    for (int jb = warp * kps + ksub; jb < n; jb += UNR * kstep) {
        uint32_t vw[UNR];
#pragma unroll
        for (int u = 0; u < UNR; u++) {
            const int jj = jb + u * kstep;
            const int j = jj < len0 ? lo0 + jj : lo1 + (jj - len0);
            vw[u] = jj < n ? __ldg(vbase + (size_t)j * (vcols / 4)) : 0u;
        }
#pragma unroll
        for (int u = 0; u < UNR; u++) {
            const int jj = jb + u * kstep;
            if (jj < n) {
                const float v0 = (float)(int8_t)(vw[u] & 0xffu), v1 = (float)(int8_t)((vw[u] >> 8) & 0xffu);
                const float v2 = (float)(int8_t)((vw[u] >> 16) & 0xffu), v3 = (float)(int8_t)(vw[u] >> 24);
#pragma unroll
                for (int r = 0; r < GS; r++) {
                    const float w = wrow[(size_t)r * lstride + jj];
                    acc[r][0] = fmaf(w, v0, acc[r][0]);
                    acc[r][1] = fmaf(w, v1, acc[r][1]);
                    acc[r][2] = fmaf(w, v2, acc[r][2]);
                    acc[r][3] = fmaf(w, v3, acc[r][3]);
                }
            }
        }
    }
    // Sum the kps key lanes of each word, then the warps.
    for (int o = rbw; o < 32; o <<= 1) {
#pragma unroll
        for (int r = 0; r < GS; r++)
#pragma unroll
            for (int q = 0; q < 4; q++) acc[r][q] += __shfl_xor_sync(0xffffffffu, acc[r][q], o);
    }
    if (ksub == 0) {
#pragma unroll
        for (int r = 0; r < GS; r++)
#pragma unroll
            for (int q = 0; q < 4; q++) part[((size_t)warp * HB + c * gs + r) * vd + d0 + q] = acc[r][q];
    }
    __syncthreads();
    for (int e = tid; e < HB * vd; e += kAttFThreads) {
        float sum = 0.0f;
        for (int w = 0; w < kAttFWarps; w++) sum += part[(size_t)w * HB * vd + e];
        p.out[(((size_t)b * p.t + i) * p.heads + h0) * vd + e] = sum;
    }
}

}  // namespace

size_t attend_any_smem_bytes(const AttendParams &p) {
    const int gs = p.heads / p.kv_heads, HB = p.kv_per_cta * gs;
    const size_t lstride = ((size_t)p.max_keys + 3) & ~(size_t)3;
    return sizeof(float) * (HB * lstride + (size_t)kAttFWarps * HB * p.vd + HB * p.qk + kAttFWarps * HB + 3 * HB) +
           (size_t)HB * p.qk + 16;
}

// The any-order kernel's templates: qk in {16, 32, 48, 64, 128}, query heads
// per KV head in {1, 2, 4, 8}, V row words of the CTA (kv_per_cta·vd/4) in
// {8, 16, 32}; false if the shape has none.
bool attend_any_supported(const AttendParams &p) {
    const int gs = p.heads / p.kv_heads;
    const int rbw = p.kv_per_cta * p.vd / 4;
    const int qkv = p.qk / 16;
    return p.qk % 16 == 0 && (qkv == 1 || qkv == 2 || qkv == 3 || qkv == 4 || qkv == 8) && p.vd % 4 == 0 &&
           (gs == 1 || gs == 2 || gs == 4 || gs == 8) && p.kv_per_cta * gs <= 8 &&
           (rbw == 8 || rbw == 16 || rbw == 32);
}

template <int QKV>
static void (*any_fn(int gs))(AttendParams) {
    switch (gs) {
        case 1: return attend_int8_any_kernel<QKV, 1>;
        case 2: return attend_int8_any_kernel<QKV, 2>;
        case 4: return attend_int8_any_kernel<QKV, 4>;
        default: return attend_int8_any_kernel<QKV, 8>;
    }
}

cudaError_t launch_attend_any(const AttendParams &p, int streams, cudaStream_t st) {
    size_t smem = attend_any_smem_bytes(p);
    const int gs = p.heads / p.kv_heads;
    void (*fn)(AttendParams);
    switch (p.qk / 16) {
        case 1: fn = any_fn<1>(gs); break;
        case 2: fn = any_fn<2>(gs); break;
        case 3: fn = any_fn<3>(gs); break;
        case 4: fn = any_fn<4>(gs); break;
        default: fn = any_fn<8>(gs); break;
    }
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    fn<<<dim3(p.kv_heads / p.kv_per_cta, p.t, streams), kAttFThreads, smem, st>>>(p);
    count_launch();
    return cudaGetLastError();
}

size_t attend_v2_smem_bytes(const AttendParams &p) {
    const int gs = p.heads / p.kv_heads, HB = p.kv_per_cta * gs;
    const size_t lstride = ((size_t)p.max_keys + 3) & ~(size_t)3;
    return (size_t)p.kv_per_cta * p.max_keys * p.vd + sizeof(float) * (HB * lstride + HB * p.qk + 2 * HB) +
           (size_t)HB * p.qk + 16;
}

cudaError_t launch_attend_v2(const AttendParams &p, int streams, cudaStream_t st) {
    size_t smem = attend_v2_smem_bytes(p);
    void (*fn)(AttendParams);
    switch (p.qk / 16) {
        case 1: fn = attend_int8_v2_kernel<1>; break;
        case 2: fn = attend_int8_v2_kernel<2>; break;
        case 3: fn = attend_int8_v2_kernel<3>; break;
        case 4: fn = attend_int8_v2_kernel<4>; break;
        case 5: fn = attend_int8_v2_kernel<5>; break;
        case 6: fn = attend_int8_v2_kernel<6>; break;
        case 7: fn = attend_int8_v2_kernel<7>; break;
        default: fn = attend_int8_v2_kernel<8>; break;
    }
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    fn<<<dim3(p.kv_heads / p.kv_per_cta, p.t, streams), kAtt2Threads, smem, st>>>(p);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_quantize_rows(const float *x, int chunks, int width, int8_t *q, float *s, cudaStream_t st) {
    if (chunks <= 0) return cudaSuccess;
    const int warps = 8;
    quantize_rows_kernel<<<(chunks + warps - 1) / warps, warps * 32, 0, st>>>(x, chunks, width, q, s);
    count_launch();
    return cudaGetLastError();
}

size_t attend_smem_bytes(const AttendParams &p) {
    return sizeof(float) * ((size_t)p.max_keys + kAttThreads / 32 + 2 + p.qk) + (size_t)p.qk + 16;
}

cudaError_t launch_attend(const AttendParams &p, int streams, cudaStream_t st) {
    size_t smem = attend_smem_bytes(p);
    cudaError_t e = cudaFuncSetAttribute(attend_int8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attend_int8_kernel<<<dim3(p.heads, p.t, streams), kAttThreads, smem, st>>>(p);
    count_launch();
    return cudaGetLastError();
}

}  // namespace wb
