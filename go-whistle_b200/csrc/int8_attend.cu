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
    const int8_t *k8 = p.k8 + (size_t)b * p.cap * kcols;
    const float *ks = p.ks + (size_t)b * p.cap * kvh;
    const int8_t *v8 = p.v8 + (size_t)b * p.cap * vcols;
    const float *vs = p.vs + (size_t)b * p.cap * kvh;

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

}  // namespace

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
