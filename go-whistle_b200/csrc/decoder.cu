// decoder.cu — Whistle's text decoder step on the device (wc_decoder_*):
// internal/decoder's Decoder.Extend (decoder.go:252) with the Best()
// hypothesis and the engine's int8 numerics, for many independent streams
// at once, every stream's state resident in HBM.
//
// One step (one token per stream) is, per layer l (decoder.go:446 layer):
//   mhc_in        RMSUnit of the 4-lane stream, int8 fake-quant (mHC φ input)
//   GEMMs         φ_pre, φ_post, φ_res (CQ4, 2048 in)
//   mhc_block_in  mHC heads: sigmoids, Sinkhorn, u = Σ h_pre·lane; engram
//                 gate at the sites; norm_in
//   GEMMs         q, k, v, gate (CQ2)
//   self_prep     causal taps, q/k ZCRMSNorm, RoPE, int8 append of k and v
//   attention     the int8 KV kernel (exact reference order)
//   gate          σ(gate) ⊙ attention
//   GEMM          out_proj
//   post_attn     post_attn_norm, gated residual, cross_norm
//   GEMMs         cross q, cross gate
//   cross_q       cross q norm
//   attention     over the int8 memory
//   gate, GEMM    σ(gate) ⊙, cross out_proj
//   block_out     post_cross_norm, residual, pre_hada norm, HadamardMLP,
//                 mHC mix back into the lanes
// then the lane mean, final norm, the tied head GEMM and the argmax. The
// engram keys and values of both sites are computed once per step before
// the layers (decoder.go:276-285).
//
// Elementwise phases run one 512-thread CTA per stream, one thread per
// model column. Every float32 operation is a separate IEEE rounding in the
// reference's order: this file is compiled with --fmad=false, and the few
// sums whose order matters in float32 (the engram gate's dot product, the
// HadamardMLP's condition and Kronecker products) run sequentially per
// output, as algo-tensor's loops do. The float64 sums of squares of the
// norms run as a tree instead of the reference's four partial sums: a
// float64 sum's rounding can change the float32 result only when it lies
// within about 2^-44 (relative) of a float32 rounding boundary.
//
// Positions live in device memory, so a step can be captured once as a
// CUDA graph and replayed.
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdarg>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "common.cuh"
#include "cq_kernels.cuh"
#include "needle_kernels.cuh"
#include "decoder_beam.cuh"

namespace wb {

namespace {

constexpr int kD = 512;        // model width this build's kernels take
constexpr int kLanes = 4;      // mHC lanes
constexpr int kQK = 48;        // query/key head width
constexpr int kVD = 64;        // value head width
constexpr int kNA = 16, kNB = 32, kRank = 8;  // HadamardMLP
constexpr int kThreads = 512;  // one thread per model column
constexpr float kEps = 1e-6f;  // internal/needle/norm.go:9 normEps as float32

// One layer's device tensors and constants.
struct LayerK {
    const float *g_norm_in, *g_post, *g_pre_hada;  // gains 1 + scale [dim]
    const float *q_taps, *k_taps, *v_taps;         // [taps][width]
    const float *g_qn, *g_kn;                      // [qk]
    const float *d1, *d2, *b2, *d3, *d4;           // [na·nb]
    const float *wa[3], *wb[3];                    // [na][na], [nb][nb]
    const float *cond_v, *cond_u;                  // [dim][rank], [rank][na·nb]
    const float *g_xn, *g_xpost, *g_xqn, *g_xkn;
    const float *b_pre, *b_post, *b_res;
    float gate;    // σ(attn_gate) (block.go:60)
    float xresid;  // σ(cross_gate) (cross.go:148)
    float a_pre, a_post, a_res;
    int lane;      // layer mod lanes: its pre/post offsets (mhc.go:123 laneOffsets)
};

__device__ __forceinline__ float sigm(float x) { return (float)(1.0 / (1.0 + exp(-(double)x))); }

// Σ of one double per thread over the CTA (warp shuffles, then the warps'
// sums in warp order), returned to every thread.
__device__ double block_sum(double v, double *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < nw; w++) t += red[w];
        red[32] = t;
    }
    __syncthreads();
    const double t = red[32];
    __syncthreads();
    return t;
}

__device__ float block_max(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < nw; w++) t = fmaxf(t, red[w]);
        red[32] = t;
    }
    __syncthreads();
    const float t = red[32];
    __syncthreads();
    return t;
}

// norm.go:104 meanSquare of the CTA's row (one value per thread, n values).
__device__ float mean_square(float x, int n, double *red) {
    const double s = block_sum((double)x * (double)x, red);
    return (float)(s / (double)n);
}

// norm.go:60 ZCRMSNorm.Apply on the CTA's row of kD values: (g·x)/rms.
__device__ float zc_norm_row(float x, float g, double *red) {
    const float ms = mean_square(x, kD, red) + kEps;
    const float rms = (float)sqrt((double)ms);
    return __fdiv_rn(g * x, rms);
}

// The same per head of 48 inside one warp: lane l < 24 holds elements l and
// l + 24 of the head. Returns the mean square + eps as float32.
__device__ float head_ms48(float a, float b, int lane) {
    double v = lane < 24 ? (double)a * (double)a + (double)b * (double)b : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return (float)(v / 48.0) + kEps;
}

// int8.go:36 QuantizeRow's rounding of one value with scale s.
__device__ __forceinline__ int8_t quant8(float x, float s) {
    float r = rintf(__fdiv_rn(x, s));
    r = fminf(fmaxf(r, -128.0f), 127.0f);
    return (int8_t)(int)r;
}

// ---------------------------------------------------------------- kernels

// Embedding row × √dim into every lane (decoder.go:270-283, mhc.go:131
// ExpandLanes); the self-attention's key count for this step.
__global__ void __launch_bounds__(kThreads) embed_kernel(const float *__restrict__ row, float scale,
                                                         const int32_t *__restrict__ pos, int32_t *nk_self,
                                                         float *__restrict__ stream) {
    const int s = blockIdx.x, c = threadIdx.x;
    const float v = row[(size_t)s * kD + c] * scale;
#pragma unroll
    for (int k = 0; k < kLanes; k++) stream[((size_t)s * kLanes + k) * kD + c] = v;
    if (c == 0) nk_self[s] = pos[s] + 1;
}

// engram.go:141 ngramHash and IndicesAt for the fed token: the table rows
// the step gathers (−1, a zero row, before order − 1 positions).
__global__ void engram_rows_kernel(const int32_t *__restrict__ tok, const int32_t *__restrict__ tokhist, int ring,
                                   const int32_t *__restrict__ pos, const int32_t *__restrict__ orders, int n_tables,
                                   int slots, int32_t *__restrict__ rows) {
    const int s = blockIdx.x, c = threadIdx.x;
    if (c >= n_tables) return;
    const int p = pos[s], order = orders[c];
    int32_t r = -1;
    if (p + 1 >= order) {
        uint32_t acc = 0x9E3779B9u * (uint32_t)(c + 1);
        for (int j = 0; j < order; j++) {
            uint32_t t = 0;
            if (j == 0)
                t = (uint32_t)tok[s];
            else if (p - j >= 0)
                t = (uint32_t)tokhist[(size_t)s * ring + (p - j) % ring];
            acc = (acc ^ t) * 0x01000193u;
        }
        acc ^= acc >> 15;
        r = c * slots + (int32_t)(acc % (uint32_t)slots);
    }
    rows[(size_t)s * n_tables + c] = r;
}

// cache.go:196-205: the dilated taps over the raw values of the last
// (taps − 1)·dil positions (a ring indexed by position) and this step's.
__global__ void __launch_bounds__(kThreads) engram_taps_kernel(const float *__restrict__ vraw, float *__restrict__ ring,
                                                               const float *__restrict__ taps, int ntaps, int dil,
                                                               const int32_t *__restrict__ pos,
                                                               float *__restrict__ ev) {
    const int s = blockIdx.x, c = threadIdx.x;
    const int p = pos[s], R = (ntaps - 1) * dil;
    const float z = vraw[(size_t)s * kD + c];
    float out = 0.0f;
    out = out + taps[c] * z;
    for (int j = 1; j < ntaps; j++) {
        const int q = p - dil * j;
        if (q < 0) break;
        out = out + taps[(size_t)j * kD + c] * ring[((size_t)s * R + q % R) * kD + c];
    }
    ev[(size_t)s * kD + c] = out;
    if (R > 0) ring[((size_t)s * R + p % R) * kD + c] = z;
}

// mhc.go:193 nx = RMSUnit(stream) over all lanes, then linear.go:108's
// int8 fake-quant of the row (the φ products' shared quantised input).
__global__ void __launch_bounds__(kThreads) mhc_in_kernel(const float *__restrict__ stream, float *__restrict__ xq) {
    __shared__ double red[33];
    __shared__ float redf[33];
    const int s = blockIdx.x, c = threadIdx.x;
    float v[kLanes];
    double sq = 0.0;
#pragma unroll
    for (int k = 0; k < kLanes; k++) {
        v[k] = stream[((size_t)s * kLanes + k) * kD + c];
        sq += (double)v[k] * (double)v[k];
    }
    const double tot = block_sum(sq, red);
    const float ms = (float)(tot / (double)(kLanes * kD)) + kEps;
    const float inv = (float)(1.0 / sqrt((double)ms));
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < kLanes; k++) {
        v[k] = v[k] * inv;
        m = fmaxf(m, fabsf(v[k]));
    }
    m = block_max(m, redf);
    const float sc = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
#pragma unroll
    for (int k = 0; k < kLanes; k++)
        xq[((size_t)s * kLanes + k) * kD + c] = (float)quant8(v[k], sc) * sc;
}

// The layer's three φ products fused with their input (mhc.go:193-205:
// nx = RMSUnit(stream), the Act int8 fake-quant of linear.go:104-114, then
// nx @ φ_pre, φ_post, φ_res): 4 + 4 + 16 rows of 2048 inputs, 4-bit, group
// 128, on the lut kernels' exact arithmetic (lut.go:213-313) without the
// table. With 24 rows a stream, tabulating 32K entries to look up 49K is the
// larger part of the work; each term is instead formed where the table
// would be read, by the table's own expression rint(cb[nib]·(x̂_q·inv_g)),
// so every integer sum, every group term float32(Σ)·(norm·step) and every
// row's sum over the groups in group order is the lut kernel's.
// One CTA per stream, a warp per group of 128: lane l holds the positions
// 4l .. 4l + 3 its row bytes 2l, 2l + 1 index, rotates them with its
// warp by registers and shuffles and forms the 24 rows' terms.
struct PhiViews {
    CqView v[3];   // φ_pre, φ_post, φ_res rows of this layer
    float *y[3];   // [streams][rows]
};
constexpr int kPhiRows = 2 * kLanes + kLanes * kLanes;  // 24
constexpr int kPhiIn = kLanes * kD;                     // 2048
constexpr int kPhiGroups = kPhiIn / 128;                // 16

__global__ void __launch_bounds__(kThreads) mhc_phi_kernel(const float *__restrict__ stream,
                                                           const __grid_constant__ CqShape sh,
                                                           const __grid_constant__ PhiViews pv) {
    __shared__ double red[33];
    __shared__ float redf[33];
    __shared__ __align__(16) float xs[kPhiIn];
    __shared__ float terms[kPhiRows][kPhiGroups];
    __shared__ float cbs[16];  // the levels in shared memory: each lane indexes its own nibble
    const int s = blockIdx.x, c = threadIdx.x, lane = c & 31, g = c >> 5;  // warp g owns group g
    static_assert(kThreads / 32 == kPhiGroups, "a warp per group");
    if (c < 16) cbs[c] = sh.cb[c];
    // Every load of the products first, so their latency passes under the
    // norm: lane l's two index bytes (positions 4l .. 4l + 3 of group g) of
    // each of the 24 rows, and lane r's norm of row r.
    uint32_t wq[kPhiRows];
    float nr = 0.0f;
#pragma unroll
    for (int row = 0; row < kPhiRows; row++) {
        const int k = row < kLanes ? 0 : row < 2 * kLanes ? 1 : 2;
        const int r = row - (k == 0 ? 0 : k == 1 ? kLanes : 2 * kLanes);
        const size_t lrow = (size_t)g * pv.v[k].ld + (size_t)(pv.v[k].row0 + r);
        wq[row] = __ldg(reinterpret_cast<const uint16_t *>(pv.v[k].idx + lrow * 64) + lane);
        if (lane == row) nr = __half2float(pv.v[k].nrm[lrow]);
    }
    // 1. RMSUnit over the lanes, the int8 fake-quant (as mhc_in_kernel).
    float v[kLanes];
    double sq = 0.0;
#pragma unroll
    for (int k = 0; k < kLanes; k++) {
        v[k] = stream[((size_t)s * kLanes + k) * kD + c];
        sq += (double)v[k] * (double)v[k];
    }
    const double tot = block_sum(sq, red);
    const float ms = (float)(tot / (double)(kLanes * kD)) + kEps;
    const float inv = (float)(1.0 / sqrt((double)ms));
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < kLanes; k++) {
        v[k] = v[k] * inv;
        m = fmaxf(m, fabsf(v[k]));
    }
    m = block_max(m, redf);
    const float sc = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
#pragma unroll
    for (int k = 0; k < kLanes; k++) xs[k * kD + c] = (float)quant8(v[k], sc) * sc;
    __syncthreads();
    // 2. x̂ of group g (kernel.go:384 fwht, stage by stage h = 1 .. 64):
    //    lane l holds positions 4l .. 4l + 3; stages 1 and 2 in registers,
    //    4 .. 64 with the lane l ^ (h / 4). Lower element a + b, upper a − b.
    const float4 x4 = *reinterpret_cast<const float4 *>(xs + g * 128 + 4 * lane);
    float x0 = x4.x, x1 = x4.y, x2 = x4.z, x3 = x4.w;
    {
        const float a0 = __fadd_rn(x0, x1), a1 = __fsub_rn(x0, x1), a2 = __fadd_rn(x2, x3), a3 = __fsub_rn(x2, x3);
        x0 = __fadd_rn(a0, a2), x2 = __fsub_rn(a0, a2), x1 = __fadd_rn(a1, a3), x3 = __fsub_rn(a1, a3);
    }
#pragma unroll
    for (int mk = 1; mk < 32; mk <<= 1) {
        const float p0 = __shfl_xor_sync(0xffffffffu, x0, mk), p1 = __shfl_xor_sync(0xffffffffu, x1, mk);
        const float p2 = __shfl_xor_sync(0xffffffffu, x2, mk), p3 = __shfl_xor_sync(0xffffffffu, x3, mk);
        if (lane & mk) {
            x0 = __fsub_rn(p0, x0), x1 = __fsub_rn(p1, x1), x2 = __fsub_rn(p2, x2), x3 = __fsub_rn(p3, x3);
        } else {
            x0 = __fadd_rn(x0, p0), x1 = __fadd_rn(x1, p1), x2 = __fadd_rn(x2, p2), x3 = __fadd_rn(x3, p3);
        }
    }
    // 3. The group bound (4-bit: max |x̂|), 8191/M and the step.
    float mx = fmaxf(fmaxf(fabsf(x0), fabsf(x1)), fmaxf(fabsf(x2), fabsf(x3)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float mm = __fmul_rn(sh.cb_max, mx);
    const float ginv = mm > 0.0f ? __fdiv_rn((float)kLutQ, mm) : 0.0f;
    const float step = __fmul_rn(mm, sh.lut_step);
    // 4. The table's operands x̂_q·inv_g.
    const float a0 = __fmul_rn(x0, ginv), a1 = __fmul_rn(x1, ginv), a2 = __fmul_rn(x2, ginv),
                a3 = __fmul_rn(x3, ginv);
    // 5. Each row's integer sum over the group and its term.
#pragma unroll
    for (int row = 0; row < kPhiRows; row++) {
        const uint32_t w = wq[row];
        int32_t sum = __float2int_rn(__fmul_rn(cbs[w & 15u], a0)) + __float2int_rn(__fmul_rn(cbs[(w >> 4) & 15u], a1)) +
                      __float2int_rn(__fmul_rn(cbs[(w >> 8) & 15u], a2)) +
                      __float2int_rn(__fmul_rn(cbs[(w >> 12) & 15u], a3));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float nrow = __shfl_sync(0xffffffffu, nr, row);
        if (lane == 0) terms[row][g] = __fmul_rn(__int2float_rn(sum), __fmul_rn(nrow, step));
    }
    __syncthreads();
    // 6. Each row's sum of its group terms in group order (lut.go:309).
    if (c < kPhiRows) {
        const int k = c < kLanes ? 0 : c < 2 * kLanes ? 1 : 2;
        const int r = c - (k == 0 ? 0 : k == 1 ? kLanes : 2 * kLanes);
        const int rows = k == 2 ? kLanes * kLanes : kLanes;
        float acc = 0.0f;
        for (int q = 0; q < kPhiGroups; q++) acc = __fadd_rn(acc, terms[c][q]);
        pv.y[k][(size_t)s * rows + r] = acc;
    }
}

// mhc.go:316 sinkhornExp / :374 sinkhornLog: h_res = sinkhorn(a_res·(nx @
// φ_res) + b_res), one stream per warp. Lane e (and its mirror e + 16)
// holds entry (e / 4, e % 4); each row or column sum is formed by every
// lane of that row or column from shuffled values in the reference's order
// (index order from 0), then the lane divides its own entry. Only the mix at
// the layer's end reads h_res, so it runs beside the block.
__global__ void sinkhorn_kernel(const LayerK L, const float *__restrict__ phi_res, float *__restrict__ hr,
                                int streams) {
    const int lane = threadIdx.x & 31;
    const int s = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (s >= streams) return;  // whole warps
    constexpr int n = kLanes;
    const int e = lane & 15, r = e >> 2, c = e & 3;
    const unsigned full = 0xffffffffu;
    const float t = L.a_res * phi_res[(size_t)s * n * n + e];
    const float k = t + L.b_res[e];
    float lo = k, hi = k;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
        lo = fminf(lo, __shfl_xor_sync(full, lo, o, 16));
        hi = fmaxf(hi, __shfl_xor_sync(full, hi, o, 16));
    }
    const double spread = (double)hi - (double)lo;
    float out;
    if (!(isinf(spread) || isnan(spread) || spread + 2.0 * 20.0 * log((double)n) > 700.0)) {
        double v = exp((double)k - (double)hi);
        for (int it = 0; it < 20; it++) {
            double sum = 0.0;
#pragma unroll
            for (int j = 0; j < n; j++) sum += __shfl_sync(full, v, r * n + j, 16);
            v = v / sum;
            sum = 0.0;
#pragma unroll
            for (int j = 0; j < n; j++) sum += __shfl_sync(full, v, j * n + c, 16);
            v = v / sum;
        }
        out = (float)v;
    } else {
        float x = k;
        for (int it = 0; it < 20; it++) {
            for (int phase = 0; phase < 2; phase++) {
                float vals[n];
#pragma unroll
                for (int j = 0; j < n; j++) vals[j] = __shfl_sync(full, x, phase == 0 ? r * n + j : j * n + c, 16);
                float m = -INFINITY;
#pragma unroll
                for (int j = 0; j < n; j++) m = fmaxf(m, vals[j]);
                if (isinf(m)) m = 0.0f;
                float sum = 0.0f;
#pragma unroll
                for (int j = 0; j < n; j++) sum += (float)exp((double)(vals[j] - m));
                x = x - (m + (float)log((double)sum));
            }
        }
        out = (float)exp((double)x);
    }
    if (lane < 16) hr[(size_t)s * n * n + e] = out;
}

// mhc.go:241 logits and :205-221 (sigmoids, u), then block.go:148
// run up to the attention: the engram gate (block.go:231 applyEngram) at a
// site, and norm_in.
__global__ void __launch_bounds__(kThreads)
    mhc_block_in_kernel(const LayerK L, const float *__restrict__ stream, const float *__restrict__ phi_pre,
                        const float *__restrict__ phi_post, const float *__restrict__ phi_res,
                        const float *__restrict__ ek, const float *__restrict__ ev, float *__restrict__ u_out,
                        float *__restrict__ h_out, float *__restrict__ n_out, float *__restrict__ hp_out) {
    __shared__ double red[33];
    __shared__ float pre[kLanes], post[kLanes];
    __shared__ float ux[kD], uk[kD];
    __shared__ float alpha;
    const int s = blockIdx.x, c = threadIdx.x, lane = c & 31, warp = c >> 5;
    if (warp == 0) {
        if (lane < kLanes) {
            const float pre_off = lane == L.lane ? 4.0f : -4.0f, post_off = lane == L.lane ? 0.0f : -4.0f;
            const float t = L.a_pre * phi_pre[(size_t)s * kLanes + lane];
            pre[lane] = sigm(t + L.b_pre[lane] + pre_off);
            const float t2 = L.a_post * phi_post[(size_t)s * kLanes + lane];
            post[lane] = 2.0f * sigm(t2 + L.b_post[lane] + post_off);
        }
    }
    __syncthreads();
    float u = 0.0f;
#pragma unroll
    for (int k = 0; k < kLanes; k++) u = u + pre[k] * stream[((size_t)s * kLanes + k) * kD + c];
    float h = u;
    if (ek) {
        const float e = ek[(size_t)s * kD + c];
        const float msx = mean_square(h, kD, red) + kEps;
        const float msk = mean_square(e, kD, red) + kEps;
        ux[c] = h * (float)(1.0 / sqrt((double)msx));
        uk[c] = e * (float)(1.0 / sqrt((double)msk));
        __syncthreads();
        if (c == 0) {
            float dp = 0.0f;  // algo-tensor DotProduct, index order
            for (int i = 0; i < kD; i++) dp = dp + ux[i] * uk[i];
            alpha = sigm(__fdiv_rn(dp, (float)sqrt((double)kD)));
        }
        __syncthreads();
        h = h + alpha * ev[(size_t)s * kD + c];
    }
    const float n = zc_norm_row(h, L.g_norm_in[c], red);
    u_out[(size_t)s * kD + c] = u;
    h_out[(size_t)s * kD + c] = h;
    n_out[(size_t)s * kD + c] = n;
    if (c < kLanes) hp_out[(size_t)s * kLanes + c] = post[c];
}

// cache.go:78-139 Attention.Extend up to the attention: the causal taps
// over the raw q/k/v history (cache.go:185 extendTaps), the per-head q/k
// ZCRMSNorm and RoPE at the position (attention.go:300 normRotate), and the
// int8 append of the key and value row (int8.go:125 Append).
__global__ void __launch_bounds__(kThreads)
    self_prep_kernel(const LayerK L, const float *__restrict__ q, const float *__restrict__ k,
                     const float *__restrict__ v, float *__restrict__ hist, int ntaps, int heads, int kv_heads,
                     const int32_t *__restrict__ pos, const float *__restrict__ rcos, const float *__restrict__ rsin,
                     int8_t *__restrict__ k8, float *__restrict__ ks, int8_t *__restrict__ v8,
                     float *__restrict__ vs, int cap, float *__restrict__ qo) {
    extern __shared__ float z[];  // [qw + kw + vw]
    const int s = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int qw = heads * kQK, kw = kv_heads * kQK, vw = kv_heads * kVD, W = qw + kw + vw;
    const int p = pos[s], th = ntaps - 1;
    for (int col = t; col < W; col += blockDim.x) {
        float raw;
        const float *tap;
        int tw, tc;
        if (col < qw) {
            raw = q[(size_t)s * qw + col], tap = L.q_taps, tw = qw, tc = col;
        } else if (col < qw + kw) {
            raw = k[(size_t)s * kw + col - qw], tap = L.k_taps, tw = kw, tc = col - qw;
        } else {
            raw = v[(size_t)s * vw + col - qw - kw], tap = L.v_taps, tw = vw, tc = col - qw - kw;
        }
        float out = 0.0f;
        out = out + tap[tc] * raw;
        for (int j = 1; j < ntaps; j++) {
            if (p - j < 0) break;
            out = out + tap[(size_t)j * tw + tc] * hist[((size_t)s * th + (p - j) % th) * W + col];
        }
        if (th > 0) hist[((size_t)s * th + p % th) * W + col] = raw;
        z[col] = out;
    }
    __syncthreads();
    // q heads, then k heads: a warp per head.
    const int nh = heads + kv_heads;
    const int half = kQK / 2;
    for (int hd = warp; hd < nh; hd += blockDim.x >> 5) {
        const int base = hd < heads ? hd * kQK : qw + (hd - heads) * kQK;
        const float *g = hd < heads ? L.g_qn : L.g_kn;
        float a = 0.0f, b = 0.0f;
        if (lane < half) {
            a = z[base + lane];
            b = z[base + lane + half];
        }
        const float rms = (float)sqrt((double)head_ms48(a, b, lane));
        if (lane < half) {
            a = __fdiv_rn(g[lane] * a, rms);
            b = __fdiv_rn(g[lane + half] * b, rms);
            const float cs = rcos[(size_t)p * half + lane], sn = rsin[(size_t)p * half + lane];
            const float ac = a * cs, bs = b * sn, bc = b * cs, as = a * sn;
            z[base + lane] = ac - bs;
            z[base + lane + half] = bc + as;
        }
    }
    __syncthreads();
    for (int col = t; col < qw; col += blockDim.x) qo[(size_t)s * qw + col] = z[col];
    // int8 codes and scales of the new key (heads of 48) and value (64) row.
    for (int hd = warp; hd < 2 * kv_heads; hd += blockDim.x >> 5) {
        const bool isk = hd < kv_heads;
        const int w = isk ? kQK : kVD, h2 = isk ? hd : hd - kv_heads;
        const int base = isk ? qw + h2 * kQK : qw + kw + h2 * kVD;
        const float a = lane < w / 2 ? z[base + lane] : 0.0f, b = lane < w / 2 ? z[base + lane + w / 2] : 0.0f;
        float m = fmaxf(fabsf(a), fabsf(b));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float sc = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
        const size_t rowi = (size_t)s * cap + p;
        if (lane < w / 2) {
            int8_t *dst = isk ? k8 + rowi * kw + h2 * kQK : v8 + rowi * vw + h2 * kVD;
            dst[lane] = quant8(a, sc);
            dst[lane + w / 2] = quant8(b, sc);
        }
        if (lane == 0) (isk ? ks : vs)[rowi * kv_heads + h2] = sc;
    }
}

// attention.go:243 output's gate: out ⊙ σ(gate).
__global__ void __launch_bounds__(kThreads) gate_kernel(float *__restrict__ out, const float *__restrict__ g, int w) {
    const int s = blockIdx.x;
    for (int i = threadIdx.x; i < w; i += blockDim.x) {
        const size_t o = (size_t)s * w + i;
        out[o] = out[o] * sigm(g[o]);
    }
}

// block.go:193-199 post_attn_norm and the gated residual, then cross.go:212
// cross_norm of the result (the cross-attention's input).
__global__ void __launch_bounds__(kThreads) post_attn_kernel(const LayerK L, const float *__restrict__ a,
                                                             float *__restrict__ h, float *__restrict__ x) {
    __shared__ double red[33];
    const int s = blockIdx.x, c = threadIdx.x;
    const float an = zc_norm_row(a[(size_t)s * kD + c], L.g_post[c], red);
    const float hv = h[(size_t)s * kD + c] + L.gate * an;
    h[(size_t)s * kD + c] = hv;
    x[(size_t)s * kD + c] = zc_norm_row(hv, L.g_xn[c], red);
}

// cross.go:218 the cross-attention's q norm, per head.
__global__ void __launch_bounds__(kThreads) cross_q_kernel(const LayerK L, const float *__restrict__ q, int heads,
                                                           float *__restrict__ qo) {
    const int s = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, half = kQK / 2;
    for (int hd = warp; hd < heads; hd += blockDim.x >> 5) {
        const size_t base = (size_t)s * heads * kQK + hd * kQK;
        float a = 0.0f, b = 0.0f;
        if (lane < half) {
            a = q[base + lane];
            b = q[base + lane + half];
        }
        const float rms = (float)sqrt((double)head_ms48(a, b, lane));
        if (lane < half) {
            qo[base + lane] = __fdiv_rn(L.g_xqn[lane] * a, rms);
            qo[base + lane + half] = __fdiv_rn(L.g_xqn[lane + half] * b, rms);
        }
    }
}

// hadamard.go:300 kronApply (+ :281 mix's permutation for stages 0 and 1)
// of z (shared, n = 512) into dst (shared): Yᵀ = bᵀ·Zᵀ, then out = aᵀ·Y,
// each output a sequential sum as tensor.MatMulTransB forms it. Y is kept
// as Y[j][i] = Yᵀ[i][j] (na × nb), and the lanes of a warp take consecutive
// i (first product) and l2 (second), so every shared load is a broadcast
// or 32 consecutive words: no bank conflicts.
__device__ void kron_mix(const float *__restrict__ wa, const float *__restrict__ wb, const int *__restrict__ perm,
                         const float *z, float *Y, float *kb, float *dst) {
    const int t = threadIdx.x;
    {
        const int j = t / kNB, i = t % kNB;  // Yᵀ[i][j], i < nb, j < na
        float acc = 0.0f;
        for (int l = 0; l < kNB; l++) acc = acc + wb[l * kNB + i] * z[j * kNB + l];
        Y[j * kNB + i] = acc;
    }
    __syncthreads();
    {
        const int kk = t / kNB, l2 = t % kNB;  // out[kk][l2], kk < na, l2 < nb
        float acc = 0.0f;
        for (int l = 0; l < kNA; l++) acc = acc + wa[l * kNA + kk] * Y[l * kNB + l2];
        (perm ? kb : dst)[t] = acc;
    }
    __syncthreads();
    if (perm) {
        dst[t] = kb[perm[t]];
        __syncthreads();
    }
}

// cross.go:236-248 post_cross_norm, the σ(cross_gate) residual; block.go:
// 203-214 pre_hada norm, HadamardMLP (hadamard.go:211 rows), the MLP
// residual; mhc.go:229 y = block(u) − u and :270 mix into the lanes.
__global__ void __launch_bounds__(kThreads)
    block_out_kernel(const LayerK L, const int *__restrict__ p1, const int *__restrict__ p2,
                     const float *__restrict__ cy, const float *__restrict__ h, const float *__restrict__ u,
                     const float *__restrict__ hp, const float *__restrict__ hr, float *__restrict__ stream) {
    __shared__ double red[33];
    __shared__ float pv[kD], z[kD], o[kD], yT[kD], kb[kD];
    __shared__ float lg[kRank];
    __shared__ float cv[kD * kRank];                         // cond_v
    __shared__ float wa_s[3][kNA * kNA], wb_s[3][kNB * kNB];  // Kronecker factors
    const int s = blockIdx.x, c = threadIdx.x;
    for (int i = c; i < kD * kRank; i += kThreads) cv[i] = L.cond_v[i];
    for (int st = 0; st < 3; st++) {
        for (int i = c; i < kNA * kNA; i += kThreads) wa_s[st][i] = L.wa[st][i];
        for (int i = c; i < kNB * kNB; i += kThreads) wb_s[st][i] = L.wb[st][i];
    }
    const float y = L.xresid * zc_norm_row(cy[(size_t)s * kD + c], L.g_xpost[c], red);
    const float h2 = h[(size_t)s * kD + c] + y;
    const float p = zc_norm_row(h2, L.g_pre_hada[c], red);
    pv[c] = p;
    __syncthreads();
    // cond = 1 + softmax(p @ cond_v) @ cond_u
    if (c < kRank) {
        float acc = 0.0f;
        for (int i = 0; i < kD; i++) acc = acc + pv[i] * cv[i * kRank + c];
        lg[c] = acc;
    }
    __syncthreads();
    if (c == 0) {  // load.go:127 softmaxInPlace with exp.go:238 expSubSumGeneric
        float m = -INFINITY;
        for (int r = 0; r < kRank; r++) m = fmaxf(m, lg[r]);
        float sum = 0.0f;
        for (int r = 0; r < kRank; r++) {
            const float e = (float)exp((double)(lg[r] - m));
            lg[r] = e;
            sum = sum + e;
        }
        for (int r = 0; r < kRank; r++) lg[r] = __fdiv_rn(lg[r], sum);
    }
    __syncthreads();
    float cond = 0.0f;
    for (int r = 0; r < kRank; r++) cond = cond + lg[r] * L.cond_u[r * kD + c];
    cond = cond + 1.0f;
    z[c] = L.d1[c] * p;
    __syncthreads();
    kron_mix(wa_s[0], wb_s[0], p1, z, yT, kb, o);
    {
        const float a2 = L.d2[c] * cond * o[c] + L.b2[c];
        z[c] = a2 * sigm(a2);
    }
    __syncthreads();
    kron_mix(wa_s[1], wb_s[1], p2, z, yT, kb, o);
    z[c] = L.d3[c] * o[c];
    __syncthreads();
    kron_mix(wa_s[2], wb_s[2], nullptr, z, yT, kb, o);
    const float m = o[c] * L.d4[c] + h2;
    const float Y = m - u[(size_t)s * kD + c];
    float st[kLanes], out[kLanes];
#pragma unroll
    for (int b = 0; b < kLanes; b++) st[b] = stream[((size_t)s * kLanes + b) * kD + c];
#pragma unroll
    for (int a = 0; a < kLanes; a++) {
        float acc = 0.0f;
#pragma unroll
        for (int b = 0; b < kLanes; b++) acc = acc + hr[(size_t)s * kLanes * kLanes + a * kLanes + b] * st[b];
        out[a] = acc + hp[(size_t)s * kLanes + a] * Y;
    }
#pragma unroll
    for (int a = 0; a < kLanes; a++) stream[((size_t)s * kLanes + a) * kD + c] = out[a];
}

// mhc.go:140 CollapseLanes and decoder.go:510 final_norm: the head's input.
__global__ void __launch_bounds__(kThreads) final_kernel(const float *__restrict__ stream, const float *__restrict__ g,
                                                         float *__restrict__ fin) {
    __shared__ double red[33];
    const int s = blockIdx.x, c = threadIdx.x;
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < kLanes; k++) m = m + stream[((size_t)s * kLanes + k) * kD + c];
    m = __fdiv_rn(m, (float)kLanes);
    fin[(size_t)s * kD + c] = zc_norm_row(m, g[c], red);
}

// The step's bookkeeping: the fed token into the engram history, the
// position forward.
__global__ void advance_kernel(const int32_t *__restrict__ tok, int32_t *__restrict__ tokhist, int ring,
                               int32_t *__restrict__ pos, int streams) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= streams) return;
    const int p = pos[s];
    if (ring > 0) tokhist[(size_t)s * ring + p % ring] = tok[s];
    pos[s] = p + 1;
}

// cross.go:188-201: the memory keys' per-head norm and the int8 codes and
// scales of keys and values, one CTA per (stream, frame) row, a warp per
// head.
__global__ void __launch_bounds__(256) xmem_kernel(const float *__restrict__ kp, const float *__restrict__ vp,
                                                   const float *__restrict__ g_xkn, int heads,
                                                   int8_t *__restrict__ k8, float *__restrict__ ks,
                                                   int8_t *__restrict__ v8, float *__restrict__ vs) {
    const size_t r = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, half = kQK / 2;
    for (int hd = warp; hd < heads; hd += blockDim.x >> 5) {
        const size_t kb = r * heads * kQK + hd * kQK;
        float a = 0.0f, b = 0.0f;
        if (lane < half) {
            a = kp[kb + lane];
            b = kp[kb + lane + half];
        }
        const float rms = (float)sqrt((double)head_ms48(a, b, lane));
        if (lane < half) {
            a = __fdiv_rn(g_xkn[lane] * a, rms);
            b = __fdiv_rn(g_xkn[lane + half] * b, rms);
        }
        float m = fmaxf(fabsf(a), fabsf(b));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float sc = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
        if (lane < half) {
            k8[kb + lane] = quant8(a, sc);
            k8[kb + lane + half] = quant8(b, sc);
        }
        if (lane == 0) ks[r * heads + hd] = sc;
        const size_t vb = r * heads * kVD + hd * kVD;
        a = vp[vb + lane];
        b = vp[vb + lane + 32];
        m = fmaxf(fabsf(a), fabsf(b));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        sc = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
        v8[vb + lane] = quant8(a, sc);
        v8[vb + lane + 32] = quant8(b, sc);
        if (lane == 0) vs[r * heads + hd] = sc;
    }
}

// greedy.go:58-66: record the argmax (already in tok) unless the stream has
// ended; EOS ends it.
__global__ void record_kernel(const int32_t *__restrict__ tok, int eos, int max_out, int32_t *__restrict__ tokens,
                              int32_t *__restrict__ counts, int32_t *__restrict__ eos_hit, int32_t *__restrict__ done,
                              int streams) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= streams || done[s]) return;
    const int t = tok[s];
    if (t == eos) {
        done[s] = 1;
        eos_hit[s] = 1;
        return;
    }
    const int n = counts[s];
    if (n < max_out) tokens[(size_t)s * max_out + n] = t;
    counts[s] = n + 1;
}

__global__ void greedy_init_kernel(int32_t *tok, int bos, int32_t *tokens, int max_out, int32_t *counts,
                                   int32_t *eos_hit, int32_t *done, int streams) {
    const int s = blockIdx.x;
    if (s >= streams) return;
    for (int i = threadIdx.x; i < max_out; i += blockDim.x) tokens[(size_t)s * max_out + i] = -1;
    if (threadIdx.x == 0) {
        tok[s] = bos;
        counts[s] = 0;
        eos_hit[s] = 0;
        done[s] = 0;
    }
}

__global__ void fill_kernel(int32_t *p, int32_t v, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

// ----------------------------------------------------- the head's choice
//
// The greedy step needs only the argmax of the tied head's logits
// (greedy.go:182), not the logits. The head (vocab × 512, CQ4) is by far
// the largest product of a step, so it runs on the tensor cores
// (WC_GEMM_TENSOR_CORES: fp16 operands, error bound stated in the header),
// and only the rows that can still be the argmax are recomputed with the
// lut kernel's exact arithmetic. Each approximate logit y_r lies within
// B_r of the lut value l_r:
//   |y_r − l_r| ≤ |y_r − e_r| + |e_r − l_r|   (e_r: the exact real product)
//   |y_r − e_r| ≤ (2^-10 + (K + log2 G + 6)·2^-24)·A_r + 2^-37·(G·max|x|·Σ|ŵ_r| + max|ŵ|·Σ|x̂|)
//   |e_r − l_r| ≤ Σ_g n_rg/√G · (G/2)·M_g/8191 + (groups + 6)·2^-24·A_r
// with A_r = Σ_k |x̂_k||ŵ_rk| ≤ ‖x̂‖·‖ŵ_r‖ = √G·‖x‖·‖ŵ_r‖ (Cauchy-Schwarz),
// Σ|ŵ_r| ≤ √K‖ŵ_r‖, Σ|x̂| ≤ √K‖x̂‖, M_g = max|cb|·max_g|x̂| ≤ max|cb|·‖x_g‖₁,
// and a margin of 1.25 for the float32 evaluation of the bound. With
// m = max_r (y_r − B_r) ≤ max_r l_r, every row whose l_r can reach the
// maximum has y_r + B_r ≥ m: those candidates (a handful) are rescored
// exactly, and the largest at its first index is the reference's argmax,
// bit for bit. More than kMaxCand candidates, or a non-finite value, and
// the stream's whole row is computed exactly instead.
constexpr int kMaxCand = 64;
constexpr int kBeamMaxCand = 64;  // candidates a beam step asks per row
constexpr int kHeadG = 128, kHeadBits = 4, kHeadGroups = kD / kHeadG, kHeadGB = kHeadG * kHeadBits / 8;

// ‖ŵ_r‖₂ (rounded up) and max_g |n_rg| of every head row.
__global__ void head_rownorm_kernel(const __grid_constant__ CqShape s, const CqView v, float *__restrict__ wn,
                                    float *__restrict__ nmax) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= v.out) return;
    double acc = 0.0;
    float nm = 0.0f;
    for (int g = 0; g < s.groups; g++) {
        const size_t lrow = (size_t)g * v.ld + (size_t)(v.row0 + r);
        const double n = fabs((double)__half2float(v.nrm[lrow]));
        nm = fmaxf(nm, (float)n);
        double c2 = 0.0;
        for (int k = 0; k < s.group; k++) {
            const int bit = k * s.bits;
            const uint32_t code = (v.idx[lrow * s.gb + (bit >> 3)] >> (bit & 7)) & ((1u << s.bits) - 1u);
            c2 += (double)s.cb[code] * (double)s.cb[code];
        }
        acc += n * n * c2 / (double)s.group;
    }
    wn[r] = (float)(sqrt(acc) * (1.0 + 1e-6));
    nmax[r] = nm;
}

// Candidates of each stream's argmax from the approximate logits y.
__global__ void __launch_bounds__(kThreads)
    head_screen_kernel(const float *__restrict__ y, int vocab, const float *__restrict__ x, const float *__restrict__ wn,
                       const float *__restrict__ nmax, float cb_max, float wmax, int32_t *__restrict__ cand,
                       int32_t *__restrict__ cnt) {
    __shared__ double red[33];
    __shared__ float redf[33];
    __shared__ int count;
    __shared__ int bad;
    const int s = blockIdx.x, t = threadIdx.x;
    const float xv = x[(size_t)s * kD + t];
    const double sq = block_sum((double)xv * (double)xv, red);
    const double l1 = block_sum(fabs((double)xv), red);
    const float xmax = block_max(fabsf(xv), redf);
    const double sqrtG = sqrt((double)kHeadG), sqrtK = sqrt((double)kD);
    const double gamma = 0x1p-10 + ((double)kD + 7.0 + 6.0) * 0x1p-24 + (kHeadGroups + 6) * 0x1p-24;
    const double xh = sqrtG * sqrt(sq);
    const float c1 = (float)(1.25 * (gamma * xh + 0x1p-37 * kHeadG * (double)xmax * sqrtK));
    const float c2 = (float)(1.25 * 0.5 * sqrtG / 8191.0 * (double)cb_max * l1);
    const float c3 = (float)(1.25 * 0x1p-37 * (double)wmax * sqrtK * xh);
    if (t == 0) {
        count = 0;
        bad = !(isfinite(sq) && isfinite(l1));
    }
    const float *yr = y + (size_t)s * vocab;
    float m = -INFINITY;
    int nonfinite = 0;
    for (int r = t; r < vocab; r += kThreads) {
        const float v = yr[r];
        if (!isfinite(v)) nonfinite = 1;
        m = fmaxf(m, v - (c1 * wn[r] + c2 * nmax[r] + c3));
    }
    if (nonfinite) bad = 1;
    // Block max of m (−inf allowed).
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((t & 31) == 0) redf[t >> 5] = m;
    __syncthreads();
    if (t == 0) {
        float mm = -INFINITY;
        for (int w = 0; w < kThreads / 32; w++) mm = fmaxf(mm, redf[w]);
        redf[32] = mm;
    }
    __syncthreads();
    m = redf[32];
    for (int r = t; r < vocab; r += kThreads) {
        if (yr[r] + (c1 * wn[r] + c2 * nmax[r] + c3) >= m) {
            const int k = atomicAdd(&count, 1);
            if (k < kMaxCand) cand[(size_t)s * kMaxCand + k] = r;
        }
    }
    __syncthreads();
    if (t == 0) cnt[s] = (bad || count > kMaxCand || count == 0) ? -1 : count;
}

// The lut kernel's exact value of head row r for the activation whose
// tables are tab (nibble tables [2·256][16]) and steps, computed by one
// warp: lane l sums the 16 nibbles of its 8 index bytes, eight lanes make
// a group's exact integer sum, and the group terms are added in order.
__device__ float head_row_exact(const CqView &v, int r, const int16_t *tab, const float *steps, int lane) {
    const int g = lane >> 3, off = (lane & 7) * 8;
    const size_t lrow = (size_t)g * v.ld + (size_t)(v.row0 + r);
    const uint2 w = __ldg(reinterpret_cast<const uint2 *>(v.idx + lrow * kHeadGB + off));
    int32_t sum = 0;
    const uint32_t ws[2] = {w.x, w.y};
#pragma unroll
    for (int b = 0; b < 8; b++) {
        const uint32_t byte = (ws[b >> 2] >> (8 * (b & 3))) & 0xffu;
        const int pos = g * kHeadGB + off + b;
        sum += tab[(2 * pos) * 16 + (byte & 15u)];
        sum += tab[(2 * pos + 1) * 16 + (byte >> 4)];
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    const float coef = __half2float(v.nrm[lrow]) * steps[g];
    const float term = (float)sum * coef;
    float acc = 0.0f;
#pragma unroll
    for (int gg = 0; gg < kHeadGroups; gg++) acc = acc + __shfl_sync(0xffffffffu, term, gg * 8);
    return acc;
}

// head_argmax's key (decode_head.cu): the largest key is the largest value
// at its first index; NaN keys are 0.
__device__ __forceinline__ unsigned long long pick_key(float v, int i) {
    if (v != v) return 0ull;
    const uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
    const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)ord << 32) | (uint32_t)(0xffffffffu - (uint32_t)i);
}

// Exact rescoring and the choice, one CTA per stream. mode 0: the
// screen's candidates (or, for cnt = −1, every row, its exact logits
// written to y); mode 1: the fixed list (the language tokens: the largest
// at its first position in the list, greedy.go:81).
__global__ void __launch_bounds__(kThreads)
    head_pick_kernel(const __grid_constant__ CqShape sh, const CqView v, const float *__restrict__ x,
                     const int32_t *__restrict__ cand, const int32_t *__restrict__ cnt, const int32_t *__restrict__ list,
                     int nlist, int mode, float *__restrict__ y, int32_t *__restrict__ tok, int32_t *__restrict__ lang) {
    __shared__ float xs[kD];
    __shared__ float steps[kHeadGroups], invs[kHeadGroups];
    __shared__ __align__(16) int16_t tab[2 * kHeadGB * kHeadGroups * 16];
    __shared__ unsigned long long bestw[kThreads / 32];
    __shared__ int nan0;
    const int s = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    // Rotation (kernel.go:384 fwht per group, stage by stage), bounds and
    // tables exactly as cq_lut.cu builds them.
    xs[t] = x[(size_t)s * kD + t];
    if (t == 0) nan0 = 0;
    __syncthreads();
    for (int h = 1; h < kHeadG; h <<= 1) {
        if (t < kD / 2) {
            const int g = t / (kHeadG / 2), q = t % (kHeadG / 2);
            const int j = g * kHeadG + (q / h) * 2 * h + (q % h);
            const float a = xs[j], c = xs[j + h];
            xs[j] = __fadd_rn(a, c);
            xs[j + h] = __fsub_rn(a, c);
        }
        __syncthreads();
    }
    if (warp < kHeadGroups) {
        float mx = 0.0f;
        for (int q = lane; q < kHeadG; q += 32) mx = fmaxf(mx, fabsf(xs[warp * kHeadG + q]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) {
            const float m = __fmul_rn(sh.cb_max, mx);
            invs[warp] = m > 0.0f ? __fdiv_rn((float)kLutQ, m) : 0.0f;
            steps[warp] = __fmul_rn(m, sh.lut_step);
        }
    }
    __syncthreads();
    for (int e = t; e < kD * 16; e += kThreads) {  // 4-bit: one nibble position per column
        const int pos = e >> 4, c = e & 15;
        const float a = __fmul_rn(xs[pos], invs[pos / kHeadG]);
        tab[e] = (int16_t)__float2int_rn(__fmul_rn(sh.cb[c], a));
    }
    __syncthreads();
    unsigned long long best = 0ull;
    const int n = cnt ? cnt[s] : 0;
    if (mode == 1) {
        for (int k = warp; k < nlist; k += kThreads / 32) {
            const float val = head_row_exact(v, list[k], tab, steps, lane);
            const unsigned long long key = pick_key(val, k);
            best = key > best ? key : best;
        }
    } else if (n >= 0) {
        for (int k = warp; k < n; k += kThreads / 32) {
            const int r = cand[(size_t)s * kMaxCand + k];
            const float val = head_row_exact(v, r, tab, steps, lane);
            const unsigned long long key = pick_key(val, r);
            best = key > best ? key : best;
        }
    } else {
        for (int r = warp; r < v.out; r += kThreads / 32) {
            const float val = head_row_exact(v, r, tab, steps, lane);
            if (lane == 0) y[(size_t)s * v.out + r] = val;
            if (r == 0 && val != val) nan0 = 1;
            const unsigned long long key = pick_key(val, r);
            best = key > best ? key : best;
        }
    }
    if (lane == 0) bestw[warp] = best;
    __syncthreads();
    if (t == 0) {
        unsigned long long b = 0ull;
        for (int w = 0; w < kThreads / 32; w++) b = bestw[w] > b ? bestw[w] : b;
        const int i = (int)(0xffffffffu - (uint32_t)(b & 0xffffffffull));
        int chosen = b == 0ull || nan0 ? 0 : i;  // all NaN, or a NaN at index 0: index 0, as the reference
        if (mode == 1) {
            chosen = list[b == 0ull ? 0 : i];
            lang[s] = chosen;
        }
        tok[s] = chosen;
    }
}

// ------------------------------------------------ beam search (search/)
//
// A fork (decoder.go:223 State.Fork) copies one stream's state into
// another: per layer the int8 self-attention rows of the positions so far
// and their scales, and the tap history; the engram value ring and token
// history, the position and key count. Block (pair, part): parts
// 0 .. layers-1 are the layers, part `layers` the rest. 4-byte words (every
// row length is a multiple of 4 bytes).
struct ForkParams {
    int8_t *k8, *v8;
    float *ks, *vs, *hist, *evring;
    int32_t *tokhist, *pos, *nk_self;
    int layers, max_streams, streams, cap, len, kw, vw, kvh, th_w, sites, ring_kd, ring;
};

__device__ __forceinline__ void copy_words(void *dst, const void *src, size_t bytes) {
    const uint32_t *s = static_cast<const uint32_t *>(src);
    uint32_t *d = static_cast<uint32_t *>(dst);
    for (size_t i = threadIdx.x; i < bytes / 4; i += blockDim.x) d[i] = s[i];
}

__global__ void fork_kernel(const int32_t *__restrict__ pairs, ForkParams f) {
    const int src = pairs[2 * blockIdx.x], dst = pairs[2 * blockIdx.x + 1];
    const int part = blockIdx.y;
    if (part < f.layers) {
        const size_t l = (size_t)part, ms = (size_t)f.max_streams, cap = (size_t)f.cap, n = (size_t)f.len;
        copy_words(f.k8 + ((l * ms + dst) * cap) * f.kw, f.k8 + ((l * ms + src) * cap) * f.kw, n * f.kw);
        copy_words(f.v8 + ((l * ms + dst) * cap) * f.vw, f.v8 + ((l * ms + src) * cap) * f.vw, n * f.vw);
        copy_words(f.ks + ((l * ms + dst) * cap) * f.kvh, f.ks + ((l * ms + src) * cap) * f.kvh, n * f.kvh * 4);
        copy_words(f.vs + ((l * ms + dst) * cap) * f.kvh, f.vs + ((l * ms + src) * cap) * f.kvh, n * f.kvh * 4);
        copy_words(f.hist + (l * ms + dst) * f.th_w, f.hist + (l * ms + src) * f.th_w, (size_t)f.th_w * 4);
        return;
    }
    for (int i = 0; i < f.sites; i++) {
        float *base = f.evring + (size_t)i * f.streams * f.ring_kd;
        copy_words(base + (size_t)dst * f.ring_kd, base + (size_t)src * f.ring_kd, (size_t)f.ring_kd * 4);
    }
    if (f.ring > 0)
        copy_words(f.tokhist + (size_t)dst * f.ring, f.tokhist + (size_t)src * f.ring, (size_t)f.ring * 4);
    if (threadIdx.x == 0) {
        f.pos[dst] = f.pos[src];
        f.nk_self[dst] = f.nk_self[src];
    }
}

// The n best next tokens of each listed row of logits (beam.go:559
// candidates, adjust off), best first, ties to the lower id; with an
// allowed list, the n best of its tokens, ties to the earlier entry. And
// the row's log-sum-exp in float64 (beam.go:605 logSoftmax: m + log Σ
// exp(x − m)), so that log p = float64(x) − lse on the host.
constexpr int kTopThreads = 256;

__device__ __forceinline__ bool top_better(float a, int ia, float b, int ib) {
    return a > b || (a == b && ia < ib);
}

__global__ void __launch_bounds__(kTopThreads) beam_topk_kernel(const float *__restrict__ logits, int vocab,
                                                                 const int32_t *__restrict__ rows, int n,
                                                                 const int32_t *__restrict__ allowed, int nallowed,
                                                                 int32_t *__restrict__ otok, float *__restrict__ ologit,
                                                                 double *__restrict__ olse) {
    __shared__ float sv[kTopThreads / 32];
    __shared__ int si[kTopThreads / 32];
    __shared__ double sd[kTopThreads / 32];
    __shared__ int picked[kBeamMaxCand];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *x = logits + (size_t)rows[blockIdx.x] * vocab;
    float m = -INFINITY;
    for (int i = tid; i < vocab; i += kTopThreads) m = fmaxf(m, x[i]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) sv[warp] = m;
    __syncthreads();
    m = sv[0];
    for (int w = 1; w < kTopThreads / 32; w++) m = fmaxf(m, sv[w]);
    double sum = 0.0;
    for (int i = tid; i < vocab; i += kTopThreads) sum += exp((double)x[i] - (double)m);
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) sd[warp] = sum;
    __syncthreads();
    if (tid == 0) {
        double t = 0.0;
        for (int w = 0; w < kTopThreads / 32; w++) t += sd[w];
        olse[blockIdx.x] = (double)m + log(t);
    }
    const int span = allowed ? nallowed : vocab;
    for (int r = 0; r < n; r++) {
        float bv = -INFINITY;
        int bi = INT_MAX;
        for (int j = tid; j < span; j += kTopThreads) {
            bool taken = false;
            for (int q = 0; q < r; q++) taken |= picked[q] == j;
            if (taken) continue;
            const float v = x[allowed ? allowed[j] : j];
            if (bi == INT_MAX || top_better(v, j, bv, bi)) bv = v, bi = j;
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != INT_MAX && (bi == INT_MAX || top_better(ov, oi, bv, bi))) bv = ov, bi = oi;
        }
        __syncthreads();  // the previous round's readers of sv/si are done
        if (lane == 0) sv[warp] = bv, si[warp] = bi;
        __syncthreads();
        if (tid == 0) {
            float v = sv[0];
            int i = si[0];
            for (int w = 1; w < kTopThreads / 32; w++)
                if (si[w] != INT_MAX && (i == INT_MAX || top_better(sv[w], si[w], v, i))) v = sv[w], i = si[w];
            picked[r] = i;
            const size_t o = (size_t)blockIdx.x * n + r;
            otok[o] = i == INT_MAX ? -1 : (allowed ? allowed[i] : i);
            ologit[o] = v;
        }
        __syncthreads();
    }
}

}  // namespace

}  // namespace wb

using namespace wb;

// A device allocation freed with the decoder.
struct DevBuf {
    void *p = nullptr;
    size_t bytes = 0;
};

// The device buffers and matrix views a model object owns, freed with it on
// its own device.
struct DevStore {
    int device = 0;
    std::vector<DevBuf> bufs;
    // views of the caller's matrices (they keep the storage alive)
    std::vector<wc_cq *> views;

    DevStore() = default;
    DevStore(const DevStore &) = delete;
    DevStore &operator=(const DevStore &) = delete;
    ~DevStore() {
        int cur = 0;
        cudaGetDevice(&cur);
        if (cur != device) cudaSetDevice(device);
        for (auto &b : bufs) cudaFree(b.p);
        for (auto *vw : views) wc_cq_destroy(vw);
        if (cur != device) cudaSetDevice(cur);
    }

    template <typename T>
    wc_status alloc(T **p, size_t count) {
        void *q = nullptr;
        const size_t bytes = (count > 0 ? count : 1) * sizeof(T);
        cudaError_t e = cudaMalloc(&q, bytes);
        if (e != cudaSuccess) return set_error(WC_ERR_NOMEM, std::string("device memory: ") + cudaGetErrorString(e));
        bufs.push_back({q, bytes});
        *p = static_cast<T *>(q);
        return WC_OK;
    }
    // A host float array copied to the device (n values); with gain, the
    // stored norm scales become gains 1 + scale (norm.go:22 NewZCRMSNorm).
    wc_status upload(const float **dst, const float *src, size_t n, bool gain = false) {
        float *p = nullptr;
        wc_status st = alloc(&p, n);
        if (st != WC_OK) return st;
        std::vector<float> tmp(src, src + n);
        if (gain)
            for (auto &x : tmp) x = 1.0f + x;
        WB_CUDA(cudaMemcpy(p, tmp.data(), n * sizeof(float), cudaMemcpyHostToDevice));
        *dst = p;
        return WC_OK;
    }
    wc_status view(const wc_cq *h, wc_cq **out) {
        wc_status st = wc_cq_rows(h, 0, wc_cq_out(h), out);
        if (st == WC_OK) views.push_back(*out);
        return st;
    }
    // rope.go:20 NewRope's tables [len][qk/2] for heads of 48, in the same
    // float32 steps (the host's libm).
    wc_status rope_tables(double theta, int len, const float **cs, const float **sn) {
        const int half = kQK / 2;
        std::vector<float> freqs(half), c((size_t)len * half), s((size_t)len * half);
        for (int i = 0; i < half; i++) {
            const float e = (float)(2 * i) / (float)kQK;
            freqs[i] = 1.0f / (float)std::pow(theta, (double)e);
        }
        for (int t = 0; t < len; t++)
            for (int i = 0; i < half; i++) {
                const double angle = (double)((float)t * freqs[i]);
                c[(size_t)t * half + i] = (float)std::cos(angle);
                s[(size_t)t * half + i] = (float)std::sin(angle);
            }
        wc_status st = upload(cs, c.data(), c.size());
        return st != WC_OK ? st : upload(sn, s.data(), s.size());
    }
    // The HadamardMLP permutations hada_p1, hada_p2 (hadamard.go:281),
    // checked and copied to the device.
    wc_status hada_perms(const int32_t *h1, const int32_t *h2, const int **p1, const int **p2) {
        std::vector<int> seen(kNA * kNB, 0);
        for (const int32_t *pp : {h1, h2}) {
            std::fill(seen.begin(), seen.end(), 0);
            for (int i = 0; i < kNA * kNB; i++) {
                if (pp[i] < 0 || pp[i] >= kNA * kNB || seen[pp[i]])
                    return set_error(WC_ERR_INVALID, fmt("needle: hada_p is not a permutation of %d (entry %d = %d)",
                                                         kNA * kNB, i, pp[i]));
                seen[pp[i]] = 1;
            }
        }
        int32_t *p = nullptr;
        wc_status st = alloc(&p, 2 * kNA * kNB);
        if (st != WC_OK) return st;
        WB_CUDA(cudaMemcpy(p, h1, kNA * kNB * sizeof(int32_t), cudaMemcpyHostToDevice));
        WB_CUDA(cudaMemcpy(p + kNA * kNB, h2, kNA * kNB * sizeof(int32_t), cudaMemcpyHostToDevice));
        *p1 = p;
        *p2 = p + kNA * kNB;
        return WC_OK;
    }
};

struct wc_decoder : DevStore {
    wc_decoder_desc d{};  // sizes (pointers not kept)
    int max_streams = 0, max_frames = 0, cap = 0, flags = 0;
    int streams = 0, frames = 0, len = 0;
    int ring_t = 0;  // token history ring: max_order − 1
    bool tc = false;
    wc_cq *emb = nullptr;
    struct Layer {
        LayerK k;
        wc_cq *q, *kk, *v, *g, *o, *xq, *xk, *xv, *xg, *xo, *ppre, *ppost, *pres;
        bool phi_fused = false;  // the φ products by mhc_phi_kernel
    };
    std::vector<Layer> layers;
    struct Site {
        wc_cq *tables, *key, *value;
        const float *taps;
        int layer;
    };
    std::vector<Site> sites;
    const float *g_final = nullptr;
    const int *p1 = nullptr, *p2 = nullptr;
    const int32_t *orders = nullptr;
    const float *rcos = nullptr, *rsin = nullptr;
    float in_scale = 1.0f, att_scale = 1.0f, xatt_scale = 1.0f;
    // per-stream state and step buffers
    float *stream = nullptr, *xq = nullptr, *phi_pre = nullptr, *phi_post = nullptr, *phi_res = nullptr;
    float *u = nullptr, *h = nullptr, *n = nullptr, *hp = nullptr, *hr = nullptr;
    float *q = nullptr, *k = nullptr, *v = nullptr, *g = nullptr, *qo = nullptr, *att = nullptr, *a = nullptr;
    float *x = nullptr, *cq = nullptr, *cg = nullptr, *cqn = nullptr, *catt = nullptr, *cy = nullptr;
    float *fin = nullptr, *logits = nullptr, *row = nullptr, *erow = nullptr, *vraw = nullptr;
    float *ek = nullptr, *ev = nullptr, *evring = nullptr, *hist = nullptr;
    int32_t *tok = nullptr, *pos = nullptr, *nk_self = nullptr, *nk_x = nullptr, *erows = nullptr;
    int32_t *tokhist = nullptr, *done = nullptr, *langs = nullptr;
    int32_t langs_host[64] = {};
    int8_t *k8 = nullptr, *v8 = nullptr, *xk8 = nullptr, *xv8 = nullptr;
    float *ks = nullptr, *vs = nullptr, *xks = nullptr, *xvs = nullptr;
    float *mk = nullptr, *mv = nullptr;  // memory projection outputs [streams·frames][x_heads·x_qk | x_vd]
    void *tcbuf = nullptr;
    size_t tcbytes = 0;
    // The head's screen (tensor cores, then exact rescoring of candidates).
    bool screen = false;
    float *wn = nullptr, *nmax = nullptr;  // [vocab] ‖ŵ_r‖, max_g |n_rg|
    float wmax = 0.0f;                     // max |ŵ| of the head
    int32_t *cand = nullptr, *ncand = nullptr;
    cudaGraphExec_t graph = nullptr;
    cudaStream_t graph_stream = nullptr;
    int graph_streams = 0;
    // Streams per cross-attention memory (the beams of a clip share one).
    int mem_group = 1;
    // Beam steps: candidate buffers and the fork list.
    int32_t *btok = nullptr, *brows = nullptr, *bpairs = nullptr, *ballowed = nullptr;
    float *blogit = nullptr;
    double *blse = nullptr;

    ~wc_decoder() {
        int cur = 0;
        cudaGetDevice(&cur);
        if (cur != device) cudaSetDevice(device);
        if (graph) cudaGraphExecDestroy(graph);
        if (cur != device) cudaSetDevice(cur);
    }
};

namespace {

float sigmoid_host(float x) { return (float)(1.0 / (1.0 + std::exp(-(double)x))); }

wc_status check_matrix(const wc_cq *m, const char *what, int layer, int out, int in) {
    if (!m) return set_error(WC_ERR_INVALID, fmt("decoder: layer %d %s: nil matrix", layer, what));
    if (wc_cq_out(m) != out || wc_cq_in(m) != in)
        return set_error(WC_ERR_INVALID, fmt("decoder: layer %d %s has shape (%d, %d), want (%d, %d)", layer, what,
                                             wc_cq_out(m), wc_cq_in(m), out, in));
    return WC_OK;
}

// The products of one GEMMs call.
wc_status gemms(wc_decoder *d, std::initializer_list<const wc_cq *> ms, const float *x,
                std::initializer_list<float *> ys, int rows, cudaStream_t st) {
    std::vector<const wc_cq *> m(ms);
    std::vector<float *> y(ys);
    return gemms_device(m.data(), (int)m.size(), x, y.data(), rows, d->tc, d->tcbuf, d->tcbytes, st);
}

#define DEC_LAUNCH(...)                                                 \
    do {                                                                \
        __VA_ARGS__;                                                    \
        count_launch();                                                 \
        cudaError_t e_ = cudaGetLastError();                            \
        if (e_ != cudaSuccess) return cuda_error(e_, "decoder kernel"); \
    } while (0)

#define DEC_ST(call)                        \
    do {                                    \
        wc_status s_ = (call);              \
        if (s_ != WC_OK) return s_;         \
    } while (0)

// One decoder step for every stream (decoder.go:252 Extend with one token
// each, the token in d->tok): up to the head's input in d->fin (the lane
// mean after the final norm), the position advanced. The head runs after
// it (run_head).
wc_status step_body(wc_decoder *d, cudaStream_t st) {
    const int S = d->streams;
    const wc_decoder_desc &D = d->d;
    // Embedding gather (matrix.go:161 Row), × √dim, into every lane.
    DEC_ST(wc_cq_row_gather(d->emb, d->tok, S, d->row, nullptr, st));
    DEC_LAUNCH(embed_kernel<<<S, kThreads, 0, st>>>(d->row, d->in_scale, d->pos, d->nk_self, d->stream));
    // Engram keys and values of every site (cache.go:166 Engram.Extend).
    if (!d->sites.empty()) {
        DEC_LAUNCH(engram_rows_kernel<<<S, 32, 0, st>>>(d->tok, d->tokhist, d->ring_t, d->pos, d->orders, D.n_tables,
                                                        D.slots, d->erows));
        for (size_t i = 0; i < d->sites.size(); i++) {
            const auto &site = d->sites[i];
            DEC_ST(wc_cq_row_gather(site.tables, d->erows, S * D.n_tables, d->erow, nullptr, st));
            float *ek = d->ek + i * (size_t)S * kD, *ev = d->ev + i * (size_t)S * kD;
            DEC_ST(gemms(d, {site.key, site.value}, d->erow, {ek, d->vraw}, S, st));
            const int R = (D.etaps - 1) * (D.n_tables > 0 ? d->ring_t + 1 : 1);
            DEC_LAUNCH(engram_taps_kernel<<<S, kThreads, 0, st>>>(
                d->vraw, d->evring + i * (size_t)S * (R > 0 ? R : 1) * kD, site.taps, D.etaps, d->ring_t + 1, d->pos,
                ev));
        }
    }
    const int qw = D.heads * kQK, kw = D.kv_heads * kQK, vw = D.kv_heads * kVD, W = qw + kw + vw;
    const int th = D.taps - 1 > 0 ? D.taps - 1 : 1;
    for (int l = 0; l < D.layers; l++) {
        auto &L = d->layers[l];
        int site = -1;
        for (size_t i = 0; i < d->sites.size(); i++)
            if (d->sites[i].layer == l) site = (int)i;
        if (L.phi_fused) {
            PhiViews pv{};
            CqShape sh{};
            cq_internal(L.ppre, &sh, &pv.v[0]);
            cq_internal(L.ppost, nullptr, &pv.v[1]);
            cq_internal(L.pres, nullptr, &pv.v[2]);
            pv.y[0] = d->phi_pre, pv.y[1] = d->phi_post, pv.y[2] = d->phi_res;
            DEC_LAUNCH(mhc_phi_kernel<<<S, kThreads, 0, st>>>(d->stream, sh, pv));
        } else {
            DEC_LAUNCH(mhc_in_kernel<<<S, kThreads, 0, st>>>(d->stream, d->xq));
            DEC_ST(gemms(d, {L.ppre, L.ppost, L.pres}, d->xq, {d->phi_pre, d->phi_post, d->phi_res}, S, st));
        }
        const float *ek = site >= 0 ? d->ek + (size_t)site * S * kD : nullptr;
        const float *ev = site >= 0 ? d->ev + (size_t)site * S * kD : nullptr;
        DEC_LAUNCH(sinkhorn_kernel<<<(S + 3) / 4, 128, 0, st>>>(L.k, d->phi_res, d->hr, S));
        DEC_LAUNCH(mhc_block_in_kernel<<<S, kThreads, 0, st>>>(L.k, d->stream, d->phi_pre, d->phi_post, d->phi_res, ek,
                                                               ev, d->u, d->h, d->n, d->hp));
        DEC_ST(gemms(d, {L.q, L.kk, L.v, L.g}, d->n, {d->q, d->k, d->v, d->g}, S, st));
        const size_t cap = (size_t)d->cap;
        int8_t *k8 = d->k8 + (size_t)l * d->max_streams * cap * kw;
        int8_t *v8 = d->v8 + (size_t)l * d->max_streams * cap * vw;
        float *ks = d->ks + (size_t)l * d->max_streams * cap * D.kv_heads;
        float *vs = d->vs + (size_t)l * d->max_streams * cap * D.kv_heads;
        DEC_LAUNCH(self_prep_kernel<<<S, kThreads, W * sizeof(float), st>>>(
            L.k, d->q, d->k, d->v, d->hist + (size_t)l * d->max_streams * th * W, D.taps, D.heads, D.kv_heads, d->pos,
            d->rcos, d->rsin, k8, ks, v8, vs, d->cap, d->qo));
        DEC_ST(wc_attend_int8_streams(S, d->qo, D.heads, k8, ks, v8, vs, d->cap, d->nk_self, D.kv_heads, kQK, kVD,
                                      d->att_scale, WC_ATTEND_QUANT_Q, d->att, st));
        DEC_LAUNCH(gate_kernel<<<S, kThreads, 0, st>>>(d->att, d->g, D.heads * kVD));
        DEC_ST(gemms(d, {L.o}, d->att, {d->a}, S, st));
        DEC_LAUNCH(post_attn_kernel<<<S, kThreads, 0, st>>>(L.k, d->a, d->h, d->x));
        DEC_ST(gemms(d, {L.xq, L.xg}, d->x, {d->cq, d->cg}, S, st));
        DEC_LAUNCH(cross_q_kernel<<<S, kThreads, 0, st>>>(L.k, d->cq, D.x_heads, d->cqn));
        const size_t F = (size_t)d->frames;
        const size_t xoff = (size_t)l * d->max_streams * d->max_frames;
        DEC_ST(attend_streams_grouped(S, d->cqn, D.x_heads, d->xk8 + xoff * D.x_heads * kQK,
                                      d->xks + xoff * D.x_heads, d->xv8 + xoff * D.x_heads * kVD,
                                      d->xvs + xoff * D.x_heads, (int)F, d->nk_x, D.x_heads, kQK, kVD,
                                      d->xatt_scale, WC_ATTEND_QUANT_Q, d->catt, d->mem_group, st));
        DEC_LAUNCH(gate_kernel<<<S, kThreads, 0, st>>>(d->catt, d->cg, D.x_heads * kVD));
        DEC_ST(gemms(d, {L.xo}, d->catt, {d->cy}, S, st));
        DEC_LAUNCH(block_out_kernel<<<S, kThreads, 0, st>>>(L.k, d->p1, d->p2, d->cy, d->h, d->u, d->hp, d->hr,
                                                            d->stream));
    }
    DEC_LAUNCH(final_kernel<<<S, kThreads, 0, st>>>(d->stream, d->g_final, d->fin));
    DEC_LAUNCH(advance_kernel<<<(S + 127) / 128, 128, 0, st>>>(d->tok, d->tokhist, d->ring_t, d->pos, S));
    return WC_OK;
}

// The step, replayed from a CUDA graph captured on first use (per stream
// count), or launched eagerly.
wc_status run_step(wc_decoder *d, cudaStream_t st) {
    if (d->len >= d->cap || d->len >= d->d.rope_len)
        return set_error(WC_ERR_INVALID, fmt("decoder: %d positions exceed the cache's %d or the RoPE tables' %d",
                                             d->len + 1, d->cap, d->d.rope_len));
    if (d->flags & WC_DECODER_NO_GRAPH) {
        DEC_ST(step_body(d, st));
        d->len++;
        return WC_OK;
    }
    if (!d->graph || d->graph_streams != d->streams) {
        if (d->graph) {
            cudaGraphExecDestroy(d->graph);
            d->graph = nullptr;
        }
        // The first step runs eagerly: it sets kernel attributes and the
        // library's one-time device words outside any capture.
        if (d->len == 0 && d->graph_streams != -d->streams) {
            d->graph_streams = -d->streams;
            DEC_ST(step_body(d, st));
            d->len++;
            return WC_OK;
        }
        cudaStream_t cs = nullptr;
        WB_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
        cudaGraph_t g = nullptr;
        WB_CUDA(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
        wc_status s = step_body(d, cs);
        cudaError_t e = cudaStreamEndCapture(cs, &g);
        if (s == WC_OK && e == cudaSuccess) e = cudaGraphInstantiate(&d->graph, g, 0);
        if (g) cudaGraphDestroy(g);
        cudaStreamDestroy(cs);
        if (s != WC_OK) return s;
        if (e != cudaSuccess) return cuda_error(e, "decoder step graph");
        d->graph_streams = d->streams;
    }
    WB_CUDA(cudaGraphLaunch(d->graph, st));
    count_launch();
    d->len++;
    return WC_OK;
}

enum HeadMode { kHeadLogits = 0, kHeadGreedy = 1, kHeadLang = 2 };

// The tied head on d->fin (decoder.go:508 logits, greedy.go:182 argmax,
// greedy.go:81 language): kHeadLogits, the exact logits into d->logits;
// kHeadGreedy, the argmax into d->tok (screened on the tensor cores and
// rescored exactly where the head's shape allows, else exact logits and
// their argmax); kHeadLang, the language token among d->langs into d->tok
// and lang.
wc_status run_head(wc_decoder *d, int mode, int nlangs, int32_t *lang, cudaStream_t st) {
    const int S = d->streams;
    CqShape sh{};
    CqView v{};
    cq_internal(d->emb, &sh, &v);
    if (mode == kHeadLang) {
        DEC_LAUNCH(head_pick_kernel<<<S, kThreads, 0, st>>>(sh, v, d->fin, nullptr, nullptr, d->langs, nlangs, 1,
                                                            d->logits, d->tok, lang));
        return WC_OK;
    }
    if (mode == kHeadLogits || !d->screen) {
        DEC_ST(gemms_device(&d->emb, 1, d->fin, &d->logits, S, false, nullptr, 0, st));
        if (mode == kHeadGreedy) {
            cudaError_t e = launch_head_argmax(d->logits, S, d->d.vocab, 1.0f, nullptr, d->tok, st);
            if (e != cudaSuccess) return cuda_error(e, "decoder argmax");
        }
        return WC_OK;
    }
    DEC_ST(gemms_device(&d->emb, 1, d->fin, &d->logits, S, true, d->tcbuf, d->tcbytes, st));
    DEC_LAUNCH(head_screen_kernel<<<S, kThreads, 0, st>>>(d->logits, d->d.vocab, d->fin, d->wn, d->nmax, sh.cb_max,
                                                          d->wmax, d->cand, d->ncand));
    DEC_LAUNCH(head_pick_kernel<<<S, kThreads, 0, st>>>(sh, v, d->fin, d->cand, d->ncand, nullptr, 0, 0, d->logits,
                                                        d->tok, nullptr));
    return WC_OK;
}

}  // namespace

static wc_status dec_check(const wc_decoder *d);

namespace wb {

wc_status dec_beam_info(const wc_decoder *d, DecBeamInfo *out) {
    DEC_ST(dec_check(d));
    if (d->streams == 0) return set_error(WC_ERR_INVALID, "decoder: no memory (call wc_decoder_memory_beams first)");
    out->streams = d->streams;
    out->group = d->mem_group;
    out->len = d->len;
    out->positions = std::min(d->cap, d->d.rope_len);
    out->vocab = d->d.vocab;
    return WC_OK;
}

static wc_status beam_buffers(wc_decoder *d) {
    if (d->btok) return WC_OK;
    const size_t S = (size_t)d->max_streams;
    DEC_ST(d->alloc(&d->btok, S * kBeamMaxCand));
    DEC_ST(d->alloc(&d->blogit, S * kBeamMaxCand));
    DEC_ST(d->alloc(&d->blse, S));
    DEC_ST(d->alloc(&d->brows, S));
    DEC_ST(d->alloc(&d->bpairs, 2 * S));
    DEC_ST(d->alloc(&d->ballowed, (size_t)kBeamMaxCand));
    return WC_OK;
}

wc_status dec_beam_feed(wc_decoder *d, const int32_t *tokens, cudaStream_t st) {
    WB_CUDA(cudaMemcpyAsync(d->tok, tokens, (size_t)d->streams * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    DEC_ST(run_step(d, st));
    return run_head(d, kHeadLogits, 0, nullptr, st);
}

wc_status dec_beam_top(wc_decoder *d, const int32_t *rows, int nrows, int n, const int32_t *allowed, int nallowed,
                       int32_t *tok, float *logit, double *lse, cudaStream_t st) {
    if (nrows <= 0) return WC_OK;
    const int span = allowed ? nallowed : d->d.vocab;
    if (n < 1 || n > kBeamMaxCand || n > span || nrows > d->streams || (allowed && nallowed > kBeamMaxCand))
        return set_error(WC_ERR_INVALID, fmt("decoder: %d candidates of %d rows among %d tokens", n, nrows, span));
    for (int i = 0; i < nrows; i++)
        if (rows[i] < 0 || rows[i] >= d->streams)
            return set_error(WC_ERR_INVALID, fmt("decoder: candidates of stream %d (%d streams)", rows[i], d->streams));
    for (int i = 0; allowed && i < nallowed; i++)
        if (allowed[i] < 0 || allowed[i] >= d->d.vocab)
            return set_error(WC_ERR_INVALID, fmt("decoder: token %d out of range [0, %d)", allowed[i], d->d.vocab));
    DEC_ST(beam_buffers(d));
    WB_CUDA(cudaMemcpyAsync(d->brows, rows, (size_t)nrows * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    if (allowed)
        WB_CUDA(cudaMemcpyAsync(d->ballowed, allowed, (size_t)nallowed * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    DEC_LAUNCH(beam_topk_kernel<<<nrows, kTopThreads, 0, st>>>(d->logits, d->d.vocab, d->brows, n,
                                                                 allowed ? d->ballowed : nullptr, nallowed, d->btok,
                                                                 d->blogit, d->blse));
    WB_CUDA(cudaMemcpyAsync(tok, d->btok, (size_t)nrows * n * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    WB_CUDA(cudaMemcpyAsync(logit, d->blogit, (size_t)nrows * n * sizeof(float), cudaMemcpyDeviceToHost, st));
    WB_CUDA(cudaMemcpyAsync(lse, d->blse, (size_t)nrows * sizeof(double), cudaMemcpyDeviceToHost, st));
    WB_CUDA(cudaStreamSynchronize(st));
    return WC_OK;
}

wc_status dec_beam_fork(wc_decoder *d, const int32_t *pairs, int npairs, cudaStream_t st) {
    if (npairs <= 0) return WC_OK;
    if (npairs > d->streams) return set_error(WC_ERR_INVALID, fmt("decoder: %d forks of %d streams", npairs, d->streams));
    for (int i = 0; i < 2 * npairs; i++)
        if (pairs[i] < 0 || pairs[i] >= d->streams)
            return set_error(WC_ERR_INVALID, fmt("decoder: fork of stream %d (%d streams)", pairs[i], d->streams));
    DEC_ST(beam_buffers(d));
    const wc_decoder_desc &D = d->d;
    WB_CUDA(cudaMemcpyAsync(d->bpairs, pairs, (size_t)npairs * 2 * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    ForkParams f{};
    f.k8 = d->k8, f.v8 = d->v8, f.ks = d->ks, f.vs = d->vs, f.hist = d->hist, f.evring = d->evring;
    f.tokhist = d->tokhist, f.pos = d->pos, f.nk_self = d->nk_self;
    f.layers = D.layers, f.max_streams = d->max_streams, f.streams = d->streams, f.cap = d->cap, f.len = d->len;
    f.kw = D.kv_heads * kQK, f.vw = D.kv_heads * kVD, f.kvh = D.kv_heads;
    const int th = D.taps - 1 > 0 ? D.taps - 1 : 1;
    f.th_w = th * (D.heads * kQK + D.kv_heads * kQK + D.kv_heads * kVD);
    f.sites = (int)d->sites.size();
    const int R = (D.etaps - 1) * (D.n_tables > 0 ? d->ring_t + 1 : 1);
    f.ring_kd = (R > 0 ? R : 1) * kD;
    f.ring = d->ring_t;
    DEC_LAUNCH(fork_kernel<<<dim3((unsigned)npairs, (unsigned)(D.layers + 1)), 256, 0, st>>>(d->bpairs, f));
    return WC_OK;
}

}  // namespace wb

extern "C" wc_status wc_decoder_create(const wc_decoder_desc *desc, int max_streams, int max_frames, int max_positions,
                                       int flags, wc_decoder **out) {
    if (!out) return set_error(WC_ERR_INVALID, "decoder: nil handle pointer");
    *out = nullptr;
    if (!desc) return set_error(WC_ERR_INVALID, "decoder: nil description");
    const wc_decoder_desc &D = *desc;
    if (D.dim != kD || D.lanes != kLanes || D.qk != kQK || D.vd != kVD || D.x_qk != kQK || D.x_vd != kVD ||
        D.na != kNA || D.nb != kNB || D.rank != kRank)
        return set_error(WC_ERR_UNSUPPORTED,
                         fmt("decoder: this build's kernels take width 512 in 4 lanes, heads of 48/64 and a 16 x 32 "
                             "HadamardMLP of rank 8 (got width %d, %d lanes, heads %d/%d, cross %d/%d, %d x %d rank %d)",
                             D.dim, D.lanes, D.qk, D.vd, D.x_qk, D.x_vd, D.na, D.nb, D.rank));
    if (D.layers <= 0 || D.vocab <= 0 || D.heads <= 0 || D.kv_heads <= 0 || D.heads % D.kv_heads != 0 ||
        D.taps < 1 || D.x_heads <= 0 || D.heads * kVD > 4 * kThreads)
        return set_error(WC_ERR_INVALID, fmt("decoder: %d layers, vocab %d, %d query heads over %d KV heads, %d taps",
                                             D.layers, D.vocab, D.heads, D.kv_heads, D.taps));
    if (D.heads * kVD != kD || D.x_heads * kVD != kD)
        return set_error(WC_ERR_UNSUPPORTED, "decoder: the attention outputs must be as wide as the model (heads·64 = 512)");
    if (max_streams <= 0 || max_streams > 65535 || max_frames <= 0 || max_positions <= 0)
        return set_error(WC_ERR_INVALID, fmt("decoder: room for %d streams, %d frames, %d positions", max_streams,
                                             max_frames, max_positions));
    if (D.n_sites < 0 || (D.n_sites > 0 && (!D.site || !D.orders || D.n_tables <= 0 || D.n_tables > 32 ||
                                            D.slots <= 0 || D.etaps < 1 || D.n_tables * D.sub != kD)))
        return set_error(WC_ERR_INVALID, fmt("decoder: %d engram sites of %d tables x %d slots x %d", D.n_sites,
                                             D.n_tables, D.slots, D.sub));
    if (!D.layer || !D.embedding || !D.final_norm || !D.hada_p1 || !D.hada_p2 || D.rope_len <= 0)
        return set_error(WC_ERR_INVALID, "decoder: nil tensor");

    std::unique_ptr<wc_decoder> d(new (std::nothrow) wc_decoder);
    if (!d) return set_error(WC_ERR_NOMEM, "decoder: out of host memory");
    WB_CUDA(cudaGetDevice(&d->device));
    d->d = D;
    d->d.layer = nullptr;
    d->d.site = nullptr;
    d->d.orders = d->d.hada_p1 = d->d.hada_p2 = nullptr;
    d->d.final_norm = nullptr;
    d->d.embedding = nullptr;
    d->max_streams = max_streams;
    d->max_frames = max_frames;
    d->cap = (max_positions + 1) & ~1;  // an even row count keeps the bulk attention's scale chunks aligned
    d->flags = flags;
    d->tc = (flags & WC_DECODER_TENSOR_CORES) != 0;
    const int qw = D.heads * kQK, kw = D.kv_heads * kQK, vw = D.kv_heads * kVD;
    const int xqw = D.x_heads * kQK, xvw = D.x_heads * kVD;

    // Matrices.
    if (wc_cq_out(D.embedding) != D.vocab || wc_cq_in(D.embedding) != kD)
        return set_error(WC_ERR_INVALID, fmt("decoder: embedding has shape (%d, %d), want (%d, %d)",
                                             wc_cq_out(D.embedding), wc_cq_in(D.embedding), D.vocab, kD));
    DEC_ST(d->view(D.embedding, &d->emb));
    for (int l = 0; l < D.layers; l++) {
        const wc_decoder_layer &S = D.layer[l];
        DEC_ST(check_matrix(S.q_proj, "q_proj", l, qw, kD));
        DEC_ST(check_matrix(S.k_proj, "k_proj", l, kw, kD));
        DEC_ST(check_matrix(S.v_proj, "v_proj", l, vw, kD));
        DEC_ST(check_matrix(S.gate_proj, "gate_proj", l, D.heads * kVD, kD));
        DEC_ST(check_matrix(S.out_proj, "out_proj", l, kD, D.heads * kVD));
        DEC_ST(check_matrix(S.x_q_proj, "cross q_proj", l, xqw, kD));
        DEC_ST(check_matrix(S.x_k_proj, "cross k_proj", l, xqw, kD));
        DEC_ST(check_matrix(S.x_v_proj, "cross v_proj", l, xvw, kD));
        DEC_ST(check_matrix(S.x_gate_proj, "cross gate_proj", l, xvw, kD));
        DEC_ST(check_matrix(S.x_out_proj, "cross out_proj", l, kD, xvw));
        DEC_ST(check_matrix(S.phi_pre, "mhc_phi_pre", l, kLanes, kLanes * kD));
        DEC_ST(check_matrix(S.phi_post, "mhc_phi_post", l, kLanes, kLanes * kD));
        DEC_ST(check_matrix(S.phi_res, "mhc_phi_res", l, kLanes * kLanes, kLanes * kD));
        const float *vecs[] = {S.norm_in, S.post_norm, S.pre_hada, S.q_taps, S.k_taps, S.v_taps, S.q_norm, S.k_norm,
                               S.d1, S.d2, S.b2, S.d3, S.d4, S.w1a, S.w1b, S.w2a, S.w2b, S.w3a, S.w3b, S.cond_v,
                               S.cond_u, S.x_norm_in, S.x_post_norm, S.x_q_norm, S.x_k_norm, S.b_pre, S.b_post,
                               S.b_res};
        for (const float *p : vecs)
            if (!p) return set_error(WC_ERR_INVALID, fmt("decoder: layer %d: nil tensor", l));
        wc_decoder::Layer L{};
        DEC_ST(d->view(S.q_proj, &L.q));
        DEC_ST(d->view(S.k_proj, &L.kk));
        DEC_ST(d->view(S.v_proj, &L.v));
        DEC_ST(d->view(S.gate_proj, &L.g));
        DEC_ST(d->view(S.out_proj, &L.o));
        DEC_ST(d->view(S.x_q_proj, &L.xq));
        DEC_ST(d->view(S.x_k_proj, &L.xk));
        DEC_ST(d->view(S.x_v_proj, &L.xv));
        DEC_ST(d->view(S.x_gate_proj, &L.xg));
        DEC_ST(d->view(S.x_out_proj, &L.xo));
        DEC_ST(d->view(S.phi_pre, &L.ppre));
        DEC_ST(d->view(S.phi_post, &L.ppost));
        DEC_ST(d->view(S.phi_res, &L.pres));
        // The fused φ kernel (exact mode): 4-bit group-128 rows of 2048
        // inputs on one codebook, 4 + 4 + 16 of them.
        {
            CqShape a{}, b{}, c{};
            CqView va{}, vb{}, vc{};
            cq_internal(L.ppre, &a, &va);
            cq_internal(L.ppost, &b, &vb);
            cq_internal(L.pres, &c, &vc);
            auto same = [](const CqShape &x, const CqShape &y) {
                return x.in == y.in && x.group == y.group && x.bits == y.bits && x.cb_max == y.cb_max &&
                       x.lut_step == y.lut_step && std::memcmp(x.cb, y.cb, sizeof x.cb) == 0;
            };
            L.phi_fused = !d->tc && a.bits == 4 && a.group == 128 && a.in == kPhiIn && a.gb == 64 &&
                          a.pad == kPhiIn && same(a, b) && same(a, c) && va.out == kLanes && vb.out == kLanes &&
                          vc.out == kLanes * kLanes;
        }
        LayerK &K = L.k;
        const int nn = kNA * kNB;
        DEC_ST(d->upload(&K.g_norm_in, S.norm_in, kD, true));
        DEC_ST(d->upload(&K.g_post, S.post_norm, kD, true));
        DEC_ST(d->upload(&K.g_pre_hada, S.pre_hada, kD, true));
        DEC_ST(d->upload(&K.q_taps, S.q_taps, (size_t)D.taps * qw));
        DEC_ST(d->upload(&K.k_taps, S.k_taps, (size_t)D.taps * kw));
        DEC_ST(d->upload(&K.v_taps, S.v_taps, (size_t)D.taps * vw));
        DEC_ST(d->upload(&K.g_qn, S.q_norm, kQK, true));
        DEC_ST(d->upload(&K.g_kn, S.k_norm, kQK, true));
        DEC_ST(d->upload(&K.d1, S.d1, nn));
        DEC_ST(d->upload(&K.d2, S.d2, nn));
        DEC_ST(d->upload(&K.b2, S.b2, nn));
        DEC_ST(d->upload(&K.d3, S.d3, nn));
        DEC_ST(d->upload(&K.d4, S.d4, nn));
        const float *wa[3] = {S.w1a, S.w2a, S.w3a}, *wbb[3] = {S.w1b, S.w2b, S.w3b};
        for (int i = 0; i < 3; i++) {
            DEC_ST(d->upload(&K.wa[i], wa[i], kNA * kNA));
            DEC_ST(d->upload(&K.wb[i], wbb[i], kNB * kNB));
        }
        DEC_ST(d->upload(&K.cond_v, S.cond_v, (size_t)kD * kRank));
        DEC_ST(d->upload(&K.cond_u, S.cond_u, (size_t)kRank * nn));
        DEC_ST(d->upload(&K.g_xn, S.x_norm_in, kD, true));
        DEC_ST(d->upload(&K.g_xpost, S.x_post_norm, kD, true));
        DEC_ST(d->upload(&K.g_xqn, S.x_q_norm, kQK, true));
        DEC_ST(d->upload(&K.g_xkn, S.x_k_norm, kQK, true));
        DEC_ST(d->upload(&K.b_pre, S.b_pre, kLanes));
        DEC_ST(d->upload(&K.b_post, S.b_post, kLanes));
        DEC_ST(d->upload(&K.b_res, S.b_res, kLanes * kLanes));
        K.gate = sigmoid_host(S.attn_gate);
        K.xresid = sigmoid_host(S.x_attn_gate);
        K.a_pre = S.a_pre;
        K.a_post = S.a_post;
        K.a_res = S.a_res;
        K.lane = l % kLanes;
        d->layers.push_back(L);
    }
    for (int i = 0; i < D.n_sites; i++) {
        const wc_engram_site &S = D.site[i];
        if (S.layer < 0 || S.layer >= D.layers || !S.taps)
            return set_error(WC_ERR_INVALID, fmt("decoder: engram site %d at layer %d", i, S.layer));
        if (!S.tables || wc_cq_out(S.tables) != D.n_tables * D.slots || wc_cq_in(S.tables) != D.sub)
            return set_error(WC_ERR_INVALID, fmt("decoder: engram site %d tables: want (%d, %d)", i,
                                                 D.n_tables * D.slots, D.sub));
        if (!S.key_proj || wc_cq_out(S.key_proj) != kD || wc_cq_in(S.key_proj) != kD || !S.value_proj ||
            wc_cq_out(S.value_proj) != kD || wc_cq_in(S.value_proj) != kD)
            return set_error(WC_ERR_INVALID, fmt("decoder: engram site %d projections: want (%d, %d)", i, kD, kD));
        wc_decoder::Site st{};
        DEC_ST(d->view(S.tables, &st.tables));
        DEC_ST(d->view(S.key_proj, &st.key));
        DEC_ST(d->view(S.value_proj, &st.value));
        DEC_ST(d->upload(&st.taps, S.taps, (size_t)D.etaps * kD));
        st.layer = S.layer;
        d->sites.push_back(st);
    }
    int max_order = 1;
    if (D.n_sites > 0) {
        for (int c = 0; c < D.n_tables; c++) {
            if (D.orders[c] < 1) return set_error(WC_ERR_INVALID, fmt("decoder: engram order %d", D.orders[c]));
            max_order = std::max(max_order, (int)D.orders[c]);
        }
        int32_t *o = nullptr;
        DEC_ST(d->alloc(&o, D.n_tables));
        WB_CUDA(cudaMemcpy(o, D.orders, D.n_tables * sizeof(int32_t), cudaMemcpyHostToDevice));
        d->orders = o;
    }
    d->ring_t = max_order - 1;
    d->d.etaps = D.etaps;
    DEC_ST(d->hada_perms(D.hada_p1, D.hada_p2, &d->p1, &d->p2));
    DEC_ST(d->upload(&d->g_final, D.final_norm, kD, true));
    DEC_ST(d->rope_tables(D.rope_theta, D.rope_len, &d->rcos, &d->rsin));
    d->in_scale = (float)std::sqrt((double)kD);    // decoder.go:313 ScaleSqrtDim
    d->att_scale = (float)std::sqrt((double)kQK);  // attention.go:407 attendScale
    d->xatt_scale = (float)std::sqrt((double)kQK); // cross.go:276

    // State and step buffers.
    const size_t S = (size_t)max_streams, cap = (size_t)d->cap, F = (size_t)max_frames, L = (size_t)D.layers;
    const int th = D.taps - 1 > 0 ? D.taps - 1 : 1;
    const int W = qw + kw + vw;
    DEC_ST(d->alloc(&d->stream, S * kLanes * kD));
    DEC_ST(d->alloc(&d->xq, S * kLanes * kD));
    DEC_ST(d->alloc(&d->phi_pre, S * kLanes));
    DEC_ST(d->alloc(&d->phi_post, S * kLanes));
    DEC_ST(d->alloc(&d->phi_res, S * kLanes * kLanes));
    for (float **p : {&d->u, &d->h, &d->n, &d->att, &d->a, &d->x, &d->cg, &d->catt, &d->cy, &d->fin, &d->row,
                      &d->erow, &d->vraw, &d->g})
        DEC_ST(d->alloc(p, S * kD));
    DEC_ST(d->alloc(&d->hp, S * kLanes));
    DEC_ST(d->alloc(&d->hr, S * kLanes * kLanes));
    DEC_ST(d->alloc(&d->q, S * qw));
    DEC_ST(d->alloc(&d->qo, S * qw));
    DEC_ST(d->alloc(&d->k, S * kw));
    DEC_ST(d->alloc(&d->v, S * vw));
    DEC_ST(d->alloc(&d->cq, S * xqw));
    DEC_ST(d->alloc(&d->cqn, S * xqw));
    DEC_ST(d->alloc(&d->logits, S * D.vocab));
    const size_t sites = D.n_sites > 0 ? D.n_sites : 1;
    DEC_ST(d->alloc(&d->ek, sites * S * kD));
    DEC_ST(d->alloc(&d->ev, sites * S * kD));
    const int R = (D.etaps - 1) * max_order;
    DEC_ST(d->alloc(&d->evring, sites * S * (R > 0 ? R : 1) * kD));
    DEC_ST(d->alloc(&d->hist, L * S * th * W));
    DEC_ST(d->alloc(&d->tok, S));
    DEC_ST(d->alloc(&d->pos, S));
    DEC_ST(d->alloc(&d->nk_self, S));
    DEC_ST(d->alloc(&d->nk_x, S));
    DEC_ST(d->alloc(&d->done, S));
    DEC_ST(d->alloc(&d->langs, 64));
    DEC_ST(d->alloc(&d->erows, S * (D.n_tables > 0 ? D.n_tables : 1)));
    DEC_ST(d->alloc(&d->tokhist, S * (d->ring_t > 0 ? d->ring_t : 1)));
    DEC_ST(d->alloc(&d->k8, L * S * cap * kw));
    DEC_ST(d->alloc(&d->v8, L * S * cap * vw));
    DEC_ST(d->alloc(&d->ks, L * S * cap * D.kv_heads));
    DEC_ST(d->alloc(&d->vs, L * S * cap * D.kv_heads));
    DEC_ST(d->alloc(&d->xk8, L * S * F * xqw));
    DEC_ST(d->alloc(&d->xv8, L * S * F * xvw));
    DEC_ST(d->alloc(&d->xks, L * S * F * D.x_heads));
    DEC_ST(d->alloc(&d->xvs, L * S * F * D.x_heads));
    DEC_ST(d->alloc(&d->mk, S * F * xqw));
    DEC_ST(d->alloc(&d->mv, S * F * xvw));
    {
        // The rotated image of the tensor-core products: the head's (S rows
        // at 512 in), and with WC_DECODER_TENSOR_CORES every product's (S·F
        // rows at 512 in for the memory, S rows at 2048 in for φ).
        size_t need = tc_a_bytes((int)S, (kD + 63) / 64);
        if (d->tc)
            need = std::max(need, std::max(tc_a_bytes((int)(S * F), (kD + 63) / 64),
                                           tc_a_bytes((int)S, (kLanes * kD + 63) / 64)));
        d->tcbytes = need;
        unsigned char *p = nullptr;
        DEC_ST(d->alloc(&p, d->tcbytes));
        d->tcbuf = p;
    }
    {
        CqShape sh{};
        CqView v{};
        cq_internal(d->emb, &sh, &v);
        d->screen = sh.group == kHeadG && sh.bits == kHeadBits && sh.in == kD && sh.groups == kHeadGroups;
        if (d->screen) {
            DEC_ST(wc_cq_prepare_tc(d->emb));
            DEC_ST(d->alloc(&d->wn, D.vocab));
            DEC_ST(d->alloc(&d->nmax, D.vocab));
            DEC_ST(d->alloc(&d->cand, S * kMaxCand));
            DEC_ST(d->alloc(&d->ncand, S));
            head_rownorm_kernel<<<(D.vocab + 255) / 256, 256>>>(sh, v, d->wn, d->nmax);
            count_launch();
            WB_CUDA(cudaGetLastError());
            std::vector<float> nm(D.vocab);
            WB_CUDA(cudaMemcpy(nm.data(), d->nmax, D.vocab * sizeof(float), cudaMemcpyDeviceToHost));
            float mx = 0.0f;
            for (float x : nm) mx = std::max(mx, x);
            d->wmax = sh.cb_max * mx * sh.inv_sqrt * 1.0001f;
        }
    }
    if (d->tc) {
        for (auto &L2 : d->layers)
            for (wc_cq *m : {L2.q, L2.kk, L2.v, L2.g, L2.o, L2.xq, L2.xk, L2.xv, L2.xg, L2.xo, L2.ppre, L2.ppost,
                             L2.pres})
                DEC_ST(wc_cq_prepare_tc(m));
        for (auto &st : d->sites) {
            DEC_ST(wc_cq_prepare_tc(st.key));
            DEC_ST(wc_cq_prepare_tc(st.value));
        }
        DEC_ST(wc_cq_prepare_tc(d->emb));
    }
    if (!err_word()) return set_error(WC_ERR_NOMEM, "cuda: error word");
    WB_CUDA(cudaDeviceSynchronize());
    *out = d.release();
    return WC_OK;
}

extern "C" void wc_decoder_destroy(wc_decoder *d) { delete d; }

extern "C" int wc_decoder_len(const wc_decoder *d) { return d ? d->len : 0; }

static wc_status dec_check(const wc_decoder *d) {
    if (!d) return set_error(WC_ERR_INVALID, "decoder: nil decoder");
    int dev = 0;
    WB_CUDA(cudaGetDevice(&dev));
    if (dev != d->device)
        return set_error(WC_ERR_DEVICE, fmt("decoder: created on device %d, called on device %d", d->device, dev));
    return WC_OK;
}

static wc_status memory_group(wc_decoder *d, const float *enc, int streams, int frames, int group, wc_stream stream);

extern "C" wc_status wc_decoder_memory(wc_decoder *d, const float *enc, int streams, int frames, wc_stream stream) {
    return memory_group(d, enc, streams, frames, 1, stream);
}

extern "C" wc_status wc_decoder_memory_beams(wc_decoder *d, const float *enc, int clips, int frames, int beams,
                                             wc_stream stream) {
    DEC_ST(dec_check(d));
    if (beams < 1 || clips <= 0 || (long long)clips * beams > d->max_streams)
        return set_error(WC_ERR_INVALID, fmt("decoder: %d clips x %d beams (room for %d streams)", clips, beams,
                                             d->max_streams));
    return memory_group(d, enc, clips, frames, beams, stream);
}

// Memory of `streams` clips, each read by `group` consecutive streams.
static wc_status memory_group(wc_decoder *d, const float *enc, int streams, int frames, int group, wc_stream stream) {
    DEC_ST(dec_check(d));
    if (streams <= 0 || streams > d->max_streams || frames <= 0 || frames > d->max_frames || !enc)
        return set_error(WC_ERR_INVALID, fmt("decoder: encoder output of %d streams x %d frames (room for %d x %d)",
                                             streams, frames, d->max_streams, d->max_frames));
    cudaStream_t st = (cudaStream_t)stream;
    const wc_decoder_desc &D = d->d;
    const size_t rows = (size_t)streams * frames;
    if (rows > (size_t)INT32_MAX) return set_error(WC_ERR_INVALID, "decoder: memory too large");
    for (int l = 0; l < D.layers; l++) {
        auto &L = d->layers[l];
        DEC_ST(gemms(d, {L.xk, L.xv}, enc, {d->mk, d->mv}, (int)rows, st));
        const size_t xoff = (size_t)l * d->max_streams * d->max_frames;
        // Memory rows of stream b start at b·frames (cap = frames for the
        // attention), so the layer's block is contiguous.
        DEC_LAUNCH(xmem_kernel<<<(unsigned)rows, 256, 0, st>>>(d->mk, d->mv, L.k.g_xkn, D.x_heads,
                                                               d->xk8 + xoff * D.x_heads * kQK, d->xks + xoff * D.x_heads,
                                                               d->xv8 + xoff * D.x_heads * kVD,
                                                               d->xvs + xoff * D.x_heads));
    }
    const int S = streams * group;
    DEC_LAUNCH(fill_kernel<<<(S + 255) / 256, 256, 0, st>>>(d->nk_x, frames, S));
    DEC_LAUNCH(fill_kernel<<<(S + 255) / 256, 256, 0, st>>>(d->pos, 0, S));
    if (d->streams != S || d->frames != frames || d->mem_group != group) {
        if (d->graph) cudaGraphExecDestroy(d->graph);
        d->graph = nullptr;
        d->graph_streams = 0;
    }
    d->streams = S;
    d->frames = frames;
    d->mem_group = group;
    d->len = 0;
    return WC_OK;
}

extern "C" wc_status wc_decoder_memory_of(const wc_decoder *d, int l, const int8_t **k8, const float **ks,
                                          const int8_t **v8, const float **vs) {
    DEC_ST(dec_check(d));
    if (l < 0 || l >= d->d.layers || !k8 || !ks || !v8 || !vs)
        return set_error(WC_ERR_INVALID, fmt("decoder: memory of layer %d", l));
    const size_t xoff = (size_t)l * d->max_streams * d->max_frames;
    *k8 = d->xk8 + xoff * d->d.x_heads * kQK;
    *ks = d->xks + xoff * d->d.x_heads;
    *v8 = d->xv8 + xoff * d->d.x_heads * kVD;
    *vs = d->xvs + xoff * d->d.x_heads;
    return WC_OK;
}

extern "C" wc_status wc_decoder_extend(wc_decoder *d, const int32_t *tokens, float *logits, int32_t *next,
                                       wc_stream stream) {
    DEC_ST(dec_check(d));
    if (d->streams == 0) return set_error(WC_ERR_INVALID, "decoder: no memory (call wc_decoder_memory first)");
    if (!tokens) return set_error(WC_ERR_INVALID, "decoder: nil tokens");
    cudaStream_t st = (cudaStream_t)stream;
    const int S = d->streams;
    WB_CUDA(cudaMemcpyAsync(d->tok, tokens, S * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
    DEC_ST(run_step(d, st));
    if (logits || next) DEC_ST(run_head(d, kHeadLogits, 0, nullptr, st));
    if (logits)
        WB_CUDA(cudaMemcpyAsync(logits, d->logits, (size_t)S * d->d.vocab * sizeof(float), cudaMemcpyDeviceToDevice,
                                st));
    if (next) {
        cudaError_t e = launch_head_argmax(d->logits, S, d->d.vocab, 1.0f, nullptr, next, st);
        if (e != cudaSuccess) return cuda_error(e, "decoder argmax");
    }
    return WC_OK;
}

extern "C" wc_status wc_decoder_greedy(wc_decoder *d, int bos, const int32_t *langs, int n_langs, int eos,
                                       int max_tokens, int32_t *tokens, int32_t *counts, int32_t *lang,
                                       int32_t *eos_hit, wc_stream stream) {
    DEC_ST(dec_check(d));
    if (d->streams == 0) return set_error(WC_ERR_INVALID, "decoder: no memory (call wc_decoder_memory first)");
    if (!langs || n_langs <= 0 || n_langs > 64 || max_tokens < 1 || !tokens || !counts || !lang || !eos_hit)
        return set_error(WC_ERR_INVALID, fmt("decoder: greedy with %d languages and %d tokens", n_langs, max_tokens));
    const wc_decoder_desc &D = d->d;
    if (bos < 0 || bos >= D.vocab || eos < 0 || eos >= D.vocab)
        return set_error(WC_ERR_INVALID, fmt("decoder: token %d out of range [0, %d)", bos < 0 || bos >= D.vocab ? bos : eos,
                                             D.vocab));
    for (int i = 0; i < n_langs; i++)
        if (langs[i] < 0 || langs[i] >= D.vocab)
            return set_error(WC_ERR_INVALID, fmt("decoder: token %d out of range [0, %d)", langs[i], D.vocab));
    if (d->len + max_tokens > d->cap || d->len + max_tokens > D.rope_len)
        return set_error(WC_ERR_INVALID, fmt("decoder: %d positions exceed the cache's %d or the RoPE tables' %d",
                                             d->len + max_tokens, d->cap, D.rope_len));
    cudaStream_t st = (cudaStream_t)stream;
    const int S = d->streams, out_w = max_tokens > 1 ? max_tokens - 1 : 1;
    // The language ids: a small device copy (the stream orders it before
    // the kernel that reads it; the host array may be reused after return
    // only once the stream has reached the copy, so copy from a staging
    // array the decoder owns).
    std::memcpy(d->langs_host, langs, n_langs * sizeof(int32_t));
    WB_CUDA(cudaMemcpyAsync(d->langs, d->langs_host, n_langs * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    int32_t *dl = d->langs;
    DEC_LAUNCH(greedy_init_kernel<<<S, 128, 0, st>>>(d->tok, bos, tokens, out_w, counts, eos_hit, d->done, S));
    (void)dl;
    DEC_ST(run_step(d, st));
    DEC_ST(run_head(d, kHeadLang, n_langs, lang, st));
    for (int step = 0; step < max_tokens - 1; step++) {
        DEC_ST(run_step(d, st));
        DEC_ST(run_head(d, kHeadGreedy, 0, nullptr, st));
        DEC_LAUNCH(record_kernel<<<(S + 127) / 128, 128, 0, st>>>(d->tok, eos, out_w, tokens, counts, eos_hit, d->done,
                                                                  S));
    }
    return WC_OK;
}

// =========================================================================
// The encoder stack (wc_encoder_*): internal/encoder's Stack (encoder.go:167)
// with the Best() hypothesis and the engine's int8 numerics, for many clips
// at once. The stack's rows are frames (clip-major), and every row-wise
// phase is the decoder's kernel or one written the same way: a 512-thread
// CTA per frame, one thread per model column, every float32 operation a
// separate rounding in the reference's order. Per layer l:
//   mhc_phi / mhc_in + GEMMs, sinkhorn, mhc_block_in (u, pre_hada_0 norm)
//   enc_ffn      FFN1: x += 1/2 · HadamardMLP, then norm_in
//   GEMMs        q, k, v, gate (one shared input)
//   enc_qkv      per-head q/k norm, RoPE at the frame's position, the int8
//                codes and scales of k and v (QuantizeRows per head)
//   attention    every frame against its clip's keys and values, no mask:
//                enc_attend_kernel (any order: a clip's keys and values
//                staged once per CTA of 32 frames) or the int8 decode
//                kernel (exact order, kv_group = frames)
//   gate, GEMM   σ(gate) ⊙, out_proj
//   post_attn    post_attn_norm, gated residual, conv_norm
//   GEMM, enc_glu, enc_dw, GEMM   pw1, GLU, depthwise + conv_out_norm +
//                SiLU, pw2
//   enc_out      conv residual, FFN2, mHC mix back into the lanes
// then the lane mean and the final norm (final_kernel).
namespace wb {
namespace {

// One HadamardMLP's device tensors.
struct HadaK {
    const float *d1, *d2, *b2, *d3, *d4;
    const float *wa[3], *wb[3];
    const float *cond_v, *cond_u;
};

// The encoder layer's tensors beside its LayerK (whose g_norm_in is
// pre_hada_0's gain, g_post post_norm's, g_xn conv_norm's).
struct EncK {
    const float *g_attn_in, *g_qn, *g_kn, *g_conv_out, *g_pre_hada;
    const float *dw;  // [dw_k][kD]
    int dw_k;
};

// The shared memory of one HadamardMLP per CTA.
struct HadaSmem {
    float pv[kD], z[kD], o[kD], yT[kD], kb[kD];
    float lg[kRank];
    float cv[kD * kRank];
    float wa[3][kNA * kNA], wb[3][kNB * kNB];
};

__device__ void hada_load(const HadaK &H, HadaSmem &S) {
    const int c = threadIdx.x;
    for (int i = c; i < kD * kRank; i += kThreads) S.cv[i] = H.cond_v[i];
    for (int st = 0; st < 3; st++) {
        for (int i = c; i < kNA * kNA; i += kThreads) S.wa[st][i] = H.wa[st][i];
        for (int i = c; i < kNB * kNB; i += kThreads) S.wb[st][i] = H.wb[st][i];
    }
}

// hadamard.go:211 rows for the CTA's row, p its normed input (column c):
// returns column c of mlp(p), the same operations as block_out_kernel's.
__device__ float hada_col(const HadaK &H, const int *__restrict__ p1, const int *__restrict__ p2, float p,
                          HadaSmem &S) {
    const int c = threadIdx.x;
    S.pv[c] = p;
    __syncthreads();
    if (c < kRank) {
        float acc = 0.0f;
        for (int i = 0; i < kD; i++) acc = acc + S.pv[i] * S.cv[i * kRank + c];
        S.lg[c] = acc;
    }
    __syncthreads();
    if (c == 0) {  // load.go:127 softmaxInPlace with exp.go:238 expSubSumGeneric
        float m = -INFINITY;
        for (int r = 0; r < kRank; r++) m = fmaxf(m, S.lg[r]);
        float sum = 0.0f;
        for (int r = 0; r < kRank; r++) {
            const float e = (float)exp((double)(S.lg[r] - m));
            S.lg[r] = e;
            sum = sum + e;
        }
        for (int r = 0; r < kRank; r++) S.lg[r] = __fdiv_rn(S.lg[r], sum);
    }
    __syncthreads();
    float cond = 0.0f;
    for (int r = 0; r < kRank; r++) cond = cond + S.lg[r] * H.cond_u[r * kD + c];
    cond = cond + 1.0f;
    S.z[c] = H.d1[c] * p;
    __syncthreads();
    kron_mix(S.wa[0], S.wb[0], p1, S.z, S.yT, S.kb, S.o);
    {
        const float a2 = H.d2[c] * cond * S.o[c] + H.b2[c];
        S.z[c] = a2 * sigm(a2);
    }
    __syncthreads();
    kron_mix(S.wa[1], S.wb[1], p2, S.z, S.yT, S.kb, S.o);
    S.z[c] = H.d3[c] * S.o[c];
    __syncthreads();
    kron_mix(S.wa[2], S.wb[2], nullptr, S.z, S.yT, S.kb, S.o);
    return S.o[c] * H.d4[c];
}

// mhc.go:131 ExpandLanes: every frame row into every lane.
__global__ void __launch_bounds__(kThreads) enc_expand_kernel(const float *__restrict__ x, float *__restrict__ stream) {
    const int r = blockIdx.x, c = threadIdx.x;
    const float v = x[(size_t)r * kD + c];
#pragma unroll
    for (int k = 0; k < kLanes; k++) stream[((size_t)r * kLanes + k) * kD + c] = v;
}

// block.go:172 ffn (FFN1): x += 1/2 · mlp(n) with n the pre_hada_0 norm of
// x; then block.go:193's norm_in of the result (the attention's input).
__global__ void __launch_bounds__(kThreads)
    enc_ffn_kernel(const __grid_constant__ HadaK H, const int *__restrict__ p1, const int *__restrict__ p2,
                   const float *__restrict__ n, float *__restrict__ h, const float *__restrict__ g_next,
                   float *__restrict__ n_out) {
    __shared__ double red[33];
    __shared__ HadaSmem S;
    const int r = blockIdx.x, c = threadIdx.x;
    hada_load(H, S);
    const float m = hada_col(H, p1, p2, n[(size_t)r * kD + c], S);
    const float hv = h[(size_t)r * kD + c] + 0.5f * m;
    h[(size_t)r * kD + c] = hv;
    n_out[(size_t)r * kD + c] = zc_norm_row(hv, g_next[c], red);
}

// attention.go:300 normRotate at the frame's position (RoPE from 0 in each
// clip) and :342 quantQKV's keys and values as int8 codes per head
// (int8.go:115 QuantizeRows: the codes fakeQuant's values stand for); the
// queries stay float (the attention quantises them per head).
__global__ void __launch_bounds__(kThreads)
    enc_qkv_kernel(const __grid_constant__ EncK K, const float *__restrict__ q, const float *__restrict__ k,
                   const float *__restrict__ v, int heads, int kv_heads, int frames, const float *__restrict__ rcos,
                   const float *__restrict__ rsin, float *__restrict__ qo, int8_t *__restrict__ k8,
                   float *__restrict__ ks, int8_t *__restrict__ v8, float *__restrict__ vs) {
    const int r = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int f = r % frames, half = kQK / 2;
    const int qw = heads * kQK, kw = kv_heads * kQK, vw = kv_heads * kVD;
    for (int hd = warp; hd < heads + 2 * kv_heads; hd += nw) {
        if (hd < heads + kv_heads) {
            const bool isq = hd < heads;
            const int h2 = isq ? hd : hd - heads;
            const float *src = isq ? q + (size_t)r * qw + h2 * kQK : k + (size_t)r * kw + h2 * kQK;
            const float *g = isq ? K.g_qn : K.g_kn;
            float a = 0.0f, b = 0.0f;
            if (lane < half) {
                a = src[lane];
                b = src[lane + half];
            }
            const float rms = (float)sqrt((double)head_ms48(a, b, lane));
            float ra = 0.0f, rb = 0.0f;
            if (lane < half) {
                a = __fdiv_rn(g[lane] * a, rms);
                b = __fdiv_rn(g[lane + half] * b, rms);
                const float cs = rcos[(size_t)f * half + lane], sn = rsin[(size_t)f * half + lane];
                const float ac = a * cs, bs = b * sn, bc = b * cs, as = a * sn;
                ra = ac - bs;
                rb = bc + as;
            }
            if (isq) {
                if (lane < half) {
                    qo[(size_t)r * qw + h2 * kQK + lane] = ra;
                    qo[(size_t)r * qw + h2 * kQK + lane + half] = rb;
                }
            } else {
                float m = fmaxf(fabsf(ra), fabsf(rb));
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                const float sc = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
                if (lane < half) {
                    k8[(size_t)r * kw + h2 * kQK + lane] = quant8(ra, sc);
                    k8[(size_t)r * kw + h2 * kQK + lane + half] = quant8(rb, sc);
                }
                if (lane == 0) ks[(size_t)r * kv_heads + h2] = sc;
            }
        } else {
            const int h2 = hd - heads - kv_heads;
            const float a = v[(size_t)r * vw + h2 * kVD + lane], b = v[(size_t)r * vw + h2 * kVD + lane + 32];
            float m = fmaxf(fabsf(a), fabsf(b));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const float sc = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
            v8[(size_t)r * vw + h2 * kVD + lane] = quant8(a, sc);
            v8[(size_t)r * vw + h2 * kVD + lane + 32] = quant8(b, sc);
            if (lane == 0) vs[(size_t)r * kv_heads + h2] = sc;
        }
    }
}

// block.go:257 gated, GLUValueGate: value · σ(gate) of pw1's two halves.
__global__ void __launch_bounds__(kThreads) enc_glu_kernel(const float *__restrict__ p, float *__restrict__ out) {
    const int r = blockIdx.x, c = threadIdx.x;
    const float a = p[(size_t)r * 2 * kD + c], g = p[(size_t)r * 2 * kD + kD + c];
    out[(size_t)r * kD + c] = a * sigm(g);
}

// block.go:290 depthwise (DWCentred: frames i − pad … i + pad of the same
// clip, zeros outside it, taps in order from 0), then block.go:236
// NormBeforeAct: conv_out_norm and SiLU (stem.go:367 applyAct).
__global__ void __launch_bounds__(kThreads)
    enc_dw_kernel(const __grid_constant__ EncK K, const float *__restrict__ g, int frames, float *__restrict__ out) {
    __shared__ double red[33];
    const int r = blockIdx.x, c = threadIdx.x;
    const int f = r % frames, r0 = r - f, pad = (K.dw_k - 1) / 2;
    float acc = 0.0f;
    for (int j = 0; j < K.dw_k; j++) {
        const int src = f - pad + j;
        if (src < 0 || src >= frames) continue;
        acc = acc + K.dw[(size_t)j * kD + c] * g[(size_t)(r0 + src) * kD + c];
    }
    const float nv = zc_norm_row(acc, K.g_conv_out[c], red);
    out[(size_t)r * kD + c] = nv * sigm(nv);
}

// block.go:246 the conv residual; block.go:172 ffn (FFN2); mhc.go:229
// y = block(u) − u and :270 mix into the lanes.
__global__ void __launch_bounds__(kThreads)
    enc_out_kernel(const __grid_constant__ HadaK H, const __grid_constant__ EncK K, const int *__restrict__ p1,
                   const int *__restrict__ p2, const float *__restrict__ conv, const float *__restrict__ h,
                   const float *__restrict__ u, const float *__restrict__ hp, const float *__restrict__ hr,
                   float *__restrict__ stream) {
    __shared__ double red[33];
    __shared__ HadaSmem S;
    const int r = blockIdx.x, c = threadIdx.x;
    hada_load(H, S);
    const float h2 = h[(size_t)r * kD + c] + conv[(size_t)r * kD + c];
    const float p = zc_norm_row(h2, K.g_pre_hada[c], red);
    const float m = hada_col(H, p1, p2, p, S);
    const float hf = h2 + 0.5f * m;
    const float Y = hf - u[(size_t)r * kD + c];
    float st[kLanes], out[kLanes];
#pragma unroll
    for (int b = 0; b < kLanes; b++) st[b] = stream[((size_t)r * kLanes + b) * kD + c];
#pragma unroll
    for (int a = 0; a < kLanes; a++) {
        float acc = 0.0f;
#pragma unroll
        for (int b = 0; b < kLanes; b++) acc = acc + hr[(size_t)r * kLanes * kLanes + a * kLanes + b] * st[b];
        out[a] = acc + hp[(size_t)r * kLanes + a] * Y;
    }
#pragma unroll
    for (int a = 0; a < kLanes; a++) stream[((size_t)r * kLanes + a) * kD + c] = out[a];
}


// ---- the log-mel front end (frontend/stft.go, mel.go) and the conv stem
// (encoder/stem.go), Best() hypothesis.
constexpr int kNFFT = 512, kHop = 160, kBins = kNFFT / 2 + 1, kMels = 80;
constexpr int kWinLo = (kNFFT - 400) / 2;  // the 400-sample window's offset in the frame

// stft.go:113 spectrum for one frame: the frame centred on sample f·160
// (zeros outside the clip) times the window in float32, then |X_k|² of
// bins 0 … 256 from a float64 radix-2 FFT (bit-reversed load, nine
// butterfly stages; twiddles cos/sin(2πm/512) from the host's libm),
// rounded to float32. One CTA of 256 threads per frame, one butterfly a
// thread per stage.
__device__ __forceinline__ int bitrev9(int j) { return (int)(__brev((unsigned)j) >> 23); }

__global__ void __launch_bounds__(256)
    logmel_spec_kernel(const float *__restrict__ samples, int n, int frames, const float *__restrict__ win,
                       const double *__restrict__ twc, const double *__restrict__ tws, float *__restrict__ spec) {
    __shared__ double re[kNFFT], im[kNFFT];
    const int f = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
    for (int j = t; j < kNFFT; j += blockDim.x) {
        const long long smp = (long long)f * kHop - kNFFT / 2 + j;
        const float v = smp >= 0 && smp < n ? samples[(size_t)b * n + smp] : 0.0f;
        const int r = bitrev9(j);
        re[r] = (double)(v * win[j]);
        im[r] = 0.0;
    }
    __syncthreads();
    for (int half = 1; half < kNFFT; half <<= 1) {
        const int pos = t & (half - 1), i0 = ((t - pos) << 1) + pos, i1 = i0 + half;
        const int m = pos * (kNFFT / (2 * half));
        const double wr = twc[m], wi = -tws[m];
        const double br = re[i1] * wr - im[i1] * wi, bi = re[i1] * wi + im[i1] * wr;
        const double ar = re[i0], ai = im[i0];
        __syncthreads();
        re[i0] = ar + br;
        im[i0] = ai + bi;
        re[i1] = ar - br;
        im[i1] = ai - bi;
        __syncthreads();
    }
    for (int k = t; k < kBins; k += blockDim.x)
        spec[((size_t)b * frames + f) * kBins + k] = (float)(re[k] * re[k] + im[k] * im[k]);
}

// mel.go:78 MelBank.apply: channel m's float64 sum over its non-zero bins.
__global__ void logmel_mel_kernel(const float *__restrict__ spec, int frames, const float *__restrict__ bank,
                                  const int *__restrict__ lo, const int *__restrict__ hi, double *__restrict__ mel) {
    const int f = blockIdx.x, b = blockIdx.y, m = threadIdx.x;
    if (m >= kMels) return;
    const float *row = spec + ((size_t)b * frames + f) * kBins;
    double sum = 0.0;
    for (int k = lo[m]; k < hi[m]; k++) sum = sum + (double)row[k] * (double)bank[k * kMels + m];
    mel[((size_t)b * frames + f) * kMels + m] = sum;
}

// mel.go:302 softLog (ε = knee·max over the clip, log10 as Go's math.Log10:
// ln(x)·(1/ln 10)) and :320 normalise, NormChannel (mean and n − 1
// deviation per channel over time): one CTA per clip, 12 threads per
// channel over interleaved frames; the float64 sums run in a fixed order
// of partial sums (their rounding vanishes in the float32 output).
constexpr int kNormGroups = 12;
__global__ void __launch_bounds__(kMels * kNormGroups)
    logmel_norm_kernel(double *__restrict__ mel, int frames, double knee, float *__restrict__ out) {
    __shared__ double red[kMels * kNormGroups];
    __shared__ double eps_s, mean_s[kMels], sd_s[kMels];
    const int b = blockIdx.x, t = threadIdx.x, m = t % kMels, g = t / kMels;
    double *base = mel + (size_t)b * frames * kMels;
    double mx = -INFINITY;
    for (int f = g; f < frames; f += kNormGroups) mx = fmax(mx, base[(size_t)f * kMels + m]);
    red[t] = mx;
    __syncthreads();
    if (t == 0) {
        double v = -INFINITY;
        for (int i = 0; i < kMels * kNormGroups; i++) v = fmax(v, red[i]);
        v = knee * v;
        eps_s = v == 0.0 ? 1e-10 : v;
    }
    __syncthreads();
    const double eps = eps_s, inv_ln10 = 1.0 / 2.30258509299404568401799145468436421;
    double sum = 0.0;
    for (int f = g; f < frames; f += kNormGroups) {
        const double v = log(base[(size_t)f * kMels + m] + eps) * inv_ln10;
        base[(size_t)f * kMels + m] = v;
        sum = sum + v;
    }
    red[t] = sum;
    __syncthreads();
    if (g == 0) {
        double s2 = 0.0;
        for (int i = 0; i < kNormGroups; i++) s2 = s2 + red[i * kMels + m];
        mean_s[m] = s2 / (double)frames;
    }
    __syncthreads();
    const double mean = mean_s[m];
    double dev = 0.0;
    for (int f = g; f < frames; f += kNormGroups) {
        const double d = base[(size_t)f * kMels + m] - mean;
        dev = dev + d * d;
    }
    red[t] = dev;
    __syncthreads();
    if (g == 0) {
        double s2 = 0.0;
        for (int i = 0; i < kNormGroups; i++) s2 = s2 + red[i * kMels + m];
        sd_s[m] = frames > 1 ? sqrt(s2 / (double)(frames - 1)) : 0.0;
    }
    __syncthreads();
    const double sd = sd_s[m];
    for (int f = g; f < frames; f += kNormGroups)
        out[((size_t)b * frames + f) * kMels + m] = (float)((base[(size_t)f * kMels + m] - mean) / (sd + 1e-5));
}

// stem.go:176 conv on one stage: a 3×3 stride-2 conv with one padding row
// and column on each side (PadSymmetric), the taps in (time, mel) order
// from 0, each product rounded before its add. Stage 0 reads one input
// channel (stem.w, then SiLU, stem.go:367); the depthwise stages read
// channel c for output channel c (groups = channels, no activation).
// x [clips][h][w][cin], out [clips][h'][w'][channels]; a CTA per
// kStemPix output pixels, a thread per channel.
constexpr int kStemPix = 16;
__global__ void stem_conv_kernel(const float *__restrict__ x, int h, int w, int cin, const float *__restrict__ k,
                                 int ho, int wo, int npix, int silu, float *__restrict__ out) {
    const int c = threadIdx.x, channels = blockDim.x, ci = cin == 1 ? 0 : c;
    float kc[9];
#pragma unroll
    for (int t = 0; t < 9; t++) kc[t] = k[t * channels + c];
    const int p0 = blockIdx.x * kStemPix, p1 = min(npix, p0 + kStemPix);
    // The first pixel's coordinates once; the next ones by stepping.
    int ow = p0 % wo, oh = (p0 / wo) % ho, b = p0 / wo / ho;
    for (int pix = p0; pix < p1; pix++) {
        const float *xb = x + (size_t)b * h * w * cin + ci;
        const int ih0 = 2 * oh - 1, iw0 = 2 * ow - 1;
        float acc = 0.0f;
#pragma unroll
        for (int kh = 0; kh < 3; kh++) {
            const int ih = ih0 + kh;
            if (ih < 0 || ih >= h) continue;
            const float *xr = xb + (size_t)ih * w * cin;
#pragma unroll
            for (int kw = 0; kw < 3; kw++) {
                const int iw = iw0 + kw;
                if (iw < 0 || iw >= w) continue;
                acc = acc + xr[iw * cin] * kc[kh * 3 + kw];
            }
        }
        out[(size_t)pix * channels + c] = silu ? acc * sigm(acc) : acc;
        if (++ow == wo) {
            ow = 0;
            if (++oh == ho) {
                oh = 0;
                ++b;
            }
        }
    }
}

// stem.go:253 pointwise's activation (SiLU) in place, or with flatten set,
// into stem.go:262 output's channel-major flatten: out[r][c·w + f] for
// pixel (r, f) of w mel positions. A CTA per kStemPix pixels, a thread
// per channel.
__global__ void stem_act_kernel(const float *__restrict__ y, int w, int npix, int flatten, float *__restrict__ out) {
    const int c = threadIdx.x, channels = blockDim.x;
    const int p1 = min(npix, (blockIdx.x + 1) * kStemPix);
    for (int pix = blockIdx.x * kStemPix; pix < p1; pix++) {
        const float v = y[(size_t)pix * channels + c];
        const float a = v * sigm(v);
        if (!flatten) {
            out[(size_t)pix * channels + c] = a;
            continue;
        }
        const int f = pix % w, r = pix / w;
        out[(size_t)r * channels * w + (size_t)c * w + f] = a;
    }
}

// The encoder's self-attention in any order (WC_ENCODER_ANY_ORDER): a CTA
// stages one clip's int8 keys and values of one KV head and their scales
// in shared memory once, then its 8 warps serve 32 query frames × the KV
// head's query heads, a (frame, head) pair per warp at a time. Per pair:
// the query quantised per head as int8.go:36 QuantizeRow does it (the int8
// kernel's codes); lane l takes keys l, l + 32, …: logits (Σ q8·k8 exact
// in int32)·(s_q·s_k)/√qk, the softmax weights with expf, and all 64
// columns of Σ_j p_j·s_v,j·v8_j by packed f32x2 FMAs; a halving shuffle
// reduction leaves each lane two finished columns, ÷ Σ p. The int8
// kernel's any-order arithmetic in another order (WC_ATTEND_ANY_ORDER's
// bound).
constexpr int kEaFrames = 32, kEaThreads = 256, kEaWarps = kEaThreads / 32, kEaMaxKeys = 1024;
constexpr int kEaVRow = kVD + 16;  // staged V row stride: 16-byte loads of 8 lanes hit distinct banks

// Shared memory: K [nk][48] and V [nk][80] int8 (offsets multiples of 16),
// the warps' query codes [8][64], the key and value scales [nk] and the
// warps' logits [8][nk] (floats).
__host__ __device__ inline size_t ea_smem(int nk) {
    return (size_t)nk * (kQK + kEaVRow) + (size_t)kEaWarps * 64 + 2 * (size_t)nk * 4 + (size_t)kEaWarps * nk * 4;
}

__global__ void __launch_bounds__(kEaThreads, 2)
    enc_attend_kernel(const float *__restrict__ q, const int8_t *__restrict__ k8, const float *__restrict__ ks,
                      const int8_t *__restrict__ v8, const float *__restrict__ vs, int frames, int heads,
                      int kv_heads, float scale, float *__restrict__ out) {
    extern __shared__ __align__(16) unsigned char sm[];
    const int nk = frames, b = blockIdx.z, g = blockIdx.y, f0 = blockIdx.x * kEaFrames;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int8_t *K = reinterpret_cast<int8_t *>(sm);
    int8_t *V = K + (size_t)nk * kQK;
    int8_t *q8 = V + (size_t)nk * kEaVRow + warp * 64;
    float *kss = reinterpret_cast<float *>(V + (size_t)nk * kEaVRow + kEaWarps * 64);
    float *vss = kss + nk;
    float *pw = vss + nk + (size_t)warp * nk;  // this warp's logits: lane l owns keys l, l + 32, ...
    const size_t row0 = (size_t)b * frames;
    for (int i = tid; i < nk * (kQK / 16); i += kEaThreads) {
        const int j = i / (kQK / 16), w = i % (kQK / 16);
        reinterpret_cast<uint4 *>(K)[i] =
            reinterpret_cast<const uint4 *>(k8 + ((row0 + j) * kv_heads + g) * kQK)[w];
    }
    for (int i = tid; i < nk * (kVD / 16); i += kEaThreads) {
        const int j = i / (kVD / 16), w = i % (kVD / 16);
        reinterpret_cast<uint4 *>(V + (size_t)j * kEaVRow)[w] =
            reinterpret_cast<const uint4 *>(v8 + ((row0 + j) * kv_heads + g) * kVD)[w];
    }
    for (int j = tid; j < nk; j += kEaThreads) {
        kss[j] = ks[(row0 + j) * kv_heads + g];
        vss[j] = vs[(row0 + j) * kv_heads + g];
    }
    __syncthreads();
    const int gs = heads / kv_heads, half = kQK / 2;
    uint64_t bias;
    asm("mov.b64 %0, {%1, %1};" : "=l"(bias) : "f"(-8388736.0f));
    for (int task = warp; task < kEaFrames * gs; task += kEaWarps) {
        const int f = f0 + task / gs, h = g * gs + task % gs;
        if (f >= frames) break;  // warp-uniform; later tasks are later frames
        const size_t r = row0 + f;
        const float *qh = q + (r * heads + h) * kQK;
        const float x0 = lane < half ? qh[lane] : 0.0f, x1 = lane < half ? qh[lane + half] : 0.0f;
        float m = fmaxf(fabsf(x0), fabsf(x1));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float sq = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
        if (lane < half) {
            q8[lane] = quant8(x0, sq);
            q8[lane + half] = quant8(x1, sq);
        }
        __syncwarp();
        uint32_t qw[kQK / 4];
#pragma unroll
        for (int w = 0; w < kQK / 16; w++) {
            const uint4 v = reinterpret_cast<const uint4 *>(q8)[w];
            qw[4 * w] = v.x, qw[4 * w + 1] = v.y, qw[4 * w + 2] = v.z, qw[4 * w + 3] = v.w;
        }
        __syncwarp();  // q8 is rewritten by the next pair
        // Logits of this lane's keys.
        float mx = -INFINITY;
        for (int j = lane; j < nk; j += 32) {
            const uint4 *kr = reinterpret_cast<const uint4 *>(K + (size_t)j * kQK);
            int32_t d0 = 0, d1 = 0;
#pragma unroll
            for (int w = 0; w < kQK / 16; w++) {
                const uint4 kv = kr[w];
                d0 = __dp4a((int)qw[4 * w], (int)kv.x, d0);
                d1 = __dp4a((int)qw[4 * w + 1], (int)kv.y, d1);
                d0 = __dp4a((int)qw[4 * w + 2], (int)kv.z, d0);
                d1 = __dp4a((int)qw[4 * w + 3], (int)kv.w, d1);
            }
            const float l = (float)(d0 + d1) * (sq * kss[j]) / scale;
            pw[j] = l;
            mx = fmaxf(mx, l);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        // Σ_j p_j·s_v·v8_j over this lane's keys, all 64 columns, packed.
        uint64_t acc[kVD / 2];
#pragma unroll
        for (int c = 0; c < kVD / 2; c++) acc[c] = 0;
        float sum = 0.0f;
        for (int j = lane; j < nk; j += 32) {
            {
                const float e = expf(pw[j] - mx);
                sum += e;
                uint64_t ww;
                asm("mov.b64 %0, {%1, %1};" : "=l"(ww) : "f"(e * vss[j]));
                const uint4 *vr = reinterpret_cast<const uint4 *>(V + (size_t)j * kEaVRow);
#pragma unroll
                for (int w = 0; w < kVD / 16; w++) {
                    const uint4 v = vr[w];
                    const uint32_t vw[4] = {v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u,
                                            v.w ^ 0x80808080u};
#pragma unroll
                    for (int u = 0; u < 4; u++) {
#pragma unroll
                        for (int bb = 0; bb < 4; bb += 2) {
                            // Two codes as floats: 2^23 + (code + 128), less the bias.
                            uint64_t cv;
                            asm("mov.b64 %0, {%1, %2};"
                                : "=l"(cv)
                                : "r"(__byte_perm(vw[u], 0x4B000000u, 0x7540u + bb)),
                                  "r"(__byte_perm(vw[u], 0x4B000000u, 0x7540u + bb + 1)));
                            asm("add.rn.f32x2 %0, %0, %1;" : "+l"(cv) : "l"(bias));
                            uint64_t &a = acc[(16 * w + 4 * u + bb) / 2];
                            asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(a) : "l"(ww), "l"(cv));
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        // Halving reduction over the lanes: after the step of width s the lane
        // keeps s of the column pairs; at the end lane l holds pair l.
        float av[kVD];
#pragma unroll
        for (int c = 0; c < kVD / 2; c++) asm("mov.b64 {%0, %1}, %2;" : "=f"(av[2 * c]), "=f"(av[2 * c + 1]) : "l"(acc[c]));
#pragma unroll
        for (int s = 16; s >= 1; s >>= 1) {
            const bool upper = (lane & s) != 0;
#pragma unroll
            for (int c = 0; c < s; c++) {
                // pairs [0, 2s): the lower half stays with the lanes without bit s
                const float k0 = upper ? av[2 * c] : av[2 * (c + s)];
                const float k1 = upper ? av[2 * c + 1] : av[2 * (c + s) + 1];
                const float g0 = __shfl_xor_sync(0xffffffffu, k0, s);
                const float g1 = __shfl_xor_sync(0xffffffffu, k1, s);
                const float m0 = upper ? av[2 * (c + s)] : av[2 * c];
                const float m1 = upper ? av[2 * (c + s) + 1] : av[2 * c + 1];
                av[2 * c] = m0 + g0;
                av[2 * c + 1] = m1 + g1;
            }
        }
        // The lanes with bit s set kept the upper half at every step, so lane
        // l holds column pair l.
        const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
        float *o = out + (r * heads + h) * kVD + 2 * lane;
        o[0] = av[0] * inv;
        o[1] = av[1] * inv;
    }
}
}  // namespace
}  // namespace wb

struct wc_encoder : DevStore {
    wc_encoder_desc d{};  // sizes (pointers not kept)
    int max_clips = 0, max_frames = 0, flags = 0, dw_k = 0;
    bool tc = false, any = false, xq_needed = false;
    struct Layer {
        LayerK k;
        EncK e;
        HadaK h0, h1;
        wc_cq *q, *kk, *v, *g, *o, *pw1, *pw2, *ppre, *ppost, *pres;
        bool phi_fused = false;
    };
    std::vector<Layer> layers;
    const float *g_final = nullptr, *rcos = nullptr, *rsin = nullptr;
    const int *p1 = nullptr, *p2 = nullptr;
    float att_scale = 1.0f;
    // [rows][…] buffers, rows = clips · frames
    float *stream = nullptr, *xq = nullptr, *phi_pre = nullptr, *phi_post = nullptr, *phi_res = nullptr;
    float *hr = nullptr, *hp = nullptr, *u = nullptr, *h = nullptr, *n = nullptr;
    float *q = nullptr, *k = nullptr, *v = nullptr, *g = nullptr, *qo = nullptr, *att = nullptr, *a = nullptr;
    float *p = nullptr, *glu = nullptr, *cv = nullptr;
    int8_t *k8 = nullptr, *v8 = nullptr;
    float *ks = nullptr, *vs = nullptr;
    int32_t *nk = nullptr;
    void *tcbuf = nullptr;
    size_t tcbytes = 0;
    // The stem and the front end (when the desc has them).
    bool has_stem = false;
    int channels = 0;
    const float *sw = nullptr, *sdw[2] = {nullptr, nullptr}, *win = nullptr, *bank = nullptr;
    const double *twc = nullptr, *tws = nullptr;
    const int *mlo = nullptr, *mhi = nullptr;
    double knee = 0.0;
    wc_cq *spw[2] = {nullptr, nullptr}, *sout = nullptr;
    float *spec = nullptr, *melf = nullptr, *s0 = nullptr, *s1 = nullptr, *s2 = nullptr, *s3 = nullptr;
    float *s4 = nullptr, *flat = nullptr, *xin = nullptr;
    double *mel64 = nullptr;
};

namespace {

wc_status enc_matrix(const wc_cq *m, const char *what, int layer, int out, int in) {
    if (!m) return set_error(WC_ERR_INVALID, fmt("encoder: layer %d %s: nil matrix", layer, what));
    if (wc_cq_out(m) != out || wc_cq_in(m) != in)
        return set_error(WC_ERR_INVALID, fmt("encoder: layer %d %s has shape (%d, %d), want (%d, %d)", layer, what,
                                             wc_cq_out(m), wc_cq_in(m), out, in));
    return WC_OK;
}

wc_status enc_gemms(wc_encoder *e, std::initializer_list<const wc_cq *> ms, const float *x,
                    std::initializer_list<float *> ys, int rows, cudaStream_t st) {
    std::vector<const wc_cq *> m(ms);
    std::vector<float *> y(ys);
    return gemms_device(m.data(), (int)m.size(), x, y.data(), rows, e->tc, e->tcbuf, e->tcbytes, st);
}

wc_status enc_hada(wc_encoder *e, const wc_hadamard_mlp &S, HadaK *H) {
    const int nn = kNA * kNB;
    if (!S.d1 || !S.d2 || !S.b2 || !S.d3 || !S.d4 || !S.w1a || !S.w1b || !S.w2a || !S.w2b || !S.w3a || !S.w3b ||
        !S.cond_v || !S.cond_u)
        return set_error(WC_ERR_INVALID, "encoder: nil HadamardMLP tensor");
    DEC_ST(e->upload(&H->d1, S.d1, nn));
    DEC_ST(e->upload(&H->d2, S.d2, nn));
    DEC_ST(e->upload(&H->b2, S.b2, nn));
    DEC_ST(e->upload(&H->d3, S.d3, nn));
    DEC_ST(e->upload(&H->d4, S.d4, nn));
    const float *wa[3] = {S.w1a, S.w2a, S.w3a}, *wbb[3] = {S.w1b, S.w2b, S.w3b};
    for (int i = 0; i < 3; i++) {
        DEC_ST(e->upload(&H->wa[i], wa[i], kNA * kNA));
        DEC_ST(e->upload(&H->wb[i], wbb[i], kNB * kNB));
    }
    DEC_ST(e->upload(&H->cond_v, S.cond_v, (size_t)kD * kRank));
    DEC_ST(e->upload(&H->cond_u, S.cond_u, (size_t)kRank * nn));
    return WC_OK;
}

// One encoder layer on R rows of `frames` frames per clip.
wc_status enc_layer(wc_encoder *e, int l, int R, int frames, cudaStream_t st) {
    auto &L = e->layers[l];
    const wc_encoder_desc &D = e->d;
    if (L.phi_fused) {
        PhiViews pv{};
        CqShape sh{};
        cq_internal(L.ppre, &sh, &pv.v[0]);
        cq_internal(L.ppost, nullptr, &pv.v[1]);
        cq_internal(L.pres, nullptr, &pv.v[2]);
        pv.y[0] = e->phi_pre, pv.y[1] = e->phi_post, pv.y[2] = e->phi_res;
        DEC_LAUNCH(mhc_phi_kernel<<<R, kThreads, 0, st>>>(e->stream, sh, pv));
    } else {
        DEC_LAUNCH(mhc_in_kernel<<<R, kThreads, 0, st>>>(e->stream, e->xq));
        DEC_ST(enc_gemms(e, {L.ppre, L.ppost, L.pres}, e->xq, {e->phi_pre, e->phi_post, e->phi_res}, R, st));
    }
    DEC_LAUNCH(sinkhorn_kernel<<<(R + 3) / 4, 128, 0, st>>>(L.k, e->phi_res, e->hr, R));
    // u, and FFN1's input: the pre_hada_0 norm of u (LayerK's g_norm_in).
    DEC_LAUNCH(mhc_block_in_kernel<<<R, kThreads, 0, st>>>(L.k, e->stream, e->phi_pre, e->phi_post, e->phi_res,
                                                           nullptr, nullptr, e->u, e->h, e->n, e->hp));
    DEC_LAUNCH(enc_ffn_kernel<<<R, kThreads, 0, st>>>(L.h0, e->p1, e->p2, e->n, e->h, L.e.g_attn_in, e->a));
    DEC_ST(enc_gemms(e, {L.q, L.kk, L.v, L.g}, e->a, {e->q, e->k, e->v, e->g}, R, st));
    DEC_LAUNCH(enc_qkv_kernel<<<R, kThreads, 0, st>>>(L.e, e->q, e->k, e->v, D.heads, D.kv_heads, frames, e->rcos,
                                                      e->rsin, e->qo, e->k8, e->ks, e->v8, e->vs));
    if (e->any && frames <= kEaMaxKeys) {
        const dim3 grid((frames + kEaFrames - 1) / kEaFrames, D.kv_heads, R / frames);
        DEC_LAUNCH(enc_attend_kernel<<<grid, kEaThreads, ea_smem(frames), st>>>(
            e->qo, e->k8, e->ks, e->v8, e->vs, frames, D.heads, D.kv_heads, e->att_scale, e->att));
    } else {
        DEC_ST(attend_streams_grouped(R, e->qo, D.heads, e->k8, e->ks, e->v8, e->vs, frames, e->nk, D.kv_heads, kQK,
                                      kVD, e->att_scale, WC_ATTEND_QUANT_Q | (e->any ? WC_ATTEND_ANY_ORDER : 0),
                                      e->att, frames, st));
    }
    DEC_LAUNCH(gate_kernel<<<R, kThreads, 0, st>>>(e->att, e->g, D.heads * kVD));
    DEC_ST(enc_gemms(e, {L.o}, e->att, {e->a}, R, st));
    // post_attn_norm, the σ(attn_gate) residual, then conv_norm (g_xn).
    DEC_LAUNCH(post_attn_kernel<<<R, kThreads, 0, st>>>(L.k, e->a, e->h, e->n));
    DEC_ST(enc_gemms(e, {L.pw1}, e->n, {e->p}, R, st));
    DEC_LAUNCH(enc_glu_kernel<<<R, kThreads, 0, st>>>(e->p, e->glu));
    DEC_LAUNCH(enc_dw_kernel<<<R, kThreads, 0, st>>>(L.e, e->glu, frames, e->cv));
    DEC_ST(enc_gemms(e, {L.pw2}, e->cv, {e->a}, R, st));
    DEC_LAUNCH(enc_out_kernel<<<R, kThreads, 0, st>>>(L.h1, L.e, e->p1, e->p2, e->a, e->h, e->u, e->hp, e->hr,
                                                      e->stream));
    return WC_OK;
}

}  // namespace

extern "C" wc_status wc_encoder_create(const wc_encoder_desc *desc, int max_clips, int max_frames, int flags,
                                       wc_encoder **out) {
    if (!out) return set_error(WC_ERR_INVALID, "encoder: nil handle pointer");
    *out = nullptr;
    if (!desc) return set_error(WC_ERR_INVALID, "encoder: nil description");
    const wc_encoder_desc &D = *desc;
    if (D.dim != kD || D.lanes != kLanes || D.qk != kQK || D.vd != kVD || D.na != kNA || D.nb != kNB ||
        D.rank != kRank)
        return set_error(WC_ERR_UNSUPPORTED,
                         fmt("encoder: this build's kernels take width 512 in 4 lanes, heads of 48/64 and a 16 x 32 "
                             "HadamardMLP of rank 8 (got width %d, %d lanes, heads %d/%d, %d x %d rank %d)",
                             D.dim, D.lanes, D.qk, D.vd, D.na, D.nb, D.rank));
    if (D.layers <= 0 || D.heads <= 0 || D.kv_heads <= 0 || D.heads % D.kv_heads != 0)
        return set_error(WC_ERR_INVALID,
                         fmt("encoder: %d layers, %d query heads over %d KV heads", D.layers, D.heads, D.kv_heads));
    if (D.heads * kVD != kD)
        return set_error(WC_ERR_UNSUPPORTED, "encoder: the attention output must be as wide as the model (heads·64 = 512)");
    if (D.dw_kernel < 1 || D.dw_kernel > 31 || D.dw_kernel % 2 == 0)
        return set_error(WC_ERR_INVALID, fmt("encoder: depthwise kernel of %d taps (odd, at most 31)", D.dw_kernel));
    if (max_clips <= 0 || max_frames <= 0 || (long long)max_clips * max_frames > 65535)
        return set_error(WC_ERR_INVALID, fmt("encoder: room for %d clips of %d frames (at most 65535 rows)", max_clips,
                                             max_frames));
    if (!D.layer || !D.final_norm || !D.hada_p1 || !D.hada_p2 || D.rope_len <= 0)
        return set_error(WC_ERR_INVALID, "encoder: nil tensor");

    std::unique_ptr<wc_encoder> e(new (std::nothrow) wc_encoder);
    if (!e) return set_error(WC_ERR_NOMEM, "encoder: out of host memory");
    WB_CUDA(cudaGetDevice(&e->device));
    e->d = D;
    e->d.layer = nullptr;
    e->d.hada_p1 = e->d.hada_p2 = nullptr;
    e->d.final_norm = nullptr;
    e->max_clips = max_clips;
    e->max_frames = max_frames;
    e->flags = flags;
    e->tc = (flags & WC_ENCODER_TENSOR_CORES) != 0;
    e->any = (flags & WC_ENCODER_ANY_ORDER) != 0;
    if (e->any)
        WB_CUDA(cudaFuncSetAttribute(enc_attend_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)ea_smem(std::min(max_frames, kEaMaxKeys))));
    e->dw_k = D.dw_kernel;
    const int qw = D.heads * kQK, kw = D.kv_heads * kQK, vw = D.kv_heads * kVD;
    for (int l = 0; l < D.layers; l++) {
        const wc_encoder_layer &S = D.layer[l];
        DEC_ST(enc_matrix(S.q_proj, "q_proj", l, qw, kD));
        DEC_ST(enc_matrix(S.k_proj, "k_proj", l, kw, kD));
        DEC_ST(enc_matrix(S.v_proj, "v_proj", l, vw, kD));
        DEC_ST(enc_matrix(S.gate_proj, "gate_proj", l, D.heads * kVD, kD));
        DEC_ST(enc_matrix(S.out_proj, "out_proj", l, kD, D.heads * kVD));
        DEC_ST(enc_matrix(S.pw1, "pw1", l, 2 * kD, kD));
        DEC_ST(enc_matrix(S.pw2, "pw2", l, kD, kD));
        DEC_ST(enc_matrix(S.phi_pre, "mhc_phi_pre", l, kLanes, kLanes * kD));
        DEC_ST(enc_matrix(S.phi_post, "mhc_phi_post", l, kLanes, kLanes * kD));
        DEC_ST(enc_matrix(S.phi_res, "mhc_phi_res", l, kLanes * kLanes, kLanes * kD));
        if (!S.pre_hada_0 || !S.norm_in || !S.post_norm || !S.conv_norm || !S.conv_out_norm || !S.pre_hada ||
            !S.q_norm || !S.k_norm || !S.dw || !S.b_pre || !S.b_post || !S.b_res)
            return set_error(WC_ERR_INVALID, fmt("encoder: layer %d: nil tensor", l));
        wc_encoder::Layer L{};
        DEC_ST(e->view(S.q_proj, &L.q));
        DEC_ST(e->view(S.k_proj, &L.kk));
        DEC_ST(e->view(S.v_proj, &L.v));
        DEC_ST(e->view(S.gate_proj, &L.g));
        DEC_ST(e->view(S.out_proj, &L.o));
        DEC_ST(e->view(S.pw1, &L.pw1));
        DEC_ST(e->view(S.pw2, &L.pw2));
        DEC_ST(e->view(S.phi_pre, &L.ppre));
        DEC_ST(e->view(S.phi_post, &L.ppost));
        DEC_ST(e->view(S.phi_res, &L.pres));
        {
            CqShape a{}, b{}, c{};
            CqView va{}, vb{}, vc{};
            cq_internal(L.ppre, &a, &va);
            cq_internal(L.ppost, &b, &vb);
            cq_internal(L.pres, &c, &vc);
            auto same = [](const CqShape &x, const CqShape &y) {
                return x.in == y.in && x.group == y.group && x.bits == y.bits && x.cb_max == y.cb_max &&
                       x.lut_step == y.lut_step && std::memcmp(x.cb, y.cb, sizeof x.cb) == 0;
            };
            L.phi_fused = !e->tc && a.bits == 4 && a.group == 128 && a.in == kPhiIn && a.gb == 64 &&
                          a.pad == kPhiIn && same(a, b) && same(a, c);
            if (!L.phi_fused) e->xq_needed = true;
        }
        LayerK &K = L.k;
        DEC_ST(e->upload(&K.g_norm_in, S.pre_hada_0, kD, true));
        DEC_ST(e->upload(&K.g_post, S.post_norm, kD, true));
        DEC_ST(e->upload(&K.g_xn, S.conv_norm, kD, true));
        DEC_ST(e->upload(&K.b_pre, S.b_pre, kLanes));
        DEC_ST(e->upload(&K.b_post, S.b_post, kLanes));
        DEC_ST(e->upload(&K.b_res, S.b_res, kLanes * kLanes));
        K.gate = sigmoid_host(S.attn_gate);
        K.a_pre = S.a_pre;
        K.a_post = S.a_post;
        K.a_res = S.a_res;
        K.lane = l % kLanes;
        EncK &E = L.e;
        DEC_ST(e->upload(&E.g_attn_in, S.norm_in, kD, true));
        DEC_ST(e->upload(&E.g_qn, S.q_norm, kQK, true));
        DEC_ST(e->upload(&E.g_kn, S.k_norm, kQK, true));
        DEC_ST(e->upload(&E.g_conv_out, S.conv_out_norm, kD, true));
        DEC_ST(e->upload(&E.g_pre_hada, S.pre_hada, kD, true));
        DEC_ST(e->upload(&E.dw, S.dw, (size_t)D.dw_kernel * kD));
        E.dw_k = D.dw_kernel;
        DEC_ST(enc_hada(e.get(), S.hada_0, &L.h0));
        DEC_ST(enc_hada(e.get(), S.hada, &L.h1));
        e->layers.push_back(L);
    }
    DEC_ST(e->hada_perms(D.hada_p1, D.hada_p2, &e->p1, &e->p2));
    DEC_ST(e->upload(&e->g_final, D.final_norm, kD, true));
    DEC_ST(e->rope_tables(D.rope_theta, D.rope_len, &e->rcos, &e->rsin));
    e->att_scale = (float)std::sqrt((double)kQK);  // attention.go:407 attendScale
    const int Tm = max_frames;
    const bool any_stem = D.stem_w || D.stem_dw_1 || D.stem_dw_2 || D.stem_pw_1 || D.stem_pw_2 || D.stem_out ||
                          D.mel_filters;
    if (any_stem) {
        const int C = D.stem_channels;
        if (!D.stem_w || !D.stem_dw_1 || !D.stem_dw_2 || !D.stem_pw_1 || !D.stem_pw_2 || !D.stem_out ||
            !D.mel_filters || C <= 0 || C > 1024)
            return set_error(WC_ERR_INVALID, fmt("encoder: stem of %d channels with a nil tensor", C));
        const int wout = wc_encoder_stem_frames(kMels);  // 10 mel positions after three stages
        auto stem_mat = [&](const wc_cq *m, const char *what, int out, int in) -> wc_status {
            if (wc_cq_out(m) != out || wc_cq_in(m) != in)
                return set_error(WC_ERR_INVALID, fmt("encoder: %s has shape (%d, %d), want (%d, %d)", what,
                                                     wc_cq_out(m), wc_cq_in(m), out, in));
            return WC_OK;
        };
        DEC_ST(stem_mat(D.stem_pw_1, "stem.pw_1", C, C));
        DEC_ST(stem_mat(D.stem_pw_2, "stem.pw_2", C, C));
        DEC_ST(stem_mat(D.stem_out, "stem.out", kD, wout * C));
        e->has_stem = true;
        e->channels = C;
        DEC_ST(e->upload(&e->sw, D.stem_w, (size_t)9 * C));
        DEC_ST(e->upload(&e->sdw[0], D.stem_dw_1, (size_t)9 * C));
        DEC_ST(e->upload(&e->sdw[1], D.stem_dw_2, (size_t)9 * C));
        DEC_ST(e->view(D.stem_pw_1, &e->spw[0]));
        DEC_ST(e->view(D.stem_pw_2, &e->spw[1]));
        DEC_ST(e->view(D.stem_out, &e->sout));
        DEC_ST(e->upload(&e->bank, D.mel_filters, (size_t)kBins * kMels));
        {
            // mel.go:30 MelBank's non-zero bin range of every channel.
            std::vector<int32_t> lh(2 * kMels, 0);
            for (int m = 0; m < kMels; m++) {
                int lo = -1, hi = -1;
                for (int k = 0; k < kBins; k++)
                    if (D.mel_filters[k * kMels + m] != 0.0f) {
                        if (lo < 0) lo = k;
                        hi = k + 1;
                    }
                lh[m] = lo < 0 ? 0 : lo;
                lh[kMels + m] = lo < 0 ? 0 : hi;
            }
            int32_t *d = nullptr;
            DEC_ST(e->alloc(&d, lh.size()));
            WB_CUDA(cudaMemcpy(d, lh.data(), lh.size() * sizeof(int32_t), cudaMemcpyHostToDevice));
            e->mlo = d;
            e->mhi = d + kMels;
        }
        {
            // stft.go:60: the 400-sample symmetric Hann window at offset 56
            // of the 512-point frame, and the DFT's twiddles.
            const double pi = 3.14159265358979323846;
            std::vector<float> w(kNFFT, 0.0f);
            for (int k = 0; k < 400; k++) w[kWinLo + k] = (float)(0.5 - 0.5 * std::cos(2.0 * pi * k / 399.0));
            DEC_ST(e->upload(&e->win, w.data(), w.size()));
            std::vector<double> c(kNFFT), sn(kNFFT);
            for (int m = 0; m < kNFFT; m++) {
                c[m] = std::cos(2.0 * pi * m / kNFFT);
                sn[m] = std::sin(2.0 * pi * m / kNFFT);
            }
            double *dc = nullptr, *ds = nullptr;
            DEC_ST(e->alloc(&dc, kNFFT));
            DEC_ST(e->alloc(&ds, kNFFT));
            WB_CUDA(cudaMemcpy(dc, c.data(), kNFFT * sizeof(double), cudaMemcpyHostToDevice));
            WB_CUDA(cudaMemcpy(ds, sn.data(), kNFFT * sizeof(double), cudaMemcpyHostToDevice));
            e->twc = dc;
            e->tws = ds;
        }
        e->knee = std::pow(10.0, -7.6);  // mel.go:24 soft76
        const size_t B = (size_t)max_clips, F = (size_t)8 * Tm;
        DEC_ST(e->alloc(&e->spec, B * F * kBins));
        DEC_ST(e->alloc(&e->mel64, B * F * kMels));
        DEC_ST(e->alloc(&e->melf, B * F * kMels));
        DEC_ST(e->alloc(&e->s0, B * 4 * Tm * 40 * C));
        DEC_ST(e->alloc(&e->s1, B * 2 * Tm * 20 * C));
        DEC_ST(e->alloc(&e->s2, B * 2 * Tm * 20 * C));
        DEC_ST(e->alloc(&e->s3, B * Tm * wout * C));
        DEC_ST(e->alloc(&e->s4, B * Tm * wout * C));
        DEC_ST(e->alloc(&e->flat, B * Tm * wout * C));
        DEC_ST(e->alloc(&e->xin, B * Tm * kD));
    }

    const size_t R = (size_t)max_clips * max_frames;
    DEC_ST(e->alloc(&e->stream, R * kLanes * kD));
    if (e->xq_needed) DEC_ST(e->alloc(&e->xq, R * kLanes * kD));
    DEC_ST(e->alloc(&e->phi_pre, R * kLanes));
    DEC_ST(e->alloc(&e->phi_post, R * kLanes));
    DEC_ST(e->alloc(&e->phi_res, R * kLanes * kLanes));
    DEC_ST(e->alloc(&e->hr, R * kLanes * kLanes));
    DEC_ST(e->alloc(&e->hp, R * kLanes));
    DEC_ST(e->alloc(&e->u, R * kD));
    DEC_ST(e->alloc(&e->h, R * kD));
    DEC_ST(e->alloc(&e->n, R * kD));
    DEC_ST(e->alloc(&e->q, R * qw));
    DEC_ST(e->alloc(&e->k, R * kw));
    DEC_ST(e->alloc(&e->v, R * vw));
    DEC_ST(e->alloc(&e->g, R * D.heads * kVD));
    DEC_ST(e->alloc(&e->qo, R * qw));
    DEC_ST(e->alloc(&e->att, R * D.heads * kVD));
    DEC_ST(e->alloc(&e->a, R * kD));
    DEC_ST(e->alloc(&e->p, R * 2 * kD));
    DEC_ST(e->alloc(&e->glu, R * kD));
    DEC_ST(e->alloc(&e->cv, R * kD));
    DEC_ST(e->alloc(&e->k8, R * kw));
    DEC_ST(e->alloc(&e->v8, R * vw));
    DEC_ST(e->alloc(&e->ks, R * D.kv_heads));
    DEC_ST(e->alloc(&e->vs, R * D.kv_heads));
    DEC_ST(e->alloc(&e->nk, R));
    if (e->tc) {
        // The rotated image of the tensor-core products: R rows at 512 in,
        // and at 2048 in for the φ products; the stem's pointwise rows at
        // its channel count and stem.out's rows at 10 · channels.
        e->tcbytes = std::max(tc_a_bytes((int)R, (kD + 63) / 64), tc_a_bytes((int)R, (kLanes * kD + 63) / 64));
        if (e->has_stem) {
            const int C = e->channels;
            e->tcbytes = std::max(e->tcbytes, tc_a_bytes((int)(max_clips * 2LL * Tm * 20), (C + 63) / 64));
            e->tcbytes = std::max(e->tcbytes, tc_a_bytes((int)R, (10 * C + 63) / 64));
        }
        unsigned char *pb = nullptr;
        DEC_ST(e->alloc(&pb, e->tcbytes));
        e->tcbuf = pb;
    }
    *out = e.release();
    return WC_OK;
}

extern "C" void wc_encoder_destroy(wc_encoder *e) { delete e; }

extern "C" wc_status wc_encoder_stack(wc_encoder *e, const float *x, int clips, int frames, float *out,
                                      wc_stream stream) {
    if (!e) return set_error(WC_ERR_INVALID, "encoder: nil encoder");
    int cur = 0;
    WB_CUDA(cudaGetDevice(&cur));
    if (cur != e->device)
        return set_error(WC_ERR_INVALID, fmt("encoder: built on device %d, called on device %d", e->device, cur));
    if (clips < 0 || frames < 0 || clips > e->max_clips || frames > e->max_frames)
        return set_error(WC_ERR_INVALID, fmt("encoder: %d clips of %d frames exceed the room for %d of %d", clips,
                                             frames, e->max_clips, e->max_frames));
    if (frames > e->d.rope_len)
        return set_error(WC_ERR_INVALID, fmt("encoder: RoPE tables for %d positions, want %d", e->d.rope_len, frames));
    if (clips == 0 || frames == 0) return WC_OK;
    if (!x || !out) return set_error(WC_ERR_INVALID, "encoder: nil input or output");
    cudaStream_t st = (cudaStream_t)stream;
    const int R = clips * frames;
    DEC_LAUNCH(fill_kernel<<<(R + 255) / 256, 256, 0, st>>>(e->nk, frames, R));
    DEC_LAUNCH(enc_expand_kernel<<<R, kThreads, 0, st>>>(x, e->stream));
    for (int l = 0; l < e->d.layers; l++) DEC_ST(enc_layer(e, l, R, frames, st));
    DEC_LAUNCH(final_kernel<<<R, kThreads, 0, st>>>(e->stream, e->g_final, out));
    return WC_OK;
}

extern "C" int wc_encoder_stem_frames(int frames) {
    int n = frames;
    for (int st = 0; st < 3; st++) {
        if (n + 2 < 3) return 0;
        n = (n + 2 - 3) / 2 + 1;  // stem.go:166 length: 3 taps, stride 2, one padding position each side
    }
    return n;
}

static wc_status enc_stem_ready(wc_encoder *e) {
    if (!e) return set_error(WC_ERR_INVALID, "encoder: nil encoder");
    int cur = 0;
    WB_CUDA(cudaGetDevice(&cur));
    if (cur != e->device)
        return set_error(WC_ERR_INVALID, fmt("encoder: built on device %d, called on device %d", e->device, cur));
    if (!e->has_stem) return set_error(WC_ERR_INVALID, "encoder: built without the stem and the mel bank");
    return WC_OK;
}

extern "C" wc_status wc_encoder_logmel(wc_encoder *e, const float *samples, int clips, int n, float *mel,
                                       wc_stream stream) {
    DEC_ST(enc_stem_ready(e));
    if (clips < 0 || n < 0 || clips > e->max_clips || n / kHop > 8 * e->max_frames)
        return set_error(WC_ERR_INVALID, fmt("encoder: %d clips of %d samples exceed the room for %d of %d", clips, n,
                                             e->max_clips, 8 * e->max_frames * kHop + kHop - 1));
    const int F = n / kHop;  // stft.go:35 FrameCount, centred framing
    if (clips == 0 || F == 0) return WC_OK;
    if (!samples || !mel) return set_error(WC_ERR_INVALID, "encoder: nil samples or mel");
    cudaStream_t st = (cudaStream_t)stream;
    DEC_LAUNCH(logmel_spec_kernel<<<dim3(F, clips), 256, 0, st>>>(samples, n, F, e->win, e->twc, e->tws, e->spec));
    DEC_LAUNCH(logmel_mel_kernel<<<dim3(F, clips), 96, 0, st>>>(e->spec, F, e->bank, e->mlo, e->mhi, e->mel64));
    DEC_LAUNCH(logmel_norm_kernel<<<clips, kMels * kNormGroups, 0, st>>>(e->mel64, F, e->knee, mel));
    return WC_OK;
}

extern "C" wc_status wc_encoder_stem(wc_encoder *e, const float *mel, int clips, int frames, float *x,
                                     wc_stream stream) {
    DEC_ST(enc_stem_ready(e));
    const int T = wc_encoder_stem_frames(frames);
    if (clips < 0 || frames < 0 || clips > e->max_clips || T > e->max_frames)
        return set_error(WC_ERR_INVALID, fmt("encoder: %d clips of %d mel frames (%d stem frames) exceed the room for "
                                             "%d of %d", clips, frames, T, e->max_clips, e->max_frames));
    if (clips == 0 || T == 0) return WC_OK;
    if (!mel || !x) return set_error(WC_ERR_INVALID, "encoder: nil mel or output");
    cudaStream_t st = (cudaStream_t)stream;
    const int C = e->channels;
    const int h1 = (frames - 1) / 2 + 1, w1 = (kMels - 1) / 2 + 1;
    const int h2 = (h1 - 1) / 2 + 1, w2 = (w1 - 1) / 2 + 1;
    const int w3 = (w2 - 1) / 2 + 1;
    const int p1 = clips * h1 * w1, p2 = clips * h2 * w2, p3 = clips * T * w3;
    auto ctas = [](int npix) { return (npix + kStemPix - 1) / kStemPix; };
    DEC_LAUNCH(stem_conv_kernel<<<ctas(p1), C, 0, st>>>(mel, frames, kMels, 1, e->sw, h1, w1, p1, 1, e->s0));
    DEC_LAUNCH(stem_conv_kernel<<<ctas(p2), C, 0, st>>>(e->s0, h1, w1, C, e->sdw[0], h2, w2, p2, 0, e->s1));
    DEC_ST(enc_gemms(e, {e->spw[0]}, e->s1, {e->s2}, p2, st));
    DEC_LAUNCH(stem_act_kernel<<<ctas(p2), C, 0, st>>>(e->s2, w2, p2, 0, e->s2));
    DEC_LAUNCH(stem_conv_kernel<<<ctas(p3), C, 0, st>>>(e->s2, h2, w2, C, e->sdw[1], T, w3, p3, 0, e->s3));
    DEC_ST(enc_gemms(e, {e->spw[1]}, e->s3, {e->s4}, p3, st));
    DEC_LAUNCH(stem_act_kernel<<<ctas(p3), C, 0, st>>>(e->s4, w3, p3, 1, e->flat));
    DEC_ST(enc_gemms(e, {e->sout}, e->flat, {x}, clips * T, st));
    return WC_OK;
}

extern "C" wc_status wc_encoder_embed(wc_encoder *e, const float *samples, int clips, int n, float *out,
                                      wc_stream stream) {
    DEC_ST(enc_stem_ready(e));
    const int F = n < 0 ? 0 : n / kHop, T = wc_encoder_stem_frames(F);
    DEC_ST(wc_encoder_logmel(e, samples, clips, n, e->melf, stream));
    DEC_ST(wc_encoder_stem(e, e->melf, clips, F, e->xin, stream));
    return wc_encoder_stack(e, e->xin, clips, T, out, stream);
}
