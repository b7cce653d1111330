// cq_lut.cu — the CQ LUT GEMV/GEMM (internal/cq/lut.go) on sm_100a.
//
// y[r] = Σ_g float32(Σ_{j∈g} v_j[idx]) · (norm[r,g] · step_g), accumulated in
// group order, where v are the activation's integer tables (lut.go:239-287)
// and the integer sums are exact. The kernel reproduces the reference's lut
// kernel bit for bit:
//   - the FWHT butterflies of kernel.go:384 fwht, stage by stage;
//   - M, 8191/M, the table products and their round-half-even conversion
//     with separate IEEE roundings (__fmul_rn/__fdiv_rn/__float2int_rn; no
//     FMA contraction);
//   - Σv in int32 (exact, so any summation order gives the same integer);
//   - step = M · lutStep, coef = norm · step, term = float32(Σv) · coef and
//     y += term in group order (lut.go:308-309).
//
// Work split. One CTA owns one activation and a tile of kTileRows rows of
// one matrix. It rotates and tabulates the activation into shared memory
// (the tables of all matrices of a GEMMs launch are the same), then its
// threads each take (row, group) items: a 16-byte (or gb-byte) coalesced
// load of the row's index bytes for the group from the group-major layout,
// table lookups, an exact integer sum, and one float term into shared
// memory. A last pass adds each row's terms in group order.
#include "common.cuh"
#include "cq_kernels.cuh"

namespace wb {

namespace {

constexpr int kThreads = 256;

// Index of the matrix that owns global tile t (tile_start is a prefix sum).
__device__ __forceinline__ int find_matrix(const LutParams &p, int t) {
    int lo = 0, hi = p.n - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (p.tile_start[mid] <= t)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

// Σ of the table entries the gb index bytes at `src` select, for the
// group's byte positions starting at pos0 (nibble tables: 16 int16 entries
// per nibble position, low nibble first).
template <int GB>
__device__ __forceinline__ int32_t lookup_group(const uint8_t *__restrict__ src, const int16_t *__restrict__ tab,
                                                int pos0) {
    int32_t sum = 0;
    if constexpr (GB >= 16) {
#pragma unroll 4
        for (int c = 0; c < GB / 16; c++) {
            uint4 w = __ldg(reinterpret_cast<const uint4 *>(src) + c);
            uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
#pragma unroll
                for (int b = 0; b < 4; b++) {
                    uint32_t byte = (ws[k] >> (8 * b)) & 0xffu;
                    int pos = pos0 + c * 16 + k * 4 + b;
                    sum += tab[(2 * pos) * 16 + (byte & 15u)];
                    sum += tab[(2 * pos + 1) * 16 + (byte >> 4)];
                }
            }
        }
    } else if constexpr (GB == 8) {
        uint2 v = __ldg(reinterpret_cast<const uint2 *>(src));
        uint32_t ws[2] = {v.x, v.y};
#pragma unroll
        for (int k = 0; k < 2; k++) {
#pragma unroll
            for (int b = 0; b < 4; b++) {
                uint32_t byte = (ws[k] >> (8 * b)) & 0xffu;
                int pos = pos0 + k * 4 + b;
                sum += tab[(2 * pos) * 16 + (byte & 15u)];
                sum += tab[(2 * pos + 1) * 16 + (byte >> 4)];
            }
        }
    } else {  // GB == 4 or 2
        uint32_t w;
        if constexpr (GB == 4)
            w = __ldg(reinterpret_cast<const uint32_t *>(src));
        else
            w = __ldg(reinterpret_cast<const uint16_t *>(src));
#pragma unroll
        for (int b = 0; b < GB; b++) {
            uint32_t byte = (w >> (8 * b)) & 0xffu;
            int pos = pos0 + b;
            sum += tab[(2 * pos) * 16 + (byte & 15u)];
            sum += tab[(2 * pos + 1) * 16 + (byte >> 4)];
        }
    }
    return sum;
}

template <int GB>
__device__ __forceinline__ int32_t lookup_dispatch(const uint8_t *src, const int16_t *tab, int pos0, int gb) {
    if constexpr (GB > 0) {
        return lookup_group<GB>(src, tab, pos0);
    } else {  // any gb that is a multiple of 16
        int32_t sum = 0;
        for (int c = 0; c < gb / 16; c++) sum += lookup_group<16>(src + 16 * c, tab, pos0 + 16 * c);
        return sum;
    }
}

// A (row, group) item's index bytes, loaded ahead of the table build so the
// load's latency overlaps it.
template <int GB>
struct ItemWords {
    uint32_t w[GB >= 4 ? GB / 4 : 1];
};

template <int GB>
__device__ __forceinline__ void load_item(ItemWords<GB> &W, const uint8_t *__restrict__ src) {
    if constexpr (GB >= 16) {
#pragma unroll
        for (int c = 0; c < GB / 16; c++) {
            const uint4 v = __ldg(reinterpret_cast<const uint4 *>(src) + c);
            W.w[4 * c] = v.x;
            W.w[4 * c + 1] = v.y;
            W.w[4 * c + 2] = v.z;
            W.w[4 * c + 3] = v.w;
        }
    } else if constexpr (GB == 8) {
        const uint2 v = __ldg(reinterpret_cast<const uint2 *>(src));
        W.w[0] = v.x;
        W.w[1] = v.y;
    } else if constexpr (GB == 4) {
        W.w[0] = __ldg(reinterpret_cast<const uint32_t *>(src));
    } else {
        W.w[0] = __ldg(reinterpret_cast<const uint16_t *>(src));
    }
}

// The same sum as lookup_group<GB> on preloaded bytes.
template <int GB>
__device__ __forceinline__ int32_t lookup_item(const ItemWords<GB> &W, const int16_t *__restrict__ tab, int pos0) {
    int32_t sum = 0;
#pragma unroll
    for (int b = 0; b < GB; b++) {
        const uint32_t byte = (W.w[b >> 2] >> (8 * (b & 3))) & 0xffu;
        const int pos = pos0 + b;
        sum += tab[(2 * pos) * 16 + (byte & 15u)];
        sum += tab[(2 * pos + 1) * 16 + (byte >> 4)];
    }
    return sum;
}

template <int GB>
__global__ void __launch_bounds__(kThreads) cq_lut_kernel(const __grid_constant__ LutParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const CqShape &s = p.shape;
    const int tid = threadIdx.x;
    const int pad = s.pad, G = s.group, groups = s.groups, gb = s.gb;
    const int npos = 2 * s.row_bytes;  // nibble positions: one table each

    float *xs = reinterpret_cast<float *>(smem);                              // [pad]
    float *steps = xs + pad;                                                  // [groups]
    float *invs = steps + groups;                                             // [groups]
    float *terms = invs + groups;                                             // [tile rows][groups+1]
    size_t tab_off = (sizeof(float) * ((size_t)pad + 2 * groups + (size_t)kTileRows * (groups + 1)) + 15) & ~(size_t)15;
    int16_t *tab = reinterpret_cast<int16_t *>(smem + tab_off);               // [npos][16]

    const int act = blockIdx.y + p.act0;
    const float *x = p.x + (size_t)act * s.in;

    // This CTA's matrix and row tile, and this thread's first (row, group)
    // item, whose index bytes and norm are loaded now.
    const int TR = p.tile_rows;
    const int k = find_matrix(p, blockIdx.x);
    const CqView v = p.views[k];
    const int r0 = (blockIdx.x - p.tile_start[k]) * TR;
    const int nrows = min(TR, v.out - r0);
    ItemWords<(GB > 0 ? GB : 4)> first;
    __half first_n = __ushort_as_half((unsigned short)0);
    bool have_first = false;
    if constexpr (GB > 0) {
        const int rl = tid % TR, g = tid / TR;
        if (tid < TR * groups && rl < nrows) {
            const size_t lrow = (size_t)g * v.ld + (size_t)(v.row0 + r0 + rl);
            load_item<GB>(first, v.idx + lrow * gb);
            first_n = v.nrm[lrow];
            have_first = true;
        }
    }

    // Rotate: x zero-padded to pad (lut.go:163-165), then fwht per group.
    for (int k = tid; k < pad; k += kThreads) xs[k] = k < s.in ? x[k] : 0.0f;
    __syncthreads();
    const int half = G >> 1;
    for (int h = 1; h < G; h <<= 1) {
        for (int b = tid; b < pad / 2; b += kThreads) {
            int g = b / half, t = b % half;
            int j = g * G + (t / h) * 2 * h + (t % h);
            float a = xs[j], c = xs[j + h];
            xs[j] = __fadd_rn(a, c);
            xs[j + h] = __fsub_rn(a, c);
        }
        __syncthreads();
    }

    // Group bounds M (lut.go:241-245, 264-269), 8191/M and the step.
    const int warp = tid >> 5, lane = tid & 31;
    for (int g = warp; g < groups; g += kThreads / 32) {
        const float *xg = xs + g * G;
        float mx = 0.0f;
        if (s.bits == 2) {
            for (int q = lane; q < half; q += 32) mx = fmaxf(mx, __fadd_rn(fabsf(xg[2 * q]), fabsf(xg[2 * q + 1])));
        } else {
            for (int q = lane; q < G; q += 32) mx = fmaxf(mx, fabsf(xg[q]));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) {
            float m = __fmul_rn(s.cb_max, mx);
            invs[g] = m > 0.0f ? __fdiv_rn((float)kLutQ, m) : 0.0f;
            steps[g] = __fmul_rn(m, s.lut_step);
        }
    }
    __syncthreads();

    // Tables (lut.go:248-255, 272-279): integer v per (nibble position, code).
    for (int e = tid; e < npos * 16; e += kThreads) {
        int pos = e >> 4, c = e & 15;
        float val;
        if (s.bits == 2) {
            int g = (2 * pos) / G;
            float inv = invs[g];
            float a = __fmul_rn(xs[2 * pos], inv), b = __fmul_rn(xs[2 * pos + 1], inv);
            val = __fadd_rn(__fmul_rn(s.cb[c & 3], a), __fmul_rn(s.cb[c >> 2], b));
        } else {
            int g = pos / G;
            float a = __fmul_rn(xs[pos], invs[g]);
            val = __fmul_rn(s.cb[c], a);
        }
        tab[e] = (int16_t)__float2int_rn(val);
    }
    __syncthreads();

    // (row, group) items: exact integer sums, one float term each.
    if constexpr (GB > 0) {
        if (have_first) {
            const int rl = tid % TR, g = tid / TR;
            const int32_t sum = lookup_item<GB>(first, tab, g * gb);
            const float coef = __fmul_rn(__half2float(first_n), steps[g]);
            terms[rl * (groups + 1) + g] = __fmul_rn(__int2float_rn(sum), coef);
        }
    }
    for (int e = tid + (GB > 0 ? kThreads : 0); e < TR * groups; e += kThreads) {
        int rl = e % TR, g = e / TR;
        if (rl >= nrows) continue;
        size_t lrow = (size_t)g * v.ld + (size_t)(v.row0 + r0 + rl);
        int32_t sum = lookup_dispatch<GB>(v.idx + lrow * gb, tab, g * gb, gb);
        float coef = __fmul_rn(__half2float(v.nrm[lrow]), steps[g]);
        terms[rl * (groups + 1) + g] = __fmul_rn(__int2float_rn(sum), coef);
    }
    __syncthreads();

    // y[r] = Σ_g term, in group order from +0 (lut.go:295, 309).
    float *y = p.y[k] + (size_t)act * v.out;
    for (int rl = tid; rl < nrows; rl += kThreads) {
        const float *t = terms + rl * (groups + 1);
        float acc = 0.0f;
        for (int g = 0; g < groups; g++) acc = __fadd_rn(acc, t[g]);
        y[r0 + rl] = acc;
    }
}

}  // namespace

size_t lut_smem_bytes(const CqShape &s) {
    size_t b = sizeof(float) * ((size_t)s.pad + 2 * s.groups + (size_t)kTileRows * (s.groups + 1));
    b = (b + 15) & ~(size_t)15;
    b += sizeof(int16_t) * (size_t)2 * s.row_bytes * 16;
    return b;
}

cudaError_t launch_lut(const LutParams &p, int tiles, int acts, cudaStream_t st) {
    size_t smem = lut_smem_bytes(p.shape);
    void (*fn)(LutParams);
    switch (p.shape.gb) {
        case 2: fn = cq_lut_kernel<2>; break;
        case 4: fn = cq_lut_kernel<4>; break;
        case 8: fn = cq_lut_kernel<8>; break;
        case 16: fn = cq_lut_kernel<16>; break;
        case 32: fn = cq_lut_kernel<32>; break;
        case 64: fn = cq_lut_kernel<64>; break;
        default: fn = cq_lut_kernel<0>; break;
    }
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid(tiles, acts);
    fn<<<grid, kThreads, smem, st>>>(p);
    count_launch();
    return cudaGetLastError();
}

}  // namespace wb
