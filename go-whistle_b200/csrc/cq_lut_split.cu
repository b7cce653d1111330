// cq_lut_split.cu — the CQ LUT product for one activation at low latency:
// the groups of a row are split over the CTAs of a thread-block cluster.
//
// Same arithmetic as cq_lut.cu and the reference's lut kernel
// (internal/cq/lut.go), bit for bit. The per-tile kernel makes every CTA
// rotate and tabulate the whole activation before its first lookup; for a
// single small product (a decode step's projections, the vocabulary head)
// that set-up is most of the time. Here a cluster of CS CTAs owns a tile of
// 32 rows, and CTA c of the cluster handles only groups
// [c·gpc, (c+1)·gpc): it rotates and tabulates just those groups (each
// group's bound, 8191/M and step depend on that group alone, lut.go:160-178),
// loads its (row, group) items' index bytes before the table build so the
// loads overlap it, and writes each item's float term into shared memory of
// the cluster's first CTA (distributed shared memory). After a cluster
// barrier that CTA adds each row's terms in group order (lut.go:309) and
// writes y. Grid: (tiles · CS, activations), cluster (CS, 1, 1), CS <= 8.
#include <cooperative_groups.h>

#include "common.cuh"
#include "cq_kernels.cuh"

namespace cg = cooperative_groups;

namespace wb {

namespace {

constexpr int kSplitThreads = 128;
constexpr int kSplitRows = 32;

__device__ __forceinline__ int split_matrix(const LutParams &p, int t) {
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

template <int GB>
struct SplitWords {
    uint32_t w[GB >= 4 ? GB / 4 : 1];
};

template <int GB>
__device__ __forceinline__ void split_load(SplitWords<GB> &W, const uint8_t *__restrict__ src) {
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

// Σ of the nibble-table entries the group's index bytes select; tab holds
// 16 int16 entries per local nibble position, the low nibble first.
template <int GB>
__device__ __forceinline__ int32_t split_sum(const SplitWords<GB> &W, const int16_t *__restrict__ tab, int lpos0) {
    int32_t sum = 0;
#pragma unroll
    for (int b = 0; b < GB; b++) {
        const uint32_t byte = (W.w[b >> 2] >> (8 * (b & 3))) & 0xffu;
        const int pos = lpos0 + b;
        sum += tab[(2 * pos) * 16 + (byte & 15u)];
        sum += tab[(2 * pos + 1) * 16 + (byte >> 4)];
    }
    return sum;
}

// Items (row, local group) per thread, loaded ahead.
constexpr int kSplitItems = 4;

template <int GB>
__global__ void __launch_bounds__(kSplitThreads) cq_lut_split_kernel(const __grid_constant__ LutParams p, int cs,
                                                                    int gpc) {
    extern __shared__ __align__(16) unsigned char smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const CqShape &s = p.shape;
    const int tid = threadIdx.x;
    const int G = s.group, groups = s.groups;
    const int rank = (int)cluster.block_rank();
    const int g0 = rank * gpc, gn = max(0, min(gpc, groups - g0));
    const int tile = blockIdx.x / cs;
    const int act = blockIdx.y + p.act0;

    // Shared memory: terms [kSplitRows][groups + 1] (read in the first CTA
    // only), this CTA's columns xs [gpc·G], bounds invs/steps [gpc], and
    // its nibble tables [2·gpc·GB][16].
    float *terms = reinterpret_cast<float *>(smem);
    float *xs = terms + kSplitRows * (groups + 1);
    float *invs = xs + gpc * G;
    float *steps = invs + gpc;
    int16_t *tab = reinterpret_cast<int16_t *>(steps + gpc + 4);

    // The tile's matrix and rows; this thread's items, loaded now.
    const int k = split_matrix(p, tile);
    const CqView v = p.views[k];
    const int r0 = (tile - p.tile_start[k]) * kSplitRows;
    const int nrows = min(kSplitRows, v.out - r0);
    const int nitems = kSplitRows * gn;
    SplitWords<GB> words[kSplitItems];
    __half nrm[kSplitItems];
#pragma unroll
    for (int i = 0; i < kSplitItems; i++) {
        const int e = tid + i * kSplitThreads;
        const int rl = e % kSplitRows, gl = e / kSplitRows;
        nrm[i] = __ushort_as_half((unsigned short)0);
        if (e < nitems && rl < nrows) {
            const size_t lrow = (size_t)(g0 + gl) * v.ld + (size_t)(v.row0 + r0 + rl);
            split_load<GB>(words[i], v.idx + lrow * GB);
            nrm[i] = v.nrm[lrow];
        }
    }

    // This CTA's columns of the activation, zero past In (lut.go:163-165),
    // and the FWHT of each of its groups (kernel.go:384), stage by stage.
    const float *x = p.x + (size_t)act * s.in;
    if (G <= 32) {
        // Groups within a warp: butterflies (same stages, same operand
        // order) and bounds by shuffles, no block barrier between stages.
        const int lane = tid & 31, ncol = gn * G;
        for (int c = tid >> 5; c * 32 < ncol; c += kSplitThreads / 32) {
            const int lc = c * 32 + lane, col = g0 * G + lc;
            float v = lc < ncol && col < s.in ? x[col] : 0.0f;
            for (int h = 1; h < G; h <<= 1) {
                const float o = __shfl_xor_sync(0xffffffffu, v, h);
                v = (lane & h) ? __fsub_rn(o, v) : __fadd_rn(v, o);
            }
            if (lc < ncol) xs[lc] = v;
            const float a = fabsf(v);
            float mv;
            if (s.bits == 2) {  // |x[2q]| + |x[2q+1]|, the even element first
                const float pa = __shfl_xor_sync(0xffffffffu, a, 1);
                mv = (lane & 1) ? __fadd_rn(pa, a) : __fadd_rn(a, pa);
            } else {
                mv = a;
            }
            mv = fmaxf(0.0f, mv);
            for (int o = 1; o < G; o <<= 1) mv = fmaxf(mv, __shfl_xor_sync(0xffffffffu, mv, o));
            if ((lane & (G - 1)) == 0 && lc < ncol) {
                const int g = lc / G;
                const float m = __fmul_rn(s.cb_max, mv);
                invs[g] = m > 0.0f ? __fdiv_rn((float)kLutQ, m) : 0.0f;
                steps[g] = __fmul_rn(m, s.lut_step);
            }
        }
    } else {
        for (int c = tid; c < gn * G; c += kSplitThreads) {
            const int col = g0 * G + c;
            xs[c] = col < s.in ? x[col] : 0.0f;
        }
        __syncthreads();
        const int half = G >> 1;
        for (int h = 1; h < G; h <<= 1) {
            for (int b = tid; b < gn * half; b += kSplitThreads) {
                const int g = b / half, t = b % half;
                const int j = g * G + (t / h) * 2 * h + (t % h);
                const float a = xs[j], c = xs[j + h];
                xs[j] = __fadd_rn(a, c);
                xs[j + h] = __fsub_rn(a, c);
            }
            __syncthreads();
        }
        // Bounds M (lut.go:241-245, 264-269), 8191/M and the step per group.
        const int warp = tid >> 5, lane = tid & 31;
        for (int g = warp; g < gn; g += kSplitThreads / 32) {
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
                const float m = __fmul_rn(s.cb_max, mx);
                invs[g] = m > 0.0f ? __fdiv_rn((float)kLutQ, m) : 0.0f;
                steps[g] = __fmul_rn(m, s.lut_step);
            }
        }
    }
    __syncthreads();
    // Nibble tables (lut.go:248-255, 272-279) for the local positions.
    const int lnpos = 2 * gn * GB;
    for (int e = tid; e < lnpos * 16; e += kSplitThreads) {
        const int pos = e >> 4, c = e & 15;
        float val;
        if (s.bits == 2) {
            const int g = (2 * pos) / G;
            const float inv = invs[g];
            const float a = __fmul_rn(xs[2 * pos], inv), b = __fmul_rn(xs[2 * pos + 1], inv);
            val = __fadd_rn(__fmul_rn(s.cb[c & 3], a), __fmul_rn(s.cb[c >> 2], b));
        } else {
            const int g = pos / G;
            val = __fmul_rn(s.cb[c], __fmul_rn(xs[pos], invs[g]));
        }
        tab[e] = (int16_t)__float2int_rn(val);
    }
    __syncthreads();

    // Every CTA of the cluster has started: its shared memory may be written.
    cluster.sync();
    float *terms0 = cluster.map_shared_rank(terms, 0);
#pragma unroll
    for (int i = 0; i < kSplitItems; i++) {
        const int e = tid + i * kSplitThreads;
        const int rl = e % kSplitRows, gl = e / kSplitRows;
        if (e < nitems && rl < nrows) {
            const int32_t sum = split_sum<GB>(words[i], tab, gl * GB);
            const float coef = __fmul_rn(__half2float(nrm[i]), steps[gl]);
            terms0[rl * (groups + 1) + g0 + gl] = __fmul_rn(__int2float_rn(sum), coef);
        }
    }
    // Items beyond kSplitItems per thread (large gpc): loaded here.
    for (int e = tid + kSplitItems * kSplitThreads; e < nitems; e += kSplitThreads) {
        const int rl = e % kSplitRows, gl = e / kSplitRows;
        if (rl >= nrows) continue;
        const size_t lrow = (size_t)(g0 + gl) * v.ld + (size_t)(v.row0 + r0 + rl);
        SplitWords<GB> w;
        split_load<GB>(w, v.idx + lrow * GB);
        const int32_t sum = split_sum<GB>(w, tab, gl * GB);
        const float coef = __fmul_rn(__half2float(v.nrm[lrow]), steps[gl]);
        terms0[rl * (groups + 1) + g0 + gl] = __fmul_rn(__int2float_rn(sum), coef);
    }
    cluster.sync();

    // y[r] = Σ_g term in group order from +0 (lut.go:295, 309).
    if (rank == 0) {
        float *y = p.y[k] + (size_t)act * v.out;
        for (int rl = tid; rl < nrows; rl += kSplitThreads) {
            const float *t = terms + rl * (groups + 1);
            float acc = 0.0f;
            for (int g = 0; g < groups; g++) acc = __fadd_rn(acc, t[g]);
            y[r0 + rl] = acc;
        }
    }
}

}  // namespace

int split_cluster_size(const CqShape &s) { return s.groups < 8 ? s.groups : 8; }

size_t split_smem_bytes(const CqShape &s) {
    const int cs = split_cluster_size(s), gpc = (s.groups + cs - 1) / cs;
    size_t b = sizeof(float) * ((size_t)kSplitRows * (s.groups + 1) + (size_t)gpc * s.group + 2 * gpc + 4);
    b = (b + 15) & ~(size_t)15;
    return b + sizeof(int16_t) * 2 * (size_t)gpc * s.gb * 16;
}

bool split_eligible(const CqShape &s) {
    return s.gb == 2 || s.gb == 4 || s.gb == 8 || s.gb == 16 || s.gb == 32 || s.gb == 64;
}

int split_tiles(int out) { return (out + kSplitRows - 1) / kSplitRows; }

cudaError_t launch_split(const LutParams &p, int tiles, int acts, cudaStream_t st) {
    const int cs = split_cluster_size(p.shape), gpc = (p.shape.groups + cs - 1) / cs;
    const size_t smem = split_smem_bytes(p.shape);
    void (*fn)(LutParams, int, int);
    switch (p.shape.gb) {
        case 2: fn = cq_lut_split_kernel<2>; break;
        case 4: fn = cq_lut_split_kernel<4>; break;
        case 8: fn = cq_lut_split_kernel<8>; break;
        case 16: fn = cq_lut_split_kernel<16>; break;
        case 32: fn = cq_lut_split_kernel<32>; break;
        default: fn = cq_lut_split_kernel<64>; break;
    }
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)(tiles * cs), (unsigned)acts);
    cfg.blockDim = dim3(kSplitThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, fn, p, cs, gpc);
    count_launch();
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace wb
