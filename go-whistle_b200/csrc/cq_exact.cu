// cq_exact.cu — the CQ Exact path (internal/cq/kernel.go:162-373) and Row
// (internal/cq/matrix.go:161) on sm_100a.
//
// Exact products sum the codebook levels in float32 (no integer tables), in
// the reference's exact operation order, so an Exact view here gives the
// same bits as the reference's purego build:
//   - rotate (kernel.go:392): fwht per group, then ×invSqrt(G);
//   - nibble tables (kernel.go:431): cb[c]·x̂ (4-bit) or cb[lo]·a + cb[hi]·b
//     (2-bit), each product and the add rounded separately;
//   - activations in whole blocks of four take nibble4's sums
//     (kernel.go:519: lo and hi entries each summed byte after byte, then
//     (a + b)·n), the leftover ones nibble's eight accumulators
//     (kernel.go:460), as gemm splits them (kernel.go:303-313).
// One thread owns one row of one activation and walks its groups in order;
// the 16-entry float tables of the activation sit in shared memory.
#include "common.cuh"
#include "cq_kernels.cuh"

namespace wb {

namespace {

constexpr int kExactThreads = 256;

__device__ __forceinline__ void rotate_scaled(float *xs, const float *x, const CqShape &s, int tid, int nthreads) {
    const int pad = s.pad, G = s.group;
    for (int k = tid; k < pad; k += nthreads) xs[k] = k < s.in ? x[k] : 0.0f;
    __syncthreads();
    const int half = G >> 1;
    for (int h = 1; h < G; h <<= 1) {
        for (int b = tid; b < pad / 2; b += nthreads) {
            int g = b / half, t = b % half;
            int j = g * G + (t / h) * 2 * h + (t % h);
            float a = xs[j], c = xs[j + h];
            xs[j] = __fadd_rn(a, c);
            xs[j + h] = __fsub_rn(a, c);
        }
        __syncthreads();
    }
    for (int k = tid; k < pad; k += nthreads) xs[k] = __fmul_rn(xs[k], s.inv_sqrt);
    __syncthreads();
}

__global__ void __launch_bounds__(kExactThreads)
    cq_exact_kernel(const __grid_constant__ CqShape s, const CqView v, const float *__restrict__ x,
                    float *__restrict__ y, int rows, int four, int act0) {
    extern __shared__ __align__(16) unsigned char smem[];
    float *xs = reinterpret_cast<float *>(smem);  // [pad]
    float *nib = xs + s.pad;                      // [2*row_bytes][16]
    const int tid = threadIdx.x;
    const int act = blockIdx.y + act0;
    const int npos = 2 * s.row_bytes;

    rotate_scaled(xs, x + (size_t)act * s.in, s, tid, kExactThreads);

    for (int e = tid; e < npos * 16; e += kExactThreads) {
        int q = e >> 4, c = e & 15;
        float val;
        if (s.bits == 4) {
            val = __fmul_rn(s.cb[c], xs[q]);
        } else {
            float a = xs[2 * q], b = xs[2 * q + 1];
            float hb = __fmul_rn(s.cb[c >> 2], b);
            val = __fadd_rn(__fmul_rn(s.cb[c & 3], a), hb);
        }
        nib[e] = val;
    }
    __syncthreads();

    const int r = blockIdx.x * kExactThreads + tid;
    if (r >= v.out) return;
    const int gb = s.gb;
    const bool by4 = act < four;
    float acc = 0.0f;
    for (int g = 0; g < s.groups; g++) {
        size_t lrow = (size_t)g * v.ld + (size_t)(v.row0 + r);
        const uint8_t *rg = v.idx + lrow * gb;
        const float *tg = nib + (size_t)2 * g * gb * 16;
        float n = __half2float(v.nrm[lrow]);
        float sum;
        if (by4) {
            float a = 0.0f, b = 0.0f;
            for (int j = 0; j < gb; j++) {
                uint32_t byte = rg[j];
                a = __fadd_rn(a, tg[(2 * j) * 16 + (byte & 15u)]);
                b = __fadd_rn(b, tg[(2 * j + 1) * 16 + (byte >> 4)]);
            }
            sum = __fadd_rn(a, b);
        } else {
            float ak[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            int j = 0;
            for (; j + 8 <= gb; j += 8) {
#pragma unroll
                for (int m = 0; m < 4; m++) {
#pragma unroll
                    for (int hh = 0; hh < 2; hh++) {
                        uint32_t b0 = rg[j + m], b1 = rg[j + 4 + m];
                        uint32_t c0 = hh ? b0 >> 4 : b0 & 15u, c1 = hh ? b1 >> 4 : b1 & 15u;
                        float t0 = tg[(2 * (j + m) + hh) * 16 + c0];
                        float t1 = tg[(2 * (j + 4 + m) + hh) * 16 + c1];
                        ak[2 * m + hh] = __fadd_rn(ak[2 * m + hh], __fadd_rn(t0, t1));
                    }
                }
            }
            for (; j < gb; j++) {
                uint32_t byte = rg[j];
                float t = __fadd_rn(tg[(2 * j) * 16 + (byte & 15u)], tg[(2 * j + 1) * 16 + (byte >> 4)]);
                ak[0] = __fadd_rn(ak[0], t);
            }
            sum = __fadd_rn(__fadd_rn(__fadd_rn(ak[0], ak[1]), __fadd_rn(ak[2], ak[3])),
                            __fadd_rn(__fadd_rn(ak[4], ak[5]), __fadd_rn(ak[6], ak[7])));
        }
        acc = __fadd_rn(acc, __fmul_rn(sum, n));
    }
    y[(size_t)act * v.out + r] = acc;
}

// matrix.go:161 Row: per group, cb[idx]·(norm·invSqrt(G)), fwht, cut at In.
__global__ void cq_row_kernel(const __grid_constant__ CqShape s, const CqView v, const int32_t *__restrict__ rows,
                              int r0, float *__restrict__ dst, int32_t *bad) {
    extern __shared__ __align__(16) unsigned char smem[];
    float *buf = reinterpret_cast<float *>(smem);  // [group]
    const int tid = threadIdx.x, nt = blockDim.x;
    const int G = s.group;
    int r = rows ? rows[blockIdx.x] : r0;
    float *out = dst + (size_t)blockIdx.x * s.in;
    if (r < 0 || r >= v.out) {
        for (int k = tid; k < s.in; k += nt) out[k] = 0.0f;
        if (tid == 0 && bad) *bad = 1;
        return;
    }
    for (int g = 0; g < s.groups; g++) {
        size_t lrow = (size_t)g * v.ld + (size_t)(v.row0 + r);
        const uint8_t *rg = v.idx + lrow * s.gb;
        float sc = __fmul_rn(__half2float(v.nrm[lrow]), s.inv_sqrt);
        for (int k = tid; k < G; k += nt) {
            int bit = k * s.bits;
            uint32_t code = (rg[bit >> 3] >> (bit & 7)) & ((1u << s.bits) - 1u);
            buf[k] = __fmul_rn(s.cb[code], sc);
        }
        __syncthreads();
        for (int h = 1; h < G; h <<= 1) {
            for (int b = tid; b < G / 2; b += nt) {
                int j = (b / h) * 2 * h + (b % h);
                float a = buf[j], c = buf[j + h];
                buf[j] = __fadd_rn(a, c);
                buf[j + h] = __fsub_rn(a, c);
            }
            __syncthreads();
        }
        int col = g * G;
        for (int k = tid; k < G && col + k < s.in; k += nt) out[col + k] = buf[k];
        __syncthreads();
    }
}

}  // namespace

size_t exact_smem_bytes(const CqShape &s) {
    return sizeof(float) * ((size_t)s.pad + (size_t)2 * s.row_bytes * 16);
}

cudaError_t launch_exact(const CqShape &s, const CqView &v, const float *x, float *y, int rows, cudaStream_t st) {
    size_t smem = exact_smem_bytes(s);
    cudaError_t e = cudaFuncSetAttribute(cq_exact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int four = rows - rows % 4;
    int tiles = (v.out + kExactThreads - 1) / kExactThreads;
    for (int a0 = 0; a0 < rows; a0 += 65535) {
        int n = rows - a0 < 65535 ? rows - a0 : 65535;
        cq_exact_kernel<<<dim3(tiles, n), kExactThreads, smem, st>>>(s, v, x, y, rows, four, a0);
        count_launch();
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_row(const CqShape &s, const CqView &v, const int32_t *rows, int r0, int n, float *dst,
                       int32_t *bad, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    int threads = s.group < 128 ? (s.group < 32 ? 32 : s.group) : 128;
    cq_row_kernel<<<n, threads, sizeof(float) * s.group, st>>>(s, v, rows, r0, dst, bad);
    count_launch();
    return cudaGetLastError();
}

}  // namespace wb
