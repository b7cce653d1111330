// cq_lut_acts.cu — the CQ lut GEMM for many activations against small
// matrices (multi-stream decode: 128–1024 streams × q/k/v/gate, φ,
// out_proj): internal/cq/lut.go's kernel, bit for bit, with each
// activation's tables built once for every row of every matrix of the
// launch.
//
// One CTA per (activation, share of the rows). The CTA rotates the
// activation (kernel.go:384 fwht per group, stage by stage), takes the
// group bounds, 8191/M and steps (lut.go:213-287) and builds the integer
// nibble tables in shared memory, as cq_lut.cu does; then each warp takes
// whole weight rows. A row is read in chunks of 32·B bytes (B = 4 bytes a
// lane for 2-bit, 8 for 4-bit rows of group 128): eight lanes cover one
// group of the chunk, each sums its bytes' two nibble entries exactly, the
// eight sums meet by shuffles (exact integers), and the group's float term
// float32(Σv)·(norm·step) joins the row's sum in group order (lut.go:309).
//
// Tables are nibble-major, T[nib][q] (q the nibble position), so a lookup's
// bank is its byte position mod 32. Each lane visits its B bytes in an
// order rotated by its lane group, which puts the 32 lanes of a warp on 32
// distinct byte positions mod 32 at every step: no bank conflicts.
#include "common.cuh"
#include "cq_kernels.cuh"

namespace wb {

namespace {

constexpr int kActsThreads = 512;

template <int B>  // bytes a lane takes per chunk: 4 (gb 32) or 8 (gb 64)
__global__ void __launch_bounds__(kActsThreads) cq_lut_acts_kernel(const __grid_constant__ ActsParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const CqShape &s = p.shape;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int pad = s.pad, G = s.group, groups = s.groups;
    const int NQ = 2 * s.row_bytes;  // nibble positions
    float *xs = reinterpret_cast<float *>(smem);  // [pad]
    float *steps = xs + pad;                      // [groups]
    float *invs = steps + groups;                 // [groups]
    int16_t *tab = reinterpret_cast<int16_t *>(smem + ((sizeof(float) * ((size_t)pad + 2 * groups) + 15) & ~15));

    const int act = blockIdx.x;
    const float *x = p.x + (size_t)act * s.in;
    for (int k = tid; k < pad; k += kActsThreads) xs[k] = k < s.in ? x[k] : 0.0f;
    __syncthreads();
    // Group sizes and table widths are powers of two: shifts, not divisions.
    const int lg2 = 31 - __clz(G);      // log2 G
    const int lq = 31 - __clz(2 * s.row_bytes);  // log2 NQ (row_bytes a power of two here)
    const int half = G >> 1;
    for (int st = 0; (1 << st) < G; st++) {
        const int h = 1 << st;
        for (int b = tid; b < pad / 2; b += kActsThreads) {
            const int g = b >> (lg2 - 1), t = b & (half - 1);
            const int j = (g << lg2) + ((t >> st) << (st + 1)) + (t & (h - 1));
            const float a = xs[j], c = xs[j + h];
            xs[j] = __fadd_rn(a, c);
            xs[j + h] = __fsub_rn(a, c);
        }
        __syncthreads();
    }
    for (int g = warp; g < groups; g += kActsThreads / 32) {
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
    __syncthreads();
    for (int e = tid; e < NQ * 16; e += kActsThreads) {
        const int nib = e >> lq, q = e & (NQ - 1);
        float val;
        if (s.bits == 2) {
            const float inv = invs[(2 * q) >> lg2];
            const float a = __fmul_rn(xs[2 * q], inv), b = __fmul_rn(xs[2 * q + 1], inv);
            val = __fadd_rn(__fmul_rn(s.cb[nib & 3], a), __fmul_rn(s.cb[nib >> 2], b));
        } else {
            val = __fmul_rn(s.cb[nib], __fmul_rn(xs[q], invs[q >> lg2]));
        }
        tab[e] = (int16_t)__float2int_rn(val);
    }
    __syncthreads();

    // Rows: this CTA's share of all matrices' rows, a warp per row.
    const int per = (p.total_rows + p.splits - 1) / p.splits;
    const int R0 = blockIdx.y * per, R1 = min(p.total_rows, R0 + per);
    constexpr int kChunk = 32 * B;           // bytes of a row per chunk
    const int gpc = kChunk / s.gb;           // groups per chunk (4)
    const int lg = lane / (32 / gpc);        // this lane's group in the chunk
    const int lo = (lane % (32 / gpc)) * B;  // its first byte in the group
    const int rot = (lane / (32 / B)) % B;   // rotation of its byte order
    const int nchunks = s.row_bytes / kChunk;
    int k = 0;
    for (int R = R0 + warp; R < R1; R += kActsThreads / 32) {
        while (k + 1 < p.n && p.row_start[k + 1] <= R) k++;
        const CqView &v = p.views[k];
        const int r = R - p.row_start[k];
        float acc = 0.0f;
        for (int c = 0; c < nchunks; c++) {
            const int g = c * gpc + lg;
            const size_t lrow = (size_t)g * v.ld + (size_t)(v.row0 + r);
            const int j0 = g * s.gb + lo;  // the byte position of this lane's first byte
            int32_t sum = 0;
            if constexpr (B == 4) {
                uint32_t w = __ldg(reinterpret_cast<const uint32_t *>(v.idx + lrow * s.gb + lo));
                w = __funnelshift_r(w, w, 8 * rot);
#pragma unroll
                for (int b = 0; b < 4; b++) {
                    const uint32_t byte = (w >> (8 * b)) & 0xffu;
                    const int j = j0 + ((b + rot) & 3);
                    sum += tab[(int)(byte & 15u) * NQ + 2 * j];
                    sum += tab[(int)(byte >> 4) * NQ + 2 * j + 1];
                }
            } else {
                const uint2 u = __ldg(reinterpret_cast<const uint2 *>(v.idx + lrow * s.gb + lo));
                unsigned long long w = ((unsigned long long)u.y << 32) | u.x;
                if (rot) w = (w >> (8 * rot)) | (w << (64 - 8 * rot));
#pragma unroll
                for (int b = 0; b < 8; b++) {
                    const uint32_t byte = (uint32_t)(w >> (8 * b)) & 0xffu;
                    const int j = j0 + ((b + rot) & 7);
                    sum += tab[(int)(byte & 15u) * NQ + 2 * j];
                    sum += tab[(int)(byte >> 4) * NQ + 2 * j + 1];
                }
            }
            // The group's exact sum over its lanes.
#pragma unroll
            for (int o = (32 / gpc) / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            const float coef = __fmul_rn(__half2float(v.nrm[lrow]), steps[g]);
            const float term = __fmul_rn(__int2float_rn(sum), coef);
            for (int q = 0; q < gpc; q++) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, term, q * (32 / gpc)));
        }
        if (lane == 0) p.y[k][(size_t)act * v.out + r] = acc;
    }
}

}  // namespace

bool acts_eligible(const CqShape &s) {
    if (!(s.bits == 2 && s.gb == 32) && !(s.bits == 4 && s.gb == 64)) return false;  // group 128
    const int chunk = 32 * (s.gb / 8);
    return s.row_bytes % chunk == 0 && (s.row_bytes & (s.row_bytes - 1)) == 0 && s.pad == s.row_bytes * 8 / s.bits &&
           acts_smem_bytes(s) <= 200 * 1024;
}

size_t acts_smem_bytes(const CqShape &s) {
    const size_t head = (sizeof(float) * ((size_t)s.pad + 2 * s.groups) + 15) & ~(size_t)15;
    return head + sizeof(int16_t) * (size_t)2 * s.row_bytes * 16;
}

cudaError_t launch_lut_acts(const ActsParams &p, int acts, cudaStream_t st) {
    if (acts <= 0 || p.total_rows <= 0) return cudaSuccess;
    const size_t smem = acts_smem_bytes(p.shape);
    void (*fn)(ActsParams) = p.shape.gb == 32 ? cq_lut_acts_kernel<4> : cq_lut_acts_kernel<8>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    fn<<<dim3((unsigned)acts, (unsigned)p.splits), kActsThreads, smem, st>>>(p);
    count_launch();
    return cudaGetLastError();
}

}  // namespace wb
