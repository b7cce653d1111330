// decode_head.cu — the decoder head's scale and the greedy choice on the
// device: logits = y·head (internal/decoder/decoder.go:508-523, when
// head != 1) and, per row, the first index of the largest logit
// (internal/decoder/greedy.go:182 argmax), so a greedy decode step hands
// the host one int32 per stream instead of a row of vocabulary logits.
//
// One CTA per row. Each thread scans a strided slice, keeping the best
// (value, index) as one 64-bit key: the value's order-preserving bits
// (+0 and -0 made equal, as `x > v[best]` treats them) in the high word and
// the complement of the index in the low word, so the largest key is the
// largest value at its first index. NaN keys are 0 and never win; a NaN at
// index 0 keeps 0, as the reference's loop does (every comparison with it
// is false).
#include <cstdint>

#include "common.cuh"

namespace wb {

namespace {

constexpr int kHeadThreads = 256;

__device__ __forceinline__ unsigned long long head_key(float v, int i) {
    if (v != v) return 0ull;
    const uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
    const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)ord << 32) | (uint32_t)(0xffffffffu - (uint32_t)i);
}

// logits may be y itself (the reference scales in place): every element is
// read and written by one thread, and v[0] is read before it is written.
__global__ void __launch_bounds__(kHeadThreads) head_argmax_kernel(const float *y, int vocab, float head,
                                                                   float *logits, int32_t *__restrict__ idx) {
    __shared__ unsigned long long best_w[kHeadThreads / 32];
    const int r = blockIdx.x, tid = threadIdx.x;
    const float *v = y + (size_t)r * vocab;
    float *o = logits ? logits + (size_t)r * vocab : nullptr;
    const bool scale = head != 1.0f;
    float x0 = 0.0f;
    if (tid == 0) x0 = scale ? __fmul_rn(v[0], head) : v[0];
    unsigned long long best = 0ull;
    auto take = [&](float x, int i) {
        if (scale) x = __fmul_rn(x, head);
        if (o) o[i] = x;
        const unsigned long long k = head_key(x, i);
        best = k > best ? k : best;
    };
    int done = 0;
    if ((vocab & 3) == 0 && (((uintptr_t)v | (uintptr_t)o) & 15) == 0) {
        // Rows of whole, aligned float4s: four loads in flight per thread.
        const float4 *v4 = reinterpret_cast<const float4 *>(v);
        const int n4 = vocab / 4;
        int i = tid;
        for (; i + 3 * kHeadThreads < n4; i += 4 * kHeadThreads) {
            float4 a[4];
#pragma unroll
            for (int u = 0; u < 4; u++) a[u] = v4[i + u * kHeadThreads];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int e = 4 * (i + u * kHeadThreads);
                take(a[u].x, e);
                take(a[u].y, e + 1);
                take(a[u].z, e + 2);
                take(a[u].w, e + 3);
            }
        }
        for (; i < n4; i += kHeadThreads) {
            const float4 a = v4[i];
            take(a.x, 4 * i);
            take(a.y, 4 * i + 1);
            take(a.z, 4 * i + 2);
            take(a.w, 4 * i + 3);
        }
        done = vocab;
    }
    for (int i = done + tid; i < vocab; i += kHeadThreads) take(v[i], i);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, s);
        best = k > best ? k : best;
    }
    if ((tid & 31) == 0) best_w[tid >> 5] = best;
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < kHeadThreads / 32; w++) best = best_w[w] > best ? best_w[w] : best;
        // NaN at 0, or every value NaN: 0 (greedy.go:182's best = 0 never moves).
        idx[r] = (x0 != x0 || best == 0ull) ? 0 : (int32_t)(0xffffffffu - (uint32_t)best);
    }
}

}  // namespace

cudaError_t launch_head_argmax(const float *y, int rows, int vocab, float head, float *logits, int32_t *idx,
                               cudaStream_t st) {
    for (int r0 = 0; r0 < rows; r0 += 65535) {
        const int n = rows - r0 < 65535 ? rows - r0 : 65535;
        head_argmax_kernel<<<n, kHeadThreads, 0, st>>>(y + (size_t)r0 * vocab, vocab, head,
                                                       logits ? logits + (size_t)r0 * vocab : nullptr, idx + r0);
        count_launch();
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace wb
