// cq_gemm_tc.cu — the batched CQ GEMM on the 5th-generation tensor cores
// (tcgen05, TMEM accumulators), for encoder prefill and many-row decode.
//
// The product is taken in the rotated domain, where a CQ matrix needs no
// Hadamard transform (internal/cq/matrix.go:1-13):
//   y[m, r] = Σ_k x̂[m, k] · ŵ[r, k],   x̂_g = H·x_g,   ŵ[r, k] = cb[idx[r,k]]·n[r,g]/√G
// Both operands go to fp16 (x̂ per activation by `rotate_f16_kernel`, ŵ once
// per matrix by `dequant_f16_kernel`), each scaled by an exact power of two
// — per activation row for x̂, per matrix for ŵ — so that its largest value
// sits just under 2^15 (no overflow, fp16's full 11-bit precision at any
// input range); the tensor cores accumulate in fp32 and the epilogue
// multiplies the scales back out, exactly. This is not the reference's lut
// arithmetic, so it is not bit-exact: every element is within the fp16
// bound stated in include/whistle_b200.h (WC_GEMM_TENSOR_CORES) of the
// float64 product. It is only used when asked for (wc_cq_gemm_ex with
// WC_GEMM_TENSOR_CORES, or WC_GEMM_AUTO past the lut kernels' crossover).
//
// Operand images in global memory are pre-swizzled 128 x 64 fp16 tiles
// (K-major, 128-byte swizzle: 16-byte chunk c of row r at chunk c ^ (r & 7)),
// so a stage of the main loop is two 1-D bulk copies (cp.async.bulk, no
// tensor map, no multicast). One CTA computes a 128 x 128 tile of y:
//   warp 0 lane 0   producer: bulk copies of the A and B chunks per stage
//   warp 1          TMEM allocation; lane 0 issues the MMAs (K = 16 each)
//   warps 2-5       epilogue: TMEM -> registers -> y (fp32)
// Every wait on an mbarrier is bounded; on timeout the CTA records an error
// code, skips its remaining work, frees its TMEM and returns.
#include <cuda_fp16.h>

#include <mutex>

#include "common.cuh"
#include "cq_kernels.cuh"

namespace wb {

namespace {

constexpr int kTcM = 128;         // UMMA M (cta_group::1)
constexpr int kTcN = 128;         // UMMA N, TMEM columns
constexpr int kTcK = 64;          // fp16 elements per 128-byte row of a chunk
constexpr int kChunkBytes = kTcM * 128;  // one 128 x 64 fp16 tile, A and B alike
constexpr int kTcThreads = 192;
constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// Bounded wait for the phase with the given parity; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t limit = kSpinLimit) {
    const uint32_t a = smem_u32(bar);
    for (uint32_t it = 0; it < limit; it++) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms
// 1024 bytes apart (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: D f32, A and B f16 (formats 0), both K-major,
// N = kTcN, M = kTcM.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kTcN >> 3) << 17) |
                            ((uint32_t)(kTcM >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(dtmem),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Byte offset of element (row, k) of a 128 x 64 fp16 swizzled chunk.
__device__ __forceinline__ uint32_t swz(int row, int k) {
    return (uint32_t)row * 128u + ((uint32_t)(((k >> 3) ^ (row & 7)) & 7) << 4) + (uint32_t)(k & 7) * 2u;
}

// kStages ring stages: 2 with three CTAs per SM; a launch of few tiles (one
// or two per SM) takes a deeper ring, more of its loads in flight at once.
template <int kStages>
__global__ void __launch_bounds__(kTcThreads, kStages <= 2 ? 3 : kStages <= 3 ? 2 : 1)
    cq_gemm_tc_kernel(const __grid_constant__ TcParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte alignment for the swizzle atoms.
    unsigned char *smem = reinterpret_cast<unsigned char *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    unsigned char *sa = smem;                                  // [kStages][kChunkBytes]
    unsigned char *sb = smem + kStages * kChunkBytes;          // [kStages][kChunkBytes]
    uint64_t *full = reinterpret_cast<uint64_t *>(sb + kStages * kChunkBytes);
    uint64_t *empty = full + kStages;
    uint64_t *done = empty + kStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    int *bail = reinterpret_cast<int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = blockIdx.y;
    const int kchunks = p.kchunks;
    // This CTA's matrix and its n-tile within it.
    int mi = 0;
    while (mi + 1 < p.nmats && p.mats[mi + 1].tile0 <= (int)blockIdx.x) mi++;
    const TcMat &mat = p.mats[mi];
    const int nt = (int)blockIdx.x - mat.tile0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        *bail = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)kTcN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    const uint32_t spin = p.spin ? p.spin : kSpinLimit;  // the waits on the other roles

    const unsigned char *ga = p.a + (size_t)mt * kchunks * kChunkBytes;
    const unsigned char *gb = mat.b + (size_t)nt * kchunks * kChunkBytes;

    if (warp == 0 && lane == 0) {
        // Producer. As a programmatic dependent of the rotation, wait for
        // it (and its writes of the x̂ image) before the first copy; the
        // set-up above already overlapped its tail.
        if (p.pdl) asm volatile("griddepcontrol.wait;" ::: "memory");
        int issued = 0;
        for (int kc = 0; kc < kchunks && !p.stall; kc++) {
            const int s = kc % kStages, round = kc / kStages;
            if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1, spin)) {
                atomicExch(p.err, 1);
                atomicExch(bail, 1);
                break;
            }
            mbar_expect_tx(&full[s], 2 * kChunkBytes);
            bulk_g2s(sa + s * kChunkBytes, ga + (size_t)kc * kChunkBytes, kChunkBytes, &full[s]);
            bulk_g2s(sb + s * kChunkBytes, gb + (size_t)kc * kChunkBytes, kChunkBytes, &full[s]);
            issued = kc + 1;
        }
        // Nothing may land in shared memory after exit: wait (bounded) for
        // the copies of the last chunk issued on each stage.
        for (int q = issued - kStages < 0 ? 0 : issued - kStages; q < issued; q++)
            if (!mbar_wait(&full[q % kStages], (q / kStages) & 1)) atomicExch(p.err, 4);
    } else if (warp == 1 && lane == 0) {
        // MMA issuer.
        bool ok = true;
        for (int kc = 0; kc < kchunks && ok; kc++) {
            const int s = kc % kStages, round = kc / kStages;
            if (!mbar_wait(&full[s], round & 1, spin)) {
                atomicExch(p.err, 2);
                atomicExch(bail, 1);
                ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a0 = smem_u32(sa + s * kChunkBytes), b0 = smem_u32(sb + s * kChunkBytes);
#pragma unroll
            for (int k = 0; k < kTcK / 16; k++)
                umma_f16(tmem, umma_desc(a0 + 32 * k), umma_desc(b0 + 32 * k), (kc > 0 || k > 0) ? 1u : 0u);
            umma_commit(&empty[s]);
        }
        umma_commit(done);
        // After a failed wait the epilogue may have given up on `done`
        // already: its arrival must still land before the CTA exits.
        if (!ok && !mbar_wait(done, 0)) atomicExch(p.err, 5);
    } else if (warp >= 2) {
        // Epilogue: warp w reads TMEM lanes 32·(w mod 4) .. +31.
        const int part = warp & 3;
        bool ok = mbar_wait(done, 0, spin);
        if (!ok) {
            atomicExch(p.err, 3);
            atomicExch(bail, 1);
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        ok = __all_sync(0xffffffffu, ok && *reinterpret_cast<volatile int *>(bail) == 0);
        // Stage 64 columns at a time through the (now idle) pipeline
        // buffers, rows padded to 68 floats, then store whole row segments:
        // each warp writes rows part, part+4, ... as 256 contiguous bytes.
        float *stage = reinterpret_cast<float *>(sa);
        constexpr int kHalf = 64, kPad = kHalf + 4;
        const int erow = part * 32 + lane;  // this thread's TMEM lane / tile row
        // Undo the row's and the matrix's power-of-two scales (exact) as the
        // accumulator leaves TMEM: one factor per thread, its tile row.
        const float fsc = __fmul_rn(p.rs[mt * kTcM + erow], mat.ws);
        for (int h = 0; h < kTcN; h += kHalf) {
            if (ok) {
#pragma unroll
                for (int c = 0; c < kHalf; c += 32) {
                    uint32_t r[32];
                    tmem_ld32(tmem + ((uint32_t)(part * 32) << 16) + (uint32_t)(h + c), r);
#pragma unroll
                    for (int q = 0; q < 8; q++)
                        *reinterpret_cast<float4 *>(stage + erow * kPad + c + 4 * q) =
                            make_float4(__fmul_rn(__uint_as_float(r[4 * q]), fsc),
                                        __fmul_rn(__uint_as_float(r[4 * q + 1]), fsc),
                                        __fmul_rn(__uint_as_float(r[4 * q + 2]), fsc),
                                        __fmul_rn(__uint_as_float(r[4 * q + 3]), fsc));
                }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (ok) {
                const int col0 = nt * kTcN + h;
                // 16 lanes per row (16 bytes each): two rows per instruction.
                const int sub = lane >> 4, c4 = (lane & 15) * 4;
                for (int rr = (warp - 2) * 2 + sub; rr < kTcM; rr += 8) {
                    const int row = mt * kTcM + rr, col = col0 + c4;
                    if (row < p.m && col < mat.n) {
                        const float4 v = *reinterpret_cast<const float4 *>(stage + rr * kPad + c4);
                        float *y = mat.y + (size_t)row * mat.ldy + col;
                        if (col + 4 <= mat.n && (mat.ldy & 3) == 0 && (((uintptr_t)y) & 15) == 0) {
                            *reinterpret_cast<float4 *>(y) = v;
                        } else {
                            const float vv[4] = {v.x, v.y, v.z, v.w};
                            for (int q = 0; q < 4 && col + q < mat.n; q++) y[q] = vv[q];
                        }
                    }
                }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)kTcN)
                     : "memory");
    }
}

// ---- persistent kernel for many rows (encoder prefill) --------------------
//
// One CTA per SM loops over 128 x 256 tiles of y (t -> n-tile t mod NT,
// m-tile t / NT, so the CTAs running together share m-tiles of x̂ in L2).
// TMEM holds two 128 x 256 fp32 accumulators (all 512 columns): while the
// epilogue warps drain one tile's accumulator, the MMA warp fills the other.
//   warp 0 lane 0   producer: per 64-wide K chunk, one bulk copy of the x̂
//                   chunk and two of the ŵ chunk (its two 128-row halves)
//                   into a 3-stage ring
//   warp 1 lane 0   MMA issuer: tcgen05.mma M = 128, N = 256, K = 16
//   warps 2-5       epilogue: TMEM -> registers -> a per-warp staging tile
//                   -> 256-byte row segments of y
// Bounded waits as in the kernel above.
constexpr int kPN = 256;
constexpr int kPStages = 3;
constexpr int kPStageBytes = 3 * kChunkBytes;  // x̂ 16 KB + ŵ 32 KB
constexpr int kPThreads = 320;  // producer, MMA, eight epilogue warps
constexpr int kPStgStride = 36;  // floats per staged row (32 + 4)
constexpr uint32_t kPIdesc = (1u << 4) | ((uint32_t)(kPN >> 3) << 17) |
                             ((uint32_t)(kTcM >> 4) << 24);

__device__ __forceinline__ void umma_f16_n256(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(dtmem),
        "l"(adesc), "l"(bdesc), "r"(kPIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_p(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// The matrix and 256-row tile of global n-tile nt (mats[].tile0 in
// 256-row units).
__device__ __forceinline__ int p_matrix(const TcParams &p, int nt) {
    int mi = 0;
    while (mi + 1 < p.nmats && p.mats[mi + 1].tile0 <= nt) mi++;
    return mi;
}

__global__ void __launch_bounds__(kPThreads, 1) cq_gemm_tc_persistent_kernel(const __grid_constant__ TcParams p,
                                                                             int ntg, int total) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    unsigned char *ring = smem;                                              // [stages][x̂ 16K | ŵ 32K]
    float *stg = reinterpret_cast<float *>(ring + kPStages * kPStageBytes);  // [8 warps][32][36]
    uint64_t *full = reinterpret_cast<uint64_t *>(stg + 8 * 32 * kPStgStride);
    uint64_t *empty = full + kPStages;
    uint64_t *accf = empty + kPStages;  // [2] accumulator b is ready
    uint64_t *acce = accf + 2;          // [2] accumulator b is drained
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acce + 2);
    int *bail = reinterpret_cast<int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kchunks = p.kchunks;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kPStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&accf[b], 1);
            mbar_init(&acce[b], 8);
        }
        *bail = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(2u * kPN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    volatile int *vbail = bail;
    const uint32_t spin = p.spin ? p.spin : kSpinLimit;  // the waits on the other roles

    if (warp == 0 && lane == 0) {
        if (p.pdl) asm volatile("griddepcontrol.wait;" ::: "memory");
        int c = 0;
        for (int t = blockIdx.x; t < total && !*vbail && !p.stall; t += gridDim.x) {
            const int nt = t % ntg, mt = t / ntg;
            const TcMat &mat = p.mats[p_matrix(p, nt)];
            const unsigned char *ga = p.a + (size_t)mt * kchunks * kChunkBytes;
            const unsigned char *gb = mat.b + (size_t)(2 * (nt - mat.tile0)) * kchunks * kChunkBytes;
            for (int kc = 0; kc < kchunks; kc++, c++) {
                const int s = c % kPStages, round = c / kPStages;
                if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1, spin)) {
                    atomicExch(p.err, 11);
                    atomicExch(bail, 1);
                    break;
                }
                unsigned char *st = ring + (size_t)s * kPStageBytes;
                mbar_expect_tx(&full[s], kPStageBytes);
                bulk_g2s(st, ga + (size_t)kc * kChunkBytes, kChunkBytes, &full[s]);
                bulk_g2s(st + kChunkBytes, gb + (size_t)kc * kChunkBytes, kChunkBytes, &full[s]);
                bulk_g2s(st + 2 * kChunkBytes, gb + (size_t)(kchunks + kc) * kChunkBytes, kChunkBytes, &full[s]);
            }
        }
        // Nothing may land in shared memory after exit.
        for (int q = c - kPStages < 0 ? 0 : c - kPStages; q < c; q++)
            if (!mbar_wait(&full[q % kPStages], (q / kPStages) & 1)) atomicExch(p.err, 12);
    } else if (warp == 1 && lane == 0) {
        int c = 0, i = 0;
        for (int t = blockIdx.x; t < total && !*vbail; t += gridDim.x, i++) {
            const int b = i & 1, u = i >> 1;
            if (u > 0 && !mbar_wait(&acce[b], (u - 1) & 1, spin)) {
                atomicExch(p.err, 13);
                atomicExch(bail, 1);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t d = tmem + (uint32_t)(b * kPN);
            bool ok = true;
            for (int kc = 0; kc < kchunks; kc++, c++) {
                const int s = c % kPStages, round = c / kPStages;
                if (!mbar_wait(&full[s], round & 1, spin)) {
                    atomicExch(p.err, 14);
                    atomicExch(bail, 1);
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t a0 = smem_u32(ring + (size_t)s * kPStageBytes);
                const uint32_t b0 = a0 + kChunkBytes;
#pragma unroll
                for (int k = 0; k < kTcK / 16; k++)
                    umma_f16_n256(d, umma_desc(a0 + 32 * k), umma_desc(b0 + 32 * k), (kc > 0 || k > 0) ? 1u : 0u);
                umma_commit(&empty[s]);
            }
            if (!ok) {
                // MMAs of this tile may still be running: let them finish
                // (bounded) before the teardown frees their TMEM. An
                // epilogue warp that sees accf[b] now also sees the bail.
                umma_commit(&accf[b]);
                if (!mbar_wait(&accf[b], u & 1)) atomicExch(p.err, 16);
                break;
            }
            umma_commit(&accf[b]);
        }
    } else if (warp >= 2) {
        const int part = warp & 3;          // TMEM lanes 32·part .. +31
        const int half = (warp - 2) >> 2;   // columns 128·half .. +127
        float *mystg = stg + (size_t)(warp - 2) * 32 * kPStgStride;
        int i = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, i++) {
            const int b = i & 1, u = i >> 1;
            bool ok = mbar_wait(&accf[b], u & 1, spin);
            ok = __all_sync(0xffffffffu, ok && *vbail == 0);
            if (!ok) {
                if (lane == 0) {
                    atomicExch(p.err, 15);
                    atomicExch(bail, 1);
                }
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int nt = t % ntg, mt = t / ntg;
            const TcMat &mat = p.mats[p_matrix(p, nt)];
            const int col_base = (nt - mat.tile0) * kPN;
            // The scales of this lane's accumulator row (TMEM lane = tile row).
            const float fsc = __fmul_rn(p.rs[mt * kTcM + part * 32 + lane], mat.ws);
            for (int cc = half * (kPN / 2); cc < (half + 1) * (kPN / 2); cc += 32) {
                {
                    uint32_t r[32];
                    tmem_ld32(tmem + ((uint32_t)(part * 32) << 16) + (uint32_t)(b * kPN + cc), r);
#pragma unroll
                    for (int q = 0; q < 8; q++)
                        *reinterpret_cast<float4 *>(mystg + lane * kPStgStride + 4 * q) =
                            make_float4(__fmul_rn(__uint_as_float(r[4 * q]), fsc),
                                        __fmul_rn(__uint_as_float(r[4 * q + 1]), fsc),
                                        __fmul_rn(__uint_as_float(r[4 * q + 2]), fsc),
                                        __fmul_rn(__uint_as_float(r[4 * q + 3]), fsc));
                }
                __syncwarp();
                // The warp's 32 rows x 32 columns: 8 lanes per row, four rows
                // per instruction.
                const int sub = lane >> 3, c4 = (lane & 7) * 4;
                for (int rr = sub; rr < 32; rr += 4) {
                    const int row = mt * kTcM + part * 32 + rr, col = col_base + cc + c4;
                    if (row < p.m && col < mat.n) {
                        const float4 v = *reinterpret_cast<const float4 *>(mystg + rr * kPStgStride + c4);
                        float *y = mat.y + (size_t)row * mat.ldy + col;
                        if (col + 4 <= mat.n && (mat.ldy & 3) == 0 && (((uintptr_t)y) & 15) == 0) {
                            *reinterpret_cast<float4 *>(y) = v;
                        } else {
                            const float vv[4] = {v.x, v.y, v.z, v.w};
                            for (int q = 0; q < 4 && col + q < mat.n; q++) y[q] = vv[q];
                        }
                    }
                }
                __syncwarp();
            }
            // This warp's quarter of accumulator b is read: release it.
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive_p(&acce[b]);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2u * kPN) : "memory");
    }
}

// x̂ = H·x per group of G (no 1/√G: it is in ŵ), scaled by a power of two
// per row, fp16, into the swizzled image [m_tile][kc][128 rows][128 B];
// rows past m and columns past In are zero. One warp per image row: lane l
// holds the columns 128·j + 4·l .. +3 (j < J), loaded as float4s (512
// contiguous bytes per warp load). The row's largest |x| fixes its scale
// 2^e, the largest with G·max|x|·2^e < 2^14, so no |x̂·2^e| reaches fp16's
// 65504 and the row keeps fp16's 11-bit precision however large or small
// its values are; rs[row] = 2^-e undoes it exactly in the GEMM's epilogue.
// The butterflies are fwht's (kernel.go:384), stage by stage: h < 4 inside
// a lane's float4, 4 <= h < 128 between lanes (xor h/4), h >= 128 between
// a lane's float4s. Each lane stores its four fp16 values as 8 bytes of a
// 128-byte chunk row.
template <int J>
__global__ void __launch_bounds__(128) rotate_f16_kernel(const float *__restrict__ x, int m, int in, int G,
                                                         int log2g, int kpad, int kchunks, long rows_total,
                                                         int vec, unsigned char *__restrict__ a,
                                                         float *__restrict__ rs) {
    // A GEMM launched as this kernel's programmatic dependent may start its
    // set-up now; it waits for this grid's completion before reading a.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int lane = threadIdx.x & 31;
    const long row = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows_total) return;  // whole warps
    float v[J][4];
    const bool real = row < m;
#pragma unroll
    for (int j = 0; j < J; j++) {
        const int c0 = 128 * j + 4 * lane;
        if (real && vec && c0 + 4 <= in) {
            const float4 f = __ldg(reinterpret_cast<const float4 *>(x + (size_t)row * in + c0));
            v[j][0] = f.x;
            v[j][1] = f.y;
            v[j][2] = f.z;
            v[j][3] = f.w;
        } else {
#pragma unroll
            for (int e = 0; e < 4; e++) v[j][e] = (real && c0 + e < in) ? x[(size_t)row * in + c0 + e] : 0.0f;
        }
    }
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < J; j++)
#pragma unroll
        for (int e = 0; e < 4; e++) amax = fmaxf(amax, fabsf(v[j][e]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    int sh = 0;  // the row's scale exponent e
    if (amax > 0.0f && amax <= 3.402823466e38f) {
        int k;
        frexpf(amax, &k);  // amax < 2^k
        sh = 14 - k - log2g;
        sh = sh < -120 ? -120 : sh > 120 ? 120 : sh;
    }
    // Butterflies inside a float4 (h = 1, 2).
#pragma unroll
    for (int h = 1; h < 4; h <<= 1) {
        if (h < G) {
#pragma unroll
            for (int j = 0; j < J; j++)
#pragma unroll
                for (int e = 0; e < 4; e++)
                    if ((e & h) == 0) {
                        const float a0 = v[j][e], b0 = v[j][e + h];
                        v[j][e] = a0 + b0;
                        v[j][e + h] = a0 - b0;
                    }
        }
    }
    // Between lanes (h = 4 .. 64).
    for (int h = 4; h < G && h < 128; h <<= 1) {
        const int pl = h >> 2;
#pragma unroll
        for (int j = 0; j < J; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float o = __shfl_xor_sync(0xffffffffu, v[j][e], pl);
                v[j][e] = (lane & pl) ? o - v[j][e] : v[j][e] + o;
            }
    }
    // Between float4s: h = 128 (G = 256, the largest group taken).
    if (G > 128) {
#pragma unroll
        for (int j = 0; j + 1 < J; j += 2)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float a0 = v[j][e], b0 = v[j + 1][e];
                v[j][e] = a0 + b0;
                v[j + 1][e] = a0 - b0;
            }
    }
    const float p2 = __int_as_float((127 + sh) << 23);
    const int mtile = (int)(row / kTcM), r = (int)(row % kTcM);
#pragma unroll
    for (int j = 0; j < J; j++) {
        const int c0 = 128 * j + 4 * lane;
        if (c0 >= kpad) continue;
        const __half2 h0 = __floats2half2_rn(__fmul_rn(v[j][0], p2), __fmul_rn(v[j][1], p2));
        const __half2 h1 = __floats2half2_rn(__fmul_rn(v[j][2], p2), __fmul_rn(v[j][3], p2));
        uint2 w;
        w.x = *reinterpret_cast<const uint32_t *>(&h0);
        w.y = *reinterpret_cast<const uint32_t *>(&h1);
        unsigned char *base = a + ((size_t)mtile * kchunks + c0 / kTcK) * kChunkBytes;
        *reinterpret_cast<uint2 *>(base + swz(r, c0 % kTcK)) = w;
    }
    if (lane == 0) rs[row] = __int_as_float((127 - sh) << 23);
}

// ŵ[r, k] = cb[idx]·n[r, g]·(1/√G)·wsc in fp16, swizzled
// [n_tile][kc][128][128 B]; rows past Out are zero. wsc is the matrix's
// power-of-two scale (its largest |ŵ| just under 2^15), undone in the
// epilogue. One thread per (row, 8 columns).
__global__ void dequant_f16_kernel(const __grid_constant__ CqShape s, const CqView v, float wsc, int ntiles,
                                   int kchunks, unsigned char *__restrict__ b) {
    const int units = ntiles * kTcN * (kchunks * kTcK / 8);
    const int u = blockIdx.x * blockDim.x + threadIdx.x;
    if (u >= units) return;
    const int per_row = kchunks * kTcK / 8;
    const int row = u / per_row, k0 = (u % per_row) * 8;
    const int ntile = row / kTcN, r = row % kTcN, kc = k0 / kTcK;
    __align__(16) __half out[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const int k = k0 + e;
        float w = 0.0f;
        if (row < v.out && k < s.pad) {
            const int g = k / s.group, kin = k % s.group;
            const size_t lrow = (size_t)g * v.ld + (size_t)(v.row0 + row);
            const int bit = kin * s.bits;
            const uint32_t code = (v.idx[lrow * s.gb + (bit >> 3)] >> (bit & 7)) & ((1u << s.bits) - 1u);
            w = __fmul_rn(__fmul_rn(__fmul_rn(s.cb[code], __half2float(v.nrm[lrow])), s.inv_sqrt), wsc);
        }
        out[e] = __float2half_rn(w);
    }
    unsigned char *base = b + ((size_t)ntile * kchunks + kc) * kChunkBytes;
    *reinterpret_cast<uint4 *>(base + swz(r, k0 % kTcK)) = *reinterpret_cast<const uint4 *>(out);
}

}  // namespace

// The x̂ image, then the rows' scales (one float per image row).
size_t tc_a_image_bytes(int m, int kchunks) { return (size_t)((m + kTcM - 1) / kTcM) * kchunks * kChunkBytes; }
size_t tc_a_bytes(int m, int kchunks) {
    return tc_a_image_bytes(m, kchunks) + (size_t)((m + kTcM - 1) / kTcM) * kTcM * sizeof(float);
}
// Weight images hold an even number of 128-row tiles (rows past Out are
// zero), so the persistent kernel's 256-row tiles never read past them.
static int tc_b_tiles(int n) { return ((n + 2 * kTcN - 1) / (2 * kTcN)) * 2; }
size_t tc_b_bytes(int n, int kchunks) { return (size_t)tc_b_tiles(n) * kchunks * kChunkBytes; }
int tc_kchunks(const CqShape &s) { return (s.pad + kTcK - 1) / kTcK; }

cudaError_t launch_dequant_f16(const CqShape &s, const CqView &v, float wsc, unsigned char *b, cudaStream_t st) {
    const int kchunks = tc_kchunks(s), ntiles = tc_b_tiles(v.out);
    const long units = (long)ntiles * kTcN * (kchunks * kTcK / 8);
    if (units == 0) return cudaSuccess;
    dequant_f16_kernel<<<(int)((units + 255) / 256), 256, 0, st>>>(s, v, wsc, ntiles, kchunks, b);
    count_launch();
    return cudaGetLastError();
}

template <int J>
static cudaError_t launch_rotate_j(const CqShape &s, const float *x, int m, int kpad, int kchunks, long rows,
                                   unsigned char *a, float *rs, cudaStream_t st) {
    int log2g = 0;
    while ((1 << log2g) < s.group) log2g++;
    const int vec = (s.in % 4 == 0) && (((uintptr_t)x) & 15) == 0;
    // Four rows (warps) per block: a call of few rows still spreads over
    // many SMs.
    rotate_f16_kernel<J><<<(int)((rows + 3) / 4), 128, 0, st>>>(x, m, s.in, s.group, log2g, kpad, kchunks, rows, vec,
                                                               a, rs);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_rotate_f16(const CqShape &s, const float *x, int m, unsigned char *a, cudaStream_t st) {
    const int kchunks = tc_kchunks(s), mtiles = (m + kTcM - 1) / kTcM;
    // The image covers kchunks·64 columns: the padding past groups·G is
    // zero (x is zero there, and H of zeros is zero within a group of
    // G <= 64; for larger G the padding is whole groups of zeros).
    const int kpad = kchunks * kTcK;
    const long rows = (long)mtiles * kTcM;
    if (rows == 0) return cudaSuccess;
    float *rs = reinterpret_cast<float *>(a + tc_a_image_bytes(m, kchunks));
    const int j = (kpad + 127) / 128;
    if (j <= 1) return launch_rotate_j<1>(s, x, m, kpad, kchunks, rows, a, rs, st);
    if (j <= 2) return launch_rotate_j<2>(s, x, m, kpad, kchunks, rows, a, rs, st);
    if (j <= 4) return launch_rotate_j<4>(s, x, m, kpad, kchunks, rows, a, rs, st);
    if (j <= 8) return launch_rotate_j<8>(s, x, m, kpad, kchunks, rows, a, rs, st);
    if (j <= 16) return launch_rotate_j<16>(s, x, m, kpad, kchunks, rows, a, rs, st);
    return launch_rotate_j<32>(s, x, m, kpad, kchunks, rows, a, rs, st);
}

static size_t tc_smem_bytes_st(int stages) { return 1024 + 2 * (size_t)stages * kChunkBytes + 8 * (2 * stages + 1) + 16; }
size_t tc_smem_bytes() { return tc_smem_bytes_st(2); }

// ---- the no-allocation entry point's scratch --------------------------------
//
// One file-scope device array holds the rotated-activation image of
// wc_cq_gemm_tc_noalloc and its rows' scales (kNoAllocScratchBytes),
// followed by its error word.
// Every GPU that loads the library carries it until the process exits.
// Host code cannot use the array's name as a device address (it names a
// host-side shadow), so each device's address is looked up once with
// cudaGetSymbolAddress, with that device current, and handed to the kernels.
// 16 MiB for the x̂ image and 512 KiB for its rows' scales (the most rows
// a 16 MiB image holds, at 64 columns, is 131,072).
constexpr size_t kNoAllocScratchBytes = ((size_t)16 << 20) + ((size_t)512 << 10);
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes + 256];

size_t noalloc_scratch_bytes() { return kNoAllocScratchBytes; }

// The array's device address per device, looked up on first use.
static unsigned char *g_noalloc_addr[64];
static std::mutex g_noalloc_mu;

static bool noalloc_ready(int dev) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    return g_noalloc_addr[dev] != nullptr;
}

// The array's device address on the current device (set-up on first use).
static cudaError_t noalloc_scratch(unsigned char **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_noalloc_addr[dev] = static_cast<unsigned char *>(p);
    }
    *out = g_noalloc_addr[dev];
    return cudaSuccess;
}

// The error word inside the array on the current device, or null when no
// no-allocation call has set the array up there yet (wc_device_status
// reads and clears it).
int *noalloc_err_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    unsigned char *base = nullptr;
    if (!noalloc_ready(dev) || noalloc_scratch(&base) != cudaSuccess) return nullptr;
    return reinterpret_cast<int *>(base + kNoAllocScratchBytes);
}

// Rotation into the static image, then the tensor-core GEMM, with no
// allocation. The caller has checked that the image fits
// (tc_a_bytes(rows, kchunks) <= kNoAllocScratchBytes) and that the weight
// image wimg exists. err: a device int for the bounded waits' error code,
// or null for the array's own word, which accumulates the codes until
// wc_device_status reads and clears it. persistent: the kernel
// wc_cq_gemm_ex picks for this many rows.
cudaError_t gemm_tc_noalloc(const CqShape &s, const unsigned char *wimg, float ws, const float *x, float *y, int rows,
                            int n, int *err, bool persistent, cudaStream_t st) {
    unsigned char *base = nullptr;
    cudaError_t e = noalloc_scratch(&base);
    if (e != cudaSuccess) return e;
    if (!err) err = reinterpret_cast<int *>(base + kNoAllocScratchBytes);
    e = launch_rotate_f16(s, x, rows, base, st);
    if (e != cudaSuccess) return e;
    TcParams p{};
    p.a = base;
    p.m = rows;
    p.kchunks = tc_kchunks(s);
    p.err = err;
    p.nmats = 1;
    p.rs = reinterpret_cast<const float *>(base + tc_a_image_bytes(rows, p.kchunks));
    p.mats[0] = TcMat{wimg, y, n, n, 0, ws};
    return persistent ? launch_gemm_tc_persistent(p, st) : launch_gemm_tc(p, st);
}

size_t tc_persistent_smem_bytes() {
    return 1024 + (size_t)kPStages * kPStageBytes + sizeof(float) * 8 * 32 * kPStgStride + 8 * (2 * kPStages + 4) + 16;
}

// The persistent kernel over mats[].tile0 in 256-row units; one CTA per SM
// (up to the tiles), as a programmatic dependent of the rotation.
cudaError_t launch_gemm_tc_persistent(const TcParams &p, cudaStream_t st) {
    const size_t smem = tc_persistent_smem_bytes();
    cudaError_t e =
        cudaFuncSetAttribute(cq_gemm_tc_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const TcMat &l = p.mats[p.nmats - 1];
    const int ntg = l.tile0 + (l.n + kPN - 1) / kPN;
    const int mtiles = (p.m + kTcM - 1) / kTcM;
    const int total = ntg * mtiles;
    if (total == 0) return cudaSuccess;
    TcParams q = p;
    q.pdl = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)(total < sms ? total : sms));
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, cq_gemm_tc_persistent_kernel, q, ntg, total);
    count_launch();
    return e != cudaSuccess ? e : cudaGetLastError();
}

int tc_total_tiles(const TcParams &p) {
    const TcMat &l = p.mats[p.nmats - 1];
    return l.tile0 + (l.n + kTcN - 1) / kTcN;
}

// The GEMM as a programmatic dependent launch of the rotation just queued
// on st: its CTAs may start while the rotation drains, and the producer
// waits for it before reading the x̂ image (griddepcontrol.wait).
cudaError_t launch_gemm_tc(const TcParams &p, cudaStream_t st) {
    const int ntiles = tc_total_tiles(p), mtiles = (p.m + kTcM - 1) / kTcM;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // The deepest ring that still holds the CTAs one wave needs per SM.
    const long long per_sm = ((long long)ntiles * mtiles + sms - 1) / sms;
    const int stages = per_sm <= 1 ? 6 : per_sm <= 2 ? 3 : 2;
    void (*fn)(TcParams) = stages == 6 ? cq_gemm_tc_kernel<6> : stages == 3 ? cq_gemm_tc_kernel<3> : cq_gemm_tc_kernel<2>;
    const size_t smem = tc_smem_bytes_st(stages);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    TcParams q = p;
    q.pdl = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)ntiles, (unsigned)mtiles);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, fn, q);
    count_launch();
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace wb
