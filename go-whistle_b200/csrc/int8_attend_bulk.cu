// int8_attend_bulk.cu — decode attention over int8 KV caches for one query
// row per stream and every key (AttendInt8 with t = 1 and no spans, and the
// batched wc_attend_int8_streams), with the cache rows staged in shared
// memory by bulk copies.
//
// Same quantities as int8_attend.cu (internal/needle/int8.go:194-285):
//   s_j = float32(dot_i32(q8, k8_j)) · (sq · sk_j) / scale   (quantised q)
//   p = softmax(s); out[d] = Σ_j float32(p_j · sv_j · float32(v8_j[d]))
// The exact-order instance keeps the reference's order and rounding
// (float64 exp, the sum in key order, the output key after key, no FMA);
// the any-order instance (WC_ATTEND_ANY_ORDER) uses expf, parallel sums and
// FMAs, and divides by the sum once at the end.
//
// One CTA per (stream, group of kvpc KV heads) and 160 threads:
//   warp 0      producer: streams the CTA's K rows (kvpc·qk bytes per key)
//               chunk after chunk, then its V rows (kvpc·vd bytes per key),
//               32 keys per chunk, through a ring of 2-8 stages (the
//               deepest that leaves room for two CTAs per SM). With every
//               KV head in the CTA a chunk is one contiguous range: one
//               cp.async.bulk for the rows and one for their scales. With
//               part of the heads, one bulk copy per row, and the row's
//               scales by 4-byte cp.async copies tracked by the same
//               mbarrier (issuing 32 copies per chunk costs the producer
//               far more time than one).
//   warps 1-4   consumers: the logits of each K chunk into shared memory
//               (thread per key and head, the query codes in registers);
//               after the last K chunk the softmax; then each V chunk
//               accumulated into registers (each thread 1, 2 or 4 adjacent
//               output columns, or several groups of 4, so that all 128
//               threads work), eight keys' loads ahead of their adds.
// The producer runs ahead by the ring's depth, so V chunks arrive while the
// consumers do the softmax. No tensor map, no multicast. Every mbarrier
// wait is bounded; on timeout the CTA records an error code and returns
// after its copies in flight have landed (also a bounded wait).
#include "common.cuh"
#include "needle_kernels.cuh"

namespace wb {

namespace {

constexpr int kBulkKeys = 32;        // keys per chunk: one row per producer lane
constexpr int kBulkMaxStages = 8;
constexpr int kBulkConsumers = 128;  // 4 warps
constexpr int kBulkThreads = 32 + kBulkConsumers;
constexpr uint32_t kBulkSpinLimit = 1u << 22;

__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void bar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void bar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(bar)) : "memory");
}

// Bounded wait for the phase of the given parity; false on timeout.
__device__ __forceinline__ bool bar_wait(uint64_t *bar, uint32_t parity) {
    const uint32_t a = su32(bar);
    for (uint32_t it = 0; it < kBulkSpinLimit; it++) {
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

__device__ __forceinline__ void bulk_row(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     su32(dst)),
                 "l"(src), "r"(bytes), "r"(su32(bar))
                 : "memory");
}

__device__ __forceinline__ void copy4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(su32(dst)), "l"(src) : "memory");
}

// The barrier counts one arrival when this thread's earlier cp.async
// copies have landed (the count was set for it at init).
__device__ __forceinline__ void copies_arrive(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(su32(bar)) : "memory");
}

__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kBulkConsumers) : "memory"); }

__device__ __forceinline__ float wmax(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// CPT adjacent int8 codes of a V row (CPT = 1, 2 or 4; aligned to CPT).
template <int CPT>
__device__ __forceinline__ uint32_t load_cols(const unsigned char *p) {
    if constexpr (CPT == 1) return *p;
    else if constexpr (CPT == 2) return *reinterpret_cast<const uint16_t *>(p);
    else return *reinterpret_cast<const uint32_t *>(p);
}

// acc[i] += w · float32(code i of v): exact order rounds the product and the
// sum separately (int8kernel.go:60), any order fuses them. float32(code) is
// formed without a conversion instruction: the biased code (code + 128) is
// the low mantissa byte of 2^23 (one byte permute), and 2^23 + 128 is
// subtracted (exact: every value is an integer below 2^24).
template <int CPT, bool EXACT>
__device__ __forceinline__ void accumulate(float *acc, float w, uint32_t v) {
    const uint32_t u = v ^ 0x80808080u;
    if constexpr (!EXACT && CPT % 2 == 0) {
        // Any order: two columns a packed f32x2 FMA (sm_100a). The exact
        // order keeps the scalar operations: its packed multiply-then-add
        // did not give the scalar path's bits (1-2 ulp apart).
        uint64_t ww, bias;
        asm("mov.b64 %0, {%1, %1};" : "=l"(ww) : "f"(w));
        asm("mov.b64 %0, {%1, %1};" : "=l"(bias) : "f"(-8388736.0f));
#pragma unroll
        for (int i = 0; i < CPT; i += 2) {
            uint64_t c, a;
            asm("mov.b64 %0, {%1, %2};"
                : "=l"(c)
                : "r"(__byte_perm(u, 0x4B000000u, 0x7540u + i)), "r"(__byte_perm(u, 0x4B000000u, 0x7540u + i + 1)));
            asm("add.rn.f32x2 %0, %0, %1;" : "+l"(c) : "l"(bias));
            asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(acc[i]), "f"(acc[i + 1]));
            asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(a) : "l"(ww), "l"(c));
            asm("mov.b64 {%0, %1}, %2;" : "=f"(acc[i]), "=f"(acc[i + 1]) : "l"(a));
        }
    } else {
#pragma unroll
        for (int i = 0; i < CPT; i++) {
            const float c = __fadd_rn(__int_as_float(__byte_perm(u, 0x4B000000u, 0x7540u + i)), -8388736.0f);
            acc[i] = EXACT ? __fadd_rn(acc[i], __fmul_rn(w, c)) : fmaf(w, c, acc[i]);
        }
    }
}

}  // namespace

// The layout for `stages` ring stages (2 .. 8).
BulkLayout attend_bulk_layout(const AttendParams &p, int stages) {
    BulkLayout L{};
    L.stages = stages < 2 ? 2 : stages > kBulkMaxStages ? kBulkMaxStages : stages;
    const int kvpc = p.kv_per_cta, hb = kvpc * (p.heads / p.kv_heads);
    const int seg = kvpc * (p.qk > p.vd ? p.qk : p.vd);
    L.scale_off = ((size_t)kBulkKeys * seg + 15) & ~(size_t)15;
    L.stage = (L.scale_off + (size_t)kBulkKeys * kvpc * 4 + 127) & ~(size_t)127;
    L.lstride = (p.max_keys + 3) & ~3;
    L.lg = L.stage * L.stages;
    L.q8 = L.lg + sizeof(float) * (size_t)hb * L.lstride;
    L.qf = (L.q8 + (size_t)hb * p.qk + 15) & ~(size_t)15;
    L.red = L.qf + sizeof(float) * (size_t)hb * p.qk;  // [hb] sq, [hb] max, [hb] sum
    L.bars = (L.red + sizeof(float) * 3 * (size_t)hb + 7) & ~(size_t)7;
    L.total = L.bars + sizeof(uint64_t) * 2 * L.stages + 16;
    return L;
}

namespace {

template <int QKV, bool EXACT, int COLS>  // qk / 16; exact order; output columns per consumer thread
__global__ void __launch_bounds__(kBulkThreads, (COLS >= 8 || QKV >= 6) ? 4 : 6) attend_int8_bulk_kernel(const __grid_constant__ AttendParams p,
                                                                       const __grid_constant__ BulkLayout L) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int qk = 16 * QKV;
    const int kvpc = p.kv_per_cta, kvh = p.kv_heads, gs = p.heads / kvh, hb = kvpc * gs;
    const int kg = blockIdx.x, b = blockIdx.y;
    const int kv0 = kg * kvpc, h0 = kv0 * gs;
    const int vd = p.vd;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    float *lg = reinterpret_cast<float *>(smem + L.lg);
    int8_t *q8 = reinterpret_cast<int8_t *>(smem + L.q8);
    float *qf = reinterpret_cast<float *>(smem + L.qf);
    float *sq = reinterpret_cast<float *>(smem + L.red);
    float *hmax = sq + hb, *hsum = hmax + hb;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bars);
    const int NS = L.stages;
    uint64_t *empty = full + NS;
    int *bail = reinterpret_cast<int *>(empty + NS);

    int nkeys = p.nkeys;
    if (p.nkeys_dev) nkeys = min(max(p.nkeys_dev[b], 0), p.cap);
    const int nch = (nkeys + kBulkKeys - 1) / kBulkKeys;
    const size_t krow = (size_t)kvh * qk, vrow = (size_t)kvh * vd;
    const uint32_t kseg = (uint32_t)(kvpc * qk), vseg = (uint32_t)(kvpc * vd);

    if (tid == 0) {
        for (int s = 0; s < NS; s++) {
            bar_init(&full[s], 33);  // lane 0's expect-tx arrival + 32 copy arrivals
            bar_init(&empty[s], kBulkConsumers / 32);
        }
        *bail = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == 0) {
        // Producer: segment s < nch is K chunk s, else V chunk s - nch.
        const size_t blk = kv_block(p, b);
        const int8_t *k8 = p.k8 + blk * p.cap * krow + (size_t)kv0 * qk;
        const int8_t *v8 = p.v8 + blk * p.cap * vrow + (size_t)kv0 * vd;
        const float *ks = p.ks + blk * p.cap * kvh + kv0;
        const float *vs = p.vs + blk * p.cap * kvh + kv0;
        int issued = 0;
        for (int s = 0; s < 2 * nch; s++) {
            const int st = s % NS, round = s / NS;
            bool ok = round == 0 || bar_wait(&empty[st], (round - 1) & 1);
            ok = __all_sync(0xffffffffu, ok && *reinterpret_cast<volatile int *>(bail) == 0);
            if (!ok) {
                if (lane == 0) {
                    atomicExch(p.err, 4);
                    atomicExch(bail, 1);
                }
                break;
            }
            const bool isk = s < nch;
            const int key0 = (isk ? s : s - nch) * kBulkKeys;
            const int rows = min(kBulkKeys, nkeys - key0);
            const uint32_t seg = isk ? kseg : vseg;
            unsigned char *dst = smem + (size_t)st * L.stage;
            float *sdst = reinterpret_cast<float *>(dst + L.scale_off);
            if (p.bulk_whole) {
                // All KV heads: the chunk's rows are one contiguous range,
                // and so are its scales (bulk-copied up to the last whole
                // 16 bytes when aligned, the rest by 4-byte copies).
                const float *ssrc = (isk ? ks : vs) + (size_t)key0 * kvh;
                const uint32_t nsc = (uint32_t)(rows * kvh);
                const uint32_t sbulk = p.bulk_scales ? (nsc * 4u) & ~15u : 0u;
                if (lane == 0) {
                    bar_expect_tx(&full[st], (uint32_t)rows * seg + sbulk);
                    bulk_row(dst, isk ? (const void *)(k8 + (size_t)key0 * krow) : (const void *)(v8 + (size_t)key0 * vrow),
                             (uint32_t)rows * seg, &full[st]);
                    if (sbulk) bulk_row(sdst, ssrc, sbulk, &full[st]);
                }
                for (uint32_t e = sbulk / 4 + lane; e < nsc; e += 32) copy4(sdst + e, ssrc + e);
            } else {
                if (lane == 0) bar_expect_tx(&full[st], (uint32_t)rows * seg);
                __syncwarp();
                if (lane < rows) {
                    const size_t key = (size_t)key0 + lane;
                    bulk_row(dst + (size_t)lane * seg,
                             isk ? (const void *)(k8 + key * krow) : (const void *)(v8 + key * vrow), seg, &full[st]);
                    const float *ssrc = (isk ? ks : vs) + key * kvh;
                    for (int c = 0; c < kvpc; c++) copy4(sdst + lane * kvpc + c, ssrc + c);
                }
            }
            copies_arrive(&full[st]);
            issued = s + 1;
        }
        // Nothing may land in shared memory after the CTA exits: wait
        // (bounded) for the last stages issued. On the normal path the
        // consumers already saw them complete.
        for (int s = max(0, issued - NS); s < issued; s++)
            if (!bar_wait(&full[s % NS], (s / NS) & 1) && lane == 0) atomicExch(p.err, 5);
        return;
    }

    // Consumers.
    const int ct = tid - 32, cw = warp - 1;
    // 1. Queries (QuantizeRow per head, int8.go:36).
    for (int e = ct; e < hb * qk; e += kBulkConsumers) qf[e] = p.q[((size_t)b * p.heads + h0) * qk + e];
    consumers_sync();
    if (p.quant_q) {
        for (int h = cw; h < hb; h += kBulkConsumers / 32) {
            const float *x = qf + h * qk;
            float m = 0.0f;
            for (int i = lane; i < qk; i += 32) m = fmaxf(m, fabsf(x[i]));
            m = wmax(m);
            const float s = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
            for (int i = lane; i < qk; i += 32) {
                int r = __float2int_rn(__fdiv_rn(x[i], s));
                q8[h * qk + i] = (int8_t)(r < -128 ? -128 : (r > 127 ? 127 : r));
            }
            if (lane == 0) sq[h] = s;
        }
    }
    consumers_sync();

    // 2. Logits: thread (key k, head h), h fixed per thread (hb divides 128).
    const int my_h = ct % hb, kstep = kBulkConsumers / hb;
    const int my_kvl = my_h / gs;
    uint32_t qw[4 * QKV];
    float my_sq = 0.0f;
    if (p.quant_q) {
#pragma unroll
        for (int v = 0; v < QKV; v++) {
            const uint4 w = *reinterpret_cast<const uint4 *>(q8 + my_h * qk + 16 * v);
            qw[4 * v] = w.x;
            qw[4 * v + 1] = w.y;
            qw[4 * v + 2] = w.z;
            qw[4 * v + 3] = w.w;
        }
        my_sq = sq[my_h];
    }
    bool ok = true;
    for (int c = 0; c < nch && ok; c++) {
        const int st = c % NS, round = c / NS;
        ok = __all_sync(0xffffffffu, bar_wait(&full[st], round & 1));
        if (!ok) break;
        const unsigned char *stage = smem + (size_t)st * L.stage;
        const float *ssc = reinterpret_cast<const float *>(stage + L.scale_off);
        const int key0 = c * kBulkKeys, rows = min(kBulkKeys, nkeys - key0);
        for (int k = ct / hb; k < rows; k += kstep) {
            const uint4 *kr = reinterpret_cast<const uint4 *>(stage + (size_t)k * kseg + my_kvl * qk);
            const float sk = ssc[k * kvpc + my_kvl];
            float logit;
            if (p.quant_q) {
                // Four partial int32 sums (exact in any order: |dot| < 2^21).
                int32_t d0 = 0, d1 = 0, d2 = 0, d3 = 0;
#pragma unroll
                for (int v = 0; v < QKV; v++) {
                    const uint4 w = kr[v];
                    d0 = __dp4a((int)qw[4 * v], (int)w.x, d0);
                    d1 = __dp4a((int)qw[4 * v + 1], (int)w.y, d1);
                    d2 = __dp4a((int)qw[4 * v + 2], (int)w.z, d2);
                    d3 = __dp4a((int)qw[4 * v + 3], (int)w.w, d3);
                }
                const int32_t dot = (d0 + d1) + (d2 + d3);
                logit = __fdiv_rn(__fmul_rn(__int2float_rn(dot), __fmul_rn(my_sq, sk)), p.scale);
            } else {
                const float *qh = qf + my_h * qk;
                float sacc = 0.0f;
#pragma unroll
                for (int v = 0; v < QKV; v++) {
                    const uint4 w = kr[v];
                    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int cc = 0; cc < 16; cc++) {
                        const float kb = (float)(int8_t)((ww[cc >> 2] >> (8 * (cc & 3))) & 0xffu);
                        sacc = __fadd_rn(sacc, __fmul_rn(qh[16 * v + cc], kb));
                    }
                }
                logit = __fdiv_rn(__fmul_rn(sacc, sk), p.scale);
            }
            lg[(size_t)my_h * L.lstride + key0 + k] = logit;
        }
        __syncwarp();
        if (lane == 0) bar_arrive(&empty[st]);
    }
    if (!ok) {
        if (lane == 0) {
            atomicExch(p.err, 6);
            atomicExch(bail, 1);
        }
        return;
    }
    consumers_sync();

    // 3. Softmax per head (load.go:127, exp.go:238): warp cw owns heads
    //    cw, cw + 4, ... and needs no other warp until the output phase.
    constexpr int kCW = kBulkConsumers / 32;
    for (int h = cw; h < hb; h += kCW) {
        float *l = lg + (size_t)h * L.lstride;
        float m = -INFINITY;
#pragma unroll 4
        for (int k = lane; k < nkeys; k += 32) m = fmaxf(m, l[k]);
        m = wmax(m);
        float sm = 0.0f;
#pragma unroll 4
        for (int k = lane; k < nkeys; k += 32) {
            const float e = EXACT ? (float)exp((double)__fsub_rn(l[k], m)) : expf(l[k] - m);
            l[k] = e;
            sm += e;
        }
        if (!EXACT) {
            sm = wsum(sm);
            if (lane == 0) hsum[h] = sm;
        }
    }
    if (EXACT) {
        __syncwarp();
        // The sum in key order: lane j of the warp takes head cw + 4j.
        const int h = cw + kCW * lane;
        if (h < hb) {
            const float *l = lg + (size_t)h * L.lstride;
            float sum = 0.0f;
            int k = 0;
#pragma unroll 4
            for (; k + 4 <= nkeys; k += 4) {
                const float4 v = *reinterpret_cast<const float4 *>(l + k);
                sum = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sum, v.x), v.y), v.z), v.w);
            }
            for (; k < nkeys; k++) sum = __fadd_rn(sum, l[k]);
            hsum[h] = sum;
        }
        __syncwarp();
        for (int hh = cw; hh < hb; hh += kCW) {
            float *l = lg + (size_t)hh * L.lstride;
            const float sum = hsum[hh];
            for (int k = lane; k < nkeys; k += 32) l[k] = __fdiv_rn(l[k], sum);
        }
    }
    consumers_sync();

    // 4. Output: thread ct owns UNITS units of CPT adjacent columns, unit u
    //    = ct + 128·j, so all 128 threads work even for narrow groups.
    constexpr int CPT = COLS < 4 ? COLS : 4, UNITS = COLS / CPT;
    float acc[COLS];
    int oh[UNITS], od[UNITS], okv[UNITS];
    bool oval[UNITS];
#pragma unroll
    for (int j = 0; j < UNITS; j++) {
        const int o = CPT * (ct + kBulkConsumers * j);
        oval[j] = o < hb * vd;
        oh[j] = oval[j] ? o / vd : 0;
        od[j] = oval[j] ? o % vd : 0;
        okv[j] = oh[j] / gs;
#pragma unroll
        for (int i = 0; i < CPT; i++) acc[CPT * j + i] = 0.0f;
    }
    for (int c = 0; c < nch && ok; c++) {
        const int s = nch + c, st = s % NS, round = s / NS;
        ok = __all_sync(0xffffffffu, bar_wait(&full[st], round & 1));
        if (!ok) break;
        const unsigned char *stage = smem + (size_t)st * L.stage;
        const float *ssc = reinterpret_cast<const float *>(stage + L.scale_off);
        const int key0 = c * kBulkKeys, rows = min(kBulkKeys, nkeys - key0);
#pragma unroll
        for (int j = 0; j < UNITS; j++) {
            if (!oval[j]) continue;
            const float *wrow = lg + (size_t)oh[j] * L.lstride + key0;
            const unsigned char *vcol = stage + okv[j] * vd + od[j];
            const float *scol = ssc + okv[j];
            int k = 0;
            // Eight keys at a time: every load first, then the adds in key order.
            for (; k + 8 <= rows; k += 8) {
                float w[8];
                uint32_t v[8];
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    w[u] = EXACT ? __fmul_rn(wrow[k + u], scol[(k + u) * kvpc]) : wrow[k + u] * scol[(k + u) * kvpc];
                    v[u] = load_cols<CPT>(vcol + (size_t)(k + u) * vseg);
                }
#pragma unroll
                for (int u = 0; u < 8; u++) accumulate<CPT, EXACT>(acc + CPT * j, w[u], v[u]);
            }
            for (; k < rows; k++) {
                const float w = EXACT ? __fmul_rn(wrow[k], scol[k * kvpc]) : wrow[k] * scol[k * kvpc];
                accumulate<CPT, EXACT>(acc + CPT * j, w, load_cols<CPT>(vcol + (size_t)k * vseg));
            }
        }
        __syncwarp();
        if (lane == 0) bar_arrive(&empty[st]);
    }
    if (!ok) {
        if (lane == 0) {
            atomicExch(p.err, 7);
            atomicExch(bail, 1);
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < UNITS; j++) {
        if (!oval[j]) continue;
        float *o = p.out + ((size_t)b * p.heads + h0 + oh[j]) * vd + od[j];
        float inv = 1.0f;
        if (!EXACT) inv = hsum[oh[j]] > 0.0f ? 1.0f / hsum[oh[j]] : 0.0f;
#pragma unroll
        for (int i = 0; i < CPT; i++) o[i] = EXACT ? acc[CPT * j + i] : acc[CPT * j + i] * inv;
    }
}

template <int QKV, bool EXACT>
void (*bulk_fn_cols(int cols))(AttendParams, BulkLayout) {
    switch (cols) {
        case 1: return attend_int8_bulk_kernel<QKV, EXACT, 1>;
        case 2: return attend_int8_bulk_kernel<QKV, EXACT, 2>;
        case 4: return attend_int8_bulk_kernel<QKV, EXACT, 4>;
        case 8: return attend_int8_bulk_kernel<QKV, EXACT, 8>;
        default: return attend_int8_bulk_kernel<QKV, EXACT, 16>;
    }
}

template <bool EXACT>
void (*bulk_fn(int qkv, int cols))(AttendParams, BulkLayout) {
    switch (qkv) {
        case 1: return bulk_fn_cols<1, EXACT>(cols);
        case 2: return bulk_fn_cols<2, EXACT>(cols);
        case 3: return bulk_fn_cols<3, EXACT>(cols);
        case 4: return bulk_fn_cols<4, EXACT>(cols);
        case 5: return bulk_fn_cols<5, EXACT>(cols);
        case 6: return bulk_fn_cols<6, EXACT>(cols);
        case 7: return bulk_fn_cols<7, EXACT>(cols);
        default: return bulk_fn_cols<8, EXACT>(cols);
    }
}

// Output columns per consumer thread: 1, 2 or 4 adjacent columns while the
// group has at most 512 columns, then 2 or 4 units of 4.
int bulk_cols(const AttendParams &p) {
    const int cols = p.kv_per_cta * (p.heads / p.kv_heads) * p.vd;
    const int per = (cols + kBulkConsumers - 1) / kBulkConsumers;
    return per <= 1 ? 1 : per <= 2 ? 2 : per <= 4 ? 4 : per <= 8 ? 8 : 16;
}

}  // namespace

// Shape conditions of the bulk kernel for a KV-head group of kvpc heads
// (alignment of the caches is the caller's check).
bool attend_bulk_shape_ok(const AttendParams &p, int kvpc) {
    const int gs = p.heads / p.kv_heads, hb = kvpc * gs;
    return p.t == 1 && !p.spans && !p.probs && p.qk % 16 == 0 && p.qk <= 128 && p.vd % 16 == 0 &&
           p.kv_heads % kvpc == 0 && kBulkConsumers % hb == 0 && hb * p.vd <= 16 * kBulkConsumers;
}

// The deepest ring (up to 8 stages) that still lets `share` CTAs share an
// SM, or, when even two stages do not, the deepest that fits one CTA.
BulkLayout attend_bulk_pick_layout(const AttendParams &p, size_t smem_per_sm, size_t smem_per_block, int share) {
    const size_t part = smem_per_sm / (size_t)(share > 0 ? share : 1);
    const size_t two = part > 1024 ? part - 1024 : 0;  // 1 KB reserved per CTA
    for (int st = kBulkMaxStages; st >= 2; st--) {
        BulkLayout L = attend_bulk_layout(p, st);
        if (L.total <= two) return L;
    }
    for (int st = kBulkMaxStages; st >= 2; st--) {
        BulkLayout L = attend_bulk_layout(p, st);
        if (L.total <= smem_per_block) return L;
    }
    return attend_bulk_layout(p, 2);
}

cudaError_t attend_bulk_occupancy(const AttendParams &p, const BulkLayout &L, bool exact, int *blocks_per_sm) {
    void (*fn)(AttendParams, BulkLayout) = exact ? bulk_fn<true>(p.qk / 16, bulk_cols(p)) : bulk_fn<false>(p.qk / 16, bulk_cols(p));
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, fn, kBulkThreads, L.total);
}

cudaError_t launch_attend_bulk(const AttendParams &p, const BulkLayout &L, int streams, bool exact, cudaStream_t st) {
    void (*fn)(AttendParams, BulkLayout) = exact ? bulk_fn<true>(p.qk / 16, bulk_cols(p)) : bulk_fn<false>(p.qk / 16, bulk_cols(p));
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
    if (e != cudaSuccess) return e;
    fn<<<dim3(p.kv_heads / p.kv_per_cta, streams), kBulkThreads, L.total, st>>>(p, L);
    count_launch();
    return cudaGetLastError();
}

}  // namespace wb
