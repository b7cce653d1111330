// cq_lut_stream.cu — the streaming CQ LUT GEMV for large batch-1 products
// (many GEMMs matrices, or one large matrix), on sm_100a.
//
// Same arithmetic as cq_lut.cu (and so the reference's lut kernel, bit for
// bit); a different shape of work, built to run at HBM speed:
//
// * Persistent CTAs, one per SM. Each rotates and tabulates the activation
//   once, then streams its share of 32-row warp tiles of every matrix.
// * Byte tables. For each index byte position j the CTA holds all 256
//   values T_j[b] = v_{2j}[b & 15] + v_{2j+1}[b >> 4] (the lo and hi nibble
//   tables of lut.go:239-282 added, stored with a +16384 bias as uint16), so
//   one shared-memory load serves one index byte (the reference's VPSHUFB
//   kernel needs two). Up to 256 byte positions (128 KB) are resident; wider
//   rows are processed in passes of 256 positions, the partial row sums
//   carried in the output between passes (the group order is kept).
// * Conflict-free lookups. Tables are laid out T[b][j] (j fastest), so the
//   bank of a lookup depends only on j. The HBM layout permutes each row's
//   64-byte superchunks by the row's lane (root row mod 32) such that, at
//   every step, the 32 lanes of a warp touch 32 distinct byte pairs of the
//   superchunk while each lane still reads its registers in a fixed order
//   and finishes one whole group per phase. The address of a lookup is one
//   PRMT: (b << 8) | colbyte, colbyte from a per-lane packed table.
// * Exactness: the integer group sums are exact; each group's term
//   float32(Σv) · (norm · step) goes through shared memory so the row's terms
//   are added in group order, as lut.go:309 does.
//
// Layouts (built by api.cu at matrix creation, "stream layout"):
//   sidx[((sc*4 + i)*ld + R)*16 + k]  byte k of quarter i of superchunk sc of
//                                     root row R, slot order (below)
//   snrm[(sc*ld + R)*NG + q]          FP16 norm of the group in phase q
// with P = gb/2 byte pairs per group, NG = 32/P groups per superchunk, lane
// id λ = R mod 32 = P·a + c, and slot s = P·q + t holding the superchunk's
// byte pair o(s) = P·((q + a) mod NG) + ((t + c) mod P).
#include <mutex>

#include "common.cuh"
#include "cq_kernels.cuh"

namespace wb {

namespace {

constexpr int kStreamThreads = 512;
constexpr int kStreamWarps = kStreamThreads / 32;
constexpr int kPassPositions = 256;               // byte positions per table pass
constexpr int kTabBytes = 2 * 256 * 128 * 2;      // two blocks of [256 b][128 j] uint16
constexpr uint32_t kTabAbs = 65536;               // shared-window address of the byte tables
constexpr int kNibBytes = 2 * 16 * kPassPositions * 2;  // lo/hi nibble tables [16][256] uint16
constexpr uint32_t kEntryBias = 8192;             // per nibble entry, so a byte entry carries 16384

// d = byte permute of {b, a} by an immediate selector.
template <uint32_t SEL>
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "n"(SEL));
    return d;
}

// A byte-table entry at shared-window address addr + IMM: one LDS, the
// table's absolute base folded into the immediate.
template <uint32_t IMM>
__device__ __forceinline__ int32_t lds_tab(uint32_t addr) {
    uint16_t v;
    asm("ld.shared.u16 %0, [%1+%2];" : "=h"(v) : "r"(addr), "n"(IMM));
    return (int32_t)v;
}

// The run holding tile t.
template <class SP>
__device__ __forceinline__ int find_run(const SP &p, int t) {
    int lo = 0, hi = p.nruns - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (p.runs[mid].tile0 <= t)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

// Tile t's run, trying k (the previous tile's) first.
template <class SP>
__device__ __forceinline__ int run_from(const SP &p, int t, int k) {
    if (k >= 0 && p.runs[k].tile0 <= t && t < p.runs[k].tile0 + p.runs[k].count * p.runs[k].tpm) return k;
    return find_run(p, t);
}

// Tile t of run k: its matrix's view and output, and the tile's first row.
struct TileLoc {
    CqView v;
    float *y;
    int r0;
};
template <class SP>
__device__ __forceinline__ TileLoc tile_loc(const SP &p, int t, int k, int act = 0) {
    const StreamRun &R = p.runs[k];
    const int u = t - R.tile0, i = u / R.tpm;
    TileLoc L;
    L.v = R.v;
    L.v.row0 += i * R.row_step;
    L.y = R.y + (long long)i * R.y_step + (long long)act * R.y_act;
    L.r0 = (u - i * R.tpm) * 32;
    return L;
}

// Rotation, group bounds, 8191/M and steps for one activation (lut.go:160-178).
__device__ void rotate_and_bound(const CqShape &s, const float *x, float *xs, float *steps, float *invs) {
    const int tid = threadIdx.x, pad = s.pad, G = s.group, half = G >> 1;
    const int nt = blockDim.x;
    if (G <= 32) {
        // Groups within a warp: lane l of chunk c holds element 32c + l; the
        // butterflies (the same stages and operand order as below) and the
        // group's bound run by shuffles, with no block barrier between.
        const int lane = tid & 31;
        for (int c = tid >> 5; c * 32 < pad; c += nt >> 5) {
            const int k = c * 32 + lane;
            float v = k < s.in ? x[k] : 0.0f;
            for (int h = 1; h < G; h <<= 1) {
                const float o = __shfl_xor_sync(0xffffffffu, v, h);
                v = (lane & h) ? __fsub_rn(o, v) : __fadd_rn(v, o);
            }
            if (k < pad) xs[k] = v;
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
            if ((lane & (G - 1)) == 0 && k < pad) {
                const int g = k / G;
                const float m = __fmul_rn(s.cb_max, mv);
                invs[g] = m > 0.0f ? __fdiv_rn((float)kLutQ, m) : 0.0f;
                steps[g] = __fmul_rn(m, s.lut_step);
            }
        }
        __syncthreads();
        return;
    }
    for (int k = tid; k < pad; k += nt) xs[k] = k < s.in ? x[k] : 0.0f;
    __syncthreads();
    const int lg2 = 31 - __clz(G);  // G is a power of two: shifts, not divisions
    for (int st = 0; (1 << st) < G; st++) {
        const int h = 1 << st;
        for (int b = tid; b < pad / 2; b += nt) {
            const int g = b >> (lg2 - 1), t = b & (half - 1);
            const int j = (g << lg2) + ((t >> st) << (st + 1)) + (t & (h - 1));
            float a = xs[j], c = xs[j + h];
            xs[j] = __fadd_rn(a, c);
            xs[j + h] = __fsub_rn(a, c);
        }
        __syncthreads();
    }
    const int warp = tid >> 5, lane = tid & 31;
    for (int g = warp; g < s.groups; g += nt / 32) {
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
}

// Byte tables for byte positions [j0, j0 + npos) of the row (npos even).
__device__ void build_pass_tables(const CqShape &s, const float *xs, const float *invs, int j0, int npos,
                                  uint16_t *nib, uint16_t *tab) {
    const int tid = threadIdx.x;
    const int lg2 = 31 - __clz(s.group);  // the group is a power of two
    // Nibble tables, biased: nib[e][c][j] for the lo (e = 0) and hi (e = 1)
    // nibble of byte position j0 + j (lut.go:248-255, 272-279).
    for (int u = tid; u < 2 * npos; u += (int)blockDim.x) {
        const int e = u >= npos, j = u - e * npos;
        uint16_t *dst = nib + e * 16 * kPassPositions + j;
        const int np = 2 * (j0 + j) + e;  // nibble position in the row
        if (s.bits == 4) {
            const float a = __fmul_rn(xs[np], invs[np >> lg2]);
#pragma unroll
            for (int c = 0; c < 16; c++)
                dst[c * kPassPositions] = (uint16_t)(__float2int_rn(__fmul_rn(s.cb[c], a)) + (int)kEntryBias);
        } else {
            const float inv = invs[(2 * np) >> lg2];
            const float a = __fmul_rn(xs[2 * np], inv), b = __fmul_rn(xs[2 * np + 1], inv);
#pragma unroll
            for (int c = 0; c < 16; c++) {
                const float v = __fadd_rn(__fmul_rn(s.cb[c & 3], a), __fmul_rn(s.cb[c >> 2], b));
                dst[c * kPassPositions] = (uint16_t)(__float2int_rn(v) + (int)kEntryBias);
            }
        }
    }
    __syncthreads();
    // Byte tables: tab[blk][b][jj] = nib[0][b & 15][j] + nib[1][b >> 4][j],
    // j = 128·blk + jj. A thread takes two adjacent positions (one word of
    // each nibble table row) and a quarter of the hi nibbles: 20 word loads,
    // 64 word stores (packed adds carry nothing: each half stays below
    // 2^15). A warp's loads and stores each cover one 128-byte row, so they
    // are conflict-free.
    const int npairs = npos / 2;
    const bool p2 = (npairs & (npairs - 1)) == 0;  // a power of two: shifts (the usual widths)
    const int lp = 31 - __clz(npairs);
    const uint32_t *nw = reinterpret_cast<const uint32_t *>(nib);
    for (int u = tid; u < 4 * npairs; u += (int)blockDim.x) {
        const int jp = p2 ? (u & (npairs - 1)) : u % npairs, hq = p2 ? (u >> lp) : u / npairs, j = 2 * jp;
        uint32_t lo[16], hi[4];
#pragma unroll
        for (int c = 0; c < 16; c++) lo[c] = nw[(c * kPassPositions + j) >> 1];
#pragma unroll
        for (int i = 0; i < 4; i++) hi[i] = nw[((16 + 4 * hq + i) * kPassPositions + j) >> 1];
        uint32_t *dst = reinterpret_cast<uint32_t *>(tab + (size_t)(j >> 7) * 256 * 128 + (j & 127)) +
                        (size_t)(4 * hq) * 16 * 64;
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int c = 0; c < 16; c++) dst[(16 * i + c) * 64] = lo[c] + hi[i];
    }
    __syncthreads();
}

// One superchunk of a 32-row tile: 32 slots of two table lookups each, one
// group per phase; the group terms go through shared memory so the row adds
// them in group order. SCL (the superchunk within the pass) fixes the table
// block and half, so every lookup is one PRMT, one LDS and one IADD.
template <int GB, int SCL>
__device__ __forceinline__ float superchunk(const uint4 (&d)[4], const uint32_t (&nw)[4], const uint32_t (&cbw)[16],
                                            const float *steps, float *wterms, int lane, int a_rot, int sc,
                                            float y) {
    constexpr int P = GB / 2, NG = 32 / P;
    constexpr uint32_t TB = kTabAbs + (SCL >> 1) * (256 * 128 * 2) + (SCL & 1) * 128;
    const uint32_t dw[16] = {d[0].x, d[0].y, d[0].z, d[0].w, d[1].x, d[1].y, d[1].z, d[1].w,
                             d[2].x, d[2].y, d[2].z, d[2].w, d[3].x, d[3].y, d[3].z, d[3].w};
#pragma unroll
    for (int q = 0; q < NG; q++) {
        int32_t acc0 = 0, acc1 = 0;
#pragma unroll
        for (int tt = 0; tt < P; tt++) {
            const int slot = P * q + tt;
            const uint32_t word = dw[slot >> 1];
            // Byte e of the pair is byte m = (2·slot & 3) + e of the data word
            // and its colbyte is byte kc = (2·slot + e) & 3 of cbw; the
            // selector puts the colbyte in byte 0, the data byte in byte 1 and
            // zeros (the colbyte's sign, colbytes < 128) above.
            // An even slot uses bytes 0 and 1 of both words, an odd one 2 and 3.
            constexpr uint32_t E0 = 0x4 | (0 << 4) | (0xc << 8) | (0xc << 12);
            constexpr uint32_t E1 = 0x5 | (1 << 4) | (0xd << 8) | (0xd << 12);
            constexpr uint32_t O0 = 0x6 | (2 << 4) | (0xe << 8) | (0xe << 12);
            constexpr uint32_t O1 = 0x7 | (3 << 4) | (0xf << 8) | (0xf << 12);
            const uint32_t cw = cbw[slot >> 1];
            int32_t v[2];
            if (slot & 1) {
                v[0] = lds_tab<TB>(prmt<O0>(word, cw));
                v[1] = lds_tab<TB>(prmt<O1>(word, cw));
            } else {
                v[0] = lds_tab<TB>(prmt<E0>(word, cw));
                v[1] = lds_tab<TB>(prmt<E1>(word, cw));
            }
            if (tt & 1)
                acc1 += v[0] + v[1];
            else
                acc0 += v[0] + v[1];
        }
        const int32_t sum = acc0 + acc1 - (int32_t)(2 * kEntryBias) * GB;
        const int gl = (q + a_rot) & (NG - 1);  // group within the superchunk
        const int g = sc * NG + gl;             // group in the row
        const uint32_t nbits = (nw[q >> 1] >> (16 * (q & 1))) & 0xffffu;
        const float nrm = __half2float(__ushort_as_half((unsigned short)nbits));
        const float coef = __fmul_rn(nrm, steps[g]);
        wterms[gl * 32 + lane] = __fmul_rn(__int2float_rn(sum), coef);
    }
#pragma unroll
    for (int gl = 0; gl < NG; gl++) y = __fadd_rn(y, wterms[gl * 32 + lane]);
    return y;
}

template <int NG>
__device__ __forceinline__ void load_superchunk(const CqView &v, int sc, int R, bool valid, uint4 (&d)[4],
                                                uint32_t (&nw)[4]) {
    if (valid) {
        const uint8_t *base = v.idx + ((size_t)sc * 4 * v.ld + R) * 16;
#pragma unroll
        for (int i = 0; i < 4; i++) d[i] = __ldg(reinterpret_cast<const uint4 *>(base + (size_t)i * v.ld * 16));
        const __half *nb = v.nrm + ((size_t)sc * v.ld + R) * NG;
        if constexpr (NG == 8) {
            uint4 t4 = __ldg(reinterpret_cast<const uint4 *>(nb));
            nw[0] = t4.x; nw[1] = t4.y; nw[2] = t4.z; nw[3] = t4.w;
        } else if constexpr (NG == 4) {
            uint2 t2 = __ldg(reinterpret_cast<const uint2 *>(nb));
            nw[0] = t2.x; nw[1] = t2.y; nw[2] = 0; nw[3] = 0;
        } else if constexpr (NG == 2) {
            nw[0] = __ldg(reinterpret_cast<const uint32_t *>(nb)); nw[1] = 0; nw[2] = 0; nw[3] = 0;
        } else {
            nw[0] = __ldg(reinterpret_cast<const uint16_t *>(nb)); nw[1] = 0; nw[2] = 0; nw[3] = 0;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            d[i] = make_uint4(0, 0, 0, 0);
            nw[i] = 0;
        }
    }
}

// Threads of an instance: 512, or 384 for 8-byte groups with four
// superchunks a pass, whose rolling prefetch needs more than 128 registers
// (registers are shared per quarter-SM: three warps a quarter leave 168).
template <int GB, int NSC>
__host__ __device__ constexpr int stream_threads() { return GB == 8 && NSC == 4 ? 384 : kStreamThreads; }

// MA: the launch has several activations. The one-activation instances
// are compiled without the activation loop, which would otherwise keep its
// bounds live across the tile loop (the 4-bit, four-superchunk instance
// spilled with it).
template <int GB, int NR, int NSC, bool MA>  // group bytes; run capacity; most superchunks a pass holds (1, 2 or 4)
__global__ void __launch_bounds__(stream_threads<GB, NSC>(), 1)
    cq_lut_stream_kernel(const __grid_constant__ StreamParamsN<NR> p) {
    constexpr int NW = stream_threads<GB, NSC>() / 32;  // warps
    constexpr int P = GB / 2;    // byte pairs per group
    constexpr int NG = 32 / P;   // groups per 64-byte superchunk
    extern __shared__ __align__(16) unsigned char smem[];
    const CqShape &s = p.shape;
    // Small buffers from the start of dynamic shared memory, the byte tables
    // at shared-window address kTabAbs (the host sized the allocation for
    // the window offset the probe kernel measured).
    const uint32_t base = (uint32_t)__cvta_generic_to_shared(smem);
    uint16_t *nib = reinterpret_cast<uint16_t *>(smem);                    // kNibBytes
    float *terms = reinterpret_cast<float *>(smem + kNibBytes);            // [warps][NG][32]
    float *steps = terms + kStreamWarps * NG * 32;                         // [groups]
    float *invs = steps + s.groups;                                        // [groups]
    float *xs = invs + s.groups;                                           // [pad]
    uint16_t *tab = reinterpret_cast<uint16_t *>(smem + (kTabAbs - base));  // kTabBytes

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // This CTA's work: a contiguous share of the (activation, 32-row tile)
    // items, activation-major: for each activation it touches, it rotates
    // and tabulates the activation once and streams that activation's tiles.
    const long long T = p.total_tiles, W = T * p.acts;
    const long long w_begin = W * blockIdx.x / gridDim.x, w_end = W * (blockIdx.x + 1) / gridDim.x;
    if (base != p.smem_base) {
        // Not the layout the host sized: leave NaN, never a wrong number,
        // and record it in the error word (wc_device_status).
        // Activation by activation as below, with no division in the loop:
        // a 64-bit division inside this never-taken loop cost the 4-bit
        // one-activation instances 2 to 4 % of their speed.
        if (tid == 0 && p.err) atomicExch(p.err, 20);
        for (int a = MA ? (int)(w_begin / T) : 0; MA ? (long long)a * T < w_end : a < 1; a++) {
            const long long a0 = (long long)a * T;
            const int lo = (int)((w_begin > a0 ? w_begin : a0) - a0);
            const int hi = (int)((w_end < a0 + T ? w_end : a0 + T) - a0);
            for (int t = lo + warp; t < hi; t += NW) {
                const TileLoc L = tile_loc(p, t, find_run(p, t), a);
                const int r = L.r0 + lane;
                if (r < L.v.out) L.y[r] = __int_as_float(0x7fc00000);
            }
        }
        return;
    }
    float *wterms = terms + warp * NG * 32;
    const int npass = (s.row_bytes + kPassPositions - 1) / kPassPositions;

    if (w_begin >= w_end) return;
    // The first and last activation and the tile bounds within them, as
    // 32-bit values: fewer registers stay live across the tile loop than
    // with the 64-bit item bounds.
    const int act_first = MA ? (int)(w_begin / T) : 0, act_last = MA ? (int)((w_end - 1) / T) : 0;
    const int tb_first = (int)(w_begin - (long long)act_first * T);
    const int te_last = (int)(w_end - (long long)act_last * T);
    int tb_next = tb_first;
  for (int act = act_first; act <= act_last; act++) {
    const int t_begin = tb_next;
    const int t_end = MA && act < act_last ? p.total_tiles : te_last;
    tb_next = 0;
    const float *x = MA ? p.x + (size_t)act * s.in : p.x;
    // The previous activation's tables and steps are read until every warp
    // has finished its tiles.
    if (MA) __syncthreads();

    // Rolling prefetch: a warp's first tile of a pass is loaded into its
    // registers before the pass's tables are built (for pass 0 before the
    // rotation); afterwards, as soon as a superchunk's registers are
    // consumed, the same superchunk of the warp's next tile is loaded into
    // them, so a tile's worth of loads is in flight while the warp computes.
    uint4 d0[4], d1[4], d2[4], d3[4];
    uint32_t n0[4], n1[4], n2[4], n3[4];
    const bool has_tile = t_begin + warp < t_end;
    auto first_tile = [&](int sc0, int nsc_pass) {
        if (has_tile) {
            const TileLoc l0 = tile_loc(p, t_begin + warp, find_run(p, t_begin + warp), act);
            const bool v0 = l0.r0 + lane < l0.v.out;
            const int R0 = l0.v.row0 + l0.r0 + lane;
            load_superchunk<NG>(l0.v, sc0, R0, v0, d0, n0);
            if (NSC > 1 && nsc_pass > 1) load_superchunk<NG>(l0.v, sc0 + 1, R0, v0, d1, n1);
            if (NSC > 2 && nsc_pass > 2) load_superchunk<NG>(l0.v, sc0 + 2, R0, v0, d2, n2);
            if (NSC > 3 && nsc_pass > 3) load_superchunk<NG>(l0.v, sc0 + 3, R0, v0, d3, n3);
        }
    };
    first_tile(0, min(min(s.row_bytes, kPassPositions) / 64, NSC));

    rotate_and_bound(s, x, xs, steps, invs);

    for (int pass = 0; pass < npass; pass++) {
        const int j0 = pass * kPassPositions;
        const int npos = min(kPassPositions, s.row_bytes - j0);
        const int sc0 = j0 / 64, nsc_pass = min(npos / 64, NSC);  // npos / 64 <= NSC by the launch
        if (pass > 0) first_tile(sc0, nsc_pass);
        __syncthreads();
        build_pass_tables(s, xs, invs, j0, npos, nib, tab);

        int cached_off = -1;
        uint32_t cbw[16];  // colbyte(slot s, half e) at byte 2s+e: 4·o(s) + 2e
#pragma unroll
        for (int w = 0; w < 16; w++) cbw[w] = 0;
        int a_rot = 0;
        int k = -1;
        for (int t = t_begin + warp; t < t_end; t += NW) {
            k = run_from(p, t, k);
            const TileLoc loc = tile_loc(p, t, k, act);
            const CqView &v = loc.v;
            const int r = loc.r0 + lane;
            const bool valid = r < v.out;
            const int off = v.row0 & 31;

            if (off != cached_off) {
                cached_off = off;
                const int lam = (off + lane) & 31;
                const int a = lam / P, c = lam % P;
                a_rot = a;
#pragma unroll
                for (int w = 0; w < 16; w++) {
                    uint32_t word = 0;
#pragma unroll
                    for (int bb = 0; bb < 4; bb++) {
                        int slot = (4 * w + bb) >> 1, e = bb & 1;
                        int q = slot / P, tt = slot % P;
                        int o = P * ((q + a) % NG) + (tt + c) % P;
                        word |= (uint32_t)(4 * o + 2 * e) << (8 * bb);
                    }
                    cbw[w] = word;
                }
            }
            // This pass reads the partial sums from, and writes them to, the
            // output or the tile's row of p.part.
            float *yk = loc.y;
            float *const pk = p.part ? p.part + (size_t)t * 32 + lane : nullptr;
            float *const src = pk ? pk : yk + r;
            float *const dst = pk && pass + 1 < npass ? pk : yk + r;
            float y = 0.0f;
            if (pass > 0 && valid) y = *src;

            // The warp's next tile.
            const int tn = t + NW;
            const bool nxt = tn < t_end;
            int kn = k;
            TileLoc ln = loc;
            int Rn = 0;
            bool vn = false;
            if (nxt) {
                kn = run_from(p, tn, k);
                ln = tile_loc(p, tn, kn, act);
                Rn = ln.v.row0 + ln.r0 + lane;
                vn = ln.r0 + lane < ln.v.out;
            }
            y = superchunk<GB, 0>(d0, n0, cbw, steps, wterms, lane, a_rot, sc0, y);
            if (nxt) load_superchunk<NG>(ln.v, sc0, Rn, vn, d0, n0);
            if (NSC > 1 && nsc_pass > 1) {
                y = superchunk<GB, 1>(d1, n1, cbw, steps, wterms, lane, a_rot, sc0 + 1, y);
                if (nxt) load_superchunk<NG>(ln.v, sc0 + 1, Rn, vn, d1, n1);
            }
            if (NSC > 2 && nsc_pass > 2) {
                y = superchunk<GB, 2>(d2, n2, cbw, steps, wterms, lane, a_rot, sc0 + 2, y);
                if (nxt) load_superchunk<NG>(ln.v, sc0 + 2, Rn, vn, d2, n2);
            }
            if (NSC > 3 && nsc_pass > 3) {
                y = superchunk<GB, 3>(d3, n3, cbw, steps, wterms, lane, a_rot, sc0 + 3, y);
                if (nxt) load_superchunk<NG>(ln.v, sc0 + 3, Rn, vn, d3, n3);
            }
            if (valid) *dst = y;
            k = kn;
        }
    }
  }
}

__global__ void smem_base_probe_kernel(int *out) {
    extern __shared__ __align__(16) unsigned char smem[];
    *out = (int)__cvta_generic_to_shared(smem);
}

}  // namespace

// Where dynamic shared memory starts in a CTA's shared window (the stream
// kernel, like the probe, declares no static shared memory). Measured once
// per device.
int stream_smem_base() {
    static int cached[64];
    static bool init[64];
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    std::lock_guard<std::mutex> lock(mu);
    if (init[dev]) return cached[dev];
    int *d = nullptr, h = -1;
    if (cudaMalloc(&d, sizeof(int)) != cudaSuccess) return -1;
    smem_base_probe_kernel<<<1, 1, 16>>>(d);
    count_launch();
    if (cudaMemcpy(&h, d, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) h = -1;
    cudaFree(d);
    cached[dev] = h;
    init[dev] = true;
    return h;
}

static size_t stream_small_bytes(const CqShape &s) {
    int ng = 64 / s.gb;
    return (size_t)kNibBytes + sizeof(float) * ((size_t)kStreamWarps * ng * 32 + 2 * s.groups + s.pad);
}

int stream_passes(const CqShape &s) { return (s.row_bytes + kPassPositions - 1) / kPassPositions; }

bool stream_eligible(const CqShape &s) {
    return (s.gb == 8 || s.gb == 16 || s.gb == 32 || s.gb == 64) && s.row_bytes % 64 == 0 && s.row_bytes >= 64;
}

// Dynamic shared memory of a launch: the small buffers must end below the
// tables' absolute address, and the tables end kTabBytes above it.
size_t stream_smem_bytes(const CqShape &s) {
    int b = stream_smem_base();
    if (b < 0 || (size_t)b + stream_small_bytes(s) > kTabAbs) return (size_t)1 << 30;  // never fits
    return (size_t)kTabAbs + kTabBytes - (size_t)b;
}

template <int NR, int NSC>
static void (*stream_fn(int gb, bool ma))(StreamParamsN<NR>) {
    switch (gb) {
        case 8: return ma ? cq_lut_stream_kernel<8, NR, NSC, true> : cq_lut_stream_kernel<8, NR, NSC, false>;
        case 16: return ma ? cq_lut_stream_kernel<16, NR, NSC, true> : cq_lut_stream_kernel<16, NR, NSC, false>;
        case 32: return ma ? cq_lut_stream_kernel<32, NR, NSC, true> : cq_lut_stream_kernel<32, NR, NSC, false>;
        default: return ma ? cq_lut_stream_kernel<64, NR, NSC, true> : cq_lut_stream_kernel<64, NR, NSC, false>;
    }
}

template <int NR>
static cudaError_t launch_stream_n(const StreamParamsN<NR> &p, int ctas, cudaStream_t st) {
    size_t smem = stream_smem_bytes(p.shape);
    // Registers for as many superchunks as a pass holds.
    const int nsc = p.shape.row_bytes / 64;
    void (*fn)(StreamParamsN<NR>) =
        nsc <= 1   ? stream_fn<NR, 1>(p.shape.gb, p.acts > 1)
        : nsc == 2 ? stream_fn<NR, 2>(p.shape.gb, p.acts > 1)
                   : stream_fn<NR, 4>(p.shape.gb, p.acts > 1);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int threads = p.shape.gb == 8 && nsc >= 3 ? stream_threads<8, 4>() : kStreamThreads;
    fn<<<ctas, threads, smem, st>>>(p);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_stream(const StreamParams &p, int ctas, cudaStream_t st) {
    if (p.nruns > kSmallStreamRuns) return launch_stream_n(p, ctas, st);
    StreamParamsN<kSmallStreamRuns> q;
    q.shape = p.shape;
    q.x = p.x;
    q.acts = p.acts;
    q.nruns = p.nruns;
    q.total_tiles = p.total_tiles;
    q.smem_base = p.smem_base;
    q.part = p.part;
    q.err = p.err;
    for (int i = 0; i < kSmallStreamRuns; i++) q.runs[i] = i < p.nruns ? p.runs[i] : StreamRun{};
    return launch_stream_n(q, ctas, st);
}

}  // namespace wb
