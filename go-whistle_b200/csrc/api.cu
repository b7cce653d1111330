// api.cu — the C ABI of libwhistle_b200.so (include/whistle_b200.h).
//
// Host-side work only: validation with the reference's messages, the
// one-time device copy of a CQ tensor into the kernels' group-major layout,
// views, and launches. No CPU compute path exists here: every product runs
// on the GPU, and a missing GPU is an error status.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <cmath>
#include <mutex>
#include <memory>
#include <new>
#include <string>
#include <vector>

#include "common.cuh"
#include "cq_kernels.cuh"
#include "needle_kernels.cuh"

// ------------------------------------------------------------- errors ----

namespace wb {

static thread_local std::string g_last_error;

wc_status set_error(wc_status st, const std::string &msg) {
    g_last_error = msg;
    return st;
}

wc_status cuda_error(cudaError_t e, const char *what) {
    std::string m = std::string("cuda: ") + what + ": " + cudaGetErrorString(e);
    return set_error(e == cudaErrorMemoryAllocation ? WC_ERR_NOMEM : WC_ERR_CUDA, m);
}

}  // namespace wb

using namespace wb;

// --------------------------------------------------------- the matrix ----

// Device storage shared by a matrix and its views.
struct CqStorage {
    uint8_t *idx = nullptr;   // group-major layout (common.cuh CqView)
    __half *nrm = nullptr;
    uint8_t *sidx = nullptr;  // stream layout (cq_lut_stream.cu), or null
    __half *snrm = nullptr;
    size_t idx_bytes = 0, nrm_bytes = 0, sidx_bytes = 0, snrm_bytes = 0;
    float nrm_max = 0.0f;  // largest |norm| (the tensor-core image's scale)
    int device = 0;
    ~CqStorage() {
        int cur = 0;
        cudaGetDevice(&cur);
        if (cur != device) cudaSetDevice(device);
        if (idx) cudaFree(idx);
        if (nrm) cudaFree(nrm);
        if (sidx) cudaFree(sidx);
        if (snrm) cudaFree(snrm);
        if (cur != device) cudaSetDevice(cur);
    }
};

// A view's bf16 weight image for the tensor-core GEMM, built on first use.
struct TcImage {
    std::mutex mu;
    unsigned char *b = nullptr;
    size_t bytes = 0;
    float ws = 1.0f;  // 1 / the image's power-of-two scale
    int device = 0;
    ~TcImage() {
        if (!b) return;
        int cur = 0;
        cudaGetDevice(&cur);
        if (cur != device) cudaSetDevice(device);
        cudaFree(b);
        if (cur != device) cudaSetDevice(cur);
    }
};

struct wc_cq {
    std::shared_ptr<CqStorage> st;
    CqShape shape;
    int out = 0, row0 = 0, ld = 0;
    bool exact = false;
    std::shared_ptr<TcImage> tc = std::make_shared<TcImage>();  // per view, not shared with copies

    CqView view() const { return CqView{st->idx, st->nrm, out, row0, ld}; }
    CqView stream_view() const { return CqView{st->sidx, st->snrm, out, row0, ld}; }
    bool lut() const { return !exact && shape.gb <= kLutMaxGroupBytes; }
    bool streamable() const { return lut() && st->sidx != nullptr; }
};

// The stream layout of cq_lut_stream.cu: superchunks of 64 index bytes, each
// row's byte pairs permuted by its lane (row mod 32), norms in phase order.
static void stream_layout(const uint8_t *index, const uint8_t *norms, int out, int groups, int gb, int row_bytes,
                          std::vector<uint8_t> &sidx, std::vector<uint16_t> &snrm) {
    const int P = gb / 2, NG = 32 / P, nsc = row_bytes / 64;
    sidx.assign((size_t)out * row_bytes, 0);
    snrm.assign((size_t)nsc * out * NG, 0);
    for (int r = 0; r < out; r++) {
        const int lam = r & 31, a = lam / P, c = lam % P;
        const uint8_t *src = index + (size_t)r * row_bytes;
        for (int sc = 0; sc < nsc; sc++) {
            uint8_t chunk[64];
            for (int slot = 0; slot < 32; slot++) {
                int q = slot / P, t = slot % P;
                int o = P * ((q + a) % NG) + (t + c) % P;
                chunk[2 * slot] = src[64 * sc + 2 * o];
                chunk[2 * slot + 1] = src[64 * sc + 2 * o + 1];
            }
            for (int i = 0; i < 4; i++)
                memcpy(&sidx[(((size_t)sc * 4 + i) * out + r) * 16], chunk + 16 * i, 16);
            for (int q = 0; q < NG; q++) {
                int g = sc * NG + (q + a) % NG;
                const uint8_t *pn = norms + 2 * ((size_t)r * groups + g);
                snrm[((size_t)sc * out + r) * NG + q] = (uint16_t)(pn[0] | (pn[1] << 8));
            }
        }
    }
}

static const char *kVersion = "whistle_b200 0.1";
static std::atomic<uint64_t> g_launches{0};

void wb::count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

extern "C" uint64_t wc_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" size_t wc_last_error(char *buf, size_t len) {
    const std::string &m = g_last_error;
    if (buf && len > 0) {
        size_t n = m.size() < len - 1 ? m.size() : len - 1;
        memcpy(buf, m.data(), n);
        buf[n] = 0;
    }
    return m.size();
}

extern "C" const char *wc_version(void) { return kVersion; }

static wc_status check_device(const wc_cq *h) {
    int cur = 0;
    WB_CUDA(cudaGetDevice(&cur));
    if (cur != h->st->device)
        return set_error(WC_ERR_DEVICE, fmt("cq: matrix lives on device %d, device %d is current", h->st->device, cur));
    return WC_OK;
}

// Shared memory the kernels need for this shape, against the device limit.
static wc_status check_smem(const CqShape &s, bool lut) {
    int dev = 0, limit = 0;
    WB_CUDA(cudaGetDevice(&dev));
    WB_CUDA(cudaDeviceGetAttribute(&limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    size_t need = lut ? lut_smem_bytes(s) : exact_smem_bytes(s);
    if (need > (size_t)limit)
        return set_error(WC_ERR_UNSUPPORTED,
                         fmt("cq: [*, %d] %d-bit group %d needs %zu bytes of shared memory, the device has %d", s.in,
                             s.bits, s.group, need, limit));
    return WC_OK;
}

extern "C" wc_status wc_cq_create(const uint8_t *index, size_t index_len, const uint8_t *norms, size_t norms_len,
                                  const float *codebook, size_t codebook_len, int out, int in, int group, int bits,
                                  int width, wc_cq **h) {
    if (!h) return set_error(WC_ERR_INVALID, "cq: nil handle pointer");
    *h = nullptr;
    // internal/cq/matrix.go:61-73, in that order.
    if ((bits != 2 && bits != 4) || width != bits)
        return set_error(WC_ERR_UNSUPPORTED,
                         fmt("cq: %d-bit CQ (index width %d) not supported, only 2 and 4", bits, width));
    if (group < 8 || (group & (group - 1)) != 0)
        return set_error(WC_ERR_UNSUPPORTED, fmt("cq: group %d is not a power of two >= 8", group));
    if (out < 0 || in <= 0) return set_error(WC_ERR_UNSUPPORTED, fmt("cq: bad shape [%d, %d]", out, in));
    if (codebook_len != ((size_t)1 << bits))
        return set_error(WC_ERR_UNSUPPORTED, fmt("cq: %zu codebook levels for %d bits", codebook_len, bits));
    const int groups = (in + group - 1) / group;
    const int row_bytes = groups * group * width / 8;
    const size_t want_idx = (size_t)out * row_bytes, want_nrm = (size_t)2 * out * groups;
    if (index_len != want_idx || norms_len != want_nrm)
        return set_error(WC_ERR_UNSUPPORTED, fmt("cq: %zu index and %zu norm bytes for [%d, %d], want %zu and %zu",
                                                 index_len, norms_len, out, in, want_idx, want_nrm));
    if ((out > 0 && (!index || !norms)) || !codebook) return set_error(WC_ERR_INVALID, "cq: nil tensor data");

    std::unique_ptr<wc_cq> m(new (std::nothrow) wc_cq);
    if (!m) return set_error(WC_ERR_NOMEM, "cq: out of host memory");
    CqShape &s = m->shape;
    memset(&s, 0, sizeof s);
    s.in = in;
    s.group = group;
    s.bits = bits;
    s.groups = groups;
    s.gb = group * bits / 8;
    s.row_bytes = row_bytes;
    s.pad = groups * group;
    s.cb_max = 0.0f;
    for (int c = 0; c < (1 << bits); c++) {
        s.cb[c] = codebook[c];
        s.cb_max = std::fmax(s.cb_max, std::fabs(codebook[c]));  // matrix.go:87-89
    }
    s.lut_step = (float)(1.0 / ((double)kLutQ * std::sqrt((double)group)));  // lut.go:213
    s.inv_sqrt = (float)(1.0 / std::sqrt((double)group));                   // kernel.go:375
    m->out = out;
    m->ld = out;
    m->row0 = 0;

    wc_status st = check_smem(s, m->lut());
    if (st != WC_OK) return st;

    auto storage = std::make_shared<CqStorage>();
    WB_CUDA(cudaGetDevice(&storage->device));
    // Group-major relayout (common.cuh CqView), done once on the host.
    const int gb = s.gb;
    std::vector<uint8_t> idx((size_t)out * row_bytes);
    std::vector<uint16_t> nrm((size_t)out * groups);
    for (int r = 0; r < out; r++) {
        for (int g = 0; g < groups; g++) {
            memcpy(&idx[((size_t)g * out + r) * gb], index + (size_t)r * row_bytes + (size_t)g * gb, gb);
            const uint8_t *p = norms + 2 * ((size_t)r * groups + g);
            nrm[(size_t)g * out + r] = (uint16_t)(p[0] | (p[1] << 8));  // little-endian FP16
            __half_raw hr;
            hr.x = nrm[(size_t)g * out + r];
            const float nv = std::fabs(__half2float(__half(hr)));
            if (nv > storage->nrm_max) storage->nrm_max = nv;  // NaN never wins
        }
    }
    storage->idx_bytes = idx.size() > 0 ? idx.size() : 16;
    storage->nrm_bytes = nrm.size() > 0 ? 2 * nrm.size() : 16;
    WB_CUDA(cudaMalloc(&storage->idx, storage->idx_bytes));
    WB_CUDA(cudaMalloc(&storage->nrm, storage->nrm_bytes));
    if (!idx.empty()) WB_CUDA(cudaMemcpy(storage->idx, idx.data(), idx.size(), cudaMemcpyHostToDevice));
    if (!nrm.empty()) WB_CUDA(cudaMemcpy(storage->nrm, nrm.data(), 2 * nrm.size(), cudaMemcpyHostToDevice));
    if (out > 0 && m->lut() && stream_eligible(s)) {
        int dev = 0, limit = 0;
        WB_CUDA(cudaGetDevice(&dev));
        WB_CUDA(cudaDeviceGetAttribute(&limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        if (stream_smem_bytes(s) <= (size_t)limit) {
            std::vector<uint8_t> sidx;
            std::vector<uint16_t> snrm;
            stream_layout(index, norms, out, groups, gb, row_bytes, sidx, snrm);
            storage->sidx_bytes = sidx.size();
            storage->snrm_bytes = 2 * snrm.size();
            WB_CUDA(cudaMalloc(&storage->sidx, storage->sidx_bytes));
            WB_CUDA(cudaMalloc(&storage->snrm, storage->snrm_bytes));
            WB_CUDA(cudaMemcpy(storage->sidx, sidx.data(), sidx.size(), cudaMemcpyHostToDevice));
            WB_CUDA(cudaMemcpy(storage->snrm, snrm.data(), 2 * snrm.size(), cudaMemcpyHostToDevice));
        }
    }
    m->st = std::move(storage);
    *h = m.release();
    return WC_OK;
}

extern "C" wc_status wc_cq_rows(const wc_cq *h, int lo, int hi, wc_cq **view) {
    if (!h || !view) return set_error(WC_ERR_INVALID, "cq: nil matrix");
    *view = nullptr;
    if (lo < 0 || hi < lo || hi > h->out)  // matrix.go:134
        return set_error(WC_ERR_INVALID, fmt("cq: Rows(%d, %d) of %d rows", lo, hi, h->out));
    wc_cq *v = new (std::nothrow) wc_cq(*h);
    if (!v) return set_error(WC_ERR_NOMEM, "cq: out of host memory");
    v->out = hi - lo;
    v->row0 = h->row0 + lo;
    v->tc = std::make_shared<TcImage>();
    *view = v;
    return WC_OK;
}

extern "C" wc_status wc_cq_exact(const wc_cq *h, wc_cq **view) {
    if (!h || !view) return set_error(WC_ERR_INVALID, "cq: nil matrix");
    *view = nullptr;
    wc_status st = check_smem(h->shape, false);
    if (st != WC_OK) return st;
    wc_cq *v = new (std::nothrow) wc_cq(*h);
    if (!v) return set_error(WC_ERR_NOMEM, "cq: out of host memory");
    v->exact = true;
    v->tc = std::make_shared<TcImage>();
    *view = v;
    return WC_OK;
}

extern "C" void wc_cq_destroy(wc_cq *h) { delete h; }
extern "C" int wc_cq_out(const wc_cq *h) { return h ? h->out : 0; }
extern "C" int wc_cq_in(const wc_cq *h) { return h ? h->shape.in : 0; }
extern "C" int wc_cq_bits(const wc_cq *h) { return h ? h->shape.bits : 0; }
extern "C" size_t wc_cq_bytes(const wc_cq *h) {
    if (!h) return 0;
    size_t one = (size_t)h->out * h->shape.row_bytes + (size_t)2 * h->out * h->shape.groups;
    return (h->st->sidx ? 2 * one : one) + 4u * (1u << h->shape.bits);
}

// lut.go:206 sharesTables.
static bool shares_tables(const wc_cq *a, const wc_cq *b) {
    if (a->st == b->st) return true;  // views of one storage: one shape and codebook
    if (a->shape.in != b->shape.in || a->shape.group != b->shape.group || a->shape.bits != b->shape.bits ||
        a->shape.cb_max != b->shape.cb_max)
        return false;
    for (int c = 0; c < (1 << a->shape.bits); c++)
        if (a->shape.cb[c] != b->shape.cb[c]) return false;
    return true;
}

// Streaming kernel threshold: index bytes of one activation's products
// below which the per-tile kernel (no per-SM table build) answers faster.
#ifndef WB_STREAM_MIN_BYTES
#define WB_STREAM_MIN_BYTES (2u << 20)
#endif
static const size_t kStreamMinBytes = WB_STREAM_MIN_BYTES;

static int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    return n;
}

// Set while a host-slice call runs its kernels straight into the caller's
// page-locked outputs: a stream launch of several table passes then keeps
// its partial sums in `part` (grown on demand, one per calling thread), so
// each output is written once, by the last pass.
namespace {
struct HostDirect {
    bool on = false;
    float *part = nullptr;
    size_t n = 0;
    int device = -1;
    ~HostDirect() {
        if (part) cudaFree(part);
    }
    cudaError_t get(size_t floats, float **out) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (n < floats || device != dev) {
            if (part) cudaFree(part);
            part = nullptr;
            n = 0;
            if ((e = cudaMalloc(&part, floats * sizeof(float))) != cudaSuccess) return e;
            n = floats;
            device = dev;
        }
        *out = part;
        return cudaSuccess;
    }
};
thread_local HostDirect t_direct;
}  // namespace

static int *device_err_word();

// The streaming kernel for one activation, if every matrix has the stream
// layout and the products are large enough; returns false otherwise.
static bool try_stream(const wc_cq *const *ms, int n, const float *x, float *const *ys, int rows, cudaStream_t st,
                       wc_status *status) {
    if (rows != 1 || n == 0) return false;
    size_t total = 0;
    for (int k = 0; k < n; k++) {
        if (!ms[k]->streamable()) return false;
        total += (size_t)ms[k]->out * ms[k]->shape.row_bytes;
    }
    if (total < kStreamMinBytes) return false;
    const int sms = sm_count();
    *status = WC_OK;
    // Consecutive matrices that are views of one storage with equal Out, a
    // constant row step and evenly spaced outputs form one run (a stack of
    // calls on one weight tensor is a single run), so one launch carries
    // up to kMaxStreamRuns runs of any length.
    auto p = std::make_unique<StreamParams>();
    auto flush = [&]() -> bool {
        if (p->nruns == 0) return true;
        const StreamRun &l = p->runs[p->nruns - 1];
        p->total_tiles = l.tile0 + l.count * l.tpm;
        p->shape = ms[0]->shape;
        p->x = x;
        p->acts = 1;
        p->smem_base = stream_smem_base();
        p->part = nullptr;
        p->err = device_err_word();
        cudaError_t e = cudaSuccess;
        if (t_direct.on && stream_passes(p->shape) > 1) e = t_direct.get((size_t)p->total_tiles * 32, &p->part);
        const int ctas = p->total_tiles < sms ? p->total_tiles : sms;
        if (e == cudaSuccess) e = launch_stream(*p, ctas, st);
        p->nruns = 0;
        if (e != cudaSuccess) {
            *status = cuda_error(e, "cq stream kernel");
            return false;
        }
        return true;
    };
    p->nruns = 0;
    long long tiles = 0;
    for (int k = 0; k < n; k++) {
        const wc_cq *m = ms[k];
        if (m->out == 0) continue;
        const CqView sv = m->stream_view();
        const int tpm = (m->out + 31) / 32;
        if (p->nruns > 0) {
            StreamRun &r = p->runs[p->nruns - 1];
            const bool same = sv.idx == r.v.idx && sv.nrm == r.v.nrm && sv.ld == r.v.ld && sv.out == r.v.out;
            const int last_row0 = r.v.row0 + (r.count - 1) * r.row_step;
            const intptr_t last_y = (intptr_t)(r.y + (long long)(r.count - 1) * r.y_step);
            const intptr_t dy = (intptr_t)ys[k] - last_y;  // bytes; a whole number of floats
            const bool fits = tiles + tpm < (1LL << 30) && dy % (intptr_t)sizeof(float) == 0;
            const long long ystep = (long long)(dy / (intptr_t)sizeof(float));
            if (same && fits && r.count == 1) {
                r.row_step = sv.row0 - last_row0;
                r.y_step = ystep;
                r.count = 2;
                tiles += tpm;
                continue;
            }
            if (same && fits && sv.row0 - last_row0 == r.row_step && ystep == r.y_step) {
                r.count++;
                tiles += tpm;
                continue;
            }
        }
        if (p->nruns == kMaxStreamRuns || tiles + tpm >= (1LL << 30)) {
            if (!flush()) return true;
            tiles = 0;
        }
        StreamRun &r = p->runs[p->nruns++];
        r.v = sv;
        r.y = ys[k];
        r.y_step = 0;
        r.y_act = 0;
        r.row_step = 0;
        r.count = 1;
        r.tpm = tpm;
        r.tile0 = (int)tiles;
        tiles += tpm;
    }
    flush();
    return true;
}

// Activations from which a product of matrices with the stream layout runs
// on the streaming kernel over all of them (each CTA tabulates the
// activations its share of (activation, tile) items touches) instead of
// the cluster, per-activation or per-tile kernels. From 2 activations it is
// the fastest lut kernel on every measured shape (the 16384 x 512 head at
// 2 and 4 activations: 7.9 and 9.4 µs, against 38 and 73 µs on the
// cluster kernel, which tabulates per tile).
static const int kStreamActsMinRows = 2;

// Rows (all matrices together) from which the streaming kernel's byte
// tables (256 entries per index byte, rebuilt per activation) pay off
// against the per-activation kernel's nibble tables; below it (the mHC φ:
// 24 rows of 2048) the table build would dominate.
static const int kStreamActsMinOut = 128;

static bool try_stream_acts(const wc_cq *const *ms, int n, const float *x, float *const *ys, int rows,
                            cudaStream_t st, wc_status *status) {
    if (rows < kStreamActsMinRows || n == 0) return false;
    long long outs = 0;
    for (int k = 0; k < n; k++) {
        if (!ms[k]->streamable()) return false;
        outs += ms[k]->out;
    }
    if (outs < kStreamActsMinOut) return false;
    const int sms = sm_count();
    *status = WC_OK;
    for (int base = 0; base < n; base += kMaxStreamRuns) {
        const int cnt = n - base < kMaxStreamRuns ? n - base : kMaxStreamRuns;
        auto p = std::make_unique<StreamParams>();
        p->shape = ms[base]->shape;
        p->x = x;
        p->acts = rows;
        p->smem_base = stream_smem_base();
        p->part = nullptr;
        p->err = device_err_word();
        p->nruns = 0;
        long long tiles = 0;
        for (int k = 0; k < cnt; k++) {
            const wc_cq *m = ms[base + k];
            if (m->out == 0) continue;
            StreamRun &r = p->runs[p->nruns++];
            r.v = m->stream_view();
            r.y = ys[base + k];
            r.y_step = 0;
            r.y_act = m->out;  // outputs [rows][out]
            r.row_step = 0;
            r.count = 1;
            r.tpm = (m->out + 31) / 32;
            r.tile0 = (int)tiles;
            tiles += r.tpm;
        }
        if (p->nruns == 0) continue;
        p->total_tiles = (int)tiles;
        const long long work = tiles * (long long)rows;
        int ctas = work < sms ? (int)work : sms;
        // A CTA's share of the (activation, tile) items is the range
        // [W·b/ctas, W·(b+1)/ctas) of W = tiles·rows: with ctas a multiple
        // k·rows no range crosses an activation, so each CTA tabulates one
        // activation. Taken while it keeps three quarters of the SMs busy.
        if (rows <= sms) {
            long long k = sms / rows;
            if (k > tiles) k = tiles;
            if (4 * k * rows >= 3LL * sms) ctas = (int)(k * rows);
        }
        cudaError_t e = launch_stream(*p, ctas, st);
        if (e != cudaSuccess) {
            *status = cuda_error(e, "cq stream kernel (activations)");
            return true;
        }
    }
    return true;
}

// One lut launch sequence for matrices that share their tables.
// Activations up to which a product below the streaming threshold runs on
// the cluster kernel (groups split over the CTAs of a cluster) instead of
// the per-tile kernel (every CTA tabulates the whole activation).
static const int kSplitMaxRows = 4;

static bool try_split(const wc_cq *const *ms, int n, const float *x, float *const *ys, int rows, cudaStream_t st,
                      wc_status *status) {
    if (rows > kSplitMaxRows || n == 0 || !split_eligible(ms[0]->shape)) return false;
    int dev = 0, limit = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
        return false;
    if (split_smem_bytes(ms[0]->shape) > (size_t)limit) return false;
    *status = WC_OK;
    for (int base = 0; base < n; base += kMaxLaunchMats) {
        int cnt = n - base < kMaxLaunchMats ? n - base : kMaxLaunchMats;
        auto p = std::make_unique<LutParams>();
        p->shape = ms[base]->shape;
        p->x = x;
        p->tile_rows = 32;
        int tiles = 0, used = 0;
        for (int k = 0; k < cnt; k++) {
            const wc_cq *m = ms[base + k];
            if (m->out == 0) continue;
            p->views[used] = m->view();
            p->y[used] = ys[base + k];
            p->tile_start[used] = tiles;
            tiles += split_tiles(m->out);
            used++;
        }
        p->tile_start[used] = tiles;
        p->n = used;
        if (used == 0) continue;
        p->act0 = 0;
        cudaError_t e = launch_split(*p, tiles, rows, st);
        if (e != cudaSuccess) {
            *status = cuda_error(e, "cq split kernel");
            return true;
        }
    }
    return true;
}

// Activations from which a product of group-128 matrices runs on the
// per-activation kernel (cq_lut_acts.cu: tables built once per activation
// for all rows) instead of the per-tile kernel (tables rebuilt per tile).
static const int kActsMinRows = 8;

// The per-activation kernel, when every matrix's shape takes it.
static bool try_acts(const wc_cq *const *ms, int n, const float *x, float *const *ys, int rows, cudaStream_t st,
                     wc_status *status) {
    if (rows < kActsMinRows || !acts_eligible(ms[0]->shape)) return false;
    const int sms = sm_count();
    *status = WC_OK;
    for (int base = 0; base < n; base += kMaxActsMats) {
        const int cnt = n - base < kMaxActsMats ? n - base : kMaxActsMats;
        ActsParams p{};
        p.shape = ms[base]->shape;
        p.x = x;
        int total = 0;
        for (int k = 0; k < cnt; k++) {
            const wc_cq *m = ms[base + k];
            if (m->out == 0) continue;
            p.views[p.n] = m->view();
            p.y[p.n] = ys[base + k];
            p.row_start[p.n] = total;
            total += m->out;
            p.n++;
        }
        p.row_start[p.n] = total;
        p.total_rows = total;
        if (p.n == 0) continue;
        // Few activations: split the rows over more CTAs (each builds the
        // tables) until about two CTAs run per SM, keeping >= 64 rows each.
        int splits = 1;
        while (rows * splits < 2 * sms && total / (2 * splits) >= 64) splits *= 2;
        p.splits = splits;
        cudaError_t e = launch_lut_acts(p, rows, st);
        if (e != cudaSuccess) {
            *status = cuda_error(e, "cq lut kernel (per activation)");
            return true;
        }
    }
    return true;
}

static wc_status run_lut(const wc_cq *const *ms, int n, const float *x, float *const *ys, int rows,
                         cudaStream_t st) {
    wc_status sst;
    if (try_stream(ms, n, x, ys, rows, st, &sst)) return sst;
    if (try_stream_acts(ms, n, x, ys, rows, st, &sst)) return sst;
    if (try_split(ms, n, x, ys, rows, st, &sst)) return sst;
    if (try_acts(ms, n, x, ys, rows, st, &sst)) return sst;
    for (int base = 0; base < n; base += kMaxLaunchMats) {
        int cnt = n - base < kMaxLaunchMats ? n - base : kMaxLaunchMats;
        auto p = std::make_unique<LutParams>();
        p->shape = ms[base]->shape;
        p->x = x;
        // One activation: smaller tiles, so more CTAs share the latency.
        p->tile_rows = rows == 1 ? kTileRowsOne : kTileRows;
        int tiles = 0, used = 0;
        for (int k = 0; k < cnt; k++) {
            const wc_cq *m = ms[base + k];
            if (m->out == 0) continue;
            p->views[used] = m->view();
            p->y[used] = ys[base + k];
            p->tile_start[used] = tiles;
            tiles += (m->out + p->tile_rows - 1) / p->tile_rows;
            used++;
        }
        p->tile_start[used] = tiles;
        p->n = used;
        if (used == 0) continue;
        for (int a0 = 0; a0 < rows; a0 += 65535) {
            int acts = rows - a0 < 65535 ? rows - a0 : 65535;
            p->act0 = a0;
            cudaError_t e = launch_lut(*p, tiles, acts, st);
            if (e != cudaSuccess) return cuda_error(e, "cq lut kernel");
        }
    }
    return WC_OK;
}

extern "C" wc_status wc_cq_gemm(const wc_cq *h, const float *x, float *y, int rows, wc_stream stream) {
    if (!h) return set_error(WC_ERR_INVALID, "cq: nil matrix");
    if (rows < 0) return set_error(WC_ERR_INVALID, fmt("cq: GEMM of %d rows on [%d, %d]", rows, h->out, h->shape.in));
    if (rows == 0 || h->out == 0) return WC_OK;  // kernel.go:110
    wc_status st = check_device(h);
    if (st != WC_OK) return st;
    cudaStream_t s = (cudaStream_t)stream;
    if (h->lut()) return run_lut(&h, 1, x, &y, rows, s);
    cudaError_t e = launch_exact(h->shape, h->view(), x, y, rows, s);
    return e == cudaSuccess ? WC_OK : cuda_error(e, "cq exact kernel");
}

extern "C" wc_status wc_cq_gemms(const wc_cq *const *hs, int n, const float *x, float *const *ys, int rows,
                                 wc_stream stream) {
    if (n < 0 || (n > 0 && (!hs || !ys))) return set_error(WC_ERR_INVALID, "cq: GEMMs of a nil list");
    if (rows < 0) return set_error(WC_ERR_INVALID, fmt("cq: GEMMs of %d rows", rows));
    for (int k = 0; k < n; k++) {
        if (!hs[k]) return set_error(WC_ERR_INVALID, "cq: nil matrix");
        if (hs[k]->shape.in != hs[0]->shape.in)
            return set_error(WC_ERR_INVALID, fmt("cq: GEMMs mixes inputs of %d and %d", hs[0]->shape.in, hs[k]->shape.in));
    }
    if (rows == 0) return WC_OK;
    cudaStream_t s = (cudaStream_t)stream;
    // Matrices sharing the first lut matrix's tables go in one launch
    // (kernel.go:328-346); each other one runs its own GEMM. Either way each
    // output is the same bits as its own GEMM.
    const wc_cq *first = nullptr;
    std::vector<const wc_cq *> shared;
    std::vector<float *> sys;
    shared.reserve(n);
    sys.reserve(n);
    int cur = 0;
    WB_CUDA(cudaGetDevice(&cur));
    for (int k = 0; k < n; k++) {
        const wc_cq *m = hs[k];
        if (m->st->device != cur)
            return set_error(WC_ERR_DEVICE,
                             fmt("cq: matrix lives on device %d, device %d is current", m->st->device, cur));
        if (m->out == 0) continue;
        if (m->lut() && (!first || shares_tables(first, m))) {
            if (!first) first = m;
            shared.push_back(m);
            sys.push_back(ys[k]);
            continue;
        }
        wc_status st = wc_cq_gemm(m, x, ys[k], rows, stream);
        if (st != WC_OK) return st;
    }
    if (!shared.empty()) return run_lut(shared.data(), (int)shared.size(), x, sys.data(), rows, s);
    return WC_OK;
}

// Device buffers for the host-slice entry points: grown on demand, one set
// per calling thread, freed at thread exit.
namespace {
// Slots: 0 and 1 the inputs and outputs of host calls, 2 the quantiser's
// scales, 3 the tensor cores' rotated image, 4 the host attention's arrays.
struct HostScratch {
    static const int kSlots = 5;
    void *p[kSlots] = {};
    size_t n[kSlots] = {};
    int device[kSlots] = {-1, -1, -1, -1, -1};
    ~HostScratch() {
        for (int i = 0; i < kSlots; i++)
            if (p[i]) cudaFree(p[i]);
    }
    cudaError_t get(int i, size_t bytes, void **out) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (n[i] < bytes || device[i] != dev) {
            if (p[i]) cudaFree(p[i]);
            p[i] = nullptr;
            n[i] = 0;
            e = cudaMalloc(&p[i], bytes < 256 ? 256 : bytes);
            if (e != cudaSuccess) return e;
            n[i] = bytes;
            device[i] = dev;
        }
        *out = p[i];
        return cudaSuccess;
    }
};
thread_local HostScratch t_scratch;
}  // namespace

extern "C" wc_status wc_cq_gemm_host(const wc_cq *h, const float *x, size_t x_len, float *y, size_t y_len, int rows) {
    if (!h) return set_error(WC_ERR_INVALID, "cq: nil matrix");
    const int out = h->out, in = h->shape.in;
    if (rows < 0 || x_len != (size_t)rows * in || y_len != (size_t)rows * out)  // kernel.go:105-107
        return set_error(WC_ERR_INVALID, fmt("cq: GEMM(len %zu, len %zu, %d rows) on [%d, %d]", y_len, x_len, rows, out, in));
    if (rows == 0 || out == 0) return WC_OK;
    return wc_cq_gemms_host(&h, 1, x, x_len, &y, &y_len, rows);
}

// Most chunks one host GEMMs call is split into.
#ifndef WB_HOST_CHUNKS
#define WB_HOST_CHUNKS 8
#endif

// Streams and events of the host-slice entry points, one set per calling
// thread: kernels run on `comp`, device-to-host copies on `copy`, so the copy
// of one chunk of outputs overlaps the kernels of the next chunk.
namespace {
struct HostPipe {
    static const int kChunks = WB_HOST_CHUNKS;
    cudaStream_t comp = nullptr, copy = nullptr;
    cudaEvent_t ev[kChunks] = {};
    int device = -1;
    void release() {
        for (int i = 0; i < kChunks; i++)
            if (ev[i]) cudaEventDestroy(ev[i]);
        if (comp) cudaStreamDestroy(comp);
        if (copy) cudaStreamDestroy(copy);
        comp = copy = nullptr;
        for (int i = 0; i < kChunks; i++) ev[i] = nullptr;
        device = -1;
    }
    ~HostPipe() { release(); }
    cudaError_t get() {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (device == dev) return cudaSuccess;
        release();
        if ((e = cudaStreamCreateWithFlags(&comp, cudaStreamNonBlocking)) != cudaSuccess) return e;
        if ((e = cudaStreamCreateWithFlags(&copy, cudaStreamNonBlocking)) != cudaSuccess) return e;
        for (int i = 0; i < kChunks; i++)
            if ((e = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming)) != cudaSuccess) return e;
        device = dev;
        return cudaSuccess;
    }
};
thread_local HostPipe t_pipe;
}  // namespace

// Output bytes per chunk below which a host GEMMs call is not split: one
// chunk's copy then costs about as much as a launch.
#ifndef WB_HOST_CHUNK_MIN_BYTES
#define WB_HOST_CHUNK_MIN_BYTES (1u << 20)
#endif
static const size_t kHostChunkMinBytes = WB_HOST_CHUNK_MIN_BYTES;
// Growth of the chunks' output bytes: about the kernels' output rate over
// the copies' (80 against 54 GB/s for the streaming kernel).
#ifndef WB_HOST_CHUNK_GROWTH
#define WB_HOST_CHUNK_GROWTH 1.4
#endif
static const double kHostChunkGrowth = WB_HOST_CHUNK_GROWTH;

// Output bytes of a host GEMMs call up to which outputs in mapped
// page-locked memory are written by the kernels themselves. Above it the
// chunked copies win: the copy engines move large blocks over PCIe faster
// than the kernels' 128-byte stores, and the first chunk's kernels are then
// a small part of the call.
#ifndef WB_HOST_DIRECT_MAX_BYTES
#define WB_HOST_DIRECT_MAX_BYTES (32u << 20)
#endif
static const size_t kHostDirectMaxBytes = WB_HOST_DIRECT_MAX_BYTES;

// The device address of page-locked host memory at p, if the current device
// can address it.
static bool host_mapped(const void *p, void **dev) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (a.type != cudaMemoryTypeHost || !a.devicePointer) return false;
    *dev = a.devicePointer;
    return true;
}

// Device addresses of the outputs when every one lies in page-locked host
// memory the device can address (each run of contiguous outputs checked at
// both ends); false otherwise.
static bool mapped_outputs(float *const *ys, const size_t *y_lens, int n, std::vector<float *> &dys) {
    dys.assign(n, nullptr);
    for (int k = 0; k < n;) {
        size_t len = y_lens[k];
        int j = k + 1;
        while (j < n && ys[j - 1] + y_lens[j - 1] == ys[j]) len += y_lens[j++];
        if (len) {
            void *d0 = nullptr, *d1 = nullptr;
            if (!host_mapped(ys[k], &d0) || !host_mapped(ys[k] + len - 1, &d1) ||
                (float *)d1 - (float *)d0 != (ptrdiff_t)(len - 1))
                return false;
            for (int i = k; i < j; i++) dys[i] = (float *)d0 + (ys[i] - ys[k]);
        }
        k = j;
    }
    return true;
}

// Outputs in mapped page-locked memory: the kernels store the results
// there themselves, so they cross PCIe once, while the products run.
static wc_status gemms_host_direct(const wc_cq *const *hs, int n, const float *x, size_t x_len,
                                   const std::vector<float *> &dys, int rows) {
    void *dx = nullptr;
    WB_CUDA(t_scratch.get(0, x_len * sizeof(float), &dx));
    wc_status st = WC_OK;
    cudaError_t e = cudaMemcpyAsync(dx, x, x_len * sizeof(float), cudaMemcpyHostToDevice, t_pipe.comp);
    if (e != cudaSuccess) st = cuda_error(e, "cq GEMMs host copy");
    if (st == WC_OK) {
        t_direct.on = true;
        st = wc_cq_gemms(hs, n, (const float *)dx, dys.data(), rows, (wc_stream)t_pipe.comp);
        t_direct.on = false;
    }
    // Nothing stays in flight into the caller's memory after return.
    e = cudaStreamSynchronize(t_pipe.comp);
    if (st != WC_OK) return st;
    if (e != cudaSuccess) return cuda_error(e, "cq GEMMs host kernels");
    return WC_OK;
}

extern "C" wc_status wc_cq_gemms_host(const wc_cq *const *hs, int n, const float *x, size_t x_len, float *const *ys,
                                      const size_t *y_lens, int rows) {
    if (n < 0 || (n > 0 && (!hs || !ys || !y_lens))) return set_error(WC_ERR_INVALID, "cq: GEMMs of a nil list");
    for (int k = 0; k < n; k++) {  // kernel.go:330-333
        if (!hs[k]) return set_error(WC_ERR_INVALID, "cq: nil matrix");
        int out = hs[k]->out, in = hs[k]->shape.in;
        if (rows < 0 || x_len != (size_t)rows * in || y_lens[k] != (size_t)rows * out)
            return set_error(WC_ERR_INVALID,
                             fmt("cq: GEMMs(len %zu, len %zu, %d rows) on [%d, %d]", y_lens[k], x_len, rows, out, in));
    }
    if (rows == 0 || n == 0) return WC_OK;
    WB_CUDA(t_pipe.get());
    size_t total = 0;
    for (int k = 0; k < n; k++) total += y_lens[k];
    if (total * sizeof(float) <= kHostDirectMaxBytes) {
        std::vector<float *> direct;
        if (mapped_outputs(ys, y_lens, n, direct)) return gemms_host_direct(hs, n, x, x_len, direct, rows);
    }
    void *dx = nullptr, *dy = nullptr;
    WB_CUDA(t_scratch.get(0, x_len * sizeof(float), &dx));
    WB_CUDA(t_scratch.get(1, (total ? total : 1) * sizeof(float), &dy));
    std::vector<float *> dys(n);
    size_t off = 0;
    for (int k = 0; k < n; k++) {
        dys[k] = (float *)dy + off;
        off += y_lens[k];
    }
    // Chunks of whole matrices whose output bytes grow by kHostChunkGrowth
    // from one chunk to the next: the first is small, so the link starts
    // copying early, and each later chunk's kernels (faster per byte than
    // the copy) finish before the copy ahead of them does. Every chunk's
    // kernels are queued before any copy, so a copy into pageable memory
    // (which returns only once it is done) never holds back the next
    // chunk's kernels.
    const size_t out_bytes = total * sizeof(float);
    int chunks = (int)(out_bytes / kHostChunkMinBytes);
    chunks = chunks < 1 ? 1 : chunks > HostPipe::kChunks ? HostPipe::kChunks : chunks;
    double wsum = 0.0, w = 1.0;
    for (int c = 0; c < chunks; c++, w *= kHostChunkGrowth) wsum += w;
    int bounds[HostPipe::kChunks + 1];
    int nb = 0;
    bounds[0] = 0;
    size_t acc = 0;
    double target = (double)total / wsum, wc = 1.0;  // cumulative output floats at the end of chunk nb
    for (int k = 0; k < n; k++) {
        acc += y_lens[k];
        if (((double)acc >= target && nb + 1 < chunks) || k == n - 1) {
            bounds[++nb] = k + 1;
            wc *= kHostChunkGrowth;
            target += (double)total * wc / wsum;
        }
    }
    wc_status st = WC_OK;
    cudaError_t e = cudaMemcpyAsync(dx, x, x_len * sizeof(float), cudaMemcpyHostToDevice, t_pipe.comp);
    int issued = 0;
    if (e != cudaSuccess) st = cuda_error(e, "cq GEMMs host copy");
    for (int c = 0; c < nb && st == WC_OK; c++) {
        st = wc_cq_gemms(hs + bounds[c], bounds[c + 1] - bounds[c], (const float *)dx, dys.data() + bounds[c], rows,
                         (wc_stream)t_pipe.comp);
        if (st != WC_OK) break;
        if ((e = cudaEventRecord(t_pipe.ev[c], t_pipe.comp)) != cudaSuccess) {
            st = cuda_error(e, "cq GEMMs host pipeline");
            break;
        }
        issued = c + 1;
    }
    // Copies of the chunks whose kernels were queued; contiguous outputs
    // (host and device) go in one copy.
    for (int c = 0; c < issued && st == WC_OK; c++) {
        if ((e = cudaStreamWaitEvent(t_pipe.copy, t_pipe.ev[c], 0)) != cudaSuccess) {
            st = cuda_error(e, "cq GEMMs host pipeline");
            break;
        }
        for (int k = bounds[c]; k < bounds[c + 1] && st == WC_OK;) {
            size_t len = y_lens[k];
            int j = k + 1;
            while (j < bounds[c + 1] && ys[j - 1] + y_lens[j - 1] == ys[j]) len += y_lens[j++];
            if (len && (e = cudaMemcpyAsync(ys[k], dys[k], len * sizeof(float), cudaMemcpyDeviceToHost,
                                            t_pipe.copy)) != cudaSuccess)
                st = cuda_error(e, "cq GEMMs host copy");
            k = j;
        }
    }
    // Nothing stays in flight into the caller's memory after return.
    cudaError_t e1 = cudaStreamSynchronize(t_pipe.copy);
    cudaError_t e2 = cudaStreamSynchronize(t_pipe.comp);
    if (st != WC_OK) return st;
    if (e1 != cudaSuccess) return cuda_error(e1, "cq GEMMs host copy");
    if (e2 != cudaSuccess) return cuda_error(e2, "cq GEMMs host kernels");
    return WC_OK;
}

extern "C" wc_status wc_cq_row(const wc_cq *h, int r, float *dst, wc_stream stream) {
    if (!h) return set_error(WC_ERR_INVALID, "cq: nil matrix");
    if (r < 0 || r >= h->out)
        return set_error(WC_ERR_INVALID, fmt("cq: Row(len %d, %d) of [%d, %d]", h->shape.in, r, h->out, h->shape.in));
    wc_status st = check_device(h);
    if (st != WC_OK) return st;
    cudaError_t e = launch_row(h->shape, h->view(), nullptr, r, 1, dst, nullptr, (cudaStream_t)stream);
    return e == cudaSuccess ? WC_OK : cuda_error(e, "cq row kernel");
}

extern "C" wc_status wc_cq_row_gather(const wc_cq *h, const int32_t *rows, int n, float *dst, int32_t *bad,
                                      wc_stream stream) {
    if (!h) return set_error(WC_ERR_INVALID, "cq: nil matrix");
    if (n < 0 || (n > 0 && (!rows || !dst))) return set_error(WC_ERR_INVALID, "cq: Row gather of a nil list");
    if (n == 0) return WC_OK;
    wc_status st = check_device(h);
    if (st != WC_OK) return st;
    cudaError_t e = launch_row(h->shape, h->view(), rows, 0, n, dst, bad, (cudaStream_t)stream);
    return e == cudaSuccess ? WC_OK : cuda_error(e, "cq row kernel");
}

extern "C" wc_status wc_cq_row_host(const wc_cq *h, int r, float *dst, size_t dst_len) {
    if (!h) return set_error(WC_ERR_INVALID, "cq: nil matrix");
    if (r < 0 || r >= h->out || dst_len != (size_t)h->shape.in)  // matrix.go:162-164
        return set_error(WC_ERR_INVALID, fmt("cq: Row(len %zu, %d) of [%d, %d]", dst_len, r, h->out, h->shape.in));
    void *d = nullptr;
    WB_CUDA(t_scratch.get(1, dst_len * sizeof(float), &d));
    wc_status st = wc_cq_row(h, r, (float *)d, nullptr);
    if (st != WC_OK) return st;
    WB_CUDA(cudaMemcpy(dst, d, dst_len * sizeof(float), cudaMemcpyDeviceToHost));
    return WC_OK;
}

// ------------------------------------------------------- tensor cores ----

// The per-device error word of the kernels' bounded waits.
static int *device_err_word() {
    static int *words[64];
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!words[dev]) {
        if (cudaMalloc(&words[dev], sizeof(int)) != cudaSuccess) return nullptr;
        if (cudaMemset(words[dev], 0, sizeof(int)) != cudaSuccess) return nullptr;
    }
    return words[dev];
}

extern "C" wc_status wc_device_status(int *code) {
    if (!code) return set_error(WC_ERR_INVALID, "nil code pointer");
    *code = 0;
    WB_CUDA(cudaDeviceSynchronize());
    int *w = device_err_word();
    if (!w) return set_error(WC_ERR_NOMEM, "cuda: error word");
    WB_CUDA(cudaMemcpy(code, w, sizeof(int), cudaMemcpyDeviceToHost));
    WB_CUDA(cudaMemset(w, 0, sizeof(int)));
    // The no-allocation GEMM's own word (its calls with err = NULL): the
    // first code recorded on either word is reported, and both are cleared.
    if (int *nw = noalloc_err_word()) {
        int c = 0;
        WB_CUDA(cudaMemcpy(&c, nw, sizeof(int), cudaMemcpyDeviceToHost));
        WB_CUDA(cudaMemset(nw, 0, sizeof(int)));
        if (*code == 0) *code = c;
    }
    return WC_OK;
}

static wc_status tc_supported(const wc_cq *h) {
    if (h->shape.group > 256)
        return set_error(WC_ERR_UNSUPPORTED, fmt("cq: tensor-core GEMM of group %d (at most 256)", h->shape.group));
    if (tc_kchunks(h->shape) > 64)
        return set_error(WC_ERR_UNSUPPORTED, fmt("cq: tensor-core GEMM of %d input columns (at most 4096)", h->shape.in));
    int dev = 0, limit = 0;
    WB_CUDA(cudaGetDevice(&dev));
    WB_CUDA(cudaDeviceGetAttribute(&limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    if (tc_smem_bytes() > (size_t)limit) return set_error(WC_ERR_UNSUPPORTED, "cq: tensor-core GEMM shared memory");
    return WC_OK;
}

extern "C" wc_status wc_cq_prepare_tc(const wc_cq *h) {
    if (!h) return set_error(WC_ERR_INVALID, "cq: nil matrix");
    wc_status st = check_device(h);
    if (st != WC_OK) return st;
    if ((st = tc_supported(h)) != WC_OK) return st;
    std::lock_guard<std::mutex> lock(h->tc->mu);
    if (h->tc->b || h->out == 0) return WC_OK;
    const int kchunks = tc_kchunks(h->shape);
    const size_t bytes = tc_b_bytes(h->out, kchunks);
    unsigned char *b = nullptr;
    // The image's power-of-two scale: its largest |ŵ| = max|cb|·max|n|/√G
    // times wsc lies in [2^13, 2^14), well inside fp16's range.
    const double wmax = (double)h->shape.cb_max * (double)h->st->nrm_max * (double)h->shape.inv_sqrt;
    int ew = 0;
    if (wmax > 0.0 && std::isfinite(wmax)) {
        int k = 0;
        std::frexp(wmax, &k);  // wmax < 2^k
        ew = std::min(120, std::max(-120, 14 - k));
    }
    const float wsc = std::ldexp(1.0f, ew);
    WB_CUDA(cudaMalloc(&b, bytes));
    cudaError_t e = launch_dequant_f16(h->shape, h->view(), wsc, b, nullptr);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(b);
        return cuda_error(e, "cq dequant kernel");
    }
    h->tc->b = b;
    h->tc->bytes = bytes;
    h->tc->ws = std::ldexp(1.0f, -ew);
    WB_CUDA(cudaGetDevice(&h->tc->device));
    return WC_OK;
}

// Where WC_GEMM_AUTO takes the tensor cores. The tensor-core call costs a
// near-constant 8-11 µs up to 256 rows (rotation, then one tile wave); the
// lut path's time grows with activations x output rows. Measured on B200,
// L2-warm weights, µs per call (lut / tensor cores):
//   qkvg 1120 x 512 CQ2 G128   64 rows 8.4 / 9.4    96 rows 12.6 / 9.9
//   2048 x 512 CQ4 G32         24 rows 8.4 / 8.5    32 rows 9.2 / 8.7
//   16384 x 512 CQ4 G32         2 rows 7.9 / 8.6     4 rows 9.4 / 8.6
// so the tensor cores once activations x output rows (all matrices of the
// call) reach 65,536, from 2 activations.
static const int kTcAutoMinRows = 2;
static const long long kTcAutoWork = 65536;
// Rows from which the tensor-core path uses the persistent kernel.
static const int kTcPersistRows = 1024;

// Tensor-core products of matrices that read the same x (same In): one
// rotation into the x̂ image per group size G, then one grouped launch per
// kMaxTcMats matrices of that G. The image lives in the calling thread's
// scratch, so one thread's calls must not overlap on the GPU (one stream
// per thread, as the header states).
static wc_status run_tc(const wc_cq *const *ms, int n, const float *x, float *const *ys, int rows, cudaStream_t s,
                        void *ext = nullptr, size_t ext_bytes = 0, bool stall = false) {
    for (int k = 0; k < n; k++) {
        wc_status st = wc_cq_prepare_tc(ms[k]);
        if (st != WC_OK) return st;
    }
    int *err = device_err_word();
    if (!err) return set_error(WC_ERR_NOMEM, "cuda: error word");
    std::vector<char> done(n, 0);
    for (int i = 0; i < n; i++) {
        if (done[i] || ms[i]->out == 0) continue;
        const CqShape &sh = ms[i]->shape;
        const int kchunks = tc_kchunks(sh);
        void *a = ext;
        if (ext) {
            if (tc_a_bytes(rows, kchunks) > ext_bytes) return set_error(WC_ERR_INVALID, "cq: tensor-core buffer too small");
        } else {
            WB_CUDA(t_scratch.get(3, tc_a_bytes(rows, kchunks), &a));
        }
        cudaError_t e = launch_rotate_f16(sh, x, rows, (unsigned char *)a, s);
        if (e != cudaSuccess) return cuda_error(e, "cq rotate kernel");
        TcParams p{};
        p.a = (const unsigned char *)a;
        p.rs = reinterpret_cast<const float *>((const unsigned char *)a + tc_a_image_bytes(rows, kchunks));
        p.m = rows;
        p.kchunks = kchunks;
        p.err = err;
        if (stall) {
            p.stall = 1;
            p.spin = 1u << 14;
        }
        // Many rows: the persistent kernel (256-row weight tiles, two TMEM
        // accumulators); few: one 128 x 128 tile per CTA.
        const bool persistent = rows >= kTcPersistRows;
        const int tile_n = persistent ? 256 : 128;
        auto launch = [&]() { return persistent ? launch_gemm_tc_persistent(p, s) : launch_gemm_tc(p, s); };
        int tiles = 0;
        for (int j = i; j < n; j++) {
            const wc_cq *m = ms[j];
            if (done[j] || m->out == 0 || m->shape.group != sh.group || m->shape.pad != sh.pad) continue;
            done[j] = 1;
            TcMat &t = p.mats[p.nmats++];
            {
                std::lock_guard<std::mutex> lock(m->tc->mu);
                t.b = m->tc->b;
                t.ws = m->tc->ws;
            }
            t.y = ys[j];
            t.n = m->out;
            t.ldy = m->out;
            t.tile0 = tiles;
            tiles += (m->out + tile_n - 1) / tile_n;
            if (p.nmats == kMaxTcMats) {
                // Full: launch, and start the next group of matrices on the
                // same image (a later launch only reads it).
                e = launch();
                if (e != cudaSuccess) return cuda_error(e, "cq tensor-core kernel");
                p.nmats = 0;
                tiles = 0;
            }
        }
        if (p.nmats > 0) {
            e = launch();
            if (e != cudaSuccess) return cuda_error(e, "cq tensor-core kernel");
        }
    }
    return WC_OK;
}

static bool use_tc(int rows, int flags, long long outs) {
    if (flags & WC_GEMM_TENSOR_CORES) return true;
    if (!(flags & WC_GEMM_AUTO)) return false;
    return rows >= kTcAutoMinRows && (long long)rows * outs >= kTcAutoWork;
}

extern "C" wc_status wc_cq_gemm_ex(const wc_cq *h, const float *x, float *y, int rows, int flags, wc_stream stream) {
    if (!use_tc(rows, flags, h ? h->out : 0)) return wc_cq_gemm(h, x, y, rows, stream);
    if (!h) return set_error(WC_ERR_INVALID, "cq: nil matrix");
    if (rows < 0) return set_error(WC_ERR_INVALID, fmt("cq: GEMM of %d rows on [%d, %d]", rows, h->out, h->shape.in));
    if (rows == 0 || h->out == 0) return WC_OK;
    wc_status st = check_device(h);
    if (st != WC_OK) return st;
    return run_tc(&h, 1, x, &y, rows, (cudaStream_t)stream);
}

// Test entry point: one tensor-core GEMM whose producer issues no copies,
// so that the kernel's bounded waits run out with nothing in flight (the
// kernel records its error code, frees its TMEM and returns; y is left
// undefined). The code is read by wc_device_status.
extern "C" wc_status wc_testing_gemm_tc_stall(const wc_cq *h, const float *x, float *y, int rows, wc_stream stream) {
    if (!h) return set_error(WC_ERR_INVALID, "cq: nil matrix");
    if (rows <= 0 || h->out == 0) return set_error(WC_ERR_INVALID, "cq: stall test of an empty product");
    wc_status st = check_device(h);
    if (st != WC_OK) return st;
    return run_tc(&h, 1, x, &y, rows, (cudaStream_t)stream, nullptr, 0, true);
}

extern "C" wc_status wc_cq_gemms_ex(const wc_cq *const *hs, int n, const float *x, float *const *ys, int rows,
                                    int flags, wc_stream stream) {
    long long outs = 0;
    for (int k = 0; hs && k < n; k++) outs += hs[k] ? hs[k]->out : 0;
    if (!use_tc(rows, flags, outs)) return wc_cq_gemms(hs, n, x, ys, rows, stream);
    if (n < 0 || (n > 0 && (!hs || !ys))) return set_error(WC_ERR_INVALID, "cq: GEMMs of a nil list");
    if (rows < 0) return set_error(WC_ERR_INVALID, fmt("cq: GEMMs of %d rows", rows));
    for (int k = 0; k < n; k++) {
        if (!hs[k]) return set_error(WC_ERR_INVALID, "cq: nil matrix");
        if (hs[k]->shape.in != hs[0]->shape.in)
            return set_error(WC_ERR_INVALID, fmt("cq: GEMMs mixes inputs of %d and %d", hs[0]->shape.in, hs[k]->shape.in));
        wc_status st = check_device(hs[k]);
        if (st != WC_OK) return st;
    }
    if (rows == 0 || n == 0) return WC_OK;
    return run_tc(hs, n, x, ys, rows, (cudaStream_t)stream);
}

namespace wb {
// GEMMs on device memory for the library's own callers (the decoder): the
// bit-exact lut kernels, or the tensor cores with the rotated image in the
// caller's buffer, so that a captured graph never points at a per-thread
// scratch that a later call could grow and free.
wc_status gemms_device(const wc_cq *const *ms, int n, const float *x, float *const *ys, int rows, bool tc,
                       void *tc_buf, size_t tc_bytes, cudaStream_t st) {
    if (rows == 0 || n == 0) return WC_OK;
    if (!tc) return wc_cq_gemms(ms, n, x, ys, rows, st);
    return run_tc(ms, n, x, ys, rows, st, tc_buf, tc_bytes);
}
int *err_word() { return device_err_word(); }
bool cq_internal(const wc_cq *h, CqShape *s, CqView *v) {
    if (!h) return false;
    if (s) *s = h->shape;
    if (v) *v = h->view();
    return true;
}
}  // namespace wb

// Tensor-core GEMM without any allocation: see whistle_b200.h.
extern "C" wc_status wc_cq_gemm_tc_noalloc(const wc_cq *h, const float *x, float *y, int rows, int *err,
                                           wc_stream stream) {
    if (!h) return set_error(WC_ERR_INVALID, "cq: nil matrix");
    if (rows < 0) return set_error(WC_ERR_INVALID, fmt("cq: GEMM of %d rows on [%d, %d]", rows, h->out, h->shape.in));
    if (rows == 0 || h->out == 0) return WC_OK;
    wc_status st = check_device(h);
    if (st != WC_OK) return st;
    if ((st = tc_supported(h)) != WC_OK) return st;
    const int kchunks = tc_kchunks(h->shape);
    const size_t need = tc_a_bytes(rows, kchunks), have = noalloc_scratch_bytes();
    if (need > have) {
        int most = 0;  // the most rows (a multiple of 128) whose image and scales fit
        while (tc_a_bytes(most + 128, kchunks) <= have) most += 128;
        return set_error(WC_ERR_INVALID,
                         fmt("cq: %d rows of %d columns need %zu bytes of scratch; the no-allocation GEMM has %zu "
                             "(at most %d rows at this width)",
                             rows, kchunks * 64, need, have, most));
    }
    const unsigned char *wimg = nullptr;
    float ws = 1.0f;
    {
        std::lock_guard<std::mutex> lock(h->tc->mu);
        wimg = h->tc->b;
        ws = h->tc->ws;
    }
    if (!wimg)
        return set_error(WC_ERR_INVALID,
                         "cq: matrix has no tensor-core weight image: call wc_cq_prepare_tc at load time first");
    cudaError_t e =
        gemm_tc_noalloc(h->shape, wimg, ws, x, y, rows, h->out, err, rows >= kTcPersistRows, (cudaStream_t)stream);
    return e == cudaSuccess ? WC_OK : cuda_error(e, "cq tensor-core kernel (no allocation)");
}

// ------------------------------------------------------------- needle ----

extern "C" wc_status wc_quantize_rows(const float *x, int rows, int cols, int width, int8_t *q, float *s,
                                      wc_stream stream) {
    if (width <= 0 || cols <= 0 || cols % width != 0)  // int8.go:108
        return set_error(WC_ERR_INVALID, fmt("needle: int8 rows of %d in chunks of %d", cols, width));
    if (rows < 0) return set_error(WC_ERR_INVALID, fmt("needle: %d rows", rows));
    long chunks = (long)rows * (cols / width);
    if (chunks == 0) return WC_OK;
    cudaError_t e = launch_quantize_rows(x, (int)chunks, width, q, s, (cudaStream_t)stream);
    return e == cudaSuccess ? WC_OK : cuda_error(e, "quantize kernel");
}

extern "C" wc_status wc_head_argmax(const float *y, int rows, int vocab, float head, float *logits, int32_t *idx,
                                    wc_stream stream) {
    if (rows < 0 || vocab < 0) return set_error(WC_ERR_INVALID, fmt("decoder: head of %d rows of %d logits", rows, vocab));
    if (rows == 0) return WC_OK;
    if (!idx || (vocab > 0 && !y)) return set_error(WC_ERR_INVALID, "decoder: nil head buffer");
    cudaError_t e;
    if (vocab == 0)  // greedy.go:182 on an empty row: 0
        e = cudaMemsetAsync(idx, 0, sizeof(int32_t) * (size_t)rows, (cudaStream_t)stream);
    else
        e = launch_head_argmax(y, rows, vocab, head, logits, idx, (cudaStream_t)stream);
    return e == cudaSuccess ? WC_OK : cuda_error(e, "head argmax kernel");
}

extern "C" wc_status wc_quantize_rows_host(const float *x, size_t x_len, int cols, int width, int8_t *q, float *s) {
    if (width <= 0 || cols <= 0 || cols % width != 0)
        return set_error(WC_ERR_INVALID, fmt("needle: int8 rows of %d in chunks of %d", cols, width));
    if (x_len % (size_t)cols != 0)  // int8.go:126-128
        return set_error(WC_ERR_INVALID, fmt("needle: %zu values are not rows of %d", x_len, cols));
    if (x_len == 0) return WC_OK;
    void *dx = nullptr, *dq = nullptr, *ds = nullptr;
    size_t chunks = x_len / width;
    WB_CUDA(t_scratch.get(0, x_len * sizeof(float), &dx));
    WB_CUDA(t_scratch.get(1, x_len, &dq));
    WB_CUDA(t_scratch.get(2, chunks * sizeof(float), &ds));
    WB_CUDA(cudaMemcpy(dx, x, x_len * sizeof(float), cudaMemcpyHostToDevice));
    wc_status st = wc_quantize_rows((const float *)dx, (int)(x_len / cols), cols, width, (int8_t *)dq, (float *)ds, nullptr);
    if (st != WC_OK) return st;
    WB_CUDA(cudaMemcpy(q, dq, x_len, cudaMemcpyDeviceToHost));
    WB_CUDA(cudaMemcpy(s, ds, chunks * sizeof(float), cudaMemcpyDeviceToHost));
    return WC_OK;
}

static wc_status check_attend(int heads, int kv_heads, int qk, int vd, int nkeys) {
    if (heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0)
        return set_error(WC_ERR_INVALID, fmt("needle: %d query heads over %d KV heads", heads, kv_heads));
    if (qk <= 0 || vd <= 0) return set_error(WC_ERR_INVALID, fmt("needle: head widths %d and %d", qk, vd));
    if (nkeys < 0) return set_error(WC_ERR_INVALID, fmt("needle: %d keys", nkeys));
    return WC_OK;
}

static wc_status attend_smem_ok(const AttendParams &p) {
    int dev = 0, limit = 0;
    WB_CUDA(cudaGetDevice(&dev));
    WB_CUDA(cudaDeviceGetAttribute(&limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    if (attend_smem_bytes(p) > (size_t)limit)
        return set_error(WC_ERR_UNSUPPORTED, fmt("needle: %d keys per query row exceed shared memory", p.max_keys));
    return WC_OK;
}

static bool aligned4(const void *p) { return ((uintptr_t)p & 3u) == 0; }
static bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

// The bulk-copy kernel (int8_attend_bulk.cu) for one query row per stream
// over all keys, when the cache rows can be bulk-copied (16-byte aligned
// rows and head slices). A CTA takes every KV head of its stream (whole
// rows: one bulk copy per chunk) when that fits and there are at least half
// as many streams as SMs; otherwise the KV-head group per CTA (kvpc) is the
// smallest whose query heads have at least 512 output columns (four per
// consumer thread), or the largest that fits, made smaller while the CTAs
// would not cover every SM. Returns false when the kernel does not apply.
static bool try_attend_bulk(AttendParams &p, int streams, cudaStream_t st, bool any_order, wc_status *status) {
    if (p.t != 1 || p.spans || p.probs || p.qk % 16 != 0 || p.vd % 16 != 0) return false;
    if (!aligned16(p.k8) || !aligned16(p.v8) || !aligned4(p.ks) || !aligned4(p.vs)) return false;
    int dev = 0, limit = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess)
        return false;
    const int gs = p.heads / p.kv_heads, sms = sm_count();
    std::vector<int> ok;  // usable group sizes, ascending
    std::vector<BulkLayout> lay;
    for (int kvpc = 1; kvpc <= p.kv_heads; kvpc++) {
        if (p.kv_heads % kvpc != 0 || !attend_bulk_shape_ok(p, kvpc)) continue;
        AttendParams q = p;
        q.kv_per_cta = kvpc;
        // A ring shallow enough for four CTAs an SM when the launch has
        // more than two CTAs an SM (1024 decode streams: the step 4.01 ->
        // 3.83 ms), else the deepest ring two CTAs an SM allow (256 streams
        // all fit at two; four there cost 4 % of the configs[3] component).
        const int share = (long long)streams * (p.kv_heads / kvpc) > 2LL * sms ? 4 : 2;
        const BulkLayout L = attend_bulk_pick_layout(q, (size_t)per_sm, (size_t)limit, share);
        if (L.total > (size_t)limit) continue;
        int blocks = 0;
        if (attend_bulk_occupancy(q, L, !any_order, &blocks) != cudaSuccess || blocks < 1) continue;
        ok.push_back(kvpc);
        lay.push_back(L);
    }
    if (ok.empty()) return false;
    size_t pick = ok.size() - 1;
    // Any order: every KV head in one CTA whenever that fits (one contiguous
    // copy a chunk). Cross attention of 1 to 128 streams x 375 keys then
    // takes 19.5 us against 33 us with a head a CTA, self attention 13 us
    // against 22.5; splitting a stream's keys over CTAs (their softmax sums
    // merged by the last) gained nothing at any stream count.
    const bool whole_any = any_order && ok.back() == p.kv_heads;
    if (!whole_any && (ok.back() != p.kv_heads || 2LL * streams < sms)) {
        for (size_t i = 0; i < ok.size(); i++)
            if (ok[i] * gs * p.vd >= 512) {
                pick = i;
                break;
            }
        while (pick > 0 && (long long)streams * (p.kv_heads / ok[pick]) < sms) pick--;
    }
    p.err = device_err_word();
    if (!p.err) return false;
    p.kv_per_cta = ok[pick];
    p.bulk_whole = ok[pick] == p.kv_heads;
    p.bulk_scales = aligned16(p.ks) && aligned16(p.vs) && ((size_t)p.cap * p.kv_heads) % 4 == 0;
    cudaError_t e = launch_attend_bulk(p, lay[pick], streams, !any_order, st);
    *status = e == cudaSuccess ? WC_OK : cuda_error(e, "attend bulk kernel");
    return true;
}

// The bulk-copy kernel when it applies; else the any-order kernel when asked
// for and its shape is supported; else the exact-order v2 kernel when its
// layout conditions hold and its shared memory fits; else the per-head
// kernel.
static wc_status run_attend(AttendParams &p, int streams, cudaStream_t st, bool any_order) {
    const int gs = p.heads / p.kv_heads;
    wc_status bst;
    if (try_attend_bulk(p, streams, st, any_order, &bst)) return bst;
    if (any_order && aligned4(p.v8) && aligned16(p.k8) && (p.kv_heads * p.qk) % 16 == 0 &&
        (p.kv_heads * p.vd) % 4 == 0) {
        int kvpc = 1;
        while (kvpc * 2 <= p.kv_heads && p.kv_heads % (kvpc * 2) == 0 && kvpc * 2 * p.vd <= 128 &&
               kvpc * 2 * gs <= 8)
            kvpc *= 2;
        p.kv_per_cta = kvpc;
        p.v_prefetch = aligned16(p.v8) && (p.kv_heads * p.vd) % 16 == 0 && (kvpc * p.vd) % 16 == 0 && p.vd % 16 == 0;
        int dev = 0, limit = 0;
        WB_CUDA(cudaGetDevice(&dev));
        WB_CUDA(cudaDeviceGetAttribute(&limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        if (attend_any_supported(p) && attend_any_smem_bytes(p) <= (size_t)limit) {
            cudaError_t e = launch_attend_any(p, streams, st);
            return e == cudaSuccess ? WC_OK : cuda_error(e, "attend kernel");
        }
    }
    const bool v2 = p.qk % 16 == 0 && p.vd % 16 == 0 && p.qk <= 128 && aligned16(p.k8) && aligned16(p.v8) &&
                    (p.kv_heads * p.qk) % 16 == 0 && (p.kv_heads * p.vd) % 16 == 0;
    if (v2) {
        int kvpc = 1;
        while (kvpc * 2 <= p.kv_heads && p.kv_heads % (kvpc * 2) == 0 && kvpc * gs * p.vd < 128) kvpc *= 2;
        p.kv_per_cta = kvpc;
        int dev = 0, limit = 0;
        WB_CUDA(cudaGetDevice(&dev));
        WB_CUDA(cudaDeviceGetAttribute(&limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        if (attend_v2_smem_bytes(p) <= (size_t)limit) {
            cudaError_t e = launch_attend_v2(p, streams, st);
            return e == cudaSuccess ? WC_OK : cuda_error(e, "attend kernel");
        }
    }
    wc_status ok = attend_smem_ok(p);
    if (ok != WC_OK) return ok;
    cudaError_t e = launch_attend(p, streams, st);
    return e == cudaSuccess ? WC_OK : cuda_error(e, "attend kernel");
}

extern "C" wc_status wc_attend_int8(const float *q, int t, int heads, const int8_t *k8, const float *ks,
                                    const int8_t *v8, const float *vs, int nkeys, int kv_heads, int qk, int vd,
                                    const int32_t *spans, float scale, int flags, float *probs, float *out,
                                    wc_stream stream) {
    wc_status st = check_attend(heads, kv_heads, qk, vd, nkeys);
    if (st != WC_OK) return st;
    if (t < 0) return set_error(WC_ERR_INVALID, fmt("needle: %d query rows", t));
    if (t == 0) return WC_OK;
    if (t > 65535) return set_error(WC_ERR_UNSUPPORTED, fmt("needle: %d query rows in one call", t));
    AttendParams p{};
    p.q = q;
    p.k8 = k8;
    p.ks = ks;
    p.v8 = v8;
    p.vs = vs;
    p.spans = spans;
    p.nkeys_dev = nullptr;
    p.probs = probs;
    p.out = out;
    p.t = t;
    p.heads = heads;
    p.kv_heads = kv_heads;
    p.qk = qk;
    p.vd = vd;
    p.nkeys = nkeys;
    p.cap = nkeys;
    p.max_keys = nkeys;
    p.scale = scale;
    p.quant_q = (flags & WC_ATTEND_QUANT_Q) ? 1 : 0;
    p.k_aligned4 = (qk % 4 == 0) && ((kv_heads * qk) % 4 == 0) && aligned4(k8);
    return run_attend(p, 1, (cudaStream_t)stream, (flags & WC_ATTEND_ANY_ORDER) != 0);
}

// AttendInt8Spans on host slices: every array is copied to one device
// buffer (the caller's probs too, so entries outside the spans keep their
// values), the kernels run, and out and probs are copied back.
extern "C" wc_status wc_attend_int8_host(const float *q, size_t q_len, int t, int heads, const int8_t *k8,
                                         size_t k8_len, const float *ks, size_t ks_len, const int8_t *v8,
                                         size_t v8_len, const float *vs, size_t vs_len, int kv_heads, int qk, int vd,
                                         const int32_t *spans, float scale, int flags, float *probs, size_t probs_len,
                                         float *out, size_t out_len) {
    if (t < 0) return set_error(WC_ERR_INVALID, fmt("needle: %d query rows", t));
    wc_status st = check_attend(heads, kv_heads, qk, vd, 0);
    if (st != WC_OK) return st;
    const size_t kcols = (size_t)kv_heads * qk, vcols = (size_t)kv_heads * vd;
    if (k8_len % kcols != 0)
        return set_error(WC_ERR_INVALID, fmt("needle: %zu key codes are not rows of %zu", k8_len, kcols));
    const size_t n = k8_len / kcols;
    if (ks_len != n * kv_heads || v8_len != n * vcols || vs_len != n * kv_heads)
        return set_error(WC_ERR_INVALID, fmt("needle: %zu keys with %zu key scales, %zu value codes and %zu value "
                                             "scales",
                                             n, ks_len, v8_len, vs_len));
    if (q_len != (size_t)t * heads * qk || out_len != (size_t)t * heads * vd ||
        (probs && probs_len < (size_t)t * heads * n))
        return set_error(WC_ERR_INVALID, fmt("needle: AttendInt8(len %zu, %d rows, %d heads of %d) into %zu outputs "
                                             "and %zu probabilities",
                                             q_len, t, heads, qk, out_len, probs ? probs_len : 0));
    if (n > (size_t)INT32_MAX) return set_error(WC_ERR_UNSUPPORTED, "needle: too many keys");
    if (t == 0) return WC_OK;
    auto up = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t b_q = up(q_len * 4), b_k = up(k8_len ? k8_len : 1), b_ks = up(ks_len * 4 + 4),
                 b_v = up(v8_len ? v8_len : 1), b_vs = up(vs_len * 4 + 4), b_sp = up((size_t)t * 16),
                 b_p = probs ? up((size_t)t * heads * n * 4 + 4) : 0, b_o = up(out_len * 4);
    void *base = nullptr;
    WB_CUDA(t_scratch.get(4, b_q + b_k + b_ks + b_v + b_vs + b_sp + b_p + b_o, &base));
    // One buffer: q, k codes, k scales, v codes, v scales, spans, probs, out.
    char *c = (char *)base;
    const size_t o_k = b_q, o_ks = o_k + b_k, o_v = o_ks + b_ks, o_vs = o_v + b_v, o_sp = o_vs + b_vs,
                 o_p = o_sp + b_sp, o_o = o_p + b_p;
    float *dq = (float *)c;
    int8_t *dk = (int8_t *)(c + o_k);
    float *dks = (float *)(c + o_ks);
    int8_t *dv = (int8_t *)(c + o_v);
    float *dvs = (float *)(c + o_vs);
    int32_t *dsp = (int32_t *)(c + o_sp);
    float *dp = probs ? (float *)(c + o_p) : nullptr;
    float *dout = (float *)(c + o_o);
    WB_CUDA(cudaMemcpy(dq, q, q_len * 4, cudaMemcpyHostToDevice));
    if (k8_len) WB_CUDA(cudaMemcpy(dk, k8, k8_len, cudaMemcpyHostToDevice));
    if (ks_len) WB_CUDA(cudaMemcpy(dks, ks, ks_len * 4, cudaMemcpyHostToDevice));
    if (v8_len) WB_CUDA(cudaMemcpy(dv, v8, v8_len, cudaMemcpyHostToDevice));
    if (vs_len) WB_CUDA(cudaMemcpy(dvs, vs, vs_len * 4, cudaMemcpyHostToDevice));
    if (spans) WB_CUDA(cudaMemcpy(dsp, spans, (size_t)t * 16, cudaMemcpyHostToDevice));
    if (probs && n) WB_CUDA(cudaMemcpy(dp, probs, (size_t)t * heads * n * 4, cudaMemcpyHostToDevice));
    st = wc_attend_int8(dq, t, heads, dk, dks, dv, dvs, (int)n, kv_heads, qk, vd, spans ? dsp : nullptr, scale, flags,
                        dp, dout, nullptr);
    if (st != WC_OK) return st;
    WB_CUDA(cudaMemcpy(out, dout, out_len * 4, cudaMemcpyDeviceToHost));
    if (probs && n) WB_CUDA(cudaMemcpy(probs, dp, (size_t)t * heads * n * 4, cudaMemcpyDeviceToHost));
    return WC_OK;
}

static wc_status attend_streams(int streams, const float *q, int heads, const int8_t *k8, const float *ks,
                                const int8_t *v8, const float *vs, int cap, const int32_t *nkeys, int kv_heads, int qk,
                                int vd, float scale, int flags, float *out, int kv_group, wc_stream stream);

extern "C" wc_status wc_attend_int8_streams(int streams, const float *q, int heads, const int8_t *k8, const float *ks,
                                            const int8_t *v8, const float *vs, int cap, const int32_t *nkeys,
                                            int kv_heads, int qk, int vd, float scale, int flags, float *out,
                                            wc_stream stream) {
    return attend_streams(streams, q, heads, k8, ks, v8, vs, cap, nkeys, kv_heads, qk, vd, scale, flags, out, 1,
                          stream);
}

namespace wb {
wc_status attend_streams_grouped(int streams, const float *q, int heads, const int8_t *k8, const float *ks,
                                 const int8_t *v8, const float *vs, int cap, const int32_t *nkeys, int kv_heads,
                                 int qk, int vd, float scale, int flags, float *out, int kv_group, cudaStream_t st) {
    if (kv_group < 1) return set_error(WC_ERR_INVALID, fmt("needle: %d streams per K/V block", kv_group));
    return attend_streams(streams, q, heads, k8, ks, v8, vs, cap, nkeys, kv_heads, qk, vd, scale, flags, out,
                          kv_group, (wc_stream)st);
}
}  // namespace wb

static wc_status attend_streams(int streams, const float *q, int heads, const int8_t *k8, const float *ks,
                                const int8_t *v8, const float *vs, int cap, const int32_t *nkeys, int kv_heads, int qk,
                                int vd, float scale, int flags, float *out, int kv_group, wc_stream stream) {
    wc_status st = check_attend(heads, kv_heads, qk, vd, cap);
    if (st != WC_OK) return st;
    if (streams < 0) return set_error(WC_ERR_INVALID, fmt("needle: %d streams", streams));
    if (streams == 0) return WC_OK;
    if (streams > 65535) return set_error(WC_ERR_UNSUPPORTED, fmt("needle: %d streams in one call", streams));
    AttendParams p{};
    p.q = q;
    p.k8 = k8;
    p.ks = ks;
    p.v8 = v8;
    p.vs = vs;
    p.spans = nullptr;
    p.nkeys_dev = nkeys;
    p.probs = nullptr;
    p.out = out;
    p.t = 1;
    p.heads = heads;
    p.kv_heads = kv_heads;
    p.qk = qk;
    p.vd = vd;
    p.nkeys = cap;
    p.cap = cap;
    p.max_keys = cap;
    p.scale = scale;
    p.quant_q = (flags & WC_ATTEND_QUANT_Q) ? 1 : 0;
    p.k_aligned4 = (qk % 4 == 0) && ((kv_heads * qk) % 4 == 0) && aligned4(k8);
    p.kv_group = kv_group;
    return run_attend(p, streams, (cudaStream_t)stream, (flags & WC_ATTEND_ANY_ORDER) != 0);
}
