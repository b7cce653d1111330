/*
 * whistle_b200.h — the C ABI of libwhistle_b200.so, the B200 (sm_100a) build of
 * go-whistle's quantized hot path: the packed 2/4-bit CQ LUT GEMV/GEMM of
 * internal/cq and the int8 KV-cache attention of internal/needle.
 *
 * Plain C: pointers, sizes and status codes; no CUDA, Go or torch types. A
 * cgo shim binds these one for one. Each entry point names
 * the reference routine it stands in for (file:line in the go-whistle
 * module).
 *
 * Conventions
 *  - Every call returns a wc_status. WC_OK is 0. On failure the message of
 *    the calling thread's last error (wc_last_error) carries the text the
 *    reference would have put in its error or panic, e.g. "cq: group 24 is
 *    not a power of two >= 8".
 *  - "device" pointers are CUDA global memory of the current device; "host"
 *    pointers are ordinary process memory. The *_host entry points copy in
 *    and out, synchronise, and so behave like the reference's Go calls.
 *  - wc_stream is a cudaStream_t (NULL: the legacy default stream). Device
 *    entry points only enqueue work; the caller orders and synchronises.
 *  - A wc_cq handle belongs to the device that was current at its creation;
 *    calls on it with another device current fail with WC_ERR_DEVICE.
 *  - Handles are safe for concurrent use from several threads (each thread
 *    on its own stream), as cq.Matrix is (internal/cq/matrix.go:22-24).
 *  - Nothing in this library aborts the process, traps, or falls back to a
 *    CPU path: a missing or unusable GPU is an error status.
 */
#ifndef WHISTLE_B200_H
#define WHISTLE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum wc_status {
    WC_OK = 0,
    WC_ERR_INVALID = 1,     /* misuse the reference panics on: shapes, lengths, ranges */
    WC_ERR_UNSUPPORTED = 2, /* a tensor the reference's constructor rejects with an error */
    WC_ERR_CUDA = 3,        /* a CUDA runtime error (message has cudaGetErrorString) */
    WC_ERR_NOMEM = 4,       /* device or host allocation failed */
    WC_ERR_DEVICE = 5,      /* handle used with another device current */
} wc_status;

typedef struct wc_cq wc_cq; /* a device-resident CQ matrix, or a view of one */
typedef void *wc_stream;    /* cudaStream_t */

/* The calling thread's last error message (NUL-terminated, truncated to
 * len). Returns the full message length. No reference counterpart: Go
 * returns the error value itself. */
size_t wc_last_error(char *buf, size_t len);

/* Library version string ("whistle_b200 <major>.<minor>"). */
const char *wc_version(void);

/* Kernels this library has launched in this process so far (all devices,
 * all threads). A diagnostic with no reference counterpart: benchmarks read
 * it before and after a timed region to count their launches. */
uint64_t wc_launch_count(void);

/* ---------------------------------------------------------------- cq ---- */

/*
 * Creates a device copy of a packed CQ tensor and prepares it for products.
 * Replaces internal/cq/matrix.go:46 New (and :60 NewGather, :111 Prepare):
 * the same validation in the same order with the same messages
 * (matrix.go:61-73). The fields are cact.Packed's
 * (internal/cact/packed.go:18-29): index = out rows of RowBytes() bytes of
 * LSB-first indices (index_len bytes), norms = out*groups little-endian FP16
 * values (norms_len BYTES, as Packed.Norms), codebook = codebook_len float32
 * levels, bits = Record.Bits, width = bits per stored index. Host pointers;
 * nothing is retained after the call.
 */
wc_status wc_cq_create(const uint8_t *index, size_t index_len, const uint8_t *norms, size_t norms_len,
                       const float *codebook, size_t codebook_len, int out, int in, int group, int bits, int width,
                       wc_cq **h);

/* Rows [lo, hi) as a view sharing h's device storage: matrix.go:133 Rows.
 * The view keeps the storage alive after wc_cq_destroy(h). */
wc_status wc_cq_rows(const wc_cq *h, int lo, int hi, wc_cq **view);

/* A view whose products run the reference's Exact (nibble/nibble4, float32
 * sums) kernels instead of the lut kernel: matrix.go:152 Exact. */
wc_status wc_cq_exact(const wc_cq *h, wc_cq **view);

/* Releases a matrix or view (device storage goes with the last of them). */
void wc_cq_destroy(wc_cq *h);

/* matrix.go:99 Out, :102 In, :105 Bits. */
int wc_cq_out(const wc_cq *h);
int wc_cq_in(const wc_cq *h);
int wc_cq_bits(const wc_cq *h);

/* Device bytes the matrix holds: packed index, FP16 norms and codebook
 * (matrix.go:121 Bytes counts the reference's host copies instead). */
size_t wc_cq_bytes(const wc_cq *h);

/*
 * y = x · Wᵀ for `rows` activations: x [rows][In], y [rows][Out], both
 * row-major fp32 DEVICE memory. internal/cq/kernel.go:85 GEMM (and :78 GEMV
 * for rows = 1). The lut kernel's result is bit-identical to the
 * reference's lut kernel; an Exact view's to its nibble4/nibble kernels.
 * rows = 0 or Out = 0 is a no-op (kernel.go:110).
 */
wc_status wc_cq_gemm(const wc_cq *h, const float *x, float *y, int rows, wc_stream stream);

/* Flags of wc_cq_gemm_ex and wc_cq_gemms_ex. */
enum {
    /* Run the product on the tensor cores (tcgen05, fp16 operands in the
     * rotated domain, each scaled by an exact power of two — per activation
     * row and per matrix — and fp32 accumulation) instead of the bit-exact
     * lut kernel: for many rows (encoder prefill, batched decode). Not
     * bit-exact: each output y is within
     *   (2^-10 + (K + log2 G + 6)·2^-24) · Σ_k |x̂_k|·|ŵ_k|
     *   + 2^-37 · (G·max|x| · Σ_k |ŵ_k| + max|ŵ| · Σ_k |x̂_k|)
     * of the exact product (K = In rounded up to the group, x̂ and ŵ the
     * rotated activation row and weight row, max|x| over the activation
     * row, max|ŵ| over the matrix; the second line covers fp16's
     * subnormals), and every row of y has cosine >= 0.99999 with the exact
     * product on the reference's test distributions, its lut kernel's
     * accept (internal/cq/cq_test.go:196-254). In <= 4096. */
    WC_GEMM_TENSOR_CORES = 1,
    /* The tensor cores once rows x output rows (all matrices of a GEMMs
     * call) reach 65,536, from 2 rows; the bit-exact lut kernels below:
     * the faster of the two on B200 at each size, the choice a batched
     * caller (multi-stream decode, prefill) makes. */
    WC_GEMM_AUTO = 2,
};

/*
 * wc_cq_gemm with options (flags above). With WC_GEMM_TENSOR_CORES the first
 * call on a matrix builds its fp16 weight image on the device (or call
 * wc_cq_prepare_tc first, outside any stream capture), and each call uses a
 * per-thread device buffer for the rotated activations, grown on demand: a
 * thread's tensor-core calls must not overlap on the GPU (use one stream
 * per calling thread). No reference counterpart: the reference has only
 * the exact kernels.
 */
wc_status wc_cq_gemm_ex(const wc_cq *h, const float *x, float *y, int rows, int flags, wc_stream stream);

/*
 * internal/cq/kernel.go:134 GEMMs with the options of wc_cq_gemm_ex. On the
 * tensor cores the matrices that share a group size share one rotation of
 * x, and up to 16 of them run as one grouped launch; otherwise it is
 * wc_cq_gemms. Each ys[k] equals what wc_cq_gemm_ex gives for hs[k].
 */
wc_status wc_cq_gemms_ex(const wc_cq *const *hs, int n, const float *x, float *const *ys, int rows, int flags,
                         wc_stream stream);

/* Builds the tensor-core weight image of h now (synchronous). */
wc_status wc_cq_prepare_tc(const wc_cq *h);

/*
 * The tensor-core GEMM (wc_cq_gemm_ex with WC_GEMM_TENSOR_CORES) for callers
 * that must not allocate GPU memory while they run. Examples: a real-time
 * transcription loop, where a cudaMalloc can synchronise the device and
 * stall a decode step for milliseconds; or a serving process that reserves
 * its GPU memory once at start-up, next to other models, and cannot let a
 * call grow it. This entry point calls no cudaMalloc, cudaFree or other
 * allocating routine: the rotated activations go to a fixed 16.5 MiB array
 * that the library keeps on every GPU it is loaded on, until the process
 * exits. It has no counterpart in the reference.
 *
 *  - R · (K · 2 + 4) bytes must fit in 16.5 MiB, R = rows rounded up to
 *    128 and K = In rounded up to the group and to 64 (16,896 rows at
 *    In = 512, 4,096 at In = 2048); larger calls
 *    fail with WC_ERR_INVALID and leave y alone.
 *  - h must already have its weight image: call wc_cq_prepare_tc when the
 *    matrix is loaded (that call allocates; this one does not).
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress) with that device current; make that first call
 *    before any stream capture.
 *  - All calls share the one array, which keeps the last call's contents:
 *    calls whose work overlaps on the GPU (on different streams, or from
 *    different threads without ordering) race and corrupt each other.
 *  - err: a device int that receives the error code of the kernels' bounded
 *    waits (0 = none; the caller clears it), or NULL to use a word inside
 *    the array. That word keeps the first code of any call until
 *    wc_device_status reports and clears it, so a caller passing NULL
 *    learns of an expired wait from wc_device_status (which synchronises,
 *    and so belongs outside the real-time loop, e.g. once per utterance).
 *    After an expired wait y is incomplete.
 * x [rows][In] and y [rows][Out] are fp32 DEVICE memory; y is what
 * wc_cq_gemm_ex with WC_GEMM_TENSOR_CORES computes, bit for bit: the same
 * kernels are chosen for the same number of rows (the persistent one from
 * 1,024 rows).
 */
wc_status wc_cq_gemm_tc_noalloc(const wc_cq *h, const float *x, float *y, int rows, int *err, wc_stream stream);

/* Synchronises the current device and reports (and clears) the error words
 * of the kernels' bounded waits — the library's word and the
 * no-allocation GEMM's — : *code = 0 if none expired. A diagnostic with no
 * reference counterpart. */
wc_status wc_device_status(int *code);

/* GEMM on HOST slices with the reference's length check and panic text
 * (kernel.go:105-107): x_len = len(x), y_len = len(dst). Synchronous; the
 * result travels as wc_cq_gemms_host's does. */
wc_status wc_cq_gemm_host(const wc_cq *h, const float *x, size_t x_len, float *y, size_t y_len, int rows);

/*
 * internal/cq/kernel.go:134 GEMMs: ys[k] = x · hs[k]ᵀ for n matrices that
 * read the same x [rows][In] (DEVICE). Matrices that share the input width,
 * group, index width and codebook (lut.go:206 sharesTables) run as ONE
 * launch that rotates and tabulates each activation once for all of them;
 * the others run one GEMM each. Every ys[k] equals wc_cq_gemm's bit for
 * bit. hs and ys are host arrays of n device pointers.
 */
wc_status wc_cq_gemms(const wc_cq *const *hs, int n, const float *x, float *const *ys, int rows, wc_stream stream);

/* GEMMs on HOST slices: y_lens[k] = len(dsts[k]). Synchronous. Outputs in
 * page-locked host memory that the device can address (cudaHostAlloc, or
 * cudaHostRegister under unified addressing) receive the results straight
 * from the kernels, which overlaps the transfer with the products; other
 * outputs are copied from device memory in chunks behind the kernels. The
 * bits are the same either way. */
wc_status wc_cq_gemms_host(const wc_cq *const *hs, int n, const float *x, size_t x_len, float *const *ys,
                           const size_t *y_lens, int rows);

/* internal/cq/matrix.go:161 Row: row r dequantised exactly as cact.CQ does
 * (bit for bit) into dst [In] (DEVICE). */
wc_status wc_cq_row(const wc_cq *h, int r, float *dst, wc_stream stream);

/* Row for n rows at once (an embedding gather for n streams): rows is a
 * DEVICE array of n row numbers, dst is [n][In] DEVICE. Rows out of range
 * produce zeros and set *bad (DEVICE int, may be NULL) to 1. */
wc_status wc_cq_row_gather(const wc_cq *h, const int32_t *rows, int n, float *dst, int32_t *bad,
                           wc_stream stream);

/* Row on a HOST dst of dst_len floats, with matrix.go:162's panic text. */
wc_status wc_cq_row_host(const wc_cq *h, int r, float *dst, size_t dst_len);

/* ------------------------------------------------------------ needle ---- */

/* Flags of the attention entry points. */
enum {
    /* Quantise each query head to int8 first (Int8.Act): exact int32 logits. */
    WC_ATTEND_QUANT_Q = 1,
    /* Let the float sums (softmax sum, the weighted sum of the values) run in
     * any order, with FMAs and expf: several times the throughput, results
     * within 1e-5 relative of the exact order. Without it the reference's
     * generic order is followed operation by operation. */
    WC_ATTEND_ANY_ORDER = 2,
};

/*
 * internal/needle/int8.go:115 QuantizeRows (and :125 Int8Rows.Append when q
 * and s point at a cache's tail): x [rows][cols] fp32 in chunks of width,
 * q [rows][cols] int8, s [rows*cols/width] fp32; all DEVICE. Each chunk is
 * int8.go:36 QuantizeRow bit for bit.
 */
wc_status wc_quantize_rows(const float *x, int rows, int cols, int width, int8_t *q, float *s, wc_stream stream);

/*
 * The decoder's head scale and greedy choice for `rows` rows of `vocab`
 * logits y (DEVICE memory), e.g. a wc_cq_gemm of the embedding matrix:
 * internal/decoder/decoder.go:508-523 logits multiplies every logit by head
 * when head != 1, and internal/decoder/greedy.go:182 argmax takes the first
 * index of the largest value (a NaN at index 0 gives 0, later NaNs never
 * win, +0 and -0 tie). logits (or NULL) receives the scaled logits and may
 * be y itself; idx[rows] receives the argmax of each row (0 for an empty
 * row). Enqueued on `stream`.
 */
wc_status wc_head_argmax(const float *y, int rows, int vocab, float head, float *logits, int32_t *idx,
                         wc_stream stream);

/* QuantizeRows on HOST memory (x_len values), with int8.go:108's checks. */
wc_status wc_quantize_rows_host(const float *x, size_t x_len, int cols, int width, int8_t *q, float *s);

/*
 * internal/needle/int8.go:208 AttendInt8Spans (int8.go:194 AttendInt8 is the
 * span pair {0,0},{0,keys(i)}). DEVICE memory:
 *   q      [t][heads][qk] fp32
 *   k8, ks the keys: [nkeys][kv_heads*qk] int8 and [nkeys][kv_heads] fp32
 *   v8, vs the values: [nkeys][kv_heads*vd] int8 and [nkeys][kv_heads] fp32
 *   spans  [t][4] int32: lo0, hi0, lo1, hi1, two ascending disjoint key
 *          ranges per query row
 *   probs  [t][heads][nkeys] fp32 or NULL; written at span keys only
 *   out    [t][heads][vd] fp32
 * Query head h reads KV head h / (heads / kv_heads). flags: WC_ATTEND_QUANT_Q
 * quantises each query head to int8 first (Int8.Act), making the logits
 * exact int32 dot products; without WC_ATTEND_ANY_ORDER the result equals
 * the reference's generic (purego) path bit for bit, up to the last-bit
 * rounding of exp: the reference rounds Go's float64 math.Exp, this library
 * CUDA's double exp; both are within one float64 ulp, so their float32
 * roundings can differ only when e^x lies within about 2^-29 (relative) of
 * a float32 rounding boundary.
 */
wc_status wc_attend_int8(const float *q, int t, int heads, const int8_t *k8, const float *ks, const int8_t *v8,
                         const float *vs, int nkeys, int kv_heads, int qk, int vd, const int32_t *spans, float scale,
                         int flags, float *probs, float *out, wc_stream stream);

/*
 * AttendInt8Spans (internal/needle/int8.go:208) on host slices, as the Go
 * shim calls it: q [t][heads][qk]; k8/ks and v8/vs the int8 rows and
 * scales of Int8Rows (nkeys = k8_len / (kv_heads·qk)); spans [t][4] or
 * NULL for every key; probs NULL or at least t·heads·nkeys values, written
 * at the spans' keys only; out [t][heads][vd]. Lengths are checked (a
 * mismatch is WC_ERR_INVALID); synchronous.
 */
wc_status wc_attend_int8_host(const float *q, size_t q_len, int t, int heads, const int8_t *k8, size_t k8_len,
                              const float *ks, size_t ks_len, const int8_t *v8, size_t v8_len, const float *vs,
                              size_t vs_len, int kv_heads, int qk, int vd, const int32_t *spans, float scale,
                              int flags, float *probs, size_t probs_len, float *out, size_t out_len);

/*
 * The decode step of `streams` independent streams, one query row each,
 * against each stream's own int8 KV cache: AttendInt8 (int8.go:194) per
 * stream with keys(0) = nkeys[b], as Attention.extendInt8 (cache.go:120)
 * and cross.attend (decoder/cross.go:273) call it. Stream b's cache starts
 * at b*cap rows of k8/ks/v8/vs (layouts as in wc_attend_int8); q is
 * [streams][heads][qk], out [streams][heads][vd], nkeys [streams] int32;
 * all DEVICE. nkeys[b] > cap is clamped to cap.
 */
wc_status wc_attend_int8_streams(int streams, const float *q, int heads, const int8_t *k8, const float *ks,
                                 const int8_t *v8, const float *vs, int cap, const int32_t *nkeys, int kv_heads,
                                 int qk, int vd, float scale, int flags, float *out, wc_stream stream);

/* ----------------------------------------------------------- decoder ---- */

/*
 * Whistle's text decoder on the device: internal/decoder's Decoder with the
 * Best() hypothesis (decoder/hypothesis.go:199: cross-attention after the
 * self-attention, ZC q/k norms, sigmoid gates and residual, √dim input
 * scale, tied head, final norm, engram on, no cross RoPE) and the engine's
 * int8 numerics (needle.Int8{Act: true, KV: true}, whistle.WithInt8). Many
 * independent sequences ("streams") advance together, one token each per
 * step; every stream's state — the mHC lanes, the int8 self-attention
 * caches with their tap history, the engram caches and the int8
 * cross-attention memory — stays in device memory.
 *
 * The tensors are the reference's, as its loaders read them from
 * whistle.cact (decoder.go:76 LoadInt8, needle.LoadBlock/LoadMHC/
 * LoadEngram): CQ matrices as wc_cq handles (the decoder keeps views of
 * them), float tensors as HOST arrays (copied at creation), norm vectors as
 * the stored scales (gain = 1 + scale), gates as their raw parameters.
 */
typedef struct wc_decoder wc_decoder;

/* One decoder layer: layerNN.* (needle.Block, block.go:21; Attention,
 * attention.go:38; HadamardMLP, hadamard.go:28), crossNN.* (cross.go:26)
 * and the layer's mHC heads (mhc.go:30; phi_* are this layer's row views of
 * the stacked mhc_phi_*, mhc.go:94-96). */
typedef struct wc_decoder_layer {
    const float *norm_in, *post_norm, *pre_hada; /* [dim] */
    float attn_gate;
    const wc_cq *q_proj, *k_proj, *v_proj, *gate_proj, *out_proj;
    const float *q_taps, *k_taps, *v_taps; /* [taps][heads·qk | kv_heads·qk | kv_heads·vd] */
    const float *q_norm, *k_norm;          /* [qk] */
    const float *d1, *d2, *b2, *d3, *d4;   /* [na·nb] */
    const float *w1a, *w1b, *w2a, *w2b, *w3a, *w3b; /* [na][na], [nb][nb] */
    const float *cond_v; /* [dim][rank] */
    const float *cond_u; /* [rank][na·nb] */
    const float *x_norm_in, *x_post_norm, *x_q_norm, *x_k_norm;
    float x_attn_gate;
    const wc_cq *x_q_proj, *x_k_proj, *x_v_proj, *x_gate_proj, *x_out_proj;
    float a_pre, a_post, a_res;
    const float *b_pre, *b_post; /* [lanes] */
    const float *b_res;          /* [lanes][lanes] */
    const wc_cq *phi_pre, *phi_post, *phi_res;
} wc_decoder_layer;

/* One engram site: engramN.* (needle/engram.go:35) and its layer. */
typedef struct wc_engram_site {
    const wc_cq *tables;            /* [n_tables·slots][sub] */
    const wc_cq *key_proj, *value_proj; /* [dim][n_tables·sub] */
    const float *taps;              /* [etaps][dim] */
    int layer;
} wc_engram_site;

typedef struct wc_decoder_desc {
    int dim, lanes, layers, vocab;
    int heads, kv_heads, qk, vd, taps;
    int x_heads, x_qk, x_vd;
    int na, nb, rank;
    int n_sites, n_tables, slots, sub, etaps;
    const int32_t *orders;           /* [n_tables]: table c's n-gram order */
    const int32_t *hada_p1, *hada_p2; /* [na·nb] */
    double rope_theta;
    int rope_len;
    const wc_cq *embedding;          /* [vocab][dim], also the head */
    const float *final_norm;         /* [dim] */
    const wc_decoder_layer *layer;   /* [layers] */
    const wc_engram_site *site;      /* [n_sites] */
} wc_decoder_desc;

/* Flags of wc_decoder_create. */
enum {
    /* Every CQ product on the tensor cores (WC_GEMM_TENSOR_CORES' fp16
     * bound) instead of the bit-exact lut kernels. */
    WC_DECODER_TENSOR_CORES = 1,
    /* Run each step as eager launches instead of a captured CUDA graph. */
    WC_DECODER_NO_GRAPH = 2,
};

/*
 * Builds a decoder (decoder.go:76 LoadInt8) with device room for up to
 * max_streams sequences of up to max_positions tokens against memories of
 * up to max_frames encoder frames. Validates the shapes with the loaders'
 * messages ("decoder: …", "needle: …"). This build's kernels take
 * Whistle's widths: dim 512 in 4 lanes, qk 48, vd 64, HadamardMLP 16 × 32.
 */
wc_status wc_decoder_create(const wc_decoder_desc *desc, int max_streams, int max_frames, int max_positions,
                            int flags, wc_decoder **out);
void wc_decoder_destroy(wc_decoder *d);

/*
 * decoder.go:157 Memory and :194 NewState for `streams` streams: enc is
 * DEVICE [streams][frames][dim] (each stream's encoder output); every
 * layer's cross-attention keys and values (cross.go:181 project: the k/v
 * products, the per-head k norm, QuantizeRows) go to the device memory,
 * and every stream starts an empty sequence.
 */
wc_status wc_decoder_memory(wc_decoder *d, const float *enc, int streams, int frames, wc_stream stream);

/*
 * decoder.go:252 Extend with one token per stream: tokens DEVICE [streams];
 * logits (or NULL) DEVICE [streams][vocab] receives the next-token logits
 * (decoder.go:508 logits); next (or NULL) DEVICE [streams] their argmax
 * (greedy.go:182).
 */
wc_status wc_decoder_extend(wc_decoder *d, const int32_t *tokens, float *logits, int32_t *next, wc_stream stream);

/*
 * decoder/greedy.go:40 GreedyMemory for every stream: the prompt [bos], the
 * language token (the largest logit among langs, the first on ties,
 * greedy.go:81), then argmax tokens until eos or max_tokens − 1 steps.
 * All on the device, with no host synchronisation between steps. DEVICE
 * outputs: tokens [streams][max_tokens − 1] (each stream's text tokens,
 * then −1), counts [streams], lang [streams] (the language token),
 * eos_hit [streams]. langs is a HOST array of n_langs token ids.
 */
wc_status wc_decoder_greedy(wc_decoder *d, int bos, const int32_t *langs, int n_langs, int eos, int max_tokens,
                            int32_t *tokens, int32_t *counts, int32_t *lang, int32_t *eos_hit, wc_stream stream);

/* Positions fed so far (every stream advances together). */
int wc_decoder_len(const wc_decoder *d);

/* ---------------------------------------------------------- beam search */

/*
 * decoder.go:157 Memory for a beam search: enc holds `clips` encoder
 * outputs (DEVICE [clips][frames][512]); the decoder then runs
 * clips × beams streams, stream c·beams + b being beam b of clip c, and the
 * beams of a clip read one shared int8 cross memory (no copy per beam).
 * Needs clips × beams <= max_streams.
 */
wc_status wc_decoder_memory_beams(wc_decoder *d, const float *enc, int clips, int frames, int beams,
                                  wc_stream stream);

/* search/options.go: Norm, Length, Stop, Admit, LangStep. */
enum {
    WC_NORM_NONE = 1, WC_NORM_LEN = 2, WC_NORM_POW = 3, WC_NORM_GNMT = 4,
    WC_LEN_TEXT = 1, WC_LEN_TEXT_EOS = 2, WC_LEN_SEQ = 3,
    WC_STOP_ALL = 1, WC_STOP_BEST = 2, WC_STOP_K = 3, WC_STOP_HF = 4,
    WC_ADMIT_TOPK = 1, WC_ADMIT_ABOVE_LIVE = 2,
    WC_LANG_ARGMAX = 1, WC_LANG_ARGMAX_SCORED = 2, WC_LANG_BEAM = 3,
};

/* search/options.go:105 Options (the Adjust hook and the probe-only
 * finished-hypothesis variants are not offered: their zero values,
 * Whisper's, apply). */
typedef struct wc_beam_options {
    int beams;      /* hypotheses kept per step, >= 1 (<= 63) */
    int max_tokens; /* tokens after the prompt, the language token included; 0: the positions the decoder holds */
    int language;   /* index into langs of a forced language, or −1 to detect it */
    int norm;       /* WC_NORM_* */
    double alpha;   /* exponent of WC_NORM_POW and WC_NORM_GNMT */
    int length;     /* WC_LEN_*: what the normalisation's L counts */
    int stop;       /* WC_STOP_* */
    int admit;      /* WC_ADMIT_* (all rules but WC_STOP_ALL) */
    int lang_step;  /* WC_LANG_* */
} wc_beam_options;

/* options.go:143 Default: 5 beams, NormLen, α 1, LenText, StopK,
 * AdmitAboveLive, LangArgmax, max_tokens 0, language −1. */
void wc_beam_default(wc_beam_options *o);

/*
 * search/beam.go:73 Beam for every clip of the last
 * wc_decoder_memory_beams (whose beams must equal o->beams): the prompt
 * [bos], the language step among langs (HOST, n_langs ids; the language's
 * code is its index), then beam steps until the stopping rule or the token
 * limit; beams share their prefix through forks of the decoder's stream
 * states (decoder.go:223 State.Fork). HOST outputs per clip: tokens
 * [clips][max_tokens − 1] (the best hypothesis' text tokens, then −1),
 * counts, lang (its language token), eos_hit, score (its ranking score),
 * and optionally lang_logprob [clips] and logprobs [clips][max_tokens] (the
 * model's log p of each text token, then of EOS when eos_hit; NULL to skip).
 */
wc_status wc_decoder_beam(wc_decoder *d, const wc_beam_options *o, int bos, const int32_t *langs, int n_langs,
                          int eos, int32_t *tokens, int32_t *counts, int32_t *lang, int32_t *eos_hit, double *score,
                          double *lang_logprob, double *logprobs, wc_stream stream);

/* Layer l's int8 cross-attention memory for the tests: device pointers to
 * k8 [streams][frames][x_heads·x_qk], ks [streams][frames][x_heads], v8, vs
 * (layouts as wc_attend_int8_streams reads them, cap = frames). */
wc_status wc_decoder_memory_of(const wc_decoder *d, int l, const int8_t **k8, const float **ks, const int8_t **v8,
                               const float **vs);

/* ------------------------------------------------------------------
 * Whistle's encoder stack on the device: internal/encoder's Stack
 * (encoder.go:167) with the Best() hypothesis (hypothesis.go:284) and the
 * engine's int8 numerics (whistle/model.go:85 WithInt8 -> encoder.go:50
 * LoadInt8): per layer, mHC (needle/mhc.go:182) around the macaron block
 * (block.go:148: FFN1 at scale 1/2, attention with no mask and RoPE
 * θ = 1e5, the conv module pw1 -> GLU value·σ(gate) -> centred depthwise
 * conv -> conv_out_norm -> SiLU -> pw2, FFN2 at scale 1/2), then the lane
 * mean and the final norm. Its input is the stem's output (encoder.go:132
 * Stem: the log-mel front end and the conv stem run before it).
 */

/* One HadamardMLP's tensors (needle/hadamard.go:28). */
typedef struct wc_hadamard_mlp {
    const float *d1, *d2, *b2, *d3, *d4;            /* [na·nb] */
    const float *w1a, *w1b, *w2a, *w2b, *w3a, *w3b; /* [na][na], [nb][nb] */
    const float *cond_v;                            /* [dim][rank] */
    const float *cond_u;                            /* [rank][na·nb] */
} wc_hadamard_mlp;

/* One encoder layer, encNN.* (block.go:17 block) and its mHC rows. Norm
 * vectors are the stored scales (gain = 1 + scale); attn_gate is raw. */
typedef struct wc_encoder_layer {
    const float *pre_hada_0, *norm_in, *post_norm, *conv_norm, *conv_out_norm, *pre_hada; /* [dim] */
    float attn_gate;
    const wc_cq *q_proj, *k_proj, *v_proj, *gate_proj, *out_proj; /* self-attention */
    const wc_cq *pw1, *pw2;                                       /* [2·dim][dim], [dim][dim] */
    const float *q_norm, *k_norm;                                 /* [qk] */
    const float *dw;                                              /* [dw_kernel][dim] */
    wc_hadamard_mlp hada_0, hada;                                 /* FFN1, FFN2 */
    float a_pre, a_post, a_res;
    const float *b_pre, *b_post; /* [lanes] */
    const float *b_res;          /* [lanes][lanes] */
    const wc_cq *phi_pre, *phi_post, *phi_res;
} wc_encoder_layer;

typedef struct wc_encoder_desc {
    int dim, lanes, layers, heads, kv_heads, qk, vd, dw_kernel, na, nb, rank;
    const int32_t *hada_p1, *hada_p2; /* [na·nb] */
    double rope_theta;
    int rope_len;
    const float *final_norm;        /* [dim] */
    const wc_encoder_layer *layer;  /* [layers] */
    /* The conv stem (stem.go:20) and the front end's mel bank, or all NULL
     * for the stack alone: 3×3 kernels as stored, (9, channels) with the
     * taps time-major; pointwise products [channels][channels]; stem.out
     * [dim][10·channels] over the channel-major flatten; mel_filters
     * [257][80] (frontend/mel.go:30 MelBank). */
    const float *stem_w, *stem_dw_1, *stem_dw_2;
    const wc_cq *stem_pw_1, *stem_pw_2, *stem_out;
    int stem_channels;
    const float *mel_filters;
} wc_encoder_desc;

typedef struct wc_encoder wc_encoder;

/* Flags of wc_encoder_create. */
enum {
    /* Every CQ product on the tensor cores (WC_GEMM_TENSOR_CORES' fp16
     * bound) instead of the bit-exact lut kernels. */
    WC_ENCODER_TENSOR_CORES = 1,
    /* The attention in any order (WC_ATTEND_ANY_ORDER's 1e-5 bound) instead
     * of int8.go's exact order. */
    WC_ENCODER_ANY_ORDER = 2,
};

/*
 * Builds an encoder stack (encoder.go:50 LoadInt8's stack part) with device
 * room for up to max_clips clips of up to max_frames frames. This build's
 * kernels take Whistle's widths: dim 512 in 4 lanes, heads of 48/64 with
 * 8·64 = 512, a 16 × 32 HadamardMLP of rank 8, an odd depthwise kernel of
 * up to 31 taps. max_clips · max_frames is at most 65,535 rows.
 */
wc_status wc_encoder_create(const wc_encoder_desc *desc, int max_clips, int max_frames, int flags, wc_encoder **out);
void wc_encoder_destroy(wc_encoder *e);

/*
 * encoder.go:167 Stack for `clips` clips of `frames` frames each: x DEVICE
 * [clips][frames][dim] (the stem's output; not written), out DEVICE
 * [clips][frames][dim]. Each clip's frames attend to that clip's frames
 * only; RoPE positions count from 0 in every clip.
 */
wc_status wc_encoder_stack(wc_encoder *e, const float *x, int clips, int frames, float *out, wc_stream stream);

/*
 * frontend/mel.go:226 LogMel with the Best() front end (hypothesis.go:288:
 * a 400-sample symmetric Hann window centred in a 512-point frame every 160
 * samples, zero padding, the power spectrum, the float64 mel sums, the soft
 * log knee 76 dB below the clip's peak, each channel standardised over
 * time): samples DEVICE [clips][n] at 16 kHz, mel DEVICE [clips][n/160][80].
 * The spectrum is a float64 DFT of the float32 windowed frame (the
 * reference's is algo-dsp's float32 FFT). Needs the desc's mel_filters.
 */
wc_status wc_encoder_logmel(wc_encoder *e, const float *samples, int clips, int n, float *mel, wc_stream stream);

/* The stem's output length for `frames` mel frames (stem.go:166 length):
 * three stride-2 stages of symmetric padding. */
int wc_encoder_stem_frames(int frames);

/*
 * encoder.go:132 Stem with Best(): mel DEVICE [clips][frames][80] to x
 * DEVICE [clips][wc_encoder_stem_frames(frames)][dim]. Each 3×3 tap sum
 * runs in tap order (time, then mel); the products are the encoder's (lut
 * or tensor cores). Needs the desc's stem tensors.
 */
wc_status wc_encoder_stem(wc_encoder *e, const float *mel, int clips, int frames, float *x, wc_stream stream);

/* encoder.go:108 Embed: LogMel, Stem and Stack on samples DEVICE
 * [clips][n]; out DEVICE [clips][wc_encoder_stem_frames(n/160)][dim]. */
wc_status wc_encoder_embed(wc_encoder *e, const float *samples, int clips, int n, float *out, wc_stream stream);

#ifdef __cplusplus
}
#endif
#endif
