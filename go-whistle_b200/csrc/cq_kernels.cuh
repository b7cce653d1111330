// cq_kernels.cuh — launch interfaces of the CQ kernels (cq_lut.cu,
// cq_exact.cu) used by the C-ABI layer (api.cu).
#pragma once

#include "common.cuh"

namespace wb {

// Rows per CTA tile of the lut kernel: kTileRows for several activations,
// kTileRowsOne for one (four times the CTAs, for latency).
constexpr int kTileRows = 64;
constexpr int kTileRowsOne = 16;
// Matrices per GEMMs launch (their views and outputs travel as kernel
// parameters).
constexpr int kMaxLaunchMats = 128;

struct LutParams {
    CqShape shape;
    const float *x;  // [rows][in] activations
    int act0;        // first activation of this launch (grid.y is relative)
    int n;           // matrices in this launch
    int tile_rows;   // kTileRows or kTileRowsOne
    CqView views[kMaxLaunchMats];
    float *y[kMaxLaunchMats];               // [rows][views[k].out] each
    int tile_start[kMaxLaunchMats + 1];     // prefix sum of row tiles
};

size_t lut_smem_bytes(const CqShape &s);
cudaError_t launch_lut(const LutParams &p, int tiles, int acts, cudaStream_t st);

// The cluster kernel for one (or a few) activations at low latency
// (cq_lut_split.cu): LutParams with tiles of 32 rows (split_tiles).
bool split_eligible(const CqShape &s);
size_t split_smem_bytes(const CqShape &s);
int split_tiles(int out);
cudaError_t launch_split(const LutParams &p, int tiles, int acts, cudaStream_t st);

// The streaming batch-1 kernel (cq_lut_stream.cu): views point at the
// "stream layout" (sidx/snrm) and tiles are 32 rows. Matrices come as
// strided runs: matrix i of a run is the view v with row0 + i·row_step,
// writing y + i·y_step (one matrix per run in general; many for a stack of
// views of one storage with evenly spaced outputs).
constexpr int kMaxStreamRuns = 256;
struct StreamRun {
    CqView v;          // the run's first matrix
    float *y;          // its output [v.out] (of the first activation)
    long long y_step;  // floats between consecutive matrices' outputs
    long long y_act;   // floats between consecutive activations' outputs
    int row_step;      // layout rows between consecutive matrices' row0
    int count;         // matrices in the run
    int tpm;           // 32-row tiles per matrix
    int tile0;         // the run's first tile in the launch
};
// Launches of few runs use a parameter block of kSmallStreamRuns runs: the
// block travels with every launch, and a small one launches faster.
constexpr int kSmallStreamRuns = 4;
template <int N>
struct StreamParamsN {
    CqShape shape;
    const float *x;   // the activations [acts][in]
    int acts;         // activations: the work is acts × total_tiles (activation-major)
    int nruns;
    int total_tiles;  // Σ count·tpm
    int smem_base;    // stream_smem_base() the launch was sized for
    // Partial row sums between table passes: null keeps them in the
    // outputs; otherwise [total_tiles][32] floats of device memory, so an
    // output is written once, by the last pass (outputs in host memory).
    float *part;
    // Device error word: the kernel records code 20 there when the shared
    // window does not start where the host sized it (and leaves NaN).
    int *err;
    StreamRun runs[N];
};
using StreamParams = StreamParamsN<kMaxStreamRuns>;
// Table passes of a stream launch (rows wider than one pass of byte tables
// take several, the partial sums carried between them).
int stream_passes(const CqShape &s);
// The tensor-core GEMM (cq_gemm_tc.cu): operand images are pre-swizzled
// 128 x 64 fp16 tiles, each scaled by a power of two.
constexpr int kMaxTcMats = 16;  // matrices one grouped tensor-core launch carries
struct TcMat {
    const unsigned char *b;  // ŵ image [n_tiles][kchunks][128][128 B]
    float *y;                // [m][ldy] fp32
    int n, ldy;
    int tile0;               // first n-tile of this matrix in the launch's grid
    float ws;                // 1 / the image's scale (a power of two)
};
struct TcParams {
    const unsigned char *a;  // x̂ image [m_tiles][kchunks][128][128 B], shared by the matrices
    const float *rs;         // [m_tiles·128]: 1 / each x̂ row's scale (a power of two)
    int m, kchunks;
    int *err;                // device error word (bounded waits)
    int nmats;               // matrices in this launch (1 .. kMaxTcMats)
    int pdl;                 // launched as a programmatic dependent of the rotation
    // Test hook (wc_testing_gemm_tc_stall): the producer issues no copies,
    // so the MMA and epilogue waits run out with nothing in flight; spin
    // bounds those waits (0: the default limit). Zero in every other call.
    int stall;
    uint32_t spin;
    TcMat mats[kMaxTcMats];
};
int tc_kchunks(const CqShape &s);
// The x̂ image of m rows alone, and with the rows' scales behind it (the
// buffer a rotation writes: tc_a_bytes).
size_t tc_a_image_bytes(int m, int kchunks);
size_t tc_a_bytes(int m, int kchunks);
size_t tc_b_bytes(int n, int kchunks);
size_t tc_smem_bytes();
// ŵ·wsc into the image b (wsc a power of two).
cudaError_t launch_dequant_f16(const CqShape &s, const CqView &v, float wsc, unsigned char *b, cudaStream_t st);
// x̂ of m rows into the buffer a (tc_a_bytes): the image, then the scales.
cudaError_t launch_rotate_f16(const CqShape &s, const float *x, int m, unsigned char *a, cudaStream_t st);
// Total n-tiles of a launch: mats[nmats - 1].tile0 + its tiles.
int tc_total_tiles(const TcParams &p);
cudaError_t launch_gemm_tc(const TcParams &p, cudaStream_t st);
// The persistent kernel for many rows: 128 x 256 tiles, mats[].tile0 in
// 256-row units.
size_t tc_persistent_smem_bytes();
cudaError_t launch_gemm_tc_persistent(const TcParams &p, cudaStream_t st);
// wc_cq_gemm_tc_noalloc's core: the same kernels on a static scratch array.
size_t noalloc_scratch_bytes();
cudaError_t gemm_tc_noalloc(const CqShape &s, const unsigned char *wimg, float ws, const float *x, float *y, int rows,
                            int n, int *err, bool persistent, cudaStream_t st);
// The static array's error word on the current device (null before the
// first no-allocation call there).
int *noalloc_err_word();

// The per-activation lut kernel (cq_lut_acts.cu): every row of up to
// kMaxActsMats matrices (group 128) per activation, tables built once.
constexpr int kMaxActsMats = 16;
struct ActsParams {
    CqShape shape;
    const float *x;  // [acts][in]
    int n;           // matrices
    int total_rows;  // Σ out
    int splits;      // CTAs per activation (grid.y), each a contiguous share of the rows
    CqView views[kMaxActsMats];
    float *y[kMaxActsMats];              // [acts][views[k].out]
    int row_start[kMaxActsMats + 1];     // prefix sum of rows
};
bool acts_eligible(const CqShape &s);
size_t acts_smem_bytes(const CqShape &s);
cudaError_t launch_lut_acts(const ActsParams &p, int acts, cudaStream_t st);

int stream_smem_base();
bool stream_eligible(const CqShape &s);
size_t stream_smem_bytes(const CqShape &s);
cudaError_t launch_stream(const StreamParams &p, int ctas, cudaStream_t st);

// The Exact path (kernel.go:162-373): one matrix, float32 nibble tables.
size_t exact_smem_bytes(const CqShape &s);
cudaError_t launch_exact(const CqShape &s, const CqView &v, const float *x, float *y, int rows, cudaStream_t st);

// matrix.go:161 Row for n rows (rows: device array, or NULL with n = 1 and
// row r0).
cudaError_t launch_row(const CqShape &s, const CqView &v, const int32_t *rows, int r0, int n, float *dst,
                       int32_t *bad, cudaStream_t st);

}  // namespace wb
