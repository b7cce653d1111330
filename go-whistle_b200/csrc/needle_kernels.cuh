// needle_kernels.cuh — launch interfaces of the int8 kernels (int8_attend.cu)
// used by the C-ABI layer (api.cu).
#pragma once

#include "common.cuh"

namespace wb {

struct AttendParams {
    const float *q;    // [streams][t][heads][qk]
    const int8_t *k8;  // stream b at b*cap rows: [cap][kv_heads*qk]
    const float *ks;   // [cap][kv_heads]
    const int8_t *v8;  // [cap][kv_heads*vd]
    const float *vs;   // [cap][kv_heads]
    const int32_t *spans;     // [t][4] or NULL (all keys)
    const int32_t *nkeys_dev; // [streams] or NULL (nkeys for every stream)
    float *probs;             // [streams][t][heads][nkeys] or NULL
    float *out;               // [streams][t][heads][vd]
    int t, heads, kv_heads, qk, vd;
    int nkeys;     // keys of the single-stream call (probs row length)
    int cap;       // rows between consecutive streams' caches
    int max_keys;  // upper bound of keys any query row sees (shared memory)
    float scale;
    int quant_q;
    int k_aligned4;  // k8 rows and q8 readable as int32 words
    int kv_per_cta;  // v2 and any-order: KV heads per CTA
    int v_prefetch;  // any-order: V row slices are 16-byte aligned (L2 prefetch)
    int *err;        // bulk kernel: device error word of its bounded waits
    int bulk_whole;  // bulk kernel: the CTA holds every KV head (contiguous chunks)
    int bulk_scales; // bulk kernel: scale chunks start 16-byte aligned (cap·kv_heads % 4 == 0)
    int kv_group;    // streams per K/V block: stream b reads block b / kv_group (0 or 1: its own)
};

// The K/V block stream b reads.
__host__ __device__ inline size_t kv_block(const AttendParams &p, int b) {
    return (size_t)(p.kv_group > 1 ? b / p.kv_group : b);
}

// Shared-memory layout of the bulk kernel (int8_attend_bulk.cu), in bytes.
struct BulkLayout {
    size_t stage, scale_off;  // one ring stage; its scale block
    size_t lg, q8, qf, red, bars, total;
    int lstride;              // floats per head row of logits
    int stages;               // ring stages
};

cudaError_t launch_quantize_rows(const float *x, int chunks, int width, int8_t *q, float *s, cudaStream_t st);
// The decoder head's scale and greedy argmax (decode_head.cu).
cudaError_t launch_head_argmax(const float *y, int rows, int vocab, float head, float *logits, int32_t *idx,
                               cudaStream_t st);
size_t attend_smem_bytes(const AttendParams &p);
cudaError_t launch_attend(const AttendParams &p, int streams, cudaStream_t st);
size_t attend_any_smem_bytes(const AttendParams &p);
bool attend_any_supported(const AttendParams &p);
cudaError_t launch_attend_any(const AttendParams &p, int streams, cudaStream_t st);
size_t attend_v2_smem_bytes(const AttendParams &p);
cudaError_t launch_attend_v2(const AttendParams &p, int streams, cudaStream_t st);
BulkLayout attend_bulk_layout(const AttendParams &p, int stages);
BulkLayout attend_bulk_pick_layout(const AttendParams &p, size_t smem_per_sm, size_t smem_per_block, int share);
bool attend_bulk_shape_ok(const AttendParams &p, int kvpc);
cudaError_t attend_bulk_occupancy(const AttendParams &p, const BulkLayout &L, bool exact, int *blocks_per_sm);
cudaError_t launch_attend_bulk(const AttendParams &p, const BulkLayout &L, int streams, bool exact, cudaStream_t st);

}  // namespace wb
