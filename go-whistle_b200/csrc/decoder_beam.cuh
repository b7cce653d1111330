// decoder_beam.cuh — the device decoder's interface for the beam search
// (beam.cu): one step for every stream with the exact head, the candidates
// of listed rows, and forks of stream states.
#pragma once

#include "common.cuh"

namespace wb {

struct DecBeamInfo {
    int streams;    // decoder streams (clips × beams)
    int group;      // streams per clip (their shared cross memory)
    int len;        // positions so far (every stream alike)
    int positions;  // positions the caches and RoPE tables hold
    int vocab;
};

wc_status dec_beam_info(const wc_decoder *d, DecBeamInfo *out);
// Feeds one token per stream (host [streams]), runs the step and the exact
// head: the logits of every stream in the decoder's buffer.
wc_status dec_beam_feed(wc_decoder *d, const int32_t *tokens, cudaStream_t st);
// For each listed stream (host rows[nrows]): its n best tokens by logit
// (ties to the lower id), or the n best of allowed (ties to the earlier
// entry), with their logits, and the row's float64 log-sum-exp; into host
// arrays tok/logit [nrows][n] and lse [nrows]. Synchronises st.
wc_status dec_beam_top(wc_decoder *d, const int32_t *rows, int nrows, int n, const int32_t *allowed, int nallowed,
                       int32_t *tok, float *logit, double *lse, cudaStream_t st);
// Copies the state of stream pairs[2i] into stream pairs[2i+1] for every
// pair (host array). No destination may be a source.
wc_status dec_beam_fork(wc_decoder *d, const int32_t *pairs, int npairs, cudaStream_t st);

}  // namespace wb
