/*
 * decoder_oracle.c — CPU restatement of the decoder's head and greedy
 * choice (TEST INFRASTRUCTURE ONLY: the checker of the CUDA kernel).
 */
#include <math.h>

#include "oracle.h"

/*
 * internal/decoder/decoder.go:508-523 logits (the scale part: out[i] *= head
 * when head != 1) and internal/decoder/greedy.go:182 argmax (the first index
 * of the largest value: best starts at 0 and moves only on x > v[best], so
 * a NaN at 0 keeps 0, later NaNs never win, and +0 and -0 tie).
 */
void wo_head_argmax(const float *y, int rows, int vocab, float head, float *logits, int32_t *idx) {
    for (int r = 0; r < rows; r++) {
        const float *v = y + (long)r * vocab;
        float *o = logits + (long)r * vocab;
        for (int i = 0; i < vocab; i++) o[i] = head != 1.0f ? v[i] * head : v[i];
        int best = 0;
        for (int i = 0; i < vocab; i++)
            if (o[i] > o[best]) best = i;
        idx[r] = best;
    }
}
