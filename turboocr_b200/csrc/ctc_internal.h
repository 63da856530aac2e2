// Launchers shared between the CTC translation units of libtocr_b200.so.
#pragma once

#include <cuda_runtime.h>

namespace tocr {

// The greedy collapse of per-step (argmax, max probability) rows into tokens,
// lengths and line scores (ctc_decode.cpp:25-48), one warp per line; lines
// [0, min(batch, *d_batch)) when d_batch is given. Returns a TOCR status.
int launch_ctc_collapse(const int *step_idx, const float *step_prob, int batch, int T,
                        int num_labels, int *tokens, int *lengths, float *scores,
                        const int *d_batch, cudaStream_t stream);

}  // namespace tocr
