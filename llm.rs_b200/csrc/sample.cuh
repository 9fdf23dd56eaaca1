// sample.cuh - device-side next-token sampling (host interface).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace llmrs {

constexpr int SAMPLE_MAX_RECENT = 4096; // recent ids the repetition penalty may look at

// scratch bytes sample_launch needs for a vocabulary of V
size_t sample_scratch_bytes(int V);
// sample one token from d_logits[V] (see sample.cu); blocks until *h_token is set
int sample_launch(const float *d_logits, int V, const int *h_recent, int n_recent, float penalty, float temperature,
                  float top_p, float u, void *scratch, int *h_token, cudaStream_t stream);

} // namespace llmrs
