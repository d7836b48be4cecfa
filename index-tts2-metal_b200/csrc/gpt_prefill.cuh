// Batched GPT prefill: all P prefix rows through each of the 24 blocks at
// once (see gpt_prefill.cu), filling the KV cache rows [0, P).
#pragma once

#include <cuda_runtime.h>

#include "gpt_persist.cuh"

namespace itts {

struct GptPrefillBuffers {
  float* x;     // [P][1280] residual stream (the prefix rows on entry; overwritten)
  float* h;     // [P][1280]
  float* xn;    // [P][1280] normalised rows
  float* q;     // [P][1280]
  float* attn;  // [P][1280]
  float* m;     // [P][5120]
  float* part;  // [4][P][1280] K-split partials
  float *kc, *vc;  // [24][4096][1280] caches
};

// Enqueues the prefill of P rows (1..4096) on `st`; returns the first launch
// error. Kernels launched: 9 per layer.
cudaError_t gpt_prefill_enqueue(const GptLayerPtrs* layers_host, const GptPrefillBuffers& b, int P, cudaStream_t st);
cudaError_t gpt_prefill_prepare();
int gpt_prefill_kernels_per_call();

}  // namespace itts
