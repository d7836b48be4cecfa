// Persistent GPT decoder kernel: one cooperative launch runs the prefill rows
// and every decode step of a generate call (see gpt_persist.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace itts {

// Device pointers of one GPT-2 block (weights [out][in] f16).
struct GptLayerPtrs {
  const float *ln1_g, *ln1_b, *b_attn, *b_proj, *ln2_g, *ln2_b, *b_fc, *b_mproj;
  const __half *w_attn, *w_proj, *w_fc, *w_mproj;
};

struct GptPersistParams {
  const GptLayerPtrs* layers;  // device [24]
  const float *lnf_g, *lnf_b, *fn_g, *fn_b, *b_head;
  const __half* w_head;       // [8194][1280]
  const float *emb, *pos;     // [8194][1280], [1818][1280]
  const float* prefix;        // [P][1280]
  float *x, *h, *qkv, *m, *logits, *kc, *vc, *part;
  float* cand_val;            // [grid] per-CTA best logit of the head stage
  int* cand_idx;              // [grid]
  uint32_t* codes;            // [max_steps]
  int* out;                   // [0] codes produced
  unsigned int* barrier;      // grid barrier arrival counter, zero at launch
  unsigned int* status;       // nonzero: a bounded wait gave up
  unsigned long long* times;  // globaltimer at start, end of prefill, end
  int P, max_steps;
  int len0;          // KV cache rows already filled (a batched prefill), prefix rows P after them
  int hf_positions;  // nonzero: decode step s > 0 takes position embedding s + 1
  // Optional stage trace of the first decode token: CTA 0's global timer when
  // the token starts and, per stage, when its prologue is done, when its first
  // warp has finished its weight slots, when its compute is done and when its
  // grid barrier is passed (kGptTraceCap entries); then every CTA's barrier
  // arrival per stage ([121][grid]).
  unsigned long long* trace;
  // Sampled decode (the reference's GptSamplingConfig with do_sample): when
  // `sample` is nonzero CTA 0 draws each code after the head stage.
  int sample;
  float temperature, top_p, repetition_penalty;
  int top_k;                 // 1..kGptSampleMaxFinite
  unsigned long long seed;
  const uint32_t* history;   // repetition history before the codes (device)
  int n_history;             // 0: [8192]
  unsigned int* seen;        // [ceil(8194 / 32)] seen-token bitmap (device scratch)
  unsigned long long* rng;   // SplitMix64 state (device scratch)
  int* sampled;              // the drawn code, read by every CTA after a barrier
};

// Largest finite set the sampler sorts in shared memory (top_k's upper bound).
constexpr int kGptSampleMaxFinite = 2048;

constexpr int kGptTraceCap = 1 + 121 * 4;
constexpr int kGptTraceStages = 121;

// Dynamic shared memory of one CTA; the one-time function attribute; the
// launch (cooperative, one CTA per SM, `grid` CTAs).
size_t gpt_persist_smem();
cudaError_t gpt_persist_prepare();
cudaError_t gpt_persist_launch(const GptPersistParams& p, int grid, cudaStream_t st);
// Smallest grid the kernel supports (the head's rows of one CTA must fit its
// per-stage task table).
int gpt_persist_min_grid();

}  // namespace itts
