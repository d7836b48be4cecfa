// GPT mel-code decoder: cached greedy decode of mel codes from a prefix of
// input embeddings.
//
// Follows run_gpt_kv_greedy_cpu (runtime/impl/gpt.cpp:1877-1909) and its
// pieces (:1060-1210, 1545-1554, 1796-1806): 24 GPT-2 blocks (LayerNorm ->
// c_attn 1280 -> 3840 -> 20-head attention over the KV cache -> c_proj +
// residual; LayerNorm -> c_fc 1280 -> 5120 -> gelu_new -> c_proj + residual),
// ln_f, final_norm, mel head (8194 codes), argmax; the next input is the
// code's mel embedding plus the step's position embedding; start code 8192,
// stop code 8193.
//
// One token at a time is bandwidth- and latency-bound (about 1 GB of f16
// weights per token, in a chain of 121 dependent all-to-all steps). The
// product path is one persistent cooperative kernel per generate call
// (gpt_persist.cu): the steps are stages separated by grid barriers, and a
// producer warp per SM streams the weights through a shared-memory ring
// ahead of them. The per-kernel path (ITTS_GPT_MODE=graph in the
// environment, a diagnostic) runs the same math as weight-streaming GEMV
// kernels with programmatic dependent launch, one CUDA graph per token. Both
// use fp32 activations, accumulation and KV cache, and split each head's
// keys over 7 ranges with the softmax merged in the next projection.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "gpt_persist.cuh"
#include "gpt_prefill.cuh"

namespace itts {

class GptDecoder {
 public:
  GptDecoder(const std::string& bundle_dir, int device, bool verify_sha256);
  ~GptDecoder();
  GptDecoder(const GptDecoder&) = delete;
  GptDecoder& operator=(const GptDecoder&) = delete;

  // prefix [P,1280] (host) -> up to max_steps codes (host); stops after the
  // stop code (included, as the reference's predicted tokens). Returns the
  // number of codes; last_logits (optional, host [8194]) of the last step.
  // hf_positions: the reference's hf_generate_positions (decode step s > 0
  // at position s + 1), as its synthesis pipeline calls the decoder.
  int generate(const float* prefix, int P, int max_steps, bool hf_positions, uint32_t* codes, float* last_logits);

  // The reference's GptSamplingConfig with do_sample (runtime/impl/gpt.cpp:
  // 1592-1599): repetition penalty, temperature, top-k, top-p, SplitMix64 seed.
  struct Sampling {
    unsigned long long seed = 0;
    float temperature = 1.0f;
    int top_k = 0;  // 1..2048 (the finite set the device sorts)
    float top_p = 1.0f;
    float repetition_penalty = 1.0f;
  };
  // As generate, drawing each code from the processed logits instead of the
  // argmax; history (host, n_history tokens; NULL/0 = [8192]) is the
  // repetition history before the codes. Persistent path only.
  int generate_sampled(const float* prefix, int P, int max_steps, bool hf_positions, const Sampling& sampling,
                       const uint32_t* history, int n_history, uint32_t* codes, float* last_logits);
  // Device time of the last generate call's prefill and decode parts (ms).
  float last_prefill_ms() const { return prefill_ms_; }
  float last_decode_ms() const { return decode_ms_; }
  int last_steps() const { return steps_; }
  int kernels_per_token() const { return decode_kernels_; }
  // Kernel launches of the last generate call (1 for the persistent kernel).
  long long last_launches() const { return launches_; }
  bool persistent() const { return persistent_; }
  // Stage trace of the last persistent generate's first decode token: the
  // microseconds since the token started at each trace point (see
  // GptPersistParams::trace); empty unless the decoder traces.
  int stage_trace(double* us, int cap);
  void set_tracing(bool on) { tracing_ = on; }
  cudaStream_t stream() const { return stream_; }
  int device() const { return device_; }
  // f16 weight bytes one decode step streams (all projections and the head).
  static double weight_bytes_per_token();

  static constexpr int kLayers = 24, kW = 1280, kQkv = 3840, kMlp = 5120, kVocab = 8194, kPositions = 1818;
  static constexpr int kHeads = 20, kHd = 64, kStart = 8192, kStop = 8193;
  static constexpr int kMaxLen = 4096;  // prefix rows + decode steps held in the KV cache

 private:
  using Layer = GptLayerPtrs;
  void check(cudaError_t e, const char* what);
  void enqueue_layers();
  void build_graphs();
  int generate_persistent(int P, int max_steps);
  int generate_common(const float* prefix, int P, int max_steps, bool hf_positions, uint32_t* codes,
                      float* last_logits);
  int generate_graphs(int P, int max_steps);

  int device_ = 0;
  cudaStream_t stream_ = nullptr;
  cudaEvent_t ev_[3] = {nullptr, nullptr, nullptr};
  void* arena_ = nullptr;
  void* state_ = nullptr;
  Layer L_[kLayers];
  const float *lnf_g_ = nullptr, *lnf_b_ = nullptr, *fn_g_ = nullptr, *fn_b_ = nullptr, *b_head_ = nullptr;
  const __half* w_head_ = nullptr;
  const float *emb_ = nullptr, *pos_ = nullptr;  // [8194][1280], [1818][1280] (fp32)
  // device state
  float *x_ = nullptr, *h_ = nullptr, *qkv_ = nullptr, *m_ = nullptr, *logits_ = nullptr;
  float* part_ = nullptr;  // attention partials [20 heads][key ranges][max, sum, 64 accumulators]
  float *kc_ = nullptr, *vc_ = nullptr;  // [24][kMaxLen][1280]
  float* prefix_ = nullptr;              // [kMaxLen][1280]
  // [0] cache length, [1] prefill row, [2] step, [3] current code, [4] stopped, [5] max steps,
  // [6] generate-style positions
  int* ctl_ = nullptr;
  uint32_t* codes_ = nullptr;  // [kPositions]
  unsigned int* status_ = nullptr;  // nonzero: a kernel abandoned a bounded wait
  int sms_ = 148;
  // persistent-kernel state
  bool persistent_ = true;
  GptLayerPtrs* layers_dev_ = nullptr;
  float* cand_val_ = nullptr;
  int* cand_idx_ = nullptr;
  unsigned int* barrier_ = nullptr;
  int* out_ = nullptr;
  unsigned long long* times_ = nullptr;
  long long launches_ = 0;
  bool hf_ = false;
  bool sample_ = false;
  Sampling sampling_;
  int n_history_ = 0;
  uint32_t* history_ = nullptr;       // [kMaxLen] device copy of the repetition history
  unsigned int* seen_ = nullptr;      // sampler scratch: seen-token bitmap
  unsigned long long* rng_ = nullptr; // sampler scratch: SplitMix64 state
  int* sampled_ = nullptr;            // sampler scratch: the drawn code
  // batched prefill (all prefix rows per layer at once) before the persistent
  // decode; ITTS_GPT_PREFILL=rows in the environment keeps the row-by-row
  // pass inside the persistent kernel (a diagnostic)
  bool batched_prefill_ = true;
  GptPrefillBuffers pf_{};
  bool tracing_ = false;
  unsigned long long* trace_ = nullptr;  // [kGptTraceCap]
  cudaGraphExec_t g_prefill_ = nullptr, g_decode_ = nullptr;
  int decode_kernels_ = 0, prefill_kernels_ = 0;
  float prefill_ms_ = 0.0f, decode_ms_ = 0.0f;
  int steps_ = 0;
};

}  // namespace itts
