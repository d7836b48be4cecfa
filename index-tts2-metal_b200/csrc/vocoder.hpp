// BigVGAN vocoder (mel [T,80] -> waveform [256 T]) on the tcgen05 GEMM.
//
// Follows run_bigvgan_vocoder_cpu (runtime/impl/dit_cfm_bigvgan.cpp:4058-4061):
// conv_pre (k=7, 80 -> 1536), six stages of { transposed-conv upsampler,
// mean of three resblocks (kernels 3, 7, 11; each three pairs of anti-aliased
// SnakeBeta -> dilated conv -> SnakeBeta -> conv, + residual) }, then the
// post activation, conv_post (k=7, 24 -> 1) and a clamp to [-1, 1].
//
// Every conv is an implicit GEMM (gemm_tc_kernel, A-mode kAConv: one row
// shift per tap, zero rows outside the utterance from TMA's out-of-bounds
// fill); a transposed conv of stride s runs as s phase GEMMs of two taps each
// whose outputs interleave (row s q + r). The activations are a tiled CUDA
// kernel; a CUDA graph per utterance length replays the whole schedule.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "engine.hpp"
#include "gemm.cuh"

namespace itts {

// One GEMM-shaped conv (or one phase of a transposed conv) in device memory.
struct VocConv {
  const __half* w = nullptr;  // [cout][taps][cin_pad] f16, zero for channels >= cin
  const float* bias = nullptr;  // [cout]
  int cin = 0, cin_pad = 0, cout = 0, taps = 0;
  int dil = 1, off = 0;  // A row of tap i: m + i * dil + off
};

// Anti-aliased SnakeBeta parameters of one activation.
struct VocAct {
  const float* alpha = nullptr;     // [C] exp(alpha_log)
  const float* inv_beta = nullptr;  // [C] 1 / (exp(beta_log) + 1e-9)
  float up[12] = {};                // anti-aliasing filters (host copies, passed to the kernel by value)
  float down[12] = {};
  int c = 0;
};

struct VocStage {
  int cin = 0, cout = 0, k = 0, s = 0, p = 0;  // upsampler
  std::vector<VocConv> phase;                  // s phase GEMMs of the upsampler
  VocConv conv1[3][3], conv2[3][3];            // [resblock][pair]
  VocAct act[3][6];                            // [resblock][activation]
};

class Vocoder {
 public:
  Vocoder(const std::string& bundle_dir, int device, bool verify_sha256);
  ~Vocoder();
  Vocoder(const Vocoder&) = delete;
  Vocoder& operator=(const Vocoder&) = delete;

  // Host mel [T,80] -> host waveform [256 T] (upload, graph replay, download).
  void run(const float* mel, int T, float* wave);
  // Device-resident pieces of run(), for timing: stage() uploads a mel and
  // builds (once per T) the plan and graph; launch() replays the graph.
  void stage(const float* mel, int T);
  void launch();
  void fetch(float* wave);
  // Event-timed launches of one vocoder pass over the staged mel, per kernel kind.
  std::vector<KernelTiming> profile(int reps);
  int launches_per_run() const;
  // Algorithmic FLOPs of one pass over T mel frames (conv MACs x 2).
  static double flops(int T);
  cudaStream_t stream() const { return stream_; }
  int device() const { return device_; }
  unsigned int read_status();
  void clear_status();

 private:
  struct Plan;
  void load(const std::string& bundle_dir, bool verify_sha256);
  Plan* plan_for(int T);
  void enqueue(Plan* p, std::vector<KernelTiming>* prof);
  void check(cudaError_t e, const char* what);

  int device_ = 0;
  cudaStream_t stream_ = nullptr;
  unsigned int* d_status_ = nullptr;
  void* arena_ = nullptr;
  VocConv pre_;
  VocStage st_[6];
  VocAct post_act_;
  const float* post_w_ = nullptr;  // [24][7] conv_post (no bias)
  std::map<int, std::unique_ptr<Plan>> plans_;
  Plan* staged_ = nullptr;
};

}  // namespace itts
