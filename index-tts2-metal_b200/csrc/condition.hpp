// Condition assembly before the CFM sampler (the length regulator and the
// prompt-condition merge): s_infer [n_in, 1024] -> length regulator -> [G, 512],
// placed after the voice prompt's P condition rows: cond [P + G, 512].
//
// Follows run_length_regulator_full_metal / _cpu (runtime/impl/gpt.cpp:
// 5298-5317, 5271-5281) and mit2_hot_condition_merge_f32
// (metal/kernels.metal:843-864, called at
// runtime/impl/tts_synthesis/synthesis_pipeline.cpp:1030-1034):
// content_in_proj (1024 -> 512, tcgen05 GEMM), nearest interpolation to G
// rows, four { k=3 conv (implicit GEMM), one-group GroupNorm, Mish }, a k=1
// conv whose epilogue writes straight into cond rows [P, P + G).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <string>
#include <tuple>

#include "gemm.cuh"

namespace itts {

class ConditionAssembler {
 public:
  ConditionAssembler(const std::string& bundle_dir, int device, bool verify_sha256);
  ~ConditionAssembler();
  ConditionAssembler(const ConditionAssembler&) = delete;
  ConditionAssembler& operator=(const ConditionAssembler&) = delete;

  // Host in / host out: s_infer [n_in,1024], prompt [P,512] -> cond [P+G,512].
  void run(const float* s_infer, int n_in, const float* prompt, int P, int G, float* cond);
  // Device-resident pieces of run(), for timing.
  void stage(const float* s_infer, int n_in, const float* prompt, int P, int G);
  void launch();
  void fetch(float* cond);
  int launches_per_run() const;
  static double flops(int n_in, int G);
  cudaStream_t stream() const { return stream_; }
  int device() const { return device_; }
  unsigned int read_status();
  void clear_status();

 private:
  struct Plan;
  Plan* plan_for(int n_in, int P, int G);
  void enqueue(Plan* p);
  void check(cudaError_t e, const char* what);

  int device_ = 0;
  cudaStream_t stream_ = nullptr;
  unsigned int* d_status_ = nullptr;
  void* arena_ = nullptr;
  const __half* w_in_ = nullptr;   // [512][1024]
  const float* b_in_ = nullptr;    // [512]
  const __half* w_conv_[4] = {};   // [512][3][512]
  const float* b_conv_[4] = {};
  const float* gn_g_[4] = {};      // GroupNorm gamma / beta [512]
  const float* gn_b_[4] = {};
  const __half* w_out_ = nullptr;  // [512][512]
  const float* b_out_ = nullptr;
  std::map<std::tuple<int, int, int>, std::unique_ptr<Plan>> plans_;
  Plan* staged_ = nullptr;
};

}  // namespace itts
