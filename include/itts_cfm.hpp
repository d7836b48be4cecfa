// itts_cfm.hpp — header-only C++ shim over the C ABI (itts_cfm.h) that keeps
// the reference's CFM stage signature, so a C++ caller of
//   run_cfm_euler_metal(MetalContext&, const Bundle&, x, prompt, cond, style,
//                       tokens, prompt_tokens, steps, cfg_rate)
// (runtime/impl/dit_cfm_bigvgan.cpp:3121-3124) switches by changing the
// context type. Errors surface as std::runtime_error, as in the reference.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "itts_cfm.h"

namespace itts {

// Owns one engine context (device weights, tables, workspaces) on one GPU.
// Like mit2::MetalContext it is single-threaded: one per (thread, GPU).
class CudaCfmContext {
 public:
  explicit CudaCfmContext(const std::string& bundle_dir, int device = 0, bool verify_sha256 = false) {
    const int rc = itts_cfm_create_ex(bundle_dir.c_str(), device, verify_sha256 ? ITTS_CREATE_VERIFY_SHA256 : 0u, &h_);
    if (rc != ITTS_OK) throw std::runtime_error(std::string("itts_cfm_create: ") + itts_cfm_create_error());
  }
  ~CudaCfmContext() { itts_cfm_destroy(h_); }
  CudaCfmContext(const CudaCfmContext&) = delete;
  CudaCfmContext& operator=(const CudaCfmContext&) = delete;
  itts_cfm_ctx* get() const { return h_; }
  void check(int rc, const char* what) const {
    if (rc != ITTS_OK)
      throw std::runtime_error(std::string(what) + ": " + itts_cfm_strerror(rc) + ": " + itts_cfm_last_error(h_));
  }

 private:
  itts_cfm_ctx* h_ = nullptr;
};

// x: [tokens, 80] initial noise; prompt: [prompt_tokens, 80]; cond:
// [tokens, 512]; style: [192]. Returns the full mel [tokens, 80] with the
// prompt rows zeroed (same contract as run_cfm_euler_metal / run_cfm_euler_cpu).
inline std::vector<float> run_cfm_euler_cuda(CudaCfmContext& ctx, std::vector<float> x, const std::vector<float>& prompt,
                                             const std::vector<float>& cond, const std::vector<float>& style,
                                             uint32_t tokens, uint32_t prompt_tokens, uint32_t steps, float cfg_rate) {
  if (x.size() != static_cast<size_t>(tokens) * 80 || cond.size() != static_cast<size_t>(tokens) * 512 ||
      style.size() != 192 || prompt.size() < static_cast<size_t>(prompt_tokens) * 80)
    throw std::runtime_error("run_cfm_euler_cuda: input size mismatch");
  std::vector<float> out(x.size());
  ctx.check(itts_cfm_run(ctx.get(), x.data(), prompt_tokens ? prompt.data() : nullptr, cond.data(), style.data(), tokens,
                         prompt_tokens, steps, cfg_rate, out.data()),
            "run_cfm_euler_cuda");
  return out;
}

// One estimator evaluation (run_dit_estimator_step_cpu, runtime/impl/dit_cfm_bigvgan.cpp:1768):
// returns the conditional-branch velocity [tokens, 80].
inline std::vector<float> run_dit_estimator_step_cuda(CudaCfmContext& ctx, const std::vector<float>& x,
                                                      const std::vector<float>& prompt_x, const std::vector<float>& cond,
                                                      const std::vector<float>& style, float timestep,
                                                      const std::vector<uint32_t>& mask, uint32_t tokens) {
  if (x.size() != static_cast<size_t>(tokens) * 80 || prompt_x.size() != x.size() ||
      cond.size() != static_cast<size_t>(tokens) * 512 || style.size() != 192 || mask.size() != tokens)
    throw std::runtime_error("run_dit_estimator_step_cuda: input size mismatch");
  std::vector<float> vel(x.size());
  ctx.check(itts_cfm_estimator(ctx.get(), 1, tokens, 1, x.data(), prompt_x.data(), cond.data(), style.data(),
                               mask.data(), timestep, vel.data()),
            "run_dit_estimator_step_cuda");
  return vel;
}

// BigVGAN vocoder context (itts_vocoder_create): one per (thread, GPU).
class CudaVocoderContext {
 public:
  explicit CudaVocoderContext(const std::string& bundle_dir, int device = 0) {
    const int rc = itts_vocoder_create(bundle_dir.c_str(), device, &h_);
    if (rc != ITTS_OK) throw std::runtime_error(std::string("itts_vocoder_create: ") + itts_vocoder_create_error());
  }
  ~CudaVocoderContext() { itts_vocoder_destroy(h_); }
  CudaVocoderContext(const CudaVocoderContext&) = delete;
  CudaVocoderContext& operator=(const CudaVocoderContext&) = delete;
  itts_vocoder_ctx* get() const { return h_; }

 private:
  itts_vocoder_ctx* h_ = nullptr;
};

// Drop-in for run_bigvgan_vocoder_metal (runtime/impl/dit_cfm_bigvgan.cpp:4196):
// mel [tokens, 80] -> waveform [256 tokens] in [-1, 1].
inline std::vector<float> run_bigvgan_vocoder_cuda(CudaVocoderContext& ctx, std::vector<float> mel, uint32_t tokens) {
  if (mel.size() != static_cast<size_t>(tokens) * 80) throw std::runtime_error("run_bigvgan_vocoder_cuda: mel size mismatch");
  std::vector<float> wave(static_cast<size_t>(tokens) * 256);
  const int rc = itts_vocoder_run(ctx.get(), mel.data(), tokens, wave.data());
  if (rc != ITTS_OK)
    throw std::runtime_error(std::string("run_bigvgan_vocoder_cuda: ") + itts_cfm_strerror(rc) + ": " +
                             itts_vocoder_last_error(ctx.get()));
  return wave;
}

}  // namespace itts
