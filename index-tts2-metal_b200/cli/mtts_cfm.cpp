// mtts_cfm — C++ host driver over the C ABI, mirroring the reference CLI's
// CFM benchmark mode (`mtts --bench-cfm BUNDLE T STEPS ITERS`,
// runtime/main.cpp:2925-2930 -> run_bench_cfm, runtime/impl/dit_cfm_bigvgan.cpp:3065-3096):
// deterministic sin/cos inputs, prompt_tokens = 6T/7, CFG 0.7, one warm-up
// call, then ITERS timed calls of the full sampler; prints a JSON report.
//
//   mtts_cfm --bench-cfm BUNDLE T STEPS ITERS [DEVICE]
//   mtts_cfm --cfm BUNDLE T P STEPS CFG IN_PREFIX OUT.f32 [DEVICE]
//       reads IN_PREFIX.{noise,prompt,cond,style}.f32 (raw little-endian
//       float32), writes the mel [T,80] to OUT.f32.
//   mtts_cfm --inspect-model-bundle DIR [cfm,length_regulator,bigvgan,gpt]
//   mtts_cfm --inspect-voice-bundle DIR
//       the bundle contract gates (reference: runtime/main.cpp:2688-2691);
//       print the JSON report, exit 0 when the contract holds, 1 otherwise.
//   mtts_cfm --gpt BUNDLE P STEPS PREFIX.f32 OUT.u32 [SEED TEMP TOP_K TOP_P PENALTY] [DEVICE]
//       GPT mel-code decode of a prefix [P,1280] (raw float32) with
//       generate-style positions, as the synthesis pipeline calls it
//       (runtime/impl/tts_synthesis/synthesis_pipeline.cpp:675, 795):
//       greedy, or sampled when the five sampling values are given; writes
//       the codes (uint32) to OUT.u32 and prints a JSON report.
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <string>
#include <vector>

#include "itts_cfm.hpp"

namespace {

std::vector<float> read_f32(const std::string& path, size_t count) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("cannot open " + path);
  std::vector<float> v(count);
  f.read(reinterpret_cast<char*>(v.data()), static_cast<std::streamsize>(count * sizeof(float)));
  if (static_cast<size_t>(f.gcount()) != count * sizeof(float)) throw std::runtime_error("short read: " + path);
  return v;
}

int bench_cfm(const std::string& bundle, uint32_t tokens, uint32_t steps, uint32_t iters, int device) {
  itts::CudaCfmContext ctx(bundle, device);
  const uint32_t prompt_tokens = tokens * 6 / 7;
  std::vector<float> x(static_cast<size_t>(tokens) * 80), prompt(static_cast<size_t>(prompt_tokens) * 80),
      cond(static_cast<size_t>(tokens) * 512), style(192);
  for (size_t i = 0; i < x.size(); ++i) x[i] = std::sin(static_cast<float>(i) * 0.013f) * 0.4f;
  for (size_t i = 0; i < prompt.size(); ++i) prompt[i] = std::cos(static_cast<float>(i) * 0.011f) * 0.5f;
  for (size_t i = 0; i < cond.size(); ++i) cond[i] = std::sin(static_cast<float>(i) * 0.007f) * 0.3f;
  for (size_t i = 0; i < style.size(); ++i) style[i] = std::cos(static_cast<float>(i) * 0.015f) * 0.18f;
  auto mel = itts::run_cfm_euler_cuda(ctx, x, prompt, cond, style, tokens, prompt_tokens, steps, 0.7f);  // warm
  const auto t0 = std::chrono::steady_clock::now();
  for (uint32_t i = 0; i < iters; ++i) mel = itts::run_cfm_euler_cuda(ctx, x, prompt, cond, style, tokens, prompt_tokens, steps, 0.7f);
  const double total = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  double checksum = 0.0;
  for (float v : mel) checksum += v;
  std::printf("{\n  \"stage\": \"bench_cfm\",\n  \"tokens\": %u,\n  \"steps\": %u,\n  \"iters\": %u,\n", tokens, steps, iters);
  std::printf("  \"seconds_per_call\": %.6f,\n  \"ms_per_step\": %.6f,\n  \"mel_checksum\": %.6f\n}\n", total / iters,
              total / iters / steps * 1000.0, checksum);
  return 0;
}

int run_cfm(int argc, char** argv) {
  if (argc < 9) {
    std::fprintf(stderr, "usage: mtts_cfm --cfm BUNDLE T P STEPS CFG IN_PREFIX OUT.f32 [DEVICE]\n");
    return 2;
  }
  const std::string bundle = argv[2];
  const uint32_t T = static_cast<uint32_t>(std::strtoul(argv[3], nullptr, 10));
  const uint32_t P = static_cast<uint32_t>(std::strtoul(argv[4], nullptr, 10));
  const uint32_t steps = static_cast<uint32_t>(std::strtoul(argv[5], nullptr, 10));
  const float cfg = std::strtof(argv[6], nullptr);
  const std::string in = argv[7];
  const int device = argc > 9 ? std::atoi(argv[9]) : 0;
  itts::CudaCfmContext ctx(bundle, device);
  auto mel = itts::run_cfm_euler_cuda(ctx, read_f32(in + ".noise.f32", T * 80ull), read_f32(in + ".prompt.f32", P * 80ull),
                                      read_f32(in + ".cond.f32", T * 512ull), read_f32(in + ".style.f32", 192), T, P,
                                      steps, cfg);
  std::ofstream o(argv[8], std::ios::binary);
  o.write(reinterpret_cast<const char*>(mel.data()), static_cast<std::streamsize>(mel.size() * sizeof(float)));
  return o ? 0 : 1;
}

int run_gpt(int argc, char** argv) {
  if (argc < 7) {
    std::fprintf(stderr, "usage: mtts_cfm --gpt BUNDLE P STEPS PREFIX.f32 OUT.u32 [SEED TEMP TOP_K TOP_P PENALTY] [DEVICE]\n");
    return 2;
  }
  const uint32_t P = static_cast<uint32_t>(std::strtoul(argv[3], nullptr, 10));
  const uint32_t steps = static_cast<uint32_t>(std::strtoul(argv[4], nullptr, 10));
  const bool sampled = argc >= 12;
  const int device = sampled ? (argc > 12 ? std::atoi(argv[12]) : 0) : (argc > 7 ? std::atoi(argv[7]) : 0);
  const std::vector<float> prefix = read_f32(argv[5], static_cast<size_t>(P) * ITTS_GPT_WIDTH);
  itts_gpt_ctx* g = nullptr;
  if (itts_gpt_create(argv[2], device, &g) != ITTS_OK) throw std::runtime_error(itts_gpt_create_error());
  std::vector<uint32_t> codes(steps > 0 ? steps : 1);
  std::vector<float> logits(ITTS_GPT_VOCAB);
  uint32_t n = 0;
  int rc;
  if (sampled) {
    itts_gpt_sampling s{std::strtoull(argv[7], nullptr, 10), std::strtof(argv[8], nullptr),
                        static_cast<uint32_t>(std::strtoul(argv[9], nullptr, 10)), std::strtof(argv[10], nullptr),
                        std::strtof(argv[11], nullptr)};
    rc = itts_gpt_generate_sampled(g, prefix.data(), P, steps, ITTS_GPT_HF_POSITIONS, &s, nullptr, 0, codes.data(), &n,
                                   logits.data());
  } else {
    rc = itts_gpt_generate_ex(g, prefix.data(), P, steps, ITTS_GPT_HF_POSITIONS, codes.data(), &n, logits.data());
  }
  if (rc != ITTS_OK) {
    const std::string msg = itts_gpt_last_error(g);
    itts_gpt_destroy(g);
    throw std::runtime_error(msg);
  }
  float prefill_ms = 0.0f, decode_ms = 0.0f;
  itts_gpt_timing(g, &prefill_ms, &decode_ms);
  itts_gpt_destroy(g);
  std::ofstream o(argv[6], std::ios::binary);
  o.write(reinterpret_cast<const char*>(codes.data()), static_cast<std::streamsize>(n * sizeof(uint32_t)));
  const int first_stop = (n > 0 && codes[n - 1] == ITTS_GPT_STOP) ? static_cast<int>(n - 1) : -1;
  std::printf("{\n  \"stage\": \"gpt_%s\",\n  \"prefix_tokens\": %u,\n  \"codes\": %u,\n", sampled ? "sampled" : "greedy",
              P, n);
  std::printf("  \"first_stop_step\": %d,\n  \"prefill_ms\": %.4f,\n  \"decode_ms_per_token\": %.5f\n}\n", first_stop,
              prefill_ms, n ? decode_ms / n : 0.0);
  return o ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
  try {
    if (argc >= 6 && std::strcmp(argv[1], "--bench-cfm") == 0) {
      return bench_cfm(argv[2], static_cast<uint32_t>(std::strtoul(argv[3], nullptr, 10)),
                       static_cast<uint32_t>(std::strtoul(argv[4], nullptr, 10)),
                       static_cast<uint32_t>(std::strtoul(argv[5], nullptr, 10)), argc > 6 ? std::atoi(argv[6]) : 0);
    }
    if (argc >= 2 && std::strcmp(argv[1], "--cfm") == 0) return run_cfm(argc, argv);
    if (argc >= 2 && std::strcmp(argv[1], "--gpt") == 0) return run_gpt(argc, argv);
    if (argc >= 3 && (std::strcmp(argv[1], "--inspect-model-bundle") == 0 ||
                      std::strcmp(argv[1], "--inspect-voice-bundle") == 0)) {
      std::string report(1 << 16, '\0');
      int rc;
      if (argv[1][10] == 'v') {
        rc = itts_inspect_voice_bundle(argv[2], &report[0], static_cast<uint32_t>(report.size()));
      } else {
        uint32_t mask = 0;
        const std::string comps = argc > 3 ? argv[3] : "cfm";
        if (comps.find("cfm") != std::string::npos) mask |= ITTS_COMPONENT_CFM;
        if (comps.find("length_regulator") != std::string::npos) mask |= ITTS_COMPONENT_LENGTH_REGULATOR;
        if (comps.find("bigvgan") != std::string::npos) mask |= ITTS_COMPONENT_BIGVGAN;
        if (comps.find("gpt") != std::string::npos) mask |= ITTS_COMPONENT_GPT;
        rc = itts_inspect_model_bundle(argv[2], mask, &report[0], static_cast<uint32_t>(report.size()));
      }
      std::printf("%s\n", report.c_str());
      return rc == ITTS_OK ? 0 : 1;
    }
    std::fprintf(stderr, "usage: mtts_cfm --bench-cfm BUNDLE T STEPS ITERS [DEVICE]\n"
                         "       mtts_cfm --cfm BUNDLE T P STEPS CFG IN_PREFIX OUT.f32 [DEVICE]\n"
                         "       mtts_cfm --inspect-model-bundle DIR [cfm,length_regulator,bigvgan,gpt]\n"
                         "       mtts_cfm --inspect-voice-bundle DIR\n"
                         "       mtts_cfm --gpt BUNDLE P STEPS PREFIX.f32 OUT.u32 [SEED TEMP TOP_K TOP_P PENALTY] [DEVICE]\n");
    return 2;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "error: %s\n", e.what());
    return 1;
  }
}
