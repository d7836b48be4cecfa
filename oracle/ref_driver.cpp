// TEST INFRASTRUCTURE — C entry points over the reference's own CPU functions.
//
// oracle/build_ref.py compiles this file together with the reference's CPU
// DiT-CFM functions, taken verbatim by line range from the read-only reference
// tree into the git-ignored oracle/_ref/ref_tu.cpp, and runtime/bundle.cpp,
// producing oracle/_ref/libref_cfm.so. Only tests/golden/make_golden.py and
// bench.py's reference arm load it; the product never does.
#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "mit2/bundle.hpp"

// Reference functions (defined in oracle/_ref/ref_tu.cpp).
std::vector<float> run_dit_estimator_step_cpu(const mit2::Bundle& bundle, const std::vector<float>& x,
                                              const std::vector<float>& prompt_x, const std::vector<float>& cond,
                                              const std::vector<float>& style, float timestep,
                                              const std::vector<uint32_t>& mask, uint32_t tokens);
std::vector<float> run_cfm_euler_cpu(const mit2::Bundle& bundle, std::vector<float> x, const std::vector<float>& prompt,
                                     const std::vector<float>& cond, const std::vector<float>& style, uint32_t tokens,
                                     uint32_t prompt_tokens, uint32_t steps, float cfg_rate);
std::vector<float> run_dit_attention_core_cpu_masked_layer(const mit2::Bundle& bundle, const std::vector<float>& input,
                                                           const std::vector<uint32_t>& key_mask, uint32_t tokens,
                                                           uint32_t layer);
std::vector<float> run_wavenet_stack_global_cond_cpu(const mit2::Bundle& bundle, const std::vector<float>& input,
                                                     const std::vector<float>& g, const std::vector<uint32_t>& mask,
                                                     uint32_t tokens);
std::vector<float> run_timestep_embedder_cpu(const mit2::Bundle& bundle, const std::vector<float>& timesteps,
                                             const std::string& prefix);
std::vector<float> make_deterministic_normal_noise(uint32_t tokens, uint32_t channels, uint64_t seed,
                                                   float temperature);
std::vector<float> run_bigvgan_vocoder_cpu(const mit2::Bundle& bundle, std::vector<float> mel, uint32_t tokens);
std::vector<float> run_length_regulator_full_cpu(const mit2::Bundle& bundle, const std::vector<float>& input,
                                                 uint32_t in_tokens, uint32_t out_tokens);
void ref_glue_gpt_kv_greedy(const mit2::Bundle& bundle, const std::vector<float>& prefix, uint32_t prefix_tokens,
                            uint32_t steps, bool hf_generate_positions, std::vector<uint32_t>* tokens,
                            std::vector<float>* last_logits, int* first_stop);
void ref_glue_gpt_sample(const std::vector<float>& logits, const std::vector<uint32_t>& history, uint64_t seed,
                         float temperature, uint32_t top_k, float top_p, float repetition_penalty, uint32_t draws,
                         std::vector<float>* processed, std::vector<uint32_t>* tokens);
std::vector<float> run_bigvgan_activation_cpu(const mit2::Bundle& bundle, const std::string& prefix,
                                              const std::vector<float>& x, uint32_t tokens, uint32_t channels);

namespace {
thread_local std::string g_err;

template <typename F>
int guard(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  } catch (...) {
    g_err = "unknown";
    return -1;
  }
}

std::vector<float> vec(const float* p, size_t n) { return std::vector<float>(p, p + n); }
}  // namespace

extern "C" {

const char* ref_last_error(void) { return g_err.c_str(); }

// run_dit_estimator_step_cpu on one branch: x, prompt_x [T,80], cond [T,512],
// style [192], mask [T] -> vel [T,80].
int ref_estimator_step(const char* bundle_dir, const float* x, const float* prompt_x, const float* cond,
                       const float* style, float t, const uint32_t* mask, uint32_t T, float* vel) {
  return guard([&] {
    mit2::Bundle b(bundle_dir);
    std::vector<uint32_t> m(mask, mask + T);
    auto v = run_dit_estimator_step_cpu(b, vec(x, T * 80ull), vec(prompt_x, T * 80ull), vec(cond, T * 512ull),
                                        vec(style, 192), t, m, T);
    std::memcpy(vel, v.data(), v.size() * sizeof(float));
  });
}

// run_cfm_euler_cpu: noise [T,80], prompt [P,80], cond [T,512], style [192] -> mel [T,80].
int ref_cfm_euler(const char* bundle_dir, const float* noise, const float* prompt, const float* cond,
                  const float* style, uint32_t T, uint32_t P, uint32_t steps, float cfg, float* out) {
  return guard([&] {
    mit2::Bundle b(bundle_dir);
    auto v = run_cfm_euler_cpu(b, vec(noise, T * 80ull), vec(prompt, P * 80ull), vec(cond, T * 512ull),
                               vec(style, 192), T, P, steps, cfg);
    std::memcpy(out, v.data(), v.size() * sizeof(float));
  });
}

// The same Euler/CFG loop as run_cfm_euler_cpu with a key-padding mask handed
// to every estimator call (the padded-batch semantics); prompt_x [T,80].
int ref_cfm_euler_masked(const char* bundle_dir, const float* noise, const float* prompt_x, const float* cond,
                         const float* style, const uint32_t* mask, uint32_t T, uint32_t P, uint32_t steps, float cfg,
                         float* out) {
  return guard([&] {
    mit2::Bundle b(bundle_dir);
    std::vector<float> x = vec(noise, T * 80ull), px = vec(prompt_x, T * 80ull), c = vec(cond, T * 512ull),
                       s = vec(style, 192);
    std::vector<float> zp(T * 80ull, 0.0f), zc(T * 512ull, 0.0f), zs(192, 0.0f);
    std::vector<uint32_t> m(mask, mask + T);
    for (uint32_t r = 0; r < P; ++r) std::fill(x.begin() + r * 80, x.begin() + (r + 1) * 80, 0.0f);
    float t = 0.0f;
    const float dt = 1.0f / static_cast<float>(steps);
    for (uint32_t i = 0; i < steps; ++i) {
      auto v = run_dit_estimator_step_cpu(b, x, px, c, s, t, m, T);
      if (cfg > 0.0f) {
        auto vu = run_dit_estimator_step_cpu(b, x, zp, zc, zs, t, m, T);
        for (size_t k = 0; k < v.size(); ++k) v[k] = (1.0f + cfg) * v[k] - cfg * vu[k];
      }
      for (size_t k = 0; k < x.size(); ++k) x[k] += dt * v[k];
      t += dt;
      for (uint32_t r = 0; r < P; ++r) std::fill(x.begin() + r * 80, x.begin() + (r + 1) * 80, 0.0f);
    }
    std::memcpy(out, x.data(), x.size() * sizeof(float));
  });
}

int ref_attention_layer(const char* bundle_dir, const float* x, const uint32_t* mask, uint32_t T, uint32_t layer,
                        float* out) {
  return guard([&] {
    mit2::Bundle b(bundle_dir);
    std::vector<uint32_t> m(mask, mask + T);
    auto v = run_dit_attention_core_cpu_masked_layer(b, vec(x, T * 512ull), m, T, layer);
    std::memcpy(out, v.data(), v.size() * sizeof(float));
  });
}

int ref_wavenet(const char* bundle_dir, const float* x, const float* g, const uint32_t* mask, uint32_t T, float* out) {
  return guard([&] {
    mit2::Bundle b(bundle_dir);
    std::vector<uint32_t> m(mask, mask + T);
    auto v = run_wavenet_stack_global_cond_cpu(b, vec(x, T * 512ull), vec(g, 512), m, T);
    std::memcpy(out, v.data(), v.size() * sizeof(float));
  });
}

int ref_timestep_embed(const char* bundle_dir, float t, int which, float* out) {
  return guard([&] {
    mit2::Bundle b(bundle_dir);
    auto v = run_timestep_embedder_cpu(b, std::vector<float>{t},
                                       which == 0 ? "s2mel.net.cfm.estimator.t_embedder"
                                                  : "s2mel.net.cfm.estimator.t_embedder2");
    std::memcpy(out, v.data(), v.size() * sizeof(float));
  });
}

int ref_noise(uint32_t T, uint32_t C, uint64_t seed, float temperature, float* out) {
  return guard([&] {
    auto v = make_deterministic_normal_noise(T, C, seed, temperature);
    std::memcpy(out, v.data(), v.size() * sizeof(float));
  });
}

// run_gpt_kv_greedy_cpu: prefix [P,1280] -> up to `steps` greedy mel codes
// (stops after the stop code 8193), the logits of the last step [8194];
// hf != 0 selects the generate-style positions (step s > 0 at position s + 1).
int ref_gpt_kv_greedy(const char* bundle_dir, const float* prefix, uint32_t P, uint32_t steps, int hf,
                      uint32_t* tokens, uint32_t* n_tokens, float* last_logits, int* first_stop) {
  return guard([&] {
    mit2::Bundle b(bundle_dir);
    std::vector<uint32_t> t;
    std::vector<float> l;
    ref_glue_gpt_kv_greedy(b, vec(prefix, static_cast<size_t>(P) * 1280), P, steps, hf != 0, &t, &l, first_stop);
    std::memcpy(tokens, t.data(), t.size() * sizeof(uint32_t));
    *n_tokens = static_cast<uint32_t>(t.size());
    std::memcpy(last_logits, l.data(), l.size() * sizeof(float));
  });
}

// apply_gpt_sampling_processors + sample_gpt_token_from_logits: the processed
// logits [n] of one step and `draws` tokens drawn from them with one SplitMix64
// stream seeded `seed`.
int ref_gpt_sample(const float* logits, uint32_t n, const uint32_t* history, uint32_t n_history, uint64_t seed,
                   float temperature, uint32_t top_k, float top_p, float repetition_penalty, uint32_t draws,
                   float* processed, uint32_t* tokens) {
  return guard([&] {
    std::vector<float> p;
    std::vector<uint32_t> t;
    ref_glue_gpt_sample(std::vector<float>(logits, logits + n), std::vector<uint32_t>(history, history + n_history),
                        seed, temperature, top_k, top_p, repetition_penalty, draws, &p, &t);
    std::memcpy(processed, p.data(), p.size() * sizeof(float));
    std::memcpy(tokens, t.data(), t.size() * sizeof(uint32_t));
  });
}

// run_length_regulator_full_cpu: s_infer [n_in,1024] -> [n_out,512].
int ref_length_regulator(const char* bundle_dir, const float* x, uint32_t n_in, uint32_t n_out, float* out) {
  return guard([&] {
    mit2::Bundle b(bundle_dir);
    auto v = run_length_regulator_full_cpu(b, vec(x, static_cast<size_t>(n_in) * 1024), n_in, n_out);
    std::memcpy(out, v.data(), v.size() * sizeof(float));
  });
}

// run_bigvgan_vocoder_cpu: mel [T,80] -> waveform [T*256] in [-1, 1].
int ref_bigvgan_vocoder(const char* bundle_dir, const float* mel, uint32_t T, float* out) {
  return guard([&] {
    mit2::Bundle b(bundle_dir);
    auto v = run_bigvgan_vocoder_cpu(b, vec(mel, T * 80ull), T);
    std::memcpy(out, v.data(), v.size() * sizeof(float));
  });
}

// run_bigvgan_activation_cpu: the anti-aliased SnakeBeta of `prefix` on x [T,C].
int ref_bigvgan_activation(const char* bundle_dir, const char* prefix, const float* x, uint32_t T, uint32_t C,
                           float* out) {
  return guard([&] {
    mit2::Bundle b(bundle_dir);
    auto v = run_bigvgan_activation_cpu(b, prefix, vec(x, static_cast<size_t>(T) * C), T, C);
    std::memcpy(out, v.data(), v.size() * sizeof(float));
  });
}

}  // extern "C"
