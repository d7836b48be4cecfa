// The S2Mel-to-waveform chain of the reference's hot synthesis path as one
// C-ABI call (include/itts_cfm.h, itts_pipeline_*): voice profile ->
// condition assembly -> CFM sampler -> BigVGAN vocoder on the generated rows.
//
// Follows synthesize_hot_condition_vectors_wav_shared and its condition input
// (runtime/impl/tts_synthesis/synthesis_pipeline.cpp:1030-1034, 1060-1089):
// cond = [s2mel_prompt rows ; length_regulator(s_infer)], prompt mel = the
// voice mel transposed to [P,80], style = s2mel_style,
// full_mel = run_cfm_euler(noise, prompt, cond, style, P + G, P, steps, cfg),
// wave = vocoder(full_mel[P:]). Each stage runs on its own context through the
// stage's public entry point; the intermediate buffers are host memory.
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "itts_cfm.h"

struct itts_pipeline {
  itts_cfm_ctx* cfm = nullptr;
  itts_cond_ctx* cond = nullptr;
  itts_vocoder_ctx* voc = nullptr;
  std::string err;
  ~itts_pipeline() {
    if (voc) itts_vocoder_destroy(voc);
    if (cond) itts_cond_destroy(cond);
    if (cfm) itts_cfm_destroy(cfm);
  }
};

namespace {

thread_local std::string g_pipe_create_err;

struct StageError : std::runtime_error {
  int code;
  StageError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

}  // namespace

extern "C" {

int itts_pipeline_create(const char* cfm_bundle_dir, const char* regulator_bundle_dir, const char* vocoder_bundle_dir,
                         int device, itts_pipeline** out) {
  g_pipe_create_err.clear();
  if (!cfm_bundle_dir || !regulator_bundle_dir || !vocoder_bundle_dir || !out) {
    g_pipe_create_err = "null argument";
    return ITTS_EINVAL_SHAPE;
  }
  *out = nullptr;
  auto p = std::make_unique<itts_pipeline>();
  int rc = itts_cfm_create(cfm_bundle_dir, device, &p->cfm);
  if (rc != ITTS_OK) {
    g_pipe_create_err = std::string("cfm: ") + itts_cfm_create_error();
    return rc;
  }
  rc = itts_cond_create(regulator_bundle_dir, device, &p->cond);
  if (rc != ITTS_OK) {
    g_pipe_create_err = std::string("length regulator: ") + itts_cond_create_error();
    return rc;
  }
  rc = itts_vocoder_create(vocoder_bundle_dir, device, &p->voc);
  if (rc != ITTS_OK) {
    g_pipe_create_err = std::string("vocoder: ") + itts_vocoder_create_error();
    return rc;
  }
  *out = p.release();
  return ITTS_OK;
}

void itts_pipeline_destroy(itts_pipeline* p) { delete p; }

const char* itts_pipeline_last_error(const itts_pipeline* p) { return p ? p->err.c_str() : "null pipeline"; }

const char* itts_pipeline_create_error(void) { return g_pipe_create_err.c_str(); }

int itts_pipeline_synthesize(itts_pipeline* p, const char* voice_bundle_dir, uint32_t prompt_tokens,
                             const float* s_infer, uint32_t n_in, uint32_t G, const float* noise, uint32_t steps,
                             float cfg_rate, float* wave, float* full_mel) {
  if (!p) return ITTS_EINVAL_SHAPE;
  p->err.clear();
  try {
    if (!voice_bundle_dir || !s_infer || !noise || !wave) throw StageError(ITTS_EINVAL_SHAPE, "null argument");
    if (G == 0) throw StageError(ITTS_EINVAL_SHAPE, "G must be >= 1 generated frame");
    uint32_t P = 0;
    char verr[512];
    int rc = itts_voice_load(voice_bundle_dir, prompt_tokens, &P, nullptr, nullptr, nullptr, verr, sizeof(verr));
    if (rc != ITTS_OK) throw StageError(rc, std::string("voice: ") + verr);
    const uint32_t T = P + G;
    std::vector<float> prompt_cond(static_cast<size_t>(P) * 512), style(192), prompt_mel(static_cast<size_t>(P) * 80);
    rc = itts_voice_load(voice_bundle_dir, prompt_tokens, &P, prompt_cond.data(), style.data(), prompt_mel.data(), verr,
                         sizeof(verr));
    if (rc != ITTS_OK) throw StageError(rc, std::string("voice: ") + verr);
    std::vector<float> cond(static_cast<size_t>(T) * 512);
    rc = itts_cond_assemble(p->cond, s_infer, n_in, prompt_cond.data(), P, G, cond.data());
    if (rc != ITTS_OK) throw StageError(rc, std::string("condition assembly: ") + itts_cond_last_error(p->cond));
    std::vector<float> mel(static_cast<size_t>(T) * 80);
    rc = itts_cfm_run(p->cfm, noise, prompt_mel.data(), cond.data(), style.data(), T, P, steps, cfg_rate, mel.data());
    if (rc != ITTS_OK) throw StageError(rc, std::string("cfm: ") + itts_cfm_last_error(p->cfm));
    rc = itts_vocoder_run(p->voc, mel.data() + static_cast<size_t>(P) * 80, G, wave);
    if (rc != ITTS_OK) throw StageError(rc, std::string("vocoder: ") + itts_vocoder_last_error(p->voc));
    if (full_mel) std::memcpy(full_mel, mel.data(), mel.size() * sizeof(float));
    return ITTS_OK;
  } catch (const StageError& e) {
    p->err = e.what();
    return e.code;
  } catch (const std::exception& e) {
    p->err = e.what();
    return ITTS_ECUDA;
  }
}

int itts_pipeline_synthesize_seeded(itts_pipeline* p, const char* voice_bundle_dir, uint32_t prompt_tokens,
                                    const float* s_infer, uint32_t n_in, uint32_t G, uint64_t seed, float temperature,
                                    uint32_t steps, float cfg_rate, float* wave, float* full_mel) {
  if (!p) return ITTS_EINVAL_SHAPE;
  p->err.clear();
  if (!voice_bundle_dir || G == 0) {
    p->err = "null voice bundle or G == 0";
    return ITTS_EINVAL_SHAPE;
  }
  uint32_t P = 0;
  char verr[512];
  int rc = itts_voice_load(voice_bundle_dir, prompt_tokens, &P, nullptr, nullptr, nullptr, verr, sizeof(verr));
  if (rc != ITTS_OK) {
    p->err = std::string("voice: ") + verr;
    return rc;
  }
  if (static_cast<uint64_t>(P) + G > ITTS_MAX_T) {
    p->err = "P + G exceeds ITTS_MAX_T";
    return ITTS_EINVAL_SHAPE;
  }
  // x0 over all P + G rows, as the reference's pipeline draws it; the
  // sampler zeroes the prompt rows itself.
  std::vector<float> noise(static_cast<size_t>(P + G) * 80);
  rc = itts_make_noise(P + G, 80, seed, temperature, noise.data());
  if (rc != ITTS_OK) {
    p->err = "noise: bad shape";
    return rc;
  }
  return itts_pipeline_synthesize(p, voice_bundle_dir, prompt_tokens, s_infer, n_in, G, noise.data(), steps, cfg_rate,
                                  wave, full_mel);
}

}  // extern "C"
