// C ABI over the GPT mel-code decoder (include/itts_cfm.h, itts_gpt_*).
// Catches every C++ exception at the boundary and turns it into a status code
// plus a message, as the estimator's entry points do.
#include <memory>
#include <stdexcept>
#include <string>

#include "gpt.hpp"
#include "itts_cfm.h"

struct itts_gpt_ctx {
  std::unique_ptr<itts::GptDecoder> dec;
  std::string err;
};

namespace {

thread_local std::string g_gpt_create_err;

int gclassify(const std::exception& e) {
  if (dynamic_cast<const std::invalid_argument*>(&e)) return ITTS_EINVAL_SHAPE;
  const std::string m = e.what();
  if (m.rfind("bundle", 0) == 0 || m.rfind("manifest", 0) == 0 || m.rfind("gpt weights", 0) == 0) return ITTS_EBUNDLE;
  if (m.rfind("timeout", 0) == 0) return ITTS_ETIMEOUT;
  if (m.rfind("device id", 0) == 0 || m.rfind("this build targets", 0) == 0) return ITTS_ENODEV;
  return ITTS_ECUDA;
}

}  // namespace

extern "C" {

int itts_gpt_create(const char* bundle_dir, int device, itts_gpt_ctx** out) {
  g_gpt_create_err.clear();
  if (!bundle_dir || !out) {
    g_gpt_create_err = "null argument";
    return ITTS_EINVAL_SHAPE;
  }
  *out = nullptr;
  try {
    auto ctx = std::make_unique<itts_gpt_ctx>();
    ctx->dec = std::make_unique<itts::GptDecoder>(bundle_dir, device, false);
    *out = ctx.release();
    return ITTS_OK;
  } catch (const std::exception& e) {
    g_gpt_create_err = e.what();
    return gclassify(e);
  }
}

void itts_gpt_destroy(itts_gpt_ctx* ctx) { delete ctx; }

const char* itts_gpt_last_error(const itts_gpt_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

const char* itts_gpt_create_error(void) { return g_gpt_create_err.c_str(); }

int itts_gpt_generate(itts_gpt_ctx* ctx, const float* prefix, uint32_t P, uint32_t steps, uint32_t* codes,
                      uint32_t* n_codes, float* last_logits) {
  return itts_gpt_generate_ex(ctx, prefix, P, steps, 0u, codes, n_codes, last_logits);
}

int itts_gpt_generate_ex(itts_gpt_ctx* ctx, const float* prefix, uint32_t P, uint32_t steps, uint32_t flags,
                         uint32_t* codes, uint32_t* n_codes, float* last_logits) {
  if (!ctx) return ITTS_EINVAL_SHAPE;
  try {
    ctx->err.clear();
    if (P > ITTS_GPT_MAX_LEN || steps > ITTS_GPT_MAX_STEPS)
      throw std::invalid_argument("gpt: need 1 <= steps <= 1818 and P + steps <= 4096");
    if (flags & ~ITTS_GPT_HF_POSITIONS) throw std::invalid_argument("gpt: unknown flag bits");
    cudaSetDevice(ctx->dec->device());
    const int n = ctx->dec->generate(prefix, static_cast<int>(P), static_cast<int>(steps),
                                     (flags & ITTS_GPT_HF_POSITIONS) != 0, codes, last_logits);
    if (n_codes) *n_codes = static_cast<uint32_t>(n);
    return ITTS_OK;
  } catch (const std::exception& e) {
    ctx->err = e.what();
    return gclassify(e);
  } catch (...) {
    ctx->err = "unknown error";
    return ITTS_ECUDA;
  }
}

int itts_gpt_generate_sampled(itts_gpt_ctx* ctx, const float* prefix, uint32_t P, uint32_t steps, uint32_t flags,
                              const itts_gpt_sampling* sampling, const uint32_t* history, uint32_t n_history,
                              uint32_t* codes, uint32_t* n_codes, float* last_logits) {
  if (!ctx) return ITTS_EINVAL_SHAPE;
  try {
    ctx->err.clear();
    if (!sampling) throw std::invalid_argument("gpt: sampling must be non-null");
    if (P > ITTS_GPT_MAX_LEN || steps > ITTS_GPT_MAX_STEPS || n_history > ITTS_GPT_MAX_LEN ||
        sampling->top_k > ITTS_GPT_SAMPLE_MAX_TOP_K)
      throw std::invalid_argument("gpt: need 1 <= steps <= 1818, P + steps <= 4096, n_history <= 4096, top_k <= 2048");
    if (flags & ~ITTS_GPT_HF_POSITIONS) throw std::invalid_argument("gpt: unknown flag bits");
    cudaSetDevice(ctx->dec->device());
    itts::GptDecoder::Sampling s;
    s.seed = sampling->seed;
    s.temperature = sampling->temperature;
    s.top_k = static_cast<int>(sampling->top_k);
    s.top_p = sampling->top_p;
    s.repetition_penalty = sampling->repetition_penalty;
    const int n = ctx->dec->generate_sampled(prefix, static_cast<int>(P), static_cast<int>(steps),
                                             (flags & ITTS_GPT_HF_POSITIONS) != 0, s, history,
                                             static_cast<int>(n_history), codes, last_logits);
    if (n_codes) *n_codes = static_cast<uint32_t>(n);
    return ITTS_OK;
  } catch (const std::exception& e) {
    ctx->err = e.what();
    return gclassify(e);
  } catch (...) {
    ctx->err = "unknown error";
    return ITTS_ECUDA;
  }
}

int itts_gpt_timing(const itts_gpt_ctx* ctx, float* prefill_ms, float* decode_ms) {
  if (!ctx) return ITTS_EINVAL_SHAPE;
  if (prefill_ms) *prefill_ms = ctx->dec->last_prefill_ms();
  if (decode_ms) *decode_ms = ctx->dec->last_decode_ms();
  return ITTS_OK;
}

int itts_gpt_launch_kernels(const itts_gpt_ctx* ctx) {
  return ctx ? static_cast<int>(ctx->dec->last_launches()) : ITTS_EINVAL_SHAPE;
}

int itts_gpt_set_tracing(itts_gpt_ctx* ctx, int on) {
  if (!ctx) return ITTS_EINVAL_SHAPE;
  ctx->dec->set_tracing(on != 0);
  return ITTS_OK;
}

int itts_gpt_stage_trace(itts_gpt_ctx* ctx, double* us, uint32_t cap) {
  if (!ctx || !us) return ITTS_EINVAL_SHAPE;
  try {
    return ctx->dec->stage_trace(us, static_cast<int>(cap));
  } catch (const std::exception& e) {
    ctx->err = e.what();
    return ITTS_ECUDA;
  }
}

double itts_gpt_weight_bytes_per_token(void) { return itts::GptDecoder::weight_bytes_per_token(); }

}  // extern "C"
