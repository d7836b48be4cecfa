// C ABI over the BigVGAN vocoder (include/itts_cfm.h, itts_vocoder_*).
// Catches every C++ exception at the boundary and turns it into a status code
// plus a message, as the estimator's entry points do.
#include <algorithm>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>

#include "itts_cfm.h"
#include "vocoder.hpp"

struct itts_vocoder_ctx {
  std::unique_ptr<itts::Vocoder> voc;
  std::string err;
};

namespace {

thread_local std::string g_voc_create_err;

struct VShapeError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct VTimeoutError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

int vclassify(const std::exception& e) {
  if (dynamic_cast<const VShapeError*>(&e)) return ITTS_EINVAL_SHAPE;
  if (dynamic_cast<const VTimeoutError*>(&e)) return ITTS_ETIMEOUT;
  const std::string m = e.what();
  if (m.rfind("bundle", 0) == 0 || m.rfind("manifest", 0) == 0 || m.rfind("vocoder weights", 0) == 0)
    return ITTS_EBUNDLE;
  if (m.rfind("device id", 0) == 0 || m.rfind("this build targets", 0) == 0) return ITTS_ENODEV;
  if (m.rfind("vocoder: T must", 0) == 0) return ITTS_EINVAL_SHAPE;
  return ITTS_ECUDA;
}

template <typename F>
int vguarded(itts_vocoder_ctx* ctx, F&& f) {
  if (!ctx) return ITTS_EINVAL_SHAPE;
  try {
    ctx->err.clear();
    cudaSetDevice(ctx->voc->device());
    f();
    return ITTS_OK;
  } catch (const std::exception& e) {
    ctx->err = e.what();
    return vclassify(e);
  } catch (...) {
    ctx->err = "unknown error";
    return ITTS_ECUDA;
  }
}

void vneed(bool ok, const char* what) {
  if (!ok) throw VShapeError(what);
}

void vcheck_status(itts::Vocoder& v) {
  const unsigned int s = v.read_status();
  if (s != 0) {
    v.clear_status();
    throw VTimeoutError("a vocoder kernel abandoned a bounded wait (device status " + std::to_string(s) + ")");
  }
}

}  // namespace

extern "C" {

int itts_vocoder_create(const char* bundle_dir, int device, itts_vocoder_ctx** out) {
  g_voc_create_err.clear();
  if (!bundle_dir || !out) {
    g_voc_create_err = "null argument";
    return ITTS_EINVAL_SHAPE;
  }
  *out = nullptr;
  try {
    auto ctx = std::make_unique<itts_vocoder_ctx>();
    ctx->voc = std::make_unique<itts::Vocoder>(bundle_dir, device, false);
    *out = ctx.release();
    return ITTS_OK;
  } catch (const std::exception& e) {
    g_voc_create_err = e.what();
    return vclassify(e);
  }
}

void itts_vocoder_destroy(itts_vocoder_ctx* ctx) { delete ctx; }

const char* itts_vocoder_last_error(const itts_vocoder_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

const char* itts_vocoder_create_error(void) { return g_voc_create_err.c_str(); }

int itts_vocoder_run(itts_vocoder_ctx* ctx, const float* mel, uint32_t T, float* wave) {
  return vguarded(ctx, [&] {
    vneed(mel && wave, "mel and wave must be non-null");
    vneed(T >= 1 && T <= ITTS_VOCODER_MAX_T, "T must be within 1..ITTS_VOCODER_MAX_T mel frames");
    ctx->voc->run(mel, static_cast<int>(T), wave);
    vcheck_status(*ctx->voc);
  });
}

int itts_vocoder_stage(itts_vocoder_ctx* ctx, const float* mel, uint32_t T) {
  return vguarded(ctx, [&] {
    vneed(mel != nullptr, "mel must be non-null");
    vneed(T >= 1 && T <= ITTS_VOCODER_MAX_T, "T must be within 1..ITTS_VOCODER_MAX_T mel frames");
    ctx->voc->stage(mel, static_cast<int>(T));
  });
}

int itts_vocoder_launch(itts_vocoder_ctx* ctx) {
  return vguarded(ctx, [&] { ctx->voc->launch(); });
}

int itts_vocoder_fetch(itts_vocoder_ctx* ctx, float* wave) {
  return vguarded(ctx, [&] {
    vneed(wave != nullptr, "wave must be non-null");
    ctx->voc->fetch(wave);
    vcheck_status(*ctx->voc);
  });
}

void* itts_vocoder_stream(itts_vocoder_ctx* ctx) { return ctx ? static_cast<void*>(ctx->voc->stream()) : nullptr; }

int itts_vocoder_launch_kernels(itts_vocoder_ctx* ctx) {
  if (!ctx) return ITTS_EINVAL_SHAPE;
  const int n = ctx->voc->launches_per_run();
  return n < 0 ? ITTS_EINVAL_SHAPE : n;
}

int itts_vocoder_profile(itts_vocoder_ctx* ctx, int reps, itts_kernel_stat* out, int cap, int* n_out) {
  return vguarded(ctx, [&] {
    vneed(reps >= 1 && out && cap > 0 && n_out, "bad profile arguments");
    auto kt = ctx->voc->profile(reps);
    vcheck_status(*ctx->voc);
    const int n = std::min<int>(cap, static_cast<int>(kt.size()));
    for (int i = 0; i < n; ++i) {
      std::memset(out[i].name, 0, sizeof(out[i].name));
      std::strncpy(out[i].name, kt[i].name.c_str(), sizeof(out[i].name) - 1);
      out[i].launches = kt[i].launches;
      out[i].ms = kt[i].ms;
      out[i].flops = kt[i].flops;
      out[i].bytes = kt[i].bytes;
    }
    *n_out = n;
  });
}

double itts_vocoder_flops(uint32_t T) { return itts::Vocoder::flops(static_cast<int>(T)); }

}  // extern "C"
