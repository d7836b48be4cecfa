// C ABI over the condition assembler (include/itts_cfm.h, itts_cond_*).
// Catches every C++ exception at the boundary and turns it into a status code
// plus a message, as the estimator's entry points do.
#include <memory>
#include <stdexcept>
#include <string>

#include "condition.hpp"
#include "itts_cfm.h"

struct itts_cond_ctx {
  std::unique_ptr<itts::ConditionAssembler> ca;
  std::string err;
};

namespace {

thread_local std::string g_cond_create_err;

struct CShapeError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct CTimeoutError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

int cclassify(const std::exception& e) {
  if (dynamic_cast<const CShapeError*>(&e)) return ITTS_EINVAL_SHAPE;
  if (dynamic_cast<const CTimeoutError*>(&e)) return ITTS_ETIMEOUT;
  const std::string m = e.what();
  if (m.rfind("bundle", 0) == 0 || m.rfind("manifest", 0) == 0 || m.rfind("condition weights", 0) == 0)
    return ITTS_EBUNDLE;
  if (m.rfind("device id", 0) == 0 || m.rfind("this build targets", 0) == 0) return ITTS_ENODEV;
  return ITTS_ECUDA;
}

template <typename F>
int cguarded(itts_cond_ctx* ctx, F&& f) {
  if (!ctx) return ITTS_EINVAL_SHAPE;
  try {
    ctx->err.clear();
    cudaSetDevice(ctx->ca->device());
    f();
    return ITTS_OK;
  } catch (const std::exception& e) {
    ctx->err = e.what();
    return cclassify(e);
  } catch (...) {
    ctx->err = "unknown error";
    return ITTS_ECUDA;
  }
}

void cneed(bool ok, const char* what) {
  if (!ok) throw CShapeError(what);
}

void check_shape(const float* s_infer, uint32_t n_in, const float* prompt, uint32_t P, uint32_t G) {
  cneed(s_infer != nullptr, "s_infer must be non-null");
  cneed(n_in >= 1 && n_in <= ITTS_MAX_T, "n_in must be within 1..ITTS_MAX_T");
  cneed(G >= 1 && static_cast<uint64_t>(P) + G <= ITTS_MAX_T, "G >= 1 and P + G <= ITTS_MAX_T");
  cneed(P == 0 || prompt != nullptr, "prompt must be non-null when P > 0");
}

void ccheck_status(itts::ConditionAssembler& c) {
  const unsigned int s = c.read_status();
  if (s != 0) {
    c.clear_status();
    throw CTimeoutError("a condition-assembly kernel abandoned a bounded wait (device status " + std::to_string(s) + ")");
  }
}

}  // namespace

extern "C" {

int itts_cond_create(const char* bundle_dir, int device, itts_cond_ctx** out) {
  g_cond_create_err.clear();
  if (!bundle_dir || !out) {
    g_cond_create_err = "null argument";
    return ITTS_EINVAL_SHAPE;
  }
  *out = nullptr;
  try {
    auto ctx = std::make_unique<itts_cond_ctx>();
    ctx->ca = std::make_unique<itts::ConditionAssembler>(bundle_dir, device, false);
    *out = ctx.release();
    return ITTS_OK;
  } catch (const std::exception& e) {
    g_cond_create_err = e.what();
    return cclassify(e);
  }
}

void itts_cond_destroy(itts_cond_ctx* ctx) { delete ctx; }

const char* itts_cond_last_error(const itts_cond_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

const char* itts_cond_create_error(void) { return g_cond_create_err.c_str(); }

int itts_cond_assemble(itts_cond_ctx* ctx, const float* s_infer, uint32_t n_in, const float* prompt_cond, uint32_t P,
                       uint32_t G, float* cond) {
  return cguarded(ctx, [&] {
    check_shape(s_infer, n_in, prompt_cond, P, G);
    cneed(cond != nullptr, "cond must be non-null");
    ctx->ca->run(s_infer, static_cast<int>(n_in), prompt_cond, static_cast<int>(P), static_cast<int>(G), cond);
    ccheck_status(*ctx->ca);
  });
}

int itts_cond_stage(itts_cond_ctx* ctx, const float* s_infer, uint32_t n_in, const float* prompt_cond, uint32_t P,
                    uint32_t G) {
  return cguarded(ctx, [&] {
    check_shape(s_infer, n_in, prompt_cond, P, G);
    ctx->ca->stage(s_infer, static_cast<int>(n_in), prompt_cond, static_cast<int>(P), static_cast<int>(G));
  });
}

int itts_cond_launch(itts_cond_ctx* ctx) {
  return cguarded(ctx, [&] { ctx->ca->launch(); });
}

int itts_cond_fetch(itts_cond_ctx* ctx, float* cond) {
  return cguarded(ctx, [&] {
    cneed(cond != nullptr, "cond must be non-null");
    ctx->ca->fetch(cond);
    ccheck_status(*ctx->ca);
  });
}

void* itts_cond_stream(itts_cond_ctx* ctx) { return ctx ? static_cast<void*>(ctx->ca->stream()) : nullptr; }

int itts_cond_launch_kernels(itts_cond_ctx* ctx) {
  if (!ctx) return ITTS_EINVAL_SHAPE;
  const int n = ctx->ca->launches_per_run();
  return n < 0 ? ITTS_EINVAL_SHAPE : n;
}

double itts_cond_flops(uint32_t n_in, uint32_t G) {
  return itts::ConditionAssembler::flops(static_cast<int>(n_in), static_cast<int>(G));
}

}  // extern "C"
