// C ABI over the DiT-CFM engine (include/itts_cfm.h). Catches every C++
// exception at the boundary and turns it into a status code plus a message.
#include "itts_cfm.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "engine.hpp"
#include "gemm.cuh"
#include "kernels.cuh"

// Page-locked ring for itts_cfm_run_batch: host threads pack one utterance
// per slot (its rows and the zero padding up to the launch length), the slot
// is copied to the launch's device buffers asynchronously, and it is reused
// once those copies are done (an event per slot); outputs come back through
// the same slots. The footprint is kSlots utterances, not the whole batch.
struct PinnedRing {
  static constexpr int kSlots = 32;
  float* p = nullptr;
  size_t slot = 0;  // floats per slot
  cudaEvent_t ev[kSlots] = {};
  bool live[kSlots] = {};  // copies reading or writing the slot may be in flight
  PinnedRing() = default;
  PinnedRing(const PinnedRing&) = delete;
  PinnedRing& operator=(const PinnedRing&) = delete;
  ~PinnedRing() { release(); }
  void release() {
    for (int i = 0; i < kSlots; ++i) {
      if (ev[i]) {
        if (live[i]) cudaEventSynchronize(ev[i]);
        cudaEventDestroy(ev[i]);
      }
      ev[i] = nullptr;
      live[i] = false;
    }
    if (p) cudaFreeHost(p);
    p = nullptr;
    slot = 0;
  }
  void reserve(size_t floats_per_slot) {
    if (floats_per_slot <= slot) return;
    release();
    void* q = nullptr;
    if (cudaHostAlloc(&q, static_cast<size_t>(kSlots) * floats_per_slot * sizeof(float), cudaHostAllocPortable) !=
        cudaSuccess)
      throw std::runtime_error("page-locked staging allocation failed");
    p = static_cast<float*>(q);
    slot = floats_per_slot;
    for (int i = 0; i < kSlots; ++i)
      if (cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming) != cudaSuccess)
        throw std::runtime_error("staging event creation failed");
  }
  float* at(int i) { return p + static_cast<size_t>(i) * slot; }
  // Waits until no copy touches slot i.
  void claim(int i) {
    if (live[i] && cudaEventSynchronize(ev[i]) != cudaSuccess) throw std::runtime_error("staging copy failed");
    live[i] = false;
  }
  void mark(int i, cudaStream_t st) {
    if (cudaEventRecord(ev[i], st) != cudaSuccess) throw std::runtime_error("staging event record failed");
    live[i] = true;
  }
};

constexpr uint32_t kRingRowsAtCreate = 1600;

struct itts_cfm_ctx {
  std::unique_ptr<itts::Engine> eng;
  std::string err;
  // staged batch
  itts::Work* staged = nullptr;
  int steps = 0;
  float cfg = 0.0f;
  PinnedRing ring;  // destroyed before the engine
};

namespace {

thread_local std::string g_create_err;

struct ShapeError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct CapError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct TimeoutError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

int classify(const std::exception& e) {
  if (dynamic_cast<const ShapeError*>(&e)) return ITTS_EINVAL_SHAPE;
  if (dynamic_cast<const CapError*>(&e)) return ITTS_ECAP;
  if (dynamic_cast<const TimeoutError*>(&e)) return ITTS_ETIMEOUT;
  const std::string m = e.what();
  if (m.rfind("bundle", 0) == 0 || m.rfind("manifest", 0) == 0 || m.rfind("weights: tensor", 0) == 0)
    return ITTS_EBUNDLE;
  if (m.rfind("device id", 0) == 0 || m.rfind("this build targets", 0) == 0) return ITTS_ENODEV;
  return ITTS_ECUDA;
}

template <typename F>
int guarded(itts_cfm_ctx* ctx, F&& f) {
  if (!ctx) return ITTS_EINVAL_SHAPE;
  try {
    ctx->err.clear();
    cudaSetDevice(ctx->eng->device());
    f();
    return ITTS_OK;
  } catch (const std::exception& e) {
    ctx->err = e.what();
    return classify(e);
  } catch (...) {
    ctx->err = "unknown error";
    return ITTS_ECUDA;
  }
}

void need(bool ok, const char* what) {
  if (!ok) throw ShapeError(what);
}

void cuda_ok(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string("cuda: ") + what + ": " + cudaGetErrorString(e));
}

void check_run_args(uint32_t B, uint32_t T, uint32_t steps, float cfg, uint32_t branches) {
  need(B >= 1, "batch must hold at least one utterance");
  need(T >= ITTS_MIN_T, "T must be >= 2 (the k=5 reflect-padded conv needs two rows)");
  need(steps >= 1, "steps must be >= 1");
  need(std::isfinite(cfg) && cfg >= 0.0f, "cfg_rate must be finite and >= 0");
  if (T > ITTS_MAX_T) throw CapError("T exceeds ITTS_MAX_T");
  if (steps > ITTS_MAX_STEPS) throw CapError("steps exceeds ITTS_MAX_STEPS");
  if (static_cast<uint64_t>(B) * branches * T > ITTS_MAX_ROWS) throw CapError("B x branches x T exceeds ITTS_MAX_ROWS");
}

void check_status(itts::Engine& e) {
  const unsigned int s = e.read_status();
  if (s != 0) {
    e.clear_status();
    throw TimeoutError("a kernel abandoned a bounded wait (device status " + std::to_string(s) + ")");
  }
}

// Copy a padded batch into workspace w (host pointers).
// Prompt lengths and the key / WaveNet mask of a launch (from valid_len, or
// per-row from mask_bt), uploaded from pageable vectors; returns after the
// stream has drained them.
void upload_masks(itts::Engine& e, itts::Work* w, const uint32_t* valid_len, const uint32_t* prompt_len,
                  const uint32_t* mask_bt) {
  cudaStream_t st = e.stream();
  std::vector<int> pl(w->B);
  std::vector<float> mask(static_cast<size_t>(w->R));
  for (int b = 0; b < w->B; ++b) {
    pl[b] = prompt_len ? static_cast<int>(prompt_len[b]) : 0;
    for (int br = 0; br < w->br; ++br) {
      for (int t = 0; t < w->T; ++t) {
        float m;
        if (mask_bt) m = mask_bt[static_cast<size_t>(b) * w->T + t] ? 1.0f : 0.0f;
        else m = static_cast<uint32_t>(t) < valid_len[b] ? 1.0f : 0.0f;
        mask[(static_cast<size_t>(b) * w->br + br) * w->T + t] = m;
      }
    }
  }
  cuda_ok(cudaMemcpyAsync(w->plen, pl.data(), pl.size() * sizeof(int), cudaMemcpyHostToDevice, st), "plen upload");
  cuda_ok(cudaMemcpyAsync(w->mask, mask.data(), mask.size() * sizeof(float), cudaMemcpyHostToDevice, st), "mask upload");
  // Pageable sources: the copies above complete before the host vectors die.
  cuda_ok(cudaStreamSynchronize(st), "upload sync");
}

void upload_padded(itts::Engine& e, itts::Work* w, const uint32_t* valid_len, const uint32_t* prompt_len,
                   const float* noise, const float* prompt_x, const float* cond, const float* style,
                   const uint32_t* mask_bt) {
  const size_t BT = static_cast<size_t>(w->B) * w->T;
  cudaStream_t st = e.stream();
  cuda_ok(cudaMemcpyAsync(w->X0, noise, BT * 80 * sizeof(float), cudaMemcpyHostToDevice, st), "noise upload");
  cuda_ok(cudaMemcpyAsync(w->prompt_x, prompt_x, BT * 80 * sizeof(float), cudaMemcpyHostToDevice, st), "prompt upload");
  cuda_ok(cudaMemcpyAsync(w->cond, cond, BT * 512 * sizeof(float), cudaMemcpyHostToDevice, st), "cond upload");
  cuda_ok(cudaMemcpyAsync(w->style, style, static_cast<size_t>(w->B) * 192 * sizeof(float), cudaMemcpyHostToDevice, st),
          "style upload");
  upload_masks(e, w, valid_len, prompt_len, mask_bt);
}

void stage(itts_cfm_ctx* ctx, uint32_t B, uint32_t T, const uint32_t* valid_len, const uint32_t* prompt_len,
           const float* noise, const float* prompt_x, const float* cond, const float* style, uint32_t steps, float cfg) {
  const uint32_t branches = cfg > 0.0f ? 2u : 1u;
  check_run_args(B, T, steps, cfg, branches);
  need(valid_len && noise && prompt_x && cond && style, "null input pointer");
  for (uint32_t b = 0; b < B; ++b) {
    need(valid_len[b] >= 1 && valid_len[b] <= T, "valid_len must be in [1, T]");
    need(!prompt_len || prompt_len[b] <= T, "prompt_len must be <= T");
  }
  itts::Work* w = ctx->eng->work(static_cast<int>(B), static_cast<int>(T), static_cast<int>(branches));
  upload_padded(*ctx->eng, w, valid_len, prompt_len, noise, prompt_x, cond, style, nullptr);
  ctx->staged = w;
  ctx->steps = static_cast<int>(steps);
  ctx->cfg = cfg;
}

void fetch(itts_cfm_ctx* ctx, float* out_mel) {
  need(ctx->staged != nullptr, "nothing staged");
  need(out_mel != nullptr, "null output pointer");
  itts::Work* w = ctx->staged;
  cuda_ok(cudaMemcpyAsync(out_mel, w->X, static_cast<size_t>(w->B) * w->T * 80 * sizeof(float), cudaMemcpyDeviceToHost,
                          ctx->eng->stream()),
          "mel download");
  cuda_ok(cudaStreamSynchronize(ctx->eng->stream()), "mel sync");
}

}  // namespace

extern "C" {

int itts_cfm_create(const char* bundle_dir, int device, itts_cfm_ctx** out) {
  return itts_cfm_create_ex(bundle_dir, device, 0u, out);
}

int itts_cfm_create_ex(const char* bundle_dir, int device, uint32_t flags, itts_cfm_ctx** out) {
  g_create_err.clear();
  if (!out || !bundle_dir) {
    g_create_err = "null argument";
    return ITTS_EINVAL_SHAPE;
  }
  *out = nullptr;
  try {
    auto ctx = std::make_unique<itts_cfm_ctx>();
    ctx->eng = std::make_unique<itts::Engine>(bundle_dir, device, (flags & ITTS_CREATE_VERIFY_SHA256) != 0);
    // The batch entry point's page-locked ring, sized for utterances of up to
    // kRingRowsAtCreate rows (~138 MB), so a first itts_cfm_run_batch does not
    // pay for pinning it; longer utterances grow it on demand. A failure here
    // only defers the allocation to that call.
    try {
      ctx->ring.reserve(static_cast<size_t>(kRingRowsAtCreate) * (2 * 80 + 512));
    } catch (const std::exception&) {
      ctx->ring.release();
    }
    *out = ctx.release();
    return ITTS_OK;
  } catch (const std::exception& e) {
    g_create_err = e.what();
    return classify(e);
  } catch (...) {
    g_create_err = "unknown error";
    return ITTS_ECUDA;
  }
}

void itts_cfm_destroy(itts_cfm_ctx* ctx) { delete ctx; }

const char* itts_cfm_last_error(const itts_cfm_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

const char* itts_cfm_create_error(void) { return g_create_err.c_str(); }

const char* itts_cfm_strerror(int code) {
  switch (code) {
    case ITTS_OK: return "ok";
    case ITTS_EINVAL_SHAPE: return "invalid shape or argument";
    case ITTS_EBUNDLE: return "invalid or incomplete MIT2 bundle";
    case ITTS_ECUDA: return "CUDA error";
    case ITTS_ETIMEOUT: return "device-side wait timed out";
    case ITTS_ECAP: return "capacity limit exceeded";
    case ITTS_ENODEV: return "no usable sm_100 device";
    default: return "unknown status";
  }
}

uint32_t itts_cfm_bucket_len(uint32_t T) {
  if (T <= 2048) return std::max<uint32_t>(128u, (T + 127u) / 128u * 128u);
  return (T + 255u) / 256u * 256u;
}

double itts_cfm_step_flops(uint32_t S, uint32_t T) { return itts::step_flops(static_cast<int>(S), static_cast<int>(T)); }

int itts_cfm_run_padded(itts_cfm_ctx* ctx, uint32_t B, uint32_t T, const uint32_t* valid_len,
                        const uint32_t* prompt_len, const float* noise, const float* prompt_x, const float* cond,
                        const float* style, uint32_t steps, float cfg_rate, float* out_mel) {
  return guarded(ctx, [&] {
    need(out_mel != nullptr, "null output pointer");
    stage(ctx, B, T, valid_len, prompt_len, noise, prompt_x, cond, style, steps, cfg_rate);
    ctx->eng->enqueue_sampler(ctx->staged, ctx->steps, ctx->cfg, true);
    check_status(*ctx->eng);
    fetch(ctx, out_mel);
  });
}

int itts_cfm_run(itts_cfm_ctx* ctx, const float* noise, const float* prompt, const float* cond, const float* style,
                 uint32_t T, uint32_t P, uint32_t steps, float cfg_rate, float* out_mel) {
  return guarded(ctx, [&] {
    need(noise && cond && style && out_mel, "null pointer");
    need(P <= T, "prompt rows exceed T");
    need(P == 0 || prompt != nullptr, "null prompt with P > 0");
    std::vector<float> prompt_x(static_cast<size_t>(T) * 80, 0.0f);
    if (P) std::memcpy(prompt_x.data(), prompt, static_cast<size_t>(P) * 80 * sizeof(float));
    const uint32_t valid = T;
    stage(ctx, 1, T, &valid, &P, noise, prompt_x.data(), cond, style, steps, cfg_rate);
    ctx->eng->enqueue_sampler(ctx->staged, ctx->steps, ctx->cfg, true);
    check_status(*ctx->eng);
    fetch(ctx, out_mel);
  });
}

int itts_cfm_run_batch(itts_cfm_ctx* ctx, uint32_t n, const itts_cfm_utt* utts, uint32_t steps, float cfg_rate) {
  return guarded(ctx, [&] {
    need(n >= 1 && utts != nullptr, "empty batch");
    for (uint32_t i = 0; i < n; ++i) {
      const itts_cfm_utt& u = utts[i];
      need(u.noise && u.cond && u.style && u.out_mel, "null utterance pointer");
      need(u.T >= ITTS_MIN_T, "T must be >= 2");
      if (u.T > ITTS_MAX_T) throw CapError("T exceeds ITTS_MAX_T");
      need(u.P <= u.T && (u.P == 0 || u.prompt), "bad prompt");
    }
    const uint32_t branches = cfg_rate > 0.0f ? 2u : 1u;
    // Group by length class, longest first within a class (ties by index),
    // cut into launches of at most ITTS_MAX_ROWS rows, and pad each launch to
    // its longest utterance: a launch whose utterances share one length runs
    // unpadded, exactly as itts_cfm_run would.
    std::map<uint32_t, std::vector<uint32_t>> buckets;
    for (uint32_t i = 0; i < n; ++i) buckets[itts_cfm_bucket_len(utts[i].T)].push_back(i);
    // Launch list.
    struct Launch {
      const std::vector<uint32_t>* idx;
      size_t off;
      uint32_t B, Tp;
    };
    std::vector<Launch> launches;
    for (auto& kv : buckets) {
      std::stable_sort(kv.second.begin(), kv.second.end(),
                       [&](uint32_t a, uint32_t b) { return utts[a].T > utts[b].T; });
      const uint32_t per = std::max<uint32_t>(1u, ITTS_MAX_ROWS / (branches * kv.first));
      for (size_t off = 0; off < kv.second.size(); off += per) {
        const uint32_t B = static_cast<uint32_t>(std::min<size_t>(per, kv.second.size() - off));
        const uint32_t Tp = utts[kv.second[off]].T;
        launches.push_back(Launch{&kv.second, off, B, Tp});
      }
    }
    // Packing and unpacking run over a group's utterances on up to 16 host threads.
    auto parallel = [](uint32_t count, const auto& body) {
      const uint32_t hw = std::max(1u, std::thread::hardware_concurrency());
      const uint32_t nt = std::min<uint32_t>(std::min<uint32_t>(hw, 16u), count);
      if (nt <= 1) {
        for (uint32_t i = 0; i < count; ++i) body(i);
        return;
      }
      std::vector<std::thread> th;
      for (uint32_t t = 0; t < nt; ++t)
        th.emplace_back([&, t] {
          for (uint32_t i = t; i < count; i += nt) body(i);
        });
      for (auto& x : th) x.join();
    };
    PinnedRing& ring = ctx->ring;
    uint32_t t_max = 0;
    for (const Launch& L : launches) t_max = std::max(t_max, L.Tp);
    ring.reserve(static_cast<size_t>(t_max) * (2 * 80 + 512));  // once, for the longest launch
    constexpr int kHalf = PinnedRing::kSlots / 2;  // utterances per group; groups alternate ring halves
    itts::Engine& e = *ctx->eng;
    cudaStream_t st = e.stream();
    for (const Launch& L : launches) {
      const uint32_t B = L.B, Tp = L.Tp;
      check_run_args(B, Tp, steps, cfg_rate, branches);
      itts::Work* w = e.work(static_cast<int>(B), static_cast<int>(Tp), static_cast<int>(branches));
      const size_t n80 = static_cast<size_t>(Tp) * 80, n512 = static_cast<size_t>(Tp) * 512;
      std::vector<uint32_t> vl(B), pl(B);
      std::vector<float> style(static_cast<size_t>(B) * 192);
      for (uint32_t b = 0; b < B; ++b) {
        const itts_cfm_utt& u = utts[(*L.idx)[L.off + b]];
        vl[b] = u.T;
        pl[b] = u.P;
        std::memcpy(&style[static_cast<size_t>(b) * 192], u.style, 192 * 4);
      }
      // Inputs: a group is packed into its ring half while the previous
      // group's copies (in the other half) run.
      for (uint32_t g0 = 0; g0 < B; g0 += kHalf) {
        const int base = static_cast<int>((g0 / kHalf) & 1) * kHalf;
        const uint32_t cnt = std::min<uint32_t>(kHalf, B - g0);
        for (uint32_t i = 0; i < cnt; ++i) ring.claim(base + static_cast<int>(i));
        parallel(cnt, [&](uint32_t i) {
          const itts_cfm_utt& u = utts[(*L.idx)[L.off + g0 + i]];
          float* sl = ring.at(base + static_cast<int>(i));
          float* noise = sl;
          float* px = sl + n80;
          float* cond = sl + 2 * n80;
          std::memcpy(noise, u.noise, static_cast<size_t>(u.T) * 80 * 4);
          std::memset(noise + static_cast<size_t>(u.T) * 80, 0, static_cast<size_t>(Tp - u.T) * 80 * 4);
          if (u.P) std::memcpy(px, u.prompt, static_cast<size_t>(u.P) * 80 * 4);
          std::memset(px + static_cast<size_t>(u.P) * 80, 0, static_cast<size_t>(Tp - u.P) * 80 * 4);
          std::memcpy(cond, u.cond, static_cast<size_t>(u.T) * 512 * 4);
          std::memset(cond + static_cast<size_t>(u.T) * 512, 0, static_cast<size_t>(Tp - u.T) * 512 * 4);
        });
        for (uint32_t i = 0; i < cnt; ++i) {
          const int sidx = base + static_cast<int>(i);
          const size_t b = g0 + i;
          const float* sl = ring.at(sidx);
          cuda_ok(cudaMemcpyAsync(w->X0 + b * n80, sl, n80 * 4, cudaMemcpyHostToDevice, st), "noise upload");
          cuda_ok(cudaMemcpyAsync(w->prompt_x + b * n80, sl + n80, n80 * 4, cudaMemcpyHostToDevice, st),
                  "prompt upload");
          cuda_ok(cudaMemcpyAsync(w->cond + b * n512, sl + 2 * n80, n512 * 4, cudaMemcpyHostToDevice, st),
                  "cond upload");
          ring.mark(sidx, st);
        }
      }
      cuda_ok(cudaMemcpyAsync(w->style, style.data(), style.size() * 4, cudaMemcpyHostToDevice, st), "style upload");
      upload_masks(e, w, vl.data(), pl.data(), nullptr);  // also drains the copies above
      ctx->staged = w;
      ctx->steps = static_cast<int>(steps);
      ctx->cfg = cfg_rate;
      e.enqueue_sampler(w, ctx->steps, ctx->cfg, true);
      check_status(e);
      // Outputs: each group is copied into a ring half, then unpacked by the
      // host threads while the next group's copies run.
      uint32_t prev_g0 = 0, prev_cnt = 0;
      int prev_base = 0;
      auto unpack = [&](uint32_t g0, uint32_t cnt, int base) {
        for (uint32_t i = 0; i < cnt; ++i) ring.claim(base + static_cast<int>(i));
        parallel(cnt, [&](uint32_t i) {
          const itts_cfm_utt& u = utts[(*L.idx)[L.off + g0 + i]];
          std::memcpy(u.out_mel, ring.at(base + static_cast<int>(i)), static_cast<size_t>(u.T) * 80 * 4);
        });
      };
      for (uint32_t g0 = 0; g0 < B; g0 += kHalf) {
        const int base = static_cast<int>((g0 / kHalf) & 1) * kHalf;
        const uint32_t cnt = std::min<uint32_t>(kHalf, B - g0);
        for (uint32_t i = 0; i < cnt; ++i) {
          const int sidx = base + static_cast<int>(i);
          ring.claim(sidx);
          cuda_ok(cudaMemcpyAsync(ring.at(sidx), w->X + (g0 + i) * n80, n80 * 4, cudaMemcpyDeviceToHost, st),
                  "mel download");
          ring.mark(sidx, st);
        }
        if (prev_cnt) unpack(prev_g0, prev_cnt, prev_base);
        prev_g0 = g0;
        prev_cnt = cnt;
        prev_base = base;
      }
      if (prev_cnt) unpack(prev_g0, prev_cnt, prev_base);
    }
  });
}

int itts_cfm_estimator(itts_cfm_ctx* ctx, uint32_t B, uint32_t T, uint32_t branches, const float* x,
                       const float* prompt_x, const float* cond, const float* style, const uint32_t* mask, float t,
                       float* vel) {
  return guarded(ctx, [&] {
    need(branches == 1 || branches == 2, "branches must be 1 or 2");
    check_run_args(B, T, 1, 0.0f, branches);
    need(x && prompt_x && cond && style && mask && vel, "null pointer");
    need(std::isfinite(t), "t must be finite");
    itts::Engine& e = *ctx->eng;
    itts::Work* w = e.work(static_cast<int>(B), static_cast<int>(T), static_cast<int>(branches));
    std::vector<uint32_t> zeros(B, 0u);
    upload_padded(e, w, nullptr, zeros.data(), x, prompt_x, cond, style, mask);
    const float* tab = e.tables_for_t(t);
    e.enqueue_prep(w);
    cuda_ok(itts::euler_init_run(w->X0, w->X, w->XD, w->plen, w->B, w->T, w->br, e.stream()), "x init");
    e.enqueue_estimator(w, tab);
    check_status(e);
    cuda_ok(cudaMemcpyAsync(vel, w->vel, static_cast<size_t>(w->R) * 80 * sizeof(float), cudaMemcpyDeviceToHost,
                            e.stream()),
            "velocity download");
    cuda_ok(cudaStreamSynchronize(e.stream()), "velocity sync");
    ctx->staged = nullptr;
  });
}

int itts_cfm_stage_padded(itts_cfm_ctx* ctx, uint32_t B, uint32_t T, const uint32_t* valid_len,
                          const uint32_t* prompt_len, const float* noise, const float* prompt_x, const float* cond,
                          const float* style, uint32_t steps, float cfg_rate) {
  return guarded(ctx, [&] {
    stage(ctx, B, T, valid_len, prompt_len, noise, prompt_x, cond, style, steps, cfg_rate);
    // Build tables and capture the graph now so launches are pure replays.
    ctx->eng->enqueue_sampler(ctx->staged, ctx->steps, ctx->cfg, true);
    check_status(*ctx->eng);
  });
}

int itts_cfm_launch(itts_cfm_ctx* ctx) {
  return guarded(ctx, [&] {
    need(ctx->staged != nullptr, "nothing staged");
    ctx->eng->enqueue_sampler(ctx->staged, ctx->steps, ctx->cfg, true);
  });
}

int itts_cfm_sync(itts_cfm_ctx* ctx) {
  return guarded(ctx, [&] {
    cuda_ok(cudaStreamSynchronize(ctx->eng->stream()), "sync");
    check_status(*ctx->eng);
  });
}

int itts_cfm_fetch(itts_cfm_ctx* ctx, float* out_mel) {
  return guarded(ctx, [&] { fetch(ctx, out_mel); });
}

void* itts_cfm_stream(itts_cfm_ctx* ctx) { return ctx ? static_cast<void*>(ctx->eng->stream()) : nullptr; }

int itts_cfm_launch_kernels(itts_cfm_ctx* ctx) {
  if (!ctx || !ctx->staged) return ITTS_EINVAL_SHAPE;
  uint32_t bits;
  std::memcpy(&bits, &ctx->cfg, 4);
  auto it = ctx->staged->graph_kernels.find(std::make_pair(ctx->steps, bits));
  return it == ctx->staged->graph_kernels.end() ? ITTS_EINVAL_SHAPE : it->second;
}

int itts_cfm_profile_step(itts_cfm_ctx* ctx, int reps, itts_kernel_stat* out, int cap, int* n_out) {
  return guarded(ctx, [&] {
    need(ctx->staged != nullptr, "nothing staged");
    need(reps >= 1 && out && cap > 0 && n_out, "bad profile arguments");
    auto kt = ctx->eng->profile_step(ctx->staged, ctx->steps, ctx->cfg, reps);
    check_status(*ctx->eng);
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

int itts_cfm_selftest_timeout(itts_cfm_ctx* ctx, uint64_t budget_cycles) {
  return guarded(ctx, [&] {
    need(budget_cycles >= 1000 && budget_cycles <= 1000000000ull, "budget_cycles must be within 1e3..1e9");
    itts::Engine& e = *ctx->eng;
    e.clear_status();
    cuda_ok(itts::bounded_wait_probe_run(e.status_ptr(), static_cast<long long>(budget_cycles), e.stream()),
            "self-test launch");
    cuda_ok(cudaStreamSynchronize(e.stream()), "self-test sync");
    check_status(e);
    throw std::runtime_error("self-test: the bounded wait did not report its expiry");
  });
}

int itts_op_gemm(itts_cfm_ctx* ctx, const void* a0, uint32_t lda0, const void* a1, uint32_t lda1, uint32_t k0,
                 const void* b, uint32_t ldb, const float* bias, float* c, uint32_t ldc, uint32_t M, uint32_t N,
                 uint32_t K, uint32_t bn) {
  return guarded(ctx, [&] {
    need(a0 && b && c && M > 0 && N > 0 && K > 0, "bad gemm arguments");
    const bool pair = (bn & ITTS_GEMM_PAIR) != 0;
    bn &= ~ITTS_GEMM_PAIR;
    need(bn == 64 || bn == 80 || bn == 128 || bn == 192 || bn == 256, "bn must be 64, 80, 128, 192 or 256");
    need(!pair || bn == 64 || bn == 128 || bn == 256, "the CTA-pair form takes bn 64, 128 or 256");
    need(N % 16 == 0 && ldc % 4 == 0, "N must be a multiple of 16, ldc of 4");
    itts::GemmLaunch g;
    std::memset(&g, 0, sizeof(g));
    const uint32_t ka = a1 ? k0 : K;
    const uint32_t kbox = static_cast<uint32_t>(itts::gemm_kbox(static_cast<int>(bn)));
    need(!a1 || (k0 % (64 * kbox) == 0 && k0 < K),
         "k0 must be below K and a multiple of 64 x the k-blocks per TMA box (256 for bn 64, 128 for bn 80/128, 64 for "
         "bn 256)");
    need(K % 64 == 0, "K must be a multiple of 64 (zero-pad the operands)");
    if (!itts::make_tmap_f16(&g.tmA0, a0, ka, M, lda0, 128, kbox)) throw ShapeError("A0 layout rejected by TMA");
    if (a1) {
      if (!itts::make_tmap_f16(&g.tmA1, a1, K - k0, M, lda1, 128, kbox)) throw ShapeError("A1 layout rejected by TMA");
    } else {
      g.tmA1 = g.tmA0;
    }
    if (!itts::make_tmap_f16(&g.tmB, b, K, N, ldb, pair ? bn / 2 : bn, kbox))
      throw ShapeError("B layout rejected by TMA");
    g.args.M = static_cast<int>(M);
    g.args.N = static_cast<int>(N);
    g.args.a_mode = a1 ? itts::kASplit : itts::kAPlain;
    g.args.kb_split = static_cast<int>(k0 / 64);
    g.args.num_kb = a1 ? static_cast<int>(k0 / 64 + (K - k0 + 63) / 64) : static_cast<int>((K + 63) / 64);
    g.args.epi = itts::kEpiF32;
    g.args.bias = bias;
    g.args.out32 = c;
    g.args.ld32 = static_cast<int>(ldc);
    g.args.seq_T = 1;
    g.bn = static_cast<int>(bn);
    g.pair = pair ? 1 : 0;
    itts::Engine& e = *ctx->eng;
    e.clear_status();
    cuda_ok(itts::gemm_run(g, e.stream()), "gemm launch");
    cuda_ok(cudaStreamSynchronize(e.stream()), "gemm sync");
    check_status(e);
  });
}

int itts_op_conv5(itts_cfm_ctx* ctx, const void* xp, uint32_t S, uint32_t T, const void* w, const float* bias,
                  float* out, uint32_t N) {
  return guarded(ctx, [&] {
    need(xp && w && out && S > 0 && T >= ITTS_MIN_T && T <= ITTS_MAX_T && N > 0 && N % 16 == 0,
         "bad conv arguments");
    const uint64_t rows = static_cast<uint64_t>(S) * (static_cast<uint64_t>(T) + 4);
    need(rows <= static_cast<uint64_t>(INT32_MAX), "conv too large: S*(T+4) padded rows must fit in 31 bits");
    itts::GemmLaunch g;
    std::memset(&g, 0, sizeof(g));
    const uint32_t Rp = static_cast<uint32_t>(rows);
    // Tile shape and form as the engine picks them for its WaveNet convs.
    const itts::GemmPick pk = itts::gemm_pick(static_cast<int>(Rp), static_cast<int>(N), false);
    const uint32_t kbox = static_cast<uint32_t>(itts::gemm_kbox(pk.bn));
    if (!itts::make_tmap_f16(&g.tmA0, xp, 512, Rp, 512, 128, kbox)) throw ShapeError("xp layout rejected by TMA");
    g.tmA1 = g.tmA0;
    if (!itts::make_tmap_f16(&g.tmB, w, 2560, N, 2560, static_cast<uint32_t>(pk.pair ? pk.bn / 2 : pk.bn), kbox))
      throw ShapeError("w layout rejected by TMA");
    g.args.M = static_cast<int>(Rp);
    g.args.N = static_cast<int>(N);
    g.args.a_mode = itts::kAConv;
    g.args.kb_per_tap = 8;
    g.args.conv_dil = 1;
    g.args.conv_off = -2;
    g.args.num_kb = 40;
    g.args.epi = itts::kEpiF32;
    g.args.pad_rows = 1;
    g.args.bias = bias;
    g.args.out32 = out;
    g.args.ld32 = static_cast<int>(N);
    g.args.seq_T = static_cast<int>(T);
    g.bn = pk.bn;
    g.pair = pk.pair;
    itts::Engine& e = *ctx->eng;
    e.clear_status();
    cuda_ok(itts::gemm_run(g, e.stream()), "conv launch");
    cuda_ok(cudaStreamSynchronize(e.stream()), "conv sync");
    check_status(e);
  });
}

int itts_op_attention(itts_cfm_ctx* ctx, const void* qkv, const float* row_mask, void* out, uint32_t S, uint32_t T) {
  return guarded(ctx, [&] {
    need(qkv && row_mask && out && S > 0 && T > 0, "bad attention arguments");
    itts::Engine& e = *ctx->eng;
    CUtensorMap tm;
    if (!itts::make_attn_tmap(&tm, static_cast<const __half*>(qkv), static_cast<int>(S * T)))
      throw ShapeError("qkv layout rejected by TMA");
    e.clear_status();
    cuda_ok(itts::attention_tc_run(tm, row_mask, static_cast<__half*>(out), static_cast<int>(S), static_cast<int>(T),
                                   e.status_ptr(), e.stream()),
            "attention launch");
    cuda_ok(cudaStreamSynchronize(e.stream()), "attention sync");
    check_status(e);
  });
}

int itts_op_adarms(itts_cfm_ctx* ctx, const float* x, uint32_t R, const float* wb, const float* gamma, void* y) {
  return guarded(ctx, [&] {
    need(x && wb && gamma && y && R > 0, "bad adarms arguments");
    itts::Engine& e = *ctx->eng;
    cuda_ok(itts::adarms_run(x, static_cast<int>(R), wb, gamma, static_cast<__half*>(y), e.stream()), "adarms launch");
    cuda_ok(cudaStreamSynchronize(e.stream()), "adarms sync");
  });
}

}  // extern "C"
