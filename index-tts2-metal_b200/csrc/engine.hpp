// DiT-CFM sampler engine: one per (host thread, GPU). Owns the resident
// weights, the per-`steps` t-conditioning tables, shape-keyed workspaces and
// their CUDA graphs.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

#include "bundle.hpp"
#include "gemm.cuh"
#include "model.hpp"

namespace itts {

// Per-kernel-kind timing gathered by Engine::profile_step.
struct KernelTiming {
  std::string name;
  int launches = 0;
  double ms = 0.0;
  double flops = 0.0;  // algorithmic FLOPs of all launches of this kind
  double bytes = 0.0;  // compulsory HBM bytes of all launches of this kind
};

// Device buffers for B utterances padded to T rows, with `branches` estimator
// branches each (2 = conditional + null for CFG, 1 = conditional only).
struct Work {
  int B = 0, T = 0, br = 0, S = 0, R = 0, Rp = 0;
  // inputs / state
  float* X0 = nullptr;        // [B*T, 80] initial noise (kept for replays)
  float* X = nullptr;         // [B*T, 80] mel state (fp32)
  __half* XD = nullptr;       // [S*T, kXdLd] f16 copy per branch (GEMM operand; columns >= 80 stay 0)
  float* prompt_x = nullptr;  // [B*T, 80]
  float* cond = nullptr;      // [B*T, 512]
  float* style = nullptr;     // [B, 192]
  int* plen = nullptr;        // [B] prompt rows
  float* mask = nullptr;      // [S*T] key / WaveNet mask
  // step-invariant merge
  __half* cond16 = nullptr;
  __half* cp16 = nullptr;
  __half* U = nullptr;    // [R, kUld] (columns >= 784 stay 0)
  float* base = nullptr;  // [R, 512]
  // transformer
  float* xres = nullptr;
  __half* skip16[6] = {};
  __half* xn16 = nullptr;  // normalised GEMM operand (folded AdaRMS: x * w * g)
  float* ss = nullptr;     // [16][R] per-32-column partial sums of squares of the normalised x
  __half* qkv16 = nullptr;
  __half* attn16 = nullptr;
  float* h = nullptr;
  // [R, 2048] f16: columns 512.. hold every layer's SwiGLU activations g;
  // columns 0..511 f16(h) of layers 6..11, whose w2 is composed into the next
  // layer's skip_in_linear (that GEMM reads [h | g | skip] directly).
  __half* cat16 = nullptr;
  // post + wavenet + final
  __half* xp16 = nullptr;  // [S*(T+4), 512]
  float* res = nullptr;
  __half* gate16 = nullptr;
  float* wacc = nullptr;
  float* fin = nullptr;
  __half* fn16 = nullptr;
  float* vel = nullptr;  // [R, 80]
  float2* rope = nullptr;
  CUtensorMap tm_attn;  // qkv16 viewed for the attention kernel
  void* arena = nullptr;
  size_t arena_bytes = 0;
  // prebuilt GEMM launches
  GemmLaunch g_cp, g_base, g_merge, g_qkv[kLayers], g_wo[kLayers], g_w13[kLayers], g_w2[kLayers],
      g_skip[kLayers], g_post, g_in[kWnLayers], g_rs[kWnLayers], g_out;
  // captured sampler graphs keyed by (steps, cfg bits)
  std::map<std::pair<int, uint32_t>, cudaGraphExec_t> graphs;
  std::map<std::pair<int, uint32_t>, int> graph_kernels;  // kernel nodes per captured graph
};

class Engine {
 public:
  Engine(const std::string& bundle_dir, int device, bool verify_sha256);
  ~Engine();

  int device() const { return device_; }
  cudaStream_t stream() const { return stream_; }
  const DevWeights& weights() const { return w_; }

  Work* work(int B, int T, int branches);
  // Device table [steps][kTcondPerStep] for the Euler schedule t_i = i/steps (fp32 accumulation).
  const float* tables_for_steps(int steps);
  // Device table [1][kTcondPerStep] for one timestep value.
  const float* tables_for_t(float t);

  // Enqueue the whole sampler on stream(): inputs must already be in the
  // workspace (X, prompt_x, cond, style, plen, mask). With use_graph the
  // sequence is captured once per (shape, steps, cfg) and replayed.
  void enqueue_sampler(Work* w, int steps, float cfg, bool use_graph);
  // Enqueue one estimator evaluation at the table row `tab` (velocity -> w->vel).
  void enqueue_estimator(Work* w, const float* tab);
  // Enqueue the step-invariant input preparation.
  void enqueue_prep(Work* w);
  // Time every kernel of one sampler step (events around each launch).
  std::vector<KernelTiming> profile_step(Work* w, int steps, float cfg, int reps);

  // Device status word (non-zero after a kernel abandoned a bounded wait).
  unsigned int read_status();
  unsigned int* status_ptr() const { return d_status_; }
  void clear_status();

 private:
  void build_work_launches(Work* w);
  void enqueue_step(Work* w, const float* tab, float dt, float cfg, bool do_update,
                    std::vector<KernelTiming>* prof);
  void check(cudaError_t e, const char* what);

  int device_ = 0;
  cudaStream_t stream_ = nullptr;
  DevWeights w_;
  unsigned int* d_status_ = nullptr;
  std::map<int, float*> step_tables_;
  std::map<uint32_t, float*> t_tables_;
  std::map<std::tuple<int, int, int>, std::unique_ptr<Work>> works_;
};

// Algorithmic FLOPs of one guided step for S sequences of T rows
// (GEMMs + attention, the per-step cost model of the sampler).
double step_flops(int S, int T);

}  // namespace itts
