// Condition assembly: weights, the interpolation / GroupNorm / Mish kernels
// and the launch schedule (see condition.hpp).
#include "condition.hpp"

#include <cmath>
#include <cstring>
#include <stdexcept>
#include <vector>

#include "bundle.hpp"
#include "kernels.cuh"

namespace itts {

namespace {

constexpr int kC = 512;
constexpr int kIn = 1024;
constexpr int kGnBlocks = 296;  // partial sums per GroupNorm pass (2 per SM)
const std::string kLr = "s2mel.net.length_regulator.";

// Nearest interpolation of cpu_nearest_interpolate
// (runtime/impl/tokenizer_tests.cpp:3127-3141): row t takes input row
// floor(t * (n_in / n_out)) (float arithmetic as the reference), clamped;
// written as the f16 operand of the first conv.
__global__ void __launch_bounds__(256) interp_kernel(const float* __restrict__ proj, int n_in, int n_out,
                                                     __half* __restrict__ out) {
  const float scale = static_cast<float>(n_in) / static_cast<float>(n_out);
  const size_t n = static_cast<size_t>(n_out) * kC;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / kC);
    const int c = static_cast<int>(i - static_cast<size_t>(t) * kC);
    unsigned src = static_cast<unsigned>(floorf(static_cast<float>(t) * scale));
    if (src >= static_cast<unsigned>(n_in)) src = static_cast<unsigned>(n_in) - 1;
    out[i] = __float2half_rn(proj[static_cast<size_t>(src) * kC + c]);
  }
}

// Block sum of 256 values (fixed tree: deterministic).
__device__ __forceinline__ float block_sum(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.0f;
  if (threadIdx.x < 32) {
    t = threadIdx.x < 8 ? sh[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  }
  return t;  // valid in thread 0
}

// Sum of the kGnBlocks partials in index order (every block gets the same value).
__device__ __forceinline__ float partials_sum(const float* __restrict__ part, float* sh) {
  float v = 0.0f;
  for (int i = threadIdx.x; i < kGnBlocks; i += 256) v += part[i];
  float s = block_sum(v, sh);
  __syncthreads();
  if (threadIdx.x == 0) sh[8] = s;
  __syncthreads();
  s = sh[8];
  __syncthreads();
  return s;
}

// GroupNorm with one group (cpu_groupnorm1, runtime/impl/tokenizer_tests.cpp:
// 3874-3896) over all n values, in three passes: partial sums of x; partial
// sums of (x - mean)^2 (each block first reduces the sums to the mean); then
// y = (x - mean) / sqrt(var + 1e-5) * gamma + beta and Mish
// (cpu_mish, :3898-3904: y tanh(log1p(exp(y)))) -> f16 operand of the next conv.
__global__ void __launch_bounds__(256) gn_sum_kernel(const float* __restrict__ x, size_t n, float* __restrict__ part) {
  __shared__ float sh[9];
  float v = 0.0f;
  for (size_t i = static_cast<size_t>(blockIdx.x) * 256 + threadIdx.x; i < n; i += static_cast<size_t>(kGnBlocks) * 256)
    v += x[i];
  const float s = block_sum(v, sh);
  if (threadIdx.x == 0) part[blockIdx.x] = s;
}

__global__ void __launch_bounds__(256) gn_var_kernel(const float* __restrict__ x, size_t n,
                                                     const float* __restrict__ part_sum, float* __restrict__ part_sq) {
  __shared__ float sh[9];
  const float mean = partials_sum(part_sum, sh) / static_cast<float>(n);
  float v = 0.0f;
  for (size_t i = static_cast<size_t>(blockIdx.x) * 256 + threadIdx.x; i < n; i += static_cast<size_t>(kGnBlocks) * 256) {
    const float d = x[i] - mean;
    v += d * d;
  }
  const float s = block_sum(v, sh);
  if (threadIdx.x == 0) part_sq[blockIdx.x] = s;
}

__global__ void __launch_bounds__(256) gn_mish_kernel(const float* __restrict__ x, size_t n,
                                                      const float* __restrict__ part_sum,
                                                      const float* __restrict__ part_sq, const float* __restrict__ gamma,
                                                      const float* __restrict__ beta, __half* __restrict__ out) {
  __shared__ float sh[9];
  const float mean = partials_sum(part_sum, sh) / static_cast<float>(n);
  const float var = partials_sum(part_sq, sh) / static_cast<float>(n);
  const float inv = 1.0f / sqrtf(var + 1e-5f);
  for (size_t i = static_cast<size_t>(blockIdx.x) * 256 + threadIdx.x; i < n; i += static_cast<size_t>(kGnBlocks) * 256) {
    const int c = static_cast<int>(i % kC);
    const float y = (x[i] - mean) * inv * gamma[c] + beta[c];
    out[i] = __float2half_rn(y * tanhf(log1pf(expf(y))));
  }
}

std::vector<uint16_t> h16_of(const Mit2Bundle& b, const std::string& n, size_t want) {
  std::vector<float> f = b.as_f32(n);
  if (f.size() != want) throw std::runtime_error("condition weights: " + n + " has an unexpected size");
  std::vector<uint16_t> h(want);
  for (size_t i = 0; i < want; ++i) h[i] = float_to_half_bits(f[i]);
  return h;
}

std::vector<float> f32_of(const Mit2Bundle& b, const std::string& n, size_t want) {
  std::vector<float> f = b.as_f32(n);
  if (f.size() != want) throw std::runtime_error("condition weights: " + n + " has an unexpected size");
  return f;
}

GemmLaunch plain_gemm(const __half* a, int M, int K, const __half* w, int N, const float* bias, float* out32,
                      unsigned int* status, int a_mode, int taps) {
  GemmLaunch g;
  std::memset(&g, 0, sizeof(g));
  const int kin = K / taps;  // channels per tap
  const GemmPick pk = gemm_pick(M, N, false);
  const uint32_t kbox = static_cast<uint32_t>(gemm_kbox(pk.bn));
  if (!make_tmap_f16(&g.tmA0, a, kin, M, kin, 128, kbox)) throw std::runtime_error("condition: tensor map for A rejected");
  g.tmA1 = g.tmA0;
  if (!make_tmap_f16(&g.tmB, w, K, N, K, pk.bn, kbox)) throw std::runtime_error("condition: tensor map for W rejected");
  g.args.M = M;
  g.args.N = N;
  g.args.num_kb = K / 64;
  g.args.a_mode = a_mode;
  g.args.kb_per_tap = kin / 64;
  g.args.conv_dil = 1;
  g.args.conv_off = -(taps / 2);
  g.args.epi = kEpiF32;
  g.args.bias = bias;
  g.args.out32 = out32;
  g.args.ld32 = N;
  g.args.seq_T = M;
  g.args.status = status;
  g.bn = pk.bn;
  g.pair = 0;
  return g;
}

unsigned grid_of(size_t n) {
  const size_t b = (n + 255) / 256;
  return static_cast<unsigned>(b < 1184 ? (b ? b : 1) : 1184);
}

}  // namespace

struct ConditionAssembler::Plan {
  int n_in = 0, P = 0, G = 0;
  void* mem = nullptr;
  float* x32 = nullptr;     // s_infer upload [n_in][1024]
  __half* x16 = nullptr;    // [n_in][1024]
  float* proj = nullptr;    // [n_in][512]
  __half* a16 = nullptr;    // [G][512] conv operand
  float* h32 = nullptr;     // [G][512] conv output
  float* part = nullptr;    // [2][kGnBlocks]
  float* cond = nullptr;    // [P + G][512]
  GemmLaunch in_proj, conv[4], out;
  cudaGraphExec_t graph = nullptr;
  int kernels = 0;
};

void ConditionAssembler::check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string("cuda: condition: ") + what + ": " + cudaGetErrorString(e));
}

ConditionAssembler::ConditionAssembler(const std::string& bundle_dir, int device, bool verify_sha256)
    : device_(device) {
  int n = 0;
  check(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
  if (device < 0 || device >= n) throw std::runtime_error("device id out of range");
  check(cudaSetDevice(device), "cudaSetDevice");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10 || minor != 0) throw std::runtime_error("this build targets sm_100a (B200) only");
  Mit2Bundle b(bundle_dir, verify_sha256);
  std::vector<uint8_t> host;
  auto put = [&](const void* p, size_t bytes) {
    const size_t off = host.size();
    host.resize(off + ((bytes + 255) & ~size_t(255)), 0);
    std::memcpy(host.data() + off, p, bytes);
    return off;
  };
  auto put_h = [&](const std::vector<uint16_t>& v) { return put(v.data(), v.size() * 2); };
  auto put_f = [&](const std::vector<float>& v) { return put(v.data(), v.size() * 4); };
  const size_t o_win = put_h(h16_of(b, kLr + "content_in_proj.weight", static_cast<size_t>(kC) * kIn));
  const size_t o_bin = put_f(f32_of(b, kLr + "content_in_proj.bias", kC));
  const int convs[4] = {0, 3, 6, 9}, norms[4] = {1, 4, 7, 10};
  size_t o_wc[4], o_bc[4], o_g[4], o_b[4];
  for (int i = 0; i < 4; ++i) {
    const std::string cp = kLr + "model." + std::to_string(convs[i]);
    const std::string np = kLr + "model." + std::to_string(norms[i]);
    // conv weight [o][i][k] -> GEMM operand [o][k][i]
    std::vector<float> w = f32_of(b, cp + ".weight", static_cast<size_t>(kC) * kC * 3);
    std::vector<uint16_t> h(w.size());
    for (int o = 0; o < kC; ++o)
      for (int ci = 0; ci < kC; ++ci)
        for (int k = 0; k < 3; ++k)
          h[(static_cast<size_t>(o) * 3 + k) * kC + ci] = float_to_half_bits(w[(static_cast<size_t>(o) * kC + ci) * 3 + k]);
    o_wc[i] = put_h(h);
    o_bc[i] = put_f(f32_of(b, cp + ".bias", kC));
    o_g[i] = put_f(f32_of(b, np + ".weight", kC));
    o_b[i] = put_f(f32_of(b, np + ".bias", kC));
  }
  const size_t o_wo = put_h(h16_of(b, kLr + "model.12.weight", static_cast<size_t>(kC) * kC));
  const size_t o_bo = put_f(f32_of(b, kLr + "model.12.bias", kC));
  check(cudaMalloc(&arena_, host.size()), "condition weights cudaMalloc");
  check(cudaMemcpy(arena_, host.data(), host.size(), cudaMemcpyHostToDevice), "condition weights upload");
  const uint8_t* base = static_cast<const uint8_t*>(arena_);
  w_in_ = reinterpret_cast<const __half*>(base + o_win);
  b_in_ = reinterpret_cast<const float*>(base + o_bin);
  for (int i = 0; i < 4; ++i) {
    w_conv_[i] = reinterpret_cast<const __half*>(base + o_wc[i]);
    b_conv_[i] = reinterpret_cast<const float*>(base + o_bc[i]);
    gn_g_[i] = reinterpret_cast<const float*>(base + o_g[i]);
    gn_b_[i] = reinterpret_cast<const float*>(base + o_b[i]);
  }
  w_out_ = reinterpret_cast<const __half*>(base + o_wo);
  b_out_ = reinterpret_cast<const float*>(base + o_bo);
  check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
  check(cudaMalloc(&d_status_, sizeof(unsigned int)), "cudaMalloc status");
  check(cudaMemset(d_status_, 0, sizeof(unsigned int)), "cudaMemset status");
}

ConditionAssembler::~ConditionAssembler() {
  cudaSetDevice(device_);
  if (stream_) cudaStreamSynchronize(stream_);
  for (auto& kv : plans_) {
    if (kv.second->graph) cudaGraphExecDestroy(kv.second->graph);
    if (kv.second->mem) cudaFree(kv.second->mem);
  }
  if (arena_) cudaFree(arena_);
  if (d_status_) cudaFree(d_status_);
  if (stream_) cudaStreamDestroy(stream_);
}

unsigned int ConditionAssembler::read_status() {
  unsigned int v = 0;
  check(cudaMemcpyAsync(&v, d_status_, sizeof(v), cudaMemcpyDeviceToHost, stream_), "status read");
  check(cudaStreamSynchronize(stream_), "status sync");
  return v;
}

void ConditionAssembler::clear_status() {
  check(cudaMemsetAsync(d_status_, 0, sizeof(unsigned int), stream_), "status clear");
}

ConditionAssembler::Plan* ConditionAssembler::plan_for(int n_in, int P, int G) {
  const auto key = std::make_tuple(n_in, P, G);
  auto it = plans_.find(key);
  if (it != plans_.end()) return it->second.get();
  auto p = std::make_unique<Plan>();
  p->n_in = n_in;
  p->P = P;
  p->G = G;
  size_t off = 0;
  auto carve = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  };
  const size_t o_x32 = carve(static_cast<size_t>(n_in) * kIn * 4), o_x16 = carve(static_cast<size_t>(n_in) * kIn * 2),
               o_proj = carve(static_cast<size_t>(n_in) * kC * 4), o_a16 = carve(static_cast<size_t>(G) * kC * 2),
               o_h = carve(static_cast<size_t>(G) * kC * 4), o_part = carve(2 * kGnBlocks * 4),
               o_cond = carve(static_cast<size_t>(P + G) * kC * 4);
  check(cudaMalloc(&p->mem, off), "condition workspace cudaMalloc");
  check(cudaMemset(p->mem, 0, off), "condition workspace memset");
  uint8_t* m = static_cast<uint8_t*>(p->mem);
  p->x32 = reinterpret_cast<float*>(m + o_x32);
  p->x16 = reinterpret_cast<__half*>(m + o_x16);
  p->proj = reinterpret_cast<float*>(m + o_proj);
  p->a16 = reinterpret_cast<__half*>(m + o_a16);
  p->h32 = reinterpret_cast<float*>(m + o_h);
  p->part = reinterpret_cast<float*>(m + o_part);
  p->cond = reinterpret_cast<float*>(m + o_cond);
  p->in_proj = plain_gemm(p->x16, n_in, kIn, w_in_, kC, b_in_, p->proj, d_status_, kAPlain, 1);
  for (int i = 0; i < 4; ++i) p->conv[i] = plain_gemm(p->a16, G, 3 * kC, w_conv_[i], kC, b_conv_[i], p->h32, d_status_, kAConv, 3);
  p->out = plain_gemm(p->a16, G, kC, w_out_, kC, b_out_, p->cond + static_cast<size_t>(P) * kC, d_status_, kAPlain, 1);
  Plan* raw = p.get();
  plans_[key] = std::move(p);
  cudaGraph_t graph = nullptr;
  check(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "condition begin capture");
  try {
    enqueue(raw);
  } catch (...) {
    cudaStreamEndCapture(stream_, &graph);
    if (graph) cudaGraphDestroy(graph);
    throw;
  }
  check(cudaStreamEndCapture(stream_, &graph), "condition end capture");
  size_t nn = 0;
  cudaGraphGetNodes(graph, nullptr, &nn);
  std::vector<cudaGraphNode_t> nodes(nn);
  if (nn) cudaGraphGetNodes(graph, nodes.data(), &nn);
  for (auto nd : nodes) {
    cudaGraphNodeType ty;
    if (cudaGraphNodeGetType(nd, &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++raw->kernels;
  }
  const cudaError_t e = cudaGraphInstantiate(&raw->graph, graph, 0);
  cudaGraphDestroy(graph);
  check(e, "condition graph instantiate");
  return raw;
}

void ConditionAssembler::enqueue(Plan* p) {
  const size_t n = static_cast<size_t>(p->G) * kC;
  check(to_half_run(p->x32, p->x16, static_cast<size_t>(p->n_in) * kIn, stream_), "s_infer to f16");
  check(gemm_run(p->in_proj, stream_), "content_in_proj");
  interp_kernel<<<grid_of(n), 256, 0, stream_>>>(p->proj, p->n_in, p->G, p->a16);
  check(cudaGetLastError(), "interpolation");
  for (int i = 0; i < 4; ++i) {
    check(gemm_run(p->conv[i], stream_), "regulator conv");
    gn_sum_kernel<<<kGnBlocks, 256, 0, stream_>>>(p->h32, n, p->part);
    check(cudaGetLastError(), "groupnorm sum");
    gn_var_kernel<<<kGnBlocks, 256, 0, stream_>>>(p->h32, n, p->part, p->part + kGnBlocks);
    check(cudaGetLastError(), "groupnorm variance");
    gn_mish_kernel<<<grid_of(n), 256, 0, stream_>>>(p->h32, n, p->part, p->part + kGnBlocks, gn_g_[i], gn_b_[i], p->a16);
    check(cudaGetLastError(), "groupnorm + mish");
  }
  check(gemm_run(p->out, stream_), "regulator output conv");
}

void ConditionAssembler::stage(const float* s_infer, int n_in, const float* prompt, int P, int G) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  Plan* p = plan_for(n_in, P, G);
  check(cudaMemcpyAsync(p->x32, s_infer, static_cast<size_t>(n_in) * kIn * 4, cudaMemcpyHostToDevice, stream_),
        "s_infer upload");
  if (P > 0)
    check(cudaMemcpyAsync(p->cond, prompt, static_cast<size_t>(P) * kC * 4, cudaMemcpyHostToDevice, stream_),
          "prompt condition upload");
  staged_ = p;
}

void ConditionAssembler::launch() {
  if (!staged_) throw std::runtime_error("condition: nothing staged");
  check(cudaGraphLaunch(staged_->graph, stream_), "condition graph launch");
}

void ConditionAssembler::fetch(float* cond) {
  if (!staged_) throw std::runtime_error("condition: nothing staged");
  check(cudaMemcpyAsync(cond, staged_->cond, static_cast<size_t>(staged_->P + staged_->G) * kC * 4,
                        cudaMemcpyDeviceToHost, stream_),
        "condition download");
  check(cudaStreamSynchronize(stream_), "condition sync");
}

void ConditionAssembler::run(const float* s_infer, int n_in, const float* prompt, int P, int G, float* cond) {
  stage(s_infer, n_in, prompt, P, G);
  launch();
  fetch(cond);
}

int ConditionAssembler::launches_per_run() const { return staged_ ? staged_->kernels : -1; }

double ConditionAssembler::flops(int n_in, int G) {
  return 2.0 * (static_cast<double>(n_in) * kIn * kC + 4.0 * G * kC * kC * 3 + static_cast<double>(G) * kC * kC);
}

}  // namespace itts
