// GPT mel-code decoder: weights, the GEMV / attention / argmax kernels and the
// per-token graphs (see gpt.hpp).
#include "gpt.hpp"

#include <algorithm>
#include <cfloat>
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "bundle.hpp"
#include "gpt_prefill.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace itts {

namespace {

constexpr int kW = GptDecoder::kW;
constexpr int kMaxLen = GptDecoder::kMaxLen;
constexpr int kHeads = GptDecoder::kHeads;
constexpr int kDecodeChunk = 8;   // decode steps per host check of the stop flag
constexpr int kSplits = 7;        // key ranges per head in the attention (7 x 20 heads = 140 CTAs)
constexpr int kPart = 66;         // per (head, range) partial: max, sum, 64 accumulators
constexpr int kSplitKeys = (kMaxLen + kSplits - 1) / kSplits + 1;  // longest key range

enum { kProPlain = 0, kProLn = 1, kProLn2 = 2, kProAttn = 3 };
enum { kEpiBias = 0, kEpiGelu = 1, kEpiResid = 2 };

struct GemvArgs {
  const float* x;                  // [K] input row (kProAttn: the attention partials)
  const float *g1, *b1, *g2, *b2;  // LayerNorm(s) of the prologue
  const __half* w;                 // [N][K] f16
  const float* bias;               // [N]
  const float* resid;              // [N] (kEpiResid)
  float* y;                        // [N]
  int n;                           // rows
  int rpc;                         // rows per CTA
  const int* ctl;                  // ctl[4] nonzero: the decode has ended, do nothing
  unsigned int* status;            // bounded-wait failures
};

// Sum of one value per thread over an NT-thread block, returned to every
// thread (fixed reduction tree: deterministic).
template <int NT>
__device__ __forceinline__ float block_sum_all(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) t += red[w];
  __syncthreads();
  return t;
}

template <int NT>
__device__ __forceinline__ float block_max_all(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = red[0];
#pragma unroll
  for (int w = 1; w < NT / 32; ++w) t = fmaxf(t, red[w]);
  __syncthreads();
  return t;
}

// cpu_layernorm (runtime/impl/tokenizer_tests.cpp:2992-3010) on the row held
// in shared memory: mean, biased variance, (x - mean) * (1 / sqrt(var + 1e-5))
// * gamma + beta.
template <int K, int NT>
__device__ __forceinline__ void layer_norm_smem(float* xs, const float* __restrict__ g, const float* __restrict__ b,
                                                float* red) {
  float s = 0.0f;
  for (int i = threadIdx.x; i < K; i += NT) s += xs[i];
  const float mean = block_sum_all<NT>(s, red) / static_cast<float>(K);
  float v = 0.0f;
  for (int i = threadIdx.x; i < K; i += NT) {
    const float d = xs[i] - mean;
    v += d * d;
  }
  const float var = block_sum_all<NT>(v, red) / static_cast<float>(K);
  const float inv = 1.0f / sqrtf(var + 1e-5f);
  for (int i = threadIdx.x; i < K; i += NT) xs[i] = (xs[i] - mean) * inv * g[i] + b[i];
  __syncthreads();
}

// gelu_new of cpu_gelu_new (runtime/impl/tokenizer_tests.cpp:3931-3945),
// with its clamps: x > 10 -> x, x < -10 -> 0.
__device__ __forceinline__ float gelu_new(float x) {
  if (x > 10.0f) return x;
  if (x < -10.0f) return 0.0f;
  const float c = 0.7978845608028654f;
  return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
}

__device__ __forceinline__ float dot8(const uint4 w, const float* xs) {
  const float4 xa = *reinterpret_cast<const float4*>(xs);
  const float4 xb = *reinterpret_cast<const float4*>(xs + 4);
  const float2 w0 = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
  const float2 w1 = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
  const float2 w2 = __half22float2(*reinterpret_cast<const __half2*>(&w.z));
  const float2 w3 = __half22float2(*reinterpret_cast<const __half2*>(&w.w));
  float s = w0.x * xa.x;
  s = fmaf(w0.y, xa.y, s);
  s = fmaf(w1.x, xa.z, s);
  s = fmaf(w1.y, xa.w, s);
  s = fmaf(w2.x, xb.x, s);
  s = fmaf(w2.y, xb.y, s);
  s = fmaf(w3.x, xb.z, s);
  s = fmaf(w3.y, xb.w, s);
  return s;
}

// Merges the attention's per-range partials into the heads' outputs
// (1280 values in xs): M = max_r m_r, out = sum_r acc_r e^(m_r - M) /
// sum_r l_r e^(m_r - M), ranges in index order.
template <int NT>
__device__ __forceinline__ void attn_combine_smem(const float* __restrict__ part, float* xs) {
  for (int i = threadIdx.x; i < kW; i += NT) {
    const int h = i >> 6, d = i & 63;
    const float* p = part + static_cast<size_t>(h) * kSplits * kPart;
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < kSplits; ++r)
      if (p[r * kPart + 1] > 0.0f) M = fmaxf(M, p[r * kPart]);
    float L = 0.0f, A = 0.0f;
#pragma unroll
    for (int r = 0; r < kSplits; ++r) {
      const float l = p[r * kPart + 1];
      if (l > 0.0f) {
        const float e = expf(p[r * kPart] - M);
        L = fmaf(l, e, L);
        A = fmaf(p[r * kPart + 2 + d], e, A);
      }
    }
    xs[i] = A / L;
  }
  __syncthreads();
}

// Weight load that bypasses L1 (each weight byte is read once per token).
// Volatile: every weight load of the kernel stays ahead of the dependency
// wait that follows them.
__device__ __forceinline__ uint4 ldg_weights(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

constexpr int kGemvThreads = 512;

// y[n] = epilogue(W[n,:] . prologue(x) + bias[n]). The work is cut into
// tasks (row, segment of K / SEG columns); warp w of CTA b takes tasks
// b * tpc + w + 16 i (i < RW). Every weight load of the CTA's tasks (f16,
// 16 bytes per lane, 512 contiguous bytes per warp load) and the biases are
// issued BEFORE the kernel waits on its predecessor (programmatic dependent
// launch), so the weight stream overlaps the previous kernel's tail and the
// prologue; then the input row is read (and normalised, or the attention
// partials merged) into shared memory and each warp reduces its tasks from
// registers: fp32 products and accumulation, a fixed butterfly, segments
// summed in order.
template <int K, int SEG, int RW, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads) gemv_stream_kernel(GemvArgs a) {
  constexpr int NT = kGemvThreads, NW = NT / 32;
  constexpr int KS = K / SEG;  // columns per task
  constexpr int C = KS / 256;  // 16-byte loads per lane per task
  static_assert(KS % 256 == 0, "segment width");
  __shared__ __align__(16) float xs[K];
  __shared__ float red[NW];
  __shared__ float part[SEG > 1 ? NW * RW : 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * a.rpc;  // rpc = tasks per CTA here (a multiple of SEG)
  const int tend = min(t0 + a.rpc, a.n * SEG);
  uint4 wv[RW][C];
  float bias[RW];
#pragma unroll
  for (int i = 0; i < RW; ++i) {
    int t = t0 + warp + NW * i;
    if (t >= tend) t = t0;  // a valid row; the result is discarded
    const int row = t / SEG, seg = t - row * SEG;
    const uint4* wr = reinterpret_cast<const uint4*>(a.w + static_cast<size_t>(row) * K + seg * KS);
#pragma unroll
    for (int c = 0; c < C; ++c) wv[i][c] = ldg_weights(wr + lane + 32 * c);
    bias[i] = a.bias[row];
  }
  griddep_launch();
  griddep_wait();
  if (a.ctl[4]) return;
  if (PRO == kProAttn) {
    attn_combine_smem<NT>(a.x, xs);
  } else {
    for (int i = threadIdx.x; i < K; i += NT) xs[i] = a.x[i];
    __syncthreads();
    if (PRO >= kProLn) layer_norm_smem<K, NT>(xs, a.g1, a.b1, red);
    if (PRO == kProLn2) layer_norm_smem<K, NT>(xs, a.g2, a.b2, red);
  }
#pragma unroll
  for (int i = 0; i < RW; ++i) {
    const int t = t0 + warp + NW * i;
    const int row = t / SEG, seg = t - row * SEG;
    float s = 0.0f;
#pragma unroll
    for (int c = 0; c < C; ++c) s += dot8(wv[i][c], xs + seg * KS + (lane + 32 * c) * 8);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0 && t < tend) {
      if (SEG == 1) {
        float v = s + bias[i];
        if (EPI == kEpiGelu) v = gelu_new(v);
        if (EPI == kEpiResid) v = a.resid[row] + v;
        a.y[row] = v;
      } else {
        part[warp + NW * i] = s;  // task index within the CTA
      }
    }
  }
  if (SEG > 1) {
    __syncthreads();
    for (int j = threadIdx.x * SEG; j < tend - t0; j += NT * SEG) {
      const int row = (t0 + j) / SEG;
      float s = 0.0f;
#pragma unroll
      for (int q = 0; q < SEG; ++q) s += part[j + q];
      float v = s + a.bias[row];
      if (EPI == kEpiGelu) v = gelu_new(v);
      if (EPI == kEpiResid) v = a.resid[row] + v;
      a.y[row] = v;
    }
  }
}

// One key range of one head of the cached single-query attention
// (cpu_attention_single_query, runtime/impl/tokenizer_tests.cpp:4034-4061,
// over the cache of runtime/impl/gpt.cpp:1060-1210). The len + 1 keys (the
// cache plus this token's, read straight from qkv) are cut into kSplits
// ranges; range r of head h writes its partial (m = max score, l = sum
// e^(s - m), acc = sum e^(s - m) v) for the combine in the next projection.
// Range 0 also appends this token's K and V at row len of the layer's cache.
__global__ void __launch_bounds__(256) gpt_attn_kernel(const float* __restrict__ qkv, float* __restrict__ kc,
                                                       float* __restrict__ vc, float* __restrict__ part,
                                                       const int* __restrict__ ctl) {
  __shared__ float s[kSplitKeys];
  __shared__ __align__(16) float q[64];
  __shared__ float red[8];
  __shared__ float acc_w[8][64];
  griddep_launch();
  griddep_wait();
  if (ctl[4]) return;
  const int r = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int len = ctl[0], n = len + 1;
  const int chunk = (n + kSplits - 1) / kSplits;
  const int j0 = r * chunk, j1 = min(n, j0 + chunk);
  const float* kcur = qkv + kW + h * 64;
  const float* vcur = qkv + 2 * kW + h * 64;
  if (r == 0) {
    const size_t cur = static_cast<size_t>(len) * kW + h * 64;
    if (tid < 64) kc[cur + tid] = kcur[tid];
    else if (tid < 128) vc[cur + tid - 64] = vcur[tid - 64];
  }
  float* out = part + (static_cast<size_t>(h) * kSplits + r) * kPart;
  if (j0 >= j1) {  // empty range (short caches)
    if (tid < kPart) out[tid] = tid == 0 ? -INFINITY : 0.0f;
    return;
  }
  if (tid < 64) q[tid] = qkv[h * 64 + tid];
  __syncthreads();
  // scores: 16 lanes per key (a float4 of the 64 dims each), 4 keys in flight per group
  const int g = tid >> 4, l = tid & 15;
  const float4 qv = reinterpret_cast<const float4*>(q)[l];
  for (int base = j0; base < j1; base += 64) {
    float4 kv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = base + g + 16 * u;
      const float* kp = j == len ? kcur : kc + static_cast<size_t>(j) * kW + h * 64;
      kv[u] = j < j1 ? *reinterpret_cast<const float4*>(kp + 4 * l) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float d = qv.x * kv[u].x;
      d = fmaf(qv.y, kv[u].y, d);
      d = fmaf(qv.z, kv[u].z, d);
      d = fmaf(qv.w, kv[u].w, d);
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      const int j = base + g + 16 * u;
      if (l == 0 && j < j1) s[j - j0] = d * 0.125f;
    }
  }
  __syncthreads();
  const int cnt = j1 - j0;
  float mx = -INFINITY;
  for (int j = tid; j < cnt; j += 256) mx = fmaxf(mx, s[j]);
  mx = block_max_all<256>(mx, red);
  float den = 0.0f;
  for (int j = tid; j < cnt; j += 256) {
    const float e = expf(s[j] - mx);
    s[j] = e;
    den += e;
  }
  den = block_sum_all<256>(den, red);  // also orders the writes of s before the reads below
  // acc: warp w takes keys w, w+8, ...; lane dims 2 lane, 2 lane + 1
  const int w = tid >> 5, lane = tid & 31;
  float2 acc = make_float2(0.f, 0.f);
  for (int base = 0; base < cnt; base += 32) {
    float2 vv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = base + w + 8 * u;
      const int jj = j0 + j;
      const float* vp = jj == len ? vcur : vc + static_cast<size_t>(jj) * kW + h * 64;
      vv[u] = j < cnt ? *reinterpret_cast<const float2*>(vp + 2 * lane) : make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = base + w + 8 * u;
      const float p = j < cnt ? s[j] : 0.0f;
      acc.x = fmaf(p, vv[u].x, acc.x);
      acc.y = fmaf(p, vv[u].y, acc.y);
    }
  }
  acc_w[w][2 * lane] = acc.x;
  acc_w[w][2 * lane + 1] = acc.y;
  __syncthreads();
  if (tid < 64) {
    float o = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) o += acc_w[i][tid];
    out[2 + tid] = o;
  } else if (tid == 64) {
    out[0] = mx;
    out[1] = den;
  }
}

// Decode input (build_gpt_greedy_current_cpu, runtime/impl/gpt.cpp:
// 1545-1554): mel_embedding[code] + mel_pos_embedding[step].
__global__ void __launch_bounds__(256) gpt_embed_kernel(const float* __restrict__ emb, const float* __restrict__ pos,
                                                        float* __restrict__ x, const int* __restrict__ ctl) {
  griddep_launch();
  griddep_wait();
  if (ctl[4]) return;
  const int i = blockIdx.x * 256 + threadIdx.x;
  const int step = ctl[2], position = ctl[6] && step > 0 ? step + 1 : step;  // ctl[6]: generate-style positions
  if (i < kW) x[i] = emb[static_cast<size_t>(ctl[3]) * kW + i] + pos[static_cast<size_t>(position) * kW + i];
}

// Prefill input: prefix row ctl[1].
__global__ void __launch_bounds__(256) gpt_prefix_row_kernel(const float* __restrict__ prefix, float* __restrict__ x,
                                                             const int* __restrict__ ctl) {
  griddep_launch();
  griddep_wait();
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i < kW) x[i] = prefix[static_cast<size_t>(ctl[1]) * kW + i];
}

__global__ void gpt_prefill_advance_kernel(int* ctl) {
  griddep_launch();
  griddep_wait();
  ctl[0] += 1;
  ctl[1] += 1;
}

// argmax_row (runtime/impl/gpt.cpp:1297-1308): the first index of the
// maximum. Records the code, makes it the next input, advances the step and
// the cache, and stops after the stop code or the last allowed step.
__global__ void __launch_bounds__(1024) gpt_argmax_kernel(const float* __restrict__ logits, int n,
                                                          uint32_t* __restrict__ codes, int* __restrict__ ctl) {
  __shared__ float bv_s[32];
  griddep_launch();
  griddep_wait();
  if (ctl[4]) return;
  __shared__ int bi_s[32];
  float bv = -INFINITY;
  int bi = INT_MAX;
  for (int i = threadIdx.x; i < n; i += 1024) {
    const float v = logits[i];
    if (bi == INT_MAX || v > bv) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    bv_s[threadIdx.x >> 5] = bv;
    bi_s[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    bv = bv_s[0];
    bi = bi_s[0];
    for (int w = 1; w < 32; ++w)
      if (bv_s[w] > bv || (bv_s[w] == bv && bi_s[w] < bi)) {
        bv = bv_s[w];
        bi = bi_s[w];
      }
    const int step = ctl[2];
    codes[step] = static_cast<uint32_t>(bi);
    ctl[3] = bi;
    ctl[2] = step + 1;
    ctl[0] += 1;
    if (bi == GptDecoder::kStop || step + 1 >= ctl[5]) ctl[4] = 1;
  }
}

// Grid of a projection: tasks (row, segment) in CTAs of 16 warps x RW tasks.
template <int K, int SEG, int RW, int PRO, int EPI>
cudaError_t launch_gemv(GemvArgs a, cudaStream_t st) {
  const int tpc = kGemvThreads / 32 * RW;
  static_assert((kGemvThreads / 32 * RW) % SEG == 0, "rows must not straddle CTAs");
  a.rpc = tpc;
  const int grid = (a.n * SEG + tpc - 1) / tpc;
  return launch_pdl(gemv_stream_kernel<K, SEG, RW, PRO, EPI>, dim3(grid), dim3(kGemvThreads), 0, st, a);
}

// Transposes a [rows][cols] f16 payload to [cols][rows] (32x32 tiles).
std::vector<uint16_t> transpose16(const uint16_t* src, size_t rows, size_t cols) {
  std::vector<uint16_t> t(rows * cols);
  for (size_t r0 = 0; r0 < rows; r0 += 32)
    for (size_t c0 = 0; c0 < cols; c0 += 32)
      for (size_t r = r0; r < std::min(rows, r0 + 32); ++r)
        for (size_t c = c0; c < std::min(cols, c0 + 32); ++c) t[c * rows + r] = src[r * cols + c];
  return t;
}

}  // namespace

double GptDecoder::weight_bytes_per_token() {
  const double per_layer = static_cast<double>(kW) * kQkv + static_cast<double>(kW) * kW + 2.0 * kW * kMlp;
  return 2.0 * (kLayers * per_layer + static_cast<double>(kVocab) * kW);
}

void GptDecoder::check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string("cuda: gpt: ") + what + ": " + cudaGetErrorString(e));
}

GptDecoder::GptDecoder(const std::string& bundle_dir, int device, bool verify_sha256) : device_(device) {
  int nd = 0;
  check(cudaGetDeviceCount(&nd), "cudaGetDeviceCount");
  if (device < 0 || device >= nd) throw std::runtime_error("device id out of range");
  check(cudaSetDevice(device), "cudaSetDevice");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10 || minor != 0) throw std::runtime_error("this build targets sm_100a (B200) only");
  Mit2Bundle b(bundle_dir, verify_sha256);

  // Device layout: every tensor at a 256-byte aligned offset of one arena.
  struct Item {
    std::string name;
    bool f16, transpose;
    size_t rows, cols, off;
  };
  std::vector<Item> items;
  size_t total = 0;
  auto add = [&](const std::string& name, bool f16, bool transpose, size_t rows, size_t cols) {
    const TensorRec& t = b.require(name);
    if (b.element_count(t) != rows * cols) throw std::runtime_error("gpt weights: " + name + " has an unexpected size");
    items.push_back({name, f16, transpose, rows, cols, total});
    total += ((rows * cols * (f16 ? 2 : 4)) + 255) & ~size_t(255);
    return items.size() - 1;
  };
  size_t idx[kLayers][12];
  for (int l = 0; l < kLayers; ++l) {
    const std::string p = "gpt.gpt.h." + std::to_string(l) + ".";
    idx[l][0] = add(p + "ln_1.weight", false, false, 1, kW);
    idx[l][1] = add(p + "ln_1.bias", false, false, 1, kW);
    idx[l][2] = add(p + "attn.c_attn.weight", true, true, kW, kQkv);  // Conv1D [in][out]
    idx[l][3] = add(p + "attn.c_attn.bias", false, false, 1, kQkv);
    idx[l][4] = add(p + "attn.c_proj.weight", true, true, kW, kW);
    idx[l][5] = add(p + "attn.c_proj.bias", false, false, 1, kW);
    idx[l][6] = add(p + "ln_2.weight", false, false, 1, kW);
    idx[l][7] = add(p + "ln_2.bias", false, false, 1, kW);
    idx[l][8] = add(p + "mlp.c_fc.weight", true, true, kW, kMlp);
    idx[l][9] = add(p + "mlp.c_fc.bias", false, false, 1, kMlp);
    idx[l][10] = add(p + "mlp.c_proj.weight", true, true, kMlp, kW);
    idx[l][11] = add(p + "mlp.c_proj.bias", false, false, 1, kW);
  }
  const size_t i_lnf_g = add("gpt.gpt.ln_f.weight", false, false, 1, kW);
  const size_t i_lnf_b = add("gpt.gpt.ln_f.bias", false, false, 1, kW);
  const size_t i_fn_g = add("gpt.final_norm.weight", false, false, 1, kW);
  const size_t i_fn_b = add("gpt.final_norm.bias", false, false, 1, kW);
  const size_t i_head = add("gpt.mel_head.weight", true, false, kVocab, kW);  // nn.Linear [out][in]
  const size_t i_bhead = add("gpt.mel_head.bias", false, false, 1, kVocab);
  const size_t i_emb = add("gpt.mel_embedding.weight", false, false, kVocab, kW);
  const size_t i_pos = add("gpt.mel_pos_embedding.emb.weight", false, false, kPositions, kW);
  check(cudaMalloc(&arena_, total), "gpt weights cudaMalloc");
  uint8_t* base = static_cast<uint8_t*>(arena_);
  for (const Item& it : items) {
    const TensorRec& t = b.require(it.name);
    if (it.f16) {
      std::vector<uint16_t> h;
      if (t.dtype == "f16") {
        size_t cnt = 0;
        const uint16_t* src = b.as_f16(it.name, &cnt);
        h = it.transpose ? transpose16(src, it.rows, it.cols) : std::vector<uint16_t>(src, src + cnt);
      } else {
        std::vector<float> f = b.as_f32(it.name);
        std::vector<uint16_t> raw(f.size());
        for (size_t i = 0; i < f.size(); ++i) raw[i] = float_to_half_bits(f[i]);
        h = it.transpose ? transpose16(raw.data(), it.rows, it.cols) : std::move(raw);
      }
      check(cudaMemcpy(base + it.off, h.data(), h.size() * 2, cudaMemcpyHostToDevice), "gpt weights upload");
    } else {
      std::vector<float> f = b.as_f32(it.name);
      check(cudaMemcpy(base + it.off, f.data(), f.size() * 4, cudaMemcpyHostToDevice), "gpt weights upload");
    }
  }
  auto F = [&](size_t i) { return reinterpret_cast<const float*>(base + items[i].off); };
  auto H = [&](size_t i) { return reinterpret_cast<const __half*>(base + items[i].off); };
  for (int l = 0; l < kLayers; ++l) {
    Layer& L = L_[l];
    L.ln1_g = F(idx[l][0]);
    L.ln1_b = F(idx[l][1]);
    L.w_attn = H(idx[l][2]);
    L.b_attn = F(idx[l][3]);
    L.w_proj = H(idx[l][4]);
    L.b_proj = F(idx[l][5]);
    L.ln2_g = F(idx[l][6]);
    L.ln2_b = F(idx[l][7]);
    L.w_fc = H(idx[l][8]);
    L.b_fc = F(idx[l][9]);
    L.w_mproj = H(idx[l][10]);
    L.b_mproj = F(idx[l][11]);
  }
  lnf_g_ = F(i_lnf_g);
  lnf_b_ = F(i_lnf_b);
  fn_g_ = F(i_fn_g);
  fn_b_ = F(i_fn_b);
  w_head_ = H(i_head);
  b_head_ = F(i_bhead);
  emb_ = F(i_emb);
  pos_ = F(i_pos);

  // State: activations, the fp32 KV caches, the prefix, control words, codes.
  size_t off = 0;
  auto carve = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  };
  const size_t o_x = carve(kW * 4), o_h = carve(kW * 4), o_qkv = carve(kQkv * 4), o_part = carve(static_cast<size_t>(kHeads) * kSplits * kPart * 4),
               o_m = carve(kMlp * 4), o_logits = carve(kVocab * 4),
               o_kc = carve(static_cast<size_t>(kLayers) * kMaxLen * kW * 4),
               o_vc = carve(static_cast<size_t>(kLayers) * kMaxLen * kW * 4),
               o_prefix = carve(static_cast<size_t>(kMaxLen) * kW * 4), o_ctl = carve(8 * 4), o_status = carve(4),
               o_codes = carve(static_cast<size_t>(kPositions) * 4);
  check(cudaDeviceGetAttribute(&sms_, cudaDevAttrMultiProcessorCount, device), "SM count");
  const size_t o_layers = carve(sizeof(GptLayerPtrs) * kLayers), o_cval = carve(static_cast<size_t>(sms_) * 4),
               o_cidx = carve(static_cast<size_t>(sms_) * 4), o_bar = carve(512), o_out = carve(16),
               o_times = carve(4 * 8), o_trace = carve((2 * static_cast<size_t>(kGptTraceCap) + static_cast<size_t>(kGptTraceStages) * sms_) * 8),
               o_hist = carve(static_cast<size_t>(kMaxLen) * 4), o_seen = carve(((kVocab + 31) / 32) * 4),
               o_rng = carve(8), o_sampled = carve(4);
  const size_t rows = static_cast<size_t>(kMaxLen);
  const size_t o_pf_h = carve(rows * kW * 4), o_pf_xn = carve(rows * kW * 4), o_pf_q = carve(rows * kW * 4),
               o_pf_attn = carve(rows * kW * 4), o_pf_m = carve(rows * kMlp * 4), o_pf_part = carve(4 * rows * kW * 4);
  check(cudaMalloc(&state_, off), "gpt state cudaMalloc");
  check(cudaMemset(state_, 0, off), "gpt state memset");
  uint8_t* s = static_cast<uint8_t*>(state_);
  x_ = reinterpret_cast<float*>(s + o_x);
  h_ = reinterpret_cast<float*>(s + o_h);
  qkv_ = reinterpret_cast<float*>(s + o_qkv);
  part_ = reinterpret_cast<float*>(s + o_part);
  m_ = reinterpret_cast<float*>(s + o_m);
  logits_ = reinterpret_cast<float*>(s + o_logits);
  kc_ = reinterpret_cast<float*>(s + o_kc);
  vc_ = reinterpret_cast<float*>(s + o_vc);
  prefix_ = reinterpret_cast<float*>(s + o_prefix);
  ctl_ = reinterpret_cast<int*>(s + o_ctl);
  status_ = reinterpret_cast<unsigned int*>(s + o_status);
  codes_ = reinterpret_cast<uint32_t*>(s + o_codes);
  layers_dev_ = reinterpret_cast<GptLayerPtrs*>(s + o_layers);
  cand_val_ = reinterpret_cast<float*>(s + o_cval);
  cand_idx_ = reinterpret_cast<int*>(s + o_cidx);
  barrier_ = reinterpret_cast<unsigned int*>(s + o_bar);
  out_ = reinterpret_cast<int*>(s + o_out);
  times_ = reinterpret_cast<unsigned long long*>(s + o_times);
  trace_ = reinterpret_cast<unsigned long long*>(s + o_trace);
  history_ = reinterpret_cast<uint32_t*>(s + o_hist);
  pf_.x = prefix_;  // the residual stream starts as the prefix rows
  pf_.h = reinterpret_cast<float*>(s + o_pf_h);
  pf_.xn = reinterpret_cast<float*>(s + o_pf_xn);
  pf_.q = reinterpret_cast<float*>(s + o_pf_q);
  pf_.attn = reinterpret_cast<float*>(s + o_pf_attn);
  pf_.m = reinterpret_cast<float*>(s + o_pf_m);
  pf_.part = reinterpret_cast<float*>(s + o_pf_part);
  pf_.kc = kc_;
  pf_.vc = vc_;
  seen_ = reinterpret_cast<unsigned int*>(s + o_seen);
  rng_ = reinterpret_cast<unsigned long long*>(s + o_rng);
  sampled_ = reinterpret_cast<int*>(s + o_sampled);
  check(cudaMemcpy(layers_dev_, L_, sizeof(GptLayerPtrs) * kLayers, cudaMemcpyHostToDevice), "gpt layer table upload");
  check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
  for (auto& e : ev_) check(cudaEventCreate(&e), "cudaEventCreate");
  const char* mode = std::getenv("ITTS_GPT_MODE");
  persistent_ = !(mode && std::string(mode) == "graph");
  if (persistent_) {
    if (sms_ < gpt_persist_min_grid()) throw std::runtime_error("gpt: too few SMs for the persistent decoder");
    check(gpt_persist_prepare(), "persistent decoder shared memory");
    check(gpt_prefill_prepare(), "prefill attention shared memory");
    const char* pm = std::getenv("ITTS_GPT_PREFILL");
    batched_prefill_ = !(pm && std::string(pm) == "rows");
  }
  build_graphs();
}

GptDecoder::~GptDecoder() {
  cudaSetDevice(device_);
  if (stream_) cudaStreamSynchronize(stream_);
  if (g_prefill_) cudaGraphExecDestroy(g_prefill_);
  if (g_decode_) cudaGraphExecDestroy(g_decode_);
  for (auto& e : ev_)
    if (e) cudaEventDestroy(e);
  if (arena_) cudaFree(arena_);
  if (state_) cudaFree(state_);
  if (stream_) cudaStreamDestroy(stream_);
}

// The 24 blocks on x_ (run_gpt_cached_block_current_cpu per layer,
// runtime/impl/gpt.cpp:1060-1210): qkv = c_attn(ln_1(x)); a = attention over
// the cache with this token appended; h = x + c_proj(a); m = gelu_new(c_fc(
// ln_2(h))); x = h + mlp.c_proj(m).
void GptDecoder::enqueue_layers() {
  for (int l = 0; l < kLayers; ++l) {
    const Layer& L = L_[l];
    float* kc = kc_ + static_cast<size_t>(l) * kMaxLen * kW;
    float* vc = vc_ + static_cast<size_t>(l) * kMaxLen * kW;
    check(launch_gemv<kW, 1, 4, kProLn, kEpiBias>(
              {x_, L.ln1_g, L.ln1_b, nullptr, nullptr, L.w_attn, L.b_attn, nullptr, qkv_, kQkv, 0, ctl_, status_}, stream_),
          "c_attn");
    check(launch_pdl(gpt_attn_kernel, dim3(kSplits, kHeads), dim3(256), 0, stream_, qkv_, kc, vc, part_, ctl_),
          "attention");
    check(launch_gemv<kW, 1, 2, kProAttn, kEpiResid>(
              {part_, nullptr, nullptr, nullptr, nullptr, L.w_proj, L.b_proj, x_, h_, kW, 0, ctl_, status_}, stream_),
          "attn.c_proj");
    check(launch_gemv<kW, 1, 4, kProLn, kEpiGelu>(
              {h_, L.ln2_g, L.ln2_b, nullptr, nullptr, L.w_fc, L.b_fc, nullptr, m_, kMlp, 0, ctl_, status_}, stream_),
          "c_fc");
    check(launch_gemv<kMlp, 2, 1, kProPlain, kEpiResid>(
              {m_, nullptr, nullptr, nullptr, nullptr, L.w_mproj, L.b_mproj, h_, x_, kW, 0, ctl_, status_}, stream_),
          "mlp.c_proj");
  }
}

void GptDecoder::build_graphs() {
  auto capture = [&](auto&& body, cudaGraphExec_t* exec, int* kernels) {
    cudaGraph_t graph = nullptr;
    check(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "gpt begin capture");
    try {
      body();
    } catch (...) {
      cudaStreamEndCapture(stream_, &graph);
      if (graph) cudaGraphDestroy(graph);
      throw;
    }
    check(cudaStreamEndCapture(stream_, &graph), "gpt end capture");
    if (kernels) {
      size_t nn = 0;
      cudaGraphGetNodes(graph, nullptr, &nn);
      std::vector<cudaGraphNode_t> nodes(nn);
      if (nn) cudaGraphGetNodes(graph, nodes.data(), &nn);
      *kernels = 0;
      for (auto nd : nodes) {
        cudaGraphNodeType ty;
        if (cudaGraphNodeGetType(nd, &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++*kernels;
      }
    }
    const cudaError_t e = cudaGraphInstantiate(exec, graph, 0);
    cudaGraphDestroy(graph);
    check(e, "gpt graph instantiate");
  };
  capture(
      [&] {
        check(launch_pdl(gpt_prefix_row_kernel, dim3(kW / 256), dim3(256), 0, stream_, prefix_, x_, ctl_),
              "prefix row");
        enqueue_layers();
        check(launch_pdl(gpt_prefill_advance_kernel, dim3(1), dim3(1), 0, stream_, ctl_), "prefill advance");
      },
      &g_prefill_, &prefill_kernels_);
  capture(
      [&] {
        check(launch_pdl(gpt_embed_kernel, dim3(kW / 256), dim3(256), 0, stream_, emb_, pos_, x_, ctl_), "embed");
        enqueue_layers();
        // ln_f then final_norm (runtime/impl/gpt.cpp:1901-1902), the mel head, argmax
        check(launch_gemv<kW, 1, 4, kProLn2, kEpiBias>(
                  {x_, lnf_g_, lnf_b_, fn_g_, fn_b_, w_head_, b_head_, nullptr, logits_, kVocab, 0, ctl_, status_}, stream_),
              "mel head");
        check(launch_pdl(gpt_argmax_kernel, dim3(1), dim3(1024), 0, stream_, logits_, kVocab, codes_, ctl_), "argmax");
      },
      &g_decode_, &decode_kernels_);
}

int GptDecoder::generate(const float* prefix, int P, int max_steps, bool hf_positions, uint32_t* codes,
                         float* last_logits) {
  sample_ = false;
  return generate_common(prefix, P, max_steps, hf_positions, codes, last_logits);
}

int GptDecoder::generate_sampled(const float* prefix, int P, int max_steps, bool hf_positions, const Sampling& sampling,
                                 const uint32_t* history, int n_history, uint32_t* codes, float* last_logits) {
  if (!persistent_) throw std::invalid_argument("gpt: sampled decode needs the persistent decoder");
  if (!(sampling.temperature > 0.0f)) throw std::invalid_argument("gpt: sampling temperature must be positive");
  if (sampling.top_k < 1 || sampling.top_k > kGptSampleMaxFinite)
    throw std::invalid_argument("gpt: sampling top_k must be within 1..2048");
  if (!(sampling.top_p > 0.0f && sampling.top_p <= 1.0f)) throw std::invalid_argument("gpt: top_p must be in (0, 1]");
  if (!(sampling.repetition_penalty > 0.0f)) throw std::invalid_argument("gpt: repetition penalty must be positive");
  if (n_history < 0 || n_history > kMaxLen || (n_history > 0 && !history))
    throw std::invalid_argument("gpt: the repetition history must hold 0..4096 tokens");
  check(cudaSetDevice(device_), "cudaSetDevice");
  if (n_history > 0)
    check(cudaMemcpyAsync(history_, history, static_cast<size_t>(n_history) * 4, cudaMemcpyHostToDevice, stream_),
          "gpt history upload");
  sample_ = true;
  sampling_ = sampling;
  n_history_ = n_history;
  return generate_common(prefix, P, max_steps, hf_positions, codes, last_logits);
}

int GptDecoder::generate_common(const float* prefix, int P, int max_steps, bool hf_positions, uint32_t* codes,
                                float* last_logits) {
  const int max_allowed = hf_positions ? kPositions - 1 : kPositions;
  if (P < 0 || max_steps < 1 || max_steps > max_allowed || P + max_steps > kMaxLen)
    throw std::invalid_argument("gpt: need 0 <= P, 1 <= max_steps <= 1818 (1817 with generate-style positions) and "
                                "P + max_steps <= 4096");
  hf_ = hf_positions;
  if (P > 0 && !prefix) throw std::invalid_argument("gpt: prefix must be non-null when P > 0");
  if (!codes) throw std::invalid_argument("gpt: codes must be non-null");
  check(cudaSetDevice(device_), "cudaSetDevice");
  if (P > 0)
    check(cudaMemcpyAsync(prefix_, prefix, static_cast<size_t>(P) * kW * 4, cudaMemcpyHostToDevice, stream_),
          "gpt prefix upload");
  const int n = persistent_ ? generate_persistent(P, max_steps) : generate_graphs(P, max_steps);
  unsigned int st = 0;
  check(cudaMemcpy(&st, status_, sizeof(st), cudaMemcpyDeviceToHost), "gpt status read");
  if (st != 0) {
    check(cudaMemset(status_, 0, sizeof(st)), "gpt status clear");
    if (st == 43) throw std::runtime_error("gpt: sampling: more than 2048 scores tie at the top-k pivot");
    throw std::runtime_error("timeout: a GPT kernel abandoned a bounded wait (device status " + std::to_string(st) + ")");
  }
  if (n < 1 || n > max_steps) throw std::runtime_error("cuda: gpt: decoder produced an invalid step count");
  check(cudaMemcpyAsync(codes, codes_, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost, stream_), "codes read");
  if (last_logits)
    check(cudaMemcpyAsync(last_logits, logits_, kVocab * 4, cudaMemcpyDeviceToHost, stream_), "logits read");
  check(cudaStreamSynchronize(stream_), "gpt sync");
  steps_ = n;
  return n;
}

// One cooperative launch for the whole call; the prefill / decode split of
// the device time comes from the kernel's global-timer stamps.
int GptDecoder::generate_persistent(int P, int max_steps) {
  GptPersistParams p;
  p.layers = layers_dev_;
  p.lnf_g = lnf_g_;
  p.lnf_b = lnf_b_;
  p.fn_g = fn_g_;
  p.fn_b = fn_b_;
  p.b_head = b_head_;
  p.w_head = w_head_;
  p.emb = emb_;
  p.pos = pos_;
  p.prefix = prefix_;
  p.x = x_;
  p.h = h_;
  p.qkv = qkv_;
  p.m = m_;
  p.logits = logits_;
  p.kc = kc_;
  p.vc = vc_;
  p.part = part_;
  p.cand_val = cand_val_;
  p.cand_idx = cand_idx_;
  p.codes = codes_;
  p.out = out_;
  p.barrier = barrier_;
  p.status = status_;
  p.times = times_;
  p.P = P;
  p.max_steps = max_steps;
  p.hf_positions = hf_ ? 1 : 0;
  p.trace = tracing_ ? trace_ : nullptr;
  p.sample = sample_ ? 1 : 0;
  p.temperature = sampling_.temperature;
  p.top_k = sampling_.top_k;
  p.top_p = sampling_.top_p;
  p.repetition_penalty = sampling_.repetition_penalty;
  p.seed = sampling_.seed;
  p.history = history_;
  p.n_history = n_history_;
  p.seen = seen_;
  p.rng = rng_;
  p.sampled = sampled_;
  if (tracing_)
    check(cudaMemsetAsync(trace_, 0,
                          (2 * static_cast<size_t>(kGptTraceCap) + static_cast<size_t>(kGptTraceStages) * sms_) * 8,
                          stream_),
          "trace reset");
  check(cudaMemsetAsync(barrier_, 0, 512, stream_), "grid barrier reset");
  check(cudaMemsetAsync(out_, 0, 16, stream_), "gpt output reset");
  const bool batched = batched_prefill_ && P > 0;
  p.len0 = 0;
  check(cudaEventRecord(ev_[0], stream_), "event");
  if (batched) {  // all prefix rows per layer at once; the decode starts from a cache of P rows
    check(gpt_prefill_enqueue(L_, pf_, P, stream_), "batched prefill launch");
    p.P = 0;
    p.len0 = P;
  }
  check(cudaEventRecord(ev_[1], stream_), "event");
  check(gpt_persist_launch(p, sms_, stream_), "persistent decoder launch");
  check(cudaEventRecord(ev_[2], stream_), "event");
  int n = 0;
  unsigned long long t[3] = {0, 0, 0};
  check(cudaMemcpyAsync(&n, out_, sizeof(int), cudaMemcpyDeviceToHost, stream_), "gpt step count read");
  check(cudaMemcpyAsync(t, times_, sizeof(t), cudaMemcpyDeviceToHost, stream_), "gpt timer read");
  check(cudaStreamSynchronize(stream_), "gpt sync");
  float total = 0.0f;
  check(cudaEventElapsedTime(&total, ev_[0], ev_[2]), "event time");
  if (batched) {
    check(cudaEventElapsedTime(&prefill_ms_, ev_[0], ev_[1]), "event time");
    decode_ms_ = total - prefill_ms_;
    launches_ = 1 + gpt_prefill_kernels_per_call();
  } else {
    const double pre = t[1] >= t[0] ? (t[1] - t[0]) * 1e-6 : 0.0;
    prefill_ms_ = static_cast<float>(pre);
    decode_ms_ = total - prefill_ms_;
    launches_ = 1;
  }
  return n;
}

// The per-kernel path: a graph per prefill row, a graph per decode step,
// the stop flag read once per chunk of steps.
int GptDecoder::generate_graphs(int P, int max_steps) {
  static_assert(kStart == 8192, "start code");
  const int ctl0[8] = {0, 0, 0, kStart, 0, max_steps, hf_ ? 1 : 0, 0};
  check(cudaMemcpyAsync(ctl_, ctl0, sizeof(ctl0), cudaMemcpyHostToDevice, stream_), "gpt control upload");
  check(cudaEventRecord(ev_[0], stream_), "event");
  for (int r = 0; r < P; ++r) check(cudaGraphLaunch(g_prefill_, stream_), "prefill graph launch");
  check(cudaEventRecord(ev_[1], stream_), "event");
  int launched = 0, stopped = 0;
  while (!stopped && launched < max_steps) {
    const int chunk = std::min(kDecodeChunk, max_steps - launched);
    for (int i = 0; i < chunk; ++i) check(cudaGraphLaunch(g_decode_, stream_), "decode graph launch");
    launched += chunk;
    check(cudaMemcpyAsync(&stopped, ctl_ + 4, sizeof(int), cudaMemcpyDeviceToHost, stream_), "stop flag read");
    check(cudaStreamSynchronize(stream_), "decode sync");
  }
  check(cudaEventRecord(ev_[2], stream_), "event");
  int ctl[8];
  check(cudaMemcpyAsync(ctl, ctl_, sizeof(ctl), cudaMemcpyDeviceToHost, stream_), "gpt control read");
  check(cudaStreamSynchronize(stream_), "gpt sync");
  check(cudaEventElapsedTime(&prefill_ms_, ev_[0], ev_[1]), "event time");
  check(cudaEventElapsedTime(&decode_ms_, ev_[1], ev_[2]), "event time");
  launches_ = static_cast<long long>(P) * prefill_kernels_ + static_cast<long long>(launched) * decode_kernels_;
  return ctl[2];
}

int GptDecoder::stage_trace(double* us, int cap) {
  if (!tracing_ || !persistent_) return 0;
  const size_t stamps = static_cast<size_t>(kGptTraceCap) + static_cast<size_t>(kGptTraceStages) * sms_;
  std::vector<unsigned long long> t(stamps + kGptTraceCap);
  check(cudaMemcpy(t.data(), trace_, t.size() * 8, cudaMemcpyDeviceToHost), "trace read");
  int n = 0;
  for (size_t i = 0; i < stamps && n < cap; ++i, ++n)
    us[n] = t[i] == 0 || t[0] == 0 ? -1.0 : (static_cast<double>(t[i]) - static_cast<double>(t[0])) * 1e-3;
  for (size_t i = stamps; i < t.size() && n < cap; ++i, ++n) us[n] = static_cast<double>(t[i]) * 1e-3;  // durations
  return n;
}

}  // namespace itts
