// GPT mel-code decoder: weights, the GEMV / attention / argmax kernels and the
// per-token graphs (see gpt.hpp).
#include "gpt.hpp"

#include <algorithm>
#include <cfloat>
#include <climits>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "bundle.hpp"

namespace itts {

namespace {

constexpr int kW = GptDecoder::kW;
constexpr int kMaxLen = GptDecoder::kMaxLen;
constexpr int kDecodeChunk = 8;  // decode steps per host check of the stop flag

enum { kProPlain = 0, kProLn = 1, kProLn2 = 2 };
enum { kEpiBias = 0, kEpiGelu = 1, kEpiResid = 2 };

struct GemvArgs {
  const float* x;  // [K] input row
  const float *g1, *b1, *g2, *b2;  // LayerNorm(s) of the prologue
  const __half* w;     // [N][K] f16
  const float* bias;   // [N]
  const float* resid;  // [N] (kEpiResid)
  float* y;            // [N]
  int n;
  const int* stopped;  // nonzero: the decode has ended, do nothing
};

// Sum of one value per thread over a 256-thread block, returned to every
// thread (fixed reduction tree: deterministic).
__device__ __forceinline__ float block_sum_all(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) t += red[w];
  __syncthreads();
  return t;
}

__device__ __forceinline__ float block_max_all(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) t = fmaxf(t, red[w]);
  __syncthreads();
  return t;
}

// cpu_layernorm (runtime/impl/tokenizer_tests.cpp:2992-3010) on the row held
// in shared memory: mean, biased variance, (x - mean) * (1 / sqrt(var + 1e-5))
// * gamma + beta.
template <int K>
__device__ __forceinline__ void layer_norm_smem(float* xs, const float* __restrict__ g, const float* __restrict__ b,
                                                float* red) {
  float s = 0.0f;
  for (int i = threadIdx.x; i < K; i += 256) s += xs[i];
  const float mean = block_sum_all(s, red) / static_cast<float>(K);
  float v = 0.0f;
  for (int i = threadIdx.x; i < K; i += 256) {
    const float d = xs[i] - mean;
    v += d * d;
  }
  const float var = block_sum_all(v, red) / static_cast<float>(K);
  const float inv = 1.0f / sqrtf(var + 1e-5f);
  for (int i = threadIdx.x; i < K; i += 256) xs[i] = (xs[i] - mean) * inv * g[i] + b[i];
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

// Streaming 16-byte load (evict-first). Volatile so that the compiler keeps
// every load of a row batch ahead of the first multiply.
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.cs.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
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

// y[n] = epilogue(W[n,:] . prologue(x) + bias[n]) for the R rows of each of
// the block's 8 warps. A warp streams its rows' f16 weights in 16-byte chunks
// (lane l takes chunks l, l+32, ...: 512 contiguous bytes per warp load),
// every load of the rows issued before the first multiply; fp32 products,
// fp32 accumulation, a fixed butterfly across the warp.
template <int K, int R, int PRO, int EPI>
__global__ void __launch_bounds__(256) gemv_kernel(GemvArgs a) {
  if (*a.stopped) return;
  __shared__ __align__(16) float xs[K];
  __shared__ float red[8];
  for (int i = threadIdx.x; i < K; i += 256) xs[i] = a.x[i];
  __syncthreads();
  if (PRO >= kProLn) layer_norm_smem<K>(xs, a.g1, a.b1, red);
  if (PRO == kProLn2) layer_norm_smem<K>(xs, a.g2, a.b2, red);
  constexpr int C = K / 256;  // 16-byte chunks per lane per row
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * 8 + warp) * R;
  uint4 wv[R][C];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int n = row0 + r;
    const uint4* wr = reinterpret_cast<const uint4*>(a.w + static_cast<size_t>(n < a.n ? n : 0) * K);
#pragma unroll
    for (int c = 0; c < C; ++c) wv[r][c] = ld_stream(wr + lane + 32 * c);
  }
  asm volatile("" ::: "memory");  // the shared-memory reads of x stay behind the weight loads
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float s = 0.0f;
#pragma unroll
    for (int c = 0; c < C; ++c) s += dot8(wv[r][c], xs + (lane + 32 * c) * 8);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    acc[r] = s;
  }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int n = row0 + r;
      if (n >= a.n) break;
      float v = acc[r] + a.bias[n];
      if (EPI == kEpiGelu) v = gelu_new(v);
      if (EPI == kEpiResid) v = a.resid[n] + v;
      a.y[n] = v;
    }
  }
}

// One head of the cached single-query attention
// (cpu_attention_single_query, runtime/impl/tokenizer_tests.cpp:4034-4061,
// over the cache of runtime/impl/gpt.cpp:1060-1210): appends this token's K
// and V at row len of the layer's cache, then scores = q . k * (1/8) over the
// len + 1 keys, p = exp(s - max) / sum, out = sum_j p_j v_j.
__global__ void __launch_bounds__(256) gpt_attn_kernel(const float* __restrict__ qkv, float* __restrict__ kc,
                                                       float* __restrict__ vc, float* __restrict__ out,
                                                       const int* __restrict__ ctl) {
  if (ctl[4]) return;
  extern __shared__ float s[];  // [len + 1] scores, then probabilities
  __shared__ __align__(16) float q[64];
  __shared__ float red[8];
  __shared__ float part[8][64];
  const int h = blockIdx.x, tid = threadIdx.x;
  const int len = ctl[0], n = len + 1;
  const size_t cur = static_cast<size_t>(len) * kW + h * 64;
  if (tid < 64) {
    q[tid] = qkv[h * 64 + tid];
    kc[cur + tid] = qkv[kW + h * 64 + tid];
  } else if (tid < 128) {
    vc[cur + tid - 64] = qkv[2 * kW + h * 64 + tid - 64];
  }
  __syncthreads();
  // scores: 16 lanes per key (a float4 of the 64 dims each), 4 keys in flight
  const int g = tid >> 4, l = tid & 15;
  const float4 qv = reinterpret_cast<const float4*>(q)[l];
  const float* kh = kc + h * 64 + 4 * l;
  for (int base = 0; base < n; base += 64) {
    float4 kv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = base + g + 16 * u;
      kv[u] = j < n ? *reinterpret_cast<const float4*>(kh + static_cast<size_t>(j) * kW) : make_float4(0.f, 0.f, 0.f, 0.f);
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
      if (l == 0 && j < n) s[j] = d * 0.125f;
    }
  }
  __syncthreads();
  float mx = -FLT_MAX;
  for (int j = tid; j < n; j += 256) mx = fmaxf(mx, s[j]);
  mx = block_max_all(mx, red);
  float den = 0.0f;
  for (int j = tid; j < n; j += 256) {
    const float e = expf(s[j] - mx);
    s[j] = e;
    den += e;
  }
  den = block_sum_all(den, red);
  for (int j = tid; j < n; j += 256) s[j] = s[j] / den;
  __syncthreads();
  // out: warp w takes keys w, w+8, ...; lane l dims 2l, 2l+1
  const int w = tid >> 5, lane = tid & 31;
  const float* vh = vc + h * 64 + 2 * lane;
  float2 acc = make_float2(0.f, 0.f);
  for (int base = 0; base < n; base += 32) {
    float2 vv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = base + w + 8 * u;
      vv[u] = j < n ? *reinterpret_cast<const float2*>(vh + static_cast<size_t>(j) * kW) : make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = base + w + 8 * u;
      const float p = j < n ? s[j] : 0.0f;
      acc.x = fmaf(p, vv[u].x, acc.x);
      acc.y = fmaf(p, vv[u].y, acc.y);
    }
  }
  part[w][2 * lane] = acc.x;
  part[w][2 * lane + 1] = acc.y;
  __syncthreads();
  if (tid < 64) {
    float o = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) o += part[i][tid];
    out[h * 64 + tid] = o;
  }
}

// Decode input (build_gpt_greedy_current_cpu, runtime/impl/gpt.cpp:
// 1545-1554): mel_embedding[code] + mel_pos_embedding[step].
__global__ void __launch_bounds__(256) gpt_embed_kernel(const float* __restrict__ emb, const float* __restrict__ pos,
                                                        float* __restrict__ x, const int* __restrict__ ctl) {
  if (ctl[4]) return;
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i < kW) x[i] = emb[static_cast<size_t>(ctl[3]) * kW + i] + pos[static_cast<size_t>(ctl[2]) * kW + i];
}

// Prefill input: prefix row ctl[1].
__global__ void __launch_bounds__(256) gpt_prefix_row_kernel(const float* __restrict__ prefix, float* __restrict__ x,
                                                             const int* __restrict__ ctl) {
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i < kW) x[i] = prefix[static_cast<size_t>(ctl[1]) * kW + i];
}

__global__ void gpt_prefill_advance_kernel(int* ctl) {
  ctl[0] += 1;
  ctl[1] += 1;
}

// argmax_row (runtime/impl/gpt.cpp:1297-1308): the first index of the
// maximum. Records the code, makes it the next input, advances the step and
// the cache, and stops after the stop code or the last allowed step.
__global__ void __launch_bounds__(1024) gpt_argmax_kernel(const float* __restrict__ logits, int n,
                                                          uint32_t* __restrict__ codes, int* __restrict__ ctl) {
  if (ctl[4]) return;
  __shared__ float bv_s[32];
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

template <int K, int R, int PRO, int EPI>
void launch_gemv(const GemvArgs& a, cudaStream_t st) {
  const int rows_per_block = 8 * R;
  gemv_kernel<K, R, PRO, EPI><<<(a.n + rows_per_block - 1) / rows_per_block, 256, 0, st>>>(a);
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
  const size_t o_x = carve(kW * 4), o_h = carve(kW * 4), o_qkv = carve(kQkv * 4), o_attn = carve(kW * 4),
               o_m = carve(kMlp * 4), o_logits = carve(kVocab * 4),
               o_kc = carve(static_cast<size_t>(kLayers) * kMaxLen * kW * 4),
               o_vc = carve(static_cast<size_t>(kLayers) * kMaxLen * kW * 4),
               o_prefix = carve(static_cast<size_t>(kMaxLen) * kW * 4), o_ctl = carve(8 * 4),
               o_codes = carve(static_cast<size_t>(kPositions) * 4);
  check(cudaMalloc(&state_, off), "gpt state cudaMalloc");
  check(cudaMemset(state_, 0, off), "gpt state memset");
  uint8_t* s = static_cast<uint8_t*>(state_);
  x_ = reinterpret_cast<float*>(s + o_x);
  h_ = reinterpret_cast<float*>(s + o_h);
  qkv_ = reinterpret_cast<float*>(s + o_qkv);
  attn_ = reinterpret_cast<float*>(s + o_attn);
  m_ = reinterpret_cast<float*>(s + o_m);
  logits_ = reinterpret_cast<float*>(s + o_logits);
  kc_ = reinterpret_cast<float*>(s + o_kc);
  vc_ = reinterpret_cast<float*>(s + o_vc);
  prefix_ = reinterpret_cast<float*>(s + o_prefix);
  ctl_ = reinterpret_cast<int*>(s + o_ctl);
  codes_ = reinterpret_cast<uint32_t*>(s + o_codes);
  check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
  for (auto& e : ev_) check(cudaEventCreate(&e), "cudaEventCreate");
  check(cudaFuncSetAttribute(gpt_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxLen * 4),
        "attention shared memory");
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
  const int* stopped = ctl_ + 4;
  for (int l = 0; l < kLayers; ++l) {
    const Layer& L = L_[l];
    float* kc = kc_ + static_cast<size_t>(l) * kMaxLen * kW;
    float* vc = vc_ + static_cast<size_t>(l) * kMaxLen * kW;
    launch_gemv<kW, 2, kProLn, kEpiBias>({x_, L.ln1_g, L.ln1_b, nullptr, nullptr, L.w_attn, L.b_attn, nullptr, qkv_, kQkv, stopped},
                                         stream_);
    gpt_attn_kernel<<<kHeads, 256, kMaxLen * 4, stream_>>>(qkv_, kc, vc, attn_, ctl_);
    launch_gemv<kW, 1, kProPlain, kEpiResid>({attn_, nullptr, nullptr, nullptr, nullptr, L.w_proj, L.b_proj, x_, h_, kW, stopped},
                                             stream_);
    launch_gemv<kW, 2, kProLn, kEpiGelu>({h_, L.ln2_g, L.ln2_b, nullptr, nullptr, L.w_fc, L.b_fc, nullptr, m_, kMlp, stopped},
                                         stream_);
    launch_gemv<kMlp, 1, kProPlain, kEpiResid>({m_, nullptr, nullptr, nullptr, nullptr, L.w_mproj, L.b_mproj, h_, x_, kW, stopped},
                                               stream_);
  }
  check(cudaGetLastError(), "layer launches");
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
        gpt_prefix_row_kernel<<<kW / 256, 256, 0, stream_>>>(prefix_, x_, ctl_);
        enqueue_layers();
        gpt_prefill_advance_kernel<<<1, 1, 0, stream_>>>(ctl_);
        check(cudaGetLastError(), "prefill launches");
      },
      &g_prefill_, nullptr);
  capture(
      [&] {
        gpt_embed_kernel<<<kW / 256, 256, 0, stream_>>>(emb_, pos_, x_, ctl_);
        enqueue_layers();
        // ln_f then final_norm (runtime/impl/gpt.cpp:1901-1902), the mel head, argmax
        launch_gemv<kW, 2, kProLn2, kEpiBias>(
            {x_, lnf_g_, lnf_b_, fn_g_, fn_b_, w_head_, b_head_, nullptr, logits_, kVocab, ctl_ + 4}, stream_);
        gpt_argmax_kernel<<<1, 1024, 0, stream_>>>(logits_, kVocab, codes_, ctl_);
        check(cudaGetLastError(), "decode launches");
      },
      &g_decode_, &decode_kernels_);
}

int GptDecoder::generate(const float* prefix, int P, int max_steps, uint32_t* codes, float* last_logits) {
  if (P < 0 || max_steps < 1 || max_steps > kPositions || P + max_steps > kMaxLen)
    throw std::invalid_argument("gpt: need 0 <= P, 1 <= max_steps <= 1818 and P + max_steps <= 4096");
  if (P > 0 && !prefix) throw std::invalid_argument("gpt: prefix must be non-null when P > 0");
  if (!codes) throw std::invalid_argument("gpt: codes must be non-null");
  check(cudaSetDevice(device_), "cudaSetDevice");
  static_assert(kStart == 8192, "start code");
  const int ctl0[8] = {0, 0, 0, kStart, 0, max_steps, 0, 0};
  check(cudaMemcpyAsync(ctl_, ctl0, sizeof(ctl0), cudaMemcpyHostToDevice, stream_), "gpt control upload");
  if (P > 0)
    check(cudaMemcpyAsync(prefix_, prefix, static_cast<size_t>(P) * kW * 4, cudaMemcpyHostToDevice, stream_),
          "gpt prefix upload");
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
  const int n = ctl[2];
  if (n < 1 || n > max_steps) throw std::runtime_error("cuda: gpt: decoder produced an invalid step count");
  check(cudaMemcpyAsync(codes, codes_, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost, stream_), "codes read");
  if (last_logits)
    check(cudaMemcpyAsync(last_logits, logits_, kVocab * 4, cudaMemcpyDeviceToHost, stream_), "logits read");
  check(cudaStreamSynchronize(stream_), "gpt sync");
  check(cudaEventElapsedTime(&prefill_ms_, ev_[0], ev_[1]), "event time");
  check(cudaEventElapsedTime(&decode_ms_, ev_[1], ev_[2]), "event time");
  steps_ = n;
  return n;
}

}  // namespace itts
