// Batched GPT prefill: the P prefix rows go through each GPT-2 block together
// (run_gpt_kv_prefill_cpu, runtime/impl/gpt.cpp:1792-1806, the causal
// full-sequence pass of run_gpt_transformer_block_cpu_layer, :658-711), in
// fp32 on the CUDA cores so that the KV cache it leaves behind matches the
// one-token-at-a-time pass up to summation order. Per layer:
//   xn = ln_1(x);  [q | K | V] = xn W_attn^T + b  (K, V straight into the cache)
//   a = causal attention;  h = x + a W_proj^T + b
//   xn = ln_2(h);  m = gelu_new(xn W_fc^T + b);  x = h + m W_mproj^T + b
// The projections are tiled fp32 GEMMs (64 x 64 output tiles, 32-deep k
// steps with the next step's loads in registers, f16 weights widened in
// shared memory); the narrow ones split K over 4 CTAs and sum the partials
// in order in a separate epilogue kernel (deterministic).
#include "gpt_prefill.cuh"

#include <cuda_fp16.h>

namespace itts {

namespace {

constexpr int kW = 1280, kQkv = 3840, kMlp = 5120, kLayers = 24, kMaxLen = 4096, kHeads = 20;
constexpr int kBM = 64, kBN = 64, kBK = 32;
constexpr int kSplitNarrow = 4;  // K splits of the 1280-row projections

enum { kEpiStore = 0, kEpiQkv = 1, kEpiGelu = 2, kEpiResid = 3, kEpiPartial = 4 };

__device__ __forceinline__ float gelu_new(float x) {
  if (x > 10.0f) return x;
  if (x < -10.0f) return 0.0f;
  const float c = 0.7978845608028654f;
  return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
}

struct RowsGemm {
  const float* x;     // [M][K]
  const __half* w;    // [N][K]
  const float* bias;  // [N]
  const float* resid; // [M][N] (kEpiResid)
  float* y;           // [M][N], or [split][M][N] partials (kEpiPartial)
  float *q, *kc, *vc; // kEpiQkv targets ([M][1280] each; the caches with row stride 1280)
  int M, N, K, kchunk;
};

// One 64 x 64 output tile (4 x 4 per thread) over K range [z * kchunk, (z + 1) * kchunk).
template <int EPI>
__global__ void __launch_bounds__(256) rows_gemm_kernel(RowsGemm g) {
  __shared__ __align__(16) float xs[kBK][kBM];
  __shared__ __align__(16) float ws[kBK][kBN];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
  const int kb = blockIdx.z * g.kchunk, ke = kb + g.kchunk;
  // loaders: x tile 64 x 32 (two float4 per thread: rows xr and xr + 32),
  // w tile 64 x 32 halves (a uint4 per thread)
  const int xr = tid >> 3, xc = (tid & 7) * 4;
  const int wr = tid >> 2, wc = (tid & 3) * 8;
  const bool xrow0 = m0 + xr < g.M, xrow1 = m0 + xr + 32 < g.M;
  const float* xp0 = g.x + static_cast<size_t>(xrow0 ? m0 + xr : 0) * g.K + xc;
  const float* xp1 = g.x + static_cast<size_t>(xrow1 ? m0 + xr + 32 : 0) * g.K + xc;
  const __half* wp = g.w + static_cast<size_t>(n0 + wr) * g.K + wc;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 xa = xrow0 ? *reinterpret_cast<const float4*>(xp0 + kb) : z4;
  float4 xb = xrow1 ? *reinterpret_cast<const float4*>(xp1 + kb) : z4;
  uint4 wa = *reinterpret_cast<const uint4*>(wp + kb);
  float acc[4][4] = {};
  for (int k0 = kb; k0 < ke; k0 += kBK) {
    __syncthreads();
    xs[xc + 0][xr] = xa.x;
    xs[xc + 1][xr] = xa.y;
    xs[xc + 2][xr] = xa.z;
    xs[xc + 3][xr] = xa.w;
    xs[xc + 0][xr + 32] = xb.x;
    xs[xc + 1][xr + 32] = xb.y;
    xs[xc + 2][xr + 32] = xb.z;
    xs[xc + 3][xr + 32] = xb.w;
    {
      const __half2* h2 = reinterpret_cast<const __half2*>(&wa);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h2[i]);
        ws[wc + 2 * i][wr] = f.x;
        ws[wc + 2 * i + 1][wr] = f.y;
      }
    }
    __syncthreads();
    if (k0 + kBK < ke) {  // the next k step's loads overlap this step's FMAs
      xa = xrow0 ? *reinterpret_cast<const float4*>(xp0 + k0 + kBK) : z4;
      xb = xrow1 ? *reinterpret_cast<const float4*>(xp1 + k0 + kBK) : z4;
      wa = *reinterpret_cast<const uint4*>(wp + k0 + kBK);
    }
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&xs[kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&ws[kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= g.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (EPI == kEpiPartial) {
        g.y[(static_cast<size_t>(blockIdx.z) * g.M + m) * g.N + n] = acc[i][j];
        continue;
      }
      const float v = acc[i][j] + g.bias[n];
      if (EPI == kEpiStore) g.y[static_cast<size_t>(m) * g.N + n] = v;
      if (EPI == kEpiGelu) g.y[static_cast<size_t>(m) * g.N + n] = gelu_new(v);
      if (EPI == kEpiResid) g.y[static_cast<size_t>(m) * g.N + n] = g.resid[static_cast<size_t>(m) * g.N + n] + v;
      if (EPI == kEpiQkv) {
        if (n < kW) g.q[static_cast<size_t>(m) * kW + n] = v;
        else if (n < 2 * kW) g.kc[static_cast<size_t>(m) * kW + n - kW] = v;
        else g.vc[static_cast<size_t>(m) * kW + n - 2 * kW] = v;
      }
    }
  }
}

// y = resid + bias + sum of the K-split partials (in split order).
__global__ void __launch_bounds__(256) rows_reduce_kernel(const float* __restrict__ part, int splits, int M, int N,
                                                          const float* __restrict__ bias,
                                                          const float* __restrict__ resid, float* __restrict__ y) {
  const size_t total = static_cast<size_t>(M) * N;
  for (size_t i = static_cast<size_t>(blockIdx.x) * 256 + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * 256) {
    float s = part[i];
    for (int z = 1; z < splits; ++z) s += part[static_cast<size_t>(z) * total + i];
    const int n = static_cast<int>(i % N);
    y[i] = resid[i] + (s + bias[n]);
  }
}

// cpu_layernorm (runtime/impl/tokenizer_tests.cpp:2992-3010) per row.
__global__ void __launch_bounds__(256) rows_layernorm_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                                             const float* __restrict__ b, float* __restrict__ y) {
  __shared__ float red[8];
  const float* row = x + static_cast<size_t>(blockIdx.x) * kW;
  float v[5];
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    v[k] = row[threadIdx.x + 256 * k];
    s += v[k];
  }
  auto block_sum = [&](float t) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = t;
    __syncthreads();
    float r = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) r += red[w];
    __syncthreads();
    return r;
  };
  const float mean = block_sum(s) / static_cast<float>(kW);
  float q = 0.0f;
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    const float d = v[k] - mean;
    q += d * d;
  }
  const float var = block_sum(q) / static_cast<float>(kW);
  const float inv = 1.0f / sqrtf(var + 1e-5f);
  float* out = y + static_cast<size_t>(blockIdx.x) * kW;
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    const int i = threadIdx.x + 256 * k;
    out[i] = (v[k] - mean) * inv * g[i] + b[i];
  }
}

// Causal attention of the prefix rows (cpu_attention_single_head_causal,
// runtime/impl/tokenizer_tests.cpp:4003-4032): row r of head h attends to
// keys 0..r: scores q.k / 8, p = e^(s - max) / sum, out = sum p v. One warp
// per (row, head): a key per lane for the scores, two dims per lane for the
// values.
__global__ void __launch_bounds__(256) rows_attention_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                                             const float* __restrict__ vc, float* __restrict__ out,
                                                             int M) {
  extern __shared__ float sc_all[];  // [8][M] scores, then [8][64] queries
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, h = blockIdx.x;
  const int r = blockIdx.y * 8 + warp;
  if (r >= M) return;  // whole warp; no block-wide barrier below
  float* sc = sc_all + static_cast<size_t>(warp) * M;
  float* qs = sc_all + static_cast<size_t>(8) * M + warp * 64;
  qs[2 * lane] = q[static_cast<size_t>(r) * kW + h * 64 + 2 * lane];
  qs[2 * lane + 1] = q[static_cast<size_t>(r) * kW + h * 64 + 2 * lane + 1];
  __syncwarp();
  float mx = -INFINITY;
  for (int j = lane; j <= r; j += 32) {
    const float4* kp = reinterpret_cast<const float4*>(kc + static_cast<size_t>(j) * kW + h * 64);
    float d = 0.0f;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const float4 kv = kp[c];
      d = fmaf(qs[4 * c], kv.x, d);
      d = fmaf(qs[4 * c + 1], kv.y, d);
      d = fmaf(qs[4 * c + 2], kv.z, d);
      d = fmaf(qs[4 * c + 3], kv.w, d);
    }
    d *= 0.125f;
    sc[j] = d;
    mx = fmaxf(mx, d);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float den = 0.0f;
  for (int j = lane; j <= r; j += 32) {
    const float e = expf(sc[j] - mx);
    sc[j] = e;
    den += e;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  __syncwarp();
  float2 acc = make_float2(0.f, 0.f);
  for (int j = 0; j <= r; ++j) {
    const float pj = sc[j] / den;
    const float2 v = *reinterpret_cast<const float2*>(vc + static_cast<size_t>(j) * kW + h * 64 + 2 * lane);
    acc.x = fmaf(pj, v.x, acc.x);
    acc.y = fmaf(pj, v.y, acc.y);
  }
  *reinterpret_cast<float2*>(out + static_cast<size_t>(r) * kW + h * 64 + 2 * lane) = acc;
}

template <int EPI>
cudaError_t launch_rows_gemm(const RowsGemm& g, int splits, cudaStream_t st) {
  RowsGemm a = g;
  a.kchunk = g.K / splits;
  const dim3 grid(g.N / kBN, (g.M + kBM - 1) / kBM, splits);
  rows_gemm_kernel<EPI><<<grid, 256, 0, st>>>(a);
  return cudaGetLastError();
}

unsigned grid_of(size_t n) {
  const size_t b = (n + 255) / 256;
  return static_cast<unsigned>(b < 1184 ? (b ? b : 1) : 1184);
}

}  // namespace

int gpt_prefill_kernels_per_call() { return kLayers * 9; }

cudaError_t gpt_prefill_prepare() {
  return cudaFuncSetAttribute(rows_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>((8 * kMaxLen + 8 * 64) * sizeof(float)));
}

cudaError_t gpt_prefill_enqueue(const GptLayerPtrs* layers, const GptPrefillBuffers& b, int P, cudaStream_t st) {
  if (P < 1 || P > kMaxLen) return cudaErrorInvalidValue;
  const size_t att_smem = (static_cast<size_t>(8) * P + 8 * 64) * sizeof(float);
  float* part = b.part;
  for (int l = 0; l < kLayers; ++l) {
    const GptLayerPtrs& L = layers[l];
    float* kc = b.kc + static_cast<size_t>(l) * kMaxLen * kW;
    float* vc = b.vc + static_cast<size_t>(l) * kMaxLen * kW;
    rows_layernorm_kernel<<<P, 256, 0, st>>>(b.x, L.ln1_g, L.ln1_b, b.xn);
    RowsGemm g{};
    g.x = b.xn;
    g.w = L.w_attn;
    g.bias = L.b_attn;
    g.q = b.q;
    g.kc = kc;
    g.vc = vc;
    g.M = P;
    g.N = kQkv;
    g.K = kW;
    cudaError_t e = launch_rows_gemm<kEpiQkv>(g, 1, st);
    if (e != cudaSuccess) return e;
    rows_attention_kernel<<<dim3(kHeads, (P + 7) / 8), 256, att_smem, st>>>(b.q, kc, vc, b.attn, P);
    // h = x + attn W_proj^T + b (K split over 4 CTAs, partials summed in order)
    g = RowsGemm{};
    g.x = b.attn;
    g.w = L.w_proj;
    g.y = part;
    g.M = P;
    g.N = kW;
    g.K = kW;
    e = launch_rows_gemm<kEpiPartial>(g, kSplitNarrow, st);
    if (e != cudaSuccess) return e;
    rows_reduce_kernel<<<grid_of(static_cast<size_t>(P) * kW), 256, 0, st>>>(part, kSplitNarrow, P, kW, L.b_proj, b.x,
                                                                            b.h);
    rows_layernorm_kernel<<<P, 256, 0, st>>>(b.h, L.ln2_g, L.ln2_b, b.xn);
    g = RowsGemm{};
    g.x = b.xn;
    g.w = L.w_fc;
    g.bias = L.b_fc;
    g.y = b.m;
    g.M = P;
    g.N = kMlp;
    g.K = kW;
    e = launch_rows_gemm<kEpiGelu>(g, 1, st);
    if (e != cudaSuccess) return e;
    // x = h + m W_mproj^T + b (K split over 4 CTAs)
    g = RowsGemm{};
    g.x = b.m;
    g.w = L.w_mproj;
    g.y = part;
    g.M = P;
    g.N = kW;
    g.K = kMlp;
    e = launch_rows_gemm<kEpiPartial>(g, kSplitNarrow, st);
    if (e != cudaSuccess) return e;
    rows_reduce_kernel<<<grid_of(static_cast<size_t>(P) * kW), 256, 0, st>>>(part, kSplitNarrow, P, kW, L.b_mproj, b.h,
                                                                            b.x);
  }
  return cudaGetLastError();
}

}  // namespace itts
