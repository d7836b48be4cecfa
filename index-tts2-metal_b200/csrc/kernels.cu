// HBM-bound kernels of the DiT-CFM sampler: adaptive RMSNorm / LayerNorm
// (warp per 512-wide row, float4 coalesced), the fused CFG + Euler + prompt-zero
// update, step-invariant merge-input assembly and the fp32 GEMVs that build the
// per-step t-conditioning tables.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace itts {

namespace {

constexpr int kC = 512;

// Kernels of the sampler graph are launched with programmatic dependent
// launch; each starts by waiting for its predecessor's memory.
__device__ __forceinline__ void pdl_entry() {
  griddep_wait();
  griddep_launch();
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void store_h4(__half* dst, float a, float b, float c, float d) {
  union {
    __half2 h[2];
    uint2 u;
  } pk;
  pk.h[0] = __floats2half2_rn(a, b);
  pk.h[1] = __floats2half2_rn(c, d);
  *reinterpret_cast<uint2*>(dst) = pk.u;
}

// Adaptive RMSNorm: run_adaptive_norm_cpu (runtime/impl/dit_cfm_bigvgan.cpp:260-276)
// with cpu_rmsnorm (runtime/impl/tokenizer_tests.cpp:3012-3024), eps 1e-5.
__global__ void __launch_bounds__(256) adarms_kernel(const float* __restrict__ x, int R, const float* __restrict__ wb,
                                                     const float* __restrict__ gamma, __half* __restrict__ out) {
  pdl_entry();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= R) return;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * kC);
  float4 v[4];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[i] = xr[lane + 32 * i];
    ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
  }
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(kC) + 1e-5f);
  const float4* w4 = reinterpret_cast<const float4*>(wb);
  const float4* b4 = reinterpret_cast<const float4*>(wb + kC);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  __half* orow = out + static_cast<size_t>(row) * kC;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c4 = lane + 32 * i;
    const float4 w = w4[c4], b = b4[c4], g = g4[c4];
    store_h4(orow + c4 * 4, w.x * (v[i].x * inv * g.x) + b.x, w.y * (v[i].y * inv * g.y) + b.y,
             w.z * (v[i].z * inv * g.z) + b.z, w.w * (v[i].w * inv * g.w) + b.w);
  }
}

// Final-layer AdaLN: run_dit_final_layer_cpu (runtime/impl/dit_cfm_bigvgan.cpp:1172-1199)
// with cpu_layernorm (runtime/impl/tokenizer_tests.cpp:2992-3010), eps 1e-6.
__global__ void __launch_bounds__(256) adaln_kernel(const float* __restrict__ x, int R, const float* __restrict__ ss,
                                                    __half* __restrict__ out) {
  pdl_entry();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= R) return;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * kC);
  float4 v[4];
  float sum = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[i] = xr[lane + 32 * i];
    sum += v[i].x + v[i].y + v[i].z + v[i].w;
  }
  const float mean = warp_sum(sum) / static_cast<float>(kC);
  float var = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
    var += a * a + b * b + c * c + d * d;
  }
  var = warp_sum(var) / static_cast<float>(kC);
  const float inv = 1.0f / sqrtf(var + 1e-6f);
  const float4* sh4 = reinterpret_cast<const float4*>(ss);
  const float4* sc4 = reinterpret_cast<const float4*>(ss + kC);
  __half* orow = out + static_cast<size_t>(row) * kC;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c4 = lane + 32 * i;
    const float4 sh = sh4[c4], sc = sc4[c4];
    store_h4(orow + c4 * 4, (v[i].x - mean) * inv * (1.0f + sc.x) + sh.x, (v[i].y - mean) * inv * (1.0f + sc.y) + sh.y,
             (v[i].z - mean) * inv * (1.0f + sc.z) + sh.z, (v[i].w - mean) * inv * (1.0f + sc.w) + sh.w);
  }
}

// Guided Euler step: run_cfm_euler_cpu (runtime/impl/dit_cfm_bigvgan.cpp:2908-2937) and
// the fused reference kernel cfm_euler_update (metal/kernels.metal:794-818).
// Sequence order in the velocity buffer: s = u * branches + branch.
__global__ void euler_kernel(float* __restrict__ X, const float* __restrict__ V, __half* __restrict__ XD,
                             const int* __restrict__ prompt_len, int B, int T, int branches, float dt, float cfg) {
  pdl_entry();
  // One thread per 4 consecutive mel bins of a frame (20 per 80-bin row).
  const size_t total = static_cast<size_t>(B) * T * 20;
  for (size_t q = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; q < total;
       q += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t f = q / 20;  // frame index u * T + t
    const int c4 = static_cast<int>(q - f * 20);
    const int u = static_cast<int>(f / static_cast<size_t>(T));
    const int t = static_cast<int>(f - static_cast<size_t>(u) * T);
    const size_t cond_row = (static_cast<size_t>(u) * branches) * T + t;
    float4 v = reinterpret_cast<const float4*>(V + cond_row * 80)[c4];
    if (branches == 2) {
      const float4 vu = reinterpret_cast<const float4*>(V + (cond_row + T) * 80)[c4];
      v.x = (1.0f + cfg) * v.x - cfg * vu.x;
      v.y = (1.0f + cfg) * v.y - cfg * vu.y;
      v.z = (1.0f + cfg) * v.z - cfg * vu.z;
      v.w = (1.0f + cfg) * v.w - cfg * vu.w;
    }
    float4* xp = reinterpret_cast<float4*>(X + f * 80) + c4;
    float4 x = *xp;
    x.x += dt * v.x;
    x.y += dt * v.y;
    x.z += dt * v.z;
    x.w += dt * v.w;
    if (t < prompt_len[u]) x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    *xp = x;
    union {
      __half2 h[2];
      uint2 u2;
    } pk;
    pk.h[0] = __floats2half2_rn(x.x, x.y);
    pk.h[1] = __floats2half2_rn(x.z, x.w);
    for (int b = 0; b < branches; ++b)
      *reinterpret_cast<uint2*>(XD + (cond_row + static_cast<size_t>(b) * T) * kXdLd + c4 * 4) = pk.u2;
  }
}

__global__ void euler_init_kernel(const float* X0, float* X, __half* __restrict__ XD,
                                  const int* __restrict__ prompt_len, int B, int T, int branches) {
  pdl_entry();
  const size_t total = static_cast<size_t>(B) * T * 80;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % 80);
    const size_t ut = i / 80;
    const int u = static_cast<int>(ut / T);
    const int t = static_cast<int>(ut - static_cast<size_t>(u) * T);
    float x = X0[i];
    if (t < prompt_len[u]) x = 0.0f;
    X[i] = x;
    const size_t cond_row = (static_cast<size_t>(u) * branches) * T + t;
    const __half xh = __float2half_rn(x);
    for (int b = 0; b < branches; ++b) XD[(cond_row + static_cast<size_t>(b) * T) * kXdLd + c] = xh;
  }
}

__global__ void to_half_kernel(const float* __restrict__ x, __half* __restrict__ y, size_t n) {
  pdl_entry();
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    y[i] = __float2half_rn(x[i]);
}

// Merge input without the x slice (run_dit_input_merge_cpu,
// runtime/impl/dit_cfm_bigvgan.cpp:1-19): columns 80..863 of the 864-wide row.
__global__ void merge_input_kernel(const float* __restrict__ prompt_x, const __half* __restrict__ cp16,
                                   const float* __restrict__ bcp, const float* __restrict__ style,
                                   __half* __restrict__ U, int B, int T, int branches) {
  pdl_entry();
  constexpr int W = kUld;
  const size_t total = static_cast<size_t>(B) * branches * T * W;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % W);
    const size_t row = i / W;  // sequence row
    const size_t seq = row / T;
    const int t = static_cast<int>(row - seq * T);
    const int u = static_cast<int>(seq / branches);
    const int br = static_cast<int>(seq - static_cast<size_t>(u) * branches);
    float v;
    if (br == 0) {
      if (c < 80) v = prompt_x[(static_cast<size_t>(u) * T + t) * 80 + c];
      else if (c < 592) v = __half2float(cp16[(static_cast<size_t>(u) * T + t) * 512 + (c - 80)]);
      else if (c < 784) v = style[static_cast<size_t>(u) * 192 + (c - 592)];
      else v = 0.0f;
    } else {
      v = (c >= 80 && c < 592) ? bcp[c - 80] : 0.0f;
    }
    U[i] = __float2half_rn(v);
  }
}

// One warp per output feature n; loops over the nb input vectors.
template <typename WT>
__global__ void __launch_bounds__(256) gemv_kernel(const WT* __restrict__ W, const float* __restrict__ bias,
                                                   const float* __restrict__ x, int ldx, float* __restrict__ y,
                                                   int ldy, int N, int K, int nb, int act_in) {
  const int n = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (n >= N) return;
  const WT* wr = W + static_cast<size_t>(n) * K;
  for (int b = 0; b < nb; ++b) {
    const float* xb = x + static_cast<size_t>(b) * ldx;
    float acc = 0.0f;
    for (int k = lane; k < K; k += 32) {
      float xv = xb[k];
      if (act_in == 1) xv = xv / (1.0f + expf(-xv));
      float wv;
      if constexpr (sizeof(WT) == 2) wv = __half2float(wr[k]);
      else wv = wr[k];
      acc += wv * xv;
    }
    acc = warp_sum(acc);
    if (lane == 0) y[static_cast<size_t>(b) * ldy + n] = acc + (bias ? bias[n] : 0.0f);
  }
}

// cpu_timestep_embedding (runtime/impl/tokenizer_tests.cpp:3947-3958).
__global__ void tembed_kernel(const float* __restrict__ t, const float* __restrict__ freqs, float* __restrict__ emb,
                              int nb, float scale) {
  const int b = blockIdx.x;
  const int i = threadIdx.x;  // 128 threads
  if (b >= nb) return;
  const float arg = scale * t[b] * freqs[i];
  emb[b * 256 + i] = cosf(arg);
  emb[b * 256 + 128 + i] = sinf(arg);
}

__global__ void silu_kernel(float* __restrict__ x, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float v = x[i];
    x[i] = v / (1.0f + expf(-v));
  }
}

inline unsigned grid_for(size_t n, int threads) {
  size_t b = (n + threads - 1) / threads;
  if (b > 148u * 16u) b = 148u * 16u;
  return static_cast<unsigned>(b == 0 ? 1 : b);
}

}  // namespace

// Failure-detection self-test: one thread waits on an mbarrier that nothing
// will complete, through the same bounded wait every kernel here uses, and
// gives up after `budget` cycles with kDevTimeoutProbe in the status word.
__global__ void bounded_wait_probe_kernel(unsigned int* status, long long budget) {
  __shared__ uint64_t bar;
  mbar_init(&bar, 1);
  fence_barrier_init();
  mbar_wait_for(&bar, 0, status, kDevTimeoutProbe, budget);
}

cudaError_t bounded_wait_probe_run(unsigned int* status, long long budget_cycles, cudaStream_t st) {
  bounded_wait_probe_kernel<<<1, 1, 0, st>>>(status, budget_cycles);
  return cudaGetLastError();
}

cudaError_t adarms_run(const float* x, int R, const float* wb, const float* gamma, __half* out, cudaStream_t st) {
  return launch_pdl(adarms_kernel, dim3((R + 7) / 8), dim3(256), 0, st, x, R, wb, gamma, out);
}

cudaError_t adaln_run(const float* x, int R, const float* ss, __half* out, cudaStream_t st) {
  return launch_pdl(adaln_kernel, dim3((R + 7) / 8), dim3(256), 0, st, x, R, ss, out);
}

cudaError_t euler_run(float* X, const float* V, __half* XD, const int* prompt_len, int B, int T, int branches,
                      float dt, float cfg, cudaStream_t st) {
  const size_t n = static_cast<size_t>(B) * T * 20;
  return launch_pdl(euler_kernel, dim3(grid_for(n, 256)), dim3(256), 0, st, X, V, XD, prompt_len, B, T, branches, dt,
                    cfg);
}

cudaError_t euler_init_run(const float* X0, float* X, __half* XD, const int* prompt_len, int B, int T, int branches,
                           cudaStream_t st) {
  const size_t n = static_cast<size_t>(B) * T * 80;
  return launch_pdl(euler_init_kernel, dim3(grid_for(n, 256)), dim3(256), 0, st, X0, X, XD, prompt_len, B, T, branches);
}

cudaError_t to_half_run(const float* x, __half* y, size_t n, cudaStream_t st) {
  return launch_pdl(to_half_kernel, dim3(grid_for(n, 256)), dim3(256), 0, st, x, y, n);
}

cudaError_t merge_input_run(const float* prompt_x, const __half* cp16, const float* bcp, const float* style,
                            __half* U, int B, int T, int branches, cudaStream_t st) {
  const size_t n = static_cast<size_t>(B) * branches * T * kUld;
  return launch_pdl(merge_input_kernel, dim3(grid_for(n, 256)), dim3(256), 0, st, prompt_x, cp16, bcp, style, U, B, T,
                    branches);
}

cudaError_t gemv_f16w_run(const __half* W, const float* bias, const float* x, int ldx, float* y, int ldy, int N,
                          int K, int nb, int act_in, cudaStream_t st) {
  gemv_kernel<__half><<<(N + 7) / 8, 256, 0, st>>>(W, bias, x, ldx, y, ldy, N, K, nb, act_in);
  return cudaGetLastError();
}

cudaError_t gemv_f32w_run(const float* W, const float* bias, const float* x, int ldx, float* y, int ldy, int N,
                          int K, int nb, int act_in, cudaStream_t st) {
  gemv_kernel<float><<<(N + 7) / 8, 256, 0, st>>>(W, bias, x, ldx, y, ldy, N, K, nb, act_in);
  return cudaGetLastError();
}

cudaError_t tembed_run(const float* t, const float* freqs, float* emb, int nb, float scale, cudaStream_t st) {
  tembed_kernel<<<nb, 128, 0, st>>>(t, freqs, emb, nb, scale);
  return cudaGetLastError();
}

cudaError_t silu_run(float* x, size_t n, cudaStream_t st) {
  silu_kernel<<<grid_for(n, 256), 256, 0, st>>>(x, n);
  return cudaGetLastError();
}

}  // namespace itts
