// Launchers for the non-GEMM kernels of the DiT-CFM sampler.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace itts {

// Row strides of the zero-padded GEMM operands: 80 mel columns padded to two
// 64-column k-blocks, 784 merge columns padded to 13 k-blocks.
constexpr int kXdLd = 128;
constexpr int kUld = 832;

// Masked MHA over packed QKV on tcgen05 (attention_tc.cu). make_attn_tmap builds
// the tensor map of qkv [R][1536]; attention_tc_run launches S x 8 heads x
// ceil(T/128) CTAs.
bool make_attn_tmap(CUtensorMap* tm, const __half* qkv, int R);
cudaError_t attention_tc_run(const CUtensorMap& tm, const float* row_mask, __half* out, int S, int T,
                             unsigned int* status, cudaStream_t st);

// y = w (.) (x * rsqrt(mean(x^2) + 1e-5) (.) gamma) + b per 512-wide row;
// wb = [w(512) | b(512)]. f32 in, f16 out.
cudaError_t adarms_run(const float* x, int R, const float* wb, const float* gamma, __half* out, cudaStream_t st);

// y = LN(x; eps 1e-6, no affine) * (1 + scale) + shift; ss = [shift(512) | scale(512)].
cudaError_t adaln_run(const float* x, int R, const float* ss, __half* out, cudaStream_t st);

// Guided Euler update of the fp32 mel state X [B*T, 80]:
//   v = (1+cfg) * V[cond row] - cfg * V[null row]  (cfg > 0; branches == 2)
//   v = V[cond row]                                (branches == 1)
//   X += dt * v; rows t < P[u] -> 0; XD (f16, one copy per branch) = X.
cudaError_t euler_run(float* X, const float* V, __half* XD, const int* prompt_len, int B, int T, int branches,
                      float dt, float cfg, cudaStream_t st);

// Sampler start: X = X0 with prompt rows zeroed, and the f16 duplicates XD.
// X0 may equal X (in place).
cudaError_t euler_init_run(const float* X0, float* X, __half* XD, const int* prompt_len, int B, int T, int branches,
                           cudaStream_t st);

// f32 -> f16 conversion.
cudaError_t to_half_run(const float* x, __half* y, size_t n, cudaStream_t st);

// Build the 784-wide (row stride kUld, zero tail) step-invariant merge input per sequence row:
//   cond branch: [prompt_x(80) | CP(512) | style(192)], null branch: [0 | bcp | 0].
cudaError_t merge_input_run(const float* prompt_x, const __half* cp16, const float* bcp, const float* style,
                            __half* U, int B, int T, int branches, cudaStream_t st);

// y[b][n] = bias[n] + sum_k W[n][k] * x[b][k] (fp32 math); W f16 or f32.
// act_in: 0 none, 1 SiLU applied to x before the product.
cudaError_t gemv_f16w_run(const __half* W, const float* bias, const float* x, int ldx, float* y, int ldy, int N,
                          int K, int nb, int act_in, cudaStream_t st);
cudaError_t gemv_f32w_run(const float* W, const float* bias, const float* x, int ldx, float* y, int ldy, int N,
                          int K, int nb, int act_in, cudaStream_t st);

// Sinusoidal timestep embedding: emb[b] = [cos(scale*t_b*freqs) | sin(...)], 128 freqs.
cudaError_t tembed_run(const float* t, const float* freqs, float* emb, int nb, float scale, cudaStream_t st);

// Failure-detection self-test kernel (see bounded_wait_probe_kernel).
cudaError_t bounded_wait_probe_run(unsigned int* status, long long budget_cycles, cudaStream_t st);

// SiLU in place on fp32 (table build).
cudaError_t silu_run(float* x, size_t n, cudaStream_t st);

}  // namespace itts
