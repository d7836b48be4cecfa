// Masked multi-head self-attention over packed QKV rows (head_dim 64, 8 heads).
//
// Input `qkv` is f16 [R, 1536] written by the QKV GEMM epilogue: q (RoPE'd and
// pre-scaled by 1/8) in columns h*64.., k (RoPE'd) in 512 + h*64.., v in
// 1024 + h*64... Each sequence s owns rows [s*T, s*T + T). Keys whose row mask
// is 0 get probability 0 (cpu_attention_single_head_masked,
// runtime/impl/tokenizer_tests.cpp:3960-3997); every query row gets an output.
// Output: f16 [R, 512], head h in columns h*64...
//
// Flash-style online softmax with fp32 statistics; K/V tiles of 64 keys are
// double-buffered with cp.async, S = QK^T and O += PV run on mma.sync
// m16n8k16 (f16 in, fp32 accumulate), P is reused from registers.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

#include "kernels.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace itts {

namespace {

constexpr int kHd = 64;
constexpr int kBQ = 64;
constexpr int kBKV = 64;
constexpr int kQkvLd = 1536;

// Swizzled offset (in halves) of 16-byte chunk `c` (0..7) of row `r` in a
// [rows][64] f16 tile: chunk index XOR (row & 7) spreads ldmatrix rows over banks.
__device__ __forceinline__ int swz(int r, int c) { return r * kHd + ((c ^ (r & 7)) << 3); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t* r, const void* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, const void* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Load a [64 rows][64 cols] f16 tile starting at sequence row `r0` and column
// `col` of the packed QKV buffer; rows >= T are zero-filled.
__device__ __forceinline__ void load_tile(__half* dst, const __half* qkv, size_t seq_base, int r0, int T, int col) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = threadIdx.x + i * 128;  // 512 chunks of 16 bytes
    const int r = idx >> 3, c = idx & 7;
    const int row = r0 + r;
    const bool valid = row < T;
    const __half* src = qkv + (seq_base + static_cast<size_t>(valid ? row : 0)) * kQkvLd + col + c * 8;
    cp_async16(dst + swz(r, c), src, valid);
  }
}

__global__ void __launch_bounds__(128) attn_fwd_kernel(const __half* __restrict__ qkv,
                                                       const float* __restrict__ row_mask,
                                                       __half* __restrict__ out, int T) {
  __shared__ __align__(128) __half sQ[kBQ * kHd];
  __shared__ __align__(128) __half sK[2][kBKV * kHd];
  __shared__ __align__(128) __half sV[2][kBKV * kHd];
  __shared__ float sBias[2][kBKV];

  griddep_wait();
  griddep_launch();
  const int qt = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t seq_base = static_cast<size_t>(s) * T;
  const int q0 = qt * kBQ;
  const int n_kv = (T + kBKV - 1) / kBKV;

  load_tile(sQ, qkv, seq_base, q0, T, h * kHd);
  load_tile(sK[0], qkv, seq_base, 0, T, 512 + h * kHd);
  load_tile(sV[0], qkv, seq_base, 0, T, 1024 + h * kHd);
  cp_commit();
  if (threadIdx.x < kBKV) {
    const int key = threadIdx.x;
    sBias[0][key] = (key < T && row_mask[seq_base + key] != 0.0f) ? 0.0f : -CUDART_INF_F;
  }

  uint32_t qf[4][4];
  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[j][e] = 0.0f;
  float m_r[2] = {-CUDART_INF_F, -CUDART_INF_F};
  float l_r[2] = {0.0f, 0.0f};
  const float kLog2e = 1.4426950408889634f;

  for (int kt = 0; kt < n_kv; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < n_kv) {
      const int nb = buf ^ 1;
      load_tile(sK[nb], qkv, seq_base, (kt + 1) * kBKV, T, 512 + h * kHd);
      load_tile(sV[nb], qkv, seq_base, (kt + 1) * kBKV, T, 1024 + h * kHd);
      cp_commit();
      if (threadIdx.x < kBKV) {
        const int key = (kt + 1) * kBKV + threadIdx.x;
        sBias[nb][threadIdx.x] = (key < T && row_mask[seq_base + key] != 0.0f) ? 0.0f : -CUDART_INF_F;
      }
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();

    if (kt == 0) {
      // Q fragments for this warp's 16 query rows, 4 k-steps of 16 dims.
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int r = warp * 16 + (lane & 15);
        const int c = kk * 2 + (lane >> 4);
        ldsm_x4(qf[kk], sQ + swz(r, c));
      }
    }

    // S = Q K^T for 16 rows x 64 keys.
    float sc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[j][e] = 0.0f;
#pragma unroll
      for (int kk2 = 0; kk2 < 2; ++kk2) {
        uint32_t b[4];
        const int r = j * 8 + (lane & 7);
        const int c = kk2 * 4 + (lane >> 3);
        ldsm_x4(b, sK[buf] + swz(r, c));
        mma16816(sc[j], qf[kk2 * 2], b[0], b[1]);
        mma16816(sc[j], qf[kk2 * 2 + 1], b[2], b[3]);
      }
    }

    // Mask, online softmax.
    const int tq = lane & 3;
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float b0 = sBias[buf][j * 8 + tq * 2];
      const float b1 = sBias[buf][j * 8 + tq * 2 + 1];
      sc[j][0] += b0;
      sc[j][1] += b1;
      sc[j][2] += b0;
      sc[j][3] += b1;
      mx[0] = fmaxf(mx[0], fmaxf(sc[j][0], sc[j][1]));
      mx[1] = fmaxf(mx[1], fmaxf(sc[j][2], sc[j][3]));
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
    }
    float ref[2], alpha[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      ref[i] = (mx[i] == -CUDART_INF_F) ? 0.0f : mx[i];
      alpha[i] = exp2f((m_r[i] - ref[i]) * kLog2e);
      m_r[i] = mx[i];
    }
    float rs[2] = {0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sc[j][0] = exp2f((sc[j][0] - ref[0]) * kLog2e);
      sc[j][1] = exp2f((sc[j][1] - ref[0]) * kLog2e);
      sc[j][2] = exp2f((sc[j][2] - ref[1]) * kLog2e);
      sc[j][3] = exp2f((sc[j][3] - ref[1]) * kLog2e);
      rs[0] += sc[j][0] + sc[j][1];
      rs[1] += sc[j][2] + sc[j][3];
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 1);
      rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 2);
      l_r[i] = l_r[i] * alpha[i] + rs[i];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o[j][0] *= alpha[0];
      o[j][1] *= alpha[0];
      o[j][2] *= alpha[1];
      o[j][3] *= alpha[1];
    }

    // O += P V.
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_h2(sc[2 * kk][0], sc[2 * kk][1]);
      pa[1] = pack_h2(sc[2 * kk][2], sc[2 * kk][3]);
      pa[2] = pack_h2(sc[2 * kk + 1][0], sc[2 * kk + 1][1]);
      pa[3] = pack_h2(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        uint32_t b[4];
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = jj * 2 + (lane >> 4);
        ldsm_x4_t(b, sV[buf] + swz(r, c));
        mma16816(o[2 * jj], pa, b[0], b[1]);
        mma16816(o[2 * jj + 1], pa, b[2], b[3]);
      }
    }
    __syncthreads();
  }

  // Normalise and store.
  const int g = lane >> 2, tq = lane & 3;
  const float inv0 = l_r[0] > 0.0f ? 1.0f / l_r[0] : 0.0f;
  const float inv1 = l_r[1] > 0.0f ? 1.0f / l_r[1] : 0.0f;
  const int r0 = q0 + warp * 16 + g;
  const int r1 = r0 + 8;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int col = h * kHd + j * 8 + tq * 2;
    if (r0 < T) {
      *reinterpret_cast<__half2*>(out + (seq_base + r0) * 512 + col) = __floats2half2_rn(o[j][0] * inv0, o[j][1] * inv0);
    }
    if (r1 < T) {
      *reinterpret_cast<__half2*>(out + (seq_base + r1) * 512 + col) = __floats2half2_rn(o[j][2] * inv1, o[j][3] * inv1);
    }
  }
}

}  // namespace

cudaError_t attention_run(const __half* qkv, const float* row_mask, __half* out, int S, int T, cudaStream_t st) {
  if (S <= 0 || T <= 0) return cudaErrorInvalidValue;
  dim3 grid((T + kBQ - 1) / kBQ, 8, S);
  return launch_pdl(attn_fwd_kernel, grid, dim3(128), 0, st, qkv, row_mask, out, T);
}

}  // namespace itts
