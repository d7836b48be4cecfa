// tcgen05 GEMM for the DiT-CFM estimator: C[M,N] = A[M,K] * B[N,K]^T with f16
// operands staged by TMA (128-byte swizzle, no multicast), fp32 accumulation
// in TMEM and fused epilogues that read the accumulator with tcgen05.ld.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace itts {

// How the A operand's k-blocks (64 columns each) are fetched.
enum GemmAMode : int {
  kAPlain = 0,  // every k-block from A0
  kASplit = 1,  // k-blocks [0, kb_split) from A0, the rest from A1 (a concat without a buffer)
  kAConv = 2,   // implicit conv: k-block kb is tap (kb / kb_per_tap), reading A0 at column
                // (kb % kb_per_tap)*64 and row (m0 + tap * conv_dil + conv_off); rows outside
                // the tensor read as zeros (the k=5 WaveNet conv: conv_dil 1, conv_off -2 over
                // a reflect-padded row space; a transposed-conv phase: conv_dil -1)
};

// Fused epilogues. "Paired" epilogues expect B rows interleaved in 64-row
// groups [a(64) | b(64)] so each 128-column slab holds matching a/b channels.
enum GemmEpi : int {
  kEpiF16 = 0,        // out16 = acc + bias
  kEpiF32 = 1,        // out32 = acc + bias (+ resid32); optional f16 copy to out16
  kEpiQKV = 2,        // RoPE on q,k columns, q scaled by 1/sqrt(64), -> out16
  kEpiSwiGLU = 3,     // paired: silu(a) * b -> out16 (N/2 channels)
  kEpiWnGate = 4,     // paired, padded row space: tanh(a + ca) * sigmoid(b + cb) -> out16 (compact rows)
  kEpiWnResSkip = 5,  // paired: xp = (xp + a) * mask (with reflect halos); acc = (first ? 0 : acc) + b
  kEpiWnLast = 6,     // out32 = (acc + a) * mask + res
  kEpiConv1Res = 7,   // columns < 512 -> xp (f16, reflect halos); columns >= 512 -> out32 (res)
};

struct GemmArgs {
  int M;        // rows of the A row space (compact R, or padded S*(T+4) in conv mode)
  int N;        // columns of the product (rows of B)
  int num_kb;   // k-blocks of 64
  int a_mode;
  int kb_split;
  int kb_per_tap;
  int conv_dil;           // kAConv: row step per tap (the dilation, or -1 for a transposed-conv phase)
  int conv_off;           // kAConv: row offset of tap 0
  int epi;
  const float* bias;      // [N] in B-row order, or null
  float* out32;
  int ld32;
  __half* out16;
  int ld16;
  const float* resid32;
  int ldr;
  int seq_T;              // rows per sequence (T)
  const float2* rope;     // [32][T] (cos, sin) of t / 10000^(2p/64) at rope[p * T + t]
  const float* wn_cond;   // [1024] WaveNet global condition of this layer: a-part | b-part
  const float* row_mask;  // [R] 0/1 per compact row
  float* wn_acc;          // [R,512] skip accumulator
  const float* wn_res;    // [R,512] residual projection
  __half* wn_xp;          // [S*(T+4),512] reflect-padded WaveNet activations
  int wn_first;
  int pad_rows;           // kEpiF32 only: A rows are the padded S*(T+4) space; write compact rows
  int tma_o32;            // kEpiF32: out32 is written by TMA stores through GemmLaunch::tmO (set by gemm_run)
  int tma_o16;            // kEpiF16 / kEpiQKV / kEpiSwiGLU: out16 likewise (set by gemm_run)
  unsigned int* status;   // device status word
  // AdaRMSNorm folded across a producer/consumer GEMM pair:
  //   y = w*g*(x*inv) + b,  inv = 1/sqrt(mean_k x^2 + 1e-5)
  //   y . W^T = inv * ((x*w*g) . W^T) + (b . W^T)
  // Producer (kEpiF32, tile width a multiple of 32): nrm16 = f16(v * nrm_w *
  // nrm_g) and, per 32-column group p of the output, ss_out[p * ss_ld + row] =
  // sum of v^2 over the group (the partial count never depends on the tile width).
  // Consumer (kEpiQKV, kEpiSwiGLU): the accumulator of row m is multiplied by
  // 1/sqrt(sum_p ss_in[p * ss_ld + m] / ss_n + 1e-5) before `bias` (which then
  // holds b . W^T) is added.
  __half* nrm16;
  int ldn;
  const float* nrm_w;
  const float* nrm_g;
  float* ss_out;
  const float* ss_in;
  int ss_parts;
  int ss_n;
  int ss_ld;
};

struct GemmLaunch {
  CUtensorMap tmA0;
  CUtensorMap tmA1;
  CUtensorMap tmB;  // box rows: bn, or bn / 2 for the CTA-pair form
  CUtensorMap tmO;  // the TMA-stored output (encoded by gemm_run): kEpiF32 out32 as fp32 {N, M} with the
                    // 128-byte swizzle, or out16 as f16 {columns, M} with the 64-byte swizzle; box 32 x 32
  GemmArgs args;
  int bn;
  int pair;  // 1: CTA-pair form (clusters of 2, cta_group::2 MMA over 256-row tiles)
};

// k-blocks (64 columns each) fetched per TMA instruction: one TMA box moves
// kbox x rows x 128 B, and larger boxes raise the per-SM ingest rate (a
// 1600x512x512 F32 GEMM at BN=64 runs 3-4% faster with 4 than with 2).
// Tiles narrower than 64 columns (32, 48: the late BigVGAN stages) fetch one
// k-block per box, so that a conv tap of a single 64-channel block fits.
__host__ __device__ constexpr int gemm_kbox(int bn) { return bn < 64 ? 1 : bn == 64 ? 4 : bn <= 128 ? 2 : 1; }

// Bytes of one pipeline stage of a CTA: kbox k-blocks of A (128 rows) and of
// B (bn rows, or bn / 2 in the CTA-pair form).
__host__ __device__ constexpr int gemm_stage_bytes(int bn, bool pair) {
  return gemm_kbox(bn) * (128 * 64 * 2 + (pair ? bn / 2 : bn) * 64 * 2);
}

// Pipeline depth for a tile width: as many stages as fit next to the
// epilogue's shared memory (constants, 8 x 4 KB store stages, barriers) in the
// 227 KB a CTA may use, at most 8.
__host__ __device__ constexpr int gemm_stages(int bn, bool pair) {
  return ((232448 - 1024 - 256 - 8 * bn - 32768 - 512) / gemm_stage_bytes(bn, pair)) > 8
             ? 8
             : ((232448 - 1024 - 256 - 8 * bn - 32768 - 512) / gemm_stage_bytes(bn, pair));
}

// Host helpers (gemm.cu).
// Tensor map of a row-major f16 matrix [rows][cols] (row stride ld_elems)
// viewed as {64, rows, cols/64}; the box is {64, box_rows, kbox}. cols must be
// a multiple of 64 (pad the matrix with zero columns).
bool make_tmap_f16(CUtensorMap* tm, const void* base, uint64_t cols, uint64_t rows, uint64_t ld_elems,
                   uint32_t box_rows, uint32_t kbox);
cudaError_t gemm_run(const GemmLaunch& g, cudaStream_t stream);
size_t gemm_smem_bytes(int bn, int stages, bool pair);
// Tile width (64, 128 or 256; paired epilogues need a multiple of 128) that
// minimises waves x per-tile cost for an M x N output on this GPU; the
// per-tile cost is dominated by the bytes a CTA ingests per k-block (16 KB of
// A plus 128 B per B row it holds). Always the single-CTA form (see gemm.cu).
struct GemmPick {
  int bn;
  int pair;
};
GemmPick gemm_pick(int M, int N, bool paired_epilogue);

}  // namespace itts
