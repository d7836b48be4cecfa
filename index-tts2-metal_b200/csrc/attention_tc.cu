// tcgen05 flash attention for the DiT blocks (sm_100a).
//
// Persistent: one CTA per SM walks work items (sequence, head, pair of
// 128-query tiles) round-robin. The two query tiles of an item share every
// K/V block and run as a ping-pong: while the tensor core computes one tile's
// S = Q K^T and O += P V, the other tile's softmax warps turn their S into P,
// so neither the tensor pipe nor the softmax warps wait on each other.
//
//   warp 0     : TMA producer: Q tiles (once per item) and K/V blocks of 128
//                keys into a kKV-deep ring; the 32 lanes also publish each
//                block's key-mask bias row
//   warp 1     : lane 0 issues every tcgen05.mma; the warp owns the TMEM
//                allocation
//   warps 2..5 : softmax of query tile 0, warps 6..9 : of query tile 1; a
//                thread owns one query row (its TMEM lane) and all 128 keys
//                of a block: S from TMEM, running maximum, P = 2^(S - m)
//                as packed f16 pairs (ex2.approx.f16x2) written back over the
//                S columns it has read (the A operand of O += P [V | 1]); O
//                stays in TMEM and is rescaled there only when the maximum
//                grows by more than 2^8 (P <= 256 stays exact in f16); at the
//                end of the item the warps normalise O and store it.
//
// TMEM (512 columns): S_t at columns 128 t (t = query tile), O_t at 256 +
// 128 t: 64 output dims, then the row sum l (column 64, from the ones column
// appended to V), 80 columns written by an N = 80 MMA.
// The S_t columns are reissued only after the O_t MMA that read P_t from them
// has completed (its commit), so no MMA writes TMEM another one still reads.
//
// Semantics follow cpu_attention_single_head_masked
// (runtime/impl/tokenizer_tests.cpp:3960-3997): keys with mask 0 get
// probability 0; q arrives RoPE'd and scaled by 1/8 from the QKV epilogue. A
// query row whose keys are all masked gets output 0 (the reference divides 0
// by 0 there; production masks always keep real keys).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

#include <cstdlib>

#include "kernels.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace itts {

namespace {

constexpr int kQ = 128;   // queries per tile
constexpr int kKB = 128;  // keys per block
constexpr int kKV = 4;    // K/V ring depth (blocks in flight)
constexpr int kSoftWarps = 4;                        // per query tile
constexpr int kThreadsA = 64 + 2 * kSoftWarps * 32;  // producer, MMA issuer, 2 x 4 softmax warps
constexpr int OFF_Q = 0;                             // 2 tiles x 16 KB
constexpr int OFF_K = 2 * 16384;                     // kKV stages x 16 KB
constexpr int OFF_V = OFF_K + kKV * 16384;           // kKV stages x 16 KB
constexpr int OFF_ONES = OFF_V + kKV * 16384;        // 16 key rows x 128 B: the ones column appended to V
constexpr int OFF_BIAS = OFF_ONES + 2048;            // kKV x 128 floats
constexpr int OFF_FLAG = OFF_BIAS + kKV * kKB * 4;   // kKV ints: block has no masked key
constexpr int OFF_BAR = OFF_FLAG + kKV * 4;
constexpr int kBars = 2 + 2 + 2 * kKV + 2 + 2 + 2 + 2;  // q_full, q_empty, kv_full/empty, s_full, p_full, o_done, o_free
constexpr int SMEM_A = 1024 + OFF_BAR + kBars * 8 + 16;
constexpr uint32_t TMEM_S = 0;    // + 128 * tile
constexpr uint32_t TMEM_O = 256;  // + 128 * tile
constexpr int kON = 80;           // O MMA width: 64 dims of V, the ones column, 15 zero columns

enum : unsigned int { kDevTimeoutAttn = 16 };

// 2^x on the special-function unit for fp32 (rescale factors).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two exponentials in one instruction: (2^lo, 2^hi) as a packed f16 pair
// (lo in the low half), i.e. exactly the f16 P operand the O MMA reads. The
// inputs are rounded to f16 first (x <= 8 here, so the rounding of x moves
// 2^x by at most 2^-9 relative; ex2.approx.f16x2 itself is within the f16
// precision of its result).
__device__ __forceinline__ uint32_t ex2_pair(float lo, float hi) {
  uint32_t h, r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(hi), "f"(lo));
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(r) : "r"(h));
  return r;
}

// 2^x on the FMA/ALU pipes, for x <= 8: x = i + f with i = round(x) (via the
// 1.5*2^23 rounding constant) and f in [-0.5, 0.5]; 2^f from a degree-3
// polynomial fitted (weighted least squares iterated towards minimax) to
// relative error 7.5e-5 on that interval, below the 4.9e-4 rounding of the
// f16 P operand; 2^i added to the exponent bits. x is clamped at -125 so the
// result stays a normal number (2^-125 rounds to 0 in the f16 P operand).
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -125.0f);
  const float kRound = 12582912.0f;  // 1.5 * 2^23
  const float t = x + kRound;
  const int i = __float_as_int(t) - __float_as_int(kRound);
  const float f = x - (t - kRound);
  float p = 0.05517167f;
  p = fmaf(p, f, 0.24261114f);
  p = fmaf(p, f, 0.69326097f);
  p = fmaf(p, f, 0.99992806f);
  return __int_as_float(__float_as_int(p) + (i << 23));
}

// f16 bits of a non-negative fp32 value v (v < 65520), without a conversion
// instruction: v * 2^-112 moves the exponent bias from 127 to 15 (and lands
// f16 subnormals on fp32 subnormals), the top 16 bits after rounding at bit 12
// are then the f16 encoding (round half up).
__device__ __forceinline__ uint32_t f16_bits_scaled(float v_times_2m112) {
  return (static_cast<uint32_t>(__float_as_int(v_times_2m112)) + 0x1000u) >> 13;
}

// SFU 2^x without flushing subnormal results (so x - 112 keeps f16 subnormals).
__device__ __forceinline__ float ex2_sfu(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Exponentials of a key pair packed as the f16 P operand (lo key in the low
// half). EXPV selects how: 0 packed f16 SFU exponential; 1 fp32 SFU, cvt pack;
// 2 as 1 with every fourth pair on the FMA pipe; 3 fp32 SFU with the f16 bias
// folded in, integer pack; 4 as 3 with every fourth pair on the FMA pipe; 5 as
// 3 with three of every eight pairs on the FMA pipe. `e` is the pair index.
template <int EXPV>
__device__ __forceinline__ uint32_t exp_pair(float s0, float s1, float kl2, float nref, int e) {
  const float x0 = fmaf(s0, kl2, nref), x1 = fmaf(s1, kl2, nref);
  if constexpr (EXPV == 0) {
    return ex2_pair(x0, x1);
  } else if constexpr (EXPV == 1 || EXPV == 2) {
    float y0, y1;
    if (EXPV == 2 && (e & 3) == 3) {
      y0 = ex2_poly(x0);
      y1 = ex2_poly(x1);
    } else {
      y0 = ex2_approx(x0);
      y1 = ex2_approx(x1);
    }
    uint32_t h;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(y1), "f"(y0));
    return h;
  } else {
    const bool poly = (EXPV == 4 && (e & 3) == 3) || (EXPV == 5 && ((e & 7) == 2 || (e & 7) == 5 || (e & 7) == 7));
    float y0, y1;
    if (poly) {
      y0 = ex2_poly(x0) * 1.92592994e-34f;  // 2^-112
      y1 = ex2_poly(x1) * 1.92592994e-34f;
    } else {
      y0 = ex2_sfu(x0 - 112.0f);
      y1 = ex2_sfu(x1 - 112.0f);
    }
    return __byte_perm(f16_bits_scaled(y0), f16_bits_scaled(y1), 0x5410);
  }
}

// Three-input maximum (one instruction on sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Work item -> (sequence, head, first query row); items enumerate sequences,
// then heads, then query-tile pairs, so the CTAs of one wave share K/V in L2.
struct Item {
  int s, h, q0;
};
__device__ __forceinline__ Item item_at(int it, int pairs) {
  const int qp = it % pairs;
  const int sh = it / pairs;
  return Item{sh >> 3, sh & 7, qp * 2 * kQ};
}

template <int EXPV>
__global__ void __launch_bounds__(kThreadsA, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm, const float* __restrict__ row_mask, __half* __restrict__ out,
                   int S, int T, unsigned int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* q_full = bars;              // [2] Q tile t landed
  uint64_t* q_empty = q_full + 2;       // [2] the item's last S_t MMA is done (Q_t may be replaced)
  uint64_t* kv_full = q_empty + 2;      // [kKV] K/V block landed and its mask row written
  uint64_t* kv_empty = kv_full + kKV;   // [kKV] every O MMA of the block is done
  uint64_t* s_full = kv_empty + kKV;    // [2] S_t of the current block landed
  uint64_t* p_full = s_full + 2;        // [2] P_t written by the tile's 4 softmax warps
  uint64_t* o_done = p_full + 2;        // [2] O_t MMA of the current block done
  uint64_t* o_free = o_done + 2;        // [2] O_t of the finished item read out by the softmax warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_free + 2);
  float* bias = reinterpret_cast<float*>(sm + OFF_BIAS);
  int* full_block = reinterpret_cast<int*>(sm + OFF_FLAG);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = (T + kKB - 1) / kKB;
  const int tiles = (T + kQ - 1) / kQ;
  const int pairs = (tiles + 1) / 2;
  const int items = S * 8 * pairs;

  if (warp == 0 && lane == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(&q_full[t], 1);
      mbar_init(&q_empty[t], 1);
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], kSoftWarps);
      mbar_init(&o_done[t], 1);
      mbar_init(&o_free[t], kSoftWarps);
    }
    for (int i = 0; i < kKV; ++i) {
      mbar_init(&kv_full[i], 1 + 32);  // producer expect_tx + 32 lanes writing the mask row
      mbar_init(&kv_empty[i], 1);
    }
    fence_barrier_init();
    fence_proxy_async_shared();
    prefetch_tmap(&tm);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // The ones column of the O MMA: element 64 of every key row of V's second
  // MN atom is 1 (so column 64 of O accumulates the row sum of P), elements
  // 65..127 are 0. 16 key rows in the 128-byte swizzle (chunk c of row r at
  // chunk c ^ (r & 7)); every K16 step of the MMA points here through its LBO.
  for (int i = threadIdx.x; i < 512; i += blockDim.x) {
    const int r = i >> 5, w = i & 31;
    reinterpret_cast<uint32_t*>(sm + OFF_ONES)[i] = ((w >> 2) == (r & 7) && (w & 3) == 0) ? 0x3C00u : 0u;
  }
  fence_proxy_async_shared();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();
  griddep_launch();

  if (warp == 0) {
    // ---- producer ----
    int g = 0;             // running K/V block count (ring position and phase)
    int nq[2] = {0, 0};    // items so far in which query tile t was active (phase of q_full / q_empty)
    bool ok = true;
    for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
      const Item I = item_at(it, pairs);
      const int seq0 = I.s * T;
      const int nt = (I.q0 + kQ < T) ? 2 : 1;
      for (int t = 0; t < nt && ok; ++t) {
        // Q_t of the tile's previous item must no longer be read by an S MMA.
        if (nq[t] > 0 && !(ok = mbar_wait(&q_empty[t], (nq[t] - 1) & 1, status, kDevTimeoutAttn))) break;
        ++nq[t];
        if (lane == 0) {
          mbar_arrive_expect_tx(&q_full[t], kQ * 128);
          tma_load_3d(sm + OFF_Q + t * 16384, &tm, &q_full[t], 0, seq0 + I.q0 + t * kQ, I.h);
        }
      }
      for (int j = 0; j < nkb && ok; ++j, ++g) {
        const int st = g % kKV;
        if (g >= kKV && !(ok = mbar_wait(&kv_empty[st], ((g / kKV) - 1) & 1, status, kDevTimeoutAttn))) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&kv_full[st], 2 * kKB * 128);
          tma_load_3d(sm + OFF_K + st * 16384, &tm, &kv_full[st], 0, seq0 + j * kKB, 8 + I.h);
          tma_load_3d(sm + OFF_V + st * 16384, &tm, &kv_full[st], 0, seq0 + j * kKB, 16 + I.h);
        }
        bool valid4 = true;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int k = lane * 4 + i;
          const int key = j * kKB + k;
          const bool valid = key < T && row_mask[seq0 + key] != 0.0f;
          valid4 = valid4 && valid;
          bias[st * kKB + k] = valid ? 0.0f : -CUDART_INF_F;
        }
        const bool all_valid = __all_sync(0xffffffffu, valid4);
        if (lane == 0) full_block[st] = all_valid ? 1 : 0;
        __syncwarp();
        mbar_arrive(&kv_full[st]);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(128, kKB);
      constexpr uint32_t idesc_o = idesc_f16_f32(128, kON) | (1u << 16);  // B (V | ones) MN-major
      const uint32_t s_ones = smem_u32(sm + OFF_ONES);
      int g = 0;             // running K/V block count
      int nblk[2] = {0, 0};  // running block count per tile (phase of s_full / p_full / o_done)
      int nq[2] = {0, 0};    // items so far in which tile t was active (phase of q_full / o_free)
      bool ok = true;
      // S_t(block) = Q_t K_block^T into S_t.
      auto issue_s = [&](int t, int st) {
        const uint32_t sq = smem_u32(sm + OFF_Q + t * 16384);
        const uint32_t sk = smem_u32(sm + OFF_K + st * 16384);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16_ss(tmem + TMEM_S + t * 128, sdesc_k_sw128(sq + k * 32), sdesc_k_sw128(sk + k * 32), idesc_s,
                      k != 0 ? 1u : 0u);
        umma_commit(&s_full[t]);
      };
      // [O_t | l_t] (+)= P_t [V | 1], P_t read from the S_t columns.
      auto issue_o = [&](int t, int st, bool first) {
        const uint32_t sv = smem_u32(sm + OFF_V + st * 16384);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t vb = sv + kk * 2048;
          umma_f16_ts(tmem + TMEM_O + t * 128, tmem + TMEM_S + t * 128 + kk * 8,
                      sdesc_mn_sw128_lbo(vb, s_ones - vb), idesc_o, (!first || kk != 0) ? 1u : 0u);
        }
        umma_commit(&o_done[t]);
      };
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
        const Item I = item_at(it, pairs);
        const int nt = (I.q0 + kQ < T) ? 2 : 1;
        // First block: S_t(0) for each tile once Q_t and K/V block 0 landed and
        // the previous item's last O_t MMA (reading P_t from S_t) is done.
        const int st0 = g % kKV;
        if (!(ok = mbar_wait(&kv_full[st0], (g / kKV) & 1, status, kDevTimeoutAttn))) break;
        for (int t = 0; t < nt && ok; ++t) {
          if (!(ok = mbar_wait(&q_full[t], nq[t] & 1, status, kDevTimeoutAttn))) break;
          if (nblk[t] > 0 && !(ok = mbar_wait(&o_done[t], (nblk[t] - 1) & 1, status, kDevTimeoutAttn))) break;
          tc_fence_after();
          issue_s(t, st0);
          if (nkb == 1) umma_commit(&q_empty[t]);
        }
        for (int j = 0; j < nkb && ok; ++j) {
          const int st = (g + j) % kKV;
          const int stn = (g + j + 1) % kKV;
          for (int t = 0; t < nt && ok; ++t) {
            const int b = nblk[t] + j;  // this tile's block index (phase)
            if (!(ok = mbar_wait(&p_full[t], b & 1, status, kDevTimeoutAttn))) break;
            // The softmax warps have read the tile's previous O_t before its first O MMA overwrites it.
            if (j == 0 && nq[t] > 0 && !(ok = mbar_wait(&o_free[t], (nq[t] - 1) & 1, status, kDevTimeoutAttn)))
              break;
            tc_fence_after();
            issue_o(t, st, j == 0);
            if (t == nt - 1) umma_commit(&kv_empty[st]);  // every O MMA of the block is issued
            if (j + 1 < nkb) {
              if (t == 0 && !(ok = mbar_wait(&kv_full[stn], ((g + j + 1) / kKV) & 1, status, kDevTimeoutAttn)))
                break;
              // S_t(j+1) overwrites the P_t(j) columns: wait for the O MMA that reads them.
              if (!(ok = mbar_wait(&o_done[t], b & 1, status, kDevTimeoutAttn))) break;
              tc_fence_after();
              issue_s(t, stn);
              if (j + 2 == nkb) umma_commit(&q_empty[t]);
            }
          }
        }
        for (int t = 0; t < nt; ++t) {
          nblk[t] += nkb;
          ++nq[t];
        }
        g += nkb;
      }
    }
    __syncwarp();
  } else {
    // ---- softmax + epilogue: warps 2..5 tile 0, warps 6..9 tile 1 ----
    const int t = (warp - 2) / kSoftWarps;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_s = tmem + lane_off + TMEM_S + t * 128;
    const uint32_t t_o = tmem + lane_off + TMEM_O + t * 128;
    const float kLog2e = 1.4426950408889634f;
    const float kLazy = 8.0f / kLog2e;
    int g = 0;     // running K/V block count (mask rows)
    int nblk = 0;  // running block count of this tile
    bool ok = true;
    for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
      const Item I = item_at(it, pairs);
      const int nt = (I.q0 + kQ < T) ? 2 : 1;
      if (t >= nt) {  // this tile is past the end of the sequence: nothing to do for the item
        g += nkb;
        continue;
      }
      float m = -CUDART_INF_F;  // reference maximum of O_t and its row sum
      for (int j = 0; j < nkb && ok; ++j) {
        const int b = nblk + j;
        if (!(ok = mbar_wait(&s_full[t], b & 1, status, kDevTimeoutAttn))) break;
        tc_fence_after();
        uint32_t sr[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32_async(t_s + c * 32, sr + c * 32);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c) reg_fence32(sr + c * 32);
        // The mask row of this block was published with kv_full (already complete).
        const int kst = (g + j) % kKV;
        if (!(ok = mbar_wait(&kv_full[kst], ((g + j) / kKV) & 1, status, kDevTimeoutAttn))) break;
        if (!full_block[kst]) {
          const float* brow = bias + kst * kKB;
#pragma unroll
          for (int k = 0; k < 128; ++k) sr[k] = __float_as_uint(__uint_as_float(sr[k]) + brow[k]);
        }
        float mp[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
          mp[e] = fmax3(__uint_as_float(sr[e]), __uint_as_float(sr[8 + e]), __uint_as_float(sr[16 + e]));
#pragma unroll
        for (int k = 24; k < 120; k += 16) {
#pragma unroll
          for (int e = 0; e < 8; ++e) mp[e] = fmax3(mp[e], __uint_as_float(sr[k + e]), __uint_as_float(sr[k + 8 + e]));
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) mp[e] = fmaxf(mp[e], __uint_as_float(sr[120 + e]));
        const float mb = fmax3(fmax3(mp[0], mp[1], mp[2]), fmax3(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7]));
        // The first live key, or a maximum grown past 2^8: move the reference
        // maximum to this block's and rescale O_t (after P is written, so the
        // S registers are free by then).
        float alpha = 1.0f;
        bool rescale = false;
        if (mb > m + kLazy) {
          if (m != -CUDART_INF_F) {
            alpha = ex2_approx((m - mb) * kLog2e);
            rescale = true;
          }
          m = mb;
        }
        // P (f16 pairs, key order) over the first 64 of the tile's S columns,
        // which this thread has already read; the O MMA takes it from there.
        const float nref = (m == -CUDART_INF_F) ? 0.0f : -m * kLog2e;
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // 4 chunks of 32 keys -> 16 columns each
          uint32_t pw[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            pw[e] = exp_pair<EXPV>(__uint_as_float(sr[c * 32 + 2 * e]), __uint_as_float(sr[c * 32 + 2 * e + 1]),
                                   kLog2e, nref, e);
          tmem_st16(t_s + c * 16, pw);
        }
        if (rescale) {
          // O_t and its row sum hold contributions relative to the old maximum.
          // The O MMA of the previous block has completed: S_t(j) was issued
          // only after it (the issuer waits for it before reusing S_t).
          if (!(ok = mbar_wait(&o_done[t], (b - 1) & 1, status, kDevTimeoutAttn))) break;
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            uint32_t ov[32];
            tmem_ld32_async(t_o + c * 32, ov);
            tmem_wait_ld();
            reg_fence32(ov);
#pragma unroll
            for (int d = 0; d < 32; ++d) ov[d] = __float_as_uint(__uint_as_float(ov[d]) * alpha);
            tmem_st32(t_o + c * 32, ov);
          }
          uint32_t lv[16];
          tmem_ld16_async(t_o + 64, lv);
          tmem_wait_ld();
          reg_fence16(lv);
          lv[0] = __float_as_uint(__uint_as_float(lv[0]) * alpha);
          tmem_st16(t_o + 64, lv);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
      }
      if (!ok) break;
      // Epilogue: the item's last O_t MMA, then O / l for this row.
      const int bl = nblk + nkb - 1;
      if (!(ok = mbar_wait(&o_done[t], bl & 1, status, kDevTimeoutAttn))) break;
      tc_fence_after();
      uint32_t ov[64], lv[16];
      tmem_ld32_async(t_o, ov);
      tmem_ld32_async(t_o + 32, ov + 32);
      tmem_ld16_async(t_o + 64, lv);
      tmem_wait_ld();
      reg_fence32(ov);
      reg_fence32(ov + 32);
      reg_fence16(lv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[t]);  // O_t may take the next item's first MMA
      const int q = I.q0 + t * kQ + row;
      if (q < T) {
        const float l = __uint_as_float(lv[0]);
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
        uint4* dst = reinterpret_cast<uint4*>(out + (static_cast<size_t>(I.s) * T + q) * 512 + I.h * 64);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          union {
            __half2 h2[4];
            uint4 u;
          } pk;
#pragma unroll
          for (int e = 0; e < 4; ++e)
            pk.h2[e] = __floats2half2_rn(__uint_as_float(ov[c * 8 + 2 * e]) * inv,
                                         __uint_as_float(ov[c * 8 + 2 * e + 1]) * inv);
          dst[c] = pk.u;
        }
      }
      nblk += nkb;
      g += nkb;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int sms() {
  static int n = [] {
    int dev = 0, v = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v > 0 ? v : 148;
  }();
  return n;
}

}  // namespace

bool make_attn_tmap(CUtensorMap* tm, const __half* qkv, int R) {
  // qkv [R][1536] viewed as {64, R, 24 k-blocks}: block h = q head h, 8+h = k, 16+h = v.
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return false;
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(R), 24};
  cuuint64_t strides[2] = {1536 * 2, 128};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(qkv), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t attention_tc_run(const CUtensorMap& tm, const float* row_mask, __half* out, int S, int T,
                             unsigned int* status, cudaStream_t st) {
  if (S <= 0 || T <= 0) return cudaErrorInvalidValue;
  static const int variant = [] {
    const char* v = std::getenv("ITTS_ATTN_EXP");
    return v ? std::atoi(v) : 0;
  }();
  const long long tiles = (T + kQ - 1) / kQ;
  const long long items = static_cast<long long>(S) * 8 * ((tiles + 1) / 2);
  const int grid = static_cast<int>(items < sms() ? items : sms());
  auto go = [&](auto kern, PerDeviceOnce& once) -> cudaError_t {
    const cudaError_t e =
        once.run([&] { return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_A); });
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, dim3(grid), dim3(kThreadsA), SMEM_A, st, tm, row_mask, out, S, T, status);
  };
  static PerDeviceOnce c0, c1, c2, c3, c4, c5;
  switch (variant) {
    case 1: return go(attn_tc_kernel<1>, c1);
    case 2: return go(attn_tc_kernel<2>, c2);
    case 3: return go(attn_tc_kernel<3>, c3);
    case 4: return go(attn_tc_kernel<4>, c4);
    case 5: return go(attn_tc_kernel<5>, c5);
    default: return go(attn_tc_kernel<0>, c0);
  }
}

}  // namespace itts
