// tcgen05 flash attention for the DiT blocks (sm_100a): one CTA computes 128
// queries of one (sequence, head) against all keys of its sequence in blocks
// of 128 keys.
//
//   warp 0      : TMA producer (Q once; K and V blocks into a 4-deep ring) and
//                 the per-block key-mask bias row
//   warps 1, 10 : tcgen05.mma issuers (lane 0), one per 64-key half h; per
//                 block j:
//                 S_j,h = Q K_j,h^T (M=128, N=64, K=64) and
//                 [O_h | l_h] += P_j,h [V_j,h | 1] (M=128, N=80, K=64; P from
//                 TMEM, V read MN-major from shared memory)
//   warps 2..9  : online softmax, two warps per query row quarter, each over
//                 its own 64-key half of every block: S_j,h from TMEM, P_j,h
//                 (f16) back into TMEM over the S columns it has read (the O
//                 MMA's A operand); O stays in TMEM (rescaled lazily there);
//                 the halves merge at the end.
// The two halves are independent pipelines (own issuer, barriers, S buffers
// and O), so the two softmax warps sharing an SM sub-partition need not run
// in phase: one can compute exponentials while the other loads S and takes
// its row maximum. The K/V ring is shared (a stage is free after both halves'
// O MMAs of its block).
// TMEM: S double buffer (2 x 128 columns: half h at columns 64 h of each) and
// one O accumulator per key half (2 x 128 columns, 80 used).
//
// Semantics follow cpu_attention_single_head_masked
// (runtime/impl/tokenizer_tests.cpp:3960-3997): keys with mask 0 get
// probability 0; q arrives RoPE'd and scaled by 1/8 from the QKV epilogue.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

#include <atomic>

#include "kernels.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace itts {

namespace {

constexpr int kQ = 128;    // queries per CTA
constexpr int kKB = 128;   // keys per block
constexpr int kThreadsA = 64 + 8 * 32 + 32;  // producer, MMA (half 0), 8 softmax warps, MMA (half 1)
constexpr int kIssuer1 = 10;                  // warp issuing the MMAs of key half 1
constexpr int kKV = 4;     // K/V ring depth (blocks in flight)
constexpr int OFF_Q = 0;
constexpr int OFF_K = 16384;                      // kKV stages x 16 KB
constexpr int OFF_V = OFF_K + kKV * 16384;        // kKV stages x 16 KB
constexpr int OFF_ONES = OFF_V + kKV * 16384;     // 16 rows x 128 B: the ones column appended to V
constexpr int OFF_BIAS = OFF_ONES + 2048;         // kKV x 128 floats
constexpr int OFF_FLAG = OFF_BIAS + kKV * kKB * 4;  // kKV ints: block has no masked key
constexpr int OFF_XCH = OFF_FLAG + 16;               // row-max / row-sum exchange: 6 x 128 floats
constexpr int OFF_XTAG = OFF_XCH + 6 * 128 * 4;      // exchange tags: 2 halves x 128 rows
constexpr int OFF_BAR = OFF_XTAG + 2 * 128 * 4;
constexpr int SMEM_A = 1024 + OFF_BAR + 256;
constexpr uint32_t TMEM_S = 0;    // + 128 * stage
constexpr uint32_t TMEM_O = 256;  // + 128 * key half: 64 output dims, then the row sum (column 64)
constexpr int kON = 80;           // O MMA width: 64 dims of V plus the ones column (and 15 zero columns)

enum : unsigned int { kDevTimeoutAttn = 16 };

// Timeline hooks for performance investigation: compiled out unless a harness
// defines ITTS_ATTN_TRACE and provides itts_attn_trace_point(slot).
#ifdef ITTS_ATTN_TRACE
#define ATTN_TRACE(slot) itts_attn_trace_point(slot)
#else
#define ATTN_TRACE(slot) ((void)0)
#endif

// 2^x on the special-function unit (|rel err| < 2^-22; inputs here are <= 8).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA/ALU pipes, for x <= 8 (the lazily rescaled softmax keeps
// exponents there): x = i + f with i = round(x) (via the 1.5*2^23 rounding
// constant) and f in [-0.5, 0.5]; 2^f from a degree-3 polynomial fitted
// (weighted least squares iterated towards minimax) to relative error 7.5e-5
// on that interval, below the 4.9e-4 rounding of the f16 P operand; 2^i added
// to the exponent bits. x is clamped at -125 so the result stays a normal
// number (2^-125 rounds to 0 in the f16 P operand).
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

// Three-input maximum (one instruction on sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__global__ void __launch_bounds__(kThreadsA, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm, const float* __restrict__ row_mask, __half* __restrict__ out,
                   int T, unsigned int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* q_full = bars;               // 1
  uint64_t* kv_full = bars + 1;          // kKV
  uint64_t* kv_empty = kv_full + kKV;    // kKV
  // Per key half h and S buffer b, index 2 h + b.
  uint64_t* s_full = kv_empty + kKV;     // 4: S_j,h landed
  uint64_t* s_free = s_full + 4;         // 4: the O MMA that read P_j,h (over S_j,h) is done
  uint64_t* p_full = s_free + 4;         // 4: P_j,h written by the half's 4 softmax warps
  uint64_t* o_full = p_full + 4;         // 4: O_h MMA of block j landed
  uint64_t* stagger = o_full + 4;        // 1: half 0 has taken the row maximum of block 0
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(stagger + 1);
  float* bias = reinterpret_cast<float*>(sm + OFF_BIAS);
  int* full_block = reinterpret_cast<int*>(sm + OFF_FLAG);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
  const int q0 = qt * kQ;
  const int seq0 = s * T;
  const int nkb = (T + kKB - 1) / kKB;

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kKV; ++i) {
      mbar_init(&kv_full[i], 1 + 32);  // producer expect_tx + 32 lanes writing the mask row
      mbar_init(&kv_empty[i], 2);  // one commit per key half
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 1);  // commit after the O MMA that read P from this S buffer
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(stagger, 4);
    fence_barrier_init();
    fence_proxy_async_shared();
    prefetch_tmap(&tm);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // Exchange tags start at 0 for every row and half (shared memory is not
  // cleared between CTAs); the barrier below publishes them.
  if (threadIdx.x < 2 * 128) reinterpret_cast<int*>(sm + OFF_XTAG)[threadIdx.x] = 0;
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
  if (threadIdx.x == 0) ATTN_TRACE(0);

  if (warp == 0) {
    // ---- producer ----
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, kQ * 128);
      tma_load_3d(sm + OFF_Q, &tm, q_full, 0, seq0 + q0, h);
    }
    for (int j = 0; j < nkb; ++j) {
      const int st = j % kKV;
      const uint32_t ph = (j / kKV) & 1;
      if (!mbar_wait(&kv_empty[st], ph ^ 1, status, kDevTimeoutAttn)) break;
      if (lane == 0) {
        if (j < 8) ATTN_TRACE(192 + j);  // slots 192..199: K/V block j requested
        mbar_arrive_expect_tx(&kv_full[st], 2 * kKB * 128);
        tma_load_3d(sm + OFF_K + st * 16384, &tm, &kv_full[st], 0, seq0 + j * kKB, 8 + h);
        tma_load_3d(sm + OFF_V + st * 16384, &tm, &kv_full[st], 0, seq0 + j * kKB, 16 + h);
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
  } else if (warp == 1 || warp == kIssuer1) {
    // ---- MMA issuers: warp 1 for key half 0, warp kIssuer1 for key half 1 ----
    const int hh = warp == 1 ? 0 : 1;
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(128, kKB / 2);
      constexpr uint32_t idesc_o = idesc_f16_f32(128, kON) | (1u << 16);  // B (V | ones) MN-major
      const uint32_t s_ones = smem_u32(sm + OFF_ONES);
      const uint32_t sq = smem_u32(sm + OFF_Q);
      bool ok = mbar_wait(q_full, 0, status, kDevTimeoutAttn);
      // S_j,h into S buffer j & 1, columns 64 h, once K/V block j has landed
      // and the O MMA that last read the buffer (block j - 2) is done. K rows
      // [64 h, 64 h + 64) of the block start 8 KB (eight 1 KB swizzle atoms)
      // into its stage.
      auto issue_s = [&](int j) -> bool {
        const int b = 2 * hh + (j & 1);
        if (!mbar_wait(&kv_full[j % kKV], (j / kKV) & 1, status, kDevTimeoutAttn)) return false;
        if (!mbar_wait(&s_free[b], ((j >> 1) & 1) ^ 1, status, kDevTimeoutAttn)) return false;
        tc_fence_after();
        if (j < 8) ATTN_TRACE(160 + 2 * j + hh);  // slots 160..175: S_j,h issued
        const uint32_t sk = smem_u32(sm + OFF_K + (j % kKV) * 16384 + hh * 8192);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16_ss(tmem + TMEM_S + (j & 1) * 128 + hh * 64, sdesc_k_sw128(sq + k * 32), sdesc_k_sw128(sk + k * 32),
                      idesc_s, k != 0 ? 1u : 0u);
        umma_commit(&s_full[b]);
        return true;
      };
      // Half 1 starts once half 0 has its first row maximum, so that the two
      // halves' exponential phases (which share the SFU) do not coincide.
      if (ok && hh == 1) ok = mbar_wait(stagger, 0, status, kDevTimeoutAttn);
      if (ok) ok = issue_s(0);
      if (ok && nkb > 1) ok = issue_s(1);
      for (int j = 0; j < nkb && ok; ++j) {
        // [O_h | l_h] += P_j,h [V_j,h | 1]; the half accumulates into its own
        // TMEM columns across all key blocks.
        const int b = 2 * hh + (j & 1);
        if (!mbar_wait(&p_full[b], (j >> 1) & 1, status, kDevTimeoutAttn)) break;
        tc_fence_after();
        if (j < 8) ATTN_TRACE(128 + 2 * j + hh);  // slots 128..143: O_j,h issued
        const uint32_t sv = smem_u32(sm + OFF_V + (j % kKV) * 16384);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t vb = sv + (hh * 4 + kk) * 2048;
          umma_f16_ts(tmem + TMEM_O + hh * 128, tmem + TMEM_S + (j & 1) * 128 + hh * 64 + kk * 8,
                      sdesc_mn_sw128_lbo(vb, s_ones - vb), idesc_o, (j | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&o_full[b]);
        umma_commit(&s_free[b]);           // P_j,h consumed: the buffer may take S_j+2,h
        umma_commit(&kv_empty[j % kKV]);   // this half is done with K/V block j
        if (j + 2 < nkb) ok = issue_s(j + 2);
      }
    }
    __syncwarp();
  } else {
    // ---- softmax: warps 2..9. The two warps of a TMEM lane quarter share 32
    // query rows; warp half hh owns keys [64 hh, 64 hh + 64) of every block
    // and runs its own online softmax over them (its own running maximum m,
    // row sum l and TMEM accumulator O_hh), so the pair never synchronises
    // inside the key loop. The halves are merged once at the end.
    // O_hh and l are rescaled lazily: only when a block's maximum exceeds the
    // reference m by more than 8 in log2 units (P <= 2^8 stays exact in f16).
    const int quarter = warp & 3;
    const int hh = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_o = tmem + lane_off + TMEM_O + hh * 128;
    const float kLog2e = 1.4426950408889634f;
    const float kLazy = 8.0f / kLog2e;
    float* xval = reinterpret_cast<float*>(sm + OFF_XCH);          // [3 slots][2 halves][128 rows]
    volatile int* xtag = reinterpret_cast<volatile int*>(sm + OFF_XTAG);  // [2 halves][128 rows]
    float m = -CUDART_INF_F;  // reference maximum of O_hh and its row sum (TMEM column 64)
    bool ok = true;
    for (int j = 0; j < nkb && ok; ++j) {
      const int st = j & 1;
      const int b = 2 * hh + st;  // this half's barriers of S buffer st
      if (!mbar_wait(&s_full[b], (j >> 1) & 1, status, kDevTimeoutAttn)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[64];
      tmem_ld32_async(tmem + lane_off + TMEM_S + st * 128 + hh * 64, sr);
      tmem_ld32_async(tmem + lane_off + TMEM_S + st * 128 + hh * 64 + 32, sr + 32);
      tmem_wait_ld();
      reg_fence32(sr);
      reg_fence32(sr + 32);
      if (quarter == 0 && lane == 0 && j < 8) ATTN_TRACE(64 * hh + 20 + j);
      // The mask row of this block was published with kv_full (already complete).
      const int kst = j % kKV;
      if (!mbar_wait(&kv_full[kst], (j / kKV) & 1, status, kDevTimeoutAttn)) {
        ok = false;
        break;
      }
      if (!full_block[kst]) {
        const float* brow = bias + kst * kKB + hh * 64;
#pragma unroll
        for (int k = 0; k < 64; ++k) sr[k] = __float_as_uint(__uint_as_float(sr[k]) + brow[k]);
      }
      float mp[8];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        mp[e] = fmax3(__uint_as_float(sr[e]), __uint_as_float(sr[8 + e]), __uint_as_float(sr[16 + e]));
#pragma unroll
      for (int k = 24; k < 56; k += 16) {
#pragma unroll
        for (int e = 0; e < 8; ++e) mp[e] = fmax3(mp[e], __uint_as_float(sr[k + e]), __uint_as_float(sr[k + 8 + e]));
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) mp[e] = fmaxf(mp[e], __uint_as_float(sr[56 + e]));
      const float mb = fmax3(fmax3(mp[0], mp[1], mp[2]), fmax3(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7]));
      if (quarter == 0 && lane == 0 && j < 8) ATTN_TRACE(64 * hh + 40 + j);
      if (j == 0 && hh == 0 && lane == 0) mbar_arrive(stagger);
      if (mb > m + kLazy) {  // the first live key, or a maximum grown past 2^8
        if (m != -CUDART_INF_F) {
          // O_hh and its row sum hold contributions relative to m: rescale
          // them once the previous block's O MMA has landed.
          const float alpha = ex2_approx((m - mb) * kLog2e);
          if (!mbar_wait(&o_full[2 * hh + ((j - 1) & 1)], ((j - 1) >> 1) & 1, status, kDevTimeoutAttn)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
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
          tmem_wait_st();
        }
        m = mb;
      }
      // P (f16 pairs, key order) overwrites the first 32 of this warp's 64 S
      // columns, which it has already read; the O MMA takes it from there.
      const float nref = (m == -CUDART_INF_F) ? 0.0f : -m * kLog2e;
      uint32_t pw[32];
#pragma unroll
      for (int c = 0; c < 8; ++c) {  // 8 chunks of 8 keys
        float p[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          // One in four on the FMA pipe, the rest on the SFU (the units run in parallel).
          const float xe = fmaf(__uint_as_float(sr[c * 8 + e]), kLog2e, nref);
          p[e] = (e & 3) == 3 ? ex2_poly(xe) : ex2_approx(xe);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __half2 h2 = __floats2half2_rn(p[2 * e], p[2 * e + 1]);
          pw[c * 4 + e] = *reinterpret_cast<const uint32_t*>(&h2);
        }
      }
      if (quarter == 0 && lane == 0 && j < 8) ATTN_TRACE(64 * hh + 50 + j);
      tmem_st32(tmem + lane_off + TMEM_S + st * 128 + hh * 64, pw);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
      if (quarter == 0 && lane == 0 && j < 8) ATTN_TRACE(64 * hh + 30 + j);
    }
    // Merge the two key halves of the row: each warp hands the partner the 32
    // output dims the partner writes (through the now idle P buffers), its
    // reference maximum and its row sum.
    uint32_t ov[32], oth[32], lv[16];  // O_hh at this warp's output dims / at the partner's; row sum
    // Both halves' last O MMAs (which follow all their S MMAs) must be done:
    // this warp's own result, and the K ring (reused for the exchange below)
    // no longer read by the other half.
    if (ok) ok = mbar_wait(&o_full[2 * hh + ((nkb - 1) & 1)], ((nkb - 1) >> 1) & 1, status, kDevTimeoutAttn);
    if (ok) ok = mbar_wait(&o_full[2 * (hh ^ 1) + ((nkb - 1) & 1)], ((nkb - 1) >> 1) & 1, status, kDevTimeoutAttn);
    if (ok) {
      tc_fence_after();
      tmem_ld32_async(t_o + hh * 32, ov);
      tmem_ld32_async(t_o + (hh ^ 1) * 32, oth);
      tmem_ld16_async(t_o + 64, lv);
      tmem_wait_ld();
      reg_fence32(ov);
      reg_fence32(oth);
      reg_fence16(lv);
      const float l = __uint_as_float(lv[0]);
      float* ox = reinterpret_cast<float*>(sm + OFF_K);  // [reader half][32 dims][128 rows] over the idle K ring
#pragma unroll
      for (int d = 0; d < 32; ++d) ox[((hh ^ 1) * 32 + d) * 128 + row] = __uint_as_float(oth[d]);
      xval[(1 * 2 + hh) * 128 + row] = l;
      xval[(0 * 2 + hh) * 128 + row] = m;
      __threadfence_block();
      xtag[hh * 128 + row] = 1;
      const long long t0 = clock64();
      while (xtag[(hh ^ 1) * 128 + row] < 1) {
        if (clock64() - t0 > kWaitBudgetCycles) {
          if (status) atomicCAS(status, 0u, static_cast<unsigned int>(kDevTimeoutAttn));
          ok = false;
          break;
        }
      }
      __threadfence_block();
      if (ok && q0 + row < T) {
        const float mo = xval[(0 * 2 + (hh ^ 1)) * 128 + row];
        const float lo = xval[(1 * 2 + (hh ^ 1)) * 128 + row];
        const float mm = fmaxf(m, mo);
        const float as = (m == -CUDART_INF_F) ? 0.0f : ex2_approx((m - mm) * kLog2e);
        const float ao = (mo == -CUDART_INF_F) ? 0.0f : ex2_approx((mo - mm) * kLog2e);
        const float lsum = l * as + lo * ao;
        const float inv = lsum > 0.0f ? 1.0f / lsum : 0.0f;
        const float* mine = ox + (hh * 32) * 128 + row;
        uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(seq0 + q0 + row) * 512 + h * 64 + hh * 32);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          union {
            __half2 h2[4];
            uint4 u;
          } pk;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int d0 = c * 8 + 2 * e;
            const float v0 = (__uint_as_float(ov[d0]) * as + mine[d0 * 128] * ao) * inv;
            const float v1 = (__uint_as_float(ov[d0 + 1]) * as + mine[(d0 + 1) * 128] * ao) * inv;
            pk.h2[e] = __floats2half2_rn(v0, v1);
          }
          dst[c] = pk.u;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) ATTN_TRACE(63);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

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
  static PerDeviceOnce configured;
  const cudaError_t e = configured.run(
      [] { return cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_A); });
  if (e != cudaSuccess) return e;
  dim3 grid((T + kQ - 1) / kQ, 8, S);
  return launch_pdl(attn_tc_kernel, grid, dim3(kThreadsA), SMEM_A, st, tm, row_mask, out, T, status);
}

}  // namespace itts
