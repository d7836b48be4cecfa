// tcgen05 flash attention for the DiT blocks (sm_100a).
//
// Persistent: one CTA per SM walks work items (sequence, head, pair of
// 128-query tiles) round-robin. The two query tiles of an item share every
// K/V block, and each tile has its own MMA issuer, so the tensor core works
// for one tile while the other tile's softmax warps compute. When pairs would
// leave SMs idle (one short utterance), an item is one query tile instead and
// both softmax warp groups work on it, each on half of every key block (own
// running maximum, row sum and O), merging through shared memory at the end.
// The softmax warps are bound by the special-function unit: one ex2 per
// score, issued at about one warp instruction per 14 cycles per SM
// sub-partition on B200 (measured); polynomial exponentials on the FMA pipe
// were measured slower here, as the warps then run out of issue slots.
//
//   warp 0     : TMA producer: Q tiles (once per item) and K/V blocks of 128
//                keys into a kKV-deep ring; the 32 lanes also publish each
//                block's key-mask bias row
//   warp 1, 10 : lane 0 issues the tcgen05.mma of query tile 0 / 1; warp 1
//                owns the TMEM allocation
//   warps 2..5 : softmax of query tile 0, warps 6..9 : of query tile 1; a
//                thread owns one query row (its TMEM lane) and all 128 keys
//                of a block. It reads S into registers and at once releases
//                the S columns (so the next block's S = Q K^T is computed
//                while it works), takes the running maximum, computes
//                P = 2^(S - m) on the SFU in fp32, adds the row sum in fp32
//                and writes P as f16 pairs into its tile's P columns, the A
//                operand of O += P V. O stays in TMEM and is rescaled there
//                only when the maximum grows by more than 2^8 (P <= 256 stays
//                exact in f16); at the end of the item the warps normalise O
//                by the row sum and store it.
//
// TMEM (512 columns): S_t at columns 128 t, P_t at 256 + 64 t (128 keys as
// f16 pairs), O_t at 384 + 64 t (t = query tile).
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

#include "kernels.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace itts {

namespace {

constexpr int kQ = 128;   // queries per tile
constexpr int kKB = 128;  // keys per block
constexpr int kKV = 4;    // K/V ring depth (blocks in flight)
constexpr int kSoftWarps = 4;                            // per query tile
constexpr int kIssuer1 = 2 + 2 * kSoftWarps;             // warp issuing the MMAs of query tile 1
constexpr int kThreadsA = 32 * (kIssuer1 + 1);           // producer, issuer 0, 2 x 4 softmax warps, issuer 1
constexpr int OFF_Q = 0;                                 // 2 tiles x 16 KB
constexpr int OFF_K = 2 * 16384;                         // kKV stages x 16 KB
constexpr int OFF_V = OFF_K + kKV * 16384;               // kKV stages x 16 KB
constexpr int OFF_BIAS = OFF_V + kKV * 16384;            // kKV x 128 floats
constexpr int OFF_FLAG = OFF_BIAS + kKV * kKB * 4;       // kKV ints: block has no masked key
constexpr int OFF_XCH = OFF_FLAG + kKV * 4;         // key-split merge: [128 rows][64 dims + m + l] floats
constexpr int kXchLd = 66;
constexpr int OFF_BAR = OFF_XCH + 128 * kXchLd * 4;
// per tile: q_full, q_empty, s_full, s_free, p_full, o_done, o_free; the kv ring; x_full, x_empty
constexpr int kBars = 2 * 7 + 2 * kKV + 2;
constexpr int SMEM_A = 1024 + OFF_BAR + kBars * 8 + 16;
constexpr uint32_t TMEM_S = 0;    // + 128 * tile
constexpr uint32_t TMEM_P = 256;  // + 64 * tile
constexpr uint32_t TMEM_O = 384;  // + 64 * tile

enum : unsigned int { kDevTimeoutAttn = 16 };

// Timeline hooks for performance investigation: compiled out unless a harness
// defines ITTS_ATTN_TRACE and provides itts_attn_trace_point(slot) (slots are
// recorded for each CTA's first item only).
#ifdef ITTS_ATTN_TRACE
#define ATTN_TRACE(cond, slot) \
  do {                          \
    if (cond) itts_attn_trace_point(slot); \
  } while (0)
#else
#define ATTN_TRACE(cond, slot) ((void)0)
#endif

// 2^x on the special-function unit.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packs two floats as f16 (round to nearest even), lo in the low half.
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
  uint32_t h;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(hi), "f"(lo));
  return h;
}

// Three-input maximum (one instruction on sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Work item -> (sequence, head, first query row); items enumerate sequences,
// then heads, then groups of `tpi` query tiles (tpi = 2: a ping-pong pair;
// tpi = 1: one tile, for grids too small to fill the GPU with pairs), so the
// CTAs of one wave share K/V in L2.
struct Item {
  int s, h, q0;
};
__device__ __forceinline__ Item item_at(int it, int units, int tpi) {
  const int qp = it % units;
  const int sh = it / units;
  return Item{sh >> 3, sh & 7, qp * tpi * kQ};
}
// Query tiles of an item that hold rows of the sequence (tile 1 may not).
__device__ __forceinline__ int item_tiles(const Item& I, int T, int tpi) {
  return (tpi == 2 && I.q0 + kQ < T) ? 2 : 1;
}

// Shared state of the kernel's roles (shared-memory and TMEM addresses,
// barriers, the launch's shape).
struct AttnCtx {
  uint8_t* sm;
  uint64_t *q_full, *q_empty, *s_full, *s_free, *p_full, *o_done, *o_free, *kv_full, *kv_empty, *x_full, *x_empty;
  float* bias;
  int* full_block;
  uint32_t tmem;
  __half* out;
  unsigned int* status;
  int T, nkb, items, units, tpi;
};

// Softmax + epilogue of one warp group (4 warps, one query row per thread).
// NK = 128: the group owns query tile `wg` of pair items and all 128 keys of
// every block. NK = 64 (single-tile items): both groups work on the item's
// one tile, group `wg` on keys [64 wg, 64 wg + 64) of every block, each with
// its own running maximum, row sum and O accumulator; at the end of the item
// group 1 hands (O, m, l) to group 0 through shared memory, which merges the
// halves and stores the rows.
template <int NK>
__device__ __forceinline__ void softmax_role(const AttnCtx& c, int wg, int quarter, int lane) {
  constexpr bool kSplit = NK == 64;
  const int row = quarter * 32 + lane;
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  const int sidx = kSplit ? 0 : wg;  // S region / barriers this group reads
  const int kofs = kSplit ? 64 * wg : 0;  // first key of the group's share of a block
  const uint32_t t_s = c.tmem + lane_off + TMEM_S + sidx * 128 + kofs;
  const uint32_t t_p = c.tmem + lane_off + TMEM_P + wg * 64;
  const uint32_t t_o = c.tmem + lane_off + TMEM_O + wg * 64;
  const float kLog2e = 1.4426950408889634f;
  const float kLazy = 8.0f / kLog2e;
  float* xch = reinterpret_cast<float*>(c.sm + OFF_XCH) + row * kXchLd;
  int g = 0;     // running K/V block count (mask rows)
  int nblk = 0;  // running block count of this group (phase of s_full / p_full / o_done)
  int nitem = 0;  // items this group has worked on (phase of the merge barriers)
  bool ok = true;
  for (int it = blockIdx.x; it < c.items && ok; it += gridDim.x) {
    const Item I = item_at(it, c.units, c.tpi);
    if (!kSplit && wg >= item_tiles(I, c.T, c.tpi)) {
      g += c.nkb;
      continue;
    }
    float m = -CUDART_INF_F;  // reference maximum of O and l
    float l = 0.0f;           // row sum of P relative to m
    for (int j = 0; j < c.nkb && ok; ++j) {
      const int b = nblk + j;
      if (!(ok = mbar_wait(&c.s_full[sidx], b & 1, c.status, kDevTimeoutAttn))) break;
      [[maybe_unused]] const bool tr = row == 0 && nblk == 0 && j < 8;
      ATTN_TRACE(tr, 84 + wg * 16 + j);
      tc_fence_after();
      uint32_t sr[NK];
#pragma unroll
      for (int q = 0; q < NK / 32; ++q) tmem_ld32_async(t_s + q * 32, sr + q * 32);
      tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < NK / 32; ++q) reg_fence32(sr + q * 32);
      ATTN_TRACE(tr, 116 + wg * 16 + j);
      // S is in registers: the next block's S may overwrite it.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&c.s_free[sidx]);
      // The mask row of this block was published with kv_full (already complete).
      const int kst = (g + j) % kKV;
      if (!(ok = mbar_wait(&c.kv_full[kst], ((g + j) / kKV) & 1, c.status, kDevTimeoutAttn))) break;
      const int bflag = c.full_block[kst];
      // Chunks of 16 keys of this group's share that hold a live key; the rest
      // (keys past the end of the sequence in its last block, or masked) have
      // P = 2^(-inf) = +0 exactly and are written as zeros without an ex2.
      const int live = (bflag >> 8) - kofs / 16;
      if (!(bflag & 1)) {
        const float* brow = c.bias + kst * kKB + kofs;
#pragma unroll
        for (int k = 0; k < NK; ++k) sr[k] = __float_as_uint(__uint_as_float(sr[k]) + brow[k]);
      }
      float mp[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        mp[e] = fmax3(__uint_as_float(sr[e]), __uint_as_float(sr[4 + e]), __uint_as_float(sr[8 + e]));
#pragma unroll
      for (int k = 12; k < NK - 4; k += 8) {
#pragma unroll
        for (int e = 0; e < 4; ++e) mp[e] = fmax3(mp[e], __uint_as_float(sr[k + e]), __uint_as_float(sr[k + 4 + e]));
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) mp[e] = fmaxf(mp[e], __uint_as_float(sr[NK - 4 + e]));
      const float mb = fmaxf(fmax3(mp[0], mp[1], mp[2]), mp[3]);
      // The first live key, or a maximum grown past 2^8: move the reference
      // maximum to this block's; O and l are rescaled below.
      float alpha = 1.0f;
      bool rescale = false;
      if (mb > m + kLazy) {
        if (m != -CUDART_INF_F) {
          alpha = ex2_approx((m - mb) * kLog2e);
          rescale = true;
        }
        m = mb;
      }
      // P(j - 1) must have been read by its O MMA before it is overwritten
      // (and O is final for the rescale below).
      if (j > 0 && !(ok = mbar_wait(&c.o_done[wg], (b - 1) & 1, c.status, kDevTimeoutAttn))) break;
      tc_fence_after();
      const float nref = (m == -CUDART_INF_F) ? 0.0f : -m * kLog2e;
      float ls[2] = {0.0f, 0.0f};
#pragma unroll
      for (int q = 0; q < NK / 16; ++q) {  // chunks of 16 keys -> 8 columns of f16 pairs
        uint32_t pw[8];
        if (q < live) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float y0 = ex2_approx(fmaf(__uint_as_float(sr[q * 16 + 2 * e]), kLog2e, nref));
            const float y1 = ex2_approx(fmaf(__uint_as_float(sr[q * 16 + 2 * e + 1]), kLog2e, nref));
            ls[e & 1] += y0 + y1;
            pw[e] = pack_f16(y0, y1);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) pw[e] = 0u;
        }
        tmem_st8(t_p + q * 8, pw);
      }
      l = l * alpha + (ls[0] + ls[1]);
      if (rescale) {
#pragma unroll 1
        for (int q = 0; q < 2; ++q) {
          uint32_t ov[32];
          tmem_ld32_async(t_o + q * 32, ov);
          tmem_wait_ld();
          reg_fence32(ov);
#pragma unroll
          for (int d = 0; d < 32; ++d) ov[d] = __float_as_uint(__uint_as_float(ov[d]) * alpha);
          tmem_st32(t_o + q * 32, ov);
        }
      }
      tmem_wait_st();
      ATTN_TRACE(tr, 148 + wg * 16 + j);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&c.p_full[wg]);
    }
    if (!ok) break;
    // Epilogue: the item's last O MMA of this group, then O / l for the row.
    if (!(ok = mbar_wait(&c.o_done[wg], (nblk + c.nkb - 1) & 1, c.status, kDevTimeoutAttn))) break;
    ATTN_TRACE(row == 0 && nblk == 0, 182 + wg);
    tc_fence_after();
    uint32_t ov[64];
    tmem_ld32_async(t_o, ov);
    tmem_ld32_async(t_o + 32, ov + 32);
    tmem_wait_ld();
    reg_fence32(ov);
    reg_fence32(ov + 32);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&c.o_free[wg]);  // O may take the next item's first MMA
    float inv = l > 0.0f ? 1.0f / l : 0.0f;
    bool store = true;
    if constexpr (kSplit) {
      // Merge the key halves: group 1 publishes (O, m, l), group 0 combines.
      if (wg == 1) {
        if (nitem > 0 && !(ok = mbar_wait(c.x_empty, (nitem - 1) & 1, c.status, kDevTimeoutAttn))) break;
#pragma unroll
        for (int d = 0; d < 64; ++d) xch[d] = __uint_as_float(ov[d]);
        xch[64] = m;
        xch[65] = l;
        __threadfence_block();
        __syncwarp();
        if (lane == 0) mbar_arrive(c.x_full);
        store = false;
      } else {
        if (!(ok = mbar_wait(c.x_full, nitem & 1, c.status, kDevTimeoutAttn))) break;
        const float mo = xch[64], lo = xch[65];
        const float mm = fmaxf(m, mo);
        const float as = (m == -CUDART_INF_F) ? 0.0f : ex2_approx((m - mm) * kLog2e);
        const float ao = (mo == -CUDART_INF_F) ? 0.0f : ex2_approx((mo - mm) * kLog2e);
        const float lsum = l * as + lo * ao;
        const float r = lsum > 0.0f ? 1.0f / lsum : 0.0f;
#pragma unroll
        for (int d = 0; d < 64; ++d) ov[d] = __float_as_uint((__uint_as_float(ov[d]) * as + xch[d] * ao) * r);
        __threadfence_block();
        __syncwarp();
        if (lane == 0) mbar_arrive(c.x_empty);
        inv = 1.0f;
      }
    }
    const int q = I.q0 + (kSplit ? 0 : wg * kQ) + row;
    if (store && q < c.T) {
      uint4* dst = reinterpret_cast<uint4*>(c.out + (static_cast<size_t>(I.s) * c.T + q) * 512 + I.h * 64);
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        union {
          __half2 h2[4];
          uint4 u;
        } pk;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          pk.h2[e] = __floats2half2_rn(__uint_as_float(ov[cc * 8 + 2 * e]) * inv,
                                       __uint_as_float(ov[cc * 8 + 2 * e + 1]) * inv);
        dst[cc] = pk.u;
      }
    }
    ATTN_TRACE(row == 0 && nblk == 0, 184 + wg);
    nblk += c.nkb;
    g += c.nkb;
    ++nitem;
  }
}

__global__ void __launch_bounds__(kThreadsA, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm, const float* __restrict__ row_mask, __half* __restrict__ out,
                   int S, int T, int tpi, unsigned int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  AttnCtx c;
  c.sm = sm;
  c.q_full = bars;              // [2] Q tile t landed
  c.q_empty = c.q_full + 2;     // [2] the item's last S_t MMA is done (Q_t may be replaced)
  c.s_full = c.q_empty + 2;     // [2] S_t of the current block landed
  c.s_free = c.s_full + 2;      // [2] the softmax warps reading S_t have read it into registers
  c.p_full = c.s_free + 2;      // [2] P of warp group t written
  c.o_done = c.p_full + 2;      // [2] O MMA of warp group t for the current block done (its P may be rewritten)
  c.o_free = c.o_done + 2;      // [2] O of warp group t read out at the end of an item
  c.kv_full = c.o_free + 2;     // [kKV] K/V block landed and its mask row written
  c.kv_empty = c.kv_full + kKV; // [kKV] both O MMAs of the block are done
  c.x_full = c.kv_empty + kKV;  // key-split merge: group 1's (O, m, l) published
  c.x_empty = c.x_full + 1;     // key-split merge: group 0 has read them
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(c.x_empty + 1);
  c.bias = reinterpret_cast<float*>(sm + OFF_BIAS);
  c.full_block = reinterpret_cast<int*>(sm + OFF_FLAG);
  c.out = out;
  c.status = status;
  c.T = T;
  c.tpi = tpi;
  c.nkb = (T + kKB - 1) / kKB;
  const int tiles = (T + kQ - 1) / kQ;
  c.units = (tiles + tpi - 1) / tpi;  // work items per (sequence, head)
  c.items = S * 8 * c.units;
  const bool split = tpi == 1;  // single-tile items: both warp groups share the tile's keys

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = c.nkb, items = c.items, units = c.units;
  uint64_t *q_full = c.q_full, *q_empty = c.q_empty, *s_full = c.s_full, *s_free = c.s_free, *p_full = c.p_full,
           *o_done = c.o_done, *o_free = c.o_free, *kv_full = c.kv_full, *kv_empty = c.kv_empty;
  float* bias = c.bias;
  int* full_block = c.full_block;

  if (warp == 0 && lane == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(&q_full[t], 1);
      mbar_init(&q_empty[t], 1);
      mbar_init(&s_full[t], 1);
      mbar_init(&s_free[t], (split && t == 0) ? 2 * kSoftWarps : kSoftWarps);
      mbar_init(&p_full[t], kSoftWarps);
      mbar_init(&o_done[t], 1);
      mbar_init(&o_free[t], kSoftWarps);
    }
    for (int i = 0; i < kKV; ++i) {
      mbar_init(&kv_full[i], 1 + 32);  // producer expect_tx + 32 lanes writing the mask row
      mbar_init(&kv_empty[i], 2);      // one commit per issuer (the only issuer of a block commits twice)
    }
    mbar_init(c.x_full, kSoftWarps);
    mbar_init(c.x_empty, kSoftWarps);
    fence_barrier_init();
    fence_proxy_async_shared();
    prefetch_tmap(&tm);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  c.tmem = tmem;
  griddep_wait();
  griddep_launch();
  ATTN_TRACE(threadIdx.x == 0, 180);

  if (warp == 0) {
    // ---- producer ----
    int g = 0;           // running K/V block count (ring position and phase)
    int nq[2] = {0, 0};  // items so far in which query tile t was active (phase of q_full / q_empty)
    bool ok = true;
    for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
      const Item I = item_at(it, units, tpi);
      const int seq0 = I.s * T;
      const int nt = item_tiles(I, T, tpi);
      for (int t = 0; t < nt && ok; ++t) {
        // Q_t of the tile's previous item must no longer be read by an S MMA.
        if (nq[t] > 0 && !(ok = mbar_wait(&q_empty[t], (nq[t] - 1) & 1, status, kDevTimeoutAttn))) break;
        ++nq[t];
        ATTN_TRACE(lane == 0 && it == static_cast<int>(blockIdx.x), 8 + t);
        if (lane == 0) {
          mbar_arrive_expect_tx(&q_full[t], kQ * 128);
          tma_load_3d(sm + OFF_Q + t * 16384, &tm, &q_full[t], 0, seq0 + I.q0 + t * kQ, I.h);
        }
      }
      for (int j = 0; j < nkb && ok; ++j, ++g) {
        const int st = g % kKV;
        if (g >= kKV && !(ok = mbar_wait(&kv_empty[st], ((g / kKV) - 1) & 1, status, kDevTimeoutAttn))) break;
        ATTN_TRACE(lane == 0 && g < 8, g);
        if (lane == 0) {
          mbar_arrive_expect_tx(&kv_full[st], 2 * kKB * 128);
          tma_load_3d(sm + OFF_K + st * 16384, &tm, &kv_full[st], 0, seq0 + j * kKB, 8 + I.h);
          tma_load_3d(sm + OFF_V + st * 16384, &tm, &kv_full[st], 0, seq0 + j * kKB, 16 + I.h);
        }
        bool valid4 = true, any4 = false;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int k = lane * 4 + i;
          const int key = j * kKB + k;
          const bool valid = key < T && row_mask[seq0 + key] != 0.0f;
          valid4 = valid4 && valid;
          any4 = any4 || valid;
          bias[st * kKB + k] = valid ? 0.0f : -CUDART_INF_F;
        }
        const bool all_valid = __all_sync(0xffffffffu, valid4);
        // 16-key chunks (4 lanes each) up to the last one holding a live key.
        const unsigned live_lanes = __ballot_sync(0xffffffffu, any4);
        const int live_chunks = live_lanes ? (31 - __clz(live_lanes)) / 4 + 1 : 0;
        if (lane == 0) full_block[st] = (all_valid ? 1 : 0) | (live_chunks << 8);
        __syncwarp();
        mbar_arrive(&kv_full[st]);
        ATTN_TRACE(lane == 0 && g < 8, 10 + g);
      }
    }
  } else if (warp == 1 || warp == kIssuer1) {
    // ---- MMA issuer t: S and O of query tile t (pairs), or, for single-tile
    // items, S and O of key half 0 (t = 0) / O of key half 1 (t = 1) ----
    const int t = warp == 1 ? 0 : 1;
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(128, kKB);
      constexpr uint32_t idesc_o = idesc_f16_f32(128, 64) | (1u << 16);  // B (V) MN-major
      const uint32_t sq = smem_u32(sm + OFF_Q + t * 16384);
      const bool issues_s = !split || t == 0;
      const int o_steps = split ? 4 : 8;                // K16 steps of the O MMA (64 or 128 keys)
      const uint32_t v_off = split ? t * 8192 : 0;       // the key rows of V this issuer's O reads
      int g = 0;     // running K/V block count
      int nblk = 0;  // running block count of this issuer (phase of s_full / s_free / p_full / o_done)
      int nq = 0;    // items so far in which this issuer was active (phase of q_full / o_free)
      int s_trace = 0;  // S MMAs issued (trace slots of the first item)
      bool ok = true;
      // S_t = Q_t K_block^T.
      auto issue_s = [&](int st) {
        ATTN_TRACE(s_trace < 8, 20 + t * 16 + s_trace);
        ++s_trace;
        const uint32_t sk = smem_u32(sm + OFF_K + st * 16384);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16_ss(tmem + TMEM_S + t * 128, sdesc_k_sw128(sq + k * 32), sdesc_k_sw128(sk + k * 32), idesc_s,
                      k != 0 ? 1u : 0u);
        umma_commit(&s_full[t]);
      };
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
        const Item I = item_at(it, units, tpi);
        const int nt = item_tiles(I, T, tpi);
        if (!split && t >= nt) {  // this tile is past the end of the sequence for the item
          g += nkb;
          continue;
        }
        if (issues_s) {
          // S_t(0): Q_t and K/V block 0 landed, and the softmax warps have read
          // the previous item's last S_t.
          if (!(ok = mbar_wait(&q_full[t], nq & 1, status, kDevTimeoutAttn))) break;
          if (!(ok = mbar_wait(&kv_full[g % kKV], (g / kKV) & 1, status, kDevTimeoutAttn))) break;
          if (nblk > 0 && !(ok = mbar_wait(&s_free[t], (nblk - 1) & 1, status, kDevTimeoutAttn))) break;
          tc_fence_after();
          issue_s(g % kKV);
          if (nkb == 1) umma_commit(&q_empty[t]);
        }
        for (int j = 0; j < nkb && ok; ++j) {
          const int b = nblk + j;
          const int st = (g + j) % kKV;
          if (issues_s && j + 1 < nkb) {
            // S_t(j+1) as soon as K/V block j+1 landed and S_t(j) has been read out.
            const int gn = g + j + 1;
            if (!(ok = mbar_wait(&kv_full[gn % kKV], (gn / kKV) & 1, status, kDevTimeoutAttn))) break;
            if (!(ok = mbar_wait(&s_free[t], b & 1, status, kDevTimeoutAttn))) break;
            tc_fence_after();
            issue_s(gn % kKV);
            if (j + 2 == nkb) umma_commit(&q_empty[t]);
          }
          // O (+)= P(j) V(j) once P(j) is written (and, for the item's first
          // block, the previous item's O has been read out).
          if (!(ok = mbar_wait(&p_full[t], b & 1, status, kDevTimeoutAttn))) break;
          if (j == 0 && nq > 0 && !(ok = mbar_wait(&o_free[t], (nq - 1) & 1, status, kDevTimeoutAttn))) break;
          tc_fence_after();
          ATTN_TRACE(nq == 0 && j < 8, 52 + t * 16 + j);
          const uint32_t sv = smem_u32(sm + OFF_V + st * 16384) + v_off;
          for (int kk = 0; kk < o_steps; ++kk)
            umma_f16_ts(tmem + TMEM_O + t * 64, tmem + TMEM_P + t * 64 + kk * 8, sdesc_mn_sw128(sv + kk * 2048),
                        idesc_o, (j != 0 || kk != 0) ? 1u : 0u);
          umma_commit(&o_done[t]);
          umma_commit(&kv_empty[st]);
          if (!split && nt == 1) umma_commit(&kv_empty[st]);  // the absent tile's share of the stage release
        }
        nblk += nkb;
        ++nq;
        g += nkb;
      }
    }
    __syncwarp();
  } else {
    // ---- softmax + epilogue: warps 2..5 group 0, warps 6..9 group 1 ----
    const int wg = (warp - 2) / kSoftWarps;
    if (split) {
      softmax_role<64>(c, wg, warp & 3, lane);
    } else {
      softmax_role<128>(c, wg, warp & 3, lane);
    }
  }
  tc_fence_before();
  __syncthreads();
  ATTN_TRACE(threadIdx.x == 0, 181);
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
  static PerDeviceOnce configured;
  const cudaError_t e = configured.run(
      [] { return cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_A); });
  if (e != cudaSuccess) return e;
  // Ping-pong pairs of query tiles when there are enough of them to give every
  // SM work; single tiles otherwise (more CTAs, each with a shorter chain).
  const long long tiles = (T + kQ - 1) / kQ;
  const int tpi = static_cast<long long>(S) * 8 * ((tiles + 1) / 2) >= sms() ? 2 : 1;
  const long long items = static_cast<long long>(S) * 8 * ((tiles + tpi - 1) / tpi);
  const int grid = static_cast<int>(items < sms() ? items : sms());
  return launch_pdl(attn_tc_kernel, dim3(grid), dim3(kThreadsA), SMEM_A, st, tm, row_mask, out, S, T, tpi, status);
}

}  // namespace itts
