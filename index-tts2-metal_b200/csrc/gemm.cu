// tcgen05/TMEM GEMM with fused DiT-CFM epilogues (sm_100a).
//
// Persistent, warp-specialised: one CTA per SM walks the 128 x BN output
// tiles (static round-robin over the grid). Warp roles (352 threads):
//   warp 0 lane 0  : TMA producer of the A k-blocks (STAGES-deep ring)
//   warp 10 lane 0 : TMA producer of the B (weight) k-blocks; the first
//                    tile's are issued before the grid-dependency wait
//   warp 1         : allocates TMEM for two accumulator buffers; lane 0
//                    issues tcgen05.mma (M=128, N=BN, K=16) into buffer
//                    (tile & 1)
//   warps 2..9     : epilogue, one accumulator row per thread (TMEM lane
//                    quarter = warp % 4), two warps per quarter each owning
//                    half of the columns; drains buffer (tile & 1) while the
//                    MMA warp fills the other one.
// Outputs leave through a per-warp shared-memory stage: by TMA stores where
// the destination rows are contiguous, else by the lanes' coalesced stores.
// Replaces the reference's MPS GEMM calls and the elementwise kernels that
// followed them (bias prefill, RoPE rotate, silu_mul_split, add, wavenet gate,
// wavenet res/skip update, reflect pad, concat), metal/kernels.metal:131-239,
// 411-464, 820-841, 2390-2428; runtime/metal_context.mm:320-381.
#include <atomic>
#include <cstdio>
#include <mutex>

#include "gemm.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace itts {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 f16 = one 128-byte swizzle row
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter, each owning half of the columns
constexpr int kBWarp = 2 + kEpiWarps;            // issues the B (weight) TMA loads
constexpr int kThreads = 64 + 32 * kEpiWarps + 32;

// Phase timestamps for performance investigation: compiled out unless a
// harness defines ITTS_GEMM_TRACE and provides itts_gemm_trace_point(slot).
#ifdef ITTS_GEMM_TRACE
#define GEMM_TRACE(slot) itts_gemm_trace_point(slot)
#else
#define GEMM_TRACE(slot) ((void)0)
#endif

__host__ __device__ constexpr int pow2_cols(int c) { return c <= 32 ? 32 : c <= 64 ? 64 : c <= 128 ? 128 : c <= 256 ? 256 : 512; }

// Source row of the reflect padding used by the WaveNet k=5 convolution
// (tokenizer_tests.cpp:3836-3854): halo position j in {-2,-1,T,T+1}.
__device__ __forceinline__ int reflect_src(int j, int T) {
  int src = j;
#pragma unroll 1
  for (int it = 0; it < 8 && (src < 0 || src >= T); ++it) {
    if (src < 0) src = -src;
    if (src >= T) src = 2 * T - 2 - src;
  }
  return src;
}

__device__ __forceinline__ void u2f16(const uint32_t (&r)[16], float* v) {
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Epilogue helpers: the 256 epilogue threads (warps 2..9) share a named barrier.
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory"); }

// Per-tile column constants, 2*BN floats staged in shared memory: [0, BN) the
// bias of columns n0 .. n0+BN; [BN, 2 BN) for a folded-norm producer the
// column scale nrm_w * nrm_g, for the WaveNet gate the global condition of
// the tile's channels (a-part then b-part, BN/2 each), else 0. Entry i
// belongs to epilogue thread i mod 256; each thread loads its entries of the
// next tile into registers while the current tile is processed, so the
// global-load latency stays off the per-tile critical path.
__host__ __device__ constexpr int tile_const_floats(int bn) { return 2 * bn; }
__host__ __device__ constexpr int consts_per_thread(int bn) { return (2 * bn + 32 * kEpiWarps - 1) / (32 * kEpiWarps); }

template <int BN, int EPI>
__device__ __forceinline__ void load_tile_consts(const GemmArgs& args, int n0, int etid,
                                                 float (&r)[consts_per_thread(BN)]) {
#pragma unroll
  for (int k = 0; k < consts_per_thread(BN); ++k) {
    const int i = etid + k * 32 * kEpiWarps;
    float x = 0.0f;
    if (i < BN) {
      const int n = n0 + i;
      if (args.bias && n < args.N) x = args.bias[n];
    } else if (i < 2 * BN) {
      const int j = i - BN;
      if constexpr (EPI == kEpiF32) {
        const int n = n0 + j;
        if (args.nrm16 && n < args.N) x = args.nrm_w[n] * args.nrm_g[n];
      } else if constexpr (EPI == kEpiWnGate) {
        const int ch = (n0 >> 1) + (j < BN / 2 ? j : j - BN / 2);
        if (2 * ch < args.N) x = args.wn_cond[(j < BN / 2 ? 0 : 512) + ch];
      }
    }
    r[k] = x;
  }
}

template <int BN>
__device__ __forceinline__ void store_tile_consts(float* sconst, int etid, const float (&r)[consts_per_thread(BN)]) {
#pragma unroll
  for (int k = 0; k < consts_per_thread(BN); ++k) {
    const int i = etid + k * 32 * kEpiWarps;
    if (i < 2 * BN) sconst[i] = r[k];
  }
}

// ---- epilogue stores through a per-warp shared-memory stage ----
// Each epilogue warp owns 32 accumulator rows (one per lane). Values of a
// 32-column group are first written row-wise into a 32 x 32 fp32 stage (16-byte
// chunk j of row r at r * 8 + (j ^ (r & 7)): the 128-byte swizzle). With
// contiguous destination rows the block leaves through one TMA store (f32, or
// an f16 copy of the block in the 64-byte swizzle, stage_put16_h); otherwise
// it is read column-wise so that 8 (fp32) or 4 (f16) lanes cover one
// destination row segment and every store is a full 128 B / 64 B line piece,
// destination rows coming from the owning lane by shuffle (any per-row
// remapping: padded WaveNet rows, compact rows).
constexpr int kStageFloats = 32 * 32;  // per warp

__device__ __forceinline__ void stage_put16(float4* stg, int r, int c16, const float* v) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int j = (c16 >> 2) + k;
    stg[r * 8 + (j ^ (r & 7))] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
  }
}

__device__ __forceinline__ const void* shfl_ptr(const void* p, int src) {
  const unsigned long long u = reinterpret_cast<unsigned long long>(p);
  const unsigned lo = __shfl_sync(0xffffffffu, static_cast<unsigned>(u), src);
  const unsigned hi = __shfl_sync(0xffffffffu, static_cast<unsigned>(u >> 32), src);
  return reinterpret_cast<const void*>((static_cast<unsigned long long>(hi) << 32) | lo);
}

// Store staged columns [0, ncols) of all 32 rows as fp32 at (row_ptr + col0).
// `sj0` is the first 16-byte chunk (4 floats) of the staged columns.
__device__ __forceinline__ void flush_f32(const float4* stg, const float* my_row, int col0, int ncols, int lane,
                                          int sj0 = 0) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = i * 4 + (lane >> 3);
    const int j = lane & 7;
    float* p = const_cast<float*>(static_cast<const float*>(shfl_ptr(my_row, r)));
    if (p && j * 4 < ncols) *reinterpret_cast<float4*>(p + col0 + j * 4) = stg[r * 8 + ((sj0 + j) ^ (r & 7))];
  }
}

// f16 stage of a 32 x 32 block for a TMA store with the 64-byte swizzle: row r
// (64 B) holds 16-byte chunk c (columns 8c .. 8c + 7) at chunk position
// c ^ ((r >> 1) & 3). Writes columns c16 .. c16 + 15 of row r, rounded as
// flush_f16 rounds.
__device__ __forceinline__ void stage_put16_h(float4* stg, int r, int c16, const float* v) {
  uint4* row = reinterpret_cast<uint4*>(stg) + r * 4;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int c = (c16 >> 3) + k;
    union {
      __half2 h[4];
      uint4 u;
    } pk;
#pragma unroll
    for (int e = 0; e < 4; ++e) pk.h[e] = __floats2half2_rn(v[8 * k + 2 * e], v[8 * k + 2 * e + 1]);
    row[c ^ ((r >> 1) & 3)] = pk.u;
  }
}

// One TMA store of the warp's staged 32-row block (this lane's staged values
// made visible to the async proxy first); lane 0 issues and commits it.
__device__ __forceinline__ void stage_tma_store(const CUtensorMap* tmo, const float4* stg, int x, int y, int lane) {
  fence_proxy_async_shared();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmo, stg, x, y);
    bulk_commit();
  }
}

// Store staged columns [0, ncols) of all 32 rows as f16 at (row_ptr + col0).
__device__ __forceinline__ void flush_f16(const float4* stg, const __half* my_row, int col0, int ncols, int lane) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = i * 8 + (lane >> 2);
    const int j = lane & 3;
    __half* p = const_cast<__half*>(static_cast<const __half*>(shfl_ptr(my_row, r)));
    if (p && j * 8 < ncols) {
      const float4 a = stg[r * 8 + ((2 * j) ^ (r & 7))];
      const float4 b = stg[r * 8 + ((2 * j + 1) ^ (r & 7))];
      union {
        __half2 h[4];
        uint4 u;
      } pk;
      pk.h[0] = __floats2half2_rn(a.x, a.y);
      pk.h[1] = __floats2half2_rn(a.z, a.w);
      pk.h[2] = __floats2half2_rn(b.x, b.y);
      pk.h[3] = __floats2half2_rn(b.z, b.w);
      *reinterpret_cast<uint4*>(p + col0 + j * 8) = pk.u;
    }
  }
}

// As flush_f16, with staged column c multiplied by scale[c] first.
__device__ __forceinline__ void flush_f16_scaled(const float4* stg, const __half* my_row, int col0, int ncols,
                                                 int lane, const float* scale) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = i * 8 + (lane >> 2);
    const int j = lane & 3;
    __half* p = const_cast<__half*>(static_cast<const __half*>(shfl_ptr(my_row, r)));
    if (p && j * 8 < ncols) {
      const float4 a = stg[r * 8 + ((2 * j) ^ (r & 7))];
      const float4 b = stg[r * 8 + ((2 * j + 1) ^ (r & 7))];
      const float* sc = scale + j * 8;
      union {
        __half2 h[4];
        uint4 u;
      } pk;
      pk.h[0] = __floats2half2_rn(a.x * sc[0], a.y * sc[1]);
      pk.h[1] = __floats2half2_rn(a.z * sc[2], a.w * sc[3]);
      pk.h[2] = __floats2half2_rn(b.x * sc[4], b.y * sc[5]);
      pk.h[3] = __floats2half2_rn(b.z * sc[6], b.w * sc[7]);
      *reinterpret_cast<uint4*>(p + col0 + j * 8) = pk.u;
    }
  }
}

// Row scale of a folded-norm consumer: 1/sqrt(mean of squares + 1e-5) from the
// producer's per-group partial sums (summed in group order), or 1.
// The 16 partials of the usual 512-wide norm are all loaded before the first
// add (one round of load latency instead of 16), then summed in group order.
__device__ __forceinline__ float folded_row_scale(const GemmArgs& args, int m, bool row_ok) {
  if (!args.ss_in || !row_ok) return 1.0f;
  const float* src = args.ss_in + m;
  const size_t ld = static_cast<size_t>(args.ss_ld);
  float t = 0.0f;
  if (args.ss_parts == 16) {
    float v[16];
#pragma unroll
    for (int p = 0; p < 16; ++p) v[p] = src[p * ld];
#pragma unroll
    for (int p = 0; p < 16; ++p) t += v[p];
  } else {
    for (int p = 0; p < args.ss_parts; ++p) t += src[p * ld];
  }
  return 1.0f / sqrtf(t / static_cast<float>(args.ss_n) + 1e-5f);
}

// Reflect-halo copies of one WaveNet row (the interior row itself goes through
// the coalesced path): rows t in {1, 2, T-2, T-3} (and more for tiny T) are
// mirrored into the 2 halo rows on each side of their sequence. NV = 16 or 32 values.
template <int NV>
__device__ __forceinline__ void write_halos(__half* xp, int s, int t, int T, int col, const float* v) {
  if (t > 2 && t < T - 3) return;
  __half* base = xp + static_cast<size_t>(s) * (T + 4) * 512;
  const int halo[4] = {-2, -1, T, T + 1};
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    if (reflect_src(halo[h], T) == t) {
#pragma unroll
      for (int k = 0; k < NV; k += 16) store_h16(base + static_cast<size_t>(halo[h] + 2) * 512 + col + k, v + k);
    }
  }
}

// Epilogue of one 128 x BN tile for this thread's row and column half.
// `taddr` addresses TMEM lane (quarter*32) at the tile's accumulator buffer.
// Row-local operands (residual, RoPE pairs, WaveNet state) of the first chunk
// are fetched before waiting for the accumulator and later ones one chunk
// ahead; TMEM loads are double-buffered. Returns false if the accumulator
// wait timed out.
template <int BN, int EPI>
__device__ __forceinline__ bool epilogue_tile(const GemmArgs& args, const CUtensorMap* tmo, int m0, int n0, int row,
                                              int half, uint32_t taddr, const float* sconst, float4* stg,
                                              uint64_t* acc_bar, uint32_t parity) {
  const int lane = row & 31;
  const int m = m0 + row;
  const int T = args.seq_T;
  if constexpr (EPI == kEpiSwiGLU || EPI == kEpiWnGate || EPI == kEpiWnResSkip) {
    static_assert(BN % 128 == 0, "paired epilogues need 128-column slabs");
    constexpr int NCH = (BN / 128) * 4;  // chunks of 16 a-columns (+16 b-columns)
    const int q_begin = half * (NCH / 2), q_end = q_begin + NCH / 2;
    bool row_ok = m < args.M;
    int r = m;  // compact row
    int s = 0, t = 0;
    if constexpr (EPI == kEpiWnGate) {
      s = m / (T + 4);
      const int j = m - s * (T + 4) - 2;
      row_ok = row_ok && j >= 0 && j < T;
      r = s * T + j;
    } else if constexpr (EPI == kEpiWnResSkip) {
      s = m / T;
      t = m - s * T;
    }
    float msk = 1.0f;
    const __half* out16_row = nullptr;  // SwiGLU / gate output row
    __half* xp_row = nullptr;           // res/skip: interior WaveNet row
    float* acc_row = nullptr;           // res/skip: skip accumulator row
    if (row_ok) {
      if constexpr (EPI == kEpiWnResSkip) {
        msk = args.row_mask[r];
        xp_row = args.wn_xp + (static_cast<size_t>(s) * (T + 4) + t + 2) * 512;
        acc_row = args.wn_acc + static_cast<size_t>(r) * 512;
      } else {
        out16_row = args.out16 + static_cast<size_t>(r) * args.ld16;
      }
    }
    uint4 xo_cur[2], xo_nxt[2];
    float ac_cur[16], ac_nxt[16];
    auto fetch = [&](int q, uint4 (&xo)[2], float (&ac)[16]) {
      if constexpr (EPI == kEpiWnResSkip) {
        const int ch = (n0 >> 1) + (q >> 2) * 64 + (q & 3) * 16;
        if (row_ok) {
          const uint4* xs = reinterpret_cast<const uint4*>(xp_row + ch);
          xo[0] = xs[0];
          xo[1] = xs[1];
          if (!args.wn_first) load_f32x16(acc_row + ch, ac);
        }
      }
    };
    auto tcol = [](int q) { return (q >> 2) * 128 + (q & 3) * 16; };  // tile column of the a-chunk
    fetch(q_begin, xo_cur, ac_cur);
    float rs = 1.0f;
    if constexpr (EPI == kEpiSwiGLU) rs = folded_row_scale(args, m, row_ok);
    if (!mbar_wait(acc_bar, parity, args.status, kDevTimeoutAccum)) return false;
    tc_fence_after();
    uint32_t ta[16], tb[16], na_[16], nb_[16];
    tmem_ld16_async(taddr + tcol(q_begin), ta);
    tmem_ld16_async(taddr + tcol(q_begin) + 64, tb);
    tmem_wait_ld();
    reg_fence16(ta);
    reg_fence16(tb);
    // Chunks per store group: two for single-output epilogues, one for the
    // res/skip update (x and skip values share the stage).
    constexpr int G = EPI == kEpiWnResSkip ? 1 : 2;
    float xg[16 * G], bg[16];
    // SwiGLU: every group is 32 output channels of contiguous rows.
    const bool t16 = EPI == kEpiSwiGLU && args.tma_o16 && m0 + (row & ~31) < args.M;
#pragma unroll 1
    for (int q2 = q_begin; q2 < q_end; q2 += G) {
      if (t16) {  // a TMA store of the previous group may still be reading the stage
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const int q = q2 + h;
        const int ca = tcol(q);
        const int ci = (q >> 2) * 64 + (q & 3) * 16;  // channel index inside the tile
        const bool more = q + 1 < q_end;
        if (more) {
          tmem_ld16_async(taddr + tcol(q + 1), na_);
          tmem_ld16_async(taddr + tcol(q + 1) + 64, nb_);
          fetch(q + 1, xo_nxt, ac_nxt);
        }
        float a[16], b[16];
        u2f16(ta, a);
        u2f16(tb, b);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          a[e] = fmaf(a[e], rs, sconst[ca + e]);
          b[e] = fmaf(b[e], rs, sconst[ca + 64 + e]);
        }
        if constexpr (EPI == kEpiSwiGLU) {
#pragma unroll
          for (int e = 0; e < 16; ++e) xg[h * 16 + e] = silu_f(a[e]) * b[e];
        } else if constexpr (EPI == kEpiWnGate) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float ga = a[e] + sconst[BN + ci + e];
            const float gb = b[e] + sconst[BN + BN / 2 + ci + e];
            xg[h * 16 + e] = tanhf(ga) * sigmoid_f(gb);
          }
        } else {  // kEpiWnResSkip
          union {
            uint4 u[2];
            __half2 hh[8];
          } pk;
          pk.u[0] = xo_cur[0];
          pk.u[1] = xo_cur[1];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float2 f = __half22float2(pk.hh[e]);
            xg[h * 16 + 2 * e] = (f.x + a[2 * e]) * msk;
            xg[h * 16 + 2 * e + 1] = (f.y + a[2 * e + 1]) * msk;
          }
#pragma unroll
          for (int e = 0; e < 16; ++e) bg[e] = args.wn_first ? b[e] : b[e] + ac_cur[e];
          xo_cur[0] = xo_nxt[0];
          xo_cur[1] = xo_nxt[1];
#pragma unroll
          for (int e = 0; e < 16; ++e) ac_cur[e] = ac_nxt[e];
        }
        if (t16) {
          stage_put16_h(stg, lane, h * 16, xg + h * 16);
        } else {
          stage_put16(stg, lane, h * 16, xg + h * 16);
        }
        if constexpr (EPI == kEpiWnResSkip) stage_put16(stg, lane, 16, bg);
        if (more) {
          tmem_wait_ld();
          reg_fence16(na_);
          reg_fence16(nb_);
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            ta[e] = na_[e];
            tb[e] = nb_[e];
          }
        }
      }
      const int ch0 = (n0 >> 1) + (q2 >> 2) * 64 + (q2 & 3) * 16;
      __syncwarp();
      if constexpr (EPI == kEpiWnResSkip) {
        flush_f16(stg, xp_row, ch0, 16, lane);
        if (row_ok) write_halos<16>(args.wn_xp, s, t, T, ch0, xg);
        flush_f32(stg, acc_row, ch0, 16, lane, 4);
      } else if (t16) {
        stage_tma_store(tmo, stg, ch0, m0 + (row & ~31), lane);
      } else {
        flush_f16(stg, out16_row, ch0, 32, lane);
      }
      __syncwarp();
    }
  } else {
    constexpr int NCH = BN / 16;
    constexpr int SPLIT = (((NCH + 1) / 2) + 1) & ~1;  // even chunk count of the first half
    const int c_begin = half ? SPLIT : 0;
    const int c_end = half ? NCH : (SPLIT < NCH ? SPLIT : NCH);
    bool row_ok = m < args.M;
    int s = 0, t = 0;
    if constexpr (EPI == kEpiQKV || EPI == kEpiConv1Res) {
      s = m / T;
      t = m - s * T;
    }
    int mo = m;  // output row
    if constexpr (EPI == kEpiF32) {
      if (args.pad_rows) {
        const int sp = m / (T + 4);
        const int j = m - sp * (T + 4) - 2;
        row_ok = row_ok && j >= 0 && j < T;
        mo = sp * T + j;
      }
    }
    // Destination rows (null when the row is out of range).
    const void* d0 = nullptr;  // primary
    const void* d1 = nullptr;  // F32: f16 copy; Conv1Res: res projection row
    const void* d2 = nullptr;  // F32: folded-norm f16 operand row
    if (row_ok) {
      if constexpr (EPI == kEpiF16 || EPI == kEpiQKV) {
        d0 = args.out16 + static_cast<size_t>(m) * args.ld16;
      } else if constexpr (EPI == kEpiF32) {
        d0 = args.out32 + static_cast<size_t>(mo) * args.ld32;
        if (args.out16) d1 = args.out16 + static_cast<size_t>(mo) * args.ld16;
        if (args.nrm16) d2 = args.nrm16 + static_cast<size_t>(mo) * args.ldn;
      } else if constexpr (EPI == kEpiWnLast) {
        d0 = args.out32 + static_cast<size_t>(m) * args.ld32;
      } else if constexpr (EPI == kEpiConv1Res) {
        d0 = args.wn_xp + (static_cast<size_t>(s) * (T + 4) + t + 2) * 512;
        d1 = args.out32 + static_cast<size_t>(m) * args.ld32;
      }
    }
    // Row-local operands: residual (F32), RoPE pairs (QKV), skip accumulator +
    // res projection (WnLast).
    float x0_cur[16], x1_cur[16], x0_nxt[16], x1_nxt[16];
    auto fetch = [&](int c, float (&x0)[16], float (&x1)[16]) {
      const int n = n0 + c * 16;
      if (!row_ok || n >= args.N) return;
      if constexpr (EPI == kEpiF32) {
        if (args.resid32) load_f32x16(args.resid32 + static_cast<size_t>(mo) * args.ldr + n, x0);
      } else if constexpr (EPI == kEpiQKV) {
        if (n < 1024) {
          // Pairs p0..p0+7 of this row: one 8-byte load per pair, coalesced
          // across the warp's consecutive rows.
          const float2* rp = args.rope + static_cast<size_t>((n & 63) >> 1) * T + t;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float2 cs = rp[static_cast<size_t>(e) * T];
            x0[2 * e] = cs.x;
            x0[2 * e + 1] = cs.y;
          }
        }
      } else if constexpr (EPI == kEpiWnLast) {
        load_f32x16(args.wn_acc + static_cast<size_t>(m) * 512 + n, x0);
        load_f32x16(args.wn_res + static_cast<size_t>(m) * 512 + n, x1);
      }
    };
    float msk = 1.0f;
    if constexpr (EPI == kEpiWnLast) msk = row_ok ? args.row_mask[m] : 0.0f;
    fetch(c_begin, x0_cur, x1_cur);
    // With two chunks per thread (F32, BN = 64) both residual chunks are in
    // flight before the accumulator wait.
    constexpr bool kPre2 = EPI == kEpiF32 && BN == 64;
    if constexpr (kPre2) fetch(c_begin + 1, x0_nxt, x1_nxt);
    float rs = 1.0f;
    if constexpr (EPI == kEpiQKV) rs = folded_row_scale(args, m, row_ok);
    if (threadIdx.x == 64 && parity == 0) GEMM_TRACE(20);
    if (!mbar_wait(acc_bar, parity, args.status, kDevTimeoutAccum)) return false;
    tc_fence_after();
    if (threadIdx.x == 64 && parity == 0) GEMM_TRACE(21);
    uint32_t tc[16], tn[16];
    if (c_begin < c_end) {  // (a half of a 32-wide tile has no columns: its TMEM lies outside the allocation)
      tmem_ld16_async(taddr + c_begin * 16, tc);
      tmem_wait_ld();
      reg_fence16(tc);
    }
    if (threadIdx.x == 64 && parity == 0) GEMM_TRACE(22);
    float vg[32];
#pragma unroll 1
    for (int cp = c_begin; cp < c_end; cp += 2) {
      float sc = 0.0f;  // folded-norm producer: sum of squares over this 32-column group
      // A TMA store of the previous group may still be reading the stage.
      if ((EPI == kEpiF32 && args.tma_o32) || ((EPI == kEpiQKV || EPI == kEpiF16) && args.tma_o16)) {
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
      }
      // QKV / F16: a full 32-column group of in-range rows is staged as f16
      // for one TMA store; other groups go through the fp32 stage.
      const bool t16 = (EPI == kEpiQKV || EPI == kEpiF16) && args.tma_o16 && cp + 1 < c_end &&
                       n0 + cp * 16 < args.N && m0 + (row & ~31) < args.M;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = cp + h;
        if (c < c_end) {
          const int n = n0 + c * 16;
          const bool more = c + 1 < c_end;
          if (more) {
            tmem_ld16_async(taddr + (c + 1) * 16, tn);
            if constexpr (!kPre2) fetch(c + 1, x0_nxt, x1_nxt);
          }
          float* v = vg + h * 16;
          u2f16(tc, v);
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = fmaf(v[e], rs, sconst[c * 16 + e]);
          if constexpr (EPI == kEpiF32) {
            if (args.resid32) {
#pragma unroll
              for (int e = 0; e < 16; ++e) v[e] += x0_cur[e];
            }
            if (args.ss_out && n < args.N) {
#pragma unroll
              for (int e = 0; e < 16; ++e) sc = fmaf(v[e], v[e], sc);
            }
          } else if constexpr (EPI == kEpiQKV) {
            if (n < 1024) {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float cs = x0_cur[2 * e], sn = x0_cur[2 * e + 1];
                const float xa = v[2 * e], xb = v[2 * e + 1];
                v[2 * e] = xa * cs - xb * sn;
                v[2 * e + 1] = xb * cs + xa * sn;
              }
              if (n < 512) {
#pragma unroll
                for (int e = 0; e < 16; ++e) v[e] *= 0.125f;
              }
            }
          } else if constexpr (EPI == kEpiWnLast) {
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] = (x0_cur[e] + v[e]) * msk + x1_cur[e];
          }
          if (t16) {
            stage_put16_h(stg, lane, h * 16, v);
          } else {
            stage_put16(stg, lane, h * 16, v);
          }
          if (more) {
            tmem_wait_ld();
            reg_fence16(tn);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              tc[e] = tn[e];
              x0_cur[e] = x0_nxt[e];
              x1_cur[e] = x1_nxt[e];
            }
          }
        }
      }
      // Flush the group (two chunks, or one at the end).
      const int ng = n0 + cp * 16;
      if constexpr (EPI == kEpiF32) {
        // n0 and the first chunk of each half are multiples of 32 columns for
        // every producer tile width (the host accepts only BN % 32 == 0).
        if (args.ss_out && row_ok && ng < args.N) args.ss_out[static_cast<size_t>(ng >> 5) * args.ss_ld + mo] = sc;
      }
      int ncols = (cp + 1 < c_end) ? 32 : 16;
      if (ng + ncols > args.N) ncols = args.N > ng ? args.N - ng : 0;
      __syncwarp();
      const bool tr = threadIdx.x == 64 && parity == 0 && cp == c_begin;
      if (tr) GEMM_TRACE(24);
      if constexpr (EPI == kEpiF16 || EPI == kEpiQKV) {
        if (t16) {
          stage_tma_store(tmo, stg, ng, m0 + (row & ~31), lane);
        } else {
          flush_f16(stg, static_cast<const __half*>(d0), ng, ncols, lane);
        }
      } else if constexpr (EPI == kEpiF32) {
        // A full 32-column group leaves through one TMA store of the stage (its
        // layout is the 128-byte swizzle of the tensor map; rows >= M and
        // columns >= N are not written); a 16-column remainder through the
        // lanes' coalesced stores.
        // (out32 may be null when only the f16 outputs are read downstream.)
        if (args.tma_o32 && cp + 1 < c_end && ng < args.N && m0 + (row & ~31) < args.M) {
          stage_tma_store(tmo, stg, ng, m0 + (row & ~31), lane);
        } else if (args.out32) {
          flush_f32(stg, static_cast<const float*>(d0), ng, ncols, lane);
        }
        if (tr) GEMM_TRACE(25);
        if (args.out16) flush_f16(stg, static_cast<const __half*>(d1), ng, ncols, lane);
        if (tr) GEMM_TRACE(26);
        if (args.nrm16) flush_f16_scaled(stg, static_cast<const __half*>(d2), ng, ncols, lane, sconst + BN + (ng - n0));
      } else if constexpr (EPI == kEpiWnLast) {
        flush_f32(stg, static_cast<const float*>(d0), ng, ncols, lane);
      } else if constexpr (EPI == kEpiConv1Res) {
        if (ng < 512) {
          flush_f16(stg, static_cast<const __half*>(d0), ng, ncols, lane);
          if (row_ok && ncols == 32) write_halos<32>(args.wn_xp, s, t, T, ng, vg);
          if (row_ok && ncols == 16) write_halos<16>(args.wn_xp, s, t, T, ng, vg);
        } else {
          flush_f32(stg, static_cast<const float*>(d1), ng - 512, ncols, lane);
        }
      }
      __syncwarp();
      if (threadIdx.x == 64 && parity == 0 && cp == c_begin) GEMM_TRACE(23);
    }
  }
  return true;
}

// PAIR: the CTA-pair form (cluster of 2, tcgen05 cta_group::2). A work unit
// is a 256 x BN tile; CTA rank r of the pair holds A rows [128 r, 128 r + 128)
// and B rows [BN/2 r, BN/2 r + BN/2) of it in its own shared memory, and its
// 128 accumulator rows in its own TMEM. The leader (rank 0) issues the M=256
// MMAs and every load of both CTAs completes on the leader's full barrier;
// the leader's commits release both CTAs' stages and accumulators. Each CTA
// ingests 16 KB + BN/2 x 128 B per k-block instead of 16 KB + BN x 128 B.
// No TMA multicast is involved.
template <int BN, int STAGES, int EPI, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
                   const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmO,
                   const GemmArgs args) {
  constexpr int KBOX = gemm_kbox(BN);      // k-blocks per stage (one TMA box per operand)
  constexpr int BNL = PAIR ? BN / 2 : BN;  // B rows held by this CTA
  constexpr int A_KB = kBM * kBK * 2;       // one 128 x 64 k-block of A
  constexpr int B_KB = BNL * kBK * 2;       // one BNL x 64 k-block of B
  constexpr int A_BYTES = KBOX * A_KB;
  constexpr int B_BYTES = KBOX * B_KB;
  constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr int UNIT_M = PAIR ? 2 * kBM : kBM;  // rows of one work unit
  constexpr int ACC_STRIDE = pow2_cols(BN);  // columns between the two accumulator buffers
  constexpr uint32_t TMEM_COLS = pow2_cols(2 * ACC_STRIDE);
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N");
  static_assert(!PAIR || BN % 32 == 0, "pair tiles split B in halves of 16-row multiples");
  static_assert(2 * ACC_STRIDE <= 512, "two accumulator buffers must fit TMEM");
  static_assert(STAGE_BYTES % 1024 == 0 && (kEpiWarps * kStageFloats * 4) % 1024 == 0,
                "every pipeline stage starts on a 1024-byte boundary (128-byte swizzle)");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // [epilogue stages: kEpiWarps x 4 KB, 1024-byte aligned as the 128-byte
  //  swizzle of the TMA stores requires][pipeline stages][barriers][constants]
  // (measured: 0.6% faster at configuration 2 than the epilogue stages after
  // the pipeline stages; equal at the batch size)
  float4* stage_all = reinterpret_cast<float4*>(smem);  // kEpiWarps x 32 x 32 fp32
  smem += kEpiWarps * kStageFloats * 4;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* acc_full = empty_bar + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  float* sconst = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES + 256);  // [tile_const_floats(BN)]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int unit0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int units = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int num_sb = (args.num_kb + KBOX - 1) / KBOX;  // stages per tile (a missing k-block reads zeros)
  const int n_tiles = (args.N + BN - 1) / BN;
  const int num_tiles = ((args.M + UNIT_M - 1) / UNIT_M) * n_tiles;
  // Barrier addresses in the cluster window: loads of both CTAs complete on
  // the leader's full barriers; epilogues release the leader's accumulators.
  auto full_addr = [&](int s) -> uint32_t { return PAIR ? mapa_shared(&full_bar[s], 0) : smem_u32(&full_bar[s]); };

  if (threadIdx.x == 0) GEMM_TRACE(0);
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], (PAIR ? 2 : 1) * kEpiWarps);  // one arrival per epilogue warp (of both CTAs)
    }
    fence_barrier_init();
    fence_proxy_async_shared();
    prefetch_tmap(&tmA0);
    if (args.a_mode == kASplit) prefetch_tmap(&tmA1);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR) {
    cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA signal
  } else {
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Two TMA issuers: warp 0 loads A and (in the leader) arrives on each full
  // barrier with the whole stage byte count of the unit; warp kBWarp loads B
  // (its bytes complete the same transaction count, possibly before the
  // arrive). B is always weights, which no kernel of the stream writes, so the
  // first tile's B loads start before the wait for the previous kernel and
  // overlap its tail.
  const int num_pre = num_sb < STAGES ? num_sb : STAGES;
  auto load_b = [&](int s, int n0, int kb) {
    uint8_t* dst = smem + s * STAGE_BYTES + A_BYTES;
    if constexpr (PAIR) {
      tma_load_3d_pair(dst, &tmB, full_addr(s), 0, n0 + static_cast<int>(rank) * BNL, kb);
    } else {
      tma_load_3d(dst, &tmB, &full_bar[s], 0, n0, kb);
    }
  };
  if (warp == kBWarp && lane == 0 && unit0 < num_tiles) {
    const int n0 = (unit0 % n_tiles) * BN;
    for (int sbk = 0; sbk < num_pre; ++sbk) load_b(sbk, n0, sbk * KBOX);
  }
  // Everything below reads or writes memory of the previous kernel in the stream.
  griddep_wait();
  griddep_launch();
  if (threadIdx.x == 0) GEMM_TRACE(1);

  if (warp == 0) {
    if (lane == 0) {
      // ---- A producer ----
      int it = 0;
      bool ok = true;
      for (int tile = unit0; tile < num_tiles && ok; tile += units) {
        const int m0 = (tile / n_tiles) * UNIT_M + static_cast<int>(rank) * kBM;
        for (int sbk = 0; sbk < num_sb; ++sbk, ++it) {
          const int kb = sbk * KBOX;  // first k-block of the stage (kb_split and kb_per_tap are multiples of KBOX)
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (it == 0) GEMM_TRACE(18);
          const bool pre = it < num_pre;  // a fresh stage: nothing to wait for
          if (!pre && !mbar_wait(&empty_bar[s], ph ^ 1, args.status, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (it == 0) GEMM_TRACE(19);
          uint8_t* sa = smem + s * STAGE_BYTES;
          if (it == 0) GEMM_TRACE(8);
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[s], (PAIR ? 2 : 1) * STAGE_BYTES);
          // Each branch names its tensor map directly (a runtime-selected
          // pointer to a grid-constant parameter costs a local copy).
          if (args.a_mode == kAConv) {
            const int tap = kb / args.kb_per_tap;
            const int kc = kb - tap * args.kb_per_tap;
            const int row = m0 + tap * args.conv_dil + args.conv_off;
            if constexpr (PAIR) {
              tma_load_3d_pair(sa, &tmA0, full_addr(s), 0, row, kc);
            } else {
              tma_load_3d(sa, &tmA0, &full_bar[s], 0, row, kc);
            }
          } else if (args.a_mode == kASplit && kb >= args.kb_split) {
            if constexpr (PAIR) {
              tma_load_3d_pair(sa, &tmA1, full_addr(s), 0, m0, kb - args.kb_split);
            } else {
              tma_load_3d(sa, &tmA1, &full_bar[s], 0, m0, kb - args.kb_split);
            }
          } else {
            if constexpr (PAIR) {
              tma_load_3d_pair(sa, &tmA0, full_addr(s), 0, m0, kb);
            } else {
              tma_load_3d(sa, &tmA0, &full_bar[s], 0, m0, kb);
            }
          }
          if (it == 0) GEMM_TRACE(2);
        }
      }
    }
    __syncwarp();
  } else if (warp == kBWarp) {
    if (lane == 0) {
      // ---- B (weight) producer: stages after the pre-issued ones ----
      int it = 0;
      bool ok = true;
      for (int tile = unit0; tile < num_tiles && ok; tile += units) {
        const int n0 = (tile % n_tiles) * BN;
        for (int sbk = 0; sbk < num_sb; ++sbk, ++it) {
          if (it < num_pre) continue;
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty_bar[s], ph ^ 1, args.status, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          load_b(s, n0, sbk * KBOX);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---- MMA issuer (the leader of a pair) ----
      constexpr uint32_t idesc = idesc_f16_f32(UNIT_M, BN);
      int it = 0, local = 0;
      bool ok = true;
      for (int tile = unit0; tile < num_tiles && ok; tile += units, ++local) {
        const int a = local & 1;
        if (!mbar_wait(&acc_empty[a], ((local >> 1) & 1) ^ 1, args.status, kDevTimeoutAccum)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(a * ACC_STRIDE);
        for (int sbk = 0; sbk < num_sb; ++sbk, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full_bar[s], ph, args.status, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (it == 0) GEMM_TRACE(3);
          const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int j = 0; j < KBOX; ++j) {
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {
              const uint64_t ad = sdesc_k_sw128(sa + j * A_KB + k * 32);
              const uint64_t bd = sdesc_k_sw128(sb + j * B_KB + k * 32);
              const uint32_t acc = (sbk | j | k) != 0 ? 1u : 0u;
              if constexpr (PAIR) {
                umma_f16_ss_pair(d, ad, bd, idesc, acc);
              } else {
                umma_f16_ss(d, ad, bd, idesc, acc);
              }
            }
          }
          if constexpr (PAIR) {
            umma_commit_pair(mapa_shared(&empty_bar[s], 0));
            umma_commit_pair(mapa_shared(&empty_bar[s], 1));
          } else {
            umma_commit(&empty_bar[s]);
          }
        }
        if constexpr (PAIR) {
          umma_commit_pair(mapa_shared(&acc_full[a], 0));
          umma_commit_pair(mapa_shared(&acc_full[a], 1));
        } else {
          umma_commit(&acc_full[a]);
        }
        if (local == 0) GEMM_TRACE(4);
      }
    }
    __syncwarp();
  } else {
    // ---- epilogue: warps 2..(2 + kEpiWarps) ----
    const int quarter = warp & 3;
    const int half = (warp - 2) / 4;
    const int row = quarter * 32 + lane;
    const int etid = threadIdx.x - 64;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    int local = 0;
    float cst[consts_per_thread(BN)];
    if (unit0 < num_tiles) load_tile_consts<BN, EPI>(args, (unit0 % n_tiles) * BN, etid, cst);
    for (int tile = unit0; tile < num_tiles; tile += units, ++local) {
      const int a = local & 1;
      const int m0 = (tile / n_tiles) * UNIT_M + static_cast<int>(rank) * kBM;
      const int n0 = (tile % n_tiles) * BN;
      epi_bar();  // every epilogue thread is done with the previous tile's constants
      store_tile_consts<BN>(sconst, etid, cst);
      epi_bar();
      if (tile + units < num_tiles) load_tile_consts<BN, EPI>(args, ((tile + units) % n_tiles) * BN, etid, cst);
      const bool ok = epilogue_tile<BN, EPI>(args, &tmO, m0, n0, row, half,
                                             tmem_base + lane_off + static_cast<uint32_t>(a * ACC_STRIDE), sconst,
                                             stage_all + (warp - 2) * (kStageFloats / 4), &acc_full[a],
                                             (local >> 1) & 1);
      if (!ok) break;
      if (local == 0 && warp == 2 && lane == 0) GEMM_TRACE(5);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR) {
          mbar_arrive_cluster(mapa_shared(&acc_empty[a], 0));
        } else {
          mbar_arrive(&acc_empty[a]);
        }
      }
      if (local == 0 && warp == 2 && lane == 0) GEMM_TRACE(6);
    }
    // This warp's TMA stores complete before it leaves.
    if ((args.tma_o32 || args.tma_o16) && lane == 0) bulk_wait_all();
    __syncwarp();
  }
  if constexpr (PAIR) {
    // Neither CTA frees its TMEM (or exits, which would drop the barriers the
    // other one signals) before both are done.
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
  } else {
    __syncthreads();
  }
  if (lane == 0 && warp < kBWarp) GEMM_TRACE(warp == 0 ? 7 : 8 + warp);
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) {
      tmem_dealloc_pair(tmem_base, TMEM_COLS);
    } else {
      tmem_dealloc(tmem_base, TMEM_COLS);
    }
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int sm_count() {
  static int n = [] {
    int dev = 0, v = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v > 0 ? v : 148;
  }();
  return n;
}

template <int BN, int EPI, bool PAIR>
cudaError_t launch_t(const GemmLaunch& g, cudaStream_t stream) {
  constexpr int STAGES = gemm_stages(BN, PAIR);
  auto kern = gemm_tc_kernel<BN, STAGES, EPI, PAIR>;
  const size_t smem = gemm_smem_bytes(BN, STAGES, PAIR);
  // The shared-memory opt-in is set once per device for each instantiation.
  static PerDeviceOnce configured;
  cudaError_t e = configured.run(
      [&] { return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)); });
  if (e != cudaSuccess) return e;
  const int unit_m = PAIR ? 2 * kBM : kBM;
  const int units = ((g.args.M + unit_m - 1) / unit_m) * ((g.args.N + BN - 1) / BN);
  if constexpr (PAIR) {
    const int slots = sm_count() / 2;
    const int clusters = units < slots ? units : slots;
    return launch_pdl_cluster(kern, dim3(2 * clusters), dim3(kThreads), smem, stream, 2u, g.tmA0, g.tmA1, g.tmB,
                              g.tmO, g.args);
  } else {
    const int grid = units < sm_count() ? units : sm_count();
    return launch_pdl(kern, dim3(grid), dim3(kThreads), smem, stream, g.tmA0, g.tmA1, g.tmB, g.tmO, g.args);
  }
}

template <int BN, bool PAIR>
cudaError_t launch_epi(const GemmLaunch& g, cudaStream_t stream) {
  if constexpr (BN < 64) {  // narrow tiles: plain epilogues only
    switch (g.args.epi) {
      case kEpiF16: return launch_t<BN, kEpiF16, PAIR>(g, stream);
      case kEpiF32: return launch_t<BN, kEpiF32, PAIR>(g, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (g.args.epi) {
    case kEpiF16: return launch_t<BN, kEpiF16, PAIR>(g, stream);
    case kEpiF32: return launch_t<BN, kEpiF32, PAIR>(g, stream);
    case kEpiQKV: return launch_t<BN, kEpiQKV, PAIR>(g, stream);
    case kEpiWnLast: return launch_t<BN, kEpiWnLast, PAIR>(g, stream);
    case kEpiConv1Res: return launch_t<BN, kEpiConv1Res, PAIR>(g, stream);
    default: break;
  }
  if constexpr (BN % 128 == 0) {
    switch (g.args.epi) {
      case kEpiSwiGLU: return launch_t<BN, kEpiSwiGLU, PAIR>(g, stream);
      case kEpiWnGate: return launch_t<BN, kEpiWnGate, PAIR>(g, stream);
      case kEpiWnResSkip: return launch_t<BN, kEpiWnResSkip, PAIR>(g, stream);
      default: break;
    }
  }
  return cudaErrorInvalidValue;
}

}  // namespace

size_t gemm_smem_bytes(int bn, int stages, bool pair) {
  return 1024 /*alignment slack*/ + static_cast<size_t>(stages) * gemm_stage_bytes(bn, pair) + 256 /*barriers*/ +
         static_cast<size_t>(tile_const_floats(bn)) * 4 + kEpiWarps * kStageFloats * 4 /*epilogue stages*/;
}

GemmPick gemm_pick(int M, int N, bool paired_epilogue) {
  // The CTA-pair form ingests fewer bytes per CTA but measured slower on every
  // DiT shape (1600 x 512 x 512: 7.99 vs 7.48 us; 1600 x 1536 x 512: 10.8 vs
  // 9.4 us; 102400 x 3072 x 512: 353 vs 337 us), so the picker keeps to the
  // single-CTA form; the pair form stays selectable per launch.
  const int sms = sm_count();
  GemmPick best{0, 0};
  double best_cost = 0.0;
  for (int pair = 0; pair >= 0; --pair) {
    for (int bn : {256, 192, 128, 64}) {
      if (bn == 192 && (pair || paired_epilogue)) continue;
      if (paired_epilogue && bn % 128) continue;
      if (N % bn && bn > N) continue;
      const int unit_m = pair ? 256 : 128;
      const int units = ((M + unit_m - 1) / unit_m) * ((N + bn - 1) / bn);
      const int slots = pair ? sms / 2 : sms;
      const int waves = (units + slots - 1) / slots;
      // Per-tile cost in units that track the measured tile times (A share 64
      // plus the B rows a CTA holds): e.g. 1600 x 3072 at bn 128 (3 waves)
      // beats bn 256 (2 waves).
      const double cost = static_cast<double>(waves) * ((pair ? bn / 2 : bn) + 64);
      if (best.bn == 0 || cost < best_cost - 1e-9) {
        best = GemmPick{bn, pair};
        best_cost = cost;
      }
    }
  }
  return best;
}

bool make_tmap_f16(CUtensorMap* tm, const void* base, uint64_t cols, uint64_t rows, uint64_t ld_elems,
                   uint32_t box_rows, uint32_t kbox) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || !base || cols % kBK != 0 || cols > ld_elems || kbox < 1) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld_elems * 2) % 16 != 0) return false;
  // {64 columns of a k-block, rows, k-blocks}; the k-block stride (128 B) is
  // smaller than the row stride, so one box gathers kbox k-blocks of box_rows rows.
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kBK), rows, cols / kBK};
  cuuint64_t strides[2] = {ld_elems * 2, static_cast<cuuint64_t>(kBK) * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(kBK), box_rows, kbox};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Tensor map of an fp32 output [rows][cols] (row stride ld floats) for the
// epilogue's TMA stores: box 32 columns x 32 rows with the 128-byte swizzle
// of the warp stages.
static bool make_tmap_out_f16(CUtensorMap* tm, const __half* base, uint64_t cols, uint64_t rows, uint64_t ld) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || !base || cols == 0 || rows == 0 || cols > ld) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld * 2) % 16 != 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static bool make_tmap_out_f32(CUtensorMap* tm, const float* base, uint64_t cols, uint64_t rows, uint64_t ld) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || !base || cols == 0 || rows == 0 || cols > ld) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld * 4) % 16 != 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

cudaError_t gemm_run(const GemmLaunch& g_in, cudaStream_t stream) {
  if (g_in.args.M <= 0 || g_in.args.N <= 0 || g_in.args.num_kb <= 0) return cudaErrorInvalidValue;
  // Plain F32 outputs (contiguous rows, single-CTA form) leave through TMA stores.
  GemmLaunch g = g_in;
  g.args.tma_o32 = 0;
  if (g.args.epi == kEpiF32 && g.args.out32 && !g.args.pad_rows && !g.pair &&
      make_tmap_out_f32(&g.tmO, g.args.out32, static_cast<uint64_t>(g.args.N), static_cast<uint64_t>(g.args.M),
                        static_cast<uint64_t>(g.args.ld32)))
    g.args.tma_o32 = 1;
  g.args.tma_o16 = 0;
  const int e = g.args.epi;
  if ((e == kEpiF16 || e == kEpiQKV || e == kEpiSwiGLU) && g.args.out16 && !g.pair &&
      make_tmap_out_f16(&g.tmO, g.args.out16, static_cast<uint64_t>(e == kEpiSwiGLU ? g.args.N / 2 : g.args.N),
                        static_cast<uint64_t>(g.args.M), static_cast<uint64_t>(g.args.ld16)))
    g.args.tma_o16 = 1;
  if (g.pair) {
    switch (g.bn) {
      case 64: return launch_epi<64, true>(g, stream);
      case 128: return launch_epi<128, true>(g, stream);
      case 256: return launch_epi<256, true>(g, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (g.bn) {
    case 32: return launch_epi<32, false>(g, stream);
    case 48: return launch_epi<48, false>(g, stream);
    case 64: return launch_epi<64, false>(g, stream);
    case 80: return launch_epi<80, false>(g, stream);
    case 128: return launch_epi<128, false>(g, stream);
    case 192: return launch_epi<192, false>(g, stream);
    case 256: return launch_epi<256, false>(g, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace itts
