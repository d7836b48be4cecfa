// Persistent GPT decoder: one cooperative kernel runs every token of a
// generate call (the P prefix rows, then the greedy decode steps until the
// stop code or the step limit), replacing run_gpt_kv_greedy_cpu
// (runtime/impl/gpt.cpp:1877-1909) with the same math as the per-kernel
// path in gpt.cu.
//
// Decoding one token is a chain of small all-to-all dependent steps (5 per
// layer: c_attn, attention, attn.c_proj, c_fc, mlp.c_proj; then the head),
// each streaming its weight matrix once. Launching a kernel per step costs
// ~3 us of launch and drain each, more than the step's own memory time, so
// here the steps are stages of one kernel, separated by a grid barrier
// (bounded spin on an arrival counter), with one CTA per SM:
//
//  * a producer warp streams the CTA's rows of every projection's f16 weight
//    matrix, in execution order, through a ring of 10 shared-memory slots of
//    20 KB (bulk copies completing on mbarriers). It runs ahead of the
//    consumers across stage and token boundaries, so the weight stream of
//    the next stages overlaps the barriers and the small steps;
//  * 16 consumer warps compute each stage: the input row into shared memory
//    (LayerNorm / the attention's split-softmax merge fused), then one task =
//    one 1280-column slice of one row per warp (fp32 products and
//    accumulation, a fixed butterfly, row slices summed in order), the
//    epilogue (bias, gelu_new, residual) and the grid barrier;
//  * the attention stage gives each of 140 CTAs one (head, key range);
//  * the head stage ends with a per-CTA argmax candidate; after the barrier
//    every CTA reduces the candidates in CTA order (the first maximum, as
//    argmax_row) and so knows the next code without another barrier.
//
// Data written by one CTA and read by another in a later stage is read with
// ld.global.cg (L2), never through L1.
#include "gpt_persist.cuh"

#include <cfloat>
#include <climits>

#include "ptx.cuh"

namespace itts {

namespace {

constexpr int kW = 1280, kQkv = 3840, kMlp = 5120, kVocab = 8194, kLayers = 24;
constexpr int kMaxLen = 4096, kStart = 8192, kStop = 8193;
constexpr int kSplits = 7, kPart = 66, kSplitKeys = (kMaxLen + kSplits - 1) / kSplits + 1;
constexpr int kAttnCtas = 20 * kSplits;
constexpr int kCons = 512;             // consumer threads (16 warps)
constexpr int kThreads = kCons + 32;   // + the producer warp
constexpr int kSlots = 10;
constexpr int kTaskCols = 1280;        // columns of one task
constexpr int kTaskBytes = kTaskCols * 2;
constexpr int kSlotTasks = 8;
constexpr int kSlotBytes = kSlotTasks * kTaskBytes;  // 20 KB
constexpr int kMaxTasks = 64;          // tasks of one CTA in one stage
enum : unsigned int { kDevTimeoutGrid = 40, kDevTimeoutRing = 41, kDevTimeoutSlot = 42 };

constexpr size_t kOffXs = static_cast<size_t>(kSlots) * kSlotBytes;
constexpr size_t kOffBars = kOffXs + static_cast<size_t>(kMlp) * 4;
constexpr size_t kOffRed = kOffBars + 2 * kSlots * 8;
constexpr size_t kOffTsum = kOffRed + 16 * 4;
constexpr size_t kOffTv = kOffTsum + kMaxTasks * 4;
constexpr size_t kOffFlags = kOffTv + kMaxTasks * 4;
constexpr size_t kSmem = kOffFlags + 16;
static_assert(kSmem <= 227 * 1024, "shared memory");
// attention scratch inside xs: scores [0, 600), q [600, 664), 16 x 64 accumulators after
constexpr int kScrQ = 600, kScrAcc = 664;
static_assert(kSplitKeys <= kScrQ && kScrAcc + 16 * 64 <= kMlp, "attention scratch");

enum Stage { kSQkv = 0, kSAttn = 1, kSProj = 2, kSFc = 3, kSMproj = 4, kSHead = 5 };

struct ProjDesc {
  const __half* w;
  const float* bias;
  int n, k;
};

__device__ __forceinline__ ProjDesc proj_of(const GptPersistParams& p, int stage, int layer) {
  if (stage == kSHead) return {p.w_head, p.b_head, kVocab, kW};
  const GptLayerPtrs& L = p.layers[layer];
  switch (stage) {
    case kSQkv: return {L.w_attn, L.b_attn, kQkv, kW};
    case kSProj: return {L.w_proj, L.b_proj, kW, kW};
    case kSFc: return {L.w_fc, L.b_fc, kMlp, kW};
    default: return {L.w_mproj, L.b_mproj, kW, kMlp};
  }
}

// Rows [r0, r1) of an n-row projection owned by CTA b of G (balanced split).
__device__ __forceinline__ void rows_of(int n, int b, int G, int& r0, int& r1) {
  r0 = static_cast<int>(static_cast<long long>(b) * n / G);
  r1 = static_cast<int>(static_cast<long long>(b + 1) * n / G);
}

// Barrier of the 512 consumer threads (the producer warp never joins it).
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Sum / max over the 512 consumer threads, returned to all of them (fixed
// reduction tree: deterministic).
__device__ __forceinline__ float csum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  cbar();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < 16; ++w) t += red[w];
  cbar();
  return t;
}

__device__ __forceinline__ float cmax(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  cbar();
  float t = red[0];
#pragma unroll
  for (int w = 1; w < 16; ++w) t = fmaxf(t, red[w]);
  cbar();
  return t;
}

// cpu_layernorm (runtime/impl/tokenizer_tests.cpp:2992-3010) on xs[0, kW).
__device__ __forceinline__ void cons_layer_norm(float* xs, const float* __restrict__ g, const float* __restrict__ b,
                                                float* red) {
  float s = 0.0f;
  for (int i = threadIdx.x; i < kW; i += kCons) s += xs[i];
  const float mean = csum(s, red) / static_cast<float>(kW);
  float v = 0.0f;
  for (int i = threadIdx.x; i < kW; i += kCons) {
    const float d = xs[i] - mean;
    v += d * d;
  }
  const float var = csum(v, red) / static_cast<float>(kW);
  const float inv = 1.0f / sqrtf(var + 1e-5f);
  for (int i = threadIdx.x; i < kW; i += kCons) xs[i] = (xs[i] - mean) * inv * g[i] + b[i];
  cbar();
}

// gelu_new of cpu_gelu_new (runtime/impl/tokenizer_tests.cpp:3931-3945).
__device__ __forceinline__ float gelu_new(float x) {
  if (x > 10.0f) return x;
  if (x < -10.0f) return 0.0f;
  const float c = 0.7978845608028654f;
  return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
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

struct Smem {
  uint8_t* ring;
  float* xs;
  uint64_t* full;
  uint64_t* empty;
  float* red;
  float* tsum;
  float* tv;
  volatile int* flags;  // [0] done (consumers finished), [1] error, [2] argmax result
};

__device__ __forceinline__ Smem smem_of(uint8_t* base) {
  Smem s;
  s.ring = base;
  s.xs = reinterpret_cast<float*>(base + kOffXs);
  s.full = reinterpret_cast<uint64_t*>(base + kOffBars);
  s.empty = s.full + kSlots;
  s.red = reinterpret_cast<float*>(base + kOffRed);
  s.tsum = reinterpret_cast<float*>(base + kOffTsum);
  s.tv = reinterpret_cast<float*>(base + kOffTv);
  s.flags = reinterpret_cast<volatile int*>(base + kOffFlags);
  return s;
}

// Grid barrier over the consumers of all CTAs: arrival counter, bounded spin.
// Returns false (and marks the CTA's error flag) when the wait gave up.
__device__ __forceinline__ bool grid_sync(const GptPersistParams& p, unsigned int target, const Smem& sm) {
  cbar();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(p.barrier, 1u);
    const long long start = clock64();
    bool ok = true;
    while (ld_acquire(p.barrier) < target) {
      if (clock64() - start > kWaitBudgetCycles) {
        atomicCAS(p.status, 0u, kDevTimeoutGrid);
        ok = false;
        break;
      }
    }
    __threadfence();
    if (!ok) sm.flags[1] = 1;
  }
  cbar();
  return sm.flags[1] == 0;
}

// ---------------------------------------------------------------- producer

// Waits for a slot's release by the consumers; gives up when the consumers
// have finished (flags[0]) or the wait budget runs out.
__device__ __forceinline__ bool wait_slot_free(uint64_t* bar, uint32_t parity, const Smem& sm, unsigned int* status) {
  const uint32_t a = smem_u32(bar);
  const long long start = clock64();
  while (!mbar_try_wait(a, parity)) {
    if (sm.flags[0]) return false;
    if (clock64() - start > kWaitBudgetCycles) {
      atomicCAS(status, 0u, kDevTimeoutRing);
      return false;
    }
  }
  return true;
}

__device__ void producer(const GptPersistParams& p, const Smem& sm) {
  const int G = gridDim.x, b = blockIdx.x;
  uint32_t it = 0;
  bool stop = false;
  auto issue = [&](int stage, int layer) {
    if (stop) return;
    const ProjDesc d = proj_of(p, stage, layer);
    int r0, r1;
    rows_of(d.n, b, G, r0, r1);
    const uint32_t bytes = static_cast<uint32_t>(r1 - r0) * d.k * 2;
    const uint8_t* src = reinterpret_cast<const uint8_t*>(d.w + static_cast<size_t>(r0) * d.k);
    for (uint32_t off = 0; off < bytes; off += kSlotBytes) {
      const int slot = static_cast<int>(it % kSlots);
      const uint32_t k = it / kSlots;
      if (k > 0 && !wait_slot_free(&sm.empty[slot], (k - 1) & 1, sm, p.status)) {
        stop = true;
        return;
      }
      const uint32_t nb = min(static_cast<uint32_t>(kSlotBytes), bytes - off);
      mbar_arrive_expect_tx(&sm.full[slot], nb);
      bulk_load(sm.ring + static_cast<size_t>(slot) * kSlotBytes, src + off, nb, &sm.full[slot]);
      ++it;
    }
  };
  const int tokens = p.P + p.max_steps;
  for (int tok = 0; tok < tokens && !stop; ++tok) {
    for (int l = 0; l < kLayers; ++l) {
      issue(kSQkv, l);
      issue(kSProj, l);
      issue(kSFc, l);
      issue(kSMproj, l);
    }
    if (tok >= p.P) issue(kSHead, 0);
  }
  // Every copy issued must land before the CTA exits.
  for (uint32_t j = it > kSlots ? it - kSlots : 0; j < it; ++j)
    mbar_wait(&sm.full[j % kSlots], (j / kSlots) & 1, nullptr, 0);
}

// ---------------------------------------------------------------- consumers

// The CTA's part of one projection: tasks (row, 1280-column slice) from the
// ring, then the epilogue per row. `it` = the ring position of the stage's
// first slot. Returns false when a slot wait gave up.
template <int STAGE>
__device__ bool cons_proj(const GptPersistParams& p, const Smem& sm, int layer, uint32_t& it) {
  const int G = gridDim.x, b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const ProjDesc d = proj_of(p, STAGE, layer);
  int r0, r1;
  rows_of(d.n, b, G, r0, r1);
  const int segs = d.k / kTaskCols;
  const int T = (r1 - r0) * segs;
  const int S = (T + kSlotTasks - 1) / kSlotTasks;
  const int wg = warp >> 3, wt = warp & 7;  // warps 0-7 take even slots, 8-15 odd ones
  for (int sp = 0; sp < S; sp += 2) {
    const int si = sp + wg;
    if (si < S) {
      const uint32_t ig = it + si;
      const int slot = static_cast<int>(ig % kSlots);
      // warp-uniform outcome, so that the shuffles below see every lane
      const bool got = __all_sync(0xffffffffu, mbar_wait(&sm.full[slot], (ig / kSlots) & 1, p.status, kDevTimeoutSlot));
      if (!got) {
        sm.flags[1] = 1;
      } else {
        const int task = si * kSlotTasks + wt;
        if (task < T) {
          const uint4* wr = reinterpret_cast<const uint4*>(sm.ring + static_cast<size_t>(slot) * kSlotBytes +
                                                          static_cast<size_t>(wt) * kTaskBytes);
          const float* xb = sm.xs + (task % segs) * kTaskCols;
          float s = 0.0f;
#pragma unroll
          for (int c = 0; c < kTaskCols / 256; ++c) s += dot8(wr[lane + 32 * c], xb + (lane + 32 * c) * 8);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
          if (lane == 0) sm.tsum[task] = s;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[slot]);
    }
  }
  it += S;
  cbar();
  if (sm.flags[1]) return false;
  for (int r = tid; r < r1 - r0; r += kCons) {
    float s = 0.0f;
    for (int q = 0; q < segs; ++q) s += sm.tsum[r * segs + q];
    const int n = r0 + r;
    const float v = s + d.bias[n];
    if (STAGE == kSQkv) p.qkv[n] = v;
    if (STAGE == kSProj) p.h[n] = __ldcg(p.x + n) + v;
    if (STAGE == kSFc) p.m[n] = gelu_new(v);
    if (STAGE == kSMproj) p.x[n] = __ldcg(p.h + n) + v;
    if (STAGE == kSHead) {
      p.logits[n] = v;
      sm.tv[r] = v;
    }
  }
  if (STAGE == kSHead) {
    cbar();
    if (tid == 0) {  // first maximum of the CTA's rows
      float bv = sm.tv[0];
      int bi = r0;
      for (int r = 1; r < r1 - r0; ++r)
        if (sm.tv[r] > bv) {
          bv = sm.tv[r];
          bi = r0 + r;
        }
      p.cand_val[b] = bv;
      p.cand_idx[b] = bi;
    }
  }
  return true;
}

// One (head, key range) of the cached single-query attention
// (cpu_attention_single_query, runtime/impl/tokenizer_tests.cpp:4034-4061):
// partial (max, sum e^(s-max), sum e^(s-max) v) over keys [j0, j1) of the
// len + 1 keys (this token's K and V read from qkv); range 0 also appends
// this token's K and V at row len of the layer's cache.
__device__ void cons_attention(const GptPersistParams& p, const Smem& sm, int layer, int len) {
  const int b = blockIdx.x, tid = threadIdx.x;
  const int h = b / kSplits, r = b - h * kSplits;
  const int n = len + 1, chunk = (n + kSplits - 1) / kSplits;
  const int j0 = r * chunk, j1 = min(n, j0 + chunk);
  float* kc = p.kc + static_cast<size_t>(layer) * kMaxLen * kW;
  float* vc = p.vc + static_cast<size_t>(layer) * kMaxLen * kW;
  const float* kcur = p.qkv + kW + h * 64;
  const float* vcur = p.qkv + 2 * kW + h * 64;
  float* s = sm.xs;
  float* q = sm.xs + kScrQ;
  float* accw = sm.xs + kScrAcc;
  if (r == 0) {
    const size_t cur = static_cast<size_t>(len) * kW + h * 64;
    if (tid < 64) kc[cur + tid] = __ldcg(kcur + tid);
    else if (tid < 128) vc[cur + tid - 64] = __ldcg(vcur + tid - 64);
  }
  float* out = p.part + (static_cast<size_t>(h) * kSplits + r) * kPart;
  if (j0 >= j1) {  // empty range (short caches)
    if (tid < kPart) out[tid] = tid == 0 ? -INFINITY : 0.0f;
    return;
  }
  if (tid < 64) q[tid] = __ldcg(p.qkv + h * 64 + tid);
  cbar();
  // scores: 16 lanes per key (a float4 of the 64 dims each), 4 keys in flight per group
  const int g = tid >> 4, l = tid & 15;
  const float4 qv = reinterpret_cast<const float4*>(q)[l];
  for (int base = j0; base < j1; base += 128) {
    float4 kv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = base + g + 32 * u;
      const float* kp = j == len ? kcur : kc + static_cast<size_t>(j) * kW + h * 64;
      kv[u] = j < j1 ? __ldcg(reinterpret_cast<const float4*>(kp + 4 * l)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float d = qv.x * kv[u].x;
      d = fmaf(qv.y, kv[u].y, d);
      d = fmaf(qv.z, kv[u].z, d);
      d = fmaf(qv.w, kv[u].w, d);
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      const int j = base + g + 32 * u;
      if (l == 0 && j < j1) s[j - j0] = d * 0.125f;
    }
  }
  cbar();
  const int cnt = j1 - j0;
  float mx = -INFINITY;
  for (int j = tid; j < cnt; j += kCons) mx = fmaxf(mx, s[j]);
  mx = cmax(mx, sm.red);
  float den = 0.0f;
  for (int j = tid; j < cnt; j += kCons) {
    const float e = expf(s[j] - mx);
    s[j] = e;
    den += e;
  }
  den = csum(den, sm.red);  // its barriers also order the writes of s before the reads below
  // acc: warp w takes keys w, w+16, ...; lane dims 2 lane, 2 lane + 1
  const int w = tid >> 5, lane = tid & 31;
  float2 acc = make_float2(0.f, 0.f);
  for (int base = 0; base < cnt; base += 64) {
    float2 vv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = base + w + 16 * u;
      const int jj = j0 + j;
      const float* vp = jj == len ? vcur : vc + static_cast<size_t>(jj) * kW + h * 64;
      vv[u] = j < cnt ? __ldcg(reinterpret_cast<const float2*>(vp + 2 * lane)) : make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = base + w + 16 * u;
      const float pj = j < cnt ? s[j] : 0.0f;
      acc.x = fmaf(pj, vv[u].x, acc.x);
      acc.y = fmaf(pj, vv[u].y, acc.y);
    }
  }
  accw[w * 64 + 2 * lane] = acc.x;
  accw[w * 64 + 2 * lane + 1] = acc.y;
  cbar();
  if (tid < 64) {
    float o = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) o += accw[i * 64 + tid];
    out[2 + tid] = o;
  } else if (tid == 64) {
    out[0] = mx;
    out[1] = den;
  }
}

// The attention partials merged into the heads' outputs (xs[0, kW)):
// M = max_r m_r, out = sum_r acc_r e^(m_r - M) / sum_r l_r e^(m_r - M).
__device__ __forceinline__ void cons_attn_combine(const GptPersistParams& p, float* xs) {
  for (int i = threadIdx.x; i < kW; i += kCons) {
    const int h = i >> 6, d = i & 63;
    const float* pp = p.part + static_cast<size_t>(h) * kSplits * kPart;
    float ms[kSplits], ls[kSplits];
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < kSplits; ++r) {
      ms[r] = __ldcg(pp + r * kPart);
      ls[r] = __ldcg(pp + r * kPart + 1);
      if (ls[r] > 0.0f) M = fmaxf(M, ms[r]);
    }
    float L = 0.0f, A = 0.0f;
#pragma unroll
    for (int r = 0; r < kSplits; ++r) {
      if (ls[r] > 0.0f) {
        const float e = expf(ms[r] - M);
        L = fmaf(ls[r], e, L);
        A = fmaf(__ldcg(pp + r * kPart + 2 + d), e, A);
      }
    }
    xs[i] = A / L;
  }
  cbar();
}

__global__ void __launch_bounds__(kThreads, 1) gpt_persist_kernel(GptPersistParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const Smem sm = smem_of(smem_raw);
  const int tid = threadIdx.x, b = blockIdx.x, G = gridDim.x;
  if (tid == 0) {
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 8);  // the 8 consumer warps that read a slot
    }
    fence_barrier_init();
    sm.flags[0] = 0;
    sm.flags[1] = 0;
  }
  __syncthreads();
  if (tid >= kCons) {
    if (tid == kCons) producer(p, sm);
    return;
  }
  if (b == 0 && tid == 0) p.times[0] = globaltimer();
  uint32_t it = 0;
  unsigned int bar_k = 0;
  int len = 0, step = 0, code = kStart;
  bool ok = true;
  auto sync = [&]() {
    ++bar_k;
    return grid_sync(p, bar_k * static_cast<unsigned int>(G), sm);
  };
  const int tokens = p.P + p.max_steps;
  for (int tok = 0; tok < tokens && ok; ++tok) {
    const bool decode = tok >= p.P;
    if (tok == p.P && b == 0 && tid == 0) p.times[1] = globaltimer();
    for (int l = 0; l < kLayers && ok; ++l) {
      const GptLayerPtrs& L = p.layers[l];
      // c_attn(ln_1(x)); layer 0 builds x (the prefix row, or mel_embedding[code]
      // + mel_pos_embedding[step] as build_gpt_greedy_current_cpu,
      // runtime/impl/gpt.cpp:1545-1554) and publishes the CTA's slice of it.
      if (l == 0) {
        const float* e0 = decode ? p.emb + static_cast<size_t>(code) * kW : p.prefix + static_cast<size_t>(tok) * kW;
        // gpt_cached_generate_position (runtime/impl/gpt.cpp:1873-1875)
        const int position = p.hf_positions && step > 0 ? step + 1 : step;
        const float* e1 = p.pos + static_cast<size_t>(position) * kW;
        const int x0 = static_cast<int>(static_cast<long long>(b) * kW / G);
        const int x1 = static_cast<int>(static_cast<long long>(b + 1) * kW / G);
        for (int i = tid; i < kW; i += kCons) {
          const float v = decode ? e0[i] + e1[i] : e0[i];
          sm.xs[i] = v;
          if (i >= x0 && i < x1) p.x[i] = v;
        }
      } else {
        for (int i = tid; i < kW; i += kCons) sm.xs[i] = __ldcg(p.x + i);
      }
      cbar();
      cons_layer_norm(sm.xs, L.ln1_g, L.ln1_b, sm.red);
      ok = cons_proj<kSQkv>(p, sm, l, it) && sync();
      if (!ok) break;
      if (b < kAttnCtas) cons_attention(p, sm, l, len);
      ok = sync();
      if (!ok) break;
      cons_attn_combine(p, sm.xs);
      ok = cons_proj<kSProj>(p, sm, l, it) && sync();
      if (!ok) break;
      for (int i = tid; i < kW; i += kCons) sm.xs[i] = __ldcg(p.h + i);
      cbar();
      cons_layer_norm(sm.xs, L.ln2_g, L.ln2_b, sm.red);
      ok = cons_proj<kSFc>(p, sm, l, it) && sync();
      if (!ok) break;
      for (int i = tid; i < kMlp; i += kCons) sm.xs[i] = __ldcg(p.m + i);
      cbar();
      ok = cons_proj<kSMproj>(p, sm, l, it) && sync();
    }
    if (!ok) break;
    ++len;
    if (!decode) continue;
    // ln_f, final_norm, mel head, argmax (runtime/impl/gpt.cpp:1901-1905)
    for (int i = tid; i < kW; i += kCons) sm.xs[i] = __ldcg(p.x + i);
    cbar();
    cons_layer_norm(sm.xs, p.lnf_g, p.lnf_b, sm.red);
    cons_layer_norm(sm.xs, p.fn_g, p.fn_b, sm.red);
    ok = cons_proj<kSHead>(p, sm, 0, it) && sync();
    if (!ok) break;
    if (tid == 0) {  // candidates in CTA order = row order: the first maximum
      float bv = __ldcg(p.cand_val);
      int bi = __ldcg(p.cand_idx);
      for (int c = 1; c < G; ++c) {
        const float v = __ldcg(p.cand_val + c);
        if (v > bv) {
          bv = v;
          bi = __ldcg(p.cand_idx + c);
        }
      }
      sm.flags[2] = bi;
      if (b == 0) p.codes[step] = static_cast<uint32_t>(bi);
    }
    cbar();
    code = sm.flags[2];
    ++step;
    if (code == kStop || step >= p.max_steps) break;
  }
  if (b == 0 && tid == 0) {
    p.out[0] = step;
    p.times[2] = globaltimer();
  }
  cbar();
  if (tid == 0) sm.flags[0] = 1;  // lets the producer stop
}

}  // namespace

size_t gpt_persist_smem() { return kSmem; }

int gpt_persist_min_grid() { return (kVocab + kMaxTasks - 1) / kMaxTasks + 1; }

cudaError_t gpt_persist_prepare() {
  return cudaFuncSetAttribute(gpt_persist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmem));
}

cudaError_t gpt_persist_launch(const GptPersistParams& p, int grid, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gpt_persist_kernel, p);
}

}  // namespace itts
