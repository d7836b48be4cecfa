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
enum : unsigned int { kDevTimeoutGrid = 40, kDevTimeoutRing = 41, kDevTimeoutSlot = 42, kDevSampleTies = 43 };

constexpr size_t kOffXs = static_cast<size_t>(kSlots) * kSlotBytes;
constexpr size_t kOffBars = kOffXs + static_cast<size_t>(kMlp) * 4;
constexpr size_t kOffRed = kOffBars + 2 * kSlots * 8;
constexpr size_t kOffTsum = kOffRed + 16 * 4;
constexpr size_t kOffTv = kOffTsum + kMaxTasks * 4;
constexpr size_t kOffFlags = kOffTv + kMaxTasks * 4;
constexpr size_t kOffLayers = kOffFlags + 16;  // the layer pointer table, copied once
constexpr size_t kSmem = kOffLayers + sizeof(GptLayerPtrs) * kLayers;
static_assert(kSmem <= 227 * 1024, "shared memory");
// attention scratch inside xs
constexpr int kScrAcc = 640;  // scores [0, kSplitKeys), 16 x 64 accumulators from here
static_assert(kSplitKeys <= kScrAcc && kScrAcc + 16 * 64 <= kMlp, "attention scratch");

enum Stage { kSQkv = 0, kSAttn = 1, kSProj = 2, kSFc = 3, kSMproj = 4, kSHead = 5 };

struct ProjDesc {
  const __half* w;
  const float* bias;
  int n, k;
};

// Rows and columns of each stage's projection (compile-time, so that loop
// bounds never wait on a load).
__host__ __device__ constexpr int stage_n(int stage) {
  return stage == kSQkv ? kQkv : stage == kSFc ? kMlp : stage == kSHead ? kVocab : kW;
}
__host__ __device__ constexpr int stage_k(int stage) { return stage == kSMproj ? kMlp : kW; }

// Weight and bias of a stage; `layers` = the pointer table in shared memory.
__device__ __forceinline__ ProjDesc proj_of(const GptPersistParams& p, const GptLayerPtrs* layers, int stage,
                                            int layer) {
  if (stage == kSHead) return {p.w_head, p.b_head, kVocab, kW};
  const GptLayerPtrs& L = layers[layer];
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

// A 1280-wide row held 3 values per consumer thread (elements tid, tid + 512,
// tid + 1024), so that its loads, the LayerNorm parameters' loads and the
// reductions need one memory round trip.
constexpr int kPer = (kW + kCons - 1) / kCons;

__device__ __forceinline__ void load_params(const float* __restrict__ g, const float* __restrict__ b, float* gg,
                                            float* bb) {
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = threadIdx.x + k * kCons;
    gg[k] = i < kW ? g[i] : 0.0f;
    bb[k] = i < kW ? b[i] : 0.0f;
  }
}

__device__ __forceinline__ void load_row_cg(const float* src, float* v) {
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = threadIdx.x + k * kCons;
    v[k] = i < kW ? __ldcg(src + i) : 0.0f;
  }
}

// cpu_layernorm (runtime/impl/tokenizer_tests.cpp:2992-3010) on the row in
// registers: mean, biased variance, (x - mean) * (1 / sqrt(var + 1e-5)) *
// gamma + beta.
__device__ __forceinline__ void layer_norm_regs(float* v, const float* gg, const float* bb, float* red) {
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < kPer; ++k)
    if (threadIdx.x + k * kCons < kW) s += v[k];
  const float mean = csum(s, red) / static_cast<float>(kW);
  float q = 0.0f;
#pragma unroll
  for (int k = 0; k < kPer; ++k)
    if (threadIdx.x + k * kCons < kW) {
      const float d = v[k] - mean;
      q += d * d;
    }
  const float var = csum(q, red) / static_cast<float>(kW);
  const float inv = 1.0f / sqrtf(var + 1e-5f);
#pragma unroll
  for (int k = 0; k < kPer; ++k) v[k] = (v[k] - mean) * inv * gg[k] + bb[k];
}

__device__ __forceinline__ void store_row(const float* v, float* xs) {
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = threadIdx.x + k * kCons;
    if (i < kW) xs[i] = v[k];
  }
  cbar();
}

// gelu_new of cpu_gelu_new (runtime/impl/tokenizer_tests.cpp:3931-3945).
__device__ __forceinline__ float gelu_new(float x) {
  if (x > 10.0f) return x;
  if (x < -10.0f) return 0.0f;
  const float c = 0.7978845608028654f;
  return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
}

// dot8 with the eight input values in registers (same order of operations).
__device__ __forceinline__ float dot8r(const uint4 w, const float* x) {
  const float2 w0 = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
  const float2 w1 = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
  const float2 w2 = __half22float2(*reinterpret_cast<const __half2*>(&w.z));
  const float2 w3 = __half22float2(*reinterpret_cast<const __half2*>(&w.w));
  float s = w0.x * x[0];
  s = fmaf(w0.y, x[1], s);
  s = fmaf(w1.x, x[2], s);
  s = fmaf(w1.y, x[3], s);
  s = fmaf(w2.x, x[4], s);
  s = fmaf(w2.y, x[5], s);
  s = fmaf(w3.x, x[6], s);
  s = fmaf(w3.y, x[7], s);
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
  GptLayerPtrs* layers;  // [24]
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
  s.layers = reinterpret_cast<GptLayerPtrs*>(base + kOffLayers);
  return s;
}

__device__ __forceinline__ void red_add_release(unsigned int* p, unsigned int v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barrier k over the consumers of all CTAs: after the CTA barrier,
// thread 0 adds one to the arrival counter with a release reduction (the
// CTA's writes, ordered before it by the CTA barrier, are released; nothing
// waits for the add to return) and polls the counter with acquire loads until
// all k * G arrivals are in (bounded spin); the CTA barrier then passes the
// acquired writes on to the CTA. Returns false (and marks the CTA's error
// flag) when the wait gave up. `arrive`, when non-null, receives the global
// timer at this CTA's arrival (stage trace).
__device__ __forceinline__ bool grid_sync(const GptPersistParams& p, unsigned int k, const Smem& sm,
                                          unsigned long long* arrive) {
  cbar();
  if (threadIdx.x == 0) {
    const unsigned int target = k * gridDim.x;
    if (arrive) *arrive = globaltimer();
    red_add_release(p.barrier, 1u);
    const long long start = clock64();
    while (ld_acquire(p.barrier) < target) {
      if (clock64() - start > kWaitBudgetCycles) {
        atomicCAS(p.status, 0u, kDevTimeoutGrid);
        sm.flags[1] = 1;
        break;
      }
    }
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
    const ProjDesc d = proj_of(p, sm.layers, stage, layer);
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

// The epilogue operands of the CTA's rows (one row per consumer thread):
// bias and residual, loaded before the stage's prologue so that their
// latency overlaps it. The residual (x for attn.c_proj, h for mlp.c_proj)
// was written at least one grid barrier earlier.
template <int STAGE>
__device__ __forceinline__ void epi_prefetch(const GptPersistParams& p, const Smem& sm, int layer, float& eb,
                                             float& er) {
  const ProjDesc d = proj_of(p, sm.layers, STAGE, layer);
  int r0, r1;
  rows_of(stage_n(STAGE), blockIdx.x, gridDim.x, r0, r1);
  const int r = r0 + threadIdx.x;
  const bool mine = r < r1;
  eb = mine ? d.bias[r] : 0.0f;
  er = 0.0f;
  if (STAGE == kSProj && mine) er = __ldcg(p.x + r);
  if (STAGE == kSMproj && mine) er = __ldcg(p.h + r);
}

// The CTA's part of one projection: tasks (row, 1280-column slice) from the
// ring, then the epilogue per row. `it` = the ring position of the stage's
// first slot. Returns false when a slot wait gave up.
template <int STAGE>
__device__ bool cons_proj(const GptPersistParams& p, const Smem& sm, int layer, uint32_t& it, float eb, float er,
                          unsigned long long* slots_done) {
  const int G = gridDim.x, b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int r0, r1;
  rows_of(stage_n(STAGE), b, G, r0, r1);
  constexpr int segs = stage_k(STAGE) / kTaskCols;
  const int T = (r1 - r0) * segs;
  const int S = (T + kSlotTasks - 1) / kSlotTasks;
  const int wg = warp >> 3, wt = warp & 7;  // warps 0-7 take even slots, 8-15 odd ones
  // A slot holds 8 tasks and segs divides 8, so a warp always works on the
  // same 1280-column segment of the input row: its lanes keep their 40 input
  // values in registers for the whole stage, and only the weights stream
  // from shared memory.
  float xr[kTaskCols / 256][8];
  {
    const float* xb = sm.xs + (wt % segs) * kTaskCols;
#pragma unroll
    for (int c = 0; c < kTaskCols / 256; ++c) {
      const float4 a = *reinterpret_cast<const float4*>(xb + (lane + 32 * c) * 8);
      const float4 e = *reinterpret_cast<const float4*>(xb + (lane + 32 * c) * 8 + 4);
      xr[c][0] = a.x, xr[c][1] = a.y, xr[c][2] = a.z, xr[c][3] = a.w;
      xr[c][4] = e.x, xr[c][5] = e.y, xr[c][6] = e.z, xr[c][7] = e.w;
    }
  }
  unsigned long long waited = 0;  // stage trace: time thread 0 spent waiting for its slots
  for (int sp = 0; sp < S; sp += 2) {
    const int si = sp + wg;
    if (si < S) {
      const uint32_t ig = it + si;
      const int slot = static_cast<int>(ig % kSlots);
      const unsigned long long w0 = slots_done ? globaltimer() : 0;
      // warp-uniform outcome, so that the shuffles below see every lane
      const bool got = __all_sync(0xffffffffu, mbar_wait(&sm.full[slot], (ig / kSlots) & 1, p.status, kDevTimeoutSlot));
      if (slots_done) waited += globaltimer() - w0;
      if (!got) {
        sm.flags[1] = 1;
      } else {
        const int task = si * kSlotTasks + wt;
        if (task < T) {
          const uint4* wr = reinterpret_cast<const uint4*>(sm.ring + static_cast<size_t>(slot) * kSlotBytes +
                                                          static_cast<size_t>(wt) * kTaskBytes);
          float s = 0.0f;
#pragma unroll
          for (int c = 0; c < kTaskCols / 256; ++c) s += dot8r(wr[lane + 32 * c], xr[c]);
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
  if (slots_done && tid == 0) {
    *slots_done = globaltimer();
    slots_done[kGptTraceCap + kGptTraceStages * gridDim.x] = waited;  // stored after the arrivals
  }
  cbar();
  if (sm.flags[1]) return false;
  if (tid < r1 - r0) {
    float s = 0.0f;
    for (int q = 0; q < segs; ++q) s += sm.tsum[tid * segs + q];
    const int n = r0 + tid;
    const float v = s + eb;
    if (STAGE == kSQkv) p.qkv[n] = v;
    if (STAGE == kSProj) p.h[n] = er + v;
    if (STAGE == kSFc) p.m[n] = gelu_new(v);
    if (STAGE == kSMproj) p.x[n] = er + v;
    if (STAGE == kSHead) {
      p.logits[n] = v;
      sm.tv[tid] = v;
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
// this token's K and V at row len of the layer's cache. q, the first keys and
// the first values are loaded together (one memory round trip).
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
  const int cnt = j1 - j0;
  const int g = tid >> 4, l = tid & 15;
  const int w = tid >> 5, lane = tid & 31;
  auto vrow = [&](int j) {  // value row of key j0 + j (this token's from qkv)
    const int jj = j0 + j;
    return jj == len ? vcur : vc + static_cast<size_t>(jj) * kW + h * 64;
  };
  const float4 qv = __ldcg(reinterpret_cast<const float4*>(p.qkv + h * 64) + l);
  float2 vv0[4];  // values of keys w, w+16, w+32, w+48 (the first PV block)
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int j = w + 16 * u;
    vv0[u] = j < cnt ? __ldcg(reinterpret_cast<const float2*>(vrow(j) + 2 * lane)) : make_float2(0.f, 0.f);
  }
  // scores: 16 lanes per key (a float4 of the 64 dims each), 4 keys in flight per group
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
  float2 acc = make_float2(0.f, 0.f);
  for (int base = 0; base < cnt; base += 64) {
    float2 vv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = base + w + 16 * u;
      vv[u] = base == 0 ? vv0[u]
                        : (j < cnt ? __ldcg(reinterpret_cast<const float2*>(vrow(j) + 2 * lane)) : make_float2(0.f, 0.f));
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
// M = max_r m_r, out = sum_r acc_r e^(m_r - M) / sum_r l_r e^(m_r - M), ranges
// in index order. Threads 0..139 read one (head, range) max and sum each, the
// others' accumulator loads are issued at the same time; the per-head
// weights e^(m_r - M) / L go through shared memory (after the scores'
// scratch, which is free by now).
__device__ __forceinline__ void cons_attn_combine(const GptPersistParams& p, float* xs, float* wsc) {
  const int tid = threadIdx.x;
  float as[kPer][kSplits];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = tid + k * kCons;
    const int ii = i < kW ? i : 0;
    const float* pp = p.part + static_cast<size_t>(ii >> 6) * kSplits * kPart + 2 + (ii & 63);
#pragma unroll
    for (int r = 0; r < kSplits; ++r) as[k][r] = __ldcg(pp + r * kPart);
  }
  float m = 0.0f, l = 0.0f;
  if (tid < kAttnCtas) {
    m = __ldcg(p.part + static_cast<size_t>(tid) * kPart);
    l = __ldcg(p.part + static_cast<size_t>(tid) * kPart + 1);
    wsc[tid] = m;
    wsc[kAttnCtas + tid] = l;
  }
  cbar();
  if (tid < kAttnCtas) {  // weight of range r of head h: e^(m_r - M) / L (0 for empty ranges)
    const int h = tid / kSplits;
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < kSplits; ++r)
      if (wsc[kAttnCtas + h * kSplits + r] > 0.0f) M = fmaxf(M, wsc[h * kSplits + r]);
    float L = 0.0f;
#pragma unroll
    for (int r = 0; r < kSplits; ++r) {
      const float lr = wsc[kAttnCtas + h * kSplits + r];
      if (lr > 0.0f) L = fmaf(lr, expf(wsc[h * kSplits + r] - M), L);
    }
    wsc[2 * kAttnCtas + tid] = l > 0.0f ? expf(m - M) / L : 0.0f;
  }
  cbar();
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = tid + k * kCons;
    if (i < kW) {
      const float* wr = wsc + 2 * kAttnCtas + (i >> 6) * kSplits;
      float A = 0.0f;
#pragma unroll
      for (int r = 0; r < kSplits; ++r) A = fmaf(as[k][r], wr[r], A);
      xs[i] = A;
    }
  }
  cbar();
}

// ---------------------------------------------------------------- sampler

// SplitMix64 of the reference (runtime/impl/gpt.cpp:1601-1616).
__device__ __forceinline__ unsigned long long splitmix_next(unsigned long long& state) {
  unsigned long long z = (state += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Order-preserving unsigned key of a float (larger float -> larger key).
__device__ __forceinline__ unsigned int fkey(float f) {
  const unsigned int b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float unfkey(unsigned int k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

constexpr int kSPer = (kVocab + kCons - 1) / kCons;  // scores per consumer thread

// Bitonic sort of n (a power of two <= 2048) (score, index) pairs in shared
// memory, ascending by index (by_score = false) or by (score, index).
__device__ void bitonic_pairs(float* ks, int* ki, int n, bool by_score) {
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int t = threadIdx.x; t < n / 2; t += kCons) {
        const int i = 2 * t - (t & (j - 1));  // lower element of the pair
        const int l = i + j;
        const bool up = (i & k) == 0;
        const bool gt = by_score ? (ks[i] > ks[l] || (ks[i] == ks[l] && ki[i] > ki[l])) : ki[i] > ki[l];
        if (gt == up) {
          const float fs = ks[i];
          ks[i] = ks[l];
          ks[l] = fs;
          const int fi = ki[i];
          ki[i] = ki[l];
          ki[l] = fi;
        }
      }
      cbar();
    }
  }
}

// The sampled step of run_gpt_kv_greedy_metal (runtime/impl/gpt.cpp:2220-2233)
// in CTA 0: apply_gpt_sampling_processors (:1618-1718) then
// sample_gpt_token_from_logits (:1720-1755) on the head's logits:
//  * repetition penalty on each distinct history token (seen bitmap), score
//    * p when negative else / p; temperature division (float, as the
//    reference);
//  * top-k: the exact k-th largest score by a 4-pass radix select over
//    order-preserving keys; scores below it -> -inf;
//  * the finite scores are gathered into shared memory and bitonic-sorted by
//    index; top-p sorts them by (score, index), accumulates the normalised
//    double probabilities in that order and drops the low tail (cumulative <=
//    1 - top_p, the largest kept), then sorts back by index;
//  * the draw: one SplitMix64 unit x the sum of e^(s - max) in index order,
//    the first index whose running sum exceeds it.
// The sums run on one thread in the reference's order (exact). Returns the
// code (-1 on a finite set larger than kGptSampleMaxFinite).
__device__ int cons_sample(const GptPersistParams& p, const Smem& sm) {
  const int tid = threadIdx.x;
  unsigned int* hist = reinterpret_cast<unsigned int*>(sm.xs);  // [256]
  float* ls = sm.xs + 256;                                       // [2048] scores
  int* li = reinterpret_cast<int*>(sm.xs + 256 + kGptSampleMaxFinite);  // [2048] indices
  volatile int* ctl = reinterpret_cast<volatile int*>(sm.xs + 256 + 2 * kGptSampleMaxFinite);  // [4]
  float s[kSPer];
  const float pen = p.repetition_penalty, temp = p.temperature;
#pragma unroll
  for (int j = 0; j < kSPer; ++j) {
    const int i = tid + j * kCons;
    float v = i < kVocab ? __ldcg(p.logits + i) : -INFINITY;
    if (i < kVocab) {
      if (pen != 1.0f && ((__ldcg(p.seen + (i >> 5)) >> (i & 31)) & 1u)) v = v < 0.0f ? v * pen : v / pen;
      if (temp != 1.0f) v = v / temp;
    }
    s[j] = v;
  }
  // top-k pivot (k-th largest), most significant byte first
  unsigned int prefix = 0;
  int remaining = p.top_k;
  if (p.top_k < kVocab) {
    for (int shift = 24; shift >= 0; shift -= 8) {
      if (tid < 256) hist[tid] = 0;
      cbar();
#pragma unroll
      for (int j = 0; j < kSPer; ++j) {
        const int i = tid + j * kCons;
        if (i < kVocab) {
          const unsigned int key = fkey(s[j]);
          const bool match = shift == 24 || (key >> (shift + 8)) == (prefix >> (shift + 8));
          if (match) atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
      }
      cbar();
      if (tid == 0) {
        int acc = 0, digit = 0;
        for (int d = 255; d >= 0; --d) {
          const int c = static_cast<int>(hist[d]);
          if (acc + c >= remaining) {
            digit = d;
            break;
          }
          acc += c;
        }
        ctl[0] = digit;
        ctl[1] = remaining - acc;
      }
      cbar();
      prefix |= static_cast<unsigned int>(ctl[0]) << shift;
      remaining = ctl[1];
      cbar();
    }
    const float pivot = unfkey(prefix);
#pragma unroll
    for (int j = 0; j < kSPer; ++j)
      if (s[j] < pivot) s[j] = -INFINITY;
  }
  // gather the finite scores
  if (tid == 0) ctl[2] = 0;
  cbar();
#pragma unroll
  for (int j = 0; j < kSPer; ++j) {
    const int i = tid + j * kCons;
    if (i < kVocab && isfinite(s[j])) {
      const int pos = atomicAdd(const_cast<int*>(&ctl[2]), 1);
      if (pos < kGptSampleMaxFinite) {
        ls[pos] = s[j];
        li[pos] = i;
      }
    }
  }
  cbar();
  const int F = ctl[2];
  cbar();
  if (F < 1 || F > kGptSampleMaxFinite) return -1;
  int n2 = 32;
  while (n2 < F) n2 <<= 1;
  for (int t = F + tid; t < n2; t += kCons) {
    ls[t] = INFINITY;  // pads sort last in both orders
    li[t] = INT_MAX;
  }
  cbar();
  bitonic_pairs(ls, li, n2, false);
  if (p.top_p < 1.0f) {
    if (tid == 0) {
      float m = -INFINITY;
      for (int t = 0; t < F; ++t) m = fmaxf(m, ls[t]);
      double total = 0.0;
      for (int t = 0; t < F; ++t) total += exp(static_cast<double>(ls[t] - m));
      reinterpret_cast<volatile double*>(sm.red)[0] = total;
      reinterpret_cast<volatile float*>(sm.red)[2] = m;
    }
    cbar();
    const double total = reinterpret_cast<volatile double*>(sm.red)[0];
    const float m = reinterpret_cast<volatile float*>(sm.red)[2];
    cbar();
    bitonic_pairs(ls, li, n2, true);
    if (tid == 0) {
      const double low_tail = 1.0 - static_cast<double>(p.top_p);
      double cumulative = 0.0;
      for (int t = 0; t < F; ++t) {
        cumulative += exp(static_cast<double>(ls[t] - m)) / total;
        if (cumulative <= low_tail && t != F - 1) ls[t] = -INFINITY;
      }
    }
    cbar();
    bitonic_pairs(ls, li, n2, false);
  }
  if (tid == 0) {
    float m = -INFINITY;
    for (int t = 0; t < F; ++t)
      if (isfinite(ls[t])) m = fmaxf(m, ls[t]);
    double total = 0.0;
    for (int t = 0; t < F; ++t)
      if (isfinite(ls[t])) total += exp(static_cast<double>(ls[t] - m));
    unsigned long long st = *p.rng;
    const double unit = static_cast<double>(splitmix_next(st) >> 11) * (1.0 / 9007199254740992.0);
    *p.rng = st;
    const double target = unit * total;
    double cumulative = 0.0;
    int pick = -1, last = -1;
    for (int t = 0; t < F && pick < 0; ++t) {
      if (!isfinite(ls[t])) continue;
      const double pr = exp(static_cast<double>(ls[t] - m));
      if (pr <= 0.0) continue;
      last = li[t];
      cumulative += pr;
      if (target < cumulative) pick = li[t];
    }
    ctl[3] = pick >= 0 ? pick : last;
  }
  cbar();
  return ctl[3];
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
  {  // the layer pointer table into shared memory
    const uint64_t* src = reinterpret_cast<const uint64_t*>(p.layers);
    uint64_t* dst = reinterpret_cast<uint64_t*>(sm.layers);
    for (int i = tid; i < static_cast<int>(sizeof(GptLayerPtrs) * kLayers / 8); i += kThreads) dst[i] = src[i];
  }
  __syncthreads();
  if (tid >= kCons) {
    if (tid == kCons) producer(p, sm);
    return;
  }
  if (b == 0 && tid == 0) p.times[0] = globaltimer();
  if (p.sample && b == 0) {  // the repetition history before the first code
    for (int i = tid; i < (kVocab + 31) / 32; i += kCons) p.seen[i] = 0u;
    cbar();
    if (p.n_history == 0) {
      if (tid == 0) atomicOr(p.seen + (kStart >> 5), 1u << (kStart & 31));
    } else {
      for (int i = tid; i < p.n_history; i += kCons) {
        const uint32_t t = p.history[i];
        if (t < static_cast<uint32_t>(kVocab)) atomicOr(p.seen + (t >> 5), 1u << (t & 31));
      }
    }
    if (tid == 0) *p.rng = p.seed;
    cbar();
  }
  uint32_t it = 0;
  unsigned int bar_k = 0;
  int len = p.len0, step = 0, code = kStart;
  bool ok = true;
  bool tracing = false, trace_arrivals = false;
  int stage_no = 0;  // stage index within the traced token
  auto sync = [&]() {
    unsigned long long* arrive = trace_arrivals && stage_no < kGptTraceStages
                                     ? p.trace + kGptTraceCap + static_cast<size_t>(stage_no) * G + b
                                     : nullptr;
    ++stage_no;
    return grid_sync(p, ++bar_k, sm, arrive);
  };
  int tr = 0;
  auto mark = [&]() {
    if (tracing && tr < kGptTraceCap) p.trace[tr++] = globaltimer();
  };
  auto slot_mark = [&]() -> unsigned long long* {  // reserves the "slots done" point
    return tracing && tr < kGptTraceCap ? p.trace + tr++ : nullptr;
  };
  float v[kPer], gg[kPer], bb[kPer];
  float eb, er;
  const int tokens = p.P + p.max_steps;
  for (int tok = 0; tok < tokens && ok; ++tok) {
    const bool decode = tok >= p.P;
    if (tok == p.P && b == 0 && tid == 0) p.times[1] = globaltimer();
    tracing = p.trace != nullptr && tok == p.P && b == 0 && tid == 0;
    trace_arrivals = p.trace != nullptr && tok == p.P && tid == 0;
    stage_no = 0;
    mark();
    for (int l = 0; l < kLayers && ok; ++l) {
      const GptLayerPtrs& L = sm.layers[l];
      // ---- c_attn(ln_1(x)). Layer 0 builds x (the prefix row, or
      // mel_embedding[code] + mel_pos_embedding[position] as
      // build_gpt_greedy_current_cpu, runtime/impl/gpt.cpp:1545-1554, with
      // gpt_cached_generate_position, :1873-1875) and publishes the CTA's
      // slice of it for the residual of attn.c_proj.
      epi_prefetch<kSQkv>(p, sm, l, eb, er);
      load_params(L.ln1_g, L.ln1_b, gg, bb);
      if (l == 0) {
        const int position = p.hf_positions && step > 0 ? step + 1 : step;
        const float* e0 = decode ? p.emb + static_cast<size_t>(code) * kW : p.prefix + static_cast<size_t>(tok) * kW;
        const float* e1 = p.pos + static_cast<size_t>(position) * kW;
        const int x0 = static_cast<int>(static_cast<long long>(b) * kW / G);
        const int x1 = static_cast<int>(static_cast<long long>(b + 1) * kW / G);
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
          const int i = tid + k * kCons;
          v[k] = i < kW ? (decode ? e0[i] + e1[i] : e0[i]) : 0.0f;
          if (i >= x0 && i < x1) p.x[i] = v[k];
        }
      } else {
        load_row_cg(p.x, v);
      }
      layer_norm_regs(v, gg, bb, sm.red);
      store_row(v, sm.xs);
      mark();
      ok = cons_proj<kSQkv>(p, sm, l, it, eb, er, slot_mark());
      mark();
      ok = ok && sync();
      mark();
      if (!ok) break;
      // ---- attention over the cache with this token appended
      mark();
      if (b < kAttnCtas) cons_attention(p, sm, l, len);
      mark();
      mark();
      ok = sync();
      mark();
      if (!ok) break;
      // ---- h = x + attn.c_proj(merged heads)
      epi_prefetch<kSProj>(p, sm, l, eb, er);
      cons_attn_combine(p, sm.xs, sm.xs + kW);
      mark();
      ok = cons_proj<kSProj>(p, sm, l, it, eb, er, slot_mark());
      mark();
      ok = ok && sync();
      mark();
      if (!ok) break;
      // ---- m = gelu_new(c_fc(ln_2(h)))
      epi_prefetch<kSFc>(p, sm, l, eb, er);
      load_params(L.ln2_g, L.ln2_b, gg, bb);
      load_row_cg(p.h, v);
      layer_norm_regs(v, gg, bb, sm.red);
      store_row(v, sm.xs);
      mark();
      ok = cons_proj<kSFc>(p, sm, l, it, eb, er, slot_mark());
      mark();
      ok = ok && sync();
      mark();
      if (!ok) break;
      // ---- x = h + mlp.c_proj(m)
      epi_prefetch<kSMproj>(p, sm, l, eb, er);
      for (int i = tid; i < kMlp; i += kCons) sm.xs[i] = __ldcg(p.m + i);
      cbar();
      mark();
      ok = cons_proj<kSMproj>(p, sm, l, it, eb, er, slot_mark());
      mark();
      ok = ok && sync();
      mark();
    }
    if (!ok) break;
    ++len;
    if (!decode) continue;
    // ---- ln_f, final_norm, mel head, argmax (runtime/impl/gpt.cpp:1901-1905)
    epi_prefetch<kSHead>(p, sm, 0, eb, er);
    float g2[kPer], b2[kPer];
    load_params(p.lnf_g, p.lnf_b, gg, bb);
    load_params(p.fn_g, p.fn_b, g2, b2);
    load_row_cg(p.x, v);
    layer_norm_regs(v, gg, bb, sm.red);
    layer_norm_regs(v, g2, b2, sm.red);
    store_row(v, sm.xs);
    mark();
    ok = cons_proj<kSHead>(p, sm, 0, it, eb, er, slot_mark());
    mark();
    ok = ok && sync();
    mark();
    if (!ok) break;
    if (p.sample) {  // CTA 0 draws the code; one more barrier publishes it
      if (b == 0) {
        const int c = cons_sample(p, sm);
        if (tid == 0) {
          if (c < 0) atomicCAS(p.status, 0u, kDevSampleTies);
          const int cc = c < 0 ? kStop : c;
          *p.sampled = cc;
          p.codes[step] = static_cast<uint32_t>(cc);
          atomicOr(p.seen + (cc >> 5), 1u << (cc & 31));
        }
      }
      ok = sync();
      if (!ok) break;
      if (tid == 0) sm.flags[2] = __ldcg(p.sampled);
    } else if (tid == 0) {  // candidates in CTA order = row order: the first maximum
      float bv = __ldcg(p.cand_val);
      int bi = __ldcg(p.cand_idx);
      for (int c = 1; c < G; ++c) {
        const float cv = __ldcg(p.cand_val + c);
        if (cv > bv) {
          bv = cv;
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
