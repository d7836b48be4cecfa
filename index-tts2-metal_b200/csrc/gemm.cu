// tcgen05/TMEM GEMM with fused DiT-CFM epilogues (sm_100a).
//
// One CTA computes a 128 x BN output tile. Warp roles (192 threads):
//   warp 0 lane 0 : TMA producer (A and B k-blocks into a STAGES-deep ring)
//   warp 1        : allocates TMEM; lane 0 issues tcgen05.mma (M=128, N=BN, K=16)
//   warps 2..5    : epilogue, one accumulator row per thread (TMEM lane quarter = warp % 4)
// Replaces the reference's MPS GEMM calls and the elementwise kernels that
// followed them (bias prefill, RoPE rotate, silu_mul_split, add, wavenet gate,
// wavenet res/skip update, reflect pad, concat), metal/kernels.metal:131-239,
// 411-464, 820-841, 2390-2428; runtime/metal_context.mm:320-381.
#include <atomic>
#include <cstdio>
#include <mutex>

#include "gemm.cuh"
#include "ptx.cuh"

namespace itts {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 f16 = one 128-byte swizzle row
constexpr int kThreads = 192;

__host__ __device__ constexpr int tmem_cols_for(int bn) { return bn <= 32 ? 32 : bn <= 64 ? 64 : bn <= 128 ? 128 : 256; }

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

// Write 16 channels of one WaveNet activation row into the reflect-padded
// buffer, including every halo slot that mirrors this row.
__device__ __forceinline__ void write_xp16(__half* xp, int s, int t, int T, int col, const float* v) {
  __half* base = xp + static_cast<size_t>(s) * (T + 4) * 512;
  store_h16(base + static_cast<size_t>(t + 2) * 512 + col, v);
  const int halo[4] = {-2, -1, T, T + 1};
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    if (reflect_src(halo[h], T) == t) store_h16(base + static_cast<size_t>(halo[h] + 2) * 512 + col, v);
  }
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
                   const __grid_constant__ CUtensorMap tmB, const GemmArgs args) {
  constexpr int A_BYTES = kBM * kBK * 2;
  constexpr int B_BYTES = BN * kBK * 2;
  constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = tmem_cols_for(BN);
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accum_bar = empty_bar + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum_bar + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM;
  const int n0 = blockIdx.y * BN;
  const int num_kb = args.num_kb;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(accum_bar, 1);
    fence_barrier_init();
    fence_proxy_async_shared();
    prefetch_tmap(&tmA0);
    if (args.a_mode == kASplit) prefetch_tmap(&tmA1);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer ----
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mbar_wait(&empty_bar[s], ph ^ 1, args.status, kDevTimeoutEmpty)) break;
        uint8_t* sa = smem + s * STAGE_BYTES;
        uint8_t* sb = sa + A_BYTES;
        mbar_arrive_expect_tx(&full_bar[s], STAGE_BYTES);
        if (args.a_mode == kAConv5) {
          const int tap = kb / args.kb_per_tap;
          const int kc = kb - tap * args.kb_per_tap;
          tma_load_2d(sa, &tmA0, &full_bar[s], kc * kBK, m0 + tap - 2);
        } else if (args.a_mode == kASplit && kb >= args.kb_split) {
          tma_load_2d(sa, &tmA1, &full_bar[s], (kb - args.kb_split) * kBK, m0);
        } else {
          tma_load_2d(sa, &tmA0, &full_bar[s], kb * kBK, m0);
        }
        tma_load_2d(sb, &tmB, &full_bar[s], kb * kBK, n0);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer ----
      constexpr uint32_t idesc = idesc_f16_f32(kBM, BN);
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mbar_wait(&full_bar[s], ph, args.status, kDevTimeoutFull)) break;
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
        const uint32_t sb = sa + A_BYTES;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          umma_f16_ss(tmem_base, sdesc_k_sw128(sa + k * 32), sdesc_k_sw128(sb + k * 32), idesc,
                      (kb | k) != 0 ? 1u : 0u);
        }
        umma_commit(&empty_bar[s]);
      }
      umma_commit(accum_bar);
    }
    __syncwarp();
  } else {
    // ---- epilogue: warps 2..5 ----
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int m = m0 + row;
    const bool ok = mbar_wait(accum_bar, 0, args.status, kDevTimeoutAccum);
    tc_fence_after();
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    if (ok) {
      const int T = args.seq_T;
      if constexpr (EPI == kEpiSwiGLU || EPI == kEpiWnGate || EPI == kEpiWnResSkip) {
        static_assert(BN % 128 == 0, "paired epilogues need 128-column slabs");
        // Row-space bookkeeping.
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
        if constexpr (EPI == kEpiWnResSkip) msk = row_ok ? args.row_mask[r] : 0.0f;
#pragma unroll 1
        for (int slab = 0; slab < BN / 128; ++slab) {
#pragma unroll 1
          for (int i = 0; i < 4; ++i) {
            const int ca = slab * 128 + i * 16;
            const int na = n0 + ca;
            float a[16], b[16];
            tmem_ld16(taddr + ca, a);
            tmem_ld16(taddr + ca + 64, b);
            if (row_ok && na < args.N) {
            const int ch = (n0 >> 1) + slab * 64 + i * 16;
            if (args.bias) {
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                a[e] += args.bias[na + e];
                b[e] += args.bias[na + 64 + e];
              }
            }
            if constexpr (EPI == kEpiSwiGLU) {
#pragma unroll
              for (int e = 0; e < 16; ++e) a[e] = silu_f(a[e]) * b[e];
              store_h16(args.out16 + static_cast<size_t>(r) * args.ld16 + ch, a);
            } else if constexpr (EPI == kEpiWnGate) {
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                const float ga = a[e] + args.wn_cond[ch + e];
                const float gb = b[e] + args.wn_cond[512 + ch + e];
                a[e] = tanhf(ga) * sigmoid_f(gb);
              }
              store_h16(args.out16 + static_cast<size_t>(r) * args.ld16 + ch, a);
            } else {  // kEpiWnResSkip
              float x[16];
              __half* xrow = args.wn_xp + (static_cast<size_t>(s) * (T + 4) + t + 2) * 512 + ch;
              load_h16(xrow, x);
#pragma unroll
              for (int e = 0; e < 16; ++e) x[e] = (x[e] + a[e]) * msk;
              write_xp16(args.wn_xp, s, t, T, ch, x);
              float* acc = args.wn_acc + static_cast<size_t>(r) * 512 + ch;
              if (!args.wn_first) {
                float o[16];
                load_f32x16(acc, o);
#pragma unroll
                for (int e = 0; e < 16; ++e) b[e] += o[e];
              }
              store_f32x16(acc, b);
            }
            }
          }
        }
      } else {
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
        float msk = 1.0f;
        if constexpr (EPI == kEpiWnLast) msk = row_ok ? args.row_mask[m] : 0.0f;
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          const int n = n0 + c;
          float v[16];
          tmem_ld16(taddr + c, v);
          if (row_ok && n < args.N) {
          if (args.bias) {
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] += args.bias[n + e];
          }
          if constexpr (EPI == kEpiF16) {
            store_h16(args.out16 + static_cast<size_t>(m) * args.ld16 + n, v);
          } else if constexpr (EPI == kEpiF32) {
            if (args.resid32) {
              float rr[16];
              load_f32x16(args.resid32 + static_cast<size_t>(mo) * args.ldr + n, rr);
#pragma unroll
              for (int e = 0; e < 16; ++e) v[e] += rr[e];
            }
            store_f32x16(args.out32 + static_cast<size_t>(mo) * args.ld32 + n, v);
            if (args.out16) store_h16(args.out16 + static_cast<size_t>(mo) * args.ld16 + n, v);
          } else if constexpr (EPI == kEpiQKV) {
            if (n < 1024) {
              const int d0 = n & 63;  // column inside the head
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float2 cs = args.rope[static_cast<size_t>(t) * 32 + (d0 >> 1) + e];
                const float x0 = v[2 * e], x1 = v[2 * e + 1];
                v[2 * e] = x0 * cs.x - x1 * cs.y;
                v[2 * e + 1] = x1 * cs.x + x0 * cs.y;
              }
              if (n < 512) {
#pragma unroll
                for (int e = 0; e < 16; ++e) v[e] *= 0.125f;
              }
            }
            store_h16(args.out16 + static_cast<size_t>(m) * args.ld16 + n, v);
          } else if constexpr (EPI == kEpiWnLast) {
            float o[16], rr[16];
            load_f32x16(args.wn_acc + static_cast<size_t>(m) * 512 + n, o);
            load_f32x16(args.wn_res + static_cast<size_t>(m) * 512 + n, rr);
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] = (o[e] + v[e]) * msk + rr[e];
            store_f32x16(args.out32 + static_cast<size_t>(m) * args.ld32 + n, v);
          } else if constexpr (EPI == kEpiConv1Res) {
            if (n < 512) {
              write_xp16(args.wn_xp, s, t, T, n, v);
            } else {
              store_f32x16(args.out32 + static_cast<size_t>(m) * args.ld32 + (n - 512), v);
            }
          }
          }
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
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

template <int BN, int STAGES, int EPI>
cudaError_t launch_t(const GemmLaunch& g, cudaStream_t stream) {
  auto kern = gemm_tc_kernel<BN, STAGES, EPI>;
  const size_t smem = gemm_smem_bytes(BN, STAGES);
  // The shared-memory opt-in is set once per device for each instantiation.
  static std::atomic<uint32_t> configured{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint32_t bit = 1u << (dev & 31);
  if ((configured.load() & bit) == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit);
  }
  dim3 grid((g.args.M + kBM - 1) / kBM, (g.args.N + BN - 1) / BN);
  kern<<<grid, kThreads, smem, stream>>>(g.tmA0, g.tmA1, g.tmB, g.args);
  return cudaGetLastError();
}

template <int BN, int STAGES>
cudaError_t launch_epi(const GemmLaunch& g, cudaStream_t stream) {
  switch (g.args.epi) {
    case kEpiF16: return launch_t<BN, STAGES, kEpiF16>(g, stream);
    case kEpiF32: return launch_t<BN, STAGES, kEpiF32>(g, stream);
    case kEpiQKV: return launch_t<BN, STAGES, kEpiQKV>(g, stream);
    case kEpiWnLast: return launch_t<BN, STAGES, kEpiWnLast>(g, stream);
    case kEpiConv1Res: return launch_t<BN, STAGES, kEpiConv1Res>(g, stream);
    default: break;
  }
  if constexpr (BN % 128 == 0) {
    switch (g.args.epi) {
      case kEpiSwiGLU: return launch_t<BN, STAGES, kEpiSwiGLU>(g, stream);
      case kEpiWnGate: return launch_t<BN, STAGES, kEpiWnGate>(g, stream);
      case kEpiWnResSkip: return launch_t<BN, STAGES, kEpiWnResSkip>(g, stream);
      default: break;
    }
  }
  return cudaErrorInvalidValue;
}

}  // namespace

size_t gemm_smem_bytes(int bn, int stages) {
  return 1024 /*alignment slack*/ + static_cast<size_t>(stages) * (kBM * kBK * 2 + bn * kBK * 2) + 256;
}

bool make_tmap_f16(CUtensorMap* tm, const void* base, uint64_t cols, uint64_t rows, uint64_t ld_elems,
                   uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || !base) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld_elems * 2) % 16 != 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld_elems * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

cudaError_t gemm_run(const GemmLaunch& g, cudaStream_t stream) {
  if (g.args.M <= 0 || g.args.N <= 0 || g.args.num_kb <= 0) return cudaErrorInvalidValue;
  switch (g.bn) {
    case 80: return launch_epi<80, 4>(g, stream);
    case 128: return g.stages <= 3 ? launch_epi<128, 3>(g, stream) : launch_epi<128, 4>(g, stream);
    case 256: return launch_epi<256, 4>(g, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace itts
