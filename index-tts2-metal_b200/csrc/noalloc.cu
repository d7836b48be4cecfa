// itts_op_conv5_noalloc: the k=5 reflect-padded WaveNet convolution for
// callers that must not allocate device memory.
//
// The conv's implicit GEMM reads a reflect-padded staging copy of its input
// (two halo rows on each side of every sequence). itts_op_conv5 makes the
// caller build that copy in memory of its own; this entry point builds it in a
// fixed device array that belongs to the library instead, so the caller passes
// only the unpadded input, the weights and the output. The array is a
// file-scope __device__ variable: it is reserved when this module is loaded on
// a device (with CUDA's default lazy module loading, at the first call on that
// device) and held until the process exits.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "gemm.cuh"
#include "itts_cfm.h"

namespace {

constexpr uint32_t kChannels = 512;                     // WaveNet hidden width (conv input channels)
constexpr size_t kStatusBytes = 256;                    // bounded-wait status word, padded to 256 B
constexpr size_t kRowBytes = kChannels * sizeof(__half);  // one padded staging row
constexpr size_t kScratchBytes = kStatusBytes + static_cast<size_t>(ITTS_NOALLOC_CONV5_MAX_ROWS) * kRowBytes;

// [status word | 252 B unused | padded rows [ITTS_NOALLOC_CONV5_MAX_ROWS][512] f16]
static __device__ __align__(256) unsigned char g_conv5_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_conv5_scratch on the current device. In host code the
// symbol names a host-side shadow, never device memory, so the address is
// looked up once per device with that device current and cached.
cudaError_t scratch_address(int dev, unsigned char** out) {
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_conv5_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_addr[dev] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_addr[dev]);
  return cudaSuccess;
}

// Source row of the reflect padding for halo position j in [-2, T+2) (the
// same repeated reflection the engine's epilogues write; T >= 2).
__device__ __forceinline__ int reflect_row(int j, int T) {
  int src = j;
#pragma unroll 1
  for (int it = 0; it < 8 && (src < 0 || src >= T); ++it) {
    if (src < 0) src = -src;
    if (src >= T) src = 2 * T - 2 - src;
  }
  return src;
}

// x [S*T][512] f16 -> scratch rows [S*(T+4)][512] f16, four rows per block of
// 256 threads (64 x 16 B per row). Block 0 also clears the status word, which
// the conv kernel only writes if one of its waits gives up.
__global__ void __launch_bounds__(256) pad_into_scratch(const uint4* __restrict__ x, int S, int T) {
  uint4* rows = reinterpret_cast<uint4*>(g_conv5_scratch + kStatusBytes);
  if (blockIdx.x == 0 && threadIdx.x == 0) *reinterpret_cast<unsigned int*>(g_conv5_scratch) = 0u;
  const long long row = static_cast<long long>(blockIdx.x) * 4 + (threadIdx.x >> 6);
  const int piece = threadIdx.x & 63;
  if (row >= static_cast<long long>(S) * (T + 4)) return;
  const long long s = row / (T + 4);
  const int t = reflect_row(static_cast<int>(row - s * (T + 4)) - 2, T);
  rows[row * 64 + piece] = x[(s * T + t) * 64 + piece];
}

void put_err(char* err, uint32_t cap, const char* msg) {
  if (err && cap > 0) std::snprintf(err, cap, "%s", msg);
}

}  // namespace

extern "C" int itts_op_conv5_noalloc(const void* x, uint32_t S, uint32_t T, const void* w, const float* bias,
                                     float* out, uint32_t N, void* stream, char* err, uint32_t err_cap) {
  put_err(err, err_cap, "");
  // N is tiled by 128-column weight boxes with no partial tile (the WaveNet
  // conv this serves has N = 1024).
  if (!x || !w || !out || S == 0 || N == 0 || N % 128 != 0 || T < ITTS_MIN_T) {
    put_err(err, err_cap, "bad conv arguments (x, w, out non-null; S > 0; T >= 2; N a positive multiple of 128)");
    return ITTS_EINVAL_SHAPE;
  }
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15)) {
    put_err(err, err_cap, "x and w must be 16-byte aligned");
    return ITTS_EINVAL_SHAPE;
  }
  const uint64_t rows = static_cast<uint64_t>(S) * (static_cast<uint64_t>(T) + 4);
  if (T > ITTS_MAX_T || rows > ITTS_NOALLOC_CONV5_MAX_ROWS) {
    char msg[192];
    std::snprintf(msg, sizeof(msg),
                  "S*(T+4) = %llu padded rows exceeds the static scratch of %u rows (16 MiB); use itts_op_conv5",
                  static_cast<unsigned long long>(rows), ITTS_NOALLOC_CONV5_MAX_ROWS);
    put_err(err, err_cap, msg);
    return ITTS_ECAP;
  }
  auto fail = [&](cudaError_t e, const char* what) {
    char msg[192];
    std::snprintf(msg, sizeof(msg), "cuda: %s: %s", what, cudaGetErrorString(e));
    put_err(err, err_cap, msg);
    return ITTS_ECUDA;
  };
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(e, "get device");
  if (dev < 0 || dev >= kMaxDevices) {
    put_err(err, err_cap, "device ordinal beyond the 64 this entry point tracks");
    return ITTS_ENODEV;
  }
  unsigned char* scratch = nullptr;
  if ((e = scratch_address(dev, &scratch)) != cudaSuccess) return fail(e, "scratch symbol address");
  unsigned int* status = reinterpret_cast<unsigned int*>(scratch);
  const __half* xp = reinterpret_cast<const __half*>(scratch + kStatusBytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  itts::GemmLaunch g;
  std::memset(&g, 0, sizeof(g));
  if (!itts::make_tmap_f16(&g.tmA0, xp, kChannels, rows, kChannels, 128, 2)) {
    put_err(err, err_cap, "scratch layout rejected by TMA");
    return ITTS_ECUDA;
  }
  g.tmA1 = g.tmA0;
  if (!itts::make_tmap_f16(&g.tmB, w, 5 * kChannels, N, 5 * kChannels, 128, 2)) {
    put_err(err, err_cap, "w layout rejected by TMA");
    return ITTS_EINVAL_SHAPE;
  }
  g.args.M = static_cast<int>(rows);
  g.args.N = static_cast<int>(N);
  g.args.a_mode = itts::kAConv;
  g.args.kb_per_tap = 8;
  g.args.conv_dil = 1;
  g.args.conv_off = -2;
  g.args.num_kb = 40;
  g.args.epi = itts::kEpiF32;
  g.args.pad_rows = 1;
  g.args.bias = bias;
  g.args.out32 = out;
  g.args.ld32 = static_cast<int>(N);
  g.args.seq_T = static_cast<int>(T);
  g.args.status = status;
  g.bn = 128;
  g.pair = 0;

  const unsigned blocks = static_cast<unsigned>((rows + 3) / 4);
  pad_into_scratch<<<blocks, 256, 0, st>>>(static_cast<const uint4*>(x), static_cast<int>(S), static_cast<int>(T));
  if ((e = cudaGetLastError()) != cudaSuccess) return fail(e, "pad launch");
  if ((e = itts::gemm_run(g, st)) != cudaSuccess) return fail(e, "conv launch");
  unsigned int s = 0;
  if ((e = cudaMemcpyAsync(&s, status, sizeof(s), cudaMemcpyDeviceToHost, st)) != cudaSuccess)
    return fail(e, "status read");
  if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return fail(e, "conv sync");
  if (s != 0) {
    char msg[96];
    std::snprintf(msg, sizeof(msg), "a kernel abandoned a bounded wait (device status %u)", s);
    put_err(err, err_cap, msg);
    return ITTS_ETIMEOUT;
  }
  return ITTS_OK;
}
