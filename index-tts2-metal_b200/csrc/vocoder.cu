// BigVGAN vocoder: weight preparation, the activation / mean / post kernels
// and the launch schedule (see vocoder.hpp).
#include "vocoder.hpp"

#include <cmath>
#include <cstring>
#include <stdexcept>

#include "bundle.hpp"
#include "launch.cuh"
#include "ptx.cuh"

namespace itts {

namespace {

constexpr int kUps[6][5] = {{1536, 768, 8, 4, 2}, {768, 384, 8, 4, 2}, {384, 192, 4, 2, 1},
                            {192, 96, 4, 2, 1},   {96, 48, 4, 2, 1},   {48, 24, 4, 2, 1}};
constexpr int kRbKernel[3] = {3, 7, 11};
constexpr int kDil[3] = {1, 3, 5};
constexpr int kHop = 256;
enum : unsigned int { kDevTimeoutVocoder = 24 };

int pad64(int c) { return (c + 63) / 64 * 64; }

// ---------------------------------------------------------------------------
// Kernels
// ---------------------------------------------------------------------------

// Anti-aliased SnakeBeta (cpu_bigvgan_activation,
// runtime/impl/tokenizer_tests.cpp:3785-3834) on x [T][ldx] (f32, channels
// [0, C)): 2x upsampling u(j) = 2 sum_k x[clamp((j + 15 - k)/2 - 5)] up[k]
// over the taps k of j's parity, v(j) = u + sin^2(alpha u) / (beta + 1e-9)
// (computed as u + sin^2(alpha u) * (1 / (beta + 1e-9)), the reciprocal folded
// at load), then out(t) = sum_k v(clamp(2t + k - 5, 0, 2T - 1)) down[k].
// With j = 2m + rho the taps of each parity are fixed:
//   u(2m)     = 2 sum_{i<6} x[m + 2 - i] up[2i + 1]
//   u(2m + 1) = 2 sum_{i<6} x[m + 3 - i] up[2i]
// (i ascending is the reference's k order). A block owns 64 tokens x 32
// channels (lanes along channels): it stages the 76 edge-replicated input rows,
// computes v at the 140 positions 2 t0 - 6 .. 2 t0 + 133 as 70 (even, odd)
// pairs (positions outside [0, 2T) hold v at the clamped position, as the
// downsampler reads it), then each warp produces 8 consecutive outputs per
// lane from a 26-value window of v.
constexpr int kActTT = 64;
constexpr int kActCC = 32;
constexpr int kActPos = 2 * kActTT + 12;  // v positions per block

// sin(x) for the snake term: x reduced to [-pi, pi] by a two-part Cody-Waite
// split of 2 pi (6.28318548f + (-1.7484556e-7f), the float nearest 2 pi and its
// remainder), then the SFU sine (absolute error about 5e-7 there, far below
// the 4.9e-4 rounding of the f16 operand the activation feeds).
__device__ __forceinline__ float sin_reduced(float x) {
  const float k = rintf(x * 0.15915494f);  // x / (2 pi), rounded to an integer
  float r = fmaf(-k, 6.28318548f, x);
  r = fmaf(-k, -1.7484556e-7f, r);
  return __sinf(r);
}

__device__ __forceinline__ float snake(float u, float a, float ib) {
  const float s = sin_reduced(u * a);
  return fmaf(s * s, ib, u);
}

// The two 12-tap filters travel by value (kernel parameters live in the
// constant bank, which FMAs read as an operand without a load). up2 holds
// 2 * up: the upsampler's factor 2 folded into the taps, which is exact (a
// power-of-two scale commutes with every rounding of the FMA chain, outside
// the subnormal range).
struct SnakeFilters {
  float up2[12];
  float down[12];
};

// One block's tile (tokens t0 .. t0 + 63, 32 channels). EDGE = false is the
// interior form: every input row, pair and output of the tile lies inside
// [0, T), so no index is clamped and no position is checked.
template <bool F16OUT, bool EDGE>
__device__ __forceinline__ void snake_tile(float (&xs)[kActTT + 12][kActCC], float (&vs)[kActPos][kActCC],
                                           const float* __restrict__ x, int ldx, int T, int C, int cw,
                                           const float* __restrict__ alpha, const float* __restrict__ inv_beta,
                                           const SnakeFilters& f, void* __restrict__ out, int ldo, int t0, int c,
                                           int lane, int w) {
  const bool cok = c < C;
  // Warp w stages rows w, w + 8, ..., all its loads issued before the first
  // shared-memory store, so their DRAM latencies overlap.
  constexpr int kRowsPerWarp = (kActTT + 12 + 7) / 8;
  float ld[kRowsPerWarp];
#pragma unroll
  for (int j = 0; j < kRowsPerWarp; ++j) {
    const int i = w + 8 * j;
    int r = t0 - 6 + i;
    if constexpr (EDGE) r = r < 0 ? 0 : (r > T - 1 ? T - 1 : r);
    ld[j] = (cok && i < kActTT + 12) ? x[static_cast<size_t>(r) * ldx + c] : 0.0f;
  }
#pragma unroll
  for (int j = 0; j < kRowsPerWarp; ++j) {
    const int i = w + 8 * j;
    if (i < kActTT + 12) xs[i][lane] = ld[j];
  }
  __syncthreads();
  const float a = cok ? alpha[c] : 1.0f;
  const float ib = cok ? inv_beta[c] : 1.0f;
  // x row index in xs of source row (m + d) for the pair at m: m + d - (t0 - 6).
  auto u_even = [&](int xi) {  // u(2m), xi = index of row m + 2
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < 6; ++i) acc += xs[xi - i][lane] * f.up2[2 * i + 1];
    return acc;
  };
  auto u_odd = [&](int xi) {  // u(2m + 1), xi = index of row m + 3
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < 6; ++i) acc += xs[xi - i][lane] * f.up2[2 * i];
    return acc;
  };
  // Warp w computes the pairs q = 9 w .. 9 w + 8 (q < 70). Interior pairs read
  // their rows q .. q + 6 of xs from a register window of rows 9 w .. 9 w + 14,
  // loaded once per warp; pairs at the sequence edges take the clamped path.
  constexpr int kPairsPerWarp = 9;
  float xw[kPairsPerWarp + 6];
#pragma unroll
  for (int i = 0; i < kPairsPerWarp + 6; ++i) {
    const int r = kPairsPerWarp * w + i;
    xw[i] = r < kActTT + 12 ? xs[r][lane] : 0.0f;
  }
#pragma unroll
  for (int jq = 0; jq < kPairsPerWarp; ++jq) {
    const int q = kPairsPerWarp * w + jq;
    if (q >= kActPos / 2) break;
    const int m = t0 - 3 + q;  // positions 2m = 2 t0 - 6 + 2q and 2m + 1
    float v0, v1;
    if (!EDGE || (m >= 0 && m < T)) {
      // Rows m - 3 .. m + 3 are xs rows q .. q + 6, i.e. xw[jq .. jq + 6].
      float ue = 0.0f, uo = 0.0f;
#pragma unroll
      for (int i = 0; i < 6; ++i) {
        ue += xw[jq + 5 - i] * f.up2[2 * i + 1];
        uo += xw[jq + 6 - i] * f.up2[2 * i];
      }
      v0 = snake(ue, a, ib);
      v1 = snake(uo, a, ib);
    } else {
      // Edge: each position takes v at its clamped position j.
      float vv[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        int j = 2 * m + h;
        j = j < 0 ? 0 : (j > 2 * T - 1 ? 2 * T - 1 : j);
        const int mj = j >> 1;
        // Row (mj + d) sits at xs index mj + d - (t0 - 6); its clamped source
        // lies in the staged rows because j is within the block's window.
        vv[h] = (j & 1) ? snake(u_odd(mj + 3 - (t0 - 6)), a, ib) : snake(u_even(mj + 2 - (t0 - 6)), a, ib);
      }
      v0 = vv[0];
      v1 = vv[1];
    }
    vs[2 * q][lane] = v0;
    vs[2 * q + 1][lane] = v1;
  }
  __syncthreads();
  // The next kernel (a conv GEMM) may start its prologue once every block is
  // in its store phase; it waits for this grid before reading `out`.
  griddep_launch();
  if (c >= cw) return;
  // Warp w: outputs t0 + 8w .. t0 + 8w + 7; output t reads positions
  // 2t - 5 .. 2t + 6, i.e. vs[2(t - t0) + 1 .. 2(t - t0) + 12].
  const int tb = 8 * w;
  float win[26];
#pragma unroll
  for (int i = 0; i < 26; ++i) win[i] = vs[2 * tb + 1 + i][lane];
  const size_t o0 = static_cast<size_t>(t0 + tb) * ldo + c;
#pragma unroll
  for (int o = 0; o < 8; ++o) {
    if (EDGE && t0 + tb + o >= T) break;
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < 12; ++k) acc += win[2 * o + k] * f.down[k];
    if (!cok) acc = 0.0f;
    if constexpr (F16OUT) {
      static_cast<__half*>(out)[o0 + static_cast<size_t>(o) * ldo] = __float2half_rn(acc);
    } else {
      static_cast<float*>(out)[o0 + static_cast<size_t>(o) * ldo] = acc;
    }
  }
}

// Output columns [C, cw) (the f16 operand's channel padding) are written as 0;
// a block whose 32 channels are all padding only writes those zeros.
template <bool F16OUT>
__global__ void __launch_bounds__(256, 6) snake_aa_kernel(const float* __restrict__ x, int ldx, int T, int C, int cw,
                                                       const float* __restrict__ alpha,
                                                       const float* __restrict__ inv_beta, const SnakeFilters f,
                                                       void* __restrict__ out, int ldo) {
  __shared__ float xs[kActTT + 12][kActCC];  // xs[i] = x[clamp(t0 - 6 + i)]
  __shared__ float vs[kActPos][kActCC];      // vs[i] = v(clamp(2 t0 - 6 + i))
  // Launched with programmatic dependent launch: nothing of the previous
  // kernel's memory (its output x, or the operand `out` it may still read) is
  // touched before this wait.
  griddep_wait();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int t0 = blockIdx.x * kActTT;
  const int c = blockIdx.y * kActCC + lane;
  if (blockIdx.y * kActCC >= C) {  // padding columns only
    if constexpr (F16OUT) {
      if (c < cw)
        for (int tt = w; tt < kActTT && t0 + tt < T; tt += 8)
          static_cast<__half*>(out)[static_cast<size_t>(t0 + tt) * ldo + c] = __float2half_rn(0.0f);
    }
    return;
  }
  // Interior tile: rows t0 - 6 .. t0 + 69 all inside [0, T).
  if (t0 >= 6 && t0 + kActTT + 6 <= T) {
    snake_tile<F16OUT, false>(xs, vs, x, ldx, T, C, cw, alpha, inv_beta, f, out, ldo, t0, c, lane, w);
  } else {
    snake_tile<F16OUT, true>(xs, vs, x, ldx, T, C, cw, alpha, inv_beta, f, out, ldo, t0, c, lane, w);
  }
}

// Mean of a stage's three resblocks, accumulated as the reference does
// (out = 0; out += rb / 3 per resblock, runtime/impl/dit_cfm_bigvgan.cpp:
// 3982-3994): acc = (first ? 0 : acc) + rb / 3 over rows x C. With h16 (the
// last resblock) it also writes the f16 operand of the next upsampler, rows
// of ldh >= C columns with the padding columns set to 0. Each thread handles
// 4 consecutive channels (C and ldh are multiples of 4: every stage width is);
// the grid covers rows x (w / 4) groups with a 32-bit row/group split per
// grid-stride step (w / 4 <= 384).
__global__ void __launch_bounds__(256) group_mean_kernel(float* __restrict__ acc, const float* __restrict__ rb,
                                                         size_t rows, int C, int first, __half* __restrict__ h16,
                                                         int ldh) {
  griddep_wait();
  griddep_launch();
  const unsigned w4 = static_cast<unsigned>((h16 ? ldh : C) >> 2);
  const unsigned c4n = static_cast<unsigned>(C >> 2);
  const size_t n = rows * w4;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  // Row and group of the first index; later steps advance by the stride's
  // (rows, groups) decomposition, so no 64-bit division runs in the loop.
  size_t r = i / w4;
  unsigned g = static_cast<unsigned>(i - r * w4);
  const size_t sr = stride / w4;
  const unsigned sg = static_cast<unsigned>(stride - sr * w4);
  for (; r < rows;) {
    if (g >= c4n) {
      const __half2 z = __float2half2_rn(0.0f);
      __half2* hp = reinterpret_cast<__half2*>(h16 + r * ldh + 4 * g);
      hp[0] = z;
      hp[1] = z;
    } else {
      const size_t k = r * C + 4 * g;
      const float4 b = *reinterpret_cast<const float4*>(rb + k);
      float4 v = first ? make_float4(0.0f, 0.0f, 0.0f, 0.0f) : *reinterpret_cast<const float4*>(acc + k);
      v.x += b.x / 3.0f;
      v.y += b.y / 3.0f;
      v.z += b.z / 3.0f;
      v.w += b.w / 3.0f;
      *reinterpret_cast<float4*>(acc + k) = v;
      if (h16) {
        __half2* hp = reinterpret_cast<__half2*>(h16 + r * ldh + 4 * g);
        hp[0] = __floats2half2_rn(v.x, v.y);
        hp[1] = __floats2half2_rn(v.z, v.w);
      }
    }
    r += sr;
    g += sg;
    if (g >= w4) {
      g -= w4;
      ++r;
    }
  }
}

// mel [T][80] f32 -> [T][128] f16 operand of conv_pre (columns >= 80 zero).
__global__ void __launch_bounds__(256) mel_to_f16_kernel(const float* __restrict__ mel, int T,
                                                         __half* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  const size_t n = static_cast<size_t>(T) * 128;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t t = i >> 7;
    const int c = static_cast<int>(i & 127);
    out[i] = __float2half_rn(c < 80 ? mel[t * 80 + c] : 0.0f);
  }
}

// conv_post (k=7, 24 -> 1, zero-padded "same", no bias; cpu_conv1d_same,
// runtime/impl/tokenizer_tests.cpp:3142-3161, sums over in-channel then tap)
// and the clamp to [-1, 1] of run_bigvgan_post_cpu
// (runtime/impl/dit_cfm_bigvgan.cpp:4030-4039). a: [T][24] f32.
__global__ void __launch_bounds__(256) conv_post_kernel(const float* __restrict__ a, int T,
                                                        const float* __restrict__ w, float* __restrict__ wave) {
  __shared__ float ws[24 * 7];
  griddep_wait();
  griddep_launch();
  for (int i = threadIdx.x; i < 24 * 7; i += blockDim.x) ws[i] = w[i];
  __syncthreads();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  float acc = 0.0f;
  for (int ci = 0; ci < 24; ++ci) {
#pragma unroll
    for (int k = 0; k < 7; ++k) {
      const int src = t + k - 3;
      if (src >= 0 && src < T) acc += a[static_cast<size_t>(src) * 24 + ci] * ws[ci * 7 + k];
    }
  }
  wave[t] = fmaxf(-1.0f, fminf(1.0f, acc));
}

unsigned grid_for(size_t n) {
  size_t b = (n + 255) / 256;
  return static_cast<unsigned>(b < 148 * 16 ? (b ? b : 1) : 148 * 16);
}

// ---------------------------------------------------------------------------
// Host weight preparation
// ---------------------------------------------------------------------------

// W[r] = g[r] v[r] / ||v[r]|| over rows of `cols` values (weight_norm_rowmajor,
// runtime/impl/gpt.cpp:5109-5136), fp32 as the reference computes it.
std::vector<float> weight_norm(const Mit2Bundle& b, const std::string& prefix, int rows, int cols) {
  std::vector<float> g = b.as_f32(prefix + ".weight_g");
  std::vector<float> v = b.as_f32(prefix + ".weight_v");
  if (g.size() != static_cast<size_t>(rows) || v.size() != static_cast<size_t>(rows) * cols)
    throw std::runtime_error("vocoder weights: " + prefix + " has an unexpected shape");
  std::vector<float> w(v.size());
  for (int r = 0; r < rows; ++r) {
    float nrm = 0.0f;
    for (int c = 0; c < cols; ++c) nrm += v[static_cast<size_t>(r) * cols + c] * v[static_cast<size_t>(r) * cols + c];
    nrm = std::sqrt(nrm);
    const float s = g[r] / nrm;
    for (int c = 0; c < cols; ++c) w[static_cast<size_t>(r) * cols + c] = v[static_cast<size_t>(r) * cols + c] * s;
  }
  return w;
}

std::vector<float> vec_of(const Mit2Bundle& b, const std::string& n, size_t want) {
  std::vector<float> v = b.as_f32(n);
  if (v.size() != want) throw std::runtime_error("vocoder weights: " + n + " has an unexpected size");
  return v;
}

// Device arena filled from host payloads (one allocation, one copy).
class Arena {
 public:
  template <typename T>
  size_t add(const std::vector<T>& v) {
    const size_t off = bytes_.size();
    const size_t n = v.size() * sizeof(T);
    bytes_.resize(off + ((n + 255) & ~size_t(255)), 0);
    std::memcpy(bytes_.data() + off, v.data(), n);
    return off;
  }
  void* upload() {
    void* d = nullptr;
    if (cudaMalloc(&d, bytes_.size()) != cudaSuccess) throw std::runtime_error("vocoder weights: cudaMalloc failed");
    if (cudaMemcpy(d, bytes_.data(), bytes_.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
      cudaFree(d);
      throw std::runtime_error("vocoder weights: upload failed");
    }
    bytes_.clear();
    bytes_.shrink_to_fit();
    return d;
  }

 private:
  std::vector<uint8_t> bytes_;
};

struct Pending {
  VocConv* conv;
  size_t w_off, b_off;
};
struct PendingAct {
  VocAct* act;
  size_t a_off, b_off;
};

}  // namespace

// ---------------------------------------------------------------------------
// Plan: buffers, GEMM launches and the graph for one utterance length
// ---------------------------------------------------------------------------

struct Vocoder::Plan {
  int T = 0;
  void* mem = nullptr;
  float* mel32 = nullptr;   // [T][80]
  __half* mel16 = nullptr;  // [T][128]
  __half* in16 = nullptr;   // upsampler / conv_pre operand
  __half* a16 = nullptr;    // activation output (conv operand)
  float* y32 = nullptr;     // upsampler output (resblock input)
  float* xr32 = nullptr;    // resblock residual stream
  float* h32 = nullptr;     // conv1 output / post activation output
  float* acc32 = nullptr;   // stage mean
  float* wave = nullptr;    // [256 T]
  GemmLaunch pre;
  std::vector<GemmLaunch> ups[6];
  GemmLaunch c1[6][3][3], c2[6][3][3];
  cudaGraphExec_t graph = nullptr;
  int kernels = 0;
};

void Vocoder::check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string("cuda: vocoder: ") + what + ": " + cudaGetErrorString(e));
}

Vocoder::Vocoder(const std::string& bundle_dir, int device, bool verify_sha256) : device_(device) {
  int n = 0;
  check(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
  if (device < 0 || device >= n) throw std::runtime_error("device id out of range");
  check(cudaSetDevice(device), "cudaSetDevice");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10 || minor != 0) throw std::runtime_error("this build targets sm_100a (B200) only");
  load(bundle_dir, verify_sha256);
  check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
  check(cudaMalloc(&d_status_, sizeof(unsigned int)), "cudaMalloc status");
  check(cudaMemset(d_status_, 0, sizeof(unsigned int)), "cudaMemset status");
}

Vocoder::~Vocoder() {
  cudaSetDevice(device_);
  if (stream_) cudaStreamSynchronize(stream_);
  for (auto& kv : plans_) {
    if (kv.second->graph) cudaGraphExecDestroy(kv.second->graph);
    if (kv.second->mem) cudaFree(kv.second->mem);
  }
  if (arena_) cudaFree(arena_);
  if (d_status_) cudaFree(d_status_);
  if (stream_) cudaStreamDestroy(stream_);
}

unsigned int Vocoder::read_status() {
  unsigned int v = 0;
  check(cudaMemcpyAsync(&v, d_status_, sizeof(v), cudaMemcpyDeviceToHost, stream_), "status read");
  check(cudaStreamSynchronize(stream_), "status sync");
  return v;
}

void Vocoder::clear_status() { check(cudaMemsetAsync(d_status_, 0, sizeof(unsigned int), stream_), "status clear"); }

void Vocoder::load(const std::string& bundle_dir, bool verify_sha256) {
  Mit2Bundle b(bundle_dir, verify_sha256);
  Arena ar;
  std::vector<Pending> pend;
  std::vector<PendingAct> pacts;
  // Conv1d weight W[o][i][k] -> GEMM operand [o][k][cin_pad] f16.
  auto conv1d = [&](VocConv* cv, const std::string& prefix, int cin, int cout, int k, int dil, bool bias) {
    std::vector<float> w = weight_norm(b, prefix, cout, cin * k);
    const int cp = pad64(cin);
    std::vector<uint16_t> h(static_cast<size_t>(cout) * k * cp, 0);
    for (int o = 0; o < cout; ++o)
      for (int i = 0; i < cin; ++i)
        for (int kk = 0; kk < k; ++kk)
          h[(static_cast<size_t>(o) * k + kk) * cp + i] = float_to_half_bits(w[(static_cast<size_t>(o) * cin + i) * k + kk]);
    std::vector<float> bv = bias ? vec_of(b, prefix + ".bias", cout) : std::vector<float>(cout, 0.0f);
    cv->cin = cin;
    cv->cin_pad = cp;
    cv->cout = cout;
    cv->taps = k;
    cv->dil = dil;
    cv->off = -(k - 1) * dil / 2;
    pend.push_back({cv, ar.add(h), ar.add(bv)});
  };
  auto act = [&](VocAct* a, const std::string& prefix, int c) {
    std::vector<float> al = vec_of(b, prefix + ".act.alpha", c);
    std::vector<float> be = vec_of(b, prefix + ".act.beta", c);
    for (int i = 0; i < c; ++i) {
      al[i] = std::exp(al[i]);
      be[i] = 1.0f / (std::exp(be[i]) + 1e-9f);
    }
    a->c = c;
    const std::vector<float> fu = vec_of(b, prefix + ".upsample.filter", 12);
    const std::vector<float> fd = vec_of(b, prefix + ".downsample.lowpass.filter", 12);
    std::memcpy(a->up, fu.data(), sizeof(a->up));
    std::memcpy(a->down, fd.data(), sizeof(a->down));
    pacts.push_back({a, ar.add(al), ar.add(be)});
  };
  conv1d(&pre_, "bigvgan.conv_pre", 80, 1536, 7, 1, true);
  for (int i = 0; i < 6; ++i) {
    VocStage& s = st_[i];
    s.cin = kUps[i][0];
    s.cout = kUps[i][1];
    s.k = kUps[i][2];
    s.s = kUps[i][3];
    s.p = kUps[i][4];
    const std::string up = "bigvgan.ups." + std::to_string(i) + ".0";
    // Transposed conv W[ci][co][kk] (runtime/impl/tokenizer_tests.cpp:3760-3783):
    // output row s q + r takes taps kk = k0 + i s (k0 = (r + p) mod s) from
    // input rows q + (r + p) / s - i, i = 0 .. k/s - 1.
    std::vector<float> w = weight_norm(b, up, s.cin, s.cout * s.k);
    std::vector<float> bv = vec_of(b, up + ".bias", s.cout);
    const int cp = pad64(s.cin);
    const int taps = s.k / s.s;
    s.phase.resize(s.s);
    for (int r = 0; r < s.s; ++r) {
      const int k0 = (r + s.p) % s.s;
      std::vector<uint16_t> h(static_cast<size_t>(s.cout) * taps * cp, 0);
      for (int co = 0; co < s.cout; ++co)
        for (int t = 0; t < taps; ++t)
          for (int ci = 0; ci < s.cin; ++ci)
            h[(static_cast<size_t>(co) * taps + t) * cp + ci] =
                float_to_half_bits(w[(static_cast<size_t>(ci) * s.cout + co) * s.k + k0 + t * s.s]);
      VocConv& cv = s.phase[r];
      cv.cin = s.cin;
      cv.cin_pad = cp;
      cv.cout = s.cout;
      cv.taps = taps;
      cv.dil = -1;
      cv.off = (r + s.p) / s.s;
      pend.push_back({&cv, ar.add(h), ar.add(bv)});
    }
    for (int j = 0; j < 3; ++j) {
      const std::string rb = "bigvgan.resblocks." + std::to_string(3 * i + j);
      for (int p = 0; p < 3; ++p) {
        conv1d(&s.conv1[j][p], rb + ".convs1." + std::to_string(p), s.cout, s.cout, kRbKernel[j], kDil[p], true);
        conv1d(&s.conv2[j][p], rb + ".convs2." + std::to_string(p), s.cout, s.cout, kRbKernel[j], 1, true);
      }
      for (int a = 0; a < 6; ++a) act(&s.act[j][a], rb + ".activations." + std::to_string(a), s.cout);
    }
  }
  act(&post_act_, "bigvgan.activation_post", 24);
  const size_t post_off = ar.add(weight_norm(b, "bigvgan.conv_post", 1, 24 * 7));
  uint8_t* base = static_cast<uint8_t*>(ar.upload());
  arena_ = base;
  for (auto& p : pend) {
    p.conv->w = reinterpret_cast<const __half*>(base + p.w_off);
    p.conv->bias = reinterpret_cast<const float*>(base + p.b_off);
  }
  for (auto& p : pacts) {
    p.act->alpha = reinterpret_cast<const float*>(base + p.a_off);
    p.act->inv_beta = reinterpret_cast<const float*>(base + p.b_off);
  }
  post_w_ = reinterpret_cast<const float*>(base + post_off);
}

namespace {

// Tile width for a vocoder conv GEMM: among the widths whose k-blocks per TMA
// box divide the k-blocks of one tap, the one minimising waves x (width + 64)
// on this GPU (the same per-tile cost model as the estimator's GEMMs).
int pick_bn(int M, int N, int kb_per_tap, int sms) {
  int best = 0;
  double best_cost = 0.0;
  for (int bn : {256, 192, 128, 80, 64, 48, 32}) {
    if (kb_per_tap % gemm_kbox(bn) != 0) continue;
    const long long tiles = static_cast<long long>((M + 127) / 128) * ((N + bn - 1) / bn);
    const long long waves = (tiles + sms - 1) / sms;
    const double cost = static_cast<double>(waves) * (bn + 64);
    if (best == 0 || cost < best_cost - 1e-9) {
      best = bn;
      best_cost = cost;
    }
  }
  return best;
}

// The conv GEMM: out32 rows m of [M][*] (row stride ld32) = bias + sum over
// taps of A rows (m + tap dil + off) x W; optional residual and f16 copy.
GemmLaunch conv_gemm(const VocConv& cv, const __half* a, int M, float* out32, int ld32, const float* resid,
                     __half* out16, int ld16, unsigned int* status, int sms) {
  GemmLaunch g;
  std::memset(&g, 0, sizeof(g));
  const int kbpt = cv.cin_pad / 64;
  const int bn = pick_bn(M, cv.cout, kbpt, sms);
  const uint32_t kbox = static_cast<uint32_t>(gemm_kbox(bn));
  if (!make_tmap_f16(&g.tmA0, a, cv.cin_pad, M, cv.cin_pad, 128, kbox))
    throw std::runtime_error("vocoder: tensor map for a conv input rejected");
  g.tmA1 = g.tmA0;
  if (!make_tmap_f16(&g.tmB, cv.w, static_cast<uint64_t>(cv.taps) * cv.cin_pad, cv.cout,
                     static_cast<uint64_t>(cv.taps) * cv.cin_pad, bn, kbox))
    throw std::runtime_error("vocoder: tensor map for conv weights rejected");
  g.args.M = M;
  g.args.N = cv.cout;
  g.args.num_kb = cv.taps * kbpt;
  g.args.a_mode = kAConv;
  g.args.kb_per_tap = kbpt;
  g.args.conv_dil = cv.dil;
  g.args.conv_off = cv.off;
  g.args.epi = kEpiF32;
  g.args.bias = cv.bias;
  g.args.out32 = out32;
  g.args.ld32 = ld32;
  g.args.resid32 = resid;
  g.args.ldr = ld32;
  g.args.out16 = out16;
  g.args.ld16 = ld16;
  g.args.seq_T = M;
  g.args.status = status;
  g.bn = bn;
  g.pair = 0;
  return g;
}

}  // namespace

Vocoder::Plan* Vocoder::plan_for(int T) {
  auto it = plans_.find(T);
  if (it != plans_.end()) return it->second.get();
  if (T < 1 || T > 65536) throw std::runtime_error("vocoder: T must be within 1..65536 mel frames");
  int sms = 0;
  check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device_), "sm count");
  auto p = std::make_unique<Plan>();
  p->T = T;
  const size_t t = static_cast<size_t>(T);
  const size_t f32n = 6144 * t;  // max over stages of rows x channels
  size_t off = 0;
  auto carve = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  };
  const size_t o_mel32 = carve(t * 80 * 4), o_mel16 = carve(t * 128 * 2), o_in16 = carve(8192 * t * 2),
               o_a16 = carve(16384 * t * 2), o_y = carve(f32n * 4), o_xr = carve(f32n * 4), o_h = carve(f32n * 4),
               o_acc = carve(f32n * 4), o_wave = carve(t * kHop * 4);
  check(cudaMalloc(&p->mem, off), "vocoder workspace cudaMalloc");
  check(cudaMemset(p->mem, 0, off), "vocoder workspace memset");
  uint8_t* m = static_cast<uint8_t*>(p->mem);
  p->mel32 = reinterpret_cast<float*>(m + o_mel32);
  p->mel16 = reinterpret_cast<__half*>(m + o_mel16);
  p->in16 = reinterpret_cast<__half*>(m + o_in16);
  p->a16 = reinterpret_cast<__half*>(m + o_a16);
  p->y32 = reinterpret_cast<float*>(m + o_y);
  p->xr32 = reinterpret_cast<float*>(m + o_xr);
  p->h32 = reinterpret_cast<float*>(m + o_h);
  p->acc32 = reinterpret_cast<float*>(m + o_acc);
  p->wave = reinterpret_cast<float*>(m + o_wave);
  // conv_pre: mel16 -> y32 (f32) and in16 (f16 operand of the first upsampler).
  p->pre = conv_gemm(pre_, p->mel16, T, p->y32, 1536, nullptr, p->in16, 1536, d_status_, sms);
  int tg = T;
  for (int i = 0; i < 6; ++i) {
    const VocStage& s = st_[i];
    // Upsampler phases: input rows tg of in16 [tg][cin_pad] -> y32 rows s q + r.
    for (int r = 0; r < s.s; ++r)
      p->ups[i].push_back(conv_gemm(s.phase[r], p->in16, tg, p->y32 + static_cast<size_t>(r) * s.cout, s.s * s.cout,
                                    nullptr, nullptr, 0, d_status_, sms));
    tg *= s.s;
    for (int j = 0; j < 3; ++j)
      for (int q = 0; q < 3; ++q) {
        p->c1[i][j][q] = conv_gemm(s.conv1[j][q], p->a16, tg, p->h32, s.cout, nullptr, nullptr, 0, d_status_, sms);
        p->c2[i][j][q] = conv_gemm(s.conv2[j][q], p->a16, tg, p->xr32, s.cout, q == 0 ? p->y32 : p->xr32, nullptr, 0,
                                   d_status_, sms);
      }
  }
  Plan* raw = p.get();
  plans_[T] = std::move(p);
  // Capture the schedule once per length.
  cudaGraph_t graph = nullptr;
  check(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "vocoder begin capture");
  try {
    enqueue(raw, nullptr);
  } catch (...) {
    cudaStreamEndCapture(stream_, &graph);
    if (graph) cudaGraphDestroy(graph);
    throw;
  }
  check(cudaStreamEndCapture(stream_, &graph), "vocoder end capture");
  size_t nn = 0;
  cudaGraphGetNodes(graph, nullptr, &nn);
  std::vector<cudaGraphNode_t> nodes(nn);
  if (nn) cudaGraphGetNodes(graph, nodes.data(), &nn);
  for (auto nd : nodes) {
    cudaGraphNodeType ty;
    if (cudaGraphNodeGetType(nd, &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++raw->kernels;
  }
  const cudaError_t e = cudaGraphInstantiate(&raw->graph, graph, 0);
  cudaGraphDestroy(graph);
  check(e, "vocoder graph instantiate");
  return raw;
}

namespace {

// Event-bracketed launch recorder (as in the estimator engine).
struct VProf {
  std::vector<KernelTiming>* out;
  cudaStream_t st;
  std::vector<std::pair<std::string, std::pair<cudaEvent_t, cudaEvent_t>>> evs;
  std::vector<std::pair<double, double>> work;
  template <typename F>
  void run(const std::string& name, double flops, double bytes, F&& f) {
    if (!out) {
      f();
      return;
    }
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaEventRecord(a, st);
    f();
    cudaEventRecord(b, st);
    evs.push_back({name, {a, b}});
    work.push_back({flops, bytes});
  }
  void finish() {
    if (!out) return;
    cudaStreamSynchronize(st);
    for (size_t i = 0; i < evs.size(); ++i) {
      float ms = 0.0f;
      cudaEventElapsedTime(&ms, evs[i].second.first, evs[i].second.second);
      KernelTiming* kt = nullptr;
      for (auto& k : *out)
        if (k.name == evs[i].first) kt = &k;
      if (!kt) {
        out->push_back(KernelTiming{evs[i].first});
        kt = &out->back();
      }
      kt->launches += 1;
      kt->ms += ms;
      kt->flops += work[i].first;
      kt->bytes += work[i].second;
      cudaEventDestroy(evs[i].second.first);
      cudaEventDestroy(evs[i].second.second);
    }
  }
};

}  // namespace

void Vocoder::enqueue(Plan* p, std::vector<KernelTiming>* prof) {
  VProf P{prof, stream_, {}, {}};
  const int T = p->T;
  auto G = [&](const char* name, const GemmLaunch& g, const VocConv& cv) {
    // Algorithmic work counts real channels only (padding excluded).
    const double flops = 2.0 * g.args.M * cv.cout * static_cast<double>(cv.taps) * cv.cin;
    const double bytes = static_cast<double>(g.args.M) * (cv.cin_pad * 2.0 + cv.cout * 4.0 * (g.args.resid32 ? 2 : 1) +
                                                          (g.args.out16 ? cv.cout * 2.0 : 0.0)) +
                         static_cast<double>(cv.cout) * cv.taps * cv.cin_pad * 2.0;
    P.run(name, flops, bytes, [&] { check(gemm_run(g, stream_), name); });
  };
  auto A = [&](const char* name, const VocAct& a, const float* x, int tg, void* out, int ldo, bool f16) {
    const int cw = f16 ? ldo : a.c;  // columns written (the f16 operand's padding as zeros)
    const dim3 grid((tg + kActTT - 1) / kActTT, (cw + kActCC - 1) / kActCC);
    const double bytes = static_cast<double>(tg) * a.c * (4.0 + (f16 ? 2.0 : 4.0));
    SnakeFilters filt;
    for (int k = 0; k < 12; ++k) filt.up2[k] = 2.0f * a.up[k];
    std::memcpy(filt.down, a.down, sizeof(filt.down));
    P.run(name, 0.0, bytes, [&] {
      check(f16 ? launch_pdl(snake_aa_kernel<true>, grid, dim3(256), 0, stream_, x, a.c, tg, a.c, cw, a.alpha,
                             a.inv_beta, filt, out, ldo)
                : launch_pdl(snake_aa_kernel<false>, grid, dim3(256), 0, stream_, x, a.c, tg, a.c, cw, a.alpha,
                             a.inv_beta, filt, out, ldo),
            "snake activation");
    });
  };
  P.run("mel_to_f16", 0.0, T * (80.0 * 4 + 128.0 * 2), [&] {
    check(launch_pdl(mel_to_f16_kernel, dim3(grid_for(static_cast<size_t>(T) * 128)), dim3(256), 0, stream_,
                     p->mel32, T, p->mel16),
          "mel to f16");
  });
  G("conv_pre", p->pre, pre_);
  int tg = T;
  for (int i = 0; i < 6; ++i) {
    const VocStage& s = st_[i];
    const std::string sg = "." + std::to_string(i);  // profile names per stage
    const std::string n_up = "upsample" + sg, n_conv = "resblock_conv" + sg, n_act = "snake_aa" + sg;
    for (int r = 0; r < s.s; ++r) G(n_up.c_str(), p->ups[i][r], s.phase[r]);
    tg *= s.s;
    const int C = s.cout, cp = pad64(C);
    for (int j = 0; j < 3; ++j) {
      for (int q = 0; q < 3; ++q) {
        A(n_act.c_str(), s.act[j][2 * q], q == 0 ? p->y32 : p->xr32, tg, p->a16, cp, true);
        G(n_conv.c_str(), p->c1[i][j][q], s.conv1[j][q]);
        A(n_act.c_str(), s.act[j][2 * q + 1], p->h32, tg, p->a16, cp, true);
        G(n_conv.c_str(), p->c2[i][j][q], s.conv2[j][q]);
      }
      // The last mean also writes in16, the next upsampler's operand (its
      // input channel padding pad64(C) is this stage's cp).
      const size_t n = static_cast<size_t>(tg) * C;
      __half* h16 = (j == 2 && i < 5) ? p->in16 : nullptr;
      P.run("group_mean", 0.0, n * (4.0 * (j == 0 ? 2 : 3)) + (h16 ? tg * cp * 2.0 : 0.0), [&] {
        check(launch_pdl(group_mean_kernel, dim3(grid_for(static_cast<size_t>(tg) * (h16 ? cp : C) / 4)), dim3(256),
                         0, stream_, p->acc32, static_cast<const float*>(p->xr32), static_cast<size_t>(tg), C,
                         j == 0 ? 1 : 0, h16, cp),
              "group mean");
      });
    }
  }
  A("snake_aa.post", post_act_, p->acc32, tg, p->h32, 24, false);
  P.run("conv_post", 2.0 * tg * 24 * 7, tg * (24.0 * 4 + 4.0), [&] {
    check(launch_pdl(conv_post_kernel, dim3((tg + 255) / 256), dim3(256), 0, stream_, static_cast<const float*>(p->h32),
                     tg, static_cast<const float*>(post_w_), p->wave),
          "conv_post");
  });
  P.finish();
}

void Vocoder::stage(const float* mel, int T) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  Plan* p = plan_for(T);
  check(cudaMemcpyAsync(p->mel32, mel, static_cast<size_t>(T) * 80 * sizeof(float), cudaMemcpyHostToDevice, stream_),
        "mel upload");
  staged_ = p;
}

void Vocoder::launch() {
  if (!staged_) throw std::runtime_error("vocoder: nothing staged");
  check(cudaGraphLaunch(staged_->graph, stream_), "vocoder graph launch");
}

void Vocoder::fetch(float* wave) {
  if (!staged_) throw std::runtime_error("vocoder: nothing staged");
  check(cudaMemcpyAsync(wave, staged_->wave, static_cast<size_t>(staged_->T) * kHop * sizeof(float),
                        cudaMemcpyDeviceToHost, stream_),
        "wave download");
  check(cudaStreamSynchronize(stream_), "vocoder sync");
}

void Vocoder::run(const float* mel, int T, float* wave) {
  stage(mel, T);
  launch();
  fetch(wave);
}

std::vector<KernelTiming> Vocoder::profile(int reps) {
  if (!staged_) throw std::runtime_error("vocoder: nothing staged");
  std::vector<KernelTiming> out;
  for (int r = 0; r < reps; ++r) enqueue(staged_, &out);
  return out;
}

int Vocoder::launches_per_run() const { return staged_ ? staged_->kernels : -1; }

double Vocoder::flops(int T) {
  // conv_pre + per stage: upsampler (in x out x k per input row) and three
  // resblocks of three pairs of two C x C x k convs, all x 2 FLOP per MAC.
  double macs = static_cast<double>(T) * 80 * 1536 * 7;
  double tg = T;
  for (int i = 0; i < 6; ++i) {
    macs += tg * kUps[i][0] * kUps[i][1] * kUps[i][2];
    tg *= kUps[i][3];
    const double c = kUps[i][1];
    for (int j = 0; j < 3; ++j) macs += 3.0 * 2.0 * tg * c * c * kRbKernel[j];
  }
  macs += tg * 24 * 7;
  return 2.0 * macs;
}

}  // namespace itts
