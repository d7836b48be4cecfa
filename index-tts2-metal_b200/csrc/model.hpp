// DiT estimator weights, prepared once per context and resident in HBM.
//
// Tensor names are the reference bundle's (prefix s2mel.net.cfm.estimator.,
// runtime/impl/dit_cfm_bigvgan.cpp:1-1800). Layout changes made at load time:
//   - weight-norm pairs folded, W = g * v / ||v_row|| (runtime/impl/gpt.cpp:5109-5130);
//   - w1/w3, WaveNet in_layers and res_skip_layers rows interleaved in 64-row
//     groups [a | b] for the paired GEMM epilogues;
//   - WaveNet k=5 conv weights permuted from [out][in][k] to [out][k][in];
//   - the merge weight split into its x slice [512][80] and the rest [512][784];
//   - linear layers with nothing between them composed into one matrix (in
//     fp32, then rounded to f16 once): [conv1 ; res_projection] . skip_linear
//     (592 -> 1024), conv2 . final_layer.linear (512 -> 80), and for layers
//     7..12 skip_in_linear with the feed_forward.w2 of layer l - 1 (the residual
//     add between them is linear): [h | g | skip] (2560) -> 512.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "bundle.hpp"

namespace itts {

constexpr int kLayers = 13;
constexpr int kWnLayers = 8;
// Offsets (floats) inside one step's table row.
constexpr int kTabAttn = 0;           // + L*1024: [w | b] of attention_norm
constexpr int kTabFfn = 13 * 1024;    // + L*1024: [w | b] of ffn_norm
constexpr int kTabNorm = 26 * 1024;   // [w | b] of transformer.norm
constexpr int kTabFinal = 27 * 1024;  // [shift | scale] of final_layer.adaLN_modulation
constexpr int kTabWn = 28 * 1024;     // + l*1024: WaveNet global condition [a | b]
// Folded AdaRMS: the shift b of each norm pushed through the following GEMM
// (b . W^T, in the GEMM's B-row order), added in that GEMM's epilogue.
constexpr int kTabQkvC = 36 * 1024;                // + L*1536: b_attn . Wqkv^T
constexpr int kTabW13C = kTabQkvC + 13 * 1536;     // + L*3072: b_ffn . W13^T (interleaved rows)
constexpr int kTcondPerStep = kTabW13C + 13 * 3072;  // floats per step in the t-conditioning table

struct LayerW {
  __half* wqkv = nullptr;   // [1536][512]
  __half* wo = nullptr;     // [512][512]
  __half* w13 = nullptr;    // [3072][512] interleaved w1/w3
  __half* w2 = nullptr;     // [512][1536]
  __half* wskip = nullptr;  // layers 7..12: [512][2560] = [Wx | Wx . W2(l-1) | Ws] over [h | g | skip]
  float* bskip = nullptr;
  float* g_attn = nullptr;  // attention_norm.norm.weight [512]
  float* g_ffn = nullptr;   // ffn_norm.norm.weight [512]
  __half* proj_attn = nullptr;  // attention_norm.project_layer.weight [1024][512]
  float* projb_attn = nullptr;
  __half* proj_ffn = nullptr;
  float* projb_ffn = nullptr;
};

struct TEmbW {
  float* freqs = nullptr;  // [128]
  __half* w0 = nullptr;    // [512][256]
  float* b0 = nullptr;
  __half* w2 = nullptr;    // [512][512]
  float* b2 = nullptr;
};

struct DevWeights {
  LayerW L[kLayers];
  float* g_norm = nullptr;
  __half* proj_norm = nullptr;
  float* projb_norm = nullptr;
  __half* wcp = nullptr;  // cond_projection [512][512]
  float* bcp = nullptr;
  __half* wx = nullptr;     // cond_x_merge_linear x slice [512][kXdLd] (zero-padded)
  __half* wrest = nullptr;  // remaining merge columns [512][kUld] (zero-padded)
  float* bm = nullptr;
  __half* wpost = nullptr;  // [conv1 ; res_projection] . skip_linear: [1024][512 + kXdLd] (x_mel columns zero-padded)
  float* bpost = nullptr;   // [1024] [conv1 ; res_projection] . skip_linear.bias + [conv1.bias ; res_projection.bias]
  __half* win[kWnLayers] = {};  // [1024][2560] paired, tap-major K
  float* bin[kWnLayers] = {};
  __half* wrs[kWnLayers] = {};  // [1024][512] paired (l < 7), [512][512] (l = 7)
  float* brs[kWnLayers] = {};
  __half* wout = nullptr;  // conv2 . final_layer.linear (weight-normed): [80][512]
  float* bout = nullptr;   // [80] conv2 . final_layer.linear.bias + conv2.bias
  __half* ada_w = nullptr;  // final_layer.adaLN_modulation.1 [1024][512]
  float* ada_b = nullptr;
  float* wcond = nullptr;  // wavenet.cond_layer (weight-normed) [8192][512] fp32
  float* bcond = nullptr;
  TEmbW te1, te2;
  void* arena = nullptr;
  size_t arena_bytes = 0;
};

// Reads, validates and prepares every estimator tensor, then uploads to the
// current device. Throws std::runtime_error on a missing or misshaped tensor.
void load_weights(const Mit2Bundle& b, DevWeights* w);
void free_weights(DevWeights* w);

// Names of every tensor the estimator needs (for contract checks and tests).
std::vector<std::string> required_tensor_names();

}  // namespace itts
