// Estimator weight preparation and upload (host C++, fp32 math).
#include "model.hpp"

#include "kernels.cuh"

#include <cmath>
#include <cstring>
#include <functional>
#include <stdexcept>

namespace itts {

namespace {

const std::string kPre = "s2mel.net.cfm.estimator.";

// Collects host payloads, then makes one device allocation and copies them in.
class Packer {
 public:
  template <typename T>
  void add(std::vector<T>&& data, T** slot) {
    Item it;
    it.bytes.resize(data.size() * sizeof(T));
    std::memcpy(it.bytes.data(), data.data(), it.bytes.size());
    it.slot = reinterpret_cast<void**>(slot);
    items_.push_back(std::move(it));
  }
  void upload(DevWeights* w) {
    size_t total = 0;
    for (auto& it : items_) {
      it.off = total;
      total += (it.bytes.size() + 255) & ~size_t(255);
    }
    void* base = nullptr;
    if (cudaMalloc(&base, total) != cudaSuccess) throw std::runtime_error("weights: cudaMalloc failed");
    std::vector<uint8_t> host(total, 0);
    for (auto& it : items_) std::memcpy(host.data() + it.off, it.bytes.data(), it.bytes.size());
    if (cudaMemcpy(base, host.data(), total, cudaMemcpyHostToDevice) != cudaSuccess) {
      cudaFree(base);
      throw std::runtime_error("weights: upload failed");
    }
    for (auto& it : items_) *it.slot = static_cast<uint8_t*>(base) + it.off;
    w->arena = base;
    w->arena_bytes = total;
  }

 private:
  struct Item {
    std::vector<uint8_t> bytes;
    void** slot = nullptr;
    size_t off = 0;
  };
  std::vector<Item> items_;
};

size_t count_of(const Mit2Bundle& b, const std::string& n) { return b.element_count(b.require(n)); }

void expect_count(const Mit2Bundle& b, const std::string& n, size_t want) {
  const size_t got = count_of(b, n);
  if (got != want)
    throw std::runtime_error("weights: tensor " + n + " has " + std::to_string(got) + " elements, expected " +
                             std::to_string(want));
}

std::vector<uint16_t> to_h(const std::vector<float>& f) {
  std::vector<uint16_t> h(f.size());
  for (size_t i = 0; i < f.size(); ++i) h[i] = float_to_half_bits(f[i]);
  return h;
}

// f16 payload exactly as stored (bundle f16) or rounded from f32.
std::vector<uint16_t> h16(const Mit2Bundle& b, const std::string& n, size_t want) {
  expect_count(b, n, want);
  const TensorRec& t = b.require(n);
  if (t.dtype == "f16") {
    std::vector<uint16_t> out(want);
    std::memcpy(out.data(), b.data(t), want * 2);
    return out;
  }
  return to_h(b.as_f32(n));
}

std::vector<float> f32(const Mit2Bundle& b, const std::string& n, size_t want) {
  expect_count(b, n, want);
  return b.as_f32(n);
}

// weight_norm_rowmajor (runtime/impl/gpt.cpp:5109-5124): W[row] = g[row] * v[row] / ||v[row]||.
std::vector<float> weight_norm(const Mit2Bundle& b, const std::string& prefix, size_t rows, size_t cols) {
  auto g = f32(b, prefix + ".weight_g", rows);
  auto v = f32(b, prefix + ".weight_v", rows * cols);
  std::vector<float> w(rows * cols);
  for (size_t r = 0; r < rows; ++r) {
    float norm = 0.0f;
    for (size_t c = 0; c < cols; ++c) norm += v[r * cols + c] * v[r * cols + c];
    norm = std::sqrt(norm);
    const float scale = g[r] / norm;
    for (size_t c = 0; c < cols; ++c) w[r * cols + c] = v[r * cols + c] * scale;
  }
  return w;
}

// Rows [a(C) | b(C)] -> 64-row groups a0 b0 a1 b1 ...; works on any element type.
template <typename T>
std::vector<T> interleave64(const std::vector<T>& src, size_t C, size_t K) {
  std::vector<T> out(src.size());
  for (size_t g = 0; g < C / 64; ++g) {
    for (size_t r = 0; r < 64; ++r) {
      std::memcpy(&out[((2 * g) * 64 + r) * K], &src[(g * 64 + r) * K], K * sizeof(T));
      std::memcpy(&out[((2 * g + 1) * 64 + r) * K], &src[(C + g * 64 + r) * K], K * sizeof(T));
    }
  }
  return out;
}

}  // namespace

std::vector<std::string> required_tensor_names() {
  std::vector<std::string> n;
  auto add = [&](const std::string& s) { n.push_back(kPre + s); };
  add("cond_projection.weight");
  add("cond_projection.bias");
  add("cond_x_merge_linear.weight");
  add("cond_x_merge_linear.bias");
  for (const char* te : {"t_embedder", "t_embedder2"}) {
    const std::string p = std::string(te) + ".";
    add(p + "freqs");
    add(p + "mlp.0.weight");
    add(p + "mlp.0.bias");
    add(p + "mlp.2.weight");
    add(p + "mlp.2.bias");
  }
  for (int l = 0; l < kLayers; ++l) {
    const std::string p = "transformer.layers." + std::to_string(l) + ".";
    for (const char* nm : {"attention_norm", "ffn_norm"}) {
      add(p + nm + ".norm.weight");
      add(p + nm + ".project_layer.weight");
      add(p + nm + ".project_layer.bias");
    }
    add(p + "attention.wqkv.weight");
    add(p + "attention.wo.weight");
    add(p + "feed_forward.w1.weight");
    add(p + "feed_forward.w2.weight");
    add(p + "feed_forward.w3.weight");
    if (l > kLayers / 2) {
      add(p + "skip_in_linear.weight");
      add(p + "skip_in_linear.bias");
    }
  }
  add("transformer.norm.norm.weight");
  add("transformer.norm.project_layer.weight");
  add("transformer.norm.project_layer.bias");
  add("skip_linear.weight");
  add("skip_linear.bias");
  add("conv1.weight");
  add("conv1.bias");
  add("res_projection.weight");
  add("res_projection.bias");
  for (const char* s : {"weight_g", "weight_v", "bias"}) add(std::string("wavenet.cond_layer.conv.conv.") + s);
  for (int l = 0; l < kWnLayers; ++l) {
    for (const char* s : {"weight_g", "weight_v", "bias"}) {
      add("wavenet.in_layers." + std::to_string(l) + ".conv.conv." + s);
      add("wavenet.res_skip_layers." + std::to_string(l) + ".conv.conv." + s);
    }
  }
  add("final_layer.adaLN_modulation.1.weight");
  add("final_layer.adaLN_modulation.1.bias");
  add("final_layer.linear.weight_g");
  add("final_layer.linear.weight_v");
  add("final_layer.linear.bias");
  add("conv2.weight");
  add("conv2.bias");
  return n;
}

void load_weights(const Mit2Bundle& b, DevWeights* w) {
  for (const auto& n : required_tensor_names()) b.require(n);
  Packer pk;
  auto P = [](const std::string& s) { return kPre + s; };

  // Input merge: cond_projection, cond_x_merge_linear split into x slice and rest.
  pk.add(h16(b, P("cond_projection.weight"), 512 * 512), reinterpret_cast<uint16_t**>(&w->wcp));
  pk.add(f32(b, P("cond_projection.bias"), 512), &w->bcp);
  {
    auto m = h16(b, P("cond_x_merge_linear.weight"), 512 * 864);
    // Zero-padded to whole 64-column k-blocks (x slice 80 -> kXdLd, rest 784 -> kUld).
    std::vector<uint16_t> wx(512 * kXdLd, 0), wr(512 * kUld, 0);
    for (int r = 0; r < 512; ++r) {
      std::memcpy(&wx[r * kXdLd], &m[r * 864], 80 * 2);
      std::memcpy(&wr[r * kUld], &m[r * 864 + 80], 784 * 2);
    }
    pk.add(std::move(wx), reinterpret_cast<uint16_t**>(&w->wx));
    pk.add(std::move(wr), reinterpret_cast<uint16_t**>(&w->wrest));
    pk.add(f32(b, P("cond_x_merge_linear.bias"), 512), &w->bm);
  }
  // Timestep embedders.
  for (int e = 0; e < 2; ++e) {
    TEmbW& te = e == 0 ? w->te1 : w->te2;
    const std::string p = P(e == 0 ? "t_embedder." : "t_embedder2.");
    pk.add(f32(b, p + "freqs", 128), &te.freqs);
    pk.add(h16(b, p + "mlp.0.weight", 512 * 256), reinterpret_cast<uint16_t**>(&te.w0));
    pk.add(f32(b, p + "mlp.0.bias", 512), &te.b0);
    pk.add(h16(b, p + "mlp.2.weight", 512 * 512), reinterpret_cast<uint16_t**>(&te.w2));
    pk.add(f32(b, p + "mlp.2.bias", 512), &te.b2);
  }
  // Transformer.
  for (int l = 0; l < kLayers; ++l) {
    LayerW& L = w->L[l];
    const std::string p = P("transformer.layers." + std::to_string(l) + ".");
    pk.add(f32(b, p + "attention_norm.norm.weight", 512), &L.g_attn);
    pk.add(h16(b, p + "attention_norm.project_layer.weight", 1024 * 512), reinterpret_cast<uint16_t**>(&L.proj_attn));
    pk.add(f32(b, p + "attention_norm.project_layer.bias", 1024), &L.projb_attn);
    pk.add(f32(b, p + "ffn_norm.norm.weight", 512), &L.g_ffn);
    pk.add(h16(b, p + "ffn_norm.project_layer.weight", 1024 * 512), reinterpret_cast<uint16_t**>(&L.proj_ffn));
    pk.add(f32(b, p + "ffn_norm.project_layer.bias", 1024), &L.projb_ffn);
    pk.add(h16(b, p + "attention.wqkv.weight", 1536 * 512), reinterpret_cast<uint16_t**>(&L.wqkv));
    pk.add(h16(b, p + "attention.wo.weight", 512 * 512), reinterpret_cast<uint16_t**>(&L.wo));
    {
      auto w1 = h16(b, p + "feed_forward.w1.weight", 1536 * 512);
      auto w3 = h16(b, p + "feed_forward.w3.weight", 1536 * 512);
      std::vector<uint16_t> cat(w1);
      cat.insert(cat.end(), w3.begin(), w3.end());
      pk.add(interleave64(cat, 1536, 512), reinterpret_cast<uint16_t**>(&L.w13));
    }
    pk.add(h16(b, p + "feed_forward.w2.weight", 512 * 1536), reinterpret_cast<uint16_t**>(&L.w2));
    if (l > kLayers / 2) {
      // skip_in_linear reads [x | skip] where x = h + W2 . g is the output of
      // layer l - 1 (h: its stream after attention, g: its SwiGLU activations;
      // feed_forward.w2 has no bias) and nothing else reads x, so
      //   Wsk . [x ; skip] = Wx . h + (Wx . W2) . g + Ws . skip
      // is one 2560 -> 512 linear map over [h | g | skip] (Wx, Ws: the x and
      // skip halves of skip_in_linear.weight). Composed in fp32, rounded to f16 once.
      const auto wsk = b.as_f32(p + "skip_in_linear.weight");  // [512][1024]
      const auto w2p = b.as_f32(P("transformer.layers." + std::to_string(l - 1) + ".feed_forward.w2.weight"));
      if (wsk.size() != 512u * 1024 || w2p.size() != 512u * 1536)
        throw std::runtime_error("bundle: skip_in_linear / feed_forward.w2 shapes");
      std::vector<float> wc(static_cast<size_t>(512) * 2560, 0.0f);
      for (int o = 0; o < 512; ++o) {
        float* dst = &wc[static_cast<size_t>(o) * 2560];
        const float* src = &wsk[static_cast<size_t>(o) * 1024];
        std::memcpy(dst, src, 512 * sizeof(float));
        std::memcpy(dst + 2048, src + 512, 512 * sizeof(float));
        float* mid = dst + 512;
        for (int j = 0; j < 512; ++j) {
          const float a = src[j];
          const float* w2r = &w2p[static_cast<size_t>(j) * 1536];
          for (int k = 0; k < 1536; ++k) mid[k] += a * w2r[k];
        }
      }
      pk.add(to_h(wc), reinterpret_cast<uint16_t**>(&L.wskip));
      pk.add(f32(b, p + "skip_in_linear.bias", 512), &L.bskip);
    }
  }
  pk.add(f32(b, P("transformer.norm.norm.weight"), 512), &w->g_norm);
  pk.add(h16(b, P("transformer.norm.project_layer.weight"), 1024 * 512), reinterpret_cast<uint16_t**>(&w->proj_norm));
  pk.add(f32(b, P("transformer.norm.project_layer.bias"), 1024), &w->projb_norm);
  // Post-transformer projections: skip_linear (592 -> 512) feeds conv1 and
  // res_projection (512 -> 512 each) with no operation between them
  // (run_dit_post_transformer_proj_cpu, runtime/impl/dit_cfm_bigvgan.cpp:
  // 1053-1079), so the three are one 592 -> 1024 linear map.
  {
    const auto sl = b.as_f32(P("skip_linear.weight"));  // [512][592]
    const auto bsl = f32(b, P("skip_linear.bias"), 512);
    auto c1 = b.as_f32(P("conv1.weight"));  // [512][512(,1)]
    const auto rp = b.as_f32(P("res_projection.weight"));
    if (sl.size() != 512u * 592 || c1.size() != 512u * 512 || rp.size() != 512u * 512)
      throw std::runtime_error("bundle: post-transformer projection shapes");
    c1.insert(c1.end(), rp.begin(), rp.end());  // [1024][512]
    auto bc = f32(b, P("conv1.bias"), 512);
    const auto br = f32(b, P("res_projection.bias"), 512);
    bc.insert(bc.end(), br.begin(), br.end());
    std::vector<float> wp(1024 * 592, 0.0f);
    for (int o = 0; o < 1024; ++o) {
      float* dst = &wp[static_cast<size_t>(o) * 592];
      double bias = bc[o];
      for (int j = 0; j < 512; ++j) {
        const float a = c1[static_cast<size_t>(o) * 512 + j];
        const float* src = &sl[static_cast<size_t>(j) * 592];
        for (int k = 0; k < 592; ++k) dst[k] += a * src[k];
        bias += static_cast<double>(a) * bsl[j];
      }
      bc[o] = static_cast<float>(bias);
    }
    // [x_normed (512) | x_mel (80 -> kXdLd, zero-padded)]
    const auto wh = to_h(wp);
    std::vector<uint16_t> padded(1024 * (512 + kXdLd), 0);
    for (int o = 0; o < 1024; ++o) std::memcpy(&padded[o * (512 + kXdLd)], &wh[o * 592], 592 * 2);
    pk.add(std::move(padded), reinterpret_cast<uint16_t**>(&w->wpost));
    pk.add(std::move(bc), &w->bpost);
  }
  // WaveNet.
  {
    auto wc = weight_norm(b, P("wavenet.cond_layer.conv.conv"), 8192, 512);
    pk.add(std::move(wc), &w->wcond);
    pk.add(f32(b, P("wavenet.cond_layer.conv.conv.bias"), 8192), &w->bcond);
  }
  for (int l = 0; l < kWnLayers; ++l) {
    const std::string ip = P("wavenet.in_layers." + std::to_string(l) + ".conv.conv");
    auto wi = weight_norm(b, ip, 1024, 512 * 5);  // [o][c][k]
    std::vector<float> perm(wi.size());
    for (int o = 0; o < 1024; ++o)
      for (int c = 0; c < 512; ++c)
        for (int k = 0; k < 5; ++k) perm[(static_cast<size_t>(o) * 5 + k) * 512 + c] = wi[(static_cast<size_t>(o) * 512 + c) * 5 + k];
    pk.add(interleave64(to_h(perm), 512, 2560), reinterpret_cast<uint16_t**>(&w->win[l]));
    pk.add(interleave64(f32(b, ip + ".bias", 1024), 512, 1), &w->bin[l]);
    const std::string rp = P("wavenet.res_skip_layers." + std::to_string(l) + ".conv.conv");
    const int rs_out = l < kWnLayers - 1 ? 1024 : 512;
    auto wr = to_h(weight_norm(b, rp, rs_out, 512));
    auto br = f32(b, rp + ".bias", rs_out);
    if (rs_out == 1024) {
      pk.add(interleave64(wr, 512, 512), reinterpret_cast<uint16_t**>(&w->wrs[l]));
      pk.add(interleave64(br, 512, 1), &w->brs[l]);
    } else {
      pk.add(std::move(wr), reinterpret_cast<uint16_t**>(&w->wrs[l]));
      pk.add(std::move(br), &w->brs[l]);
    }
  }
  // Final layer.
  pk.add(h16(b, P("final_layer.adaLN_modulation.1.weight"), 1024 * 512), reinterpret_cast<uint16_t**>(&w->ada_w));
  pk.add(f32(b, P("final_layer.adaLN_modulation.1.bias"), 1024), &w->ada_b);
  // final_layer.linear (512 -> 512, weight-normed) then conv2 (1x1, 512 -> 80)
  // with nothing between them (run_dit_final_layer_cpu, :1172-1199, and the
  // conv2 that follows it): one 512 -> 80 linear map.
  {
    const auto fl = weight_norm(b, P("final_layer.linear"), 512, 512);
    const auto bfl = f32(b, P("final_layer.linear.bias"), 512);
    const auto c2 = b.as_f32(P("conv2.weight"));  // [80][512(,1)]
    if (c2.size() != 80u * 512) throw std::runtime_error("bundle: conv2 shape");
    auto bo = f32(b, P("conv2.bias"), 80);
    std::vector<float> wo(80 * 512, 0.0f);
    for (int o = 0; o < 80; ++o) {
      double bias = bo[o];
      for (int j = 0; j < 512; ++j) {
        const float a = c2[static_cast<size_t>(o) * 512 + j];
        const float* src = &fl[static_cast<size_t>(j) * 512];
        float* dst = &wo[static_cast<size_t>(o) * 512];
        for (int k = 0; k < 512; ++k) dst[k] += a * src[k];
        bias += static_cast<double>(a) * bfl[j];
      }
      bo[o] = static_cast<float>(bias);
    }
    pk.add(to_h(wo), reinterpret_cast<uint16_t**>(&w->wout));
    pk.add(std::move(bo), &w->bout);
  }

  pk.upload(w);
}

void free_weights(DevWeights* w) {
  if (w->arena) cudaFree(w->arena);
  *w = DevWeights{};
}

}  // namespace itts
