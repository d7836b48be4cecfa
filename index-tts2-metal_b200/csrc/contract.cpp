// Bundle contract gates and the cached-voice loader (host only; no GPU).
//
// itts_inspect_voice_bundle follows inspect_voice_bundle_contract
// (runtime/impl/tokenizer_tests.cpp:5699-5755): full integrity check with
// every payload's SHA-256 present and verified (validate_bundle_integrity,
// :4666-4708), then four f32 component=voice tensors spk_cond_emb [1,S>0,1024],
// s2mel_style [1,192], s2mel_prompt [1,P>0,512] and mel [1,80,P] with the
// prompt token count equal to the mel frame count; a JSON report.
// itts_inspect_model_bundle applies the same integrity check and then the
// required tensors (name, shape, component) of the stages this library runs,
// in the manner of inspect_model_bundle_contract (:4776-4864).
// itts_voice_load reads a voice bundle the way the synthesis pipeline does
// (runtime/impl/tts_synthesis/synthesis_pipeline.cpp:1060-1084): the first P
// rows of s2mel_prompt, s2mel_style, and the prompt mel transposed from
// [1,80,T_voice] to [P,80].
#include <cstdio>
#include <cstring>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "bundle.hpp"
#include "itts_cfm.h"

namespace {

struct Integrity {
  uint64_t aligned = 0;
  uint64_t intervals = 0;
  uint64_t sha_verified = 0;
  uint64_t tensor_bytes = 0;
};

// The reader has already checked format, version, endianness, header,
// alignment, duplicates, zero-byte payloads, dtype byte counts, bounds and
// overlaps; the gate additionally requires every payload's SHA-256 and
// verifies it.
Integrity integrity(const itts::Mit2Bundle& b) {
  Integrity r;
  for (const itts::TensorRec& t : b.tensors()) {
    if (t.shape.empty()) throw std::runtime_error("tensor has empty shape: " + t.name);
    if (t.sha256.empty()) throw std::runtime_error("tensor missing sha256: " + t.name);
    if (itts::sha256_hex(b.data(t), t.nbytes) != t.sha256) throw std::runtime_error("tensor sha256 mismatch: " + t.name);
    ++r.aligned;
    ++r.intervals;
    ++r.sha_verified;
    r.tensor_bytes += t.nbytes;
  }
  return r;
}

std::string esc(const std::string& s) {
  std::string o;
  for (char c : s) {
    if (c == '"' || c == '\\') {
      o += '\\';
      o += c;
    } else if (static_cast<unsigned char>(c) < 0x20) {
      char buf[8];
      std::snprintf(buf, sizeof(buf), "\\u%04x", c);
      o += buf;
    } else {
      o += c;
    }
  }
  return o;
}

std::string shape_json(const std::vector<int64_t>& s) {
  std::string o = "[";
  for (size_t i = 0; i < s.size(); ++i) o += (i ? "," : "") + std::to_string(s[i]);
  return o + "]";
}

std::string tensor_json(const itts::TensorRec& t) {
  return "{\"name\": \"" + esc(t.name) + "\", \"dtype\": \"" + esc(t.dtype) + "\", \"shape\": " + shape_json(t.shape) +
         ", \"nbytes\": " + std::to_string(t.nbytes) + ", \"component\": \"" + esc(t.component) + "\"}";
}

void put_report(char* out, uint32_t cap, const std::string& s) {
  if (out && cap > 0) std::snprintf(out, cap, "%s", s.c_str());
}

std::string head_json(const char* stage, const std::string& dir, const itts::Mit2Bundle& b, const Integrity& in) {
  std::ostringstream o;
  o << "{\"stage\": \"" << stage << "\", \"bundle_dir\": \"" << esc(dir) << "\", \"ok\": true, \"format\": \"MIT2\", "
    << "\"version\": " << b.version() << ", \"endianness\": \"little\", \"alignment\": " << b.alignment()
    << ", \"weights_bytes\": " << b.weights_bytes() << ", \"tensor_count\": " << b.tensors().size()
    << ", \"tensor_bytes\": " << in.tensor_bytes << ", \"integrity\": {\"aligned_tensor_count\": " << in.aligned
    << ", \"checked_interval_count\": " << in.intervals << ", \"sha256_verified_count\": " << in.sha_verified << "}";
  return o.str();
}

std::string fail_json(const char* stage, const std::string& dir, const std::string& err) {
  return std::string("{\"stage\": \"") + stage + "\", \"bundle_dir\": \"" + esc(dir) + "\", \"ok\": false, \"error\": \"" +
         esc(err) + "\"}";
}

const itts::TensorRec& voice_tensor(const itts::Mit2Bundle& b, const std::string& name) {
  const itts::TensorRec* t = b.find(name);
  if (!t) throw std::runtime_error("voice bundle missing tensor: " + name);
  if (t->dtype != "f32") throw std::runtime_error("voice tensor must use f32 dtype: " + name + " dtype=" + t->dtype);
  if (t->component != "voice")
    throw std::runtime_error("voice tensor must have component=voice: " + name + " component=" + t->component);
  return *t;
}

struct VoiceShapes {
  int64_t spk = 0, prompt = 0, mel = 0;
};

VoiceShapes check_voice(const itts::Mit2Bundle& b) {
  const auto& spk = voice_tensor(b, "spk_cond_emb");
  const auto& style = voice_tensor(b, "s2mel_style");
  const auto& prompt = voice_tensor(b, "s2mel_prompt");
  const auto& mel = voice_tensor(b, "mel");
  if (spk.shape.size() != 3 || spk.shape[0] != 1 || spk.shape[1] <= 0 || spk.shape[2] != 1024)
    throw std::runtime_error("voice spk_cond_emb must have shape [1,tokens>0,1024]");
  if (style.shape.size() != 2 || style.shape[0] != 1 || style.shape[1] != 192)
    throw std::runtime_error("voice s2mel_style must have shape [1,192]");
  if (prompt.shape.size() != 3 || prompt.shape[0] != 1 || prompt.shape[1] <= 0 || prompt.shape[2] != 512)
    throw std::runtime_error("voice s2mel_prompt must have shape [1,tokens>0,512]");
  if (mel.shape.size() != 3 || mel.shape[0] != 1 || mel.shape[1] != 80 || mel.shape[2] <= 0)
    throw std::runtime_error("voice mel must have shape [1,80,tokens>0]");
  if (prompt.shape[1] != mel.shape[2]) throw std::runtime_error("voice prompt token count must match mel frame count");
  return VoiceShapes{spk.shape[1], prompt.shape[1], mel.shape[2]};
}

struct Required {
  std::string name;
  std::string component;
  std::vector<int64_t> shape;
};

// Sentinel tensors of each stage (first, middle and last layers, every kind of
// weight the stage loads); the stage loaders check every other tensor's size.
std::vector<Required> required_for(uint32_t components) {
  std::vector<Required> r;
  if (components & ITTS_COMPONENT_CFM) {
    const char* p = "s2mel.net.cfm.estimator.";
    auto n = [&](const char* s) { return std::string(p) + s; };
    const std::vector<std::string> names = {n("cond_projection.weight"),
             n("cond_x_merge_linear.weight"),
             n("t_embedder.mlp.0.weight"),
             n("transformer.layers.0.attention.wqkv.weight"),
             n("transformer.layers.12.feed_forward.w2.weight"),
             n("transformer.layers.7.skip_in_linear.weight"),
             n("transformer.norm.project_layer.weight"),
             n("wavenet.cond_layer.conv.conv.weight_v"),
             n("wavenet.in_layers.0.conv.conv.weight_v"),
             n("wavenet.res_skip_layers.7.conv.conv.weight_v"),
             n("final_layer.linear.weight_v"),
             n("conv2.weight")};
    const std::vector<std::vector<int64_t>> shapes = {{512, 512},      {512, 864},       {512, 256},
                                                      {1536, 512},     {512, 1536},      {512, 1024},
                                                      {1024, 512},     {8192, 512, 1},   {1024, 512, 5},
                                                      {512, 512, 1},   {512, 512},       {80, 512, 1}};
    for (size_t i = 0; i < names.size(); ++i) r.push_back({names[i], "s2mel", shapes[i]});
  }
  if (components & ITTS_COMPONENT_LENGTH_REGULATOR) {
    r.push_back({"s2mel.net.length_regulator.content_in_proj.weight", "s2mel", {512, 1024}});
    r.push_back({"s2mel.net.length_regulator.model.0.weight", "s2mel", {512, 512, 3}});
    r.push_back({"s2mel.net.length_regulator.model.10.weight", "s2mel", {512}});
    r.push_back({"s2mel.net.length_regulator.model.12.weight", "s2mel", {512, 512, 1}});
  }
  if (components & ITTS_COMPONENT_BIGVGAN) {
    r.push_back({"bigvgan.conv_pre.weight_v", "bigvgan", {1536, 80, 7}});
    r.push_back({"bigvgan.ups.0.0.weight_v", "bigvgan", {1536, 768, 8}});
    r.push_back({"bigvgan.ups.5.0.weight_v", "bigvgan", {48, 24, 4}});
    r.push_back({"bigvgan.resblocks.0.convs1.0.weight_v", "bigvgan", {768, 768, 3}});
    r.push_back({"bigvgan.resblocks.17.convs2.2.weight_v", "bigvgan", {24, 24, 11}});
    r.push_back({"bigvgan.resblocks.17.activations.5.act.beta", "bigvgan", {24}});
    r.push_back({"bigvgan.activation_post.upsample.filter", "bigvgan", {1, 1, 12}});
    r.push_back({"bigvgan.conv_post.weight_v", "bigvgan", {1, 24, 7}});
  }
  if (components & ITTS_COMPONENT_GPT) {  // Conv1D weights are stored [in, out]
    r.push_back({"gpt.gpt.h.0.attn.c_attn.weight", "gpt", {1280, 3840}});
    r.push_back({"gpt.gpt.h.12.ln_1.weight", "gpt", {1280}});
    r.push_back({"gpt.gpt.h.23.mlp.c_fc.weight", "gpt", {1280, 5120}});
    r.push_back({"gpt.gpt.h.23.mlp.c_proj.weight", "gpt", {5120, 1280}});
    r.push_back({"gpt.gpt.ln_f.weight", "gpt", {1280}});
    r.push_back({"gpt.final_norm.weight", "gpt", {1280}});
    r.push_back({"gpt.mel_head.weight", "gpt", {8194, 1280}});
    r.push_back({"gpt.mel_embedding.weight", "gpt", {8194, 1280}});
    r.push_back({"gpt.mel_pos_embedding.emb.weight", "gpt", {1818, 1280}});
  }
  return r;
}

}  // namespace

extern "C" {

int itts_inspect_voice_bundle(const char* bundle_dir, char* report, uint32_t cap) {
  const std::string dir = bundle_dir ? bundle_dir : "";
  try {
    if (!bundle_dir) throw std::runtime_error("null bundle directory");
    itts::Mit2Bundle b(dir, false);
    const Integrity in = integrity(b);
    const VoiceShapes v = check_voice(b);
    std::string o = head_json("voice_bundle_contract", dir, b, in);
    o += ", \"spk_cond_tokens\": " + std::to_string(v.spk) + ", \"prompt_tokens\": " + std::to_string(v.prompt) +
         ", \"mel_frames\": " + std::to_string(v.mel) + ", \"required_tensors\": [";
    const char* names[4] = {"spk_cond_emb", "s2mel_style", "s2mel_prompt", "mel"};
    for (int i = 0; i < 4; ++i) o += (i ? ", " : "") + tensor_json(*b.find(names[i]));
    put_report(report, cap, o + "]}");
    return ITTS_OK;
  } catch (const std::exception& e) {
    put_report(report, cap, fail_json("voice_bundle_contract", dir, e.what()));
    return ITTS_EBUNDLE;
  }
}

int itts_inspect_model_bundle(const char* bundle_dir, uint32_t components, char* report, uint32_t cap) {
  const std::string dir = bundle_dir ? bundle_dir : "";
  try {
    if (!bundle_dir) throw std::runtime_error("null bundle directory");
    if (components == 0 || (components & ~ITTS_COMPONENT_ALL) != 0) throw std::runtime_error("bad component mask");
    itts::Mit2Bundle b(dir, false);
    const Integrity in = integrity(b);
    std::string list;
    for (const Required& r : required_for(components)) {
      const itts::TensorRec* t = b.find(r.name);
      if (!t) throw std::runtime_error("model bundle missing tensor: " + r.name);
      if (t->dtype != "f32" && t->dtype != "f16")
        throw std::runtime_error("model tensor must use f32 or f16 dtype: " + r.name + " dtype=" + t->dtype);
      if (!t->component.empty() && t->component != r.component)
        throw std::runtime_error("model tensor component mismatch: " + r.name + " component=" + t->component);
      if (t->shape != r.shape) throw std::runtime_error("model tensor shape mismatch: " + r.name);
      list += (list.empty() ? "" : ", ") + tensor_json(*t);
    }
    std::string comps;
    if (components & ITTS_COMPONENT_CFM) comps += "\"cfm_estimator\"";
    if (components & ITTS_COMPONENT_LENGTH_REGULATOR) comps += std::string(comps.empty() ? "" : ", ") + "\"length_regulator\"";
    if (components & ITTS_COMPONENT_BIGVGAN) comps += std::string(comps.empty() ? "" : ", ") + "\"bigvgan\"";
    if (components & ITTS_COMPONENT_GPT) comps += std::string(comps.empty() ? "" : ", ") + "\"gpt\"";
    put_report(report, cap,
               head_json("model_bundle_contract", dir, b, in) + ", \"components\": [" + comps +
                   "], \"required_tensors\": [" + list + "]}");
    return ITTS_OK;
  } catch (const std::exception& e) {
    put_report(report, cap, fail_json("model_bundle_contract", dir, e.what()));
    return ITTS_EBUNDLE;
  }
}

int itts_voice_load(const char* bundle_dir, uint32_t prompt_tokens, uint32_t* P_out, float* prompt_cond, float* style,
                    float* prompt_mel, char* err, uint32_t err_cap) {
  put_report(err, err_cap, "");
  try {
    if (!bundle_dir || !P_out) throw std::runtime_error("null argument");
    itts::Mit2Bundle b(bundle_dir, false);
    const VoiceShapes v = check_voice(b);
    const uint32_t P = prompt_tokens ? prompt_tokens : static_cast<uint32_t>(v.prompt);
    if (P > static_cast<uint32_t>(v.prompt))
      throw std::runtime_error("requested prompt_tokens exceeds the voice's " + std::to_string(v.prompt) + " prompt rows");
    *P_out = P;
    if (prompt_cond) {
      const std::vector<float> pc = b.as_f32("s2mel_prompt");
      std::memcpy(prompt_cond, pc.data(), static_cast<size_t>(P) * 512 * sizeof(float));
    }
    if (style) {
      const std::vector<float> s = b.as_f32("s2mel_style");
      std::memcpy(style, s.data(), 192 * sizeof(float));
    }
    if (prompt_mel) {
      const std::vector<float> m = b.as_f32("mel");  // [1][80][T_voice]
      const size_t tv = static_cast<size_t>(v.mel);
      for (uint32_t t = 0; t < P; ++t)
        for (int c = 0; c < 80; ++c) prompt_mel[static_cast<size_t>(t) * 80 + c] = m[static_cast<size_t>(c) * tv + t];
    }
    return ITTS_OK;
  } catch (const std::exception& e) {
    put_report(err, err_cap, e.what());
    return ITTS_EBUNDLE;
  }
}

}  // extern "C"
