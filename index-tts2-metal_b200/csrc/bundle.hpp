// MIT2 weight bundle reader: `manifest.json` + `weights.bin` (magic "MIT2",
// u32 version 1, u32 alignment, payloads at aligned offsets), mapped read-only.
// Format and validation rules follow the reference's bundle contract
// (docs/native_bundle.md:1-80; runtime/bundle.cpp:172-281; writer
// metal_indextts2/bundle.py:98-144).
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

namespace itts {

struct TensorRec {
  std::string name;
  std::vector<int64_t> shape;
  std::string dtype;  // f32 f16 i64 i32 u32 u8
  uint64_t offset = 0;
  uint64_t nbytes = 0;
  std::string sha256;
  std::string component;  // manifest "component" (gpt, semantic_codec, s2mel, bigvgan, voice, ...), may be empty
};

// True when `path` names a regular file: a single-file bundle (the reference's
// bundle_path_is_single_file, runtime/bundle.cpp:163).
bool bundle_is_single_file(const std::string& path);

class Mit2Bundle {
 public:
  // Opens and validates a bundle: a directory (manifest.json + weights file)
  // or a single file (weights stream + appended manifest + "MIT2VOIC"
  // footer); throws std::runtime_error with a message naming the violated
  // rule. With verify_sha256, every payload's SHA-256 is checked against the
  // manifest.
  explicit Mit2Bundle(const std::string& dir, bool verify_sha256 = false);
  ~Mit2Bundle();
  Mit2Bundle(const Mit2Bundle&) = delete;
  Mit2Bundle& operator=(const Mit2Bundle&) = delete;

  const TensorRec* find(const std::string& name) const;
  const TensorRec& require(const std::string& name) const;
  const uint8_t* data(const TensorRec& t) const { return base_ + t.offset; }
  size_t element_count(const TensorRec& t) const;
  // Decode to f32 (f16 decoding is exact); throws for non-float dtypes.
  std::vector<float> as_f32(const std::string& name) const;
  // Raw f16 payload (throws if the tensor is not f16).
  const uint16_t* as_f16(const std::string& name, size_t* count) const;
  const std::vector<TensorRec>& tensors() const { return tensors_; }
  uint32_t version() const { return version_; }
  uint64_t alignment() const { return alignment_; }
  size_t weights_bytes() const { return size_; }

 private:
  void map_file(const std::string& path);  // maps `path` read-only into base_ / size_
  std::string dir_;
  int fd_ = -1;
  const uint8_t* base_ = nullptr;
  size_t size_ = 0;
  std::vector<TensorRec> tensors_;
  std::unordered_map<std::string, size_t> by_name_;
  uint32_t version_ = 0;
  uint64_t alignment_ = 0;
};

// FIPS 180-4 SHA-256, lower-case hex digest.
std::string sha256_hex(const uint8_t* data, size_t n);

// IEEE binary16 -> binary32 (exact).
float half_bits_to_float(uint16_t h);
uint16_t float_to_half_bits(float f);  // round to nearest even

}  // namespace itts
