// MIT2 bundle reader with a small JSON parser and SHA-256 (no dependencies).
#include "bundle.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>
#include <stdexcept>

namespace itts {

namespace {

// ---- minimal JSON value + recursive-descent parser ----
struct JVal {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string numtext;
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* get(const std::string& k) const {
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

class JParser {
 public:
  explicit JParser(const std::string& s) : s_(s) {}
  JVal parse() {
    JVal v = value(0);
    ws();
    if (i_ != s_.size()) fail("trailing characters");
    return v;
  }

 private:
  const std::string& s_;
  size_t i_ = 0;
  [[noreturn]] void fail(const char* what) {
    throw std::runtime_error(std::string("manifest.json parse error: ") + what + " at offset " + std::to_string(i_));
  }
  void ws() {
    while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
  }
  JVal value(int depth) {
    if (depth > 64) fail("nesting too deep");
    ws();
    if (i_ >= s_.size()) fail("unexpected end");
    const char c = s_[i_];
    JVal v;
    if (c == '{') {
      v.kind = JVal::Obj;
      ++i_;
      ws();
      if (i_ < s_.size() && s_[i_] == '}') {
        ++i_;
        return v;
      }
      while (true) {
        ws();
        if (i_ >= s_.size() || s_[i_] != '"') fail("expected key");
        std::string k = string();
        ws();
        if (i_ >= s_.size() || s_[i_] != ':') fail("expected ':'");
        ++i_;
        v.obj.emplace_back(std::move(k), value(depth + 1));
        ws();
        if (i_ < s_.size() && s_[i_] == ',') {
          ++i_;
          continue;
        }
        if (i_ < s_.size() && s_[i_] == '}') {
          ++i_;
          break;
        }
        fail("expected ',' or '}'");
      }
    } else if (c == '[') {
      v.kind = JVal::Arr;
      ++i_;
      ws();
      if (i_ < s_.size() && s_[i_] == ']') {
        ++i_;
        return v;
      }
      while (true) {
        v.arr.push_back(value(depth + 1));
        ws();
        if (i_ < s_.size() && s_[i_] == ',') {
          ++i_;
          continue;
        }
        if (i_ < s_.size() && s_[i_] == ']') {
          ++i_;
          break;
        }
        fail("expected ',' or ']'");
      }
    } else if (c == '"') {
      v.kind = JVal::Str;
      v.str = string();
    } else if (c == 't' && s_.compare(i_, 4, "true") == 0) {
      v.kind = JVal::Bool;
      v.b = true;
      i_ += 4;
    } else if (c == 'f' && s_.compare(i_, 5, "false") == 0) {
      v.kind = JVal::Bool;
      i_ += 5;
    } else if (c == 'n' && s_.compare(i_, 4, "null") == 0) {
      i_ += 4;
    } else if (c == '-' || (c >= '0' && c <= '9')) {
      const size_t b = i_;
      ++i_;
      while (i_ < s_.size() && (std::isdigit(static_cast<unsigned char>(s_[i_])) || s_[i_] == '.' || s_[i_] == 'e' ||
                                s_[i_] == 'E' || s_[i_] == '+' || s_[i_] == '-'))
        ++i_;
      v.kind = JVal::Num;
      v.numtext = s_.substr(b, i_ - b);
      v.num = std::strtod(v.numtext.c_str(), nullptr);
    } else {
      fail("unexpected character");
    }
    return v;
  }
  std::string string() {
    ++i_;  // opening quote
    std::string out;
    while (true) {
      if (i_ >= s_.size()) fail("unterminated string");
      const char c = s_[i_++];
      if (c == '"') break;
      if (c != '\\') {
        out.push_back(c);
        continue;
      }
      if (i_ >= s_.size()) fail("bad escape");
      const char e = s_[i_++];
      switch (e) {
        case '"': out.push_back('"'); break;
        case '\\': out.push_back('\\'); break;
        case '/': out.push_back('/'); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'n': out.push_back('\n'); break;
        case 'r': out.push_back('\r'); break;
        case 't': out.push_back('\t'); break;
        case 'u': {
          if (i_ + 4 > s_.size()) fail("bad \\u escape");
          const unsigned cp = static_cast<unsigned>(std::stoul(s_.substr(i_, 4), nullptr, 16));
          i_ += 4;
          if (cp < 0x80) {
            out.push_back(static_cast<char>(cp));
          } else if (cp < 0x800) {
            out.push_back(static_cast<char>(0xC0 | (cp >> 6)));
            out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
          } else {
            out.push_back(static_cast<char>(0xE0 | (cp >> 12)));
            out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
            out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
          }
          break;
        }
        default: fail("bad escape");
      }
    }
    return out;
  }
};

uint64_t as_u64(const JVal* v, const std::string& what) {
  if (!v || v->kind != JVal::Num || v->numtext.empty() || v->numtext[0] == '-' ||
      v->numtext.find_first_of(".eE") != std::string::npos)
    throw std::runtime_error("manifest: " + what + " must be a non-negative integer");
  return std::stoull(v->numtext);
}

std::string as_str(const JVal* v, const std::string& what) {
  if (!v || v->kind != JVal::Str) throw std::runtime_error("manifest: " + what + " must be a string");
  return v->str;
}

size_t dtype_size(const std::string& d) {
  if (d == "f32" || d == "i32" || d == "u32") return 4;
  if (d == "f16") return 2;
  if (d == "i64") return 8;
  if (d == "u8") return 1;
  return 0;
}

uint32_t rd_u32(const uint8_t* p) {
  return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) | (static_cast<uint32_t>(p[2]) << 16) |
         (static_cast<uint32_t>(p[3]) << 24);
}

// ---- SHA-256 ----
constexpr uint32_t kK[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

void sha_block(uint32_t* h, const uint8_t* blk) {
  uint32_t w[64];
  for (int i = 0; i < 16; ++i)
    w[i] = (static_cast<uint32_t>(blk[4 * i]) << 24) | (static_cast<uint32_t>(blk[4 * i + 1]) << 16) |
           (static_cast<uint32_t>(blk[4 * i + 2]) << 8) | blk[4 * i + 3];
  for (int i = 16; i < 64; ++i) {
    const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
    const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
    w[i] = w[i - 16] + s0 + w[i - 7] + s1;
  }
  uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
  for (int i = 0; i < 64; ++i) {
    const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
    const uint32_t ch = (e & f) ^ (~e & g);
    const uint32_t t1 = hh + S1 + ch + kK[i] + w[i];
    const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
    const uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
    const uint32_t t2 = S0 + mj;
    hh = g;
    g = f;
    f = e;
    e = d + t1;
    d = c;
    c = b;
    b = a;
    a = t1 + t2;
  }
  h[0] += a;
  h[1] += b;
  h[2] += c;
  h[3] += d;
  h[4] += e;
  h[5] += f;
  h[6] += g;
  h[7] += hh;
}

}  // namespace

std::string sha256_hex(const uint8_t* data, size_t n) {
  uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  size_t i = 0;
  for (; i + 64 <= n; i += 64) sha_block(h, data + i);
  uint8_t tail[128];
  std::memset(tail, 0, sizeof(tail));
  const size_t rem = n - i;
  std::memcpy(tail, data + i, rem);
  tail[rem] = 0x80;
  const size_t tail_len = rem + 1 + 8 <= 64 ? 64 : 128;
  const uint64_t bits = static_cast<uint64_t>(n) * 8;
  for (int k = 0; k < 8; ++k) tail[tail_len - 1 - k] = static_cast<uint8_t>(bits >> (8 * k));
  sha_block(h, tail);
  if (tail_len == 128) sha_block(h, tail + 64);
  static const char* hex = "0123456789abcdef";
  std::string out(64, '0');
  for (int k = 0; k < 8; ++k)
    for (int j = 0; j < 8; ++j) out[k * 8 + j] = hex[(h[k] >> (28 - 4 * j)) & 0xF];
  return out;
}

float half_bits_to_float(uint16_t hbits) {
  const uint32_t sign = static_cast<uint32_t>(hbits & 0x8000u) << 16;
  const uint32_t exp = (hbits >> 10) & 0x1Fu;
  const uint32_t man = hbits & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: value = man * 2^-24
      float f = static_cast<float>(man) * 5.9604644775390625e-8f;
      std::memcpy(&bits, &f, 4);
      bits |= sign;
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}

uint16_t float_to_half_bits(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return static_cast<uint16_t>(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
  if (ax >= 0x477FF000u) return static_cast<uint16_t>(sign | 0x7C00u);  // rounds to >= 65520 -> inf
  if (ax < 0x38800000u) {                                               // subnormal or zero in f16
    if (ax < 0x33000000u) return static_cast<uint16_t>(sign);          // < 2^-25 -> 0
    const uint32_t e = ax >> 23;
    const uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
    const uint32_t shift = 126u - e;  // 14 - (e - 112)
    uint32_t r = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (r & 1u))) ++r;
    return static_cast<uint16_t>(sign | r);
  }
  uint32_t r = ((ax >> 13) - (112u << 10));
  const uint32_t rem = ax & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;
  return static_cast<uint16_t>(sign | r);
}

void Mit2Bundle::map_file(const std::string& path) {
  fd_ = ::open(path.c_str(), O_RDONLY);
  if (fd_ < 0) throw std::runtime_error("bundle: missing weights file " + path);
  struct stat st {};
  if (fstat(fd_, &st) != 0) throw std::runtime_error("bundle: cannot stat " + path);
  size_ = static_cast<size_t>(st.st_size);
  if (size_ < 12) throw std::runtime_error("bundle: weights file too small for the MIT2 header");
  void* p = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
  if (p == MAP_FAILED) throw std::runtime_error("bundle: mmap failed for " + path);
  base_ = static_cast<const uint8_t*>(p);
}

bool bundle_is_single_file(const std::string& path) {
  struct stat st {};
  return ::stat(path.c_str(), &st) == 0 && S_ISREG(st.st_mode);
}

Mit2Bundle::Mit2Bundle(const std::string& dir, bool verify_sha256) : dir_(dir) {
  // Two forms (the reference's Bundle constructor, runtime/bundle.cpp:172-213):
  // a directory holding manifest.json + the weights file, or ONE file that is a
  // valid MIT2 weights stream with the manifest JSON appended after the
  // payloads and a 24-byte footer [u64 manifest offset][u64 manifest size]
  // ["MIT2VOIC"] (little endian) at its very end.
  const bool single_file = bundle_is_single_file(dir);
  std::string text;
  if (single_file) {
    map_file(dir);
    constexpr size_t kFooter = 24;
    if (size_ < 12 + kFooter) throw std::runtime_error("bundle: single-file bundle is too small: " + dir);
    const uint8_t* foot = base_ + size_ - kFooter;
    if (std::memcmp(foot + 16, "MIT2VOIC", 8) != 0)
      throw std::runtime_error("bundle: single-file bundle footer magic missing: " + dir);
    uint64_t moff = 0, msize = 0;
    for (int b = 7; b >= 0; --b) {
      moff = (moff << 8) | foot[b];
      msize = (msize << 8) | foot[8 + b];
    }
    const uint64_t limit = size_ - kFooter;
    if (moff > limit || msize > limit - moff)
      throw std::runtime_error("bundle: single-file bundle manifest exceeds the file: " + dir);
    text.assign(reinterpret_cast<const char*>(base_ + moff), static_cast<size_t>(msize));
  } else {
    std::ifstream mf(dir + "/manifest.json");
    if (!mf) throw std::runtime_error("bundle: cannot open " + dir + "/manifest.json");
    std::stringstream ss;
    ss << mf.rdbuf();
    text = ss.str();
  }
  JVal root = JParser(text).parse();
  if (root.kind != JVal::Obj) throw std::runtime_error("manifest: root must be an object");
  const std::string format = as_str(root.get("format"), "format");
  if (format != "MIT2") throw std::runtime_error("bundle: unsupported format '" + format + "'");
  const uint64_t version = as_u64(root.get("version"), "version");
  if (version != 1) throw std::runtime_error("bundle: unsupported version " + std::to_string(version));
  const JVal* endian = root.get("endianness");
  if (endian && as_str(endian, "endianness") != "little")
    throw std::runtime_error("bundle: unsupported endianness '" + endian->str + "'");
  const uint64_t alignment = as_u64(root.get("alignment"), "alignment");
  if (alignment == 0) throw std::runtime_error("bundle: alignment must be non-zero");
  version_ = static_cast<uint32_t>(version);
  alignment_ = alignment;
  if (!single_file) {
    std::string wname = "weights.bin";
    if (const JVal* wf = root.get("weights_file")) wname = as_str(wf, "weights_file");
    map_file(dir + "/" + wname);
  }
  if (std::memcmp(base_, "MIT2", 4) != 0) throw std::runtime_error("bundle: weights file has an invalid MIT2 magic");
  if (rd_u32(base_ + 4) != version) throw std::runtime_error("bundle: weights header version mismatch");
  if (rd_u32(base_ + 8) != alignment) throw std::runtime_error("bundle: weights header alignment mismatch");

  const JVal* tl = root.get("tensors");
  if (!tl || tl->kind != JVal::Arr) throw std::runtime_error("manifest: missing tensors array");
  for (const JVal& o : tl->arr) {
    if (o.kind != JVal::Obj) throw std::runtime_error("manifest: tensor record must be an object");
    TensorRec t;
    t.name = as_str(o.get("name"), "tensor name");
    if (t.name.empty()) throw std::runtime_error("manifest: tensor record has an empty name");
    const JVal* sh = o.get("shape");
    if (!sh || sh->kind != JVal::Arr) throw std::runtime_error("manifest: tensor " + t.name + " has no shape");
    for (const JVal& d : sh->arr) t.shape.push_back(static_cast<int64_t>(as_u64(&d, "shape dim")));
    t.dtype = as_str(o.get("dtype"), "dtype");
    t.offset = as_u64(o.get("offset"), "offset");
    t.nbytes = as_u64(o.get("nbytes"), "nbytes");
    if (const JVal* h = o.get("sha256")) t.sha256 = as_str(h, "sha256");
    if (const JVal* c = o.get("component")) t.component = as_str(c, "component");
    if (by_name_.count(t.name)) throw std::runtime_error("bundle: duplicate tensor " + t.name);
    if (t.nbytes == 0) throw std::runtime_error("bundle: zero-byte tensor " + t.name);
    if (t.offset % alignment != 0) throw std::runtime_error("bundle: unaligned tensor offset for " + t.name);
    const size_t es = dtype_size(t.dtype);
    if (es == 0) throw std::runtime_error("bundle: unsupported dtype '" + t.dtype + "' for " + t.name);
    uint64_t count = 1;
    for (int64_t d : t.shape) count *= static_cast<uint64_t>(d);
    if (count * es != t.nbytes) throw std::runtime_error("bundle: dtype/shape byte count mismatch for " + t.name);
    if (t.offset < 12 || t.offset + t.nbytes > size_) throw std::runtime_error("bundle: tensor " + t.name + " extends beyond the weights file");
    by_name_[t.name] = tensors_.size();
    tensors_.push_back(std::move(t));
  }
  // Overlap check over payload ranges.
  std::vector<size_t> order(tensors_.size());
  for (size_t i = 0; i < order.size(); ++i) order[i] = i;
  std::sort(order.begin(), order.end(), [&](size_t a, size_t b) { return tensors_[a].offset < tensors_[b].offset; });
  for (size_t i = 1; i < order.size(); ++i) {
    const TensorRec& a = tensors_[order[i - 1]];
    const TensorRec& b = tensors_[order[i]];
    if (a.offset + a.nbytes > b.offset) throw std::runtime_error("bundle: overlapping payloads " + a.name + " / " + b.name);
  }
  if (verify_sha256) {
    for (const TensorRec& t : tensors_) {
      if (t.sha256.empty()) continue;
      if (sha256_hex(data(t), t.nbytes) != t.sha256) throw std::runtime_error("bundle: checksum mismatch for " + t.name);
    }
  }
}

Mit2Bundle::~Mit2Bundle() {
  if (base_) munmap(const_cast<uint8_t*>(base_), size_);
  if (fd_ >= 0) ::close(fd_);
}

const TensorRec* Mit2Bundle::find(const std::string& name) const {
  auto it = by_name_.find(name);
  return it == by_name_.end() ? nullptr : &tensors_[it->second];
}

const TensorRec& Mit2Bundle::require(const std::string& name) const {
  const TensorRec* t = find(name);
  if (!t) throw std::runtime_error("bundle: missing tensor " + name);
  return *t;
}

size_t Mit2Bundle::element_count(const TensorRec& t) const {
  size_t c = 1;
  for (int64_t d : t.shape) c *= static_cast<size_t>(d);
  return c;
}

std::vector<float> Mit2Bundle::as_f32(const std::string& name) const {
  const TensorRec& t = require(name);
  const size_t n = element_count(t);
  std::vector<float> out(n);
  if (t.dtype == "f32") {
    std::memcpy(out.data(), data(t), n * 4);
  } else if (t.dtype == "f16") {
    const uint8_t* p = data(t);
    for (size_t i = 0; i < n; ++i) {
      uint16_t h;
      std::memcpy(&h, p + 2 * i, 2);
      out[i] = half_bits_to_float(h);
    }
  } else {
    throw std::runtime_error("bundle: tensor " + name + " is not floating point (" + t.dtype + ")");
  }
  return out;
}

const uint16_t* Mit2Bundle::as_f16(const std::string& name, size_t* count) const {
  const TensorRec& t = require(name);
  if (t.dtype != "f16") throw std::runtime_error("bundle: tensor " + name + " is not f16");
  if (count) *count = element_count(t);
  return reinterpret_cast<const uint16_t*>(data(t));
}

}  // namespace itts
