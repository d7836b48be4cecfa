// itts_make_noise: the sampler's seeded initial noise x0, bit-identical to the
// reference's make_deterministic_normal_noise
// (runtime/impl/tokenizer_tests.cpp:2102-2140), which its synthesis pipeline
// draws for every utterance (runtime/impl/tts_synthesis/synthesis_pipeline.cpp:1333).
//
// The generator is a SplitMix64 stream; each pair of draws becomes two
// normals by the Box-Muller transform in single precision. Bit identity with
// the reference needs the same float operations in the same order and the
// host C library's logf/sqrtf/cosf/sinf, so this runs on the host (it is a
// few microseconds per utterance, before the sampler's upload).
#include <cmath>
#include <cstdint>
#include <cstring>

#include "itts_cfm.h"

namespace {

// One step of the SplitMix64 sequence (Steele, Lea and Flood 2014): a Weyl
// increment followed by two xor-shift-multiply rounds.
inline uint64_t splitmix_step(uint64_t* state) {
  *state += 0x9e3779b97f4a7c15ull;
  uint64_t z = *state;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// A uniform draw in the open interval (0, 1): the top 53 bits centred in
// their cell, clamped one cell inside both ends, then rounded to float.
inline float open_unit_draw(uint64_t* state) {
  const double cell = 1.0 / 9007199254740992.0;  // 2^-53
  double v = (static_cast<double>(splitmix_step(state) >> 11) + 0.5) * cell;
  if (v <= 0.0) v = cell;
  if (v >= 1.0) v = 1.0 - cell;
  return static_cast<float>(v);
}

}  // namespace

extern "C" int itts_make_noise(uint32_t tokens, uint32_t channels, uint64_t seed, float temperature, float* out) {
  if (!out || tokens == 0 || channels == 0 || tokens > ITTS_MAX_T || channels > ITTS_NOISE_MAX_CHANNELS)
    return ITTS_EINVAL_SHAPE;
  const size_t n = static_cast<size_t>(tokens) * channels;
  const float kTwoPi = 6.2831853071795864769f;
  uint64_t state = seed;
  for (size_t i = 0; i < n; i += 2) {
    const float u1 = open_unit_draw(&state);
    const float u2 = open_unit_draw(&state);
    const float r = std::sqrt(-2.0f * std::log(u1));
    const float a = kTwoPi * u2;
    out[i] = r * std::cos(a) * temperature;
    if (i + 1 < n) out[i + 1] = r * std::sin(a) * temperature;
  }
  return ITTS_OK;
}
