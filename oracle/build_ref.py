"""TEST INFRASTRUCTURE — build the checkers under oracle/.

1. oracle/lib/libdit_oracle.so from oracle/dit_oracle.c,
   oracle/bigvgan_oracle.c and oracle/condition_oracle.c (the C restatements).
2. oracle/_ref/libref_cfm.so: the reference's own CPU DiT-CFM functions,
   compiled where they lie in the read-only reference tree. The functions live
   inside large translation units that also hold Metal code, so this script
   writes a git-ignored translation unit oracle/_ref/ref_tu.cpp that pulls the
   needed function definitions by line range (each preceded by a #line
   directive naming its origin), then compiles it with g++ together with the
   reference's runtime/bundle.cpp and oracle/ref_driver.cpp. Nothing from the
   reference is committed; outputs stay in oracle/_ref/. Step 2 is skipped
   when the reference tree is absent (the prebuilt .so travels instead).

    python oracle/build_ref.py [--reference DIR]
"""
from __future__ import annotations

import argparse
import os
import subprocess
from pathlib import Path

ORACLE = Path(__file__).resolve().parent
REF_OUT = ORACLE / "_ref"
LIB_OUT = ORACLE / "lib"
# The reference tree: $ITTS_REFERENCE_DIR, else a `reference` checkout next to
# this repository's directory (when neither exists, build_ref() skips).
DEFAULT_REF = Path(os.environ.get("ITTS_REFERENCE_DIR", str(ORACLE.parent.parent / "reference")))

# (file inside the reference, first line, last line) of each function group.
RANGES = [
    ("runtime/impl/tokenizer_tests.cpp", 2102, 2140),  # splitmix64 noise
    ("runtime/impl/tokenizer_tests.cpp", 2992, 3036),  # layernorm, rmsnorm, linear
    ("runtime/impl/tokenizer_tests.cpp", 3097, 3104),  # silu
    ("runtime/impl/tokenizer_tests.cpp", 3127, 3141),  # nearest interpolation
    ("runtime/impl/tokenizer_tests.cpp", 3142, 3161),  # conv1d same
    ("runtime/impl/tokenizer_tests.cpp", 3739, 3834),  # dilated conv, transposed conv, anti-aliased SnakeBeta
    ("runtime/impl/tokenizer_tests.cpp", 3836, 3872),  # reflect pad, slice, reflect conv
    ("runtime/impl/tokenizer_tests.cpp", 3874, 3904),  # groupnorm (one group), mish
    ("runtime/impl/tokenizer_tests.cpp", 3931, 3945),  # gelu_new
    ("runtime/impl/tokenizer_tests.cpp", 3947, 4001),  # timestep embedding, masked attention
    ("runtime/impl/tokenizer_tests.cpp", 4003, 4061),  # causal and single-query attention
    ("runtime/impl/tokenizer_tests.cpp", 4266, 4333),  # rope, half_to_float, tensor_as_f32
    ("runtime/impl/gpt.cpp", 5109, 5136),  # weight norm (linear, conv, transposed conv)
    ("runtime/impl/gpt.cpp", 208, 216),  # GPT Conv1D weight transpose
    ("runtime/impl/gpt.cpp", 371, 395),  # GPT causal attention core
    ("runtime/impl/gpt.cpp", 658, 711),  # GPT transformer block (full sequence)
    ("runtime/impl/gpt.cpp", 1060, 1077),  # GPT layer QKV
    ("runtime/impl/gpt.cpp", 1115, 1170),  # GPT KV cache, cached attention
    ("runtime/impl/gpt.cpp", 1180, 1210),  # GPT cached block
    ("runtime/impl/gpt.cpp", 1297, 1308),  # argmax
    ("runtime/impl/gpt.cpp", 1545, 1554),  # GPT current-token embedding
    ("runtime/impl/gpt.cpp", 1583, 1590),  # GPT greedy outputs
    ("runtime/impl/gpt.cpp", 1592, 1755),  # GPT sampling: config, SplitMix64, logits processors, sampler
    ("runtime/impl/gpt.cpp", 1792, 1806),  # GPT KV prefill
    ("runtime/impl/gpt.cpp", 1873, 1909),  # GPT KV greedy decode
    ("runtime/impl/gpt.cpp", 5271, 5281),  # length regulator front (content_in_proj + interpolation)
    ("runtime/impl/gpt.cpp", 5298, 5317),  # length regulator (conv / groupnorm / mish blocks)
    ("runtime/impl/gpt.cpp", 5404, 5422),  # timestep embedder
    ("runtime/impl/dit_cfm_bigvgan.cpp", 1, 19),  # input merge
    ("runtime/impl/dit_cfm_bigvgan.cpp", 260, 276),  # adaptive norm
    ("runtime/impl/dit_cfm_bigvgan.cpp", 469, 512),  # attention core
    ("runtime/impl/dit_cfm_bigvgan.cpp", 727, 746),  # feed forward
    ("runtime/impl/dit_cfm_bigvgan.cpp", 785, 798),  # skip in
    ("runtime/impl/dit_cfm_bigvgan.cpp", 816, 832),  # block
    ("runtime/impl/dit_cfm_bigvgan.cpp", 868, 886),  # stack
    ("runtime/impl/dit_cfm_bigvgan.cpp", 1038, 1049),  # post-transformer structs
    ("runtime/impl/dit_cfm_bigvgan.cpp", 1053, 1079),  # post-transformer projections
    ("runtime/impl/dit_cfm_bigvgan.cpp", 1172, 1199),  # final layer
    ("runtime/impl/dit_cfm_bigvgan.cpp", 1464, 1514),  # wavenet
    ("runtime/impl/dit_cfm_bigvgan.cpp", 1768, 1788),  # estimator step
    ("runtime/impl/dit_cfm_bigvgan.cpp", 2908, 2937),  # euler sampler
    ("runtime/impl/dit_cfm_bigvgan.cpp", 3606, 3610),  # BigVGAN conv_pre
    ("runtime/impl/dit_cfm_bigvgan.cpp", 3672, 3694),  # BigVGAN upsamplers
    ("runtime/impl/dit_cfm_bigvgan.cpp", 3810, 3816),  # BigVGAN activation
    ("runtime/impl/dit_cfm_bigvgan.cpp", 3885, 3900),  # BigVGAN resblock pair
    ("runtime/impl/dit_cfm_bigvgan.cpp", 3939, 3945),  # BigVGAN resblock
    ("runtime/impl/dit_cfm_bigvgan.cpp", 3955, 3994),  # BigVGAN resblock specs, group
    ("runtime/impl/dit_cfm_bigvgan.cpp", 4008, 4017),  # BigVGAN body
    ("runtime/impl/dit_cfm_bigvgan.cpp", 4030, 4039),  # BigVGAN post
    ("runtime/impl/dit_cfm_bigvgan.cpp", 4058, 4061),  # BigVGAN vocoder
]

PRELUDE = """// Generated by oracle/build_ref.py from the reference tree; do not commit.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>
#include "mit2/bundle.hpp"
"""


# Our own glue inside the generated unit: the greedy decoder returns a struct
# the driver (a separate unit) cannot see, so it is unpacked here.
GLUE = """
// ---- glue written by oracle/build_ref.py (not reference code) ----
void ref_glue_gpt_kv_greedy(const mit2::Bundle& bundle, const std::vector<float>& prefix, uint32_t prefix_tokens,
                            uint32_t steps, bool hf_generate_positions, std::vector<uint32_t>* tokens,
                            std::vector<float>* last_logits, int* first_stop) {
  GptGreedyOutputs o = run_gpt_kv_greedy_cpu(bundle, prefix, prefix_tokens, steps, hf_generate_positions);
  *tokens = o.predicted_tokens;
  *last_logits = o.last_logits;
  *first_stop = o.first_stop_step;
}

void ref_glue_gpt_sample(const std::vector<float>& logits, const std::vector<uint32_t>& history, uint64_t seed,
                         float temperature, uint32_t top_k, float top_p, float repetition_penalty, uint32_t draws,
                         std::vector<float>* processed, std::vector<uint32_t>* tokens) {
  GptSamplingConfig c;
  c.do_sample = true;
  c.seed = seed;
  c.temperature = temperature;
  c.top_k = top_k;
  c.top_p = top_p;
  c.repetition_penalty = repetition_penalty;
  *processed = apply_gpt_sampling_processors(logits, history, c);
  SplitMix64 rng(seed);
  tokens->clear();
  for (uint32_t d = 0; d < draws; ++d) tokens->push_back(sample_gpt_token_from_logits(*processed, rng));
}
"""


def build_port(cc: str = "gcc") -> Path:
    LIB_OUT.mkdir(parents=True, exist_ok=True)
    out = LIB_OUT / "libdit_oracle.so"
    srcs = [ORACLE / "dit_oracle.c", ORACLE / "bigvgan_oracle.c", ORACLE / "condition_oracle.c"]
    if out.exists() and out.stat().st_mtime >= max(s.stat().st_mtime for s in srcs):
        return out
    cmd = [cc, "-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", "-std=c11", "-o", str(out),
           *[str(s) for s in srcs], "-lm"]
    subprocess.run(cmd, check=True)
    return out


def build_ref(reference: Path = DEFAULT_REF, cxx: str = "g++") -> Path | None:
    if not (reference / "runtime" / "impl" / "dit_cfm_bigvgan.cpp").exists():
        return None
    REF_OUT.mkdir(parents=True, exist_ok=True)
    out = REF_OUT / "libref_cfm.so"
    driver = ORACLE / "ref_driver.cpp"
    if out.exists() and out.stat().st_mtime >= max(driver.stat().st_mtime, Path(__file__).stat().st_mtime):
        return out
    parts = [PRELUDE]
    for rel, a, b in RANGES:
        lines = (reference / rel).read_text(encoding="utf-8", errors="replace").splitlines()
        parts.append(f'#line {a} "{rel}"')
        parts.extend(lines[a - 1 : b])
        parts.append("")
    parts.append(GLUE)
    tu = REF_OUT / "ref_tu.cpp"
    tu.write_text("\n".join(parts) + "\n", encoding="utf-8")
    inc = reference / "runtime" / "include"
    flags = ["-O3", "-std=c++17", "-fPIC", "-include", "memory", "-I", str(inc), "-w"]
    objs = []
    for src in (tu, reference / "runtime" / "bundle.cpp", driver):
        obj = REF_OUT / (src.stem + ".o")
        subprocess.run([cxx, *flags, "-c", str(src), "-o", str(obj)], check=True)
        objs.append(str(obj))
    subprocess.run([cxx, "-shared", "-o", str(out), *objs], check=True)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=DEFAULT_REF)
    a = ap.parse_args()
    print(build_port())
    print(build_ref(a.reference))
