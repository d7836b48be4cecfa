/*
 * TEST INFRASTRUCTURE — CPU oracle for the condition assembly before the CFM
 * sampler: the S2Mel length regulator and the prompt/generated merge.
 *
 * A plain-C restatement (fp32) used only by tests/ and bench.py's CPU-baseline
 * leg as the checker; the product library never links or calls it. Its parity
 * is pinned against the reference's own compiled CPU functions (oracle/_ref)
 * through tests/golden/kat_length_regulator.npz (tests/golden/make_golden.py).
 * Tensors come from the table of oracle/bigvgan_oracle.c (full bundle names).
 *
 * Reference functions restated here (paths inside raoqu/index-tts2-metal):
 *   cpu_linear                    runtime/impl/tokenizer_tests.cpp:3026-3036
 *   cpu_nearest_interpolate       runtime/impl/tokenizer_tests.cpp:3127-3141
 *   cpu_conv1d_same               runtime/impl/tokenizer_tests.cpp:3142-3161
 *   cpu_groupnorm1, cpu_mish      runtime/impl/tokenizer_tests.cpp:3874-3904
 *   run_length_regulator_front_cpu runtime/impl/gpt.cpp:5271-5281
 *   run_length_regulator_full_cpu runtime/impl/gpt.cpp:5298-5317
 *   mit2_hot_condition_merge_f32  metal/kernels.metal:843-864 (prompt rows, then generated rows)
 *
 * The GroupNorm statistics are sequential fp32 sums in element order, as in
 * the reference; the conv and linear dot products use vectorised partial sums.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct voc_model voc_model;
const float* voc_lookup(const voc_model* m, const char* name, size_t want);

static int c_err = 0;
int cond_last_error(void) { return c_err; }

static float cdot(const float* a, const float* b, int n) {
  float acc = 0.0f;
#pragma omp simd reduction(+ : acc)
  for (int k = 0; k < n; ++k) acc += a[k] * b[k];
  return acc;
}

#define LRP "s2mel.net.length_regulator."

/* "same" zero-padded conv, weight [Cout][Cin][k] (C = 512). */
static void conv_same(const float* x, const float* w, const float* b, int T, int k, float* out) {
  const int C = 512, pad = k / 2;
  float* wt = (float*)calloc((size_t)C * k * C, sizeof(float)); /* [o][k][i] */
  for (int o = 0; o < C; ++o)
    for (int i = 0; i < C; ++i)
      for (int kk = 0; kk < k; ++kk) wt[((size_t)o * k + kk) * C + i] = w[((size_t)o * C + i) * k + kk];
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t)
    for (int o = 0; o < C; ++o) {
      float acc = b[o];
      for (int kk = 0; kk < k; ++kk) {
        const int s = t + kk - pad;
        if (s >= 0 && s < T) acc += cdot(x + (size_t)s * C, wt + ((size_t)o * k + kk) * C, C);
      }
      out[(size_t)t * C + o] = acc;
    }
  free(wt);
}

/* run_length_regulator_full_cpu: x [n_in][1024] -> out [n_out][512]. */
int cond_length_regulator(const voc_model* m, const float* x, int n_in, int n_out, float* out) {
  const int C = 512;
  const float* W = voc_lookup(m, LRP "content_in_proj.weight", (size_t)C * 1024);
  const float* B = voc_lookup(m, LRP "content_in_proj.bias", C);
  if (!W || !B || n_in < 1 || n_out < 1) {
    c_err = __LINE__;
    return -1;
  }
  float* proj = (float*)calloc((size_t)n_in * C, sizeof(float));
  float* a = (float*)calloc((size_t)n_out * C, sizeof(float));
  float* h = (float*)calloc((size_t)n_out * C, sizeof(float));
#pragma omp parallel for schedule(static)
  for (int t = 0; t < n_in; ++t)
    for (int o = 0; o < C; ++o) proj[(size_t)t * C + o] = B[o] + cdot(W + (size_t)o * 1024, x + (size_t)t * 1024, 1024);
  const float scale = (float)n_in / (float)n_out;
  for (int t = 0; t < n_out; ++t) {
    uint32_t src = (uint32_t)floorf((float)t * scale);
    if (src >= (uint32_t)n_in) src = (uint32_t)n_in - 1;
    memcpy(a + (size_t)t * C, proj + (size_t)src * C, C * sizeof(float));
  }
  const int convs[4] = {0, 3, 6, 9}, norms[4] = {1, 4, 7, 10};
  const size_t n = (size_t)n_out * C;
  int rc = 0;
  for (int blk = 0; blk < 4 && rc == 0; ++blk) {
    char nw[96], nb[96], gw[96], gb[96];
    snprintf(nw, sizeof(nw), LRP "model.%d.weight", convs[blk]);
    snprintf(nb, sizeof(nb), LRP "model.%d.bias", convs[blk]);
    snprintf(gw, sizeof(gw), LRP "model.%d.weight", norms[blk]);
    snprintf(gb, sizeof(gb), LRP "model.%d.bias", norms[blk]);
    const float* cw = voc_lookup(m, nw, (size_t)C * C * 3);
    const float* cb = voc_lookup(m, nb, C);
    const float* g = voc_lookup(m, gw, C);
    const float* be = voc_lookup(m, gb, C);
    if (!cw || !cb || !g || !be) {
      c_err = __LINE__;
      rc = -1;
      break;
    }
    conv_same(a, cw, cb, n_out, 3, h);
    float mean = 0.0f;
    for (size_t i = 0; i < n; ++i) mean += h[i];
    mean /= (float)n;
    float var = 0.0f;
    for (size_t i = 0; i < n; ++i) {
      const float d = h[i] - mean;
      var += d * d;
    }
    var /= (float)n;
    const float inv = 1.0f / sqrtf(var + 1e-5f);
    for (size_t i = 0; i < n; ++i) {
      const int c = (int)(i % C);
      const float v = (h[i] - mean) * inv * g[c] + be[c];
      a[i] = v * tanhf(log1pf(expf(v)));
    }
  }
  if (rc == 0) {
    const float* fw = voc_lookup(m, LRP "model.12.weight", (size_t)C * C);
    const float* fb = voc_lookup(m, LRP "model.12.bias", C);
    if (!fw || !fb) {
      c_err = __LINE__;
      rc = -1;
    } else {
      conv_same(a, fw, fb, n_out, 1, out);
    }
  }
  free(proj);
  free(a);
  free(h);
  return rc;
}

/* Condition assembly: cond = [prompt rows (P); length-regulated rows (G)]. */
int cond_assemble(const voc_model* m, const float* x, int n_in, const float* prompt, int P, int G, float* cond) {
  if (P > 0) memcpy(cond, prompt, (size_t)P * 512 * sizeof(float));
  return cond_length_regulator(m, x, n_in, G, cond + (size_t)P * 512);
}
