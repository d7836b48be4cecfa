/*
 * TEST INFRASTRUCTURE — CPU oracle for the BigVGAN vocoder.
 *
 * A plain-C restatement (fp32 throughout) of the reference's CPU vocoder,
 * used only by tests/ and bench.py's CPU-baseline leg as the checker; the
 * product library never links or calls it. Its parity is pinned against the
 * reference's own compiled CPU functions (oracle/_ref) through the golden
 * vectors of tests/golden/make_golden.py.
 *
 * Reference functions restated here (paths inside raoqu/index-tts2-metal):
 *   cpu_conv1d_same                   runtime/impl/tokenizer_tests.cpp:3142-3161
 *   cpu_conv1d_dilated_same           runtime/impl/tokenizer_tests.cpp:3739-3758
 *   cpu_conv_transpose1d              runtime/impl/tokenizer_tests.cpp:3760-3783
 *   clamped_channel_sample, bigvgan_upsample_value, cpu_bigvgan_activation
 *                                     runtime/impl/tokenizer_tests.cpp:3785-3834
 *   weight_norm_conv_weight / _transpose_weight runtime/impl/gpt.cpp:5126-5136
 *   run_bigvgan_conv_pre_cpu          runtime/impl/dit_cfm_bigvgan.cpp:3606-3610
 *   kBigVGANUpsamplers, run_bigvgan_upsample_cpu runtime/impl/dit_cfm_bigvgan.cpp:3672-3694
 *   run_bigvgan_activation_cpu        runtime/impl/dit_cfm_bigvgan.cpp:3810-3816
 *   run_bigvgan_resblock_pair_cpu     runtime/impl/dit_cfm_bigvgan.cpp:3885-3900
 *   run_bigvgan_resblock_cpu          runtime/impl/dit_cfm_bigvgan.cpp:3939-3945
 *   kBigVGANResblocks, run_bigvgan_resblock_group_cpu runtime/impl/dit_cfm_bigvgan.cpp:3955-3994
 *   run_bigvgan_body_cpu              runtime/impl/dit_cfm_bigvgan.cpp:4008-4017
 *   run_bigvgan_post_cpu              runtime/impl/dit_cfm_bigvgan.cpp:4030-4039
 *   run_bigvgan_vocoder_cpu           runtime/impl/dit_cfm_bigvgan.cpp:4058-4061
 *
 * Dot products run over input channels with vectorised partial sums, so
 * results differ from the reference's sequential fp32 sums by rounding only.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
  char name[128];
  const float* p;
  size_t n;
} voc_tensor;

typedef struct {
  voc_tensor* t;
  int count;
  int cap;
} voc_model;

voc_model* voc_model_new(void) {
  voc_model* m = (voc_model*)calloc(1, sizeof(voc_model));
  m->cap = 1024;
  m->t = (voc_tensor*)calloc((size_t)m->cap, sizeof(voc_tensor));
  return m;
}

void voc_model_free(voc_model* m) {
  if (!m) return;
  free(m->t);
  free(m);
}

/* Registers a caller-owned fp32 buffer under its full bundle tensor name. */
int voc_model_set(voc_model* m, const char* name, const float* p, size_t n) {
  if (m->count == m->cap) {
    m->cap *= 2;
    m->t = (voc_tensor*)realloc(m->t, (size_t)m->cap * sizeof(voc_tensor));
  }
  voc_tensor* e = &m->t[m->count++];
  strncpy(e->name, name, sizeof(e->name) - 1);
  e->name[sizeof(e->name) - 1] = 0;
  e->p = p;
  e->n = n;
  return 0;
}

static const float* VW(const voc_model* m, const char* name, size_t want) {
  for (int i = 0; i < m->count; ++i)
    if (strcmp(m->t[i].name, name) == 0) return (want && m->t[i].n != want) ? NULL : m->t[i].p;
  return NULL;
}

/* Tensor lookup for the other stage oracles sharing this table. */
const float* voc_lookup(const voc_model* m, const char* name, size_t want) { return VW(m, name, want); }

static int v_err = 0;
int voc_last_error(void) { return v_err; }

#define VNEED(ptr)       \
  do {                   \
    if (!(ptr)) {        \
      v_err = __LINE__;  \
      goto fail;         \
    }                    \
  } while (0)

static float* vzalloc(size_t n) { return (float*)calloc(n ? n : 1, sizeof(float)); }

static float vdot(const float* a, const float* b, int n) {
  float acc = 0.0f;
#pragma omp simd reduction(+ : acc)
  for (int k = 0; k < n; ++k) acc += a[k] * b[k];
  return acc;
}

/* W[r] = g[r] * v[r] / ||v[r]|| over rows of `cols` values (weight_norm_rowmajor). */
static float* vweight_norm(const voc_model* m, const char* prefix, int rows, int cols) {
  char a[160], b[160];
  snprintf(a, sizeof(a), "%s.weight_g", prefix);
  snprintf(b, sizeof(b), "%s.weight_v", prefix);
  const float* g = VW(m, a, (size_t)rows);
  const float* v = VW(m, b, (size_t)rows * cols);
  if (!g || !v) return NULL;
  float* w = vzalloc((size_t)rows * cols);
  for (int r = 0; r < rows; ++r) {
    float nrm = 0.0f;
    for (int c = 0; c < cols; ++c) nrm += v[(size_t)r * cols + c] * v[(size_t)r * cols + c];
    nrm = sqrtf(nrm);
    const float s = g[r] / nrm;
    for (int c = 0; c < cols; ++c) w[(size_t)r * cols + c] = v[(size_t)r * cols + c] * s;
  }
  return w;
}

/* Zero-padded "same" conv with dilation: out[t][o] = b[o] + sum_{i,k}
 * x[t + k dil - pad][i] w[o][i][k], pad = (k - 1) dil / 2 (k/2 for dil 1). */
static void conv1d_zero(const float* x, const float* w, const float* bias, int T, int Cin, int Cout, int k, int dil,
                        float* out) {
  const int pad = (k - 1) * dil / 2;
  float* wt = vzalloc((size_t)Cout * k * Cin); /* [Cout][k][Cin] */
  for (int o = 0; o < Cout; ++o)
    for (int i = 0; i < Cin; ++i)
      for (int kk = 0; kk < k; ++kk) wt[((size_t)o * k + kk) * Cin + i] = w[((size_t)o * Cin + i) * k + kk];
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    for (int o = 0; o < Cout; ++o) {
      float acc = bias ? bias[o] : 0.0f;
      for (int kk = 0; kk < k; ++kk) {
        const int src = t + kk * dil - pad;
        if (src >= 0 && src < T) acc += vdot(x + (size_t)src * Cin, wt + ((size_t)o * k + kk) * Cin, Cin);
      }
      out[(size_t)t * Cout + o] = acc;
    }
  }
  free(wt);
}

/* Transposed conv, weight [Cin][Cout][k]: out_t = (T-1) s + k - 2 p rows. */
static void conv_transpose(const float* x, const float* w, const float* bias, int T, int Cin, int Cout, int k, int s,
                           int p, float* out) {
  const int To = (T - 1) * s + k - 2 * p;
  float* wt = vzalloc((size_t)k * Cout * Cin); /* [k][Cout][Cin] */
  for (int i = 0; i < Cin; ++i)
    for (int o = 0; o < Cout; ++o)
      for (int kk = 0; kk < k; ++kk) wt[((size_t)kk * Cout + o) * Cin + i] = w[((size_t)i * Cout + o) * k + kk];
#pragma omp parallel for schedule(static)
  for (int t = 0; t < To; ++t) {
    for (int o = 0; o < Cout; ++o) {
      float acc = bias[o];
      for (int kk = 0; kk < k; ++kk) {
        const int num = t + p - kk;
        if (num >= 0 && num % s == 0 && num / s < T)
          acc += vdot(x + (size_t)(num / s) * Cin, wt + ((size_t)kk * Cout + o) * Cin, Cin);
      }
      out[(size_t)t * Cout + o] = acc;
    }
  }
  free(wt);
}

static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* Anti-aliased SnakeBeta on x [T][C]: 2x upsampling by a 12-tap filter over
 * the edge-replicated signal (input pad 5, crop 15), y + sin^2(alpha y) /
 * (beta + 1e-9) with alpha = exp(alpha_log), beta = exp(beta_log), then the
 * 12-tap low-pass back to T samples over the edge-clamped upsampled signal. */
static int activation(const voc_model* m, const char* prefix, const float* x, int T, int C, float* out) {
  char n[4][192];
  snprintf(n[0], sizeof(n[0]), "%s.upsample.filter", prefix);
  snprintf(n[1], sizeof(n[1]), "%s.downsample.lowpass.filter", prefix);
  snprintf(n[2], sizeof(n[2]), "%s.act.alpha", prefix);
  snprintf(n[3], sizeof(n[3]), "%s.act.beta", prefix);
  const float* up = VW(m, n[0], 12);
  const float* dn = VW(m, n[1], 12);
  const float* al = VW(m, n[2], (size_t)C);
  const float* be = VW(m, n[3], (size_t)C);
  if (!up || !dn || !al || !be) {
    v_err = __LINE__;
    return -1;
  }
  const int U = 2 * T;
#pragma omp parallel for schedule(static)
  for (int c = 0; c < C; ++c) {
    const float alpha = expf(al[c]), beta = expf(be[c]);
    float* v = vzalloc((size_t)U);
    for (int j = 0; j < U; ++j) {
      const int full = j + 15;
      float acc = 0.0f;
      for (int k = 0; k < 12; ++k) {
        if (full >= k && ((full - k) % 2) == 0) {
          const int src = clampi((full - k) / 2 - 5, 0, T - 1);
          acc += x[(size_t)src * C + c] * up[k];
        }
      }
      const float y = 2.0f * acc;
      const float s = sinf(y * alpha);
      v[j] = y + (s * s) / (beta + 1e-9f);
    }
    for (int t = 0; t < T; ++t) {
      float acc = 0.0f;
      for (int k = 0; k < 12; ++k) acc += v[clampi(2 * t + k - 5, 0, U - 1)] * dn[k];
      out[(size_t)t * C + c] = acc;
    }
    free(v);
  }
  return 0;
}

int voc_activation(const voc_model* m, const char* prefix, const float* x, int T, int C, float* out) {
  return activation(m, prefix, x, T, C, out);
}

static const int kUps[6][5] = {{1536, 768, 8, 4, 2}, {768, 384, 8, 4, 2}, {384, 192, 4, 2, 1},
                               {192, 96, 4, 2, 1},   {96, 48, 4, 2, 1},   {48, 24, 4, 2, 1}};
static const int kRbKernel[3] = {3, 7, 11};
static const int kDil[3] = {1, 3, 5};

/* One resblock (three act -> dilated conv -> act -> conv -> + x pairs). */
static int resblock(const voc_model* m, const char* rb, const float* xin, int T, int C, int k, float* xout) {
  const size_t n = (size_t)T * C;
  float* x = vzalloc(n);
  float* a = vzalloc(n);
  float* h = vzalloc(n);
  float *w1 = NULL, *w2 = NULL;
  memcpy(x, xin, n * sizeof(float));
  for (int p = 0; p < 3; ++p) {
    char pre[160], cv[160], bn[192];
    snprintf(pre, sizeof(pre), "%s.activations.%d", rb, 2 * p);
    if (activation(m, pre, x, T, C, a)) goto fail;
    snprintf(cv, sizeof(cv), "%s.convs1.%d", rb, p);
    VNEED(w1 = vweight_norm(m, cv, C, C * k));
    snprintf(bn, sizeof(bn), "%s.bias", cv);
    const float* b1 = VW(m, bn, (size_t)C);
    VNEED(b1);
    conv1d_zero(a, w1, b1, T, C, C, k, kDil[p], h);
    snprintf(pre, sizeof(pre), "%s.activations.%d", rb, 2 * p + 1);
    if (activation(m, pre, h, T, C, a)) goto fail;
    snprintf(cv, sizeof(cv), "%s.convs2.%d", rb, p);
    VNEED(w2 = vweight_norm(m, cv, C, C * k));
    snprintf(bn, sizeof(bn), "%s.bias", cv);
    const float* b2 = VW(m, bn, (size_t)C);
    VNEED(b2);
    conv1d_zero(a, w2, b2, T, C, C, k, 1, h);
    for (size_t i = 0; i < n; ++i) x[i] = h[i] + x[i];
    free(w1);
    free(w2);
    w1 = w2 = NULL;
  }
  memcpy(xout, x, n * sizeof(float));
  free(x);
  free(a);
  free(h);
  return 0;
fail:
  free(x);
  free(a);
  free(h);
  free(w1);
  free(w2);
  return -1;
}

/* run_bigvgan_vocoder_cpu: mel [T][80] -> waveform [256 T] in [-1, 1]. */
int voc_vocoder(const voc_model* m, const float* mel, int T, float* wave) {
  float *x = NULL, *y = NULL, *rb = NULL, *acc = NULL, *w = NULL;
  const float* b;
  int t = T, C = 1536;
  VNEED(w = vweight_norm(m, "bigvgan.conv_pre", 1536, 80 * 7));
  VNEED(b = VW(m, "bigvgan.conv_pre.bias", 1536));
  x = vzalloc((size_t)T * 1536);
  conv1d_zero(mel, w, b, T, 80, 1536, 7, 1, x);
  free(w);
  w = NULL;
  for (int i = 0; i < 6; ++i) {
    const int cin = kUps[i][0], cout = kUps[i][1], k = kUps[i][2], s = kUps[i][3], p = kUps[i][4];
    char pre[64], bn[80];
    snprintf(pre, sizeof(pre), "bigvgan.ups.%d.0", i);
    VNEED(w = vweight_norm(m, pre, cin, cout * k));
    snprintf(bn, sizeof(bn), "%s.bias", pre);
    VNEED(b = VW(m, bn, (size_t)cout));
    const int to = (t - 1) * s + k - 2 * p;
    y = vzalloc((size_t)to * cout);
    conv_transpose(x, w, b, t, cin, cout, k, s, p, y);
    free(w);
    w = NULL;
    free(x);
    x = NULL;
    t = to;
    C = cout;
    /* Mean of the stage's three resblocks, accumulated as out += rb / 3. */
    acc = vzalloc((size_t)t * C);
    rb = vzalloc((size_t)t * C);
    for (int j = 0; j < 3; ++j) {
      char rbn[64];
      snprintf(rbn, sizeof(rbn), "bigvgan.resblocks.%d", 3 * i + j);
      if (resblock(m, rbn, y, t, C, kRbKernel[j], rb)) goto fail;
      for (size_t q = 0; q < (size_t)t * C; ++q) acc[q] += rb[q] / 3.0f;
    }
    free(rb);
    rb = NULL;
    free(y);
    y = NULL;
    x = acc;
    acc = NULL;
  }
  y = vzalloc((size_t)t * 24);
  if (activation(m, "bigvgan.activation_post", x, t, 24, y)) goto fail;
  VNEED(w = vweight_norm(m, "bigvgan.conv_post", 1, 24 * 7));
  conv1d_zero(y, w, NULL, t, 24, 1, 7, 1, wave);
  for (int q = 0; q < t; ++q) wave[q] = fmaxf(-1.0f, fminf(1.0f, wave[q]));
  free(w);
  free(x);
  free(y);
  return 0;
fail:
  free(x);
  free(y);
  free(rb);
  free(acc);
  free(w);
  return -1;
}
