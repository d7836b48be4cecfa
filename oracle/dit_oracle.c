/*
 * TEST INFRASTRUCTURE — CPU oracle for the DiT-CFM mel decoder.
 *
 * A plain-C restatement of the reference's CPU path (fp32 throughout) used
 * only by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as
 * the checker. The product (libitts_cfm.so) never links or calls this file.
 *
 * Parity of this restatement is pinned against the reference's own compiled
 * CPU functions (oracle/_ref, built by oracle/build_ref.py) through the golden
 * vectors under tests/golden/ (see tests/golden/make_golden.py).
 *
 * Reference functions restated here (paths inside raoqu/index-tts2-metal):
 *   cpu_linear                 runtime/impl/tokenizer_tests.cpp:3026-3036
 *   cpu_rmsnorm                runtime/impl/tokenizer_tests.cpp:3012-3024
 *   cpu_layernorm              runtime/impl/tokenizer_tests.cpp:2992-3010
 *   cpu_conv1d_same            runtime/impl/tokenizer_tests.cpp:3142-3161
 *   reflect_pad_1d             runtime/impl/tokenizer_tests.cpp:3836-3854
 *   cpu_conv1d_reflect_same    runtime/impl/tokenizer_tests.cpp:3866-3872
 *   cpu_timestep_embedding     runtime/impl/tokenizer_tests.cpp:3947-3958
 *   cpu_attention_single_head_masked runtime/impl/tokenizer_tests.cpp:3960-3997
 *   apply_rope_inplace         runtime/impl/tokenizer_tests.cpp:4266-4281
 *   weight_norm_rowmajor       runtime/impl/gpt.cpp:5109-5124
 *   run_timestep_embedder_cpu  runtime/impl/gpt.cpp:5404-5422
 *   run_dit_input_merge_cpu    runtime/impl/dit_cfm_bigvgan.cpp:1-19
 *   run_adaptive_norm_cpu      runtime/impl/dit_cfm_bigvgan.cpp:260-276
 *   run_dit_attention_core_cpu_masked_layer runtime/impl/dit_cfm_bigvgan.cpp:469-512
 *   run_dit_feed_forward_cpu_layer runtime/impl/dit_cfm_bigvgan.cpp:727-746
 *   run_skip_in_cpu            runtime/impl/dit_cfm_bigvgan.cpp:785-798
 *   run_dit_transformer_block_cpu_layer runtime/impl/dit_cfm_bigvgan.cpp:816-832
 *   run_dit_transformer_stack_cpu runtime/impl/dit_cfm_bigvgan.cpp:868-886
 *   run_dit_post_transformer_proj_cpu runtime/impl/dit_cfm_bigvgan.cpp:1053-1079
 *   run_dit_final_layer_cpu    runtime/impl/dit_cfm_bigvgan.cpp:1172-1199
 *   run_wavenet_stack_global_cond_cpu runtime/impl/dit_cfm_bigvgan.cpp:1464-1514
 *   run_dit_estimator_step_cpu runtime/impl/dit_cfm_bigvgan.cpp:1768-1788
 *   run_cfm_euler_cpu          runtime/impl/dit_cfm_bigvgan.cpp:2908-2937
 *   make_deterministic_normal_noise runtime/impl/tokenizer_tests.cpp:2102-2140
 *
 * Dot products use vectorised partial sums (OpenMP simd), so results differ
 * from the reference's strictly sequential fp32 sums by rounding only.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct {
  char name[128];
  const float* p;
  size_t n;
} orc_tensor;

typedef struct {
  orc_tensor* t;
  int count;
  int cap;
} orc_model;

/* ---------------- tensor table ---------------- */

orc_model* orc_model_new(void) {
  orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
  m->cap = 512;
  m->t = (orc_tensor*)calloc((size_t)m->cap, sizeof(orc_tensor));
  return m;
}

void orc_model_free(orc_model* m) {
  if (!m) return;
  free(m->t);
  free(m);
}

/* Registers a caller-owned fp32 buffer under the bundle tensor name. */
int orc_model_set(orc_model* m, const char* name, const float* p, size_t n) {
  if (m->count == m->cap) {
    m->cap *= 2;
    m->t = (orc_tensor*)realloc(m->t, (size_t)m->cap * sizeof(orc_tensor));
  }
  orc_tensor* e = &m->t[m->count++];
  strncpy(e->name, name, sizeof(e->name) - 1);
  e->name[sizeof(e->name) - 1] = 0;
  e->p = p;
  e->n = n;
  return 0;
}

static const float* W(const orc_model* m, const char* name, size_t want) {
  static const char* pre = "s2mel.net.cfm.estimator.";
  char full[256];
  snprintf(full, sizeof(full), "%s%s", pre, name);
  for (int i = 0; i < m->count; ++i) {
    if (strcmp(m->t[i].name, full) == 0) {
      if (want && m->t[i].n != want) return NULL;
      return m->t[i].p;
    }
  }
  return NULL;
}

static int g_err = 0;
int orc_last_error(void) { return g_err; }

#define NEED(ptr)          \
  do {                     \
    if (!(ptr)) {          \
      g_err = __LINE__;    \
      return -1;           \
    }                      \
  } while (0)

static float* fzalloc(size_t n) { return (float*)calloc(n ? n : 1, sizeof(float)); }

/* ---------------- primitives ---------------- */

static float dot(const float* a, const float* b, int n) {
  float acc = 0.0f;
#pragma omp simd reduction(+ : acc)
  for (int k = 0; k < n; ++k) acc += a[k] * b[k];
  return acc;
}

/* out[t][n] = bias[n] + W[n] . x[t]  (cpu_linear applied per token row). */
static void linear_rows(const float* Wt, const float* bias, const float* x, int T, int N, int K, float* out) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int t = 0; t < T; ++t)
    for (int n = 0; n < N; ++n)
      out[(size_t)t * N + n] = (bias ? bias[n] : 0.0f) + dot(Wt + (size_t)n * K, x + (size_t)t * K, K);
}

static float silu(float v) { return v / (1.0f + expf(-v)); }

/* weight_norm_rowmajor: W[r] = g[r] * v[r] / ||v[r]||. */
static float* weight_norm(const float* g, const float* v, int rows, int cols) {
  float* w = fzalloc((size_t)rows * cols);
  for (int r = 0; r < rows; ++r) {
    float nrm = 0.0f;
    for (int c = 0; c < cols; ++c) nrm += v[(size_t)r * cols + c] * v[(size_t)r * cols + c];
    nrm = sqrtf(nrm);
    const float s = g[r] / nrm;
    for (int c = 0; c < cols; ++c) w[(size_t)r * cols + c] = v[(size_t)r * cols + c] * s;
  }
  return w;
}

static float* weight_norm_named(const orc_model* m, const char* prefix, int rows, int cols) {
  char a[160], b[160];
  snprintf(a, sizeof(a), "%s.weight_g", prefix);
  snprintf(b, sizeof(b), "%s.weight_v", prefix);
  const float* g = W(m, a, (size_t)rows);
  const float* v = W(m, b, (size_t)rows * cols);
  if (!g || !v) return NULL;
  return weight_norm(g, v, rows, cols);
}

/* Reflect source row of padded position j (reflect_pad_1d); T >= 2. */
static int reflect_row(int j, int T) {
  int s = j;
  while (s < 0 || s >= T) {
    if (s < 0) s = -s;
    if (s >= T) s = 2 * T - 2 - s;
  }
  return s;
}

/* "same" conv with reflect padding, weight [Cout][Cin][k]. */
static void conv1d_reflect_same(const float* x, const float* w, const float* bias, int T, int Cin, int Cout, int k,
                                float* out) {
  const int pad = k / 2;
  /* Gather the padded rows once, then per output row a tap-major dot. */
  float* wt = fzalloc((size_t)Cout * Cin * k); /* [Cout][k][Cin] */
  for (int o = 0; o < Cout; ++o)
    for (int c = 0; c < Cin; ++c)
      for (int j = 0; j < k; ++j) wt[((size_t)o * k + j) * Cin + c] = w[((size_t)o * Cin + c) * k + j];
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    int src[16];
    for (int j = 0; j < k; ++j) src[j] = reflect_row(t + j - pad, T);
    for (int o = 0; o < Cout; ++o) {
      float acc = bias[o];
      for (int j = 0; j < k; ++j) acc += dot(wt + ((size_t)o * k + j) * Cin, x + (size_t)src[j] * Cin, Cin);
      out[(size_t)t * Cout + o] = acc;
    }
  }
  free(wt);
}

/* cpu_rmsnorm then adaptive affine: y = w*(x*inv*gamma) + b. */
static int adaptive_norm(const orc_model* m, const float* x, const float* t1, int T, const char* prefix, float* out) {
  char a[160], b[160], c[160];
  snprintf(a, sizeof(a), "%s.norm.weight", prefix);
  snprintf(b, sizeof(b), "%s.project_layer.weight", prefix);
  snprintf(c, sizeof(c), "%s.project_layer.bias", prefix);
  const float* gamma = W(m, a, 512);
  const float* pw = W(m, b, 1024 * 512);
  const float* pb = W(m, c, 1024);
  NEED(gamma && pw && pb);
  float wb[1024];
  linear_rows(pw, pb, t1, 1, 1024, 512, wb);
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    const float* r = x + (size_t)t * 512;
    float ms = 0.0f;
    for (int i = 0; i < 512; ++i) ms += r[i] * r[i];
    ms /= 512.0f;
    const float inv = 1.0f / sqrtf(ms + 1e-5f);
    for (int i = 0; i < 512; ++i) out[(size_t)t * 512 + i] = wb[i] * (r[i] * inv * gamma[i]) + wb[512 + i];
  }
  return 0;
}

/* ---------------- DiT components ---------------- */

/* run_timestep_embedder_cpu for one timestep: MLP(256 -> 512 SiLU -> 512). */
int orc_timestep_embed(const orc_model* m, float t, const char* which, float* out) {
  char a[160];
  snprintf(a, sizeof(a), "%s.freqs", which);
  const float* fr = W(m, a, 128);
  snprintf(a, sizeof(a), "%s.mlp.0.weight", which);
  const float* w0 = W(m, a, 512 * 256);
  snprintf(a, sizeof(a), "%s.mlp.0.bias", which);
  const float* b0 = W(m, a, 512);
  snprintf(a, sizeof(a), "%s.mlp.2.weight", which);
  const float* w2 = W(m, a, 512 * 512);
  snprintf(a, sizeof(a), "%s.mlp.2.bias", which);
  const float* b2 = W(m, a, 512);
  NEED(fr && w0 && b0 && w2 && b2);
  float emb[256], h[512];
  for (int i = 0; i < 128; ++i) {
    const float arg = 1000.0f * t * fr[i];
    emb[i] = cosf(arg);
    emb[128 + i] = sinf(arg);
  }
  linear_rows(w0, b0, emb, 1, 512, 256, h);
  for (int i = 0; i < 512; ++i) h[i] = silu(h[i]);
  linear_rows(w2, b2, h, 1, 512, 512, out);
  return 0;
}

/* Adjacent-pair RoPE on a [T][512] block (8 heads x 64), positions 0..T-1. */
static void rope_inplace(float* x, int T) {
  for (int t = 0; t < T; ++t) {
    for (int p = 0; p < 32; ++p) {
      const float theta = (float)t / powf(10000.0f, (float)(p * 2) / 64.0f);
      const float c = cosf(theta), s = sinf(theta);
      for (int h = 0; h < 8; ++h) {
        float* e = x + (size_t)t * 512 + h * 64 + p * 2;
        const float a = e[0], b = e[1];
        e[0] = a * c - b * s;
        e[1] = b * c + a * s;
      }
    }
  }
}

/* Masked attention core of one layer: QKV projection, RoPE, softmax(QK^T/8)V, out-proj. */
int orc_attention_layer(const orc_model* m, const float* xin, const uint32_t* mask, int T, int layer, float* out) {
  char a[160];
  snprintf(a, sizeof(a), "transformer.layers.%d.attention.wqkv.weight", layer);
  const float* wqkv = W(m, a, 1536 * 512);
  snprintf(a, sizeof(a), "transformer.layers.%d.attention.wo.weight", layer);
  const float* wo = W(m, a, 512 * 512);
  NEED(wqkv && wo);
  float* qkv = fzalloc((size_t)T * 1536);
  float* q = fzalloc((size_t)T * 512);
  float* k = fzalloc((size_t)T * 512);
  float* v = fzalloc((size_t)T * 512);
  float* cat = fzalloc((size_t)T * 512);
  linear_rows(wqkv, NULL, xin, T, 1536, 512, qkv);
  for (int t = 0; t < T; ++t) {
    memcpy(q + (size_t)t * 512, qkv + (size_t)t * 1536, 512 * sizeof(float));
    memcpy(k + (size_t)t * 512, qkv + (size_t)t * 1536 + 512, 512 * sizeof(float));
    memcpy(v + (size_t)t * 512, qkv + (size_t)t * 1536 + 1024, 512 * sizeof(float));
  }
  rope_inplace(q, T);
  rope_inplace(k, T);
  const float scale = 1.0f / sqrtf(64.0f);
#pragma omp parallel for collapse(2) schedule(static)
  for (int h = 0; h < 8; ++h) {
    for (int tq = 0; tq < T; ++tq) {
      float* sc = fzalloc((size_t)T);
      float mx = -INFINITY;
      for (int tk = 0; tk < T; ++tk) {
        if (mask[tk] == 0) {
          sc[tk] = -INFINITY;
          continue;
        }
        sc[tk] = dot(q + (size_t)tq * 512 + h * 64, k + (size_t)tk * 512 + h * 64, 64) * scale;
        if (sc[tk] > mx) mx = sc[tk];
      }
      float den = 0.0f;
      for (int tk = 0; tk < T; ++tk) {
        if (!isfinite(sc[tk])) {
          sc[tk] = 0.0f;
          continue;
        }
        sc[tk] = expf(sc[tk] - mx);
        den += sc[tk];
      }
      /* acc[d] = sum over tk (ascending) of (sc[tk] / den) * v[tk][d]: the
       * same operands and order per output as a d-outer loop, walked key-major
       * so that V is read contiguously. */
      float acc[64];
      for (int d = 0; d < 64; ++d) acc[d] = 0.0f;
      for (int tk = 0; tk < T; ++tk) {
        const float pk = sc[tk] / den;
        const float* vr = v + (size_t)tk * 512 + h * 64;
        for (int d = 0; d < 64; ++d) acc[d] += pk * vr[d];
      }
      for (int d = 0; d < 64; ++d) cat[(size_t)tq * 512 + h * 64 + d] = acc[d];
      free(sc);
    }
  }
  linear_rows(wo, NULL, cat, T, 512, 512, out);
  free(qkv);
  free(q);
  free(k);
  free(v);
  free(cat);
  return 0;
}

static int feed_forward(const orc_model* m, const float* xin, int T, int layer, float* out) {
  char a[160];
  snprintf(a, sizeof(a), "transformer.layers.%d.feed_forward.w1.weight", layer);
  const float* w1 = W(m, a, 1536 * 512);
  snprintf(a, sizeof(a), "transformer.layers.%d.feed_forward.w3.weight", layer);
  const float* w3 = W(m, a, 1536 * 512);
  snprintf(a, sizeof(a), "transformer.layers.%d.feed_forward.w2.weight", layer);
  const float* w2 = W(m, a, 512 * 1536);
  NEED(w1 && w2 && w3);
  float* h1 = fzalloc((size_t)T * 1536);
  float* h3 = fzalloc((size_t)T * 1536);
  linear_rows(w1, NULL, xin, T, 1536, 512, h1);
  linear_rows(w3, NULL, xin, T, 1536, 512, h3);
  for (size_t i = 0; i < (size_t)T * 1536; ++i) h1[i] = silu(h1[i]) * h3[i];
  linear_rows(w2, NULL, h1, T, 512, 1536, out);
  free(h1);
  free(h3);
  return 0;
}

/* One transformer block (with the optional UViT skip-in) into `out`. */
static int block(const orc_model* m, const float* xin, const float* skip, const float* t1, const uint32_t* mask, int T,
                 int layer, float* out) {
  const size_t n = (size_t)T * 512;
  float* x = fzalloc(n);
  if (skip) {
    char a[160], b[160];
    snprintf(a, sizeof(a), "transformer.layers.%d.skip_in_linear.weight", layer);
    snprintf(b, sizeof(b), "transformer.layers.%d.skip_in_linear.bias", layer);
    const float* ws = W(m, a, 512 * 1024);
    const float* bs = W(m, b, 512);
    NEED(ws && bs);
    float* cat = fzalloc((size_t)T * 1024);
    for (int t = 0; t < T; ++t) {
      memcpy(cat + (size_t)t * 1024, xin + (size_t)t * 512, 512 * sizeof(float));
      memcpy(cat + (size_t)t * 1024 + 512, skip + (size_t)t * 512, 512 * sizeof(float));
    }
    linear_rows(ws, bs, cat, T, 512, 1024, x);
    free(cat);
  } else {
    memcpy(x, xin, n * sizeof(float));
  }
  char pre[160];
  float* nrm = fzalloc(n);
  float* att = fzalloc(n);
  float* hh = fzalloc(n);
  snprintf(pre, sizeof(pre), "transformer.layers.%d.attention_norm", layer);
  if (adaptive_norm(m, x, t1, T, pre, nrm)) return -1;
  if (orc_attention_layer(m, nrm, mask, T, layer, att)) return -1;
  for (size_t i = 0; i < n; ++i) hh[i] = x[i] + att[i];
  snprintf(pre, sizeof(pre), "transformer.layers.%d.ffn_norm", layer);
  if (adaptive_norm(m, hh, t1, T, pre, nrm)) return -1;
  if (feed_forward(m, nrm, T, layer, att)) return -1;
  for (size_t i = 0; i < n; ++i) out[i] = hh[i] + att[i];
  free(x);
  free(nrm);
  free(att);
  free(hh);
  return 0;
}

/* WaveNet stack with a global (timestep) condition. */
int orc_wavenet(const orc_model* m, const float* input, const float* t2, const uint32_t* mask, int T, float* output) {
  float* wc = weight_norm_named(m, "wavenet.cond_layer.conv.conv", 8192, 512);
  const float* bc = W(m, "wavenet.cond_layer.conv.conv.bias", 8192);
  NEED(wc && bc);
  float* cond = fzalloc(8192);
  linear_rows(wc, bc, t2, 1, 8192, 512, cond);
  free(wc);
  const size_t n = (size_t)T * 512;
  float* x = fzalloc(n);
  memcpy(x, input, n * sizeof(float));
  memset(output, 0, n * sizeof(float));
  float* in = fzalloc((size_t)T * 1024);
  float* gate = fzalloc(n);
  float* rs = fzalloc((size_t)T * 1024);
  for (int l = 0; l < 8; ++l) {
    char p[160], b[160];
    snprintf(p, sizeof(p), "wavenet.in_layers.%d.conv.conv", l);
    snprintf(b, sizeof(b), "wavenet.in_layers.%d.conv.conv.bias", l);
    float* wi = weight_norm_named(m, p, 1024, 512 * 5);
    const float* bi = W(m, b, 1024);
    NEED(wi && bi);
    conv1d_reflect_same(x, wi, bi, T, 512, 1024, 5, in);
    free(wi);
    for (int t = 0; t < T; ++t) {
      for (int c = 0; c < 512; ++c) {
        const float a = in[(size_t)t * 1024 + c] + cond[l * 1024 + c];
        const float bb = in[(size_t)t * 1024 + 512 + c] + cond[l * 1024 + 512 + c];
        gate[(size_t)t * 512 + c] = tanhf(a) * (1.0f / (1.0f + expf(-bb)));
      }
    }
    const int rsc = l < 7 ? 1024 : 512;
    snprintf(p, sizeof(p), "wavenet.res_skip_layers.%d.conv.conv", l);
    snprintf(b, sizeof(b), "wavenet.res_skip_layers.%d.conv.conv.bias", l);
    float* wr = weight_norm_named(m, p, rsc, 512);
    const float* br = W(m, b, (size_t)rsc);
    NEED(wr && br);
    linear_rows(wr, br, gate, T, rsc, 512, rs);
    free(wr);
    if (l < 7) {
      for (int t = 0; t < T; ++t) {
        const float mk = mask[t] ? 1.0f : 0.0f;
        for (int c = 0; c < 512; ++c) {
          x[(size_t)t * 512 + c] = (x[(size_t)t * 512 + c] + rs[(size_t)t * 1024 + c]) * mk;
          output[(size_t)t * 512 + c] += rs[(size_t)t * 1024 + 512 + c];
        }
      }
    } else {
      for (size_t i = 0; i < n; ++i) output[i] += rs[i];
    }
  }
  for (int t = 0; t < T; ++t) {
    const float mk = mask[t] ? 1.0f : 0.0f;
    for (int c = 0; c < 512; ++c) output[(size_t)t * 512 + c] *= mk;
  }
  free(cond);
  free(x);
  free(in);
  free(gate);
  free(rs);
  return 0;
}

/*
 * One estimator evaluation: x [T,80], prompt_x [T,80], cond [T,512],
 * style [192], timestep t, key mask [T] -> velocity [T,80].
 */
int orc_estimator(const orc_model* m, const float* x, const float* prompt_x, const float* cond, const float* style,
                  float timestep, const uint32_t* mask, int T, float* vel) {
  float t1[512], t2[512];
  if (orc_timestep_embed(m, timestep, "t_embedder", t1)) return -1;
  if (orc_timestep_embed(m, timestep, "t_embedder2", t2)) return -1;
  const size_t n = (size_t)T * 512;
  /* input merge */
  const float* wcp = W(m, "cond_projection.weight", 512 * 512);
  const float* bcp = W(m, "cond_projection.bias", 512);
  const float* wm = W(m, "cond_x_merge_linear.weight", 512 * 864);
  const float* bm = W(m, "cond_x_merge_linear.bias", 512);
  NEED(wcp && bcp && wm && bm);
  float* cp = fzalloc(n);
  linear_rows(wcp, bcp, cond, T, 512, 512, cp);
  float* merged = fzalloc((size_t)T * 864);
  for (int t = 0; t < T; ++t) {
    float* r = merged + (size_t)t * 864;
    memcpy(r, x + (size_t)t * 80, 80 * sizeof(float));
    memcpy(r + 80, prompt_x + (size_t)t * 80, 80 * sizeof(float));
    memcpy(r + 160, cp + (size_t)t * 512, 512 * sizeof(float));
    memcpy(r + 672, style, 192 * sizeof(float));
  }
  float* xs = fzalloc(n);
  linear_rows(wm, bm, merged, T, 512, 864, xs);
  free(merged);
  free(cp);
  /* transformer stack with UViT skips: push outputs of layers 0..5, pop in 7..12 */
  float* skips[6];
  int nskip = 0;
  float* y = fzalloc(n);
  for (int l = 0; l < 13; ++l) {
    const float* sk = l > 6 ? skips[nskip - 1] : NULL;
    if (block(m, xs, sk, t1, mask, T, l, y)) return -1;
    memcpy(xs, y, n * sizeof(float));
    if (l > 6) free(skips[--nskip]);
    if (l < 6) {
      skips[nskip] = fzalloc(n);
      memcpy(skips[nskip++], xs, n * sizeof(float));
    }
  }
  if (adaptive_norm(m, xs, t1, T, "transformer.norm", y)) return -1;
  /* post-transformer projections */
  const float* wsl = W(m, "skip_linear.weight", 512 * 592);
  const float* bsl = W(m, "skip_linear.bias", 512);
  const float* wc1 = W(m, "conv1.weight", 512 * 512);
  const float* bc1 = W(m, "conv1.bias", 512);
  const float* wrp = W(m, "res_projection.weight", 512 * 512);
  const float* brp = W(m, "res_projection.bias", 512);
  NEED(wsl && bsl && wc1 && bc1 && wrp && brp);
  float* cat = fzalloc((size_t)T * 592);
  for (int t = 0; t < T; ++t) {
    memcpy(cat + (size_t)t * 592, y + (size_t)t * 512, 512 * sizeof(float));
    memcpy(cat + (size_t)t * 592 + 512, x + (size_t)t * 80, 80 * sizeof(float));
  }
  float* ls = fzalloc(n);
  float* c1 = fzalloc(n);
  float* res = fzalloc(n);
  linear_rows(wsl, bsl, cat, T, 512, 592, ls);
  linear_rows(wc1, bc1, ls, T, 512, 512, c1);
  linear_rows(wrp, brp, ls, T, 512, 512, res);
  free(cat);
  /* wavenet */
  float* wav = fzalloc(n);
  if (orc_wavenet(m, c1, t2, mask, T, wav)) return -1;
  for (size_t i = 0; i < n; ++i) wav[i] += res[i];
  /* final layer: LN(eps 1e-6) * (1 + scale) + shift, weight-normed linear */
  const float* aw = W(m, "final_layer.adaLN_modulation.1.weight", 1024 * 512);
  const float* ab = W(m, "final_layer.adaLN_modulation.1.bias", 1024);
  const float* lg = W(m, "final_layer.linear.weight_g", 512);
  const float* lv = W(m, "final_layer.linear.weight_v", 512 * 512);
  const float* lb = W(m, "final_layer.linear.bias", 512);
  const float* w2 = W(m, "conv2.weight", 80 * 512);
  const float* b2 = W(m, "conv2.bias", 80);
  NEED(aw && ab && lg && lv && lb && w2 && b2);
  float ts[512], ss[1024];
  for (int i = 0; i < 512; ++i) ts[i] = silu(t1[i]);
  linear_rows(aw, ab, ts, 1, 1024, 512, ss);
  float* lw = weight_norm(lg, lv, 512, 512);
  for (int t = 0; t < T; ++t) {
    float* r = wav + (size_t)t * 512;
    float mean = 0.0f;
    for (int i = 0; i < 512; ++i) mean += r[i];
    mean /= 512.0f;
    float var = 0.0f;
    for (int i = 0; i < 512; ++i) var += (r[i] - mean) * (r[i] - mean);
    var /= 512.0f;
    const float inv = 1.0f / sqrtf(var + 1e-6f);
    for (int i = 0; i < 512; ++i) r[i] = ((r[i] - mean) * inv * 1.0f + 0.0f) * (1.0f + ss[512 + i]) + ss[i];
  }
  linear_rows(lw, lb, wav, T, 512, 512, ls);
  linear_rows(w2, b2, ls, T, 80, 512, vel);
  free(lw);
  free(ls);
  free(c1);
  free(res);
  free(wav);
  free(xs);
  free(y);
  return 0;
}

/*
 * Euler sampler with CFG; the estimator sees `mask` (all ones in the
 * reference's run_cfm_euler_cpu; a key-padding mask for padded batches).
 * prompt_x [T,80] holds the prompt in rows < P. x is updated in place.
 * vel_trace (optional, [steps][T][80]) receives the guided velocity per step.
 */
int orc_euler(const orc_model* m, float* x, const float* prompt_x, const float* cond, const float* style,
              const uint32_t* mask, int T, int P, int steps, float cfg, float* vel_trace) {
  const size_t n80 = (size_t)T * 80;
  float* zp = fzalloc(n80);
  float* zc = fzalloc((size_t)T * 512);
  float zs[192];
  memset(zs, 0, sizeof(zs));
  float* v = fzalloc(n80);
  float* vu = fzalloc(n80);
  for (int t = 0; t < P; ++t) memset(x + (size_t)t * 80, 0, 80 * sizeof(float));
  float tt = 0.0f;
  const float dt = 1.0f / (float)steps;
  for (int s = 0; s < steps; ++s) {
    if (orc_estimator(m, x, prompt_x, cond, style, tt, mask, T, v)) return -1;
    if (cfg > 0.0f) {
      if (orc_estimator(m, x, zp, zc, zs, tt, mask, T, vu)) return -1;
      for (size_t i = 0; i < n80; ++i) v[i] = (1.0f + cfg) * v[i] - cfg * vu[i];
    }
    if (vel_trace) memcpy(vel_trace + (size_t)s * n80, v, n80 * sizeof(float));
    for (size_t i = 0; i < n80; ++i) x[i] += dt * v[i];
    tt += dt;
    for (int p = 0; p < P; ++p) memset(x + (size_t)p * 80, 0, 80 * sizeof(float));
  }
  free(zp);
  free(zc);
  free(v);
  free(vu);
  return 0;
}

/* splitmix64 + Box-Muller noise (make_deterministic_normal_noise). */
static uint64_t sm64(uint64_t* s) {
  uint64_t z = (*s += 0x9e3779b97f4a7c15ull);
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

static float sm64_u01(uint64_t* s) {
  const double scale = 1.0 / (double)(1ull << 53);
  double v = ((double)(sm64(s) >> 11) + 0.5) * scale;
  if (v <= 0.0) v = scale;
  else if (v >= 1.0) v = 1.0 - scale;
  return (float)v;
}

int orc_noise(int T, int C, uint64_t seed, float temperature, float* out) {
  if (T <= 0 || C <= 0) return -1;
  const size_t n = (size_t)T * C;
  uint64_t st = seed;
  size_t i = 0;
  const float two_pi = 6.2831853071795864769f;
  while (i < n) {
    const float u1 = sm64_u01(&st), u2 = sm64_u01(&st);
    const float r = sqrtf(-2.0f * logf(u1));
    const float a = two_pi * u2;
    out[i++] = r * cosf(a) * temperature;
    if (i < n) out[i++] = r * sinf(a) * temperature;
  }
  return 0;
}

int orc_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
