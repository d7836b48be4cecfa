/*
 * itts_cfm.h — C ABI of the B200 (sm_100a) IndexTTS2 S2Mel stage: the DiT
 * estimator inside the conditional-flow-matching Euler sampler with
 * classifier-free guidance.
 *
 * Every entry point returns an int status (ITTS_OK = 0, negative on error);
 * no C++ exception crosses this boundary. Host buffers are owned by the
 * caller; the context owns the device weights, t-conditioning tables,
 * workspaces and CUDA graphs. A context is bound to one GPU and must be used
 * from one host thread at a time.
 *
 * Layouts are row-major, token-major: a mel is [T, 80] float32, the content
 * condition [T, 512], the style vector [192].
 */
#ifndef ITTS_CFM_H
#define ITTS_CFM_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct itts_cfm_ctx itts_cfm_ctx;

enum {
  ITTS_OK = 0,
  ITTS_EINVAL_SHAPE = -1, /* a size, count or pointer argument is out of range */
  ITTS_EBUNDLE = -2,      /* the MIT2 bundle is missing, malformed or incomplete */
  ITTS_ECUDA = -3,        /* a CUDA call failed (message in itts_cfm_last_error) */
  ITTS_ETIMEOUT = -4,     /* a kernel abandoned a bounded device-side wait */
  ITTS_ECAP = -5,         /* the request exceeds a documented capacity limit */
  ITTS_ENODEV = -6        /* no usable sm_100 device with that id */
};

/* itts_cfm_create_ex flags */
#define ITTS_CREATE_VERIFY_SHA256 0x1u

/* Capacity limits. */
#define ITTS_MAX_T 65536u          /* frames per utterance */
#define ITTS_MIN_T 2u              /* reflect padding of the k=5 conv needs two rows */
#define ITTS_MAX_STEPS 1000u
#define ITTS_MAX_ROWS (1u << 22)   /* estimator rows per launch: utterances x branches x T */

/* One utterance for itts_cfm_run_batch. */
typedef struct {
  const float* noise;  /* [T, 80] initial x (prompt rows are zeroed by the sampler) */
  const float* prompt; /* [P, 80] prompt mel rows (may be NULL when P == 0) */
  const float* cond;   /* [T, 512] content condition */
  const float* style;  /* [192] style vector */
  uint32_t T;
  uint32_t P;
  float* out_mel; /* [T, 80] result; prompt rows are 0 */
} itts_cfm_utt;

/* Per-kernel timing of one profiled sampler step (itts_cfm_profile_step). */
typedef struct {
  char name[32];
  int32_t launches;
  double ms;
  double flops;
  double bytes;
} itts_kernel_stat;

/*
 * Load the estimator weights of an MIT2 bundle (manifest.json + weights.bin)
 * onto `device`. Replaces mit2::Bundle construction plus the lazy resident
 * weight upload of mit2::MetalContext (runtime/bundle.cpp:172,
 * runtime/include/mit2/metal_context.hpp:151-234).
 */
int itts_cfm_create(const char* bundle_dir, int device, itts_cfm_ctx** out);
int itts_cfm_create_ex(const char* bundle_dir, int device, uint32_t flags, itts_cfm_ctx** out);
void itts_cfm_destroy(itts_cfm_ctx* ctx);
/* Message of the last failure on this context ("" when none). */
const char* itts_cfm_last_error(const itts_cfm_ctx* ctx);
/* Message of the last itts_cfm_create failure on this thread. */
const char* itts_cfm_create_error(void);
const char* itts_cfm_strerror(int code);

/*
 * Full CFM sampler for one utterance: replaces run_cfm_euler_metal /
 * run_cfm_euler_cpu (runtime/impl/dit_cfm_bigvgan.cpp:3121-3124, 2908).
 * x starts at `noise`, prompt rows (< P) are zeroed before the loop and after
 * every step, t runs 0 -> 1 in `steps` Euler steps of dt = 1/steps, and with
 * cfg_rate > 0 the velocity is (1+cfg)·v(cond) − cfg·v(null), the null branch
 * using zero prompt, condition and style. Writes the full mel [T, 80].
 */
int itts_cfm_run(itts_cfm_ctx* ctx, const float* noise, const float* prompt, const float* cond, const float* style,
                 uint32_t T, uint32_t P, uint32_t steps, float cfg_rate, float* out_mel);

/*
 * Batched serving: utterances are grouped into length classes
 * (itts_cfm_bucket_len), sorted longest first within a class (ties by index),
 * cut into launches of at most ITTS_MAX_ROWS rows, and each launch is padded
 * to its longest utterance with zero rows and key-padding masks. A padded
 * utterance equals the single-utterance sampler run at the padded length with
 * its mask (reflect padding and masking make it differ slightly from the
 * unpadded run; an utterance as long as its launch gives itts_cfm_run's
 * result, bitwise when the attention splits its work the same way for both
 * launch sizes, else up to that split's summation order). Inputs and outputs
 * pass through a page-locked ring of the context (reserved at creation for
 * utterances of up to 1600 rows, grown for longer ones): host threads pack
 * each utterance and the copies run asynchronously. Has no single reference
 * function: it batches calls of run_cfm_euler_metal
 * (runtime/impl/tts_synthesis/synthesis_pipeline.cpp:1085).
 */
int itts_cfm_run_batch(itts_cfm_ctx* ctx, uint32_t n, const itts_cfm_utt* utts, uint32_t steps, float cfg_rate);
/* Length class of an utterance of T frames in itts_cfm_run_batch (an upper
 * bound of the length its launch is padded to). */
uint32_t itts_cfm_bucket_len(uint32_t T);

/*
 * B utterances that already share one padded length T. valid_len[b] frames
 * are real (mask 1), the rest padding (mask 0); prompt_x is [B, T, 80] with
 * the prompt mel in rows < prompt_len[b] and zeros elsewhere (the reference's
 * prompt_x, runtime/impl/dit_cfm_bigvgan.cpp:2909-2913). Output [B, T, 80].
 */
int itts_cfm_run_padded(itts_cfm_ctx* ctx, uint32_t B, uint32_t T, const uint32_t* valid_len,
                        const uint32_t* prompt_len, const float* noise, const float* prompt_x, const float* cond,
                        const float* style, uint32_t steps, float cfg_rate, float* out_mel);

/*
 * One DiT estimator evaluation at timestep t for B utterances of T rows:
 * replaces run_dit_estimator_step_cpu (runtime/impl/dit_cfm_bigvgan.cpp:1768-1788)
 * and, with branches == 2, the batched conditional + null pass
 * (run_dit_estimator_step_metal_cfg_transformer_batched_pass, :2001).
 * x, prompt_x: [B, T, 80]; cond: [B, T, 512]; style: [B, 192];
 * mask: [B, T] (0 = padded key); vel: [B, branches, T, 80] (branch 0 = conditional,
 * branch 1 = null: zero prompt_x, cond and style).
 */
int itts_cfm_estimator(itts_cfm_ctx* ctx, uint32_t B, uint32_t T, uint32_t branches, const float* x,
                       const float* prompt_x, const float* cond, const float* style, const uint32_t* mask, float t,
                       float* vel);

/*
 * Device-resident staging (benchmarks): copy a padded batch into the
 * context's workspace once, enqueue the sampler any number of times on the
 * context's stream (inputs never leave HBM), then fetch the mel.
 */
int itts_cfm_stage_padded(itts_cfm_ctx* ctx, uint32_t B, uint32_t T, const uint32_t* valid_len,
                          const uint32_t* prompt_len, const float* noise, const float* prompt_x, const float* cond,
                          const float* style, uint32_t steps, float cfg_rate);
int itts_cfm_launch(itts_cfm_ctx* ctx);
int itts_cfm_sync(itts_cfm_ctx* ctx);
int itts_cfm_fetch(itts_cfm_ctx* ctx, float* out_mel);
/* The context's cudaStream_t (as void*), for event timing by the caller. */
void* itts_cfm_stream(itts_cfm_ctx* ctx);
/* Kernel launches one itts_cfm_launch of the staged batch performs (the
 * kernel nodes of its captured CUDA graph), or a negative status. */
int itts_cfm_launch_kernels(itts_cfm_ctx* ctx);

/*
 * Time every kernel of `reps` sampler steps of the staged batch with CUDA
 * events around each launch (no graph). Fills up to `cap` entries.
 */
int itts_cfm_profile_step(itts_cfm_ctx* ctx, int reps, itts_kernel_stat* out, int cap, int* n_out);

/* Algorithmic FLOPs of one guided step over S sequences of T rows. */
double itts_cfm_step_flops(uint32_t S, uint32_t T);

/*
 * Failure-detection self-test: launches one kernel that waits on a barrier
 * nothing completes, through the bounded wait every kernel of this library
 * uses, with a budget of `budget_cycles` SM clock cycles (1e3..1e9). Returns
 * ITTS_ETIMEOUT once the kernel has given up and reported it through the
 * context's device status word, exactly as a stalled production kernel would;
 * the context stays usable afterwards. No counterpart in the reference (its
 * Metal kernels have no device-side wait).
 */
int itts_cfm_selftest_timeout(itts_cfm_ctx* ctx, uint64_t budget_cycles);

/*
 * Kernel-level entry points on caller-owned DEVICE pointers, for parity tests
 * of single kernels. They run on the context's stream and synchronise.
 *
 * itts_op_gemm: C[M,N] (f32, row stride ldc) = A[M,K] · B[N,K]^T + bias, A and B
 * f16 row-major; with a1 != NULL the first k0 columns of K come from a0 and
 * the rest from a1 (a concat without a buffer). bn is the tile width (64, 80,
 * 128, 192 or 256); bn | ITTS_GEMM_PAIR selects the CTA-pair form (256-row tiles
 * over two CTAs, bn 64/128/256). Replaces the MPS GEMM of
 * linear_rows_f32_pass (runtime/metal_context.mm:344-381).
 */
#define ITTS_GEMM_PAIR 0x10000u
int itts_op_gemm(itts_cfm_ctx* ctx, const void* a0, uint32_t lda0, const void* a1, uint32_t lda1, uint32_t k0,
                 const void* b, uint32_t ldb, const float* bias, float* c, uint32_t ldc, uint32_t M, uint32_t N,
                 uint32_t K, uint32_t bn);
/*
 * itts_op_conv5: reflect-padded k=5 "same" conv as an implicit GEMM.
 * xp: [S*(T+4), 512] f16 rows already reflect-padded (2 halo rows each side per
 * sequence); w: [N][5*512] f16 tap-major; out: [S*T, N] f32. Replaces
 * cpu_conv1d_reflect_same (runtime/impl/tokenizer_tests.cpp:3866-3872).
 */
int itts_op_conv5(itts_cfm_ctx* ctx, const void* xp, uint32_t S, uint32_t T, const void* w, const float* bias,
                  float* out, uint32_t N);
/*
 * itts_op_attention: masked MHA over packed qkv [S*T, 1536] f16 (q pre-scaled,
 * RoPE already applied) -> out [S*T, 512] f16; row_mask [S*T] f32 (0 = masked key).
 * Replaces mit2_dit_attention_sgq_batched_f32 (metal/kernels.metal:2625-2807).
 */
int itts_op_attention(itts_cfm_ctx* ctx, const void* qkv, const float* row_mask, void* out, uint32_t S, uint32_t T);
/*
 * itts_op_adarms: y = w ⊙ (x·rsqrt(mean x² + 1e-5) ⊙ gamma) + b, x [R,512] f32,
 * wb = [w | b] (1024 f32), y f16. Replaces mit2_adaptive_rmsnorm_f32_rows
 * (metal/kernels.metal:755-792).
 */
int itts_op_adarms(itts_cfm_ctx* ctx, const float* x, uint32_t R, const float* wb, const float* gamma, void* y);

/*
 * itts_op_conv5_noalloc: the k=5 reflect-padded conv of itts_op_conv5 for
 * callers that cannot allocate device memory. Examples are a serving process
 * whose own memory pool already holds the GPU's memory, and a real-time audio
 * thread that must not take cudaMalloc's implicit device-wide synchronisation.
 * It needs no context: nothing here calls cudaMalloc, cudaFree or an
 * allocating library routine. No counterpart in the reference.
 *
 * x: [S*T, 512] f16 UNPADDED rows (16-byte aligned); w, bias, out as for
 * itts_op_conv5, with N a multiple of 128 (other N: ITTS_EINVAL_SHAPE). The reflect-padded staging copy the conv reads lives in one
 * static device array of ITTS_NOALLOC_CONV5_MAX_ROWS x 512 f16 (16 MiB) per
 * GPU, held from the first call on that GPU until the process exits;
 * S*(T+4) above that limit returns ITTS_ECAP. Runs on the calling thread's
 * current device and on `stream` (a cudaStream_t of that device; NULL = the
 * legacy default stream), and synchronises that stream before returning.
 * The first call on each device looks up the array's device address; make
 * that call before any stream capture. Every call shares the array, so calls
 * that overlap on the GPU (several host threads, or streams that are not
 * ordered) race on it. On failure a message goes to err (err_cap bytes,
 * may be NULL).
 */
#define ITTS_NOALLOC_CONV5_MAX_ROWS 16384u
int itts_op_conv5_noalloc(const void* x, uint32_t S, uint32_t T, const void* w, const float* bias, float* out,
                          uint32_t N, void* stream, char* err, uint32_t err_cap);

/* ------------------------------------------------------------------------
 * BigVGAN vocoder: mel [T,80] (token-major, the CFM output rows after the
 * prompt) -> waveform [256 T] in [-1, 1]. Replaces
 * run_bigvgan_vocoder_metal(MetalContext&, const Bundle&, std::vector<float>
 * mel, uint32_t tokens) (runtime/impl/dit_cfm_bigvgan.cpp:4196-4223; CPU twin
 * run_bigvgan_vocoder_cpu, :4058-4061), which the synthesis pipeline calls on
 * the generated mel rows (runtime/impl/tts_synthesis/synthesis_pipeline.cpp:1085-1089).
 * ------------------------------------------------------------------------ */
typedef struct itts_vocoder_ctx itts_vocoder_ctx;

#define ITTS_VOCODER_MAX_T 16384u /* mel frames per call (4.2 M samples) */

/* Loads the bundle's bigvgan.* tensors (weight norm folded at load) onto
 * `device`. Replaces the lazy resident upload of the vocoder weights
 * (runtime/impl/dit_cfm_bigvgan.cpp:4064-4101). */
int itts_vocoder_create(const char* bundle_dir, int device, itts_vocoder_ctx** out);
void itts_vocoder_destroy(itts_vocoder_ctx* ctx);
const char* itts_vocoder_last_error(const itts_vocoder_ctx* ctx);
const char* itts_vocoder_create_error(void);

/* Host mel [T,80] f32 -> host wave [256 T] f32 (the caller owns both). The
 * first call for a length T builds that length's workspace and CUDA graph. */
int itts_vocoder_run(itts_vocoder_ctx* ctx, const float* mel, uint32_t T, float* wave);

/* The pieces of itts_vocoder_run for timing: stage (upload + plan), launch
 * (graph replay on the context's stream, asynchronous), fetch (download and
 * synchronise). No reference counterpart. */
int itts_vocoder_stage(itts_vocoder_ctx* ctx, const float* mel, uint32_t T);
int itts_vocoder_launch(itts_vocoder_ctx* ctx);
int itts_vocoder_fetch(itts_vocoder_ctx* ctx, float* wave);
void* itts_vocoder_stream(itts_vocoder_ctx* ctx);
/* Kernels in the staged length's graph (>= 0), or a negative status. */
int itts_vocoder_launch_kernels(itts_vocoder_ctx* ctx);
/* Event-timed launches of one vocoder pass over the staged mel, per kind. */
int itts_vocoder_profile(itts_vocoder_ctx* ctx, int reps, itts_kernel_stat* out, int cap, int* n_out);
/* Algorithmic FLOPs of one pass over T mel frames (conv MACs x 2). */
double itts_vocoder_flops(uint32_t T);

/* ------------------------------------------------------------------------
 * Condition assembly (the step right before the sampler): the S2Mel length
 * regulator on s_infer [n_in,1024] (GPT layer + VQ embedding, token-major) to
 * G frames, placed after the voice prompt's P condition rows:
 * cond [P+G,512] = [prompt_cond ; length_regulator(s_infer, G)]. Replaces
 * run_length_regulator_full_metal (runtime/impl/gpt.cpp:5319-5357; CPU twin
 * :5298-5317) followed by MetalContext::hot_condition_merge_f32
 * (runtime/metal_context.mm:2207-2257; kernel metal/kernels.metal:843-864),
 * as run at runtime/impl/tts_synthesis/synthesis_pipeline.cpp:1030-1034.
 * ------------------------------------------------------------------------ */
typedef struct itts_cond_ctx itts_cond_ctx;

/* Loads the bundle's s2mel.net.length_regulator.* tensors onto `device`. */
int itts_cond_create(const char* bundle_dir, int device, itts_cond_ctx** out);
void itts_cond_destroy(itts_cond_ctx* ctx);
const char* itts_cond_last_error(const itts_cond_ctx* ctx);
const char* itts_cond_create_error(void);

/* Host s_infer [n_in,1024] f32, prompt_cond [P,512] f32 (may be NULL when
 * P = 0) -> host cond [P+G,512] f32. The first call for a shape (n_in, P, G)
 * builds its workspace and CUDA graph. */
int itts_cond_assemble(itts_cond_ctx* ctx, const float* s_infer, uint32_t n_in, const float* prompt_cond, uint32_t P,
                       uint32_t G, float* cond);

/* The pieces of itts_cond_assemble for timing (no reference counterpart). */
int itts_cond_stage(itts_cond_ctx* ctx, const float* s_infer, uint32_t n_in, const float* prompt_cond, uint32_t P,
                    uint32_t G);
int itts_cond_launch(itts_cond_ctx* ctx);
int itts_cond_fetch(itts_cond_ctx* ctx, float* cond);
void* itts_cond_stream(itts_cond_ctx* ctx);
int itts_cond_launch_kernels(itts_cond_ctx* ctx);
/* Algorithmic FLOPs of one length-regulator pass (GEMM MACs x 2). */
double itts_cond_flops(uint32_t n_in, uint32_t G);

/* ------------------------------------------------------------------------
 * Bundle contract gates and the cached-voice loader (host only, no GPU, no
 * context). Replace the reference's --inspect-voice-bundle / --inspect-model-
 * bundle gates (inspect_voice_bundle_contract / inspect_model_bundle_contract,
 * runtime/impl/tokenizer_tests.cpp:5699, 4776; rules docs/native_bundle.md:
 * 55-112) and the voice reads of the synthesis pipeline
 * (runtime/impl/tts_synthesis/synthesis_pipeline.cpp:1060-1084). Return ITTS_OK
 * or ITTS_EBUNDLE; the gates write a JSON report ("ok": true/false, integrity
 * counters, the required tensors or the error) into `report` (cap bytes, may
 * be NULL).
 * ------------------------------------------------------------------------ */
#define ITTS_COMPONENT_CFM 0x1u              /* s2mel.net.cfm.estimator.* */
#define ITTS_COMPONENT_LENGTH_REGULATOR 0x2u /* s2mel.net.length_regulator.* */
#define ITTS_COMPONENT_BIGVGAN 0x4u          /* bigvgan.* */
#define ITTS_COMPONENT_GPT 0x8u              /* gpt.* (the mel-code decoder's tensors) */
#define ITTS_COMPONENT_ALL 0xfu

/* Voice gate: every payload's SHA-256 present and verified; f32 component=voice
 * spk_cond_emb [1,S>0,1024], s2mel_style [1,192], s2mel_prompt [1,P>0,512],
 * mel [1,80,P]. */
int itts_inspect_voice_bundle(const char* bundle_dir, char* report, uint32_t cap);
/* Model gate: every payload's SHA-256 present and verified; the sentinel
 * tensors (name, shape, component) of each stage in `components`. */
int itts_inspect_model_bundle(const char* bundle_dir, uint32_t components, char* report, uint32_t cap);
/* Reads a voice bundle (after the voice gate's shape rules): *P_out = the
 * prompt rows used (prompt_tokens, or all of the voice's when 0); then, for
 * each non-NULL buffer, prompt_cond [P,512] (s2mel_prompt rows), style [192]
 * and prompt_mel [P,80] (mel transposed from [1,80,T_voice]). */
int itts_voice_load(const char* bundle_dir, uint32_t prompt_tokens, uint32_t* P_out, float* prompt_cond, float* style,
                    float* prompt_mel, char* err, uint32_t err_cap);

/* ------------------------------------------------------------------------
 * The S2Mel-to-waveform chain of the reference's hot synthesis path
 * (synthesize_hot_condition_vectors_wav_shared,
 * runtime/impl/tts_synthesis/synthesis_pipeline.cpp:1030-1034, 1060-1089),
 * from the semantic features on: voice profile -> condition assembly -> CFM
 * sampler -> vocoder on the generated rows. Holds one context of each stage
 * on one GPU.
 * ------------------------------------------------------------------------ */
typedef struct itts_pipeline itts_pipeline;

/* The three bundle directories may be the same (a full model bundle). */
int itts_pipeline_create(const char* cfm_bundle_dir, const char* regulator_bundle_dir, const char* vocoder_bundle_dir,
                         int device, itts_pipeline** out);
void itts_pipeline_destroy(itts_pipeline* p);
const char* itts_pipeline_last_error(const itts_pipeline* p);
const char* itts_pipeline_create_error(void);

/* voice_bundle_dir: a cached voice (itts_inspect_voice_bundle contract);
 * prompt_tokens: prompt rows P taken from it (0 = all). s_infer [n_in,1024]
 * (GPT layer + VQ embedding), G generated frames, noise [(P+G),80], steps,
 * cfg_rate -> wave [256 G] (and, if full_mel is non-NULL, the sampler's
 * mel [(P+G),80]). */
int itts_pipeline_synthesize(itts_pipeline* p, const char* voice_bundle_dir, uint32_t prompt_tokens,
                             const float* s_infer, uint32_t n_in, uint32_t G, const float* noise, uint32_t steps,
                             float cfg_rate, float* wave, float* full_mel);

/* As itts_pipeline_synthesize, with the sampler's initial noise drawn the
 * way the reference's synthesis pipeline draws it:
 * itts_make_noise(P + G, 80, seed, temperature) (synthesis_pipeline.cpp:1333,
 * make_deterministic_normal_noise(tokens, mel_dim, seed, temperature)). */
int itts_pipeline_synthesize_seeded(itts_pipeline* p, const char* voice_bundle_dir, uint32_t prompt_tokens,
                                    const float* s_infer, uint32_t n_in, uint32_t G, uint64_t seed, float temperature,
                                    uint32_t steps, float cfg_rate, float* wave, float* full_mel);

/* ------------------------------------------------------------------------
 * Seeded noise. itts_make_noise writes tokens x channels normals (row-major)
 * scaled by temperature, bit-identical to the reference's
 * make_deterministic_normal_noise(tokens, channels, seed, temperature)
 * (runtime/impl/tokenizer_tests.cpp:2102-2140): SplitMix64 uniforms in (0, 1),
 * Box-Muller pairs (cos then sin) in single precision. Host code; no context
 * or GPU needed. tokens in [1, ITTS_MAX_T], channels in
 * [1, ITTS_NOISE_MAX_CHANNELS]; out holds tokens * channels floats.
 * ------------------------------------------------------------------------ */
#define ITTS_NOISE_MAX_CHANNELS 4096u
int itts_make_noise(uint32_t tokens, uint32_t channels, uint64_t seed, float temperature, float* out);

/* ------------------------------------------------------------------------
 * GPT mel-code decoder: cached greedy decode of mel codes (24 GPT-2 blocks,
 * width 1280, 20 heads, vocabulary 8194; start code 8192, stop code 8193)
 * from a prefix of input embeddings. Replaces run_gpt_kv_greedy_cpu
 * (runtime/impl/gpt.cpp:1877-1909, its GptGreedyOutputs :1857-1863 as codes
 * plus last_logits; hf_generate_positions = false) and the Metal cached decode
 * it stands for. f16 weights, fp32 activations and KV cache.
 * ------------------------------------------------------------------------ */
typedef struct itts_gpt_ctx itts_gpt_ctx;

#define ITTS_GPT_WIDTH 1280u
#define ITTS_GPT_VOCAB 8194u
#define ITTS_GPT_START 8192u
#define ITTS_GPT_STOP 8193u
#define ITTS_GPT_MAX_STEPS 1818u /* rows of gpt.mel_pos_embedding */
#define ITTS_GPT_MAX_LEN 4096u   /* prefix rows + steps held in the KV cache */

/* Loads the bundle's gpt.* decoder tensors onto `device`. */
int itts_gpt_create(const char* bundle_dir, int device, itts_gpt_ctx** out);
void itts_gpt_destroy(itts_gpt_ctx* ctx);
const char* itts_gpt_last_error(const itts_gpt_ctx* ctx);
const char* itts_gpt_create_error(void);

/* prefix [P,1280] f32 (may be NULL when P = 0), at most `steps` decode steps
 * -> codes [steps] (the predicted codes; the stop code, when predicted, is the
 * last one), *n_codes = how many, last_logits [8194] (may be NULL) = the last
 * step's logits. Needs 1 <= steps <= ITTS_GPT_MAX_STEPS and
 * P + steps <= ITTS_GPT_MAX_LEN. */
int itts_gpt_generate(itts_gpt_ctx* ctx, const float* prefix, uint32_t P, uint32_t steps, uint32_t* codes,
                      uint32_t* n_codes, float* last_logits);
/* itts_gpt_generate with flags. ITTS_GPT_HF_POSITIONS = the reference's
 * hf_generate_positions = true (decode step s > 0 takes position embedding
 * s + 1; steps <= 1817), which is how its synthesis pipeline calls the decoder
 * (runtime/impl/tts_synthesis/synthesis_pipeline.cpp:675, 795). */
#define ITTS_GPT_HF_POSITIONS 0x1u
int itts_gpt_generate_ex(itts_gpt_ctx* ctx, const float* prefix, uint32_t P, uint32_t steps, uint32_t flags,
                         uint32_t* codes, uint32_t* n_codes, float* last_logits);

/* The reference's GptSamplingConfig with do_sample = true
 * (runtime/impl/gpt.cpp:1592-1599). */
typedef struct {
  uint64_t seed;            /* SplitMix64 seed */
  float temperature;        /* > 0 */
  uint32_t top_k;           /* 1..ITTS_GPT_SAMPLE_MAX_TOP_K */
  float top_p;              /* (0, 1] */
  float repetition_penalty; /* > 0 (1 = off) */
} itts_gpt_sampling;
#define ITTS_GPT_SAMPLE_MAX_TOP_K 2048u

/* Sampled decode: as itts_gpt_generate_ex, but each code is drawn as the
 * reference's sampled step of run_gpt_kv_greedy_metal (runtime/impl/gpt.cpp:
 * 2220-2233, apply_gpt_sampling_processors :1618-1718 and
 * sample_gpt_token_from_logits :1720-1755): repetition penalty over
 * history + the codes so far, temperature, top-k, top-p, one SplitMix64 draw
 * per step. history [n_history] is its repetition_history_prefix (the
 * synthesis pipeline passes the prefix's fake_inputs,
 * runtime/impl/tts_synthesis/synthesis_pipeline.cpp:795-802); NULL / 0 means
 * [8192]. top_k is bounded (the reference also accepts 0 = off): the finite
 * set is sorted on the device. */
int itts_gpt_generate_sampled(itts_gpt_ctx* ctx, const float* prefix, uint32_t P, uint32_t steps, uint32_t flags,
                              const itts_gpt_sampling* sampling, const uint32_t* history, uint32_t n_history,
                              uint32_t* codes, uint32_t* n_codes, float* last_logits);
/* Device time (ms) of the last generate's prefill and decode (no reference
 * counterpart); kernel launches of the last generate (1: the whole call is one
 * persistent kernel); f16 weight bytes one decode step streams. */
int itts_gpt_timing(const itts_gpt_ctx* ctx, float* prefill_ms, float* decode_ms);
int itts_gpt_launch_kernels(const itts_gpt_ctx* ctx);
double itts_gpt_weight_bytes_per_token(void);
/* Profiling aid (no reference counterpart): with tracing on, the persistent
 * decoder stamps its first decode token's stages; itts_gpt_stage_trace writes
 * the microseconds since that token started at each point (the token start,
 * then per stage: prologue done, weight slots done, compute done, grid
 * barrier passed; 5 stages
 * per layer, then the head; 485 values), then every CTA's barrier arrival
 * ([121 stages][SM count]), then (at the "weight slots done" positions of
 * the first block) how long CTA 0's first thread waited for its weight slots;
 * -1 marks points not reached. Returns how many. */
int itts_gpt_set_tracing(itts_gpt_ctx* ctx, int on);
int itts_gpt_stage_trace(itts_gpt_ctx* ctx, double* us, uint32_t cap);

#ifdef __cplusplus
}
#endif

#endif /* ITTS_CFM_H */
