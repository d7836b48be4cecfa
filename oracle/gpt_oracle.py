"""TEST INFRASTRUCTURE — numpy restatement of the reference's cached greedy
GPT mel-code decoder (fp32), used only by tests/ as the checker; the product
never imports it. Pinned to the reference's own compiled CPU decoder
(oracle/_ref) through tests/golden/kat_gpt_decode.npz.

Reference functions restated (paths inside raoqu/index-tts2-metal):
  cpu_layernorm                      runtime/impl/tokenizer_tests.cpp:2992-3010
  cpu_gelu_new                       runtime/impl/tokenizer_tests.cpp:3931-3945
  cpu_attention_single_head_causal / cpu_attention_single_query
                                     runtime/impl/tokenizer_tests.cpp:4003-4061
  transpose_gpt_conv1d_weight        runtime/impl/gpt.cpp:208-216
  run_gpt_transformer_block_cpu_layer runtime/impl/gpt.cpp:658-711
  run_gpt_layer_qkv_cpu, KV cache, cached attention/block
                                     runtime/impl/gpt.cpp:1060-1210
  argmax_row                         runtime/impl/gpt.cpp:1297-1308
  build_gpt_greedy_current_cpu       runtime/impl/gpt.cpp:1545-1554
  run_gpt_kv_prefill_cpu             runtime/impl/gpt.cpp:1796-1806
  GptSamplingConfig, SplitMix64     runtime/impl/gpt.cpp:1592-1616
  apply_gpt_sampling_processors      runtime/impl/gpt.cpp:1618-1718
  sample_gpt_token_from_logits       runtime/impl/gpt.cpp:1720-1755
  sampled step of run_gpt_kv_greedy_metal (history = prefix history or [8192],
  then the predicted codes)          runtime/impl/gpt.cpp:2220-2233
  gpt_cached_generate_position       runtime/impl/gpt.cpp:1873-1875
  run_gpt_kv_greedy_cpu              runtime/impl/gpt.cpp:1877-1909
"""
from __future__ import annotations

import numpy as np

START, STOP, VOCAB, W, HEADS, HD, LAYERS = 8192, 8193, 8194, 1280, 20, 64, 24


def _ln(x, g, b, eps=1e-5):
    x = x.astype(np.float32)
    m = x.mean(axis=-1, keepdims=True, dtype=np.float32)
    v = ((x - m) ** 2).mean(axis=-1, keepdims=True, dtype=np.float32)
    return ((x - m) / np.sqrt(v + np.float32(eps))) * g + b


def _gelu_new(x):
    c = np.float32(0.7978845608028654)
    y = np.float32(0.5) * x * (np.float32(1.0) + np.tanh(c * (x + np.float32(0.044715) * x * x * x)))
    return np.where(x > 10.0, x, np.where(x < -10.0, np.float32(0.0), y)).astype(np.float32)


_M64 = (1 << 64) - 1


class SplitMix64:
    """The reference's seeded stream (64-bit arithmetic, 53-bit unit draws)."""

    def __init__(self, seed: int):
        self.state = int(seed) & _M64

    def next_u64(self) -> int:
        self.state = (self.state + 0x9E3779B97F4A7C15) & _M64
        z = self.state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
        return z ^ (z >> 31)

    def next_unit(self) -> float:
        return float(self.next_u64() >> 11) * (1.0 / 9007199254740992.0)


def sampling_processors(logits, history, temperature: float, top_k: int, top_p: float, penalty: float):
    """apply_gpt_sampling_processors: repetition penalty on each distinct
    history token (score * p if negative, else / p; float32), temperature
    (float32 division), top-k (scores below the k-th largest -> -inf), top-p
    (ascending (score, index) order, normalised double probabilities summed in
    that order, the low tail with cumulative <= 1 - top_p removed, the largest
    kept)."""
    s = np.array(logits, np.float32, copy=True)
    n = s.size
    pen, temp, tp = np.float32(penalty), np.float32(temperature), float(np.float32(top_p))
    if pen != np.float32(1.0):
        for tok in dict.fromkeys(int(t) for t in history):
            if tok < n:
                s[tok] = s[tok] * pen if s[tok] < 0 else s[tok] / pen
    if temp != np.float32(1.0):
        s = (s / temp).astype(np.float32)
    if 0 < top_k < n:
        pivot = np.sort(s)[::-1][top_k - 1]
        s[s < pivot] = -np.inf
    if tp < 1.0:
        order = np.lexsort((np.arange(n), s))  # ascending score, ties by index
        fin = np.isfinite(s)
        m = s[fin].max()
        probs = np.zeros(n, np.float64)
        probs[fin] = np.exp((s[fin] - m).astype(np.float64))
        total = np.cumsum(probs[fin])[-1]
        remove = ~fin.copy()
        cum = 0.0
        for idx in order:
            if not fin[idx]:
                continue
            cum += probs[idx] / total
            if cum <= 1.0 - tp:
                remove[idx] = True
        remove[order[-1]] = False
        s[remove] = -np.inf
    return s


def sample_token(processed, rng: SplitMix64) -> int:
    """sample_gpt_token_from_logits: double probabilities e^(s - max) of the
    finite scores, target = unit draw x their sum (in index order), the first
    index whose running sum exceeds it."""
    s = np.asarray(processed, np.float32)
    fin = np.isfinite(s)
    m = s[fin].max()
    probs = np.zeros(s.size, np.float64)
    probs[fin] = np.exp((s[fin] - m).astype(np.float64))
    idx = np.nonzero(probs > 0.0)[0]
    csum = np.cumsum(probs[idx])
    target = rng.next_unit() * csum[-1]
    hit = np.nonzero(target < csum)[0]
    return int(idx[hit[0]]) if hit.size else int(idx[-1])


class GptOracle:
    def __init__(self, tensors: dict[str, np.ndarray]):
        f = {k: np.asarray(v, np.float32) for k, v in tensors.items() if k.startswith("gpt.")}
        self.t = f
        self.layers = []
        for l in range(LAYERS):
            p = f"gpt.gpt.h.{l}."
            self.layers.append({
                "ln1": (f[p + "ln_1.weight"], f[p + "ln_1.bias"]),
                "attn": (f[p + "attn.c_attn.weight"], f[p + "attn.c_attn.bias"]),  # [in, out]: x @ W
                "proj": (f[p + "attn.c_proj.weight"], f[p + "attn.c_proj.bias"]),
                "ln2": (f[p + "ln_2.weight"], f[p + "ln_2.bias"]),
                "fc": (f[p + "mlp.c_fc.weight"], f[p + "mlp.c_fc.bias"]),
                "mproj": (f[p + "mlp.c_proj.weight"], f[p + "mlp.c_proj.bias"]),
            })

    @staticmethod
    def _attend(q, k, v):
        """q [H,64] against keys/values [L,H,64] -> [H*64]."""
        s = np.einsum("hd,lhd->hl", q, k) * np.float32(1.0 / np.sqrt(np.float32(HD)))
        s = np.exp(s - s.max(axis=1, keepdims=True))
        p = s / s.sum(axis=1, keepdims=True)
        return np.einsum("hl,lhd->hd", p, v).reshape(-1).astype(np.float32)

    def _block_current(self, L, x, cache_k, cache_v):
        """One token through layer L with its KV cache (appended in place)."""
        qkv = _ln(x, *L["ln1"]) @ L["attn"][0] + L["attn"][1]
        q, k, v = qkv[:W].reshape(HEADS, HD), qkv[W:2 * W].reshape(HEADS, HD), qkv[2 * W:].reshape(HEADS, HD)
        cache_k.append(k)
        cache_v.append(v)
        a = self._attend(q, np.stack(cache_k), np.stack(cache_v))
        h = x + (a @ L["proj"][0] + L["proj"][1])
        m = _gelu_new(_ln(h, *L["ln2"]) @ L["fc"][0] + L["fc"][1])
        return (h + (m @ L["mproj"][0] + L["mproj"][1])).astype(np.float32)

    def greedy(self, prefix, steps: int, hf_positions: bool = False, sampling: dict | None = None,
               history_prefix=None):
        """(predicted codes, logits of each step) as run_gpt_kv_greedy_cpu;
        the prefix is processed token by token (the causal full-sequence
        prefill of the reference computes the same values). hf_positions:
        its hf_generate_positions (step s > 0 uses position s + 1, as the
        synthesis pipeline calls it). sampling (dict: seed, temperature, top_k,
        top_p, repetition_penalty) replaces argmax by the reference's sampled
        step; history_prefix: the repetition history before the codes
        (default [8192])."""
        prefix = np.asarray(prefix, np.float32)
        caches = [([], []) for _ in range(LAYERS)]
        for x in prefix:
            for L, (ck, cv) in zip(self.layers, caches):
                x = self._block_current(L, x, ck, cv)
        emb, pos = self.t["gpt.mel_embedding.weight"], self.t["gpt.mel_pos_embedding.emb.weight"]
        tok, out, logits = START, [], []
        rng = SplitMix64(sampling["seed"]) if sampling else None
        for step in range(steps):
            x = emb[tok] + pos[step + 1 if hf_positions and step > 0 else step]
            for L, (ck, cv) in zip(self.layers, caches):
                x = self._block_current(L, x, ck, cv)
            h = _ln(_ln(x, self.t["gpt.gpt.ln_f.weight"], self.t["gpt.gpt.ln_f.bias"]),
                    self.t["gpt.final_norm.weight"], self.t["gpt.final_norm.bias"])
            lg = (self.t["gpt.mel_head.weight"] @ h + self.t["gpt.mel_head.bias"]).astype(np.float32)
            logits.append(lg)
            if sampling:
                hist = (list(history_prefix) if history_prefix is not None else [START]) + out
                proc = sampling_processors(lg, hist, sampling["temperature"], sampling["top_k"], sampling["top_p"],
                                           sampling["repetition_penalty"])
                tok = sample_token(proc, rng)
            else:
                tok = int(np.argmax(lg))
            out.append(tok)
            if tok == STOP:
                break
        return out, logits
