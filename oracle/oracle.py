"""TEST INFRASTRUCTURE — Python access to the CPU checkers.

* ``PortOracle``: the C restatement in oracle/dit_oracle.c (always available;
  built by oracle/build_ref.py into oracle/lib/).
* ``RefOracle``: the reference's own CPU functions compiled into
  oracle/_ref/libref_cfm.so (available where that library was built).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs use
this module, always as the checker or the timed CPU baseline.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

ORACLE = Path(__file__).resolve().parent
PORT_LIB = ORACLE / "lib" / "libdit_oracle.so"
REF_LIB = ORACLE / "_ref" / "libref_cfm.so"


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _u32(a):
    return np.ascontiguousarray(a, dtype=np.uint32)


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


class PortOracle:
    """fp32 CPU restatement of the reference's estimator and Euler sampler."""

    def __init__(self, tensors: dict[str, np.ndarray], lib_path: Path = PORT_LIB):
        self.lib = C.CDLL(str(lib_path))
        L = self.lib
        L.orc_model_new.restype = C.c_void_p
        L.orc_model_free.argtypes = [C.c_void_p]
        L.orc_model_set.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]
        L.orc_estimator.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_void_p,
                                    C.c_int, C.c_void_p]
        L.orc_euler.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                C.c_int, C.c_int, C.c_float, C.c_void_p]
        L.orc_attention_layer.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.orc_wavenet.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        L.orc_timestep_embed.argtypes = [C.c_void_p, C.c_float, C.c_char_p, C.c_void_p]
        L.orc_noise.argtypes = [C.c_int, C.c_int, C.c_uint64, C.c_float, C.c_void_p]
        L.orc_threads.restype = C.c_int
        L.orc_set_threads.argtypes = [C.c_int]
        self._keep = {k: _f32(v) for k, v in tensors.items()}
        self.m = C.c_void_p(L.orc_model_new())
        for k, v in self._keep.items():
            L.orc_model_set(self.m, k.encode(), _p(v), v.size)

    def __del__(self):
        try:
            self.lib.orc_model_free(self.m)
        except Exception:
            pass

    def threads(self) -> int:
        return int(self.lib.orc_threads())

    def set_threads(self, n: int) -> None:
        self.lib.orc_set_threads(int(n))

    def estimator(self, x, prompt_x, cond, style, t, mask=None):
        x, prompt_x, cond, style = _f32(x), _f32(prompt_x), _f32(cond), _f32(style)
        T = x.shape[0]
        mask = _u32(np.ones(T) if mask is None else mask)
        v = np.empty((T, 80), np.float32)
        rc = self.lib.orc_estimator(self.m, _p(x), _p(prompt_x), _p(cond), _p(style), float(t), _p(mask), T, _p(v))
        if rc:
            raise RuntimeError(f"oracle estimator failed (line {self.lib.orc_last_error()})")
        return v

    def euler(self, noise, prompt_x, cond, style, P, steps, cfg, mask=None, trace=False):
        x = _f32(noise).copy()
        prompt_x, cond, style = _f32(prompt_x), _f32(cond), _f32(style)
        T = x.shape[0]
        mask = _u32(np.ones(T) if mask is None else mask)
        tr = np.empty((steps, T, 80), np.float32) if trace else None
        rc = self.lib.orc_euler(self.m, _p(x), _p(prompt_x), _p(cond), _p(style), _p(mask), T, int(P), int(steps),
                                float(cfg), None if tr is None else _p(tr))
        if rc:
            raise RuntimeError(f"oracle euler failed (line {self.lib.orc_last_error()})")
        return (x, tr) if trace else x

    def attention_layer(self, x, mask, layer):
        x = _f32(x)
        T = x.shape[0]
        out = np.empty((T, 512), np.float32)
        rc = self.lib.orc_attention_layer(self.m, _p(x), _p(_u32(mask)), T, layer, _p(out))
        if rc:
            raise RuntimeError("oracle attention failed")
        return out

    def wavenet(self, x, g, mask):
        x, g = _f32(x), _f32(g)
        T = x.shape[0]
        out = np.empty((T, 512), np.float32)
        rc = self.lib.orc_wavenet(self.m, _p(x), _p(g), _p(_u32(mask)), T, _p(out))
        if rc:
            raise RuntimeError("oracle wavenet failed")
        return out

    def timestep_embed(self, t, which=0):
        out = np.empty(512, np.float32)
        rc = self.lib.orc_timestep_embed(self.m, float(t), b"t_embedder" if which == 0 else b"t_embedder2", _p(out))
        if rc:
            raise RuntimeError("oracle timestep embed failed")
        return out

    def noise(self, T, C_, seed, temperature=1.0):
        out = np.empty((T, C_), np.float32)
        if self.lib.orc_noise(T, C_, seed, temperature, _p(out)):
            raise RuntimeError("noise shape must be non-empty")
        return out


class VocoderOracle:
    """fp32 CPU restatement of the reference's BigVGAN vocoder
    (oracle/bigvgan_oracle.c), over the bundle's bigvgan.* tensors."""

    def __init__(self, tensors: dict[str, np.ndarray], lib_path: Path = PORT_LIB):
        self.lib = C.CDLL(str(lib_path))
        L = self.lib
        L.voc_model_new.restype = C.c_void_p
        L.voc_model_free.argtypes = [C.c_void_p]
        L.voc_model_set.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]
        L.voc_vocoder.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        L.voc_activation.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        self._keep = {k: _f32(v) for k, v in tensors.items() if k.startswith("bigvgan.")}
        self.m = C.c_void_p(L.voc_model_new())
        for k, v in self._keep.items():
            L.voc_model_set(self.m, k.encode(), _p(v), v.size)

    def __del__(self):
        try:
            self.lib.voc_model_free(self.m)
        except Exception:
            pass

    def vocoder(self, mel):
        mel = _f32(mel)
        T = mel.shape[0]
        out = np.empty(T * 256, np.float32)
        if self.lib.voc_vocoder(self.m, _p(mel), T, _p(out)):
            raise RuntimeError(f"oracle vocoder failed (line {self.lib.voc_last_error()})")
        return out

    def activation(self, prefix: str, x):
        x = _f32(x)
        T, Cc = x.shape
        out = np.empty_like(x)
        if self.lib.voc_activation(self.m, prefix.encode(), _p(x), T, Cc, _p(out)):
            raise RuntimeError(f"oracle activation failed (line {self.lib.voc_last_error()})")
        return out


class ConditionOracle:
    """fp32 CPU restatement of the reference's length regulator and condition
    merge (oracle/condition_oracle.c), over s2mel.net.length_regulator.* tensors."""

    def __init__(self, tensors: dict[str, np.ndarray], lib_path: Path = PORT_LIB):
        self.lib = C.CDLL(str(lib_path))
        L = self.lib
        L.voc_model_new.restype = C.c_void_p
        L.voc_model_free.argtypes = [C.c_void_p]
        L.voc_model_set.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]
        L.cond_length_regulator.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.cond_assemble.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        self._keep = {k: _f32(v) for k, v in tensors.items() if k.startswith("s2mel.net.length_regulator.")}
        self.m = C.c_void_p(L.voc_model_new())
        for k, v in self._keep.items():
            L.voc_model_set(self.m, k.encode(), _p(v), v.size)

    def __del__(self):
        try:
            self.lib.voc_model_free(self.m)
        except Exception:
            pass

    def length_regulator(self, x, n_out: int):
        x = _f32(x)
        out = np.empty((n_out, 512), np.float32)
        if self.lib.cond_length_regulator(self.m, _p(x), x.shape[0], int(n_out), _p(out)):
            raise RuntimeError(f"oracle length regulator failed (line {self.lib.cond_last_error()})")
        return out

    def assemble(self, x, prompt, G: int):
        x, prompt = _f32(x), _f32(prompt)
        P = prompt.shape[0]
        out = np.empty((P + G, 512), np.float32)
        if self.lib.cond_assemble(self.m, _p(x), x.shape[0], _p(prompt), P, int(G), _p(out)):
            raise RuntimeError(f"oracle condition assembly failed (line {self.lib.cond_last_error()})")
        return out


def ref_available() -> bool:
    return REF_LIB.exists()


class RefOracle:
    """The reference's own compiled CPU functions (single-threaded, scalar)."""

    def __init__(self, bundle_dir: str | Path, lib_path: Path = REF_LIB):
        self.lib = C.CDLL(str(lib_path))
        self.dir = str(bundle_dir).encode()
        L = self.lib
        L.ref_last_error.restype = C.c_char_p
        L.ref_estimator_step.argtypes = [C.c_char_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_float,
                                         C.c_void_p, C.c_uint32, C.c_void_p]
        L.ref_cfm_euler.argtypes = [C.c_char_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32,
                                    C.c_uint32, C.c_float, C.c_void_p]
        L.ref_cfm_euler_masked.argtypes = [C.c_char_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                           C.c_uint32, C.c_uint32, C.c_uint32, C.c_float, C.c_void_p]
        L.ref_attention_layer.argtypes = [C.c_char_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p]
        L.ref_wavenet.argtypes = [C.c_char_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p]
        L.ref_timestep_embed.argtypes = [C.c_char_p, C.c_float, C.c_int, C.c_void_p]
        L.ref_noise.argtypes = [C.c_uint32, C.c_uint32, C.c_uint64, C.c_float, C.c_void_p]
        L.ref_bigvgan_vocoder.argtypes = [C.c_char_p, C.c_void_p, C.c_uint32, C.c_void_p]
        L.ref_length_regulator.argtypes = [C.c_char_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p]
        L.ref_gpt_kv_greedy.argtypes = [C.c_char_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_int, C.c_void_p,
                                        C.POINTER(C.c_uint32), C.c_void_p, C.POINTER(C.c_int)]
        L.ref_gpt_sample.argtypes = [C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32, C.c_uint64, C.c_float,
                                     C.c_uint32, C.c_float, C.c_float, C.c_uint32, C.c_void_p, C.c_void_p]
        L.ref_bigvgan_activation.argtypes = [C.c_char_p, C.c_char_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p]

    def _ok(self, rc):
        if rc:
            raise RuntimeError("reference: " + self.lib.ref_last_error().decode())

    def estimator(self, x, prompt_x, cond, style, t, mask=None):
        x, prompt_x, cond, style = _f32(x), _f32(prompt_x), _f32(cond), _f32(style)
        T = x.shape[0]
        mask = _u32(np.ones(T) if mask is None else mask)
        v = np.empty((T, 80), np.float32)
        self._ok(self.lib.ref_estimator_step(self.dir, _p(x), _p(prompt_x), _p(cond), _p(style), float(t), _p(mask), T,
                                             _p(v)))
        return v

    def euler(self, noise, prompt, cond, style, P, steps, cfg):
        noise, cond, style = _f32(noise), _f32(cond), _f32(style)
        T = noise.shape[0]
        prompt = _f32(prompt if P else np.zeros((1, 80)))
        out = np.empty((T, 80), np.float32)
        self._ok(self.lib.ref_cfm_euler(self.dir, _p(noise), _p(prompt), _p(cond), _p(style), T, int(P), int(steps),
                                        float(cfg), _p(out)))
        return out

    def euler_masked(self, noise, prompt_x, cond, style, mask, P, steps, cfg):
        noise, prompt_x, cond, style = _f32(noise), _f32(prompt_x), _f32(cond), _f32(style)
        T = noise.shape[0]
        out = np.empty((T, 80), np.float32)
        self._ok(self.lib.ref_cfm_euler_masked(self.dir, _p(noise), _p(prompt_x), _p(cond), _p(style), _p(_u32(mask)),
                                               T, int(P), int(steps), float(cfg), _p(out)))
        return out

    def attention_layer(self, x, mask, layer):
        x = _f32(x)
        T = x.shape[0]
        out = np.empty((T, 512), np.float32)
        self._ok(self.lib.ref_attention_layer(self.dir, _p(x), _p(_u32(mask)), T, layer, _p(out)))
        return out

    def wavenet(self, x, g, mask):
        x, g = _f32(x), _f32(g)
        T = x.shape[0]
        out = np.empty((T, 512), np.float32)
        self._ok(self.lib.ref_wavenet(self.dir, _p(x), _p(g), _p(_u32(mask)), T, _p(out)))
        return out

    def timestep_embed(self, t, which=0):
        out = np.empty(512, np.float32)
        self._ok(self.lib.ref_timestep_embed(self.dir, float(t), which, _p(out)))
        return out

    def noise(self, T, C_, seed, temperature=1.0):
        out = np.empty((T, C_), np.float32)
        self._ok(self.lib.ref_noise(T, C_, seed, temperature, _p(out)))
        return out

    def gpt_greedy(self, prefix, steps: int, hf_positions: bool = False):
        """run_gpt_kv_greedy_cpu: (codes, logits of the last step, first stop step);
        hf_positions = its hf_generate_positions argument."""
        prefix = _f32(prefix)
        toks = np.zeros(steps, np.uint32)
        n = C.c_uint32(0)
        stop = C.c_int(-1)
        logits = np.zeros(8194, np.float32)
        self._ok(self.lib.ref_gpt_kv_greedy(self.dir, _p(prefix), prefix.shape[0], int(steps), int(bool(hf_positions)),
                                            _p(toks), C.byref(n),
                                            _p(logits), C.byref(stop)))
        return toks[: n.value].tolist(), logits, stop.value

    def gpt_sample(self, logits, history, seed: int, temperature: float, top_k: int, top_p: float,
                   repetition_penalty: float, draws: int):
        """apply_gpt_sampling_processors + `draws` x sample_gpt_token_from_logits
        (one SplitMix64 stream): (processed logits, tokens)."""
        logits = _f32(logits)
        history = np.ascontiguousarray(history, np.uint32)
        proc = np.empty_like(logits)
        toks = np.zeros(max(draws, 1), np.uint32)
        self._ok(self.lib.ref_gpt_sample(_p(logits), logits.size, _p(history), history.size, int(seed),
                                         float(temperature), int(top_k), float(top_p), float(repetition_penalty),
                                         int(draws), _p(proc), _p(toks)))
        return proc, toks[:draws].tolist()

    def length_regulator(self, x, n_out: int):
        x = _f32(x)
        out = np.empty((n_out, 512), np.float32)
        self._ok(self.lib.ref_length_regulator(self.dir, _p(x), x.shape[0], int(n_out), _p(out)))
        return out

    def vocoder(self, mel):
        mel = _f32(mel)
        T = mel.shape[0]
        out = np.empty(T * 256, np.float32)
        self._ok(self.lib.ref_bigvgan_vocoder(self.dir, _p(mel), T, _p(out)))
        return out

    def activation(self, prefix: str, x):
        x = _f32(x)
        T, Cc = x.shape
        out = np.empty_like(x)
        self._ok(self.lib.ref_bigvgan_activation(self.dir, prefix.encode(), _p(x), T, Cc, _p(out)))
        return out


def compare(ref, got) -> dict:
    """max-abs, rel-L2 and cosine of got vs ref (compare_arrays semantics,
    metal_indextts2/metrics.py:38-54)."""
    r = np.asarray(ref, np.float64).ravel()
    g = np.asarray(got, np.float64).ravel()
    d = g - r
    rn, gn = np.linalg.norm(r), np.linalg.norm(g)
    return {
        "max_abs": float(np.abs(d).max()) if d.size else 0.0,
        "rel_l2": float(np.linalg.norm(d) / max(rn, 1e-30)),
        "cosine": float(r @ g / max(rn * gn, 1e-30)),
    }
