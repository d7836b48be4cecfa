"""ctypes binding of libitts_cfm.so (include/itts_cfm.h) for Python callers.

The library is the product; this module only marshals numpy arrays and raises
``IttsError`` for non-zero status codes. It never falls back to another
implementation: if the library cannot be loaded, ``load()`` raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "lib" / "libitts_cfm.so"

ITTS_OK = 0
ITTS_EINVAL_SHAPE = -1
ITTS_EBUNDLE = -2
ITTS_ECUDA = -3
ITTS_ETIMEOUT = -4
ITTS_ECAP = -5
ITTS_ENODEV = -6
ITTS_CREATE_VERIFY_SHA256 = 0x1
ITTS_GEMM_PAIR = 0x10000

EXPORTED = [
    "itts_cfm_create", "itts_cfm_create_ex", "itts_cfm_destroy", "itts_cfm_last_error", "itts_cfm_create_error",
    "itts_cfm_strerror", "itts_cfm_run", "itts_cfm_run_batch", "itts_cfm_bucket_len", "itts_cfm_run_padded",
    "itts_cfm_estimator", "itts_cfm_stage_padded", "itts_cfm_launch", "itts_cfm_sync", "itts_cfm_fetch",
    "itts_cfm_stream", "itts_cfm_launch_kernels", "itts_cfm_profile_step", "itts_cfm_step_flops", "itts_op_gemm", "itts_op_conv5",
    "itts_op_attention", "itts_op_adarms", "itts_op_conv5_noalloc", "itts_cfm_selftest_timeout",
    "itts_vocoder_create", "itts_vocoder_destroy", "itts_vocoder_last_error", "itts_vocoder_create_error",
    "itts_vocoder_run", "itts_vocoder_stage", "itts_vocoder_launch", "itts_vocoder_fetch", "itts_vocoder_stream",
    "itts_vocoder_launch_kernels", "itts_vocoder_profile", "itts_vocoder_flops",
    "itts_cond_create", "itts_cond_destroy", "itts_cond_last_error", "itts_cond_create_error", "itts_cond_assemble",
    "itts_cond_stage", "itts_cond_launch", "itts_cond_fetch", "itts_cond_stream", "itts_cond_launch_kernels",
    "itts_cond_flops", "itts_inspect_voice_bundle", "itts_inspect_model_bundle", "itts_voice_load",
    "itts_pipeline_create", "itts_pipeline_destroy", "itts_pipeline_last_error", "itts_pipeline_create_error",
    "itts_pipeline_synthesize", "itts_pipeline_synthesize_seeded", "itts_make_noise",
    "itts_gpt_create", "itts_gpt_destroy", "itts_gpt_last_error", "itts_gpt_create_error", "itts_gpt_generate",
    "itts_gpt_generate_ex", "itts_gpt_set_tracing", "itts_gpt_stage_trace", "itts_gpt_generate_sampled",
    "itts_gpt_timing", "itts_gpt_launch_kernels", "itts_gpt_weight_bytes_per_token",
]
GPT_WIDTH = 1280
GPT_VOCAB = 8194
GPT_START = 8192
GPT_STOP = 8193
GPT_MAX_STEPS = 1818
GPT_MAX_LEN = 4096
GPT_HF_POSITIONS = 0x1
ITTS_COMPONENT_CFM = 0x1
ITTS_COMPONENT_LENGTH_REGULATOR = 0x2
ITTS_COMPONENT_BIGVGAN = 0x4
ITTS_COMPONENT_GPT = 0x8
ITTS_COMPONENT_ALL = 0xF
VOCODER_HOP = 256
VOCODER_MAX_T = 16384
NOISE_MAX_CHANNELS = 4096


class GptSampling(C.Structure):
    """itts_gpt_sampling: the reference's GptSamplingConfig with do_sample."""
    _fields_ = [("seed", C.c_uint64), ("temperature", C.c_float), ("top_k", C.c_uint32), ("top_p", C.c_float),
                ("repetition_penalty", C.c_float)]


class IttsError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"itts error {code}: {msg}")
        self.code = code


class Utt(C.Structure):
    _fields_ = [
        ("noise", C.c_void_p), ("prompt", C.c_void_p), ("cond", C.c_void_p), ("style", C.c_void_p),
        ("T", C.c_uint32), ("P", C.c_uint32), ("out_mel", C.c_void_p),
    ]


class KernelStat(C.Structure):
    _fields_ = [("name", C.c_char * 32), ("launches", C.c_int32), ("ms", C.c_double), ("flops", C.c_double),
                ("bytes", C.c_double)]


_lib = None


def load(path: str | Path | None = None) -> C.CDLL:
    """Load the C-ABI library (raises OSError if it is missing)."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    lib = C.CDLL(str(p))
    vp, u32, i32, f32, f64 = C.c_void_p, C.c_uint32, C.c_int, C.c_float, C.c_double
    sig = {
        "itts_cfm_create": (i32, [C.c_char_p, i32, C.POINTER(vp)]),
        "itts_cfm_create_ex": (i32, [C.c_char_p, i32, u32, C.POINTER(vp)]),
        "itts_cfm_destroy": (None, [vp]),
        "itts_cfm_last_error": (C.c_char_p, [vp]),
        "itts_cfm_create_error": (C.c_char_p, []),
        "itts_cfm_strerror": (C.c_char_p, [i32]),
        "itts_cfm_run": (i32, [vp, vp, vp, vp, vp, u32, u32, u32, f32, vp]),
        "itts_cfm_run_batch": (i32, [vp, u32, vp, u32, f32]),
        "itts_cfm_bucket_len": (u32, [u32]),
        "itts_cfm_run_padded": (i32, [vp, u32, u32, vp, vp, vp, vp, vp, vp, u32, f32, vp]),
        "itts_cfm_estimator": (i32, [vp, u32, u32, u32, vp, vp, vp, vp, vp, f32, vp]),
        "itts_cfm_stage_padded": (i32, [vp, u32, u32, vp, vp, vp, vp, vp, vp, u32, f32]),
        "itts_cfm_launch": (i32, [vp]),
        "itts_cfm_sync": (i32, [vp]),
        "itts_cfm_fetch": (i32, [vp, vp]),
        "itts_cfm_stream": (vp, [vp]),
        "itts_cfm_launch_kernels": (i32, [vp]),
        "itts_cfm_profile_step": (i32, [vp, i32, vp, i32, C.POINTER(i32)]),
        "itts_cfm_step_flops": (f64, [u32, u32]),
        "itts_op_gemm": (i32, [vp, vp, u32, vp, u32, u32, vp, u32, vp, vp, u32, u32, u32, u32, u32]),
        "itts_op_conv5": (i32, [vp, vp, u32, u32, vp, vp, vp, u32]),
        "itts_op_attention": (i32, [vp, vp, vp, vp, u32, u32]),
        "itts_op_adarms": (i32, [vp, vp, u32, vp, vp, vp]),
        "itts_op_conv5_noalloc": (i32, [vp, u32, u32, vp, vp, vp, u32, vp, C.c_char_p, u32]),
        "itts_cfm_selftest_timeout": (i32, [vp, C.c_uint64]),
        "itts_vocoder_create": (i32, [C.c_char_p, i32, C.POINTER(vp)]),
        "itts_vocoder_destroy": (None, [vp]),
        "itts_vocoder_last_error": (C.c_char_p, [vp]),
        "itts_vocoder_create_error": (C.c_char_p, []),
        "itts_vocoder_run": (i32, [vp, vp, u32, vp]),
        "itts_vocoder_stage": (i32, [vp, vp, u32]),
        "itts_vocoder_launch": (i32, [vp]),
        "itts_vocoder_fetch": (i32, [vp, vp]),
        "itts_vocoder_stream": (vp, [vp]),
        "itts_vocoder_launch_kernels": (i32, [vp]),
        "itts_vocoder_profile": (i32, [vp, i32, vp, i32, C.POINTER(i32)]),
        "itts_vocoder_flops": (f64, [u32]),
        "itts_cond_create": (i32, [C.c_char_p, i32, C.POINTER(vp)]),
        "itts_cond_destroy": (None, [vp]),
        "itts_cond_last_error": (C.c_char_p, [vp]),
        "itts_cond_create_error": (C.c_char_p, []),
        "itts_cond_assemble": (i32, [vp, vp, u32, vp, u32, u32, vp]),
        "itts_cond_stage": (i32, [vp, vp, u32, vp, u32, u32]),
        "itts_cond_launch": (i32, [vp]),
        "itts_cond_fetch": (i32, [vp, vp]),
        "itts_cond_stream": (vp, [vp]),
        "itts_cond_launch_kernels": (i32, [vp]),
        "itts_cond_flops": (f64, [u32, u32]),
        "itts_inspect_voice_bundle": (i32, [C.c_char_p, C.c_char_p, u32]),
        "itts_inspect_model_bundle": (i32, [C.c_char_p, u32, C.c_char_p, u32]),
        "itts_voice_load": (i32, [C.c_char_p, u32, C.POINTER(u32), vp, vp, vp, C.c_char_p, u32]),
        "itts_pipeline_create": (i32, [C.c_char_p, C.c_char_p, C.c_char_p, i32, C.POINTER(vp)]),
        "itts_pipeline_destroy": (None, [vp]),
        "itts_pipeline_last_error": (C.c_char_p, [vp]),
        "itts_pipeline_create_error": (C.c_char_p, []),
        "itts_pipeline_synthesize": (i32, [vp, C.c_char_p, u32, vp, u32, u32, vp, u32, f32, vp, vp]),
        "itts_pipeline_synthesize_seeded": (i32, [vp, C.c_char_p, u32, vp, u32, u32, C.c_uint64, f32, u32, f32, vp,
                                                  vp]),
        "itts_make_noise": (i32, [u32, u32, C.c_uint64, f32, vp]),
        "itts_gpt_create": (i32, [C.c_char_p, i32, C.POINTER(vp)]),
        "itts_gpt_destroy": (None, [vp]),
        "itts_gpt_last_error": (C.c_char_p, [vp]),
        "itts_gpt_create_error": (C.c_char_p, []),
        "itts_gpt_generate": (i32, [vp, vp, u32, u32, vp, C.POINTER(u32), vp]),
        "itts_gpt_generate_ex": (i32, [vp, vp, u32, u32, u32, vp, C.POINTER(u32), vp]),
        "itts_gpt_set_tracing": (i32, [vp, i32]),
        "itts_gpt_generate_sampled": (i32, [vp, vp, u32, u32, u32, C.POINTER(GptSampling), vp, u32, vp,
                                            C.POINTER(u32), vp]),
        "itts_gpt_stage_trace": (i32, [vp, vp, u32]),
        "itts_gpt_timing": (i32, [vp, C.POINTER(f32), C.POINTER(f32)]),
        "itts_gpt_launch_kernels": (i32, [vp]),
        "itts_gpt_weight_bytes_per_token": (f64, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class Context:
    """One engine context bound to one GPU (itts_cfm_create)."""

    def __init__(self, bundle_dir: str | Path, device: int = 0, verify_sha256: bool = False):
        self.lib = load()
        h = C.c_void_p()
        flags = ITTS_CREATE_VERIFY_SHA256 if verify_sha256 else 0
        rc = self.lib.itts_cfm_create_ex(str(bundle_dir).encode(), int(device), flags, C.byref(h))
        if rc != ITTS_OK:
            raise IttsError(rc, self.lib.itts_cfm_create_error().decode())
        self.h = h

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.itts_cfm_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int) -> None:
        if rc != ITTS_OK:
            raise IttsError(rc, self.lib.itts_cfm_last_error(self.h).decode())

    # ---- sampler ----
    def run(self, noise, prompt, cond, style, steps: int, cfg_rate: float) -> np.ndarray:
        noise, cond, style = _f32(noise), _f32(cond), _f32(style)
        T = noise.shape[0]
        prompt = _f32(prompt) if prompt is not None and len(prompt) else None
        P = 0 if prompt is None else prompt.shape[0]
        out = np.empty((T, 80), np.float32)
        self._check(self.lib.itts_cfm_run(self.h, _ptr(noise), _ptr(prompt), _ptr(cond), _ptr(style), T, P, steps,
                                          float(cfg_rate), _ptr(out)))
        return out

    def run_padded(self, valid_len, prompt_len, noise, prompt_x, cond, style, steps: int, cfg_rate: float):
        noise, prompt_x, cond, style = _f32(noise), _f32(prompt_x), _f32(cond), _f32(style)
        B, T = noise.shape[0], noise.shape[1]
        vl = np.ascontiguousarray(valid_len, dtype=np.uint32)
        pl = np.ascontiguousarray(prompt_len, dtype=np.uint32)
        out = np.empty((B, T, 80), np.float32)
        self._check(self.lib.itts_cfm_run_padded(self.h, B, T, _ptr(vl), _ptr(pl), _ptr(noise), _ptr(prompt_x),
                                                 _ptr(cond), _ptr(style), steps, float(cfg_rate), _ptr(out)))
        return out

    def run_batch(self, utts: list[dict], steps: int, cfg_rate: float) -> list[np.ndarray]:
        keep = []
        arr = (Utt * len(utts))()
        outs = []
        for i, u in enumerate(utts):
            n, c, s = _f32(u["noise"]), _f32(u["cond"]), _f32(u["style"])
            p = _f32(u["prompt"]) if u.get("prompt") is not None and len(u["prompt"]) else None
            o = np.empty((n.shape[0], 80), np.float32)
            keep += [n, c, s, p, o]
            outs.append(o)
            arr[i] = Utt(n.ctypes.data, None if p is None else p.ctypes.data, c.ctypes.data, s.ctypes.data,
                         n.shape[0], 0 if p is None else p.shape[0], o.ctypes.data)
        self._check(self.lib.itts_cfm_run_batch(self.h, len(utts), C.cast(arr, C.c_void_p), steps, float(cfg_rate)))
        return outs

    def estimator(self, x, prompt_x, cond, style, mask, t: float, branches: int = 2) -> np.ndarray:
        """x, prompt_x [B,T,80]; cond [B,T,512]; style [B,192]; mask [B,T] -> vel [B,branches,T,80]."""
        x, prompt_x, cond, style = _f32(x), _f32(prompt_x), _f32(cond), _f32(style)
        mask = np.ascontiguousarray(mask, dtype=np.uint32)
        B, T = x.shape[0], x.shape[1]
        vel = np.empty((B, branches, T, 80), np.float32)
        self._check(self.lib.itts_cfm_estimator(self.h, B, T, branches, _ptr(x), _ptr(prompt_x), _ptr(cond),
                                                _ptr(style), _ptr(mask), float(t), _ptr(vel)))
        return vel

    # ---- staged (device-resident) ----
    def stage_padded(self, valid_len, prompt_len, noise, prompt_x, cond, style, steps: int, cfg_rate: float):
        noise, prompt_x, cond, style = _f32(noise), _f32(prompt_x), _f32(cond), _f32(style)
        B, T = noise.shape[0], noise.shape[1]
        vl = np.ascontiguousarray(valid_len, dtype=np.uint32)
        pl = np.ascontiguousarray(prompt_len, dtype=np.uint32)
        self._check(self.lib.itts_cfm_stage_padded(self.h, B, T, _ptr(vl), _ptr(pl), _ptr(noise), _ptr(prompt_x),
                                                   _ptr(cond), _ptr(style), steps, float(cfg_rate)))
        self._staged_shape = (B, T)

    def launch(self) -> None:
        self._check(self.lib.itts_cfm_launch(self.h))

    def sync(self) -> None:
        self._check(self.lib.itts_cfm_sync(self.h))

    def fetch(self) -> np.ndarray:
        B, T = self._staged_shape
        out = np.empty((B, T, 80), np.float32)
        self._check(self.lib.itts_cfm_fetch(self.h, _ptr(out)))
        return out

    def stream(self) -> int:
        return int(self.lib.itts_cfm_stream(self.h) or 0)

    def launch_kernels(self) -> int:
        n = int(self.lib.itts_cfm_launch_kernels(self.h))
        if n < 0:
            raise IttsError(n, "no captured launch for the staged batch")
        return n

    def profile_step(self, reps: int = 1) -> list[dict]:
        cap = 64
        buf = (KernelStat * cap)()
        n = C.c_int(0)
        self._check(self.lib.itts_cfm_profile_step(self.h, reps, C.cast(buf, C.c_void_p), cap, C.byref(n)))
        return [dict(name=buf[i].name.decode(), launches=buf[i].launches, ms=buf[i].ms, flops=buf[i].flops,
                     bytes=buf[i].bytes) for i in range(n.value)]

    # ---- kernel-level (device pointers as ints) ----
    def op_gemm(self, a0, lda0, a1, lda1, k0, b, ldb, bias, c, ldc, M, N, K, bn=128) -> None:
        self._check(self.lib.itts_op_gemm(self.h, a0, lda0, a1, lda1, k0, b, ldb, bias, c, ldc, M, N, K, bn))

    def selftest_timeout(self, budget_cycles: int) -> tuple[int, str]:
        """Run the bounded-wait self-test; returns (status code, message)."""
        rc = self.lib.itts_cfm_selftest_timeout(self.h, int(budget_cycles))
        return rc, self.lib.itts_cfm_last_error(self.h).decode()

    def op_conv5(self, xp, S, T, w, bias, out, N) -> None:
        self._check(self.lib.itts_op_conv5(self.h, xp, S, T, w, bias, out, N))

    def op_attention(self, qkv, mask, out, S, T) -> None:
        self._check(self.lib.itts_op_attention(self.h, qkv, mask, out, S, T))

    def op_adarms(self, x, R, wb, gamma, y) -> None:
        self._check(self.lib.itts_op_adarms(self.h, x, R, wb, gamma, y))


NOALLOC_CONV5_MAX_ROWS = 16384


def conv5_noalloc(x, S: int, T: int, w, bias, out, N: int, stream=None) -> None:
    """itts_op_conv5_noalloc on device pointers: the k=5 reflect conv from
    UNPADDED rows x [S*T, 512] f16, for callers that cannot allocate device
    memory. It needs no Context; the padded staging copy lives in a static
    device array of NOALLOC_CONV5_MAX_ROWS rows that every call shares."""
    lib = load()
    err = C.create_string_buffer(256)
    rc = lib.itts_op_conv5_noalloc(x, S, T, w, bias, out, N, stream, err, len(err))
    if rc != ITTS_OK:
        raise IttsError(rc, err.value.decode())


def bucket_len(T: int) -> int:
    return int(load().itts_cfm_bucket_len(T))


def step_flops(S: int, T: int) -> float:
    return float(load().itts_cfm_step_flops(S, T))


MAX_ROWS = 1 << 22


def batch_plan(lengths: list[int], cfg_rate: float) -> list[list[int]]:
    """The launches itts_cfm_run_batch makes, as lists of utterance indices
    (longest first): utterances are grouped by bucket_len (ascending), sorted
    longest first within a group (ties by index) and cut into launches of at
    most MAX_ROWS rows; each launch is padded to its first (longest) member."""
    branches = 2 if cfg_rate > 0 else 1
    groups: dict[int, list[int]] = {}
    for i, T in enumerate(lengths):
        groups.setdefault(bucket_len(T), []).append(i)
    plan = []
    for cls in sorted(groups):
        idx = sorted(groups[cls], key=lambda i: -lengths[i])
        per = max(1, MAX_ROWS // (branches * cls))
        plan += [idx[off : off + per] for off in range(0, len(idx), per)]
    return plan


def batch_padded_lengths(lengths: list[int], cfg_rate: float) -> list[int]:
    """The padded length itts_cfm_run_batch runs each utterance at (the
    longest utterance of its launch, see batch_plan)."""
    out = [0] * len(lengths)
    for launch in batch_plan(lengths, cfg_rate):
        for i in launch:
            out[i] = lengths[launch[0]]
    return out


class Vocoder:
    """BigVGAN vocoder bound to one GPU (itts_vocoder_create): mel [T, 80] ->
    waveform [256 T] in [-1, 1]."""

    def __init__(self, bundle_dir: str | Path, device: int = 0):
        self.lib = load()
        h = C.c_void_p()
        rc = self.lib.itts_vocoder_create(str(bundle_dir).encode(), int(device), C.byref(h))
        if rc != ITTS_OK:
            raise IttsError(rc, self.lib.itts_vocoder_create_error().decode())
        self.h = h
        self.T = 0

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.itts_vocoder_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int) -> None:
        if rc != ITTS_OK:
            raise IttsError(rc, self.lib.itts_vocoder_last_error(self.h).decode())

    def run(self, mel) -> np.ndarray:
        mel = _f32(mel)
        if mel.ndim != 2 or mel.shape[1] != 80:
            raise ValueError("mel must be [T, 80]")
        wave = np.empty(mel.shape[0] * VOCODER_HOP, np.float32)
        self._check(self.lib.itts_vocoder_run(self.h, _ptr(mel), mel.shape[0], _ptr(wave)))
        return wave

    def stage(self, mel) -> None:
        mel = _f32(mel)
        self._check(self.lib.itts_vocoder_stage(self.h, _ptr(mel), mel.shape[0]))
        self.T = mel.shape[0]

    def launch(self) -> None:
        self._check(self.lib.itts_vocoder_launch(self.h))

    def fetch(self) -> np.ndarray:
        wave = np.empty(self.T * VOCODER_HOP, np.float32)
        self._check(self.lib.itts_vocoder_fetch(self.h, _ptr(wave)))
        return wave

    def stream(self) -> int:
        return int(self.lib.itts_vocoder_stream(self.h) or 0)

    def launch_kernels(self) -> int:
        n = int(self.lib.itts_vocoder_launch_kernels(self.h))
        if n < 0:
            raise IttsError(n, "nothing staged")
        return n

    def profile(self, reps: int = 1) -> list[dict]:
        cap = 64
        buf = (KernelStat * cap)()
        n = C.c_int(0)
        self._check(self.lib.itts_vocoder_profile(self.h, reps, C.cast(buf, C.c_void_p), cap, C.byref(n)))
        return [dict(name=buf[i].name.decode(), launches=buf[i].launches, ms=buf[i].ms, flops=buf[i].flops,
                     bytes=buf[i].bytes) for i in range(n.value)]

    @staticmethod
    def flops(T: int) -> float:
        return float(load().itts_vocoder_flops(int(T)))


class ConditionAssembler:
    """Length regulator + condition merge bound to one GPU (itts_cond_create):
    s_infer [n_in, 1024], prompt_cond [P, 512] -> cond [P + G, 512]."""

    def __init__(self, bundle_dir: str | Path, device: int = 0):
        self.lib = load()
        h = C.c_void_p()
        rc = self.lib.itts_cond_create(str(bundle_dir).encode(), int(device), C.byref(h))
        if rc != ITTS_OK:
            raise IttsError(rc, self.lib.itts_cond_create_error().decode())
        self.h = h
        self.rows = 0

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.itts_cond_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int) -> None:
        if rc != ITTS_OK:
            raise IttsError(rc, self.lib.itts_cond_last_error(self.h).decode())

    @staticmethod
    def _args(s_infer, prompt):
        s_infer = _f32(s_infer)
        if s_infer.ndim != 2 or s_infer.shape[1] != 1024:
            raise ValueError("s_infer must be [n_in, 1024]")
        prompt = None if prompt is None or len(prompt) == 0 else _f32(prompt)
        if prompt is not None and (prompt.ndim != 2 or prompt.shape[1] != 512):
            raise ValueError("prompt_cond must be [P, 512]")
        return s_infer, prompt, 0 if prompt is None else prompt.shape[0]

    def assemble(self, s_infer, prompt, G: int) -> np.ndarray:
        s_infer, prompt, P = self._args(s_infer, prompt)
        out = np.empty((P + int(G), 512), np.float32)
        self._check(self.lib.itts_cond_assemble(self.h, _ptr(s_infer), s_infer.shape[0], _ptr(prompt), P, int(G),
                                                _ptr(out)))
        return out

    def length_regulator(self, s_infer, G: int) -> np.ndarray:
        return self.assemble(s_infer, None, G)

    def stage(self, s_infer, prompt, G: int) -> None:
        s_infer, prompt, P = self._args(s_infer, prompt)
        self._check(self.lib.itts_cond_stage(self.h, _ptr(s_infer), s_infer.shape[0], _ptr(prompt), P, int(G)))
        self.rows = P + int(G)

    def launch(self) -> None:
        self._check(self.lib.itts_cond_launch(self.h))

    def fetch(self) -> np.ndarray:
        out = np.empty((self.rows, 512), np.float32)
        self._check(self.lib.itts_cond_fetch(self.h, _ptr(out)))
        return out

    def stream(self) -> int:
        return int(self.lib.itts_cond_stream(self.h) or 0)

    def launch_kernels(self) -> int:
        n = int(self.lib.itts_cond_launch_kernels(self.h))
        if n < 0:
            raise IttsError(n, "nothing staged")
        return n

    @staticmethod
    def flops(n_in: int, G: int) -> float:
        return float(load().itts_cond_flops(int(n_in), int(G)))


def inspect_voice_bundle(bundle_dir: str | Path) -> tuple[int, dict]:
    """The voice-bundle contract gate (host only): (status, JSON report)."""
    import json

    buf = C.create_string_buffer(1 << 16)
    rc = load().itts_inspect_voice_bundle(str(bundle_dir).encode(), buf, len(buf))
    return rc, json.loads(buf.value.decode())


def inspect_model_bundle(bundle_dir: str | Path, components: int = ITTS_COMPONENT_CFM) -> tuple[int, dict]:
    """The model-bundle contract gate for `components` (host only): (status, JSON report)."""
    import json

    buf = C.create_string_buffer(1 << 16)
    rc = load().itts_inspect_model_bundle(str(bundle_dir).encode(), int(components), buf, len(buf))
    return rc, json.loads(buf.value.decode())


def voice_load(bundle_dir: str | Path, prompt_tokens: int = 0) -> dict:
    """prompt_cond [P,512], style [192] and prompt_mel [P,80] of a voice bundle."""
    lib = load()
    P = C.c_uint32(0)
    err = C.create_string_buffer(512)
    rc = lib.itts_voice_load(str(bundle_dir).encode(), int(prompt_tokens), C.byref(P), None, None, None, err, len(err))
    if rc != ITTS_OK:
        raise IttsError(rc, err.value.decode())
    pc = np.empty((P.value, 512), np.float32)
    st = np.empty(192, np.float32)
    pm = np.empty((P.value, 80), np.float32)
    rc = lib.itts_voice_load(str(bundle_dir).encode(), int(prompt_tokens), C.byref(P), _ptr(pc), _ptr(st), _ptr(pm),
                             err, len(err))
    if rc != ITTS_OK:
        raise IttsError(rc, err.value.decode())
    return {"prompt_cond": pc, "style": st, "prompt_mel": pm, "P": P.value}


class Pipeline:
    """Voice profile -> condition assembly -> CFM sampler -> vocoder on one GPU
    (itts_pipeline_create / itts_pipeline_synthesize)."""

    def __init__(self, cfm_bundle: str | Path, regulator_bundle: str | Path, vocoder_bundle: str | Path,
                 device: int = 0):
        self.lib = load()
        h = C.c_void_p()
        rc = self.lib.itts_pipeline_create(str(cfm_bundle).encode(), str(regulator_bundle).encode(),
                                           str(vocoder_bundle).encode(), int(device), C.byref(h))
        if rc != ITTS_OK:
            raise IttsError(rc, self.lib.itts_pipeline_create_error().decode())
        self.h = h

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.itts_pipeline_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def synthesize(self, voice_bundle: str | Path, s_infer, G: int, noise, steps: int, cfg: float,
                   prompt_tokens: int = 0) -> tuple[np.ndarray, np.ndarray]:
        s_infer, noise = _f32(s_infer), _f32(noise)
        wave = np.empty(int(G) * VOCODER_HOP, np.float32)
        mel = np.empty_like(noise)
        rc = self.lib.itts_pipeline_synthesize(self.h, str(voice_bundle).encode(), int(prompt_tokens), _ptr(s_infer),
                                               s_infer.shape[0], int(G), _ptr(noise), int(steps), float(cfg),
                                               _ptr(wave), _ptr(mel))
        if rc != ITTS_OK:
            raise IttsError(rc, self.lib.itts_pipeline_last_error(self.h).decode())
        return wave, mel

    def synthesize_seeded(self, voice_bundle: str | Path, s_infer, G: int, seed: int, temperature: float, steps: int,
                          cfg: float, prompt_tokens: int = 0) -> tuple[np.ndarray, np.ndarray]:
        """As synthesize, with x0 = make_noise(P + G, 80, seed, temperature)
        (the reference pipeline's draw)."""
        s_infer = _f32(s_infer)
        P = voice_load(voice_bundle, prompt_tokens)["P"]
        wave = np.empty(int(G) * VOCODER_HOP, np.float32)
        mel = np.empty((P + int(G), 80), np.float32)
        rc = self.lib.itts_pipeline_synthesize_seeded(self.h, str(voice_bundle).encode(), int(prompt_tokens),
                                                      _ptr(s_infer), s_infer.shape[0], int(G), int(seed),
                                                      float(temperature), int(steps), float(cfg), _ptr(wave),
                                                      _ptr(mel))
        if rc != ITTS_OK:
            raise IttsError(rc, self.lib.itts_pipeline_last_error(self.h).decode())
        return wave, mel


def make_noise(tokens: int, channels: int, seed: int, temperature: float = 1.0) -> np.ndarray:
    """itts_make_noise: [tokens, channels] seeded normals, bit-identical to the
    reference's make_deterministic_normal_noise (host code, no GPU)."""
    out = np.empty((int(tokens), int(channels)), np.float32)
    rc = load().itts_make_noise(int(tokens), int(channels), int(seed) & (2**64 - 1), float(temperature), _ptr(out))
    if rc != ITTS_OK:
        raise IttsError(rc, f"noise shape out of range: {tokens} x {channels}")
    return out


class GptDecoder:
    """Cached greedy mel-code decoder bound to one GPU (itts_gpt_create):
    prefix [P, 1280] -> predicted codes (the stop code last when predicted)
    and the last step's logits, as run_gpt_kv_greedy_cpu."""

    def __init__(self, bundle_dir: str | Path, device: int = 0):
        self.lib = load()
        h = C.c_void_p()
        rc = self.lib.itts_gpt_create(str(bundle_dir).encode(), int(device), C.byref(h))
        if rc != ITTS_OK:
            raise IttsError(rc, self.lib.itts_gpt_create_error().decode())
        self.h = h

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.itts_gpt_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def generate(self, prefix, steps: int, hf_positions: bool = False) -> tuple[list[int], np.ndarray]:
        """hf_positions: the reference's hf_generate_positions (as its
        synthesis pipeline calls the decoder)."""
        prefix = None if prefix is None or len(prefix) == 0 else _f32(prefix)
        if prefix is not None and (prefix.ndim != 2 or prefix.shape[1] != GPT_WIDTH):
            raise ValueError("prefix must be [P, 1280]")
        P = 0 if prefix is None else prefix.shape[0]
        codes = np.zeros(max(int(steps), 1), np.uint32)
        logits = np.empty(GPT_VOCAB, np.float32)
        n = C.c_uint32(0)
        rc = self.lib.itts_gpt_generate_ex(self.h, _ptr(prefix), P, int(steps), GPT_HF_POSITIONS if hf_positions else 0,
                                           _ptr(codes), C.byref(n), _ptr(logits))
        if rc != ITTS_OK:
            raise IttsError(rc, self.lib.itts_gpt_last_error(self.h).decode())
        return [int(c) for c in codes[:n.value]], logits

    def generate_sampled(self, prefix, steps: int, sampling: dict, history=None,
                         hf_positions: bool = False) -> tuple[list[int], np.ndarray]:
        """Sampled decode (itts_gpt_generate_sampled). sampling: seed,
        temperature, top_k, top_p, repetition_penalty; history: the
        repetition history before the codes (default [8192])."""
        prefix = None if prefix is None or len(prefix) == 0 else _f32(prefix)
        P = 0 if prefix is None else prefix.shape[0]
        cfg = GptSampling(int(sampling["seed"]), float(sampling["temperature"]), int(sampling["top_k"]),
                          float(sampling["top_p"]), float(sampling["repetition_penalty"]))
        hist = None if history is None else np.ascontiguousarray(history, np.uint32)
        codes = np.zeros(max(int(steps), 1), np.uint32)
        logits = np.empty(GPT_VOCAB, np.float32)
        n = C.c_uint32(0)
        rc = self.lib.itts_gpt_generate_sampled(self.h, _ptr(prefix), P, int(steps),
                                                GPT_HF_POSITIONS if hf_positions else 0, C.byref(cfg), _ptr(hist),
                                                0 if hist is None else hist.size, _ptr(codes), C.byref(n),
                                                _ptr(logits))
        if rc != ITTS_OK:
            raise IttsError(rc, self.lib.itts_gpt_last_error(self.h).decode())
        return [int(c) for c in codes[:n.value]], logits

    def timing(self) -> tuple[float, float]:
        """Device ms of the last generate's (prefill, decode)."""
        a, b = C.c_float(0.0), C.c_float(0.0)
        self.lib.itts_gpt_timing(self.h, C.byref(a), C.byref(b))
        return a.value, b.value

    def launch_kernels(self) -> int:
        return int(self.lib.itts_gpt_launch_kernels(self.h))

    def set_tracing(self, on: bool) -> None:
        self.lib.itts_gpt_set_tracing(self.h, int(bool(on)))

    def stage_trace(self) -> np.ndarray:
        """Microseconds since the first decode token started at each trace
        point of the persistent decoder (empty unless tracing)."""
        buf = np.zeros(2 * 485 + 121 * 160, np.float64)
        n = int(self.lib.itts_gpt_stage_trace(self.h, _ptr(buf), buf.size))
        return buf[:max(n, 0)]

    @staticmethod
    def weight_bytes_per_token() -> float:
        return float(load().itts_gpt_weight_bytes_per_token())
