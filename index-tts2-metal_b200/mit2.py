"""MIT2 weight bundles: writer, reader and the synthetic DiT estimator bundle.

Format (the reference's native bundle, docs/native_bundle.md:1-80, writer
metal_indextts2/bundle.py:98-144): ``weights.bin`` starts with b"MIT2", u32
version 1, u32 alignment (4096); every tensor payload starts at an aligned
offset. ``manifest.json`` lists name, shape, dtype, offset, nbytes and sha256
per tensor.

``make_dit_bundle`` writes every tensor the DiT-CFM estimator reads, under the
reference's names (prefix ``s2mel.net.cfm.estimator.``), from a seeded
``numpy.random.default_rng``:

* ``init="baseline"`` — the benchmark configuration: f16 weights ~ N(0, 0.02),
  RMSNorm gammas 1, timestep frequencies exp(-ln(10000) i / 128), weight-norm
  pairs with g = ||v_row|| * U(0.5, 1.5) (a per-row gain, so the folded
  weight differs from v and the fold is visible in every output).
* ``init="unit"`` — same tensors with fan-in scaled weights (std 1/sqrt(K))
  and AdaRMS project_layer biases of 1 on the scale half, so every block
  contributes O(1) to the output; used by parity tests so no sub-path hides
  under rounding.
"""
from __future__ import annotations

import hashlib
import json
import math
import struct
from pathlib import Path
from typing import Iterable

import numpy as np

MAGIC = b"MIT2"
VERSION = 1
ALIGNMENT = 4096
PREFIX = "s2mel.net.cfm.estimator."

_DTYPES = {
    np.dtype(np.float32): "f32",
    np.dtype(np.float16): "f16",
    np.dtype(np.int64): "i64",
    np.dtype(np.int32): "i32",
    np.dtype(np.uint32): "u32",
    np.dtype(np.uint8): "u8",
}
_NP = {v: k for k, v in _DTYPES.items()}


VOICE_TENSORS = ("spk_cond_emb", "s2mel_style", "s2mel_prompt", "mel")


def component_of(name: str) -> str:
    """The manifest `component` of a tensor, by its name (the reference's
    bundle writer groups tensors the same way: gpt, semantic_codec, s2mel,
    bigvgan; the four cached-voice tensors are component voice)."""
    if name in VOICE_TENSORS:
        return "voice"
    for prefix in ("gpt", "semantic_codec", "s2mel", "bigvgan", "campplus"):
        if name.startswith(prefix + "."):
            return prefix
    return "s2mel"


def write_bundle(out_dir: str | Path, tensors: Iterable[tuple[str, np.ndarray]], metadata: dict | None = None) -> dict:
    """Write ``(name, array)`` pairs as an MIT2 bundle; returns the manifest."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    records = []
    with (out / "weights.bin").open("wb") as fp:
        fp.write(struct.pack("<4sII", MAGIC, VERSION, ALIGNMENT))
        for name, arr in tensors:
            arr = np.ascontiguousarray(arr)
            if arr.dtype not in _DTYPES:
                raise TypeError(f"unsupported dtype {arr.dtype} for {name}")
            pos = fp.tell()
            off = (pos + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
            fp.write(b"\0" * (off - pos))
            payload = arr.tobytes()
            fp.write(payload)
            records.append(
                {
                    "name": name,
                    "shape": [int(d) for d in arr.shape],
                    "dtype": _DTYPES[arr.dtype],
                    "offset": off,
                    "nbytes": len(payload),
                    "sha256": hashlib.sha256(payload).hexdigest(),
                    "layout": "row_major",
                    "component": component_of(name),
                }
            )
    manifest = {
        "format": "MIT2",
        "version": VERSION,
        "endianness": "little",
        "alignment": ALIGNMENT,
        "weights_file": "weights.bin",
        "metadata": metadata or {},
        "tensors": records,
    }
    (out / "manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True), encoding="utf-8")
    return manifest


SINGLE_FILE_FOOTER_MAGIC = b"MIT2VOIC"


def write_single_file_bundle(path: str | Path, tensors: Iterable[tuple[str, np.ndarray]],
                             metadata: dict | None = None) -> dict:
    """Write the single-file form of an MIT2 bundle (the reference reads it
    wherever it takes a bundle path, runtime/bundle.cpp:153-200): the weights
    stream, then the manifest JSON, then a 24-byte footer
    [u64 manifest offset][u64 manifest size][b"MIT2VOIC"], little endian."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.parent / (path.name + ".dir")
    man = write_bundle(tmp, tensors, metadata)
    body = (tmp / "weights.bin").read_bytes()
    man = dict(man)
    man.pop("weights_file", None)
    text = json.dumps(man, indent=2, sort_keys=True).encode("utf-8")
    with path.open("wb") as fp:
        fp.write(body)
        fp.write(text)
        fp.write(struct.pack("<QQ8s", len(body), len(text), SINGLE_FILE_FOOTER_MAGIC))
    for f in tmp.iterdir():
        f.unlink()
    tmp.rmdir()
    return man


def _single_file_manifest(path: Path) -> dict:
    raw = path.read_bytes()
    off, size, magic = struct.unpack("<QQ8s", raw[-24:])
    if magic != SINGLE_FILE_FOOTER_MAGIC:
        raise ValueError(f"single-file bundle footer magic missing: {path}")
    return json.loads(raw[off : off + size].decode("utf-8"))


def read_bundle(bundle_dir: str | Path, names: Iterable[str] | None = None, verify: bool = False) -> dict[str, np.ndarray]:
    """Read tensors (all, or ``names``) as numpy arrays in their stored dtype,
    from a bundle directory or a single-file bundle."""
    d = Path(bundle_dir)
    if d.is_file():
        man = _single_file_manifest(d)
        weights = d
    else:
        man = json.loads((d / "manifest.json").read_text(encoding="utf-8"))
        weights = d / man.get("weights_file", "weights.bin")
    want = set(names) if names is not None else None
    out = {}
    raw = np.memmap(weights, dtype=np.uint8, mode="r")
    for rec in man["tensors"]:
        if want is not None and rec["name"] not in want:
            continue
        buf = raw[rec["offset"] : rec["offset"] + rec["nbytes"]]
        if verify and hashlib.sha256(buf.tobytes()).hexdigest() != rec["sha256"]:
            raise ValueError(f"checksum mismatch for {rec['name']}")
        out[rec["name"]] = np.frombuffer(buf.tobytes(), dtype=_NP[rec["dtype"]]).reshape(rec["shape"])
    return out


def dit_tensor_specs() -> list[tuple[str, tuple[int, ...], str]]:
    """(name without prefix, shape, kind) of every estimator tensor.

    kind: "w" weight (fan-in = last dims), "b" bias, "gamma" norm weight,
    "freqs", "wg" weight-norm g, "wv" weight-norm v, "proj_b" AdaRMS project bias.
    """
    s: list[tuple[str, tuple[int, ...], str]] = []
    s += [("cond_projection.weight", (512, 512), "w"), ("cond_projection.bias", (512,), "b")]
    s += [("cond_x_merge_linear.weight", (512, 864), "w"), ("cond_x_merge_linear.bias", (512,), "b")]
    for te in ("t_embedder", "t_embedder2"):
        s += [
            (f"{te}.freqs", (128,), "freqs"),
            (f"{te}.mlp.0.weight", (512, 256), "w"),
            (f"{te}.mlp.0.bias", (512,), "b"),
            (f"{te}.mlp.2.weight", (512, 512), "w"),
            (f"{te}.mlp.2.bias", (512,), "b"),
        ]
    for l in range(13):
        p = f"transformer.layers.{l}."
        for nm in ("attention_norm", "ffn_norm"):
            s += [
                (f"{p}{nm}.norm.weight", (512,), "gamma"),
                (f"{p}{nm}.project_layer.weight", (1024, 512), "w"),
                (f"{p}{nm}.project_layer.bias", (1024,), "proj_b"),
            ]
        s += [
            (f"{p}attention.wqkv.weight", (1536, 512), "w"),
            (f"{p}attention.wo.weight", (512, 512), "w"),
            (f"{p}feed_forward.w1.weight", (1536, 512), "w"),
            (f"{p}feed_forward.w2.weight", (512, 1536), "w"),
            (f"{p}feed_forward.w3.weight", (1536, 512), "w"),
        ]
        if l > 6:
            s += [(f"{p}skip_in_linear.weight", (512, 1024), "w"), (f"{p}skip_in_linear.bias", (512,), "b")]
    s += [
        ("transformer.norm.norm.weight", (512,), "gamma"),
        ("transformer.norm.project_layer.weight", (1024, 512), "w"),
        ("transformer.norm.project_layer.bias", (1024,), "proj_b"),
        ("skip_linear.weight", (512, 592), "w"),
        ("skip_linear.bias", (512,), "b"),
        ("conv1.weight", (512, 512, 1), "w"),
        ("conv1.bias", (512,), "b"),
        ("res_projection.weight", (512, 512), "w"),
        ("res_projection.bias", (512,), "b"),
        ("wavenet.cond_layer.conv.conv.weight_g", (8192, 1, 1), "wg"),
        ("wavenet.cond_layer.conv.conv.weight_v", (8192, 512, 1), "wv"),
        ("wavenet.cond_layer.conv.conv.bias", (8192,), "b"),
    ]
    for l in range(8):
        s += [
            (f"wavenet.in_layers.{l}.conv.conv.weight_g", (1024, 1, 1), "wg"),
            (f"wavenet.in_layers.{l}.conv.conv.weight_v", (1024, 512, 5), "wv"),
            (f"wavenet.in_layers.{l}.conv.conv.bias", (1024,), "b"),
        ]
        rs = 1024 if l < 7 else 512
        s += [
            (f"wavenet.res_skip_layers.{l}.conv.conv.weight_g", (rs, 1, 1), "wg"),
            (f"wavenet.res_skip_layers.{l}.conv.conv.weight_v", (rs, 512, 1), "wv"),
            (f"wavenet.res_skip_layers.{l}.conv.conv.bias", (rs,), "b"),
        ]
    s += [
        ("final_layer.adaLN_modulation.1.weight", (1024, 512), "w"),
        ("final_layer.adaLN_modulation.1.bias", (1024,), "b"),
        ("final_layer.linear.weight_g", (512, 1), "wg"),
        ("final_layer.linear.weight_v", (512, 512), "wv"),
        ("final_layer.linear.bias", (512,), "b"),
        ("conv2.weight", (80, 512, 1), "w"),
        ("conv2.bias", (80,), "b"),
    ]
    return s


def make_dit_tensors(seed: int, init: str = "baseline") -> list[tuple[str, np.ndarray]]:
    """Generate the estimator tensors (f16 except freqs, f32) deterministically."""
    if init not in ("baseline", "unit"):
        raise ValueError("init must be 'baseline' or 'unit'")
    rng = np.random.default_rng(seed)
    out: list[tuple[str, np.ndarray]] = []
    pending_v: dict[str, np.ndarray] = {}
    specs = dit_tensor_specs()
    # Draw weight_v before weight_g: g is ||v_row|| times a per-row gain drawn
    # from U(0.5, 1.5) (its own generator, so the other tensors do not move),
    # so the folded W = g * v / ||v_row|| differs from v and a wrong gain, norm
    # or norm axis in the fold changes the estimator's output.
    gain_rng = np.random.default_rng(seed + 7919)
    for name, shape, kind in specs:
        if kind == "wv":
            fan_in = int(np.prod(shape[1:]))
            std = 0.02 if init == "baseline" else 1.0 / math.sqrt(fan_in)
            pending_v[name] = (rng.standard_normal(shape, dtype=np.float32) * std).astype(np.float16)
    for name, shape, kind in specs:
        full = PREFIX + name
        if kind == "w":
            fan_in = int(np.prod(shape[1:]))
            std = 0.02 if init == "baseline" else 1.0 / math.sqrt(fan_in)
            arr = (rng.standard_normal(shape, dtype=np.float32) * std).astype(np.float16)
        elif kind == "b":
            std = 0.02 if init == "baseline" else 0.1
            arr = (rng.standard_normal(shape, dtype=np.float32) * std).astype(np.float16)
        elif kind == "proj_b":
            std = 0.02 if init == "baseline" else 0.1
            b = rng.standard_normal(shape, dtype=np.float32) * std
            if init == "unit":
                b[:512] += 1.0  # AdaRMS scale half centred on 1
            arr = b.astype(np.float16)
        elif kind == "gamma":
            arr = np.ones(shape, dtype=np.float16)
        elif kind == "freqs":
            i = np.arange(128, dtype=np.float32)
            arr = np.exp(-math.log(10000.0) * i / 128.0).astype(np.float32)
        elif kind == "wv":
            arr = pending_v[name]
        elif kind == "wg":
            v = pending_v[name[: -len("weight_g")] + "weight_v"].astype(np.float32)
            norms = np.sqrt((v.reshape(v.shape[0], -1) ** 2).sum(axis=1))
            gains = gain_rng.uniform(0.5, 1.5, size=norms.shape).astype(np.float32)
            arr = (norms * gains).reshape(shape).astype(np.float16)
        else:
            raise AssertionError(kind)
        out.append((full, arr))
    return out


def make_dit_bundle(out_dir: str | Path, seed: int = 0, init: str = "baseline") -> Path:
    """Write the synthetic estimator bundle; skips work when an identical one exists."""
    out = Path(out_dir)
    stamp = out / ".synthetic"
    key = f"seed={seed} init={init} v2"
    if stamp.exists() and stamp.read_text() == key and (out / "weights.bin").exists():
        return out
    write_bundle(out, make_dit_tensors(seed, init), metadata={"synthetic": True, "seed": seed, "init": init})
    stamp.write_text(key)
    return out


# BigVGAN generator layout (runtime/impl/dit_cfm_bigvgan.cpp:3681-3688, 3961-3980):
# transposed-conv upsamplers (in, out, kernel, stride, padding) and the three
# resblock kernels of each upsampling stage (dilations 1, 3, 5 in every resblock).
BIGVGAN_UPSAMPLERS = [(1536, 768, 8, 4, 2), (768, 384, 8, 4, 2), (384, 192, 4, 2, 1),
                      (192, 96, 4, 2, 1), (96, 48, 4, 2, 1), (48, 24, 4, 2, 1)]
BIGVGAN_RESBLOCK_KERNELS = (3, 7, 11)
BIGVGAN_DILATIONS = (1, 3, 5)
BIGVGAN_HOP = 256


def kaiser_sinc_lowpass(cutoff: float, half_width: float, taps: int = 12) -> np.ndarray:
    """Kaiser-windowed sinc low-pass filter (the anti-aliasing filter design of
    the BigVGAN paper: Kaiser's beta formula for the stop-band attenuation of
    the transition width, window times sinc, normalised to unit DC gain)."""
    half = taps // 2
    delta_f = 4.0 * half_width
    atten = 2.285 * (half - 1) * math.pi * delta_f + 7.95
    if atten > 50.0:
        beta = 0.1102 * (atten - 8.7)
    elif atten >= 21.0:
        beta = 0.5842 * (atten - 21.0) ** 0.4 + 0.07886 * (atten - 21.0)
    else:
        beta = 0.0
    t = np.arange(-half, half, dtype=np.float64) + 0.5
    f = 2.0 * cutoff * np.kaiser(taps, beta) * np.sinc(2.0 * cutoff * t)
    return (f / f.sum()).astype(np.float32)


def bigvgan_tensor_specs() -> list[tuple[str, tuple[int, ...], str]]:
    """(full name, shape, kind) of every BigVGAN tensor the vocoder reads.

    kind: "wv"/"wg" weight norm (v, g), "b" bias, "filt" 12-tap filter,
    "logscale" SnakeBeta alpha/beta (log scale)."""
    s: list[tuple[str, tuple[int, ...], str]] = []

    def conv(prefix: str, rows: int, inner: int, k: int, bias: bool = True):
        s.extend([(f"{prefix}.weight_g", (rows, 1, 1), "wg"), (f"{prefix}.weight_v", (rows, inner, k), "wv")])
        if bias:
            s.append((f"{prefix}.bias", (inner if prefix.startswith("bigvgan.ups") else rows,), "b"))

    def act(prefix: str, c: int):
        s.extend([(f"{prefix}.upsample.filter", (1, 1, 12), "filt"),
                  (f"{prefix}.downsample.lowpass.filter", (1, 1, 12), "filt"),
                  (f"{prefix}.act.alpha", (c,), "logscale"), (f"{prefix}.act.beta", (c,), "logscale")])

    conv("bigvgan.conv_pre", 1536, 80, 7)
    for i, (cin, cout, k, _, _) in enumerate(BIGVGAN_UPSAMPLERS):
        conv(f"bigvgan.ups.{i}.0", cin, cout, k)  # transposed: rows = input channels
        for j, rk in enumerate(BIGVGAN_RESBLOCK_KERNELS):
            r = f"bigvgan.resblocks.{3 * i + j}"
            for p in range(3):
                conv(f"{r}.convs1.{p}", cout, cout, rk)
                conv(f"{r}.convs2.{p}", cout, cout, rk)
            for a in range(6):
                act(f"{r}.activations.{a}", cout)
    act("bigvgan.activation_post", 24)
    conv("bigvgan.conv_post", 1, 24, 7, bias=False)
    return s


def make_bigvgan_tensors(seed: int) -> list[tuple[str, np.ndarray]]:
    """Deterministic synthetic BigVGAN weights: weight_v ~ N(0, 1/fan_in)
    (f16) with weight_g = 0.8 ||v_row|| so each folded conv keeps roughly unit
    gain, biases N(0, 0.02), SnakeBeta log-scale alpha/beta N(0, 0.1), and the
    anti-aliasing filters of a ratio-2 resampler (cutoff 0.25, half-width 0.3)."""
    rng = np.random.default_rng(seed)
    lp = kaiser_sinc_lowpass(0.25, 0.3)
    out: list[tuple[str, np.ndarray]] = []
    v_rows: dict[str, np.ndarray] = {}
    for name, shape, kind in bigvgan_tensor_specs():
        if kind == "wv":
            fan_in = int(np.prod(shape[1:]))
            arr = (rng.standard_normal(shape, dtype=np.float32) / math.sqrt(fan_in)).astype(np.float16)
            v_rows[name[: -len("weight_v")]] = arr
        elif kind == "wg":
            continue  # written after its v (below), in spec order
        elif kind == "b":
            arr = (rng.standard_normal(shape, dtype=np.float32) * 0.02).astype(np.float16)
        elif kind == "filt":
            arr = lp.reshape(shape).copy()
        elif kind == "logscale":
            arr = (rng.standard_normal(shape, dtype=np.float32) * 0.1).astype(np.float32)
        else:
            raise AssertionError(kind)
        out.append((name, arr))
    by_name = dict(out)
    ordered: list[tuple[str, np.ndarray]] = []
    for name, shape, kind in bigvgan_tensor_specs():
        if kind == "wg":
            v = v_rows[name[: -len("weight_g")]].astype(np.float32)
            norms = np.sqrt((v.reshape(v.shape[0], -1) ** 2).sum(axis=1))
            ordered.append((name, (0.8 * norms).reshape(shape).astype(np.float16)))
        else:
            ordered.append((name, by_name[name]))
    return ordered


def make_vocoder_bundle(out_dir: str | Path, seed: int = 0) -> Path:
    """Write the synthetic BigVGAN bundle; skips work when an identical one exists."""
    out = Path(out_dir)
    stamp = out / ".synthetic"
    key = f"bigvgan seed={seed} v2"
    if stamp.exists() and stamp.read_text() == key and (out / "weights.bin").exists():
        return out
    write_bundle(out, make_bigvgan_tensors(seed), metadata={"synthetic": True, "seed": seed, "model": "bigvgan"})
    stamp.write_text(key)
    return out


LR_PREFIX = "s2mel.net.length_regulator."


def length_regulator_tensor_specs() -> list[tuple[str, tuple[int, ...], str]]:
    """(full name, shape, kind) of the length-regulator tensors
    (runtime/impl/gpt.cpp:5271-5317): content_in_proj (1024 -> 512), four
    {k=3 conv, one-group GroupNorm} blocks (model.0/1 .. 9/10), model.12 (k=1)."""
    s = [(LR_PREFIX + "content_in_proj.weight", (512, 1024), "w"), (LR_PREFIX + "content_in_proj.bias", (512,), "b")]
    for conv, norm in ((0, 1), (3, 4), (6, 7), (9, 10)):
        s += [(f"{LR_PREFIX}model.{conv}.weight", (512, 512, 3), "w"), (f"{LR_PREFIX}model.{conv}.bias", (512,), "b"),
              (f"{LR_PREFIX}model.{norm}.weight", (512,), "gamma"), (f"{LR_PREFIX}model.{norm}.bias", (512,), "b")]
    s += [(LR_PREFIX + "model.12.weight", (512, 512, 1), "w"), (LR_PREFIX + "model.12.bias", (512,), "b")]
    return s


def make_length_regulator_tensors(seed: int) -> list[tuple[str, np.ndarray]]:
    """Deterministic synthetic length-regulator weights (f16): weights
    N(0, 1/fan_in), biases N(0, 0.02), GroupNorm gamma 1 + N(0, 0.1)."""
    rng = np.random.default_rng(seed)
    out = []
    for name, shape, kind in length_regulator_tensor_specs():
        if kind == "w":
            arr = rng.standard_normal(shape, dtype=np.float32) / math.sqrt(int(np.prod(shape[1:])))
        elif kind == "b":
            arr = rng.standard_normal(shape, dtype=np.float32) * 0.02
        else:
            arr = 1.0 + rng.standard_normal(shape, dtype=np.float32) * 0.1
        out.append((name, arr.astype(np.float16)))
    return out


def make_condition_bundle(out_dir: str | Path, seed: int = 0) -> Path:
    """Write the synthetic length-regulator bundle; skips work when an identical one exists."""
    out = Path(out_dir)
    stamp = out / ".synthetic"
    key = f"length_regulator seed={seed} v1"
    if stamp.exists() and stamp.read_text() == key and (out / "weights.bin").exists():
        return out
    write_bundle(out, make_length_regulator_tensors(seed),
                 metadata={"synthetic": True, "seed": seed, "model": "length_regulator"})
    stamp.write_text(key)
    return out


def make_voice_tensors(seed: int, prompt_tokens: int = 200, spk_tokens: int = 170) -> list[tuple[str, np.ndarray]]:
    """A synthetic cached-voice profile in the reference's voice-bundle layout
    (f32, component voice): spk_cond_emb [1, S, 1024], s2mel_style [1, 192],
    s2mel_prompt [1, P, 512] and the prompt mel [1, 80, P]."""
    rng = np.random.default_rng(seed)
    return [("spk_cond_emb", rng.standard_normal((1, spk_tokens, 1024), dtype=np.float32)),
            ("s2mel_style", rng.standard_normal((1, 192), dtype=np.float32)),
            ("s2mel_prompt", rng.standard_normal((1, prompt_tokens, 512), dtype=np.float32)),
            ("mel", rng.standard_normal((1, 80, prompt_tokens), dtype=np.float32))]


def make_voice_bundle(out_dir: str | Path, seed: int = 0, prompt_tokens: int = 200, single_file: bool = False) -> Path:
    """Write a synthetic voice bundle (a directory, or with single_file the
    one-file form at out_dir); skips work when an identical directory exists."""
    out = Path(out_dir)
    if single_file:
        write_single_file_bundle(out, make_voice_tensors(seed, prompt_tokens),
                                 metadata={"synthetic": True, "seed": seed, "model": "voice"})
        return out
    stamp = out / ".synthetic"
    key = f"voice seed={seed} P={prompt_tokens} v1"
    if stamp.exists() and stamp.read_text() == key and (out / "weights.bin").exists():
        return out
    write_bundle(out, make_voice_tensors(seed, prompt_tokens), metadata={"synthetic": True, "seed": seed,
                                                                        "model": "voice"})
    stamp.write_text(key)
    return out


GPT_LAYERS, GPT_WIDTH, GPT_MLP, GPT_VOCAB, GPT_POSITIONS = 24, 1280, 5120, 8194, 1818


def gpt_tensor_specs() -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, kind) of the GPT mel-code decoder tensors the reference's
    cached decode reads (runtime/impl/gpt.cpp:1060-1210, 1545-1554, 1877-1909):
    24 GPT-2 blocks (Conv1D weights stored [in, out]), ln_f, final_norm, the
    mel head, the mel-code and position embeddings."""
    s: list[tuple[str, tuple[int, ...], str]] = []
    W, M = GPT_WIDTH, GPT_MLP
    for l in range(GPT_LAYERS):
        p = f"gpt.gpt.h.{l}."
        s += [(p + "ln_1.weight", (W,), "gamma"), (p + "ln_1.bias", (W,), "b"),
              (p + "attn.c_attn.weight", (W, 3 * W), "w"), (p + "attn.c_attn.bias", (3 * W,), "b"),
              (p + "attn.c_proj.weight", (W, W), "w"), (p + "attn.c_proj.bias", (W,), "b"),
              (p + "ln_2.weight", (W,), "gamma"), (p + "ln_2.bias", (W,), "b"),
              (p + "mlp.c_fc.weight", (W, M), "w"), (p + "mlp.c_fc.bias", (M,), "b"),
              (p + "mlp.c_proj.weight", (M, W), "w"), (p + "mlp.c_proj.bias", (W,), "b")]
    s += [("gpt.gpt.ln_f.weight", (W,), "gamma"), ("gpt.gpt.ln_f.bias", (W,), "b"),
          ("gpt.final_norm.weight", (W,), "gamma"), ("gpt.final_norm.bias", (W,), "b"),
          ("gpt.mel_head.weight", (GPT_VOCAB, W), "w"), ("gpt.mel_head.bias", (GPT_VOCAB,), "b"),
          ("gpt.mel_embedding.weight", (GPT_VOCAB, W), "emb"),
          ("gpt.mel_pos_embedding.emb.weight", (GPT_POSITIONS, W), "emb")]
    return s


def make_gpt_tensors(seed: int, stop_bias: float | None = None) -> list[tuple[str, np.ndarray]]:
    """Deterministic synthetic GPT decoder weights (f16): linear weights and
    embeddings N(0, 0.02) (GPT-2's initialisation scale), biases N(0, 0.02),
    LayerNorm gammas 1 + N(0, 0.02). stop_bias, when given, replaces the mel
    head's bias of the stop code (8193), to make the decode stop early."""
    rng = np.random.default_rng(seed)
    out = []
    for name, shape, kind in gpt_tensor_specs():
        a = rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
        if kind == "gamma":
            a += np.float32(1.0)
        if name == "gpt.mel_head.bias" and stop_bias is not None:
            a[GPT_VOCAB - 1] = np.float32(stop_bias)
        out.append((name, a.astype(np.float16)))
    return out


def make_gpt_bundle(out_dir: str | Path, seed: int = 0, stop_bias: float | None = None) -> Path:
    """Write the synthetic GPT decoder bundle (about 1 GB); skips work when an identical one exists."""
    out = Path(out_dir)
    stamp = out / ".synthetic"
    key = f"gpt seed={seed} v1" + ("" if stop_bias is None else f" stop_bias={float(stop_bias)!r}")
    if stamp.exists() and stamp.read_text() == key and (out / "weights.bin").exists():
        return out
    write_bundle(out, make_gpt_tensors(seed, stop_bias), metadata={"synthetic": True, "seed": seed, "model": "gpt"})
    stamp.write_text(key)
    return out


def bundle_f32(bundle_dir: str | Path) -> dict[str, np.ndarray]:
    """All estimator tensors decoded to contiguous float32 (f16 decoding is exact)."""
    return {k: np.ascontiguousarray(v, dtype=np.float32) for k, v in read_bundle(bundle_dir).items()}
