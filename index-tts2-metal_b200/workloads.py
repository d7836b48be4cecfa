"""Seeded synthetic inputs for the benchmark configurations of the DiT-CFM stage.

No public dataset is involved: every configuration is defined by shapes and
distributions (noise, content condition, style and prompt mel ~ N(0, 1)) drawn
from ``numpy.random.default_rng(seed)``.

Configurations (token-major layouts):
  1  one guided step, T=400, P=150, t=0.5                       seed 0
  2  25 steps, T=800, P=200, cfg 0.7                            seed 1
  3  64 utterances, T ~ U{200..1500}, 16 steps, cfg 0.7, padded seed 2
  4  T=4096, P=300, 25 steps, cfg 0.7                           seed 3
  5  1024 x T=800, 12 steps, cfg 0.7, sharded over GPUs         seed 4
     (utterance i from default_rng((4, i)))
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class Utterance:
    noise: np.ndarray   # [T, 80]
    prompt: np.ndarray  # [P, 80]
    cond: np.ndarray    # [T, 512]
    style: np.ndarray   # [192]

    @property
    def T(self) -> int:
        return self.noise.shape[0]

    @property
    def P(self) -> int:
        return self.prompt.shape[0]

    def prompt_x(self) -> np.ndarray:
        px = np.zeros((self.T, 80), np.float32)
        px[: self.P] = self.prompt
        return px


CONFIGS = {
    1: dict(n=1, T=400, P=150, steps=1, cfg=0.7, seed=0),
    2: dict(n=1, T=800, P=200, steps=25, cfg=0.7, seed=1),
    3: dict(n=64, T=(200, 1500), P=None, steps=16, cfg=0.7, seed=2),
    4: dict(n=1, T=4096, P=300, steps=25, cfg=0.7, seed=3),
    5: dict(n=1024, T=800, P=200, steps=12, cfg=0.7, seed=4),
}


def utterance(rng: np.random.Generator, T: int, P: int) -> Utterance:
    return Utterance(
        noise=rng.standard_normal((T, 80), dtype=np.float32),
        prompt=rng.standard_normal((P, 80), dtype=np.float32),
        cond=rng.standard_normal((T, 512), dtype=np.float32),
        style=rng.standard_normal(192, dtype=np.float32),
    )


def utterance_at(cfg_id: int, index: int) -> Utterance:
    """Utterance `index` of a fixed-length configuration, drawn from its own
    stream default_rng((seed, index)), so that any shard of a large job can be
    drawn without the utterances before it."""
    c = CONFIGS[cfg_id]
    if isinstance(c["T"], tuple):
        raise ValueError("utterance_at needs a fixed-length configuration")
    return utterance(np.random.default_rng((c["seed"], index)), c["T"], c["P"])


def config_utterances(cfg_id: int, n: int | None = None, seed_offset: int = 0) -> list[Utterance]:
    """Utterances of a configuration (optionally only the first n, or a shard
    drawn with a distinct seed offset for multi-GPU runs). Configuration 5's
    utterances come from utterance_at (one stream per utterance)."""
    c = CONFIGS[cfg_id]
    if cfg_id == 5:
        count = c["n"] if n is None else n
        return [utterance_at(5, seed_offset + i) for i in range(count)]
    rng = np.random.default_rng(c["seed"] + seed_offset)
    count = c["n"] if n is None else n
    out = []
    for _ in range(count):
        if isinstance(c["T"], tuple):
            T = int(rng.integers(c["T"][0], c["T"][1] + 1))
            P = int(rng.integers(T // 8, T // 3 + 1))
        else:
            T, P = c["T"], c["P"]
        out.append(utterance(rng, T, P))
    return out


def pad_batch(utts: list[Utterance], T_pad: int):
    """Stack utterances into the padded [B, T_pad, ...] arrays of
    itts_cfm_run_padded (zero rows beyond each utterance's length)."""
    B = len(utts)
    noise = np.zeros((B, T_pad, 80), np.float32)
    px = np.zeros((B, T_pad, 80), np.float32)
    cond = np.zeros((B, T_pad, 512), np.float32)
    style = np.zeros((B, 192), np.float32)
    vl = np.zeros(B, np.uint32)
    pl = np.zeros(B, np.uint32)
    for b, u in enumerate(utts):
        noise[b, : u.T] = u.noise
        px[b, : u.P] = u.prompt
        cond[b, : u.T] = u.cond
        style[b] = u.style
        vl[b] = u.T
        pl[b] = u.P
    return vl, pl, noise, px, cond, style


def sincos_inputs(T: int, P: int):
    """The reference self-test's deterministic inputs (cfm_euler tests,
    runtime/impl/dit_cfm_bigvgan.cpp:3306-3325), in float32."""
    i = np.arange(T * 80, dtype=np.float32)
    x = np.sin(i * np.float32(0.018)) * np.float32(0.07) + np.cos((np.arange(T * 80) % 61).astype(np.float32) * np.float32(0.011)) * np.float32(0.03)
    ip = np.arange(P * 80, dtype=np.float32)
    prompt = np.cos(ip * np.float32(0.022)) * np.float32(0.09) + np.sin((np.arange(P * 80) % 37).astype(np.float32) * np.float32(0.019)) * np.float32(0.02)
    ic = np.arange(T * 512, dtype=np.float32)
    cond = np.sin(ic * np.float32(0.009)) * np.float32(0.08) + np.cos((np.arange(T * 512) % 109).astype(np.float32) * np.float32(0.014)) * np.float32(0.04)
    style = np.cos(np.arange(192, dtype=np.float32) * np.float32(0.015)) * np.float32(0.18)
    return (x.reshape(T, 80).astype(np.float32), prompt.reshape(P, 80).astype(np.float32),
            cond.reshape(T, 512).astype(np.float32), style.astype(np.float32))
