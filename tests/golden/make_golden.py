"""Generate the golden vectors that pin the CPU oracle to the reference.

Runs the reference's own CPU functions (oracle/_ref/libref_cfm.so, compiled
from the reference sources by oracle/build_ref.py) on small seeded cases and
stores inputs + outputs as compressed .npz files next to this script. The
synthetic bundles are regenerated from their seeds (index-tts2-metal_b200/mit2.py);
each file records the sha256 of the bundle's weights.bin so generator drift
is detected.

    python tests/golden/make_golden.py

Cases (inputs follow the reference's self-tests where it has them):
  kat_tembed        t_embedder / t_embedder2 at t in {0, 0.37, 0.96}
  kat_noise         make_deterministic_normal_noise(5, 80, 1234) and (3, 7, 0)
  kat_estimator_t6  run_dit_estimator_step_test inputs (T=6, t=0.37, mask 111100),
                    unit and baseline bundles
  kat_estimator_t33 seeded N(0,1) inputs, T=33, t=0.5, 3 padded keys (unit)
  kat_attention_t6  attention core of layers 0 and 12, masks 111100 / 101110
  kat_wavenet_t6    WaveNet stack with a global condition, mask 111100
  kat_euler_t5      run_cfm_euler_test inputs (T=5, P=2): 3 steps cfg 0 and 25 steps cfg 0.5
  kat_euler_masked  T=8 (2 padded), P=2, 2 steps, cfg 0.7 (padded-batch semantics)
  kat_bigvgan       BigVGAN vocoder (run_bigvgan_vocoder_cpu) on a seeded T=3 mel,
                    and two anti-aliased SnakeBeta activations (768 and 24
                    channels) on seeded inputs, synthetic vocoder bundle seed 0

  kat_length_regulator  run_length_regulator_full_cpu on its self-test input
                    (run_length_regulator_full_test: 7 -> 11 frames) and on a
                    seeded 40 -> 63 case, synthetic length-regulator bundle seed 0

  kat_gpt_decode    run_gpt_kv_greedy_cpu (cached greedy mel-code decode, 24 layers)
                    on a seeded 4-row prefix for 3 steps, synthetic GPT bundle seed 0
  kat_gpt_decode_hf the same with hf_generate_positions = true (the synthesis
                    pipeline's call) on a seeded 5-row prefix for 3 steps
  kat_gpt_sampling  apply_gpt_sampling_processors + sample_gpt_token_from_logits
                    (repetition penalty, temperature, top-k, top-p, SplitMix64
                    draws) on the reference's own test vector and on the GPT
                    golden's last logits under five configurations

    python tests/golden/make_golden.py [--only bigvgan|lr|gpt|gpt_hf|gpt_sampling]
"""
from __future__ import annotations

import hashlib
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "index-tts2-metal_b200"))
sys.path.insert(0, str(REPO / "oracle"))

import mit2  # noqa: E402
import oracle  # noqa: E402
import workloads  # noqa: E402

ROOT = Path(tempfile.gettempdir()) / "itts_golden_bundles"


def f32(a):
    return np.asarray(a, dtype=np.float32)


def weights_sha(d: Path) -> str:
    h = hashlib.sha256()
    with (d / "weights.bin").open("rb") as f:
        for chunk in iter(lambda: f.read(1 << 22), b""):
            h.update(chunk)
    return h.hexdigest()


def estimator_selftest_inputs():
    """run_dit_estimator_step_test inputs (runtime/impl/dit_cfm_bigvgan.cpp:2829-2848)."""
    T = 6
    i = np.arange(T * 80, dtype=np.float32)
    m53 = (np.arange(T * 80) % 53).astype(np.float32)
    m47 = (np.arange(T * 80) % 47).astype(np.float32)
    x = np.sin(i * np.float32(0.021)) * np.float32(0.10) + np.cos(m53 * np.float32(0.017)) * np.float32(0.04)
    px = np.cos(i * np.float32(0.019)) * np.float32(0.08) + np.sin(m47 * np.float32(0.023)) * np.float32(0.03)
    ic = np.arange(T * 512, dtype=np.float32)
    m127 = (np.arange(T * 512) % 127).astype(np.float32)
    cond = np.sin(ic * np.float32(0.010)) * np.float32(0.09) + np.cos(m127 * np.float32(0.013)) * np.float32(0.05)
    style = np.cos(np.arange(192, dtype=np.float32) * np.float32(0.016)) * np.float32(0.20)
    return f32(x).reshape(T, 80), f32(px).reshape(T, 80), f32(cond).reshape(T, 512), f32(style)


def bigvgan_cases():
    voc = mit2.make_vocoder_bundle(ROOT / "bigvgan_seed0", seed=0)
    rv = oracle.RefOracle(voc)
    rng = np.random.default_rng(9)
    mel = f32(rng.standard_normal((3, 80)))
    xa = f32(rng.standard_normal((13, 768)))
    xp = f32(rng.standard_normal((41, 24)) * 0.5)
    np.savez_compressed(HERE / "kat_bigvgan.npz", mel=mel, wave=rv.vocoder(mel), x_act=xa,
                        act_rb0=rv.activation("bigvgan.resblocks.0.activations.0", xa), x_post=xp,
                        act_post=rv.activation("bigvgan.activation_post", xp), bundle_seed=0,
                        weights_sha256=weights_sha(voc))


def length_regulator_cases():
    lrb = mit2.make_condition_bundle(ROOT / "length_regulator_seed0", seed=0)
    r = oracle.RefOracle(lrb)
    # run_length_regulator_full_test inputs (runtime/impl/gpt.cpp:5382-5390)
    i = np.arange(7 * 1024, dtype=np.float32)
    x7 = f32(np.sin(i * np.float32(0.017)) * np.float32(0.1) +
             np.cos((np.arange(7 * 1024) % 131).astype(np.float32) * np.float32(0.013)) * np.float32(0.2)).reshape(7, 1024)
    x40 = f32(np.random.default_rng(12).standard_normal((40, 1024)))
    np.savez_compressed(HERE / "kat_length_regulator.npz", x7=x7, out7_11=r.length_regulator(x7, 11), x40=x40,
                        out40_63=r.length_regulator(x40, 63), bundle_seed=0, weights_sha256=weights_sha(lrb))


def gpt_cases():
    gb = mit2.make_gpt_bundle(ROOT / "gpt_seed0", seed=0)
    r = oracle.RefOracle(gb)
    prefix = f32(np.random.default_rng(7).standard_normal((4, 1280)))
    toks, logits, stop = r.gpt_greedy(prefix, 3)
    np.savez_compressed(HERE / "kat_gpt_decode.npz", prefix=prefix, codes=np.array(toks, np.uint32),
                        last_logits=logits, first_stop=np.int32(stop), bundle_seed=0, weights_sha256=weights_sha(gb))


SAMPLING_CASES = [
    # (name, seed, temperature, top_k, top_p, repetition_penalty, draws)
    ("ref_test", 20240605, 0.5, 4, 0.95, 2.0, 8),          # the reference's own processors test
    ("production", 20240605, 0.8, 30, 0.8, 10.0, 32),     # the synthesis pipeline's sampled call
    ("wide", 7, 1.0, 200, 0.95, 1.0, 32),
    ("greedy_k1", 11, 0.8, 1, 1.0, 1.3, 8),
    ("big_topp", 3, 1.2, 2048, 0.5, 1.0, 32),
]


def gpt_sampling_cases():
    """apply_gpt_sampling_processors + sample_gpt_token_from_logits of the
    reference on its own test vector and on the GPT golden's last logits."""
    gb = mit2.make_gpt_bundle(ROOT / "gpt_seed0", seed=0)
    r = oracle.RefOracle(gb)
    g = np.load(HERE / "kat_gpt_decode.npz")
    big = g["last_logits"].astype(np.float32)
    hist_big = np.array([1] * 30 + [8192] + [int(c) for c in g["codes"]], np.uint32)
    out = {}
    for name, seed, t, k, p, pen, draws in SAMPLING_CASES:
        logits = np.arange(-2, 8, dtype=np.float32) if name == "ref_test" else big
        hist = np.array([2, 7, 3, 7], np.uint32) if name == "ref_test" else hist_big
        proc, toks = r.gpt_sample(logits, hist, seed, t, k, p, pen, draws)
        out[f"{name}_logits"] = logits
        out[f"{name}_history"] = hist
        out[f"{name}_config"] = np.array([seed, t, k, p, pen, draws], np.float64)
        out[f"{name}_processed"] = proc
        out[f"{name}_tokens"] = np.array(toks, np.uint32)
    np.savez_compressed(HERE / "kat_gpt_sampling.npz", **out)


def gpt_hf_cases():
    """The synthesis pipeline's call (hf_generate_positions = true,
    runtime/impl/tts_synthesis/synthesis_pipeline.cpp:675, 795)."""
    gb = mit2.make_gpt_bundle(ROOT / "gpt_seed0", seed=0)
    r = oracle.RefOracle(gb)
    prefix = f32(np.random.default_rng(8).standard_normal((5, 1280)))
    toks, logits, stop = r.gpt_greedy(prefix, 3, hf_positions=True)
    np.savez_compressed(HERE / "kat_gpt_decode_hf.npz", prefix=prefix, codes=np.array(toks, np.uint32),
                        last_logits=logits, first_stop=np.int32(stop), bundle_seed=0, weights_sha256=weights_sha(gb))


def main():
    only = sys.argv[sys.argv.index("--only") + 1] if "--only" in sys.argv else None
    if only == "gpt_sampling":
        gpt_sampling_cases()
        print("golden vectors written to", HERE)
        return
    if only in ("gpt", "gpt_hf"):
        if only == "gpt":
            gpt_cases()
            gpt_sampling_cases()
        gpt_hf_cases()
        print("golden vectors written to", HERE)
        return
    if only == "bigvgan":
        bigvgan_cases()
        print("golden vectors written to", HERE)
        return
    if only == "lr":
        length_regulator_cases()
        print("golden vectors written to", HERE)
        return
    bigvgan_cases()
    length_regulator_cases()
    gpt_cases()
    gpt_hf_cases()
    gpt_sampling_cases()
    unit = mit2.make_dit_bundle(ROOT / "seed0_unit", seed=0, init="unit")
    base = mit2.make_dit_bundle(ROOT / "seed0_baseline", seed=0, init="baseline")
    ru, rb = oracle.RefOracle(unit), oracle.RefOracle(base)
    meta = lambda d, init: dict(bundle_seed=0, bundle_init=init, weights_sha256=weights_sha(d))  # noqa: E731

    ts = np.array([0.0, 0.37, 0.96], np.float32)
    np.savez_compressed(HERE / "kat_tembed.npz", t=ts, t1=np.stack([ru.timestep_embed(t, 0) for t in ts]),
                        t2=np.stack([ru.timestep_embed(t, 1) for t in ts]), **meta(unit, "unit"))

    np.savez_compressed(HERE / "kat_noise.npz", a=ru.noise(5, 80, 1234), b=ru.noise(3, 7, 0))

    x, px, cond, style = estimator_selftest_inputs()
    mask = np.array([1, 1, 1, 1, 0, 0], np.uint32)
    np.savez_compressed(HERE / "kat_estimator_t6.npz", x=x, prompt_x=px, cond=cond, style=style, mask=mask,
                        t=np.float32(0.37), vel_unit=ru.estimator(x, px, cond, style, 0.37, mask),
                        vel_baseline=rb.estimator(x, px, cond, style, 0.37, mask),
                        baseline_weights_sha256=weights_sha(base), **meta(unit, "unit"))

    rng = np.random.default_rng(33)
    T = 33
    x = f32(rng.standard_normal((T, 80)))
    px = np.zeros((T, 80), np.float32)
    px[:5] = rng.standard_normal((5, 80))
    cond = f32(rng.standard_normal((T, 512)))
    style = f32(rng.standard_normal(192))
    mask = np.ones(T, np.uint32)
    mask[-3:] = 0
    np.savez_compressed(HERE / "kat_estimator_t33.npz", x=x, prompt_x=px, cond=cond, style=style, mask=mask,
                        t=np.float32(0.5), vel=ru.estimator(x, px, cond, style, 0.5, mask), **meta(unit, "unit"))

    rng = np.random.default_rng(6)
    xa = f32(rng.standard_normal((6, 512)))
    ma = np.array([1, 1, 1, 1, 0, 0], np.uint32)
    mb = np.array([1, 0, 1, 1, 1, 0], np.uint32)
    np.savez_compressed(HERE / "kat_attention_t6.npz", x=xa, mask_a=ma, mask_b=mb,
                        l0_a=ru.attention_layer(xa, ma, 0), l0_b=ru.attention_layer(xa, mb, 0),
                        l12_a=ru.attention_layer(xa, ma, 12), **meta(unit, "unit"))

    i = np.arange(6 * 512, dtype=np.float32)
    xw = f32(np.sin(i * np.float32(0.010)) * np.float32(0.08) +
             np.cos((np.arange(6 * 512) % 181).astype(np.float32) * np.float32(0.013)) * np.float32(0.04)).reshape(6, 512)
    gi = np.arange(512, dtype=np.float32)
    g = f32(np.sin(gi * np.float32(0.019)) * np.float32(0.04) + np.cos((np.arange(512) % 71).astype(np.float32) * np.float32(0.023)) * np.float32(0.02))
    np.savez_compressed(HERE / "kat_wavenet_t6.npz", x=xw, g=g, mask=ma, out=ru.wavenet(xw, g, ma), **meta(unit, "unit"))

    x5, p5, c5, s5 = workloads.sincos_inputs(5, 2)
    np.savez_compressed(HERE / "kat_euler_t5.npz", noise=x5, prompt=p5, cond=c5, style=s5,
                        mel_3_cfg0=ru.euler(x5, p5, c5, s5, 2, 3, 0.0),
                        mel_25_cfg05=ru.euler(x5, p5, c5, s5, 2, 25, 0.5), **meta(unit, "unit"))

    rng = np.random.default_rng(8)
    T = 8
    n8 = f32(rng.standard_normal((T, 80)))
    p8 = np.zeros((T, 80), np.float32)
    p8[:2] = rng.standard_normal((2, 80))
    c8 = f32(rng.standard_normal((T, 512)))
    s8 = f32(rng.standard_normal(192))
    m8 = np.array([1] * 6 + [0] * 2, np.uint32)
    np.savez_compressed(HERE / "kat_euler_masked.npz", noise=n8, prompt_x=p8, cond=c8, style=s8, mask=m8,
                        mel=ru.euler_masked(n8, p8, c8, s8, m8, 2, 2, 0.7), **meta(unit, "unit"))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
