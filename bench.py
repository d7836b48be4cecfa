#!/usr/bin/env python
"""DiT-CFM sampler benchmark: mel frames/s through the 25-step CFG sampler.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload 2|5] [--utts B]

A bench "step" is one full sampler run (all CFM steps) over the rank's batch.
The headline workload is configuration 2 per rank: one utterance of T=800
frames (P=200 prompt frames), 25 Euler steps, CFG 0.7, random-init f16
weights ~N(0, 0.02), inputs ~N(0, 1) (seed 1 + rank). Under torchrun each
rank owns one GPU and its own utterance (weak scaling, no data-path
collective); timing is CUDA events on the engine's stream, max over ranks.
Every line also carries `scale_out`: configuration 5 (1024 utterances of
T=800, 12 steps) as ONE job split over the ranks by shard.shard and run
through itts_cfm_run_batch, timed as the max over ranks.

--impl reference times the reference's own CPU path (oracle/_ref, the
reference's run_dit_estimator_step_cpu compiled from its sources) on the
host's cores: K guided CFM steps of the configuration-2 utterance at its full
length (each a conditional and a null estimator call at T=800), spread over
all host threads; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
PKG = REPO / "index-tts2-metal_b200"
for _p in (str(PKG), str(REPO / "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import mit2  # noqa: E402
import workloads  # noqa: E402

METRIC = "mel frames/s, 25-step CFG DiT CFM at 1/2/4/8 B200; ms per CFM step"
UNIT = "mel frames/s"
BUNDLE_DIR = Path(tempfile.gettempdir()) / "itts_bench_bundle_seed0_baseline"
VOC_BUNDLE_DIR = Path(tempfile.gettempdir()) / "itts_bench_bundle_bigvgan_seed0"
VOC_REF_FRAMES = 4  # mel frames per reference CPU vocoder call in the baseline sample
COND_BUNDLE_DIR = Path(tempfile.gettempdir()) / "itts_bench_bundle_length_regulator_seed0"
COND_SEM_PER_MEL = 175 / 600  # semantic frames per generated mel frame in the condition workload
REF_SAMPLE_FRAMES = 32
GPT_BUNDLE_DIR = Path(tempfile.gettempdir()) / "itts_bench_bundle_gpt_seed0"
GPT_PREFIX, GPT_STEPS = 100, 175  # prefix rows; mel codes for 600 mel frames at 175 codes per 600 frames


def step_flops_total(B: int, T: int, cfg: dict) -> float:
    """Algorithmic FLOPs of one guided CFM step for B utterances of T frames."""
    import itts_cfm

    branches = 2 if cfg["cfg"] > 0 else 1
    return itts_cfm.step_flops(B * branches, T)


def gemm_family(prof: list[dict]) -> dict:
    """Sum of the per-op GEMM entries ("gemm.<op>") of a profiled step."""
    rows = [d for d in prof if d["name"].startswith("gemm")]
    return {"name": "gemm", "launches": sum(d["launches"] for d in rows), "ms": sum(d["ms"] for d in rows),
            "flops": sum(d["flops"] for d in rows), "bytes": sum(d["bytes"] for d in rows)}


def gemm_bound_frac(prof: list[dict], tflops_peak: float, hbm_peak: float) -> dict:
    """Fraction of each GEMM's own roofline: the time the measured peaks allow
    a launch (the larger of its FLOPs at the tensor peak and its compulsory
    bytes at the HBM peak), summed over the GEMM family and divided by the
    family's measured time. Also the share of that family time whose bound is
    HBM (the f32 residual-stream epilogues at large M)."""
    rows = [d for d in prof if d["name"].startswith("gemm")]
    bound = hbm_bound = meas = 0.0
    for d in rows:
        t_f = d["flops"] / (tflops_peak * 1e12)
        t_b = d["bytes"] / (hbm_peak * 1e9)
        bound += max(t_f, t_b)
        meas += d["ms"] / 1e3
        if t_b > t_f:
            hbm_bound += d["ms"] / 1e3
    return {"frac": bound / meas if meas > 0 else None,
            "hbm_bound_time_share": hbm_bound / meas if meas > 0 else None,
            "method": "sum over GEMM launches of max(FLOPs / tensor peak, compulsory bytes / HBM peak) "
                      "/ summed event-timed GEMM time"}


def kernel_row(d: dict, reps: int) -> dict:
    """One profiled kernel kind per CFM step: launches, time, TFLOP/s and
    compulsory-HBM GB/s over its summed event-timed launch durations."""
    s = d["ms"] / 1e3
    return {"name": d["name"], "launches_per_step": d["launches"] // reps, "ms_per_step": round(d["ms"] / reps, 4),
            "tflops": round(d["flops"] / s / 1e12, 1) if s > 0 else None,
            "hbm_gbs": round(d["bytes"] / s / 1e9, 1) if s > 0 else None}


def _env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return d, "measured"
        except Exception:
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, interval_ms: int = 20):
        self.gpu = gpu_index
        self.interval = interval_ms
        self.proc = None
        self.path = Path(tempfile.mkstemp(prefix="itts_clocks_", suffix=".csv")[1])

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", str(self.interval)], stdout=self.path.open("w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        self.path.unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------- reference arm

def _ref_guided_step_sample(ref, u, frames: int, threads: int) -> float:
    """Wall time of one guided CFM step (conditional + null estimator calls of
    the reference's run_dit_estimator_step_cpu) on a `frames`-row slice of the
    utterance, run concurrently on `threads` host threads."""
    x = u.noise[:frames].copy()
    px = u.prompt_x()[:frames]
    cond = u.cond[:frames]
    mask = np.ones(frames, np.uint32)
    zp, zc, zs = np.zeros_like(px), np.zeros_like(cond), np.zeros_like(u.style)
    errs = []

    def work():
        try:
            ref.estimator(x, px, cond, u.style, 0.0, mask)
            ref.estimator(x, zp, zc, zs, 0.0, mask)
        except Exception as e:  # pragma: no cover
            errs.append(e)

    ths = [threading.Thread(target=work) for _ in range(threads)]
    t0 = time.perf_counter()
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    dt = time.perf_counter() - t0
    if errs:
        raise errs[0]
    return dt


def _host_threads() -> int:
    n = os.cpu_count() or 1
    try:
        import psutil

        # the reference decodes every weight to fp32 per estimator call (~0.4 GB)
        n = min(n, max(1, int(psutil.virtual_memory().available / 1.0e9)))
    except Exception:
        pass
    return max(1, min(n, 64))


def cpu_vocoder_rate(threads: int):
    """The reference's run_bigvgan_vocoder_cpu on `threads` host threads at
    once, each on a VOC_REF_FRAMES-frame mel: mel frames/s and the wall time."""
    import oracle

    ref = oracle.RefOracle(VOC_BUNDLE_DIR)
    mel = np.random.default_rng(4).standard_normal((VOC_REF_FRAMES, 80)).astype(np.float32)
    errs = []

    def work():
        try:
            ref.vocoder(mel)
        except Exception as e:  # pragma: no cover
            errs.append(e)

    ths = [threading.Thread(target=work) for _ in range(threads)]
    t0 = time.perf_counter()
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    dt = time.perf_counter() - t0
    if errs:
        raise errs[0]
    return threads * VOC_REF_FRAMES / dt, dt


def vocoder_line(args, cfg, rank, world, local, barrier, max_over_ranks, peak, hbm_peak):
    """BigVGAN vocoder throughput on this rank's generated mel rows (T - P of
    the workload's utterance): device-timed graph replays, e2e through
    itts_vocoder_run with pinned host buffers, per-kind profile, roofline of
    the conv GEMMs and of the activation kernel, and the reference CPU vocoder."""
    import ctypes as C

    import torch

    import itts_cfm

    if rank == 0 or world == 1:
        mit2.make_vocoder_bundle(VOC_BUNDLE_DIR, seed=0)
    barrier()
    Tv = cfg["T"] - cfg["P"]
    mel = np.random.default_rng(1000 + rank).standard_normal((Tv, 80)).astype(np.float32)
    voc = itts_cfm.Vocoder(VOC_BUNDLE_DIR, device=local)
    voc.stage(mel)
    for _ in range(3):
        voc.launch()
    voc.fetch()
    st = torch.cuda.ExternalStream(voc.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    nv = 10
    barrier()
    e0.record(st)
    for _ in range(nv):
        voc.launch()
    e1.record(st)
    e1.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1)) / nv
    pin = torch.from_numpy(mel).pin_memory().numpy()
    wave = torch.empty(Tv * itts_cfm.VOCODER_HOP, dtype=torch.float32).pin_memory().numpy()
    lib = itts_cfm.load()

    def e2e_once():
        rc = lib.itts_vocoder_run(voc.h, pin.ctypes.data_as(C.c_void_p), Tv, wave.ctypes.data_as(C.c_void_p))
        if rc != 0:
            raise RuntimeError(lib.itts_vocoder_last_error(voc.h).decode())

    e2e_once()
    barrier()
    t0 = time.perf_counter()
    for _ in range(nv):
        e2e_once()
    t_e2e = max_over_ranks(time.perf_counter() - t0) / nv
    prof = sorted(voc.profile(2), key=lambda d: -d["ms"])
    gem = [d for d in prof if d["name"].startswith(("upsample", "resblock_conv", "conv_pre"))]
    act = [d for d in prof if d["name"].startswith("snake_aa")]
    g_ms = sum(d["ms"] for d in gem)
    a_ms = sum(d["ms"] for d in act)
    g_ach = sum(d["flops"] for d in gem) / (g_ms / 1e3) / 1e12
    a_ach = sum(d["bytes"] for d in act) / (a_ms / 1e3) / 1e9
    launches = voc.launch_kernels()
    voc.close()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle

        if oracle.ref_available():
            threads = max(1, min(_host_threads(), 16))
            fps, t = cpu_vocoder_rate(threads)
            cpu = {"value": fps, "unit": UNIT, "cores": threads, "kind": "reference",
                   "sample": f"{threads} threads, each one run_bigvgan_vocoder_cpu call on a {VOC_REF_FRAMES}-frame "
                             f"mel; {t:.2f} s"}
    return {"metric": "BigVGAN vocoder mel frames/s (mel -> 256 samples per frame)",
            "value": Tv * world / (ms / 1e3), "unit": UNIT, "T": Tv, "ms_per_utterance": ms,
            "tflops": itts_cfm.Vocoder.flops(Tv) / (ms / 1e3) / 1e12, "gpu_launches": launches,
            "e2e": {"value": Tv * world / t_e2e, "unit": UNIT, "h2d_bytes_per_step": int(mel.nbytes),
                    "d2h_bytes_per_step": int(wave.nbytes)},
            "roofline": {"conv_gemm": {"bound": "tensor", "achieved": g_ach, "peak": peak, "unit": "TFLOP/s",
                                       "frac": g_ach / peak},
                         "snake_activation": {"bound": "hbm", "achieved": a_ach, "peak": hbm_peak, "unit": "GB/s",
                                              "frac": a_ach / hbm_peak}},
            "cpu_baseline": cpu,
            "kernels": [kernel_row(d, 2) for d in prof]}


def condition_line(args, cfg, rank, world, local, barrier, max_over_ranks):
    """Condition assembly (length regulator + merge) for this rank's utterance:
    s_infer of round(G * 175/600) semantic frames -> G = T - P generated rows
    after the P prompt rows. Device-timed graph replays, e2e through
    itts_cond_assemble, and the reference CPU length regulator."""
    import ctypes as C

    import torch

    import itts_cfm

    if rank == 0 or world == 1:
        mit2.make_condition_bundle(COND_BUNDLE_DIR, seed=0)
    barrier()
    P, G = cfg["P"], cfg["T"] - cfg["P"]
    n_in = max(1, round(G * COND_SEM_PER_MEL))
    rng = np.random.default_rng(2000 + rank)
    s_infer = rng.standard_normal((n_in, 1024)).astype(np.float32)
    prompt = rng.standard_normal((P, 512)).astype(np.float32)
    ca = itts_cfm.ConditionAssembler(COND_BUNDLE_DIR, device=local)
    ca.stage(s_infer, prompt, G)
    for _ in range(3):
        ca.launch()
    ca.fetch()
    st = torch.cuda.ExternalStream(ca.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    nv = 20
    barrier()
    e0.record(st)
    for _ in range(nv):
        ca.launch()
    e1.record(st)
    e1.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1)) / nv
    ps = torch.from_numpy(s_infer).pin_memory().numpy()
    pp = torch.from_numpy(prompt).pin_memory().numpy()
    out = torch.empty((P + G, 512), dtype=torch.float32).pin_memory().numpy()
    lib = itts_cfm.load()

    def e2e_once():
        rc = lib.itts_cond_assemble(ca.h, ps.ctypes.data_as(C.c_void_p), n_in, pp.ctypes.data_as(C.c_void_p), P, G,
                                    out.ctypes.data_as(C.c_void_p))
        if rc != 0:
            raise RuntimeError(lib.itts_cond_last_error(ca.h).decode())

    e2e_once()
    barrier()
    t0 = time.perf_counter()
    for _ in range(nv):
        e2e_once()
    t_e2e = max_over_ranks(time.perf_counter() - t0) / nv
    launches = ca.launch_kernels()
    ca.close()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle

        if oracle.ref_available():
            ref = oracle.RefOracle(COND_BUNDLE_DIR)
            g_s, n_s = 64, max(1, round(64 * COND_SEM_PER_MEL))
            t0 = time.perf_counter()
            ref.length_regulator(s_infer[:n_s], g_s)
            dt = time.perf_counter() - t0
            cpu = {"value": g_s / dt, "unit": "generated mel frames/s", "cores": 1, "kind": "reference",
                   "sample": f"one run_length_regulator_full_cpu call, {n_s} -> {g_s} frames; {dt:.2f} s"}
    return {"metric": "condition assembly, generated mel frames/s (length regulator + prompt merge)",
            "value": G * world / (ms / 1e3), "unit": "generated mel frames/s", "n_in": n_in, "P": P, "G": G,
            "ms_per_utterance": ms, "tflops": itts_cfm.ConditionAssembler.flops(n_in, G) / (ms / 1e3) / 1e12,
            "gpu_launches": launches,
            "e2e": {"value": G * world / t_e2e, "unit": "generated mel frames/s",
                    "h2d_bytes_per_step": int(s_infer.nbytes + prompt.nbytes), "d2h_bytes_per_step": int(out.nbytes)},
            "cpu_baseline": cpu}


def gpt_line(args, rank, world, local, barrier, max_over_ranks, hbm_peak):
    """GPT mel-code decoder for this rank's utterance: a GPT_PREFIX-row prefix,
    then GPT_STEPS greedy decode steps (random weights never predict the stop
    code, so every step runs). Device-timed prefill and decode from the
    decoder's own events, e2e = wall clock of itts_gpt_generate with the prefix
    in and the codes and logits out; the dominant cost is streaming the f16
    weights once per token, so the roofline is HBM bytes per token."""
    import itts_cfm

    if rank == 0 or world == 1:
        mit2.make_gpt_bundle(GPT_BUNDLE_DIR, seed=0)
    barrier()
    P_rows, S_steps = args.gpt_prefix, args.gpt_steps
    rng = np.random.default_rng(3000 + rank)
    prefix = rng.standard_normal((P_rows, 1280)).astype(np.float32)
    dec = itts_cfm.GptDecoder(GPT_BUNDLE_DIR, device=local)
    dec.generate(prefix, min(16, S_steps))
    runs, pre, dcd, wall = 3, [], [], []
    for _ in range(runs):
        barrier()
        t0 = time.perf_counter()
        codes, _ = dec.generate(prefix, S_steps)
        wall.append(time.perf_counter() - t0)
        p_ms, d_ms = dec.timing()
        pre.append(p_ms)
        dcd.append(d_ms)
    n = len(codes)
    pre_ms, dec_ms, t_e2e = (max_over_ranks(float(np.median(v))) for v in (pre, dcd, wall))
    launches = dec.launch_kernels()
    sampled = None
    if os.environ.get("ITTS_GPT_MODE") != "graph":  # the synthesis pipeline's sampled call (persistent path)
        cfg_s = dict(seed=20240605, temperature=0.8, top_k=30, top_p=0.8, repetition_penalty=10.0)
        hist = [1] * P_rows + [8192]
        dec.generate_sampled(prefix, min(16, S_steps), cfg_s, history=hist, hf_positions=True)
        s_codes, _ = dec.generate_sampled(prefix, S_steps, cfg_s, history=hist, hf_positions=True)
        s_pre, s_dec = dec.timing()
        s_dec = max_over_ranks(s_dec)
        sampled = {"config": "temperature 0.8, top_k 30, top_p 0.8, repetition_penalty 10, generate-style positions",
                   "steps": len(s_codes), "ms_per_token": s_dec / len(s_codes),
                   "value": len(s_codes) * world / (s_dec / 1e3), "unit": "tokens/s"}
    trace = gpt_stage_trace(dec, prefix) if args.gpt_trace else None
    dec.close()
    wb = itts_cfm.GptDecoder.weight_bytes_per_token()
    kv = 24 * 1280 * 2 * 4 * (P_rows + 0.5 * (n + 1))  # fp32 K and V rows read per token, mean over the run
    gbs = (wb + kv) / (dec_ms / n / 1e3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import gpt_oracle
        import threadpoolctl

        o = gpt_oracle.GptOracle(mit2.bundle_f32(GPT_BUNDLE_DIR))
        th = threadpoolctl.threadpool_info()
        cores = max([int(i.get("num_threads", 1)) for i in th if i.get("user_api") == "blas"] or [1])
        ps, ss = 16, 8
        t0 = time.perf_counter()
        o.greedy(prefix[:ps], ss)
        dt = time.perf_counter() - t0
        cpu = {"value": (ps + ss) / dt, "unit": "tokens/s (prefix rows + decode steps)", "cores": cores, "kind": "port",
               "sample": f"oracle/gpt_oracle.py greedy, {ps} prefix rows + {ss} steps, numpy BLAS; {dt:.2f} s"}
    return {"metric": "GPT mel-code decode, tokens/s (cached greedy, one utterance per GPU)",
            "value": n * world / (dec_ms / 1e3), "unit": "tokens/s", "prefix_rows": P_rows, "steps": n,
            "ms_per_token": dec_ms / n, "prefill_ms": pre_ms, "prefill_ms_per_row": pre_ms / max(P_rows, 1),
            "gpu_launches": launches,
            "path": ("graphs per token" if os.environ.get("ITTS_GPT_MODE") == "graph" else
                     "one persistent decode kernel per call" + ("" if os.environ.get("ITTS_GPT_PREFILL") == "rows"
                                                                else ", after the batched prefill kernels")),
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                         "bytes_per_token": wb + kv, "note": "f16 weights once per token + mean fp32 KV-cache reads"},
            "e2e": {"value": n * world / t_e2e, "unit": "tokens/s (prefill included)",
                    "h2d_bytes_per_step": int(prefix.nbytes), "d2h_bytes_per_step": int(n * 4 + 8194 * 4)},
            "cpu_baseline": cpu, "sampled": sampled, "stage_trace": trace}


def gpt_stage_trace(dec, prefix):
    """Per-stage time split of the persistent decoder's first decode token
    (mean over the 24 layers, microseconds), from its global-timer trace:
    prologue, weight slots (ring compute), epilogue, barrier wait of CTA 0;
    the barrier's latency after the last CTA arrived, the arrival skew (last
    minus median), and CTA 0's wait for weight slots."""
    dec.set_tracing(True)
    dec.generate(prefix, 4)
    t = dec.stage_trace()
    dec.set_tracing(False)
    H, S = 485, 121
    G = (len(t) - 2 * H) // S
    if G <= 0:
        return None
    cta0, arr, wait = t[:H], t[H:H + S * G].reshape(S, G), t[H + S * G:]
    names = ["c_attn", "attention", "attn.c_proj", "c_fc", "mlp.c_proj"]
    acc = {}
    for s in range(S):
        nm = "head" if s == S - 1 else names[s % 5]
        start, pro, slots, comp, syn = cta0[4 * s:4 * s + 5]
        acc.setdefault(nm, []).append((pro - start, slots - pro, comp - slots, syn - comp, syn - arr[s].max(),
                                       arr[s].max() - np.median(arr[s]), wait[4 * s + 2]))
    keys = ["prologue", "slots", "epilogue", "barrier_wait", "barrier_latency", "arrival_skew", "slot_wait"]
    out = {nm: dict(zip(keys, (round(float(x), 3) for x in np.mean(v, axis=0)))) for nm, v in acc.items()}
    out["token_us"] = round(float(cta0[H - 1]), 1)
    return out


def pipeline_line(cfg, rank, world, local, barrier, max_over_ranks):
    """End to end from semantic features to waveform through
    itts_pipeline_synthesize (voice profile -> condition assembly -> CFM
    sampler -> vocoder), host buffers in and out, for this rank's utterance of
    the workload's shape; wall-clock per call, max over ranks."""
    import itts_cfm

    voice_dir = Path(tempfile.gettempdir()) / f"itts_bench_voice_P{cfg['P']}"
    if rank == 0 or world == 1:
        mit2.make_dit_bundle(BUNDLE_DIR, seed=0, init="baseline")
        mit2.make_condition_bundle(COND_BUNDLE_DIR, seed=0)
        mit2.make_vocoder_bundle(VOC_BUNDLE_DIR, seed=0)
        mit2.make_voice_bundle(voice_dir, seed=0, prompt_tokens=cfg["P"])
    barrier()
    P, G = cfg["P"], cfg["T"] - cfg["P"]
    n_in = max(1, round(G * COND_SEM_PER_MEL))
    rng = np.random.default_rng(3000 + rank)
    s_infer = rng.standard_normal((n_in, 1024)).astype(np.float32)
    noise = rng.standard_normal((P + G, 80)).astype(np.float32)
    pipe = itts_cfm.Pipeline(BUNDLE_DIR, COND_BUNDLE_DIR, VOC_BUNDLE_DIR, device=local)
    pipe.synthesize(voice_dir, s_infer, G, noise, cfg["steps"], cfg["cfg"])
    nv = 5
    barrier()
    t0 = time.perf_counter()
    for _ in range(nv):
        pipe.synthesize(voice_dir, s_infer, G, noise, cfg["steps"], cfg["cfg"])
    dt = max_over_ranks(time.perf_counter() - t0) / nv
    pipe.close()
    audio_s = G * 256 / 22050.0
    return {"metric": "generated mel frames/s end to end (semantic features + voice -> waveform)",
            "value": G * world / dt, "unit": "generated mel frames/s", "P": P, "G": G, "n_in": n_in,
            "steps_cfm": cfg["steps"], "ms_per_utterance": 1e3 * dt,
            "real_time_factor": dt / audio_s, "audio_seconds_per_second": world * audio_s / dt,
            "timing": "host wall clock around itts_pipeline_synthesize (host buffers in and out)"}


def cpu_reference_rate(u, steps_cfm: int, threads: int, reps: int = 1):
    """Our arm's bounded CPU sample: `threads` host threads each run one guided
    step of the reference on a REF_SAMPLE_FRAMES-frame slice; frames/s of a
    `steps_cfm`-step run, and the seconds per guided step per slice."""
    import oracle

    ref = oracle.RefOracle(BUNDLE_DIR)
    ts = [_ref_guided_step_sample(ref, u, REF_SAMPLE_FRAMES, threads) for _ in range(reps)]
    t = min(ts)
    fps = threads * REF_SAMPLE_FRAMES / (steps_cfm * t)
    return fps, t


def _ref_call_pool(calls, threads: int, durations: list | None = None) -> float:
    """Run reference estimator calls (zero-argument callables) on `threads`
    host threads, each thread taking the next call as it frees up; returns
    the wall seconds until the last call ends (and appends each call's own
    seconds to `durations`)."""
    import queue

    q = queue.Queue()
    for c in calls:
        q.put(c)
    errs = []

    def worker():
        while True:
            try:
                c = q.get_nowait()
            except queue.Empty:
                return
            try:
                t0 = time.perf_counter()
                c()
                if durations is not None:
                    durations.append(time.perf_counter() - t0)
            except Exception as e:  # pragma: no cover
                errs.append(e)

    ths = [threading.Thread(target=worker) for _ in range(max(1, min(threads, len(calls))))]
    t0 = time.perf_counter()
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    dt = time.perf_counter() - t0
    if errs:
        raise errs[0]
    return dt


def _guided_step_calls(ref, u, t: float = 0.0):
    """The two reference estimator calls of one guided CFM step over the
    whole utterance (conditional, then null with zero prompt/cond/style)."""
    x = u.noise.copy()
    x[: u.P] = 0
    px = u.prompt_x()
    mask = np.ones(u.T, np.uint32)
    zp, zc, zs = np.zeros_like(px), np.zeros_like(u.cond), np.zeros_like(u.style)
    return [lambda: ref.estimator(x, px, u.cond, u.style, t, mask), lambda: ref.estimator(x, zp, zc, zs, t, mask)]


def run_reference(args, rank):
    """The reference arm: the reference's compiled run_dit_estimator_step_cpu
    on the configuration-2 utterance at its full length (T=800). The timed
    region runs `steps` guided CFM steps (2 * steps estimator calls at
    T=800), rounded up to whole rounds of the host threads, spread over all
    of them; frames/s is that of full 25-step sampler runs. Configuration 1 (one guided step at T=400, P=150, t=0.5) is
    measured exactly on one thread while the warm-up calls run."""
    if rank != 0:
        return 0
    import oracle

    cfg = workloads.CONFIGS[args.workload]
    if not oracle.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libref_cfm.so was not built"}))
        return 0
    mit2.make_dit_bundle(BUNDLE_DIR, seed=0, init="baseline")
    u = workloads.config_utterances(args.workload, n=1)[0]
    threads = _host_threads()
    ref = oracle.RefOracle(BUNDLE_DIR)
    # Configuration 1 exactly, on its own thread, during the warm-up calls.
    u1 = workloads.config_utterances(1)[0]
    c1 = {}

    def config1():
        px1 = u1.prompt_x()
        m1 = np.ones(u1.T, np.uint32)
        t0 = time.perf_counter()
        ref.estimator(u1.noise, px1, u1.cond, u1.style, 0.5, m1)
        ref.estimator(u1.noise, np.zeros_like(px1), np.zeros_like(u1.cond), np.zeros_like(u1.style), 0.5, m1)
        c1["s"] = time.perf_counter() - t0

    th1 = threading.Thread(target=config1)
    th1.start()
    warm = [c for _ in range(args.warmup) for c in _guided_step_calls(ref, u)]
    _ref_call_pool(warm, max(1, threads - 1))
    th1.join()
    # Whole rounds of calls keep every host thread busy: `steps` guided steps
    # rounded up to a multiple of threads / 2 (a partly idle last round would
    # understate the reference's throughput).
    per_round = max(1, threads // 2)
    steps_run = ((args.steps + per_round - 1) // per_round) * per_round
    calls = [c for _ in range(steps_run) for c in _guided_step_calls(ref, u)]
    per_call = []
    wall = _ref_call_pool(calls, threads, per_call)
    fps = steps_run * u.T / (cfg["steps"] * wall)
    sample = (f"{steps_run} guided CFM steps ({args.steps} requested, rounded up to whole rounds of the host "
              f"threads) of the config-{args.workload} utterance at its full length (T={u.T}, P={u.P}): "
              f"{2 * steps_run} run_dit_estimator_step_cpu calls (conditional + null) over {threads} host threads, "
              f"{wall:.1f} s; frames/s = guided steps*T/({cfg['steps']} CFM steps * wall)")
    line = {
        "impl": "reference", "metric": METRIC, "value": fps, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * wall / steps_run, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"config {args.workload}", "T": u.T, "P": u.P, "steps_cfm": cfg["steps"],
                   "cfg_rate": cfg["cfg"]},
        "s_per_estimator_call_median": statistics.median(per_call),
        "ms_per_guided_step_one_thread": 2e3 * statistics.median(per_call),
        "cpu_baseline": {"value": fps, "unit": UNIT, "cores": threads, "kind": "reference", "sample": sample,
                         "host": _host_model()},
        "config1": {"workload": "config 1: one guided step (cond + null), T=400, P=150, t=0.5, seed 0",
                    "ms_per_guided_step": 1e3 * c1.get("s", float("nan")), "cores": 1,
                    "note": "measured on one thread while the warm-up calls ran on the other threads"},
        "e2e": {"value": fps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def _host_model() -> str:
    try:
        for line in subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout.splitlines():
            if line.startswith("Model name"):
                return f"{line.split(':', 1)[1].strip()}, nproc {os.cpu_count()}"
    except Exception:
        pass
    return f"nproc {os.cpu_count()}"


# ---------------------------------------------------------------- configurations 3, 4 and 5

def _timed_launches(ctx, launches, steps: int, cfg_rate: float, reps: int = 1) -> float:
    """Device milliseconds of the sampler over a list of padded batches
    (vl, pl, noise, px, cond, style) with inputs resident: each batch is
    staged, warmed once, then its graph launches are bracketed by CUDA events
    on the context's stream; the sum over batches of the mean per launch."""
    import torch

    st = torch.cuda.ExternalStream(ctx.stream())
    total = 0.0
    for vl, pl, noise, px, cond, style in launches:
        ctx.stage_padded(vl, pl, noise, px, cond, style, steps, cfg_rate)
        ctx.launch()
        ctx.sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            ctx.launch()
        e1.record(st)
        e1.synchronize()
        total += e0.elapsed_time(e1) / reps
    return total


def scale_out_line(ctx, rank, world, barrier, max_over_ranks, gather_ranks, peak):
    """Configuration 5 as ONE job: 1024 utterances of T=800 (utterance i from
    default_rng((4, i))), 12 CFM steps, CFG 0.7, partitioned over the ranks by
    shard.shard (longest-processing-time on F(T), no communication) and run
    through the sampler. `value`: the whole job's frames over the max over
    ranks of each rank's device time with its share resident in HBM (its
    share is one padded batch, as itts_cfm_run_batch plans it); `e2e`: the same
    job through itts_cfm_run_batch with host buffers (wall clock, max over
    ranks)."""
    import itts_cfm
    import shard

    c = workloads.CONFIGS[5]
    n, T = c["n"], c["T"]
    lengths = [T] * n
    parts = shard.shard(lengths, world)
    mine = parts[rank]
    utts = [workloads.utterance_at(5, i) for i in mine]
    plan = itts_cfm.batch_plan([u.T for u in utts], c["cfg"])
    launches = [workloads.pad_batch([utts[i] for i in idx], utts[idx[0]].T) for idx in plan]
    barrier()
    dev_ms = _timed_launches(ctx, launches, c["steps"], c["cfg"])
    del launches
    per_rank_ms = gather_ranks(dev_ms)
    job_ms = max(per_rank_ms)
    batch = [dict(noise=u.noise, prompt=u.prompt, cond=u.cond, style=u.style) for u in utts]
    barrier()
    t0 = time.perf_counter()
    ctx.run_batch(batch, c["steps"], c["cfg"])
    host_s = time.perf_counter() - t0
    job_host_s = max_over_ranks(host_s)
    flops = n * itts_cfm.step_flops(2, T) * c["steps"]
    h2d = sum(u.noise.nbytes + u.prompt.nbytes + u.cond.nbytes + u.style.nbytes for u in utts)
    return {"metric": "mel frames/s, configuration 5 as one job sharded over the GPUs",
            "workload": f"{n} utterances x T={T} (P={c['P']}), {c['steps']} CFM steps, CFG {c['cfg']}, "
                        f"shard.shard over {world} rank(s), utterance i from default_rng((4, i))",
            "value": n * T / (job_ms / 1e3), "unit": UNIT, "job_ms": job_ms, "per_rank_ms": per_rank_ms,
            "utterances_per_rank": [len(p) for p in parts], "imbalance": shard.imbalance(lengths, parts),
            "tflops": flops / (job_ms / 1e3) / 1e12, "frac": flops / (job_ms / 1e3) / 1e12 / peak,
            "gpus_active": sum(1 for v in per_rank_ms if v > 0), "scaling": "strong (fixed job)",
            "e2e": {"value": n * T / job_host_s, "unit": UNIT, "job_s": job_host_s,
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(len(utts) * T * 80 * 4),
                    "path": "itts_cfm_run_batch, host buffers in and out (this rank's share)"}}


def config3_line(ctx, rank, world, barrier, max_over_ranks, peak, cpu_sec_per_flop):
    """Configuration 3 on every GPU: 64 utterances with lengths drawn from
    200..1500 (seed 2), 16 CFM steps, CFG 0.7, planned into padded launches as
    itts_cfm_run_batch plans them (length classes, each launch padded to its
    longest utterance, key-padding masks). Frames and FLOPs count the real
    (unpadded) lengths."""
    import itts_cfm

    c = workloads.CONFIGS[3]
    utts = workloads.config_utterances(3)
    Ts = [u.T for u in utts]
    plan = itts_cfm.batch_plan(Ts, c["cfg"])
    launches = [workloads.pad_batch([utts[i] for i in idx], Ts[idx[0]]) for idx in plan]
    barrier()
    dev_ms = max_over_ranks(_timed_launches(ctx, launches, c["steps"], c["cfg"]))
    del launches
    batch = [dict(noise=u.noise, prompt=u.prompt, cond=u.cond, style=u.style) for u in utts]
    barrier()
    t0 = time.perf_counter()
    ctx.run_batch(batch, c["steps"], c["cfg"])
    host_s = max_over_ranks(time.perf_counter() - t0)
    frames = sum(Ts)
    padded = sum(Ts[idx[0]] * len(idx) for idx in plan)
    flops = sum(itts_cfm.step_flops(2, T) for T in Ts) * c["steps"]
    cpu = None
    if cpu_sec_per_flop:
        cpu_s = flops * cpu_sec_per_flop
        cpu = {"value": frames / cpu_s, "unit": UNIT, "kind": "reference", "extrapolated": True,
               "sample": "the configuration-2 CPU sample's seconds per algorithmic FLOP times this workload's "
                         "F(T) summed over the drawn lengths and 16 steps"}
    return {"metric": "mel frames/s, configuration 3 (bucketed serving batch)",
            "workload": f"{len(utts)} utterances, T in [{min(Ts)}, {max(Ts)}] (seed 2), {c['steps']} CFM steps, "
                        f"CFG {c['cfg']}, {len(plan)} padded launches, padding {padded / frames - 1:.1%}",
            "value": world * frames / (dev_ms / 1e3), "unit": UNIT, "ms_per_run": dev_ms,
            "tflops": flops / (dev_ms / 1e3) / 1e12, "frac": flops / (dev_ms / 1e3) / 1e12 / peak,
            "e2e": {"value": world * frames / host_s, "unit": UNIT, "s_per_run": host_s,
                    "path": "itts_cfm_run_batch, host buffers in and out"},
            "cpu_baseline": cpu}


def config4_line(ctx, rank, world, barrier, max_over_ranks, peak, cpu_sec_per_flop):
    """Configuration 4 on every GPU: one utterance of T=4096 (P=300, seed 3),
    25 CFM steps, CFG 0.7; device-timed graph runs with inputs resident and
    the per-kernel split of one CFM step."""
    import itts_cfm

    c = workloads.CONFIGS[4]
    u = workloads.config_utterances(4)[0]
    launches = [workloads.pad_batch([u], u.T)]
    barrier()
    dev_ms = max_over_ranks(_timed_launches(ctx, launches, c["steps"], c["cfg"], reps=3))
    prof = ctx.profile_step(reps=1)
    prof.sort(key=lambda d: -d["ms"])
    flops = itts_cfm.step_flops(2, u.T) * c["steps"]
    attn = [d for d in prof if d["name"] == "attention"]
    tot = sum(d["ms"] for d in prof)
    cpu = None
    if cpu_sec_per_flop:
        cpu_s = flops * cpu_sec_per_flop
        cpu = {"value": u.T / cpu_s, "unit": UNIT, "kind": "reference", "extrapolated": True,
               "sample": "the configuration-2 CPU sample's seconds per algorithmic FLOP times F(4096) x 25 steps"}
    return {"metric": "mel frames/s, configuration 4 (T=4096 long utterance)",
            "workload": f"1 utterance, T={u.T}, P={u.P}, {c['steps']} CFM steps, CFG {c['cfg']}",
            "value": world * u.T / (dev_ms / 1e3), "unit": UNIT, "ms_per_run": dev_ms,
            "ms_per_cfm_step": dev_ms / c["steps"], "tflops": flops / (dev_ms / 1e3) / 1e12,
            "frac": flops / (dev_ms / 1e3) / 1e12 / peak,
            "attention_share": attn[0]["ms"] / tot if attn and tot else None,
            "kernels": [kernel_row(d, 1) for d in prof], "cpu_baseline": cpu}


# ---------------------------------------------------------------- our arm

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", type=int, choices=[2, 5], default=2)
    ap.add_argument("--utts", type=int, default=None, help="utterances per GPU (default: 1 for config 2)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batched", type=int, default=64,
                    help="also time a padded batch of this many utterances per GPU (0 = skip)")
    ap.add_argument("--vocoder", type=int, default=1, help="also time the BigVGAN vocoder (0 = skip)")
    ap.add_argument("--condition", type=int, default=1,
                    help="also time the condition assembly before the sampler (0 = skip)")
    ap.add_argument("--pipeline", type=int, default=1,
                    help="also time the whole semantic-features-to-waveform chain (0 = skip)")
    ap.add_argument("--gpt", type=int, default=1, help="also time the GPT mel-code decoder (0 = skip)")
    ap.add_argument("--gpt-only", action="store_true", help="time only the GPT decoder and print its line")
    ap.add_argument("--gpt-prefix", type=int, default=GPT_PREFIX, help="GPT prefix rows")
    ap.add_argument("--gpt-steps", type=int, default=GPT_STEPS, help="GPT decode steps")
    ap.add_argument("--gpt-trace", action="store_true", help="add the persistent decoder's stage trace to the gpt line")
    ap.add_argument("--vocoder-only", action="store_true",
                    help="time only the BigVGAN vocoder and print its line (profiling aid)")
    ap.add_argument("--scale-out", type=int, default=1,
                    help="also run configuration 5 as one job sharded over the ranks (0 = skip)")
    ap.add_argument("--config3", type=int, default=1, help="also time configuration 3 (0 = skip)")
    ap.add_argument("--config4", type=int, default=1, help="also time configuration 4 (0 = skip)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg (profiling aid)")
    ap.add_argument("--no-profile", action="store_true", help="skip the per-launch profile (profiling aid)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = _env_int("RANK", 0)
    world = _env_int("WORLD_SIZE", 1)
    local = _env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        return run_reference(args, rank)

    import torch

    import itts_cfm

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def gather_ranks(v: float) -> list[float]:
        if dist is None:
            return [v]
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        out = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        return [float(x.item()) for x in out]

    cfg = workloads.CONFIGS[args.workload]
    if args.gpt_only:
        peaks, _ = measured_peaks()
        g = gpt_line(args, rank, world, local, barrier, max_over_ranks, float(peaks.get("hbm_gbs", 6546.0)))
        if rank == 0:
            print(json.dumps(dict(g, n_gpus=world, higher_is_better=True, scaling="weak", data="synthetic",
                                  dtype="f32 activations, f16 weights",
                                  config={"workload": f"GPT decode: {g['prefix_rows']} prefix rows + "
                                                      f"{g['steps']} steps, random-init f16 weights seed 0"})))
        if dist is not None:
            dist.destroy_process_group()
        return 0
    if args.vocoder_only:
        peaks, _ = measured_peaks()
        v = vocoder_line(args, cfg, rank, world, local, barrier, max_over_ranks,
                         float(peaks.get("bf16_tflops", 1590.0)), float(peaks.get("hbm_gbs", 6546.0)))
        if rank == 0:
            print(json.dumps(dict(v, n_gpus=world, higher_is_better=True, scaling="weak", data="synthetic",
                                  dtype="f16", config={"workload": f"BigVGAN vocoder on the {v['T']} generated mel "
                                                                   f"rows of a config-{args.workload} utterance"})))
        if dist is not None:
            dist.destroy_process_group()
        return 0
    if rank == 0 or world == 1:
        mit2.make_dit_bundle(BUNDLE_DIR, seed=0, init="baseline")
    barrier()
    B = args.utts or (1 if args.workload == 2 else 64)
    utts = workloads.config_utterances(args.workload, n=B, seed_offset=rank * 1000)
    T = cfg["T"]
    vl, pl, noise, px, cond, style = workloads.pad_batch(utts, T)
    ctx = itts_cfm.Context(BUNDLE_DIR, device=local)
    ctx.stage_padded(vl, pl, noise, px, cond, style, cfg["steps"], cfg["cfg"])
    launches_per_step = ctx.launch_kernels()
    stream = torch.cuda.ExternalStream(ctx.stream())

    for _ in range(args.warmup):
        ctx.launch()
    ctx.sync()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.05)
    barrier()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        ctx.launch()
    ev1.record(stream)
    ev1.synchronize()
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    ctx.sync()
    frames_per_step = B * T * world
    value = frames_per_step * args.steps / (ms / 1e3)

    # e2e through the public API with pinned host buffers and host<->device copies.
    pin = lambda a: torch.from_numpy(a).pin_memory().numpy()  # noqa: E731
    h_noise, h_px, h_cond, h_style = pin(noise), pin(px), pin(cond), pin(style)
    h_out = torch.empty((B, T, 80), dtype=torch.float32).pin_memory().numpy()
    import ctypes as C

    lib = itts_cfm.load()
    vl_c, pl_c = np.ascontiguousarray(vl), np.ascontiguousarray(pl)

    def e2e_once():
        rc = lib.itts_cfm_run_padded(ctx.h, B, T, vl_c.ctypes.data_as(C.c_void_p), pl_c.ctypes.data_as(C.c_void_p),
                                     h_noise.ctypes.data_as(C.c_void_p), h_px.ctypes.data_as(C.c_void_p),
                                     h_cond.ctypes.data_as(C.c_void_p), h_style.ctypes.data_as(C.c_void_p),
                                     cfg["steps"], float(cfg["cfg"]), h_out.ctypes.data_as(C.c_void_p))
        if rc != 0:
            raise RuntimeError(lib.itts_cfm_last_error(ctx.h).decode())

    e2e_value = None
    if not args.no_e2e:
        for _ in range(2):
            e2e_once()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_once()
        t_e2e = time.perf_counter() - t0
        barrier()
        t_e2e = max_over_ranks(t_e2e)
        e2e_value = frames_per_step * args.steps / t_e2e
    h2d = noise.nbytes + px.nbytes + cond.nbytes + style.nbytes + vl.nbytes + pl.nbytes + B * 2 * T * 4
    d2h = B * T * 80 * 4 + 4

    # Roofline of the dominant kernel family (all tcgen05 GEMM launches of a
    # CFM step). The per-launch event profile gives each kernel kind's share
    # of the summed launch time; the GEMM family's time INSIDE the timed graph
    # is that share of the device-timed CFM step, so the family's time never
    # exceeds the step it belongs to.
    ms_per_cfm = ms / args.steps / cfg["steps"]
    peaks, peaks_kind = measured_peaks()
    peak = float(peaks.get("bf16_tflops", 1590.0))
    roofline = None
    if not args.no_profile:
        ctx.stage_padded(vl, pl, noise, px, cond, style, cfg["steps"], cfg["cfg"])
        prof = ctx.profile_step(reps=3)
        prof.sort(key=lambda d: -d["ms"])
        total_prof_ms = sum(d["ms"] for d in prof)
        gemm = gemm_family(prof)
        share = gemm["ms"] / total_prof_ms
        gemm_ms_in_graph = share * ms_per_cfm
        gemm_flops_per_step = gemm["flops"] / 3
        achieved = gemm_flops_per_step / (gemm_ms_in_graph / 1e3) / 1e12
        assert gemm_ms_in_graph <= ms_per_cfm * (1 + 1e-9)
        traffic = None
        tf = REPO / "profiles" / "gemm_traffic.json"
        if tf.exists():
            try:
                traffic = json.loads(tf.read_text()).get(f"config{args.workload}_bytes_per_launch")
            except Exception:
                traffic = None
        launches = gemm["launches"] // 3
        roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                    "traffic": traffic, "kernel": "gemm_tc_kernel (tcgen05, all GEMM launches of one CFM step)",
                    "launches_per_cfm_step": launches, "gemm_flops_per_cfm_step": gemm_flops_per_step,
                    "time_share": share, "gemm_ms_per_cfm_step_in_graph": gemm_ms_in_graph,
                    "avg_launch_us": 1e3 * gemm_ms_in_graph / max(launches, 1),
                    "event_sum_ms_per_cfm_step": total_prof_ms / 3, "ms_per_cfm_step": ms_per_cfm,
                    "method": "achieved = GEMM FLOPs per CFM step / (GEMM share of the per-launch event profile x "
                              "device-timed CFM step of the graph run)",
                    "peak_source": f"MEASURED_PEAKS.json bf16_tflops ({peaks_kind}, burst)",
                    "kernels": [kernel_row(d, 3) for d in prof]}

    # Batched serving throughput on the same utterance shape (supplementary):
    # utterances per GPU share one padded batch, so the GEMMs see large M.
    batched = None
    if args.batched > 0:
        Bb = args.batched
        butts = workloads.config_utterances(args.workload, n=Bb, seed_offset=rank * 1000 + 500)
        bvl, bpl, bno, bpx, bco, bst = workloads.pad_batch(butts, T)
        ctx.stage_padded(bvl, bpl, bno, bpx, bco, bst, cfg["steps"], cfg["cfg"])
        ctx.launch()
        ctx.sync()
        bev0 = torch.cuda.Event(enable_timing=True)
        bev1 = torch.cuda.Event(enable_timing=True)
        barrier()
        bev0.record(stream)
        nb = 3
        for _ in range(nb):
            ctx.launch()
        bev1.record(stream)
        bev1.synchronize()
        barrier()
        bms = max_over_ranks(bev0.elapsed_time(bev1)) / nb
        bprof = ctx.profile_step(reps=2)
        bprof.sort(key=lambda d: -d["ms"])
        bg = gemm_family(bprof)
        b_ach = bg["flops"] / (bg["ms"] / 1e3) / 1e12
        batched = {"utterances_per_gpu": Bb, "value": Bb * T * world / (bms / 1e3), "unit": UNIT,
                   "ms_per_run": bms, "ms_per_cfm_step": bms / cfg["steps"],
                   "tflops": step_flops_total(Bb, T, cfg) * cfg["steps"] / (bms / 1e3) / 1e12,
                   "gemm_tflops": b_ach, "gemm_frac": b_ach / peak,
                   "gemm_roofline_bound": gemm_bound_frac(bprof, peak, float(peaks.get("hbm_gbs", 6546.0))),
                   "kernels": [kernel_row(d, 2) for d in bprof]}

    condition = None
    if args.condition:
        condition = condition_line(args, cfg, rank, world, local, barrier, max_over_ranks)

    pipeline = None
    if args.pipeline:
        pipeline = pipeline_line(cfg, rank, world, local, barrier, max_over_ranks)

    vocoder = None
    if args.vocoder:
        vocoder = vocoder_line(args, cfg, rank, world, local, barrier, max_over_ranks, peak,
                               float(peaks.get("hbm_gbs", 6546.0)))

    gpt = None
    if args.gpt:
        gpt = gpt_line(args, rank, world, local, barrier, max_over_ranks, float(peaks.get("hbm_gbs", 6546.0)))

    cpu = None
    cpu_sec_per_flop = None  # reference CPU seconds per algorithmic FLOP, from the sample (for extrapolation)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle

        if oracle.ref_available():
            threads = _host_threads()
            fps, t = cpu_reference_rate(utts[0], cfg["steps"], threads)
            cpu_sec_per_flop = t / (threads * itts_cfm.step_flops(2, REF_SAMPLE_FRAMES))
            cpu = {"value": fps, "unit": UNIT, "cores": threads, "kind": "reference",
                   "sample": (f"{threads} threads, each one guided CFM step (cond + null run_dit_estimator_step_cpu) "
                              f"on a {REF_SAMPLE_FRAMES}-frame slice of the T={T} utterance; {t:.2f} s; scaled to "
                              f"frames/s of a {cfg['steps']}-step run (the full-length measurement is the "
                              f"--impl reference arm)"), "host": _host_model()}

    scale_out = None
    if args.scale_out:
        scale_out = scale_out_line(ctx, rank, world, barrier, max_over_ranks, gather_ranks, peak)
    config3 = None
    if args.config3:
        config3 = config3_line(ctx, rank, world, barrier, max_over_ranks, peak, cpu_sec_per_flop)
    config4 = None
    if args.config4:
        config4 = config4_line(ctx, rank, world, barrier, max_over_ranks, peak, cpu_sec_per_flop)

    ctx.close()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": f"config {args.workload}: {B} utterance(s)/GPU, T={T}, P={cfg['P']}, "
                                   f"{cfg['steps']} CFM steps, CFG {cfg['cfg']}",
                       "utterances_per_gpu": B, "T": T, "steps_cfm": cfg["steps"], "cfg_rate": cfg["cfg"],
                       "global_batch": B * world, "parallelism": f"utterance-sharded x{world}",
                       "l2": "working set > L2: 182 MB of weights re-read every CFM step (126 MB L2)",
                       "weights": "random-init f16 ~N(0,0.02), seed 0"},
            "ms_per_cfm_step": ms_per_cfm,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "clocks": clk,
            "batched": batched,
            "scale_out": scale_out,
            "config3": config3,
            "config4": config4,
            "condition": condition,
            "vocoder": vocoder,
            "pipeline": pipeline,
            "gpt": gpt,
        }
        print(json.dumps(line))
    if dist is not None:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
