#!/usr/bin/env python
"""Stream-frames/s of the streaming-transformer LM step (semantic-voice-local's STT / TTS
language-model token loop) on B200s, one process per GPU.

A step is one frame of the LM for every stream the GPU holds: embeddings, every layer (norm,
QKV + RoPE + KV-ring write, sliding-window attention, out-proj, FFN) and the head with the
greedy argmax, fed back on the device. Streams are independent, so N GPUs run N independent
batches ("weak" scaling, no collective on the data path).

  python bench.py [--config 2] [--gpus N --steps K --warmup W] [--impl ours|reference]
                  [--layers L] [--no-config3] [--no-cpu-baseline]

The default workload is BASELINE config 2 (STT-1b, q8_0 weights, batch 1), timed at a steady
state (every frame attends to the full 750-key window); the same run then measures BASELINE
config 3 (STT-1b bf16, 256 streams per GPU at staggered fills) under the key "config3", and the
Mimi codec (encoder + quantizer, decoder; 64 streams per GPU) under the key "codec".
--layers L builds the workload with its first L layers only: the small cases for ncu
captures (such a line is a profiling case, not a benchmark number).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT / "semantic-ai_b200"), str(ROOT / "oracle")]

from svl import config as C  # noqa: E402
from svl import synth  # noqa: E402

CONFIGS = {
    "1": dict(workload="stt-1b f32 batch 1 (BASELINE config 1)", preset="stt_1b", wdt="f32",
              kv="f32", batch=1, frames=1000, steady=True),
    "2": dict(workload="stt-1b q8_0 batch 1 (BASELINE config 2)", preset="stt_1b", wdt="q8_0",
              kv="f32", batch=1, frames=1000, steady=True),
    "3": dict(workload="stt-1b bf16 256 streams/GPU, staggered fills (BASELINE config 3)",
              preset="stt_1b", wdt="bf16", kv="bf16", batch=256, frames=1000, stagger=750),
    "4": dict(workload="stt-2.6b q4_1 batch 1 (BASELINE config 4)", preset="stt_2b6",
              wdt="q4_1", kv="bf16", batch=1, frames=1500, steady=True),
    "4b": dict(workload="stt-2.6b q4_1 128 streams/GPU (BASELINE config 4)", preset="stt_2b6",
               wdt="q4_1", kv="bf16", batch=128, frames=1500, stagger=375),
    "5": dict(workload="pocket-tts bf16 512 streams/GPU, 64-token prompts (BASELINE config 5)",
              kind="tts", wdt="bf16", kv="bf16", batch=512, frames=500, prompt=64),
    "codec": dict(workload="codec: STT Mimi encoder + 32-codebook RVQ, and Pocket-TTS Mimi decoder, "
                           "64 streams/GPU, one 80 ms frame per stream per step",
                  kind="codec", wdt="f32", kv="f32", batch=64, frames=100),
}


def profiled_traffic(config: str, family: str):
    """DRAM bytes (read + write) per launch of the dominant kernel from the ncu capture
    summarised in profiles/ (`traffic: <config> <family prefix> <bytes>` lines), or None."""
    f = ROOT / "profiles" / "traffic.txt"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        parts = line.split()
        if len(parts) == 4 and parts[0] == "traffic:" and parts[1] == config and family.startswith(parts[2]):
            return int(parts[3])
    return None


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def preset(name: str) -> C.SttConfig:
    return getattr(C, name)()


def matmul_params(stt, cfg) -> int:
    """Weights of the step's matrix products (layers + text head): FLOPs per stream-frame = 2x."""
    d, qd, kvd, F = cfg.d_model, cfg.num_heads * cfg.head_dim, cfg.num_kv_heads * cfg.head_dim, cfg.ffn_hidden
    per_layer = (qd + 2 * kvd) * d + d * qd + 2 * F * d + d * F
    return cfg.num_layers * per_layer + stt.text_card * d


def init_dist(world, local_rank):
    if world <= 1:
        return None
    import datetime
    import torch
    import torch.distributed as dist
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local_rank))
    return dist


def max_over_ranks(dist, x: float, device) -> float:
    """The largest x over all ranks (x itself without a process group): every multi-GPU time
    is the slowest rank's."""
    if not dist:
        return float(x)
    import torch
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def rank_streams(rank: int, per_rank: int) -> range:
    """The global indices of the streams rank `rank` runs: ranks shard the streams in contiguous
    blocks of per_rank, so stream g's inputs (seeded by g) do not depend on the GPU count."""
    return range(rank * per_rank, (rank + 1) * per_rank)


def stt_spec_config(spec, layers):
    import dataclasses
    stt = preset(spec["preset"])
    if layers:
        stt = dataclasses.replace(stt, num_layers=layers)
    return stt, stt.transformer(spec["wdt"], spec["kv"])


def measure_stt(args, spec, rank, world, local_rank, dist, weights=None, full=True):
    """One STT workload: device-timed stream-frames/s (K frames after W warm-up frames), the
    same end to end through the host-buffer C-ABI call, the kernel families' rooflines."""
    import torch
    from svl import LanguageModel
    from svl import _lib

    stt, cfg = stt_spec_config(spec, args.layers)
    B, K, W = spec["batch"], args.steps, args.warmup
    if weights is None:
        weights = synth.stt_weights(stt, cfg, seed=0)
    model = LanguageModel(stt, cfg, weights, device=local_rank)
    L = _lib.lib()
    wbytes = model.weight_bytes
    dev = f"cuda:{local_rank}"

    # Per-stream audio: global stream g draws from seed 1 + g; frame 0 sees the initial tokens.
    g0 = rank_streams(rank, B).start
    audio = synth.audio_tokens(stt, K + W, seed=1 + g0, streams=B)
    rng = np.random.default_rng(2 + rank)
    if spec.get("stagger"):
        offsets = rng.integers(0, spec["stagger"], size=B)
    elif spec.get("steady") and cfg.context:
        # Steady state: every timed frame attends to the full window (the stream has run for
        # at least `window` frames).
        offsets = np.full(B, cfg.context, int)
    else:
        offsets = np.zeros(B, int)

    stream = torch.cuda.Stream()
    sptr = ctypes.c_void_p(stream.cuda_stream)

    def fresh_state():
        st = model.init_state(B)
        for b in range(B):
            if offsets[b]:
                # Position the stream at its fill level (len 0: the ring contents stand in for
                # the history, so the attention reads exactly min(pos + 1, window) keys).
                _lib.check(L.svl_state_import(st.handle, b, 0, None, None, 0, int(offsets[b])))
        return st

    def to_dev(a):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).to(dev)

    a_dev = to_dev(audio)  # [frames][B][n_q]
    for b in range(B):
        if offsets[b] == 0:
            a_dev[0, b] = stt.card
    text = [torch.full((B,), stt.text_card, dtype=torch.int32, device=dev),
            torch.zeros(B, dtype=torch.int32, device=dev)]
    row = B * stt.n_q * 4

    def device_steps(st, first, n):
        for i in range(n):
            src, dst = text[i % 2], text[(i + 1) % 2]
            _lib.check(L.svl_stt_step_device(model.handle, st.handle, B, ctypes.c_void_p(src.data_ptr()),
                                             ctypes.c_void_p(a_dev.data_ptr() + (first + i) * row),
                                             ctypes.c_void_p(dst.data_ptr()), None, sptr))

    # Warm-up (also captures the step's CUDA graph), then a fresh state for the timed run.
    st = fresh_state()
    with torch.cuda.stream(stream):
        device_steps(st, 0, W)
    stream.synchronize()
    st.close()
    st = fresh_state()
    text[0].fill_(stt.text_card)
    torch.cuda.synchronize()

    clocks = ClockSampler(local_rank)
    clocks.start()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        device_steps(st, W, K)
        e1.record(stream)
    stream.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(dist, ms, dev)
    value = world * B * K / (ms_max / 1000.0)
    st.close()

    out = {"value": round(value, 2), "ms_per_step": round(ms_max / K, 4), "clocks": clk}
    if not full:
        return out, model, weights

    # End to end through the host-buffer C-ABI call: H2D of the step's tokens and D2H of the
    # argmax inside the timed region, every step.
    st = fresh_state()
    prev = np.full(B, stt.text_card, np.uint32)
    aud = audio.copy()
    for b in range(B):
        if offsets[b] == 0:
            aud[0, b] = stt.card
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(K):
        prev = model.step(prev, aud[i], st)
    e2e_s = time.perf_counter() - t0
    e2e_value = world * B * K / max_over_ranks(dist, e2e_s, dev)
    st.close()

    # Kernel families, timed on their launching stream with every stream at its mean fill of
    # the timed frames.
    peaks, peak_kind = load_peaks()
    kern = {}
    st = fresh_state()
    fills = [int(min(o + K // 2, cfg.context or o + K)) for o in offsets]
    for b in range(B):
        _lib.check(L.svl_state_import(st.handle, b, 0, None, None, 0, fills[b]))
    for which, name in ((0, "products (all weight products of a step)"), (1, "attention (all layers)")):
        nbytes = ctypes.c_int64()
        iters = 20
        with torch.cuda.stream(stream):
            _lib.check(L.svl_profile_kernels(model.handle, st.handle, B, which, 3, sptr, ctypes.byref(nbytes)))
            stream.synchronize()
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record(stream)
            _lib.check(L.svl_profile_kernels(model.handle, st.handle, B, which, iters, sptr, ctypes.byref(nbytes)))
            a1.record(stream)
        stream.synchronize()
        per = a0.elapsed_time(a1) / iters
        kern[name] = {"ms_per_step": round(per, 5), "bytes_per_step": nbytes.value,
                      "gbs": round(nbytes.value / (per / 1e3) / 1e9, 1)}
    st.close()
    prod = kern["products (all weight products of a step)"]
    flops = 2.0 * matmul_params(stt, cfg) * B
    prod["tflops"] = round(flops / (prod["ms_per_step"] / 1e3) / 1e12, 2)
    dom = max(kern, key=lambda k: kern[k]["ms_per_step"])
    nk = ctypes.c_int32()
    st = fresh_state()
    _lib.check(L.svl_step_kernel_count(model.handle, st.handle, B, ctypes.byref(nk)))
    st.close()
    n_launch_dom = (cfg.num_layers * 4 + 1) if dom.startswith("products") else cfg.num_layers
    hbm = peaks["hbm_gbs"]
    src = f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback"
    roofline = {"bound": "hbm", "kernel": dom, "achieved": kern[dom]["gbs"],
                "peak": hbm, "unit": "GB/s", "frac": round(kern[dom]["gbs"] / hbm, 4),
                "peak_source": src, "traffic": profiled_traffic(spec["key"], dom) if not args.layers else None,
                "launches_per_step": n_launch_dom,
                "algorithmic_bytes_per_launch": kern[dom]["bytes_per_step"] // n_launch_dom}
    if B >= 16:
        tpk = peaks.get("bf16_tflops_sustained", 1400.0)
        roofline["tensor"] = {"kernel": "products (tcgen05 GEMMs with their operand preparation)",
                              "achieved": prod["tflops"], "peak": tpk, "unit": "TFLOP/s",
                              "frac": round(prod["tflops"] / tpk, 4),
                              "peak_source": "MEASURED_PEAKS.json bf16_tflops_sustained"}
    # Step-level roofline: weights + KV read + KV written per step over HBM bandwidth.
    el = 2 if cfg.kv_dtype == "bf16" else 4
    kv = sum(C.kv_bytes_per_stream(cfg, f) for f in fills)
    step_bytes = wbytes + kv + B * cfg.num_layers * 2 * cfg.num_kv_heads * cfg.head_dim * el
    step_frac = step_bytes / (ms_max / K / 1e3) / (hbm * 1e9)
    out.update({
        "e2e": {"value": round(e2e_value, 2), "unit": "stream-frames/s",
                "h2d_bytes_per_step": B * (1 + stt.n_q) * 4, "d2h_bytes_per_step": B * 4},
        "gpu_launches": nk.value * K,
        "roofline": roofline,
        "step_roofline": {"bytes_per_step": int(step_bytes), "frac": round(step_frac, 4),
                          "unit": "of measured HBM GB/s"},
        "kernels": kern,
        "config": {"workload": spec["workload"] + (f", first {args.layers} layers only (profiling case)" if args.layers else ""),
                   "streams_per_gpu": B, "frames": K,
                   "d_model": cfg.d_model, "layers": cfg.num_layers, "window": cfg.context,
                   "kv_dtype": cfg.kv_dtype,
                   "positions": ("steady state: every timed frame attends to the full window"
                                 if spec.get("steady") else
                                 f"staggered fills: stream start offsets U[0, {spec['stagger']}) seed 2+rank"
                                 if spec.get("stagger") else "from position 0"),
                   "parallelism": f"{world} GPU(s) x {B} independent streams, no collective",
                   "l2": f"inputs larger than L2: {wbytes / 1e9:.3f} GB of weights + "
                         f"{kv / 1e9:.3f} GB of KV read per step"},
    })
    return out, model, weights


def run_ours(args, spec, rank, world, local_rank):
    import gc
    import torch
    torch.cuda.set_device(local_rank)
    dist = init_dist(world, local_rank)
    res, model, weights = measure_stt(args, spec, rank, world, local_rank, dist)
    stt, cfg = stt_spec_config(spec, args.layers)
    out = {
        "metric": "stream-frames/s", "value": res["value"], "unit": "stream-frames/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": spec["wdt"], "data": "synthetic (random-init N(0,0.02) weights seed 0, uniform audio tokens seed 1+stream)",
        "config": res["config"], "e2e": res["e2e"], "gpu_launches": res["gpu_launches"],
        "roofline": res["roofline"], "step_roofline": res["step_roofline"],
        "kernels": res["kernels"], "clocks": res["clocks"],
    }
    del model
    gc.collect()
    # BASELINE config 3 in the same run (the north star's many-stream and scaling target):
    # STT-1b bf16, 256 streams per GPU, from the same seed-0 f32 weights.
    if args.config == "2" and not args.no_config3 and not args.layers:
        s3 = dict(CONFIGS["3"], key="3")
        r3, m3, _ = measure_stt(args, s3, rank, world, local_rank, dist, weights=weights)
        out["config3"] = {"metric": "stream-frames/s", "value": r3["value"], "unit": "stream-frames/s",
                          "ms_per_step": r3["ms_per_step"], "dtype": "bf16", "config": r3["config"],
                          "e2e": r3["e2e"], "gpu_launches": r3["gpu_launches"],
                          "roofline": r3["roofline"], "step_roofline": r3["step_roofline"],
                          "kernels": r3["kernels"], "clocks": r3["clocks"]}
        del m3
        gc.collect()
    # The codec around the LMs in the same run: 64 streams per GPU, one
    # frame per step, 50 timed steps.
    if args.config == "2" and not args.no_codec and not args.layers:
        sc = dict(CONFIGS["codec"], key="codec")
        cd = measure_codec(args, sc, rank, world, local_rank, dist, 50, 5, cpu=False)
        out["codec"] = {k: cd[k] for k in ("metric", "value", "unit", "ms_per_step", "dtype", "config",
                                           "e2e", "roofline", "decoder")}
        gc.collect()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(spec, stt, cfg, weights, budget_s=args.cpu_seconds)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def tts_config(spec):
    import dataclasses
    cfg, tts = C.pocket_tts()
    return dataclasses.replace(cfg, weight_dtype=spec["wdt"], kv_dtype=spec["kv"]), tts


def run_tts(args, spec, rank, world, local_rank):
    """FlowLm::step for every stream of the GPU per frame: a 64-token text prompt prefilled
    per stream (FlowLm::prompt_text), then frames of latent feedback (LatentGenerator::advance,
    tts/mod.rs:494) with the noise passed in as an input tensor (seed 4, temperature 1)."""
    import torch
    from svl import FlowLm
    from svl import _lib

    torch.cuda.set_device(local_rank)
    dist = init_dist(world, local_rank)
    cfg, tts = tts_config(spec)
    B, K, W, P = spec["batch"], args.steps, args.warmup, spec["prompt"]
    weights = synth.tts_weights(cfg, tts, seed=0)
    model = FlowLm(cfg, tts, weights, device=local_rank)
    L = _lib.lib()
    g0 = rank_streams(rank, B).start
    tokens = np.stack([np.random.default_rng(3 + g0 + b).integers(0, tts.text_bins, size=P, dtype=np.uint32)
                       for b in range(B)])
    noise = np.random.default_rng(4 + rank).standard_normal((K + W, B, tts.latent_dim)).astype(np.float32)
    dev = f"cuda:{local_rank}"
    d_noise = torch.from_numpy(noise).to(dev)
    lat = [torch.zeros((B, tts.latent_dim), dtype=torch.float32, device=dev) for _ in range(2)]
    eos = torch.zeros(B, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream()
    sptr = ctypes.c_void_p(stream.cuda_stream)
    row = B * tts.latent_dim * 4

    def fresh_state():
        st = model.init_state(B, max_positions=P + K + W + 1)
        model.prompt_text_batch(tokens, st)
        return st

    def device_steps(st, first, n):
        for i in range(n):
            src = None if first + i == 0 else ctypes.c_void_p(lat[i % 2].data_ptr())
            _lib.check(L.svl_tts_step_device(model.handle, st.handle, B, src,
                                             ctypes.c_void_p(d_noise.data_ptr() + (first + i) * row), 1,
                                             ctypes.c_void_p(lat[(i + 1) % 2].data_ptr()),
                                             ctypes.c_void_p(eos.data_ptr()), sptr))

    st = fresh_state()
    with torch.cuda.stream(stream):
        device_steps(st, 0, W)
    stream.synchronize()
    st.close()
    st = fresh_state()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        device_steps(st, 0, K)
        e1.record(stream)
    stream.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms_max = max_over_ranks(dist, e0.elapsed_time(e1), dev)
    value = world * B * K / (ms_max / 1000.0)
    st.close()

    # End to end through the host-buffer call: noise H2D, latent + EOS D2H every step.
    st = fresh_state()
    prev = None
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(K):
        prev, _ = model.step(prev, noise[i], st)
    e2e_s = time.perf_counter() - t0
    e2e_value = world * B * K / max_over_ranks(dist, e2e_s, dev)
    st.close()

    # Kernel families: transformer products, attention (at the run's mean fill), flow head.
    peaks, peak_kind = load_peaks()
    kern = {}
    st = model.init_state(B, max_positions=P + K + W + 1)
    fill = P + K // 2
    for b in range(B):
        _lib.check(L.svl_state_import(st.handle, b, 0, None, None, 0, fill))
    names = {0: "products (transformer linears)", 1: "attention (all layers)", 2: "flow head"}
    for which, name in names.items():
        nbytes = ctypes.c_int64()
        iters = 20
        with torch.cuda.stream(stream):
            _lib.check(L.svl_profile_kernels(model.handle, st.handle, B, which, 3, sptr, ctypes.byref(nbytes)))
            stream.synchronize()
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record(stream)
            _lib.check(L.svl_profile_kernels(model.handle, st.handle, B, which, iters, sptr, ctypes.byref(nbytes)))
            a1.record(stream)
        stream.synchronize()
        per = a0.elapsed_time(a1) / iters
        kern[name] = {"ms_per_step": per, "bytes_per_step": nbytes.value,
                      "gbs": nbytes.value / (per / 1e3) / 1e9}
    nk = ctypes.c_int32()
    _lib.check(L.svl_step_kernel_count(model.handle, st.handle, B, ctypes.byref(nk)))
    st.close()
    dom = max(kern, key=lambda k: kern[k]["ms_per_step"])
    hbm = peaks["hbm_gbs"]
    n_launch_dom = cfg.num_layers if dom.startswith("attention") else None
    roofline = {"bound": "hbm", "kernel": dom, "achieved": round(kern[dom]["gbs"], 1), "peak": hbm,
                "unit": "GB/s", "frac": round(kern[dom]["gbs"] / hbm, 4),
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
                "traffic": None, "launches_per_step": n_launch_dom,
                "algorithmic_bytes_per_launch": kern[dom]["bytes_per_step"] // (n_launch_dom or 1)}
    kv = B * C.kv_bytes_per_stream(cfg, P + K // 2)
    step_bytes = model.weight_bytes + kv
    step_frac = step_bytes / (ms_max / K / 1e3) / (hbm * 1e9)
    out = {
        "metric": "stream-frames/s", "value": round(value, 2), "unit": "stream-frames/s",
        "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(ms_max / K, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": spec["wdt"],
        "data": "synthetic (random-init N(0,0.02) weights seed 0, prompt ids seed 3+stream, noise N(0,1) seed 4)",
        "config": {"workload": spec["workload"], "streams_per_gpu": B, "frames": K, "prompt": P,
                   "d_model": cfg.d_model, "layers": cfg.num_layers, "flow_depth": tts.flow_depth,
                   "kv_dtype": cfg.kv_dtype,
                   "parallelism": f"{world} GPU(s) x {B} independent streams, no collective",
                   "l2": f"inputs larger than L2: {kv / 1e9:.2f} GB of KV read per step"},
        "e2e": {"value": round(e2e_value, 2), "unit": "stream-frames/s",
                "h2d_bytes_per_step": B * tts.latent_dim * 4 * 2,
                "d2h_bytes_per_step": B * (tts.latent_dim + 1) * 4},
        "gpu_launches": nk.value * K,
        "roofline": roofline,
        "step_roofline": {"bytes_per_step": int(step_bytes), "frac": round(step_frac, 4),
                          "unit": "of measured HBM GB/s"},
        "kernels": kern,
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline_tts(cfg, tts, weights, tokens[0], budget_s=args.cpu_seconds)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def codec_flops(cfg, part) -> int:
    """Multiply-adds x 2 of one codec frame of one stream: every convolution, the transformer's
    products and attention at its window, and (encoder) the quantizer's 32 x 2048 distances."""
    from svl import codec
    fl = 0
    fs = cfg.frame_size
    if part == codec.ENCODER:
        s, t, mult = cfg.encoder, fs, 1
        fl += 2 * s.n_filters * s.channels * s.kernel_size * t
        for r in reversed(s.ratios):
            dim = mult * s.n_filters
            fl += s.n_residual_layers * 2 * t * (dim * (dim // s.compress) * (s.residual_kernel_size + 1))
            t //= r
            fl += 2 * (2 * dim) * dim * 2 * r * t
            mult *= 2
        fl += 2 * s.dimension * mult * s.n_filters * s.last_kernel_size * t
        p = cfg.encoder_transformer
        fl += t * 2 * p.num_layers * (4 * p.d_model * p.d_model + 2 * p.d_model * p.dim_feedforward
                                      + 2 * p.d_model * p.context)
        st = cfg.resample_stride(s)
        fl += 2 * cfg.inner_dim * p.output_dimension * 2 * st * (t // st)
        fl += 2 * (2 * 256 * 512 + 32 * 2048 * 256)
    else:
        s = cfg.decoder
        st = cfg.resample_stride(s)
        fl += 2 * s.dimension * 2 * st  # depthwise up-sampling of one latent frame
        t = st
        p = cfg.decoder_transformer
        fl += t * 2 * p.num_layers * (4 * p.d_model * p.d_model + 2 * p.d_model * p.dim_feedforward
                                      + 2 * p.d_model * p.context)
        mult = 1 << len(s.ratios)
        fl += 2 * mult * s.n_filters * s.dimension * s.kernel_size * t
        for r in s.ratios:
            dim = mult * s.n_filters
            fl += 2 * dim * (dim // 2) * 2 * r * t
            t *= r
            h = dim // 2
            fl += s.n_residual_layers * 2 * t * (h * (h // s.compress) * (s.residual_kernel_size + 1))
            mult //= 2
        fl += 2 * s.channels * s.n_filters * s.last_kernel_size * t
    return int(fl)


def run_codec(args, spec, rank, world, local_rank):
    import torch
    torch.cuda.set_device(local_rank)
    dist = init_dist(world, local_rank)
    out = measure_codec(args, spec, rank, world, local_rank, dist, args.steps, args.warmup,
                        cpu=not args.no_cpu_baseline)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def measure_codec(args, spec, rank, world, local_rank, dist, K, W, cpu=True):
    """The codec on both sides of the LMs, one codec frame (80 ms) of every stream per step: the
    STT Mimi encoder followed by the quantizer (audio -> the LM's 32 audio tokens, stt/mod.rs:
    532-541), and the Pocket-TTS Mimi decoder (latents -> audio, tts/mod.rs:441-447). f32 on the
    CUDA cores; the roofline is the FP32 FMA rate (nominal: SMs x 128 lanes x 2 x max clock)."""
    import torch
    import oracle
    from svl import codec

    B = spec["batch"]
    peaks, src = load_peaks()
    props = torch.cuda.get_device_properties(local_rank)
    fp32_peak = props.multi_processor_count * 128 * 2 * peaks.get("sm_max_mhz", 1965.0) * 1e6 / 1e12
    stream = torch.cuda.Stream()
    out = {"metric": "stream-frames/s", "unit": "stream-frames/s", "n_gpus": world, "steps": K,
           "warmup": W, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "f32", "data": "synthetic (random-init weights seed 0, N(0, 0.09) audio seed 11+rank)",
           "config": {"workload": spec["workload"], "streams_per_gpu": B,
                      "inputs": "one frame per step, distinct per step; 1.1 GB of inputs per leg > L2"}}
    legs = {}
    for part, name in ((codec.ENCODER, "encoder+rvq"), (codec.DECODER, "decoder")):
        cfg = codec.stt_mimi(codec.ENCODER) if part == codec.ENCODER else codec.tts_mimi(codec.DECODER)
        w = synth.mimi_weights(cfg)
        if part == codec.ENCODER:
            w.update(synth.rvq_weights(32, 2048))
        m = codec.Mimi(cfg, w, device=local_rank)
        q = codec.Quantizer(32, 2048, w, device=local_rank) if part == codec.ENCODER else None
        st = m.init_state(B, 1)
        fs = m.frame_size
        g = torch.Generator(device="cuda").manual_seed(11 + rank)
        n_in = min(K + W, 16)
        if part == codec.ENCODER:
            ins = [0.3 * torch.randn((B, 1, fs), generator=g, device="cuda") for _ in range(n_in)]
        else:
            ins = [torch.randn((B, cfg.outer_dim, 1), generator=g, device="cuda") for _ in range(n_in)]

        def step(i):
            if part == codec.ENCODER:
                return q.encode(m.encode_step(ins[i % n_in], st, stream), stream)
            return m.decode_step(ins[i % n_in], st, stream)

        with torch.cuda.stream(stream):
            for i in range(W):
                step(i)
            stream.synchronize()
            if dist:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for i in range(K):
                step(W + i)
            e1.record(stream)
            e1.synchronize()
        ms = e0.elapsed_time(e1) / K
        ms = max_over_ranks(dist, ms, "cuda")
        # End to end: the frame from pinned host memory, the result back to the host.
        host_in = [x.cpu().pin_memory() for x in ins[:4]]
        h2d = host_in[0].numel() * 4
        with torch.cuda.stream(stream):
            res = step(0)
            d2h = res.numel() * res.element_size()
            stream.synchronize()
            t0 = time.perf_counter()
            for i in range(K):
                x = host_in[i % 4].to("cuda", non_blocking=True)
                y = (q.encode(m.encode_step(x, st, stream), stream) if part == codec.ENCODER
                     else m.decode_step(x, st, stream))
                y.cpu()
            stream.synchronize()
            e2e_ms = (time.perf_counter() - t0) * 1e3 / K
        e2e_ms = max_over_ranks(dist, e2e_ms, "cuda")
        flops = codec_flops(cfg, part) * B
        leg = {"value": round(B * world * 1e3 / ms, 1), "ms_per_step": round(ms, 4),
               "e2e": {"value": round(B * world * 1e3 / e2e_ms, 1), "unit": "stream-frames/s",
                       "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
               "roofline": {"bound": "fp32", "achieved": round(flops / (ms * 1e-3) / 1e12, 2),
                            "peak": round(fp32_peak, 1), "unit": "TFLOP/s",
                            "frac": round(flops / (ms * 1e-3) / 1e12 / fp32_peak, 4),
                            "peak_source": "nominal FP32 FMA rate (SMs x 128 x 2 x max SM clock)",
                            "flops_per_step": flops}}
        if rank == 0 and world == 1 and cpu:
            om = oracle.OracleMimi(cfg, w)
            oq = oracle.OracleQuantizer(32, 2048, w) if part == codec.ENCODER else None
            os_ = om.init_state()
            x = ins[0][0].cpu().numpy()
            n, t0 = 0, time.perf_counter()
            while time.perf_counter() - t0 < min(args.cpu_seconds, 10.0):
                if part == codec.ENCODER:
                    oq.encode(om.encode_step(x, os_))
                else:
                    om.decode_step(x, os_)
                n += 1
            v = n / (time.perf_counter() - t0)
            leg["cpu_baseline"] = {"value": round(v, 3), "unit": "stream-frames/s", "cores": os.cpu_count(),
                                   "kind": "port", "sample": f"{n} frames of one stream"}
        legs[name] = leg
        del m, q, st
    out.update(value=legs["encoder+rvq"]["value"], ms_per_step=legs["encoder+rvq"]["ms_per_step"],
               e2e=legs["encoder+rvq"]["e2e"], roofline=legs["encoder+rvq"]["roofline"],
               decoder=legs["decoder"])
    if "cpu_baseline" in legs["encoder+rvq"]:
        out["cpu_baseline"] = legs["encoder+rvq"]["cpu_baseline"]
    return out


def cpu_baseline_tts(cfg, tts, weights, prompt, budget_s=15.0, frames_cap=None):
    """The oracle's FlowLm step on the host's cores: stream 0's prompt, then frames until the
    time budget is spent."""
    import oracle as O
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    om = O.OracleModel(1, cfg, weights, tts=tts)
    st = om.init_state()
    om.prompt_text(prompt, st)
    noise = np.random.default_rng(4).standard_normal((4096, tts.latent_dim)).astype(np.float32)
    prev, n = None, 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s and (frames_cap is None or n < frames_cap) and n < 4096:
        prev, _ = om.tts_step(prev, noise[n], st)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 3), "unit": "stream-frames/s", "cores": threads, "kind": "port",
            "sample": f"{n} frames of one stream after a {len(prompt)}-token prompt ({cfg.weight_dtype} "
                      f"weights), {dt:.1f} s on {threads} threads"}


def cpu_baseline(spec, stt, cfg, weights, budget_s=15.0, frames_cap=None):
    """The oracle (a C restatement of the reference CPU path) on the host's cores: stream 0 of
    the workload from position 0, frames until the time budget is spent."""
    import oracle as O
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    om = O.OracleModel(0, cfg, weights, stt=stt)
    st = om.init_state()
    audio = synth.audio_tokens(stt, 4096, seed=1)
    prev = stt.text_card
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s and (frames_cap is None or n < frames_cap):
        a = np.full(stt.n_q, stt.card, np.uint32) if n == 0 else audio[n]
        prev, _, _ = om.stt_step(prev, a, st)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 3), "unit": "stream-frames/s", "cores": threads, "kind": "port",
            "sample": f"{n} frames of one stream from position 0 ({spec['wdt']} weights, "
                      f"{cfg.kv_dtype} KV), {dt:.1f} s on {threads} threads"}


def run_reference(args, spec, rank):
    """The reference's CPU implementation of the path: the oracle port (the Rust reference
    cannot be built in this image), all host threads, bounded samples of the workload."""
    if rank != 0:
        return
    if spec.get("kind") == "codec":
        # The STT Mimi encoder + quantizer of one stream on the oracle port, frame after frame.
        import oracle as O
        from svl import codec
        O.set_threads(os.cpu_count() or 1)
        cfg = codec.stt_mimi(codec.ENCODER)
        w = synth.mimi_weights(cfg)
        w.update(synth.rvq_weights(32, 2048))
        om, oq = O.OracleMimi(cfg, w), O.OracleQuantizer(32, 2048, w)
        st = om.init_state()
        pcm = (0.3 * np.random.default_rng(11).standard_normal((1, om.frame_size))).astype(np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < min(args.ref_seconds, 30.0) and n < args.steps + args.warmup:
            oq.encode(om.encode_step(pcm, st))
            n += 1
        value = round(n / (time.perf_counter() - t0), 3)
        cb = {"value": value, "unit": "stream-frames/s", "cores": os.cpu_count(), "kind": "port",
              "sample": f"{n} frames of one stream (C restatement of the reference CPU path)"}
        print(json.dumps({"metric": "stream-frames/s", "value": value, "unit": "stream-frames/s",
                          "n_gpus": args.gpus, "steps": n, "warmup": 0,
                          "ms_per_step": round(1e3 / max(value, 1e-9), 3), "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                          "config": {"workload": spec["workload"], "streams_per_gpu": spec["batch"]},
                          "impl": "reference", "cpu_baseline": cb,
                          "e2e": {"value": value, "unit": "stream-frames/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    if spec.get("kind") == "tts":
        cfg, tts = tts_config(spec)
        weights = synth.tts_weights(cfg, tts, seed=0)
        prompt = np.random.default_rng(3).integers(0, tts.text_bins, size=spec["prompt"], dtype=np.uint32)
        t0 = time.perf_counter()
        cb = cpu_baseline_tts(cfg, tts, weights, prompt, budget_s=args.ref_seconds,
                              frames_cap=args.steps + args.warmup)
        value = cb["value"]
        out = {"metric": "stream-frames/s", "value": value, "unit": "stream-frames/s",
               "n_gpus": args.gpus, "steps": args.steps, "warmup": 0,
               "ms_per_step": round(1e3 / max(value, 1e-9), 3), "higher_is_better": True,
               "scaling": "weak", "vs_baseline": None, "dtype": spec["wdt"], "data": "synthetic",
               "config": {"workload": spec["workload"], "streams_per_gpu": spec["batch"]},
               "impl": "reference",
               "cpu_baseline": dict(cb, sample=cb["sample"] + " (C restatement of the reference "
                                    "CPU path; the Rust reference needs cargo and candle 0.11.1)"),
               "e2e": {"value": value, "unit": "stream-frames/s", "h2d_bytes_per_step": 0,
                       "d2h_bytes_per_step": 0}}
        print(json.dumps(out), flush=True)
        return
    stt = preset(spec["preset"])
    cfg = stt.transformer(spec["wdt"], spec["kv"])
    weights = synth.stt_weights(stt, cfg, seed=0)
    import oracle as O
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    om = O.OracleModel(0, cfg, weights, stt=stt)
    del weights
    # The streams our arm runs at this N: n_gpus x streams per GPU, independent. The sample
    # steps up to 8 of them round-robin (each with its own state and audio, seed 1 + stream),
    # one frame each per step: the CPU reads every weight once per stream-frame whatever the
    # stream count, so the sample's stream-frames/s stands for all of them.
    total = args.gpus * spec["batch"]
    ns = min(total, 8)
    audio = [synth.audio_tokens(stt, args.steps + args.warmup + 1, seed=1 + s) for s in range(ns)]
    states = [om.init_state() for _ in range(ns)]
    prev = [stt.text_card] * ns

    def frame(s, i):
        a = np.full(stt.n_q, stt.card, np.uint32) if i == 0 else audio[s][i]
        prev[s], _, _ = om.stt_step(prev[s], a, states[s])

    for i in range(args.warmup):
        for s in range(ns):
            frame(s, i)
    # Each step: one frame of each sampled stream, stopping early once the time budget is spent.
    n = 0
    t0 = time.perf_counter()
    for i in range(args.steps):
        if time.perf_counter() - t0 > args.ref_seconds:
            break
        for s in range(ns):
            frame(s, args.warmup + i)
        n += 1
    dt = time.perf_counter() - t0
    value = n * ns / dt
    sample = (f"{n} frames of each of {ns} streams (of the {total} the GPU arm runs at this N) after "
              f"{args.warmup} warm-up frames, {dt:.1f} s on {threads} threads (C restatement of the "
              f"reference CPU path; the Rust reference needs cargo and candle 0.11.1, absent here)")
    out = {"metric": "stream-frames/s", "value": round(value, 3), "unit": "stream-frames/s",
           "n_gpus": args.gpus, "steps": n, "warmup": args.warmup,
           "ms_per_step": round(dt / max(n, 1) * 1e3, 3), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": spec["wdt"], "data": "synthetic",
           "config": {"workload": spec["workload"], "streams_per_gpu": spec["batch"],
                      "streams_sampled": ns},
           "impl": "reference",
           "cpu_baseline": {"value": round(value, 3), "unit": "stream-frames/s", "cores": threads,
                            "kind": "port", "sample": sample},
           "e2e": {"value": round(value, 3), "unit": "stream-frames/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", default="2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--ref-seconds", type=float, default=120.0)
    ap.add_argument("--layers", type=int, default=0,
                    help="first L layers only: a small case for profiling captures")
    ap.add_argument("--no-config3", action="store_true",
                    help="skip the config-3 block of the default (config 2) run")
    ap.add_argument("--no-codec", action="store_true",
                    help="skip the codec block of the default (config 2) run")
    args = ap.parse_args()
    spec = dict(CONFIGS[args.config], key=args.config)
    if args.steps is None:
        args.steps = spec["frames"]
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus > 1 and world == 1:
        sys.exit("--gpus N > 1 runs under torchrun: python -m torch.distributed.run "
                 "--nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N")
    if args.impl == "reference":
        run_reference(args, spec, rank)
    elif spec.get("kind") == "tts":
        run_tts(args, spec, rank, world, local_rank)
    elif spec.get("kind") == "codec":
        run_codec(args, spec, rank, world, local_rank)
    else:
        run_ours(args, spec, rank, world, local_rank)


if __name__ == "__main__":
    main()
