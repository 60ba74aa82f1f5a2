"""Small cases of the BASELINE workloads for ncu captures.

A full-size workload holds up to tens of GB on the device and runs thousands of launches,
too large for a many-pass ncu capture. This driver builds the same shapes with fewer layers
(synthetic seed-0 weights, the workload's stream count, streams at a full attention window)
and runs the step's kernel families through svl_profile_kernels:

    PYTHONPATH=semantic-ai_b200 python -m svl.profile_case --config 3 --layers 2 --passes 3

--which products: the weight products of every layer and the head (with their operand
preparation); attention: the attention of every layer; both (default): products, then
attention. It prints the time per pass of each family (CUDA events on the launching stream).
The numbers are for profiling only: the step throughput is bench.py's.
"""
from __future__ import annotations

import argparse
import ctypes
import dataclasses

from . import _lib, config, synth
from .model import LanguageModel

CASES = {
    "1": ("stt_1b", "f32", "f32", 1),
    "2": ("stt_1b", "q8_0", "f32", 1),
    "3": ("stt_1b", "bf16", "bf16", 256),
    "4": ("stt_2b6", "q4_1", "bf16", 1),
    "4b": ("stt_2b6", "q4_1", "bf16", 128),
}


def main(argv=None):
    import torch

    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="2", choices=sorted(CASES))
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--passes", type=int, default=3)
    ap.add_argument("--which", default="both", choices=["products", "attention", "both"])
    args = ap.parse_args(argv)
    preset, wdt, kv, batch = CASES[args.config]
    stt = dataclasses.replace(getattr(config, preset)(), num_layers=args.layers)
    cfg = stt.transformer(wdt, kv)
    model = LanguageModel(stt, cfg, synth.stt_weights(stt, cfg))
    state = model.init_state(batch)
    lib = _lib.lib()
    for b in range(batch):  # every stream at a full window
        _lib.check(lib.svl_state_import(state.handle, b, 0, None, None, 0, cfg.context or 1))
    stream = torch.cuda.Stream()
    sp = ctypes.c_void_p(stream.cuda_stream)
    nbytes = ctypes.c_int64()
    fams = {"products": [0], "attention": [1], "both": [0, 1]}[args.which]
    for which in fams:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        _lib.check(lib.svl_profile_kernels(model.handle, state.handle, batch, which, args.passes,
                                           sp, ctypes.byref(nbytes)))
        e1.record(stream)
        stream.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / args.passes
        name = "products" if which == 0 else "attention"
        print(f"config {args.config} ({args.layers} layers, {batch} streams) {name}: "
              f"{us:.1f} us per pass, {nbytes.value / 1e6:.1f} MB, "
              f"{nbytes.value / us / 1e3:.1f} GB/s", flush=True)


if __name__ == "__main__":
    main()
