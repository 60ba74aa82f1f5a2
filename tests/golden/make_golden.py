"""Golden fixtures of the CPU oracle: `python tests/golden/make_golden.py` rewrites them.

The reference ships no golden vectors for the LM step (its parity fixtures are generated
outside the repository), so these pin the oracle itself: once the oracle is held to the
reference's unit-test bounds and the float64 restatement (tests/test_oracle.py), any later
change to it must reproduce these outputs bit for bit or regenerate them deliberately.
Seeded synthetic inputs only (N(0, 0.02) weights from seed 0, uniform tokens from seed 1).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path[:0] = [str(ROOT / "semantic-ai_b200"), str(ROOT / "oracle")]

import oracle as O  # noqa: E402
from svl import config, synth  # noqa: E402


def _stt(wdt: str, kvdt: str, frames: int = 12) -> dict[str, np.ndarray]:
    stt = config.stt_toy(extra_heads_num_heads=2, extra_heads_dim=6)
    cfg = stt.transformer(wdt, kvdt)
    om = O.OracleModel(0, cfg, synth.stt_weights(stt, cfg), stt=stt)
    toks, lg = O.greedy_stt(om, synth.audio_tokens(stt, frames), frames)
    return {"tokens": np.asarray(toks, np.uint32), "logits": np.asarray(lg, np.float32)}


def _tts(kind: str) -> dict[str, np.ndarray]:
    cfg, tts = config.tts_toy(kind)
    om = O.OracleModel(1, cfg, synth.tts_weights(cfg, tts), tts=tts)
    st = om.init_state()
    om.prompt_text(np.array([3, 1, 4, 1, 5], np.uint32), st)
    noise = np.random.default_rng(4).standard_normal((3, tts.latent_dim)).astype(np.float32)
    lat, lats, eos = None, [], []
    for i in range(3):
        lat, e = om.tts_step(lat, noise[i], st)
        lats.append(lat)
        eos.append(e)
    return {"latents": np.stack(lats).astype(np.float32), "eos": np.array(eos, np.float32)}


CASES = {
    "stt_toy_f32": lambda: _stt("f32", "f32"),
    "stt_toy_q8_0": lambda: _stt("q8_0", "f32"),
    "stt_toy_q4_1": lambda: _stt("q4_1", "bf16"),
    "stt_toy_bf16": lambda: _stt("bf16", "bf16"),
    "tts_toy_lsd": lambda: _tts("lsd"),
    "tts_toy_pointwise": lambda: _tts("pointwise"),
}

if __name__ == "__main__":
    O.set_threads(1)
    for name, make in CASES.items():
        np.savez(HERE / f"{name}.npz", **make())
        print("wrote", name)
