"""The persistent batch-1 step kernel (stepk.cu) against the separate-kernel path and the
oracle.

A one-stream state runs the whole step as one persistent kernel; SVL_STEP_KERNEL=0 (read
when a state is created) runs the same step as separate kernels (the multi-stream path).
Both are checked against each other on identical inputs, teacher-forced, and the persistent
path against the oracle with the north-star bars (f32 2e-3 max-abs, quantised / bf16 2e-2
relative with margin-aware argmax).
"""
import os

import numpy as np
import pytest

import oracle as O
from svl import LanguageModel, config, synth

pytestmark = pytest.mark.gpu


def make_state(gm, split):
    old = os.environ.get("SVL_STEP_KERNEL")
    os.environ["SVL_STEP_KERNEL"] = "0" if split else "1"
    try:
        return gm.init_state(1)
    finally:
        if old is None:
            del os.environ["SVL_STEP_KERNEL"]
        else:
            os.environ["SVL_STEP_KERNEL"] = old


def mid(**kw):
    return config.stt_toy(dim=1024, num_heads=8, num_layers=3, context=40, text_card=1000,
                          card=64, n_q=4, **kw)


@pytest.mark.parametrize("shape,wdt,kvdt", [("toy", "f32", "f32"), ("toy", "q8_0", "f32"),
                                            ("toy", "q4_1", "bf16"), ("toy", "bf16", "bf16"),
                                            ("mid", "f32", "f32"), ("mid", "q8_0", "f32")])
def test_step_kernel_matches_split_path_and_oracle(svl_lib, oracle_lib, shape, wdt, kvdt):
    stt = config.stt_toy() if shape == "toy" else mid()
    cfg = stt.transformer(wdt, kvdt)
    w = synth.stt_weights(stt, cfg)
    frames = 50 if shape == "toy" else 48  # past the window: the ring wraps
    audio = synth.audio_tokens(stt, frames)
    om = O.OracleModel(0, cfg, w, stt=stt)
    ref_tok, ref_lg = O.greedy_stt(om, audio, frames)
    gm = LanguageModel(stt, cfg, w)
    sk, sp = make_state(gm, False), make_state(gm, True)
    prev = stt.text_card
    worst_split, worst_ref = 0.0, 0.0
    for i in range(frames):
        a = np.full((1, stt.n_q), stt.card, np.uint32) if i == 0 else audio[i][None]
        tk, lk = gm.step([prev], a, sk, logits=True)
        ts, ls = gm.step([prev], a, sp, logits=True)
        if wdt == "f32":
            d_split = float(np.max(np.abs(lk[0] - ls[0])))
            d_ref = float(np.max(np.abs(lk[0] - ref_lg[i])))
            assert d_ref <= 2e-3, f"step {i}: {d_ref} from the oracle"
            assert tk[0] == ref_tok[i]
        else:
            d_split = float(np.linalg.norm(lk[0] - ls[0]) / np.linalg.norm(ls[0]))
            d_ref = float(np.linalg.norm(lk[0] - ref_lg[i]) / np.linalg.norm(ref_lg[i]))
            assert d_ref <= 2e-2, f"step {i}: {d_ref} relative from the oracle"
            if tk[0] != ref_tok[i]:
                s = np.sort(ref_lg[i])
                assert s[-1] - s[-2] <= 2 * float(np.max(np.abs(lk[0] - ref_lg[i])))
        worst_split, worst_ref = max(worst_split, d_split), max(worst_ref, d_ref)
        prev = int(ref_tok[i])
    assert sk.position() == frames and sp.position() == frames
    print(f"{shape} {wdt}: step kernel vs split path {worst_split:.3g}, vs oracle {worst_ref:.3g}")


def test_step_kernel_device_loop_deterministic(svl_lib):
    stt = mid()
    cfg = stt.transformer("q8_0", "f32")
    gm = LanguageModel(stt, cfg, synth.stt_weights(stt, cfg))
    audio = synth.audio_tokens(stt, 60, seed=5)
    a = gm.run_frames(audio, make_state(gm, False))
    b = gm.run_frames(audio, make_state(gm, False))
    np.testing.assert_array_equal(a, b)
