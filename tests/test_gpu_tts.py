"""GPU parity of the Pocket-TTS FlowLm step (tts/flow_lm.rs:150-387) against the CPU oracle.

The step: input_linear on the previous latent (BOS first), the streaming transformer
(LayerNorm, GELU-tanh FFN, no window), out_norm + out_eos, then the flow head (cond_embed,
timestep embeddings, residual AdaLN blocks, final layer) applied to the noise. The latents
are fed back from the oracle (teacher forcing), so every step compares one step's arithmetic.

Bars (north star): f32 weights within 2e-3 max-abs; bf16 weights within 2e-2 relative
(||diff||_2 / ||oracle||_2). The latent out is noise + flow, so the flow part (out - noise)
is what the relative bar is applied to.
"""
import numpy as np
import pytest

import oracle as O
from svl import FlowLm, config, synth
from svl._lib import SvlError

pytestmark = pytest.mark.gpu

F32_TOL = 2e-3
REL_TOL = 2e-2


def run(kind="lsd", wdt="f32", B=1, steps=6, decode_steps=1, prompt=5):
    cfg, tts = config.tts_toy(kind, wdt, "bf16" if wdt == "bf16" else "f32")
    w = synth.tts_weights(cfg, tts)
    om = O.OracleModel(1, cfg, w, tts=tts)
    gm = FlowLm(cfg, tts, w)
    rng = np.random.default_rng(3)
    tokens = rng.integers(0, tts.text_bins + 1, size=(B, prompt), dtype=np.uint32)
    noise = np.random.default_rng(4).standard_normal((steps, B, tts.latent_dim)).astype(np.float32)
    osts = []
    for b in range(B):
        st = om.init_state()
        om.prompt_text(tokens[b], st)
        osts.append(st)
    gst = gm.init_state(B, max_positions=prompt + steps + 2)
    gm.prompt_text_batch(tokens, gst)
    worst_flow, worst_eos = 0.0, 0.0
    latent = None
    for i in range(steps):
        ref = [om.tts_step(None if latent is None else latent[b], noise[i, b], osts[b], decode_steps)
               for b in range(B)]
        ref_lat = np.stack([r[0] for r in ref])
        ref_eos = np.array([r[1] for r in ref], np.float32)
        got_lat, got_eos = gm.step(latent, noise[i], gst, decode_steps)
        if wdt == "f32":
            d_lat = float(np.max(np.abs(got_lat - ref_lat)))
            d_eos = float(np.max(np.abs(got_eos - ref_eos)))
            assert d_lat <= F32_TOL and d_eos <= F32_TOL, f"step {i}: latent {d_lat:.3g}, eos {d_eos:.3g}"
        else:
            fl_got, fl_ref = got_lat - noise[i], ref_lat - noise[i]
            if kind == "drifting":
                fl_got, fl_ref = got_lat, ref_lat
            d_lat = float(np.linalg.norm(fl_got - fl_ref) / np.linalg.norm(fl_ref))
            d_eos = float(np.linalg.norm(got_eos - ref_eos) / max(np.linalg.norm(ref_eos), 1e-6))
            assert d_lat <= REL_TOL and d_eos <= REL_TOL, f"step {i}: flow {d_lat:.3g}, eos {d_eos:.3g}"
        worst_flow, worst_eos = max(worst_flow, d_lat), max(worst_eos, d_eos)
        latent = ref_lat  # teacher forcing
    for b in range(B):
        assert gst.position(b) == prompt + steps
    return worst_flow, worst_eos


@pytest.mark.parametrize("kind", ["lsd", "flow_matching", "pointwise", "drifting"])
def test_toy_tts_f32(svl_lib, oracle_lib, kind):
    wl, we = run(kind=kind)
    print(f"tts f32 {kind}: latent {wl:.3g}, eos {we:.3g}")


def test_toy_tts_f32_two_decode_steps(svl_lib, oracle_lib):
    wl, we = run(decode_steps=2)
    print(f"tts f32 lsd x2: latent {wl:.3g}, eos {we:.3g}")


@pytest.mark.parametrize("B", [1, 3, 20, 130])
def test_toy_tts_bf16(svl_lib, oracle_lib, B):
    """B >= 16: the weight products run on the tensor cores."""
    wl, we = run(wdt="bf16", B=B, steps=4)
    print(f"tts bf16 B={B}: flow rel {wl:.3g}, eos rel {we:.3g}")


def test_prompt_batch_equals_per_stream(svl_lib):
    cfg, tts = config.tts_toy()
    w = synth.tts_weights(cfg, tts)
    gm = FlowLm(cfg, tts, w)
    tokens = np.random.default_rng(5).integers(0, tts.text_bins, size=(3, 4), dtype=np.uint32)
    noise = np.random.default_rng(6).standard_normal((3, tts.latent_dim)).astype(np.float32)
    a = gm.init_state(3, max_positions=8)
    gm.prompt_text_batch(tokens, a)
    b = gm.init_state(3, max_positions=8)
    for s in range(3):
        gm.prompt_text(tokens[s], b, stream=s)
    la, ea = gm.step(None, noise, a)
    lb, eb = gm.step(None, noise, b)
    np.testing.assert_array_equal(la, lb)
    np.testing.assert_array_equal(ea, eb)


def test_tts_rejects_bad_input(svl_lib):
    cfg, tts = config.tts_toy()
    gm = FlowLm(cfg, tts, synth.tts_weights(cfg, tts))
    st = gm.init_state(1, max_positions=4)
    with pytest.raises(SvlError):
        gm.prompt_text([tts.text_bins + 1], st)
    with pytest.raises(SvlError):
        gm.prompt_text([1, 2, 3, 4, 5], st)  # beyond max_positions
    gm.prompt_text([1, 2, 3], st)
    noise = np.zeros((1, tts.latent_dim), np.float32)
    gm.step(None, noise, st)
    with pytest.raises(SvlError):
        gm.step(None, noise, st)  # position 4 of 4
