"""Reference-order states (svl_state_create_ex with SVL_STATE_REFERENCE_ORDER) against the CPU
oracle: bit-exact logits and tokens.

In a reference-order state every reduction whose order the reference's CPU path fixes runs in
that order (norm sums, attention, RoPE table, f32 / bf16 dot lanes); the quantised products
use the reference order in every state. The step is then the reference CPU arithmetic on the
GPU, so the north-star bars (tokens bit-exact over 256 greedy steps; logits within 2e-3
max-abs for f32, 2e-2 relative for bf16 / quantised weights) hold with equality: these tests
assert identical logits and tokens, and report the bars' margins.

The oracle is the C restatement of the reference CPU path (oracle/svl_oracle.c).
"""
import numpy as np
import pytest

import oracle as O
from svl import LanguageModel, config, synth

pytestmark = pytest.mark.gpu

CASES = [("f32", "f32"), ("q8_0", "f32"), ("q4_1", "bf16"), ("bf16", "bf16")]


def host_greedy(gm, stt, audio, frames, state):
    """The Recognizer loop through svl_stt_step: tokens and logits per step."""
    prev, toks, lgs = stt.text_card, [], []
    for i in range(frames):
        a = np.full((1, stt.n_q), stt.card, np.uint32) if i == 0 else audio[i][None]
        tok, lg = gm.step([prev], a, state, logits=True)
        toks.append(int(tok[0]))
        lgs.append(lg[0])
        prev = int(tok[0])
    return np.array(toks, np.uint32), np.stack(lgs)


def assert_exact(toks, lgs, ref_tok, ref_lg, label):
    same = int(np.sum(toks == ref_tok))
    first = int(np.argmax(toks != ref_tok)) if same < len(ref_tok) else None
    diff = float(np.max(np.abs(lgs - ref_lg)))
    print(f"{label}: {same}/{len(ref_tok)} free-running tokens equal (first difference: {first}), "
          f"max |logit diff| {diff:.3g}")
    np.testing.assert_array_equal(toks, ref_tok)
    np.testing.assert_array_equal(lgs, ref_lg)


@pytest.mark.parametrize("wdt,kvdt", CASES)
def test_toy_reference_order_bit_exact(svl_lib, oracle_lib, wdt, kvdt):
    """64 free-running steps (the window-12 ring wraps five times): identical logits and
    tokens, through the host-buffer step and through the device token loop."""
    stt = config.stt_toy(extra_heads_num_heads=2, extra_heads_dim=6)
    cfg = stt.transformer(wdt, kvdt)
    w = synth.stt_weights(stt, cfg)
    frames = 64
    audio = synth.audio_tokens(stt, frames)
    om = O.OracleModel(0, cfg, w, stt=stt)
    ref_tok, ref_lg = O.greedy_stt(om, audio, frames)
    gm = LanguageModel(stt, cfg, w)
    toks, lgs = host_greedy(gm, stt, audio, frames, gm.init_state(1, reference_order=True))
    assert_exact(toks, lgs, ref_tok, ref_lg, f"toy {wdt}/{kvdt}")
    st = gm.init_state(1, reference_order=True)
    np.testing.assert_array_equal(gm.run_frames(audio[:, None, :], st)[:, 0], ref_tok)


@pytest.mark.parametrize("wdt,kvdt", [("q8_0", "f32"), ("f32", "f32"), ("q4_1", "bf16")])
def test_reference_order_batched_staggered(svl_lib, oracle_lib, wdt, kvdt):
    """Seven streams at different positions in one batch (the multi-stream templates of the
    matrix-vector kernels): each stream equals its own oracle run bit for bit."""
    stt = config.stt_toy()
    cfg = stt.transformer(wdt, kvdt)
    w = synth.stt_weights(stt, cfg)
    om = O.OracleModel(0, cfg, w, stt=stt)
    gm = LanguageModel(stt, cfg, w)
    B, frames = 7, 20
    offsets = [0, 1, 5, 11, 12, 13, 30]
    audio = synth.audio_tokens(stt, max(offsets) + frames, seed=1, streams=B)
    big = gm.init_state(B, reference_order=True)
    refs = []
    for b in range(B):
        one = gm.init_state(1, reference_order=True)
        if offsets[b]:
            gm.run_frames(audio[: offsets[b], b][:, None, :], one)
        big.copy_from(one, 0, b)
        toks, _ = O.greedy_stt(om, audio[:, b], offsets[b] + frames)
        refs.append(toks)
    got = gm.run_frames(np.stack([audio[offsets[b]: offsets[b] + frames, b] for b in range(B)], 1), big)
    for b in range(B):
        np.testing.assert_array_equal(got[:, b], refs[b][offsets[b]:], err_msg=f"stream {b}")


@pytest.mark.slow
@pytest.mark.parametrize("wdt", ["q8_0", "f32"])
def test_stt_1b_reference_order_256_steps(svl_lib, oracle_lib, wdt):
    """BASELINE configs 2 (q8_0) and 1 (f32): STT-1b, batch 1, 256 free-running greedy steps.
    tokens bit-exact over 256 steps, logits within 2e-2 relative (q8_0) /
    2e-3 max-abs (f32). Reference order meets them with identical logits."""
    stt = config.stt_1b()
    cfg = stt.transformer(wdt, "f32")
    w = synth.stt_weights(stt, cfg)
    frames = 256
    audio = synth.audio_tokens(stt, frames)
    om = O.OracleModel(0, cfg, w, stt=stt)
    ref_tok, ref_lg = O.greedy_stt(om, audio, frames)
    del om
    gm = LanguageModel(stt, cfg, w)
    del w
    toks, lgs = host_greedy(gm, stt, audio, frames, gm.init_state(1, reference_order=True))
    rel = np.linalg.norm(lgs - ref_lg, axis=1) / np.linalg.norm(ref_lg, axis=1)
    print(f"STT-1b {wdt} reference order: max L2-relative logit difference {rel.max():.3g} "
          f"(bar 2e-2)")
    assert_exact(toks, lgs, ref_tok, ref_lg, f"STT-1b {wdt} reference order")


@pytest.mark.slow
def test_stt_2b6_q4_1_reference_order_256_steps(svl_lib, oracle_lib):
    """BASELINE config 4 at batch 1: STT-2.6b, q4_1 weights, bf16 KV (window 375), 256
    free-running greedy steps, bit-exact."""
    stt = config.stt_2b6()
    cfg = stt.transformer("q4_1", "bf16")
    w = synth.stt_weights(stt, cfg)
    frames = 256
    audio = synth.audio_tokens(stt, frames)
    om = O.OracleModel(0, cfg, w, stt=stt)
    ref_tok, ref_lg = O.greedy_stt(om, audio, frames)
    del om
    gm = LanguageModel(stt, cfg, w)
    del w
    toks, lgs = host_greedy(gm, stt, audio, frames, gm.init_state(1, reference_order=True))
    assert_exact(toks, lgs, ref_tok, ref_lg, "STT-2.6b q4_1 reference order")
