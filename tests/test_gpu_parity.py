"""GPU parity: the CUDA step (through the C ABI) against the CPU oracle on identical seeded
inputs and random-init weights.

Bars (north star): logits within 2e-3 max-abs for f32 weights and within 2e-2 relative
(||diff||_2 / ||oracle||_2 per step) for bf16 and quantised weights; f32 token ids bit-exact
over the greedy steps (free-running and teacher-forced). For bf16 / quantised weights see
teacher_forced() for the token rule.
"""
import numpy as np
import pytest

import oracle as O
from svl import LanguageModel, config, synth
from svl._lib import SvlError

pytestmark = pytest.mark.gpu

F32_TOL = 2e-3
REL_TOL = 2e-2


def logits_ok(got, ref, wdt):
    """f32: max |diff| <= 2e-3. bf16 / quantised: ||diff||_2 / ||ref||_2 <= 2e-2."""
    diff = float(np.max(np.abs(got - ref)))
    if wdt == "f32":
        return diff <= F32_TOL, diff
    rel = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
    return rel <= REL_TOL, diff


def margin(lg):
    s = np.sort(lg)
    return float(s[-1] - s[-2])


def teacher_forced(gm, om_tokens, om_logits, stt, audio, wdt, state=None, stream=0):
    """Feeds the oracle's tokens to the GPU step and compares argmax and logits per step.

    f32: every argmax equals the oracle's. bf16 / quantised weights: the activation rounding
    (bf16, Q8_0 / Q8_1 blocks) is discontinuous, so a 1-ulp difference in any f32 reduction
    order flips some rounded activations and the flips propagate; an argmax may then differ
    only where the oracle's top-2 margin is within twice that step's max logit deviation.
    Returns (worst max-abs logit diff, steps with the same argmax)."""
    st = state or gm.init_state(1)
    prev = stt.text_card
    worst, same = 0.0, 0
    for i in range(len(om_tokens)):
        a = np.full((1, stt.n_q), stt.card, np.uint32) if i == 0 else audio[i][None]
        tok, lg = gm.step([prev], a, st, logits=True)
        ok, diff = logits_ok(lg[0], om_logits[i], wdt)
        worst = max(worst, diff)
        assert ok, f"step {i}: logits differ by {diff} (max abs)"
        if tok[0] == om_tokens[i]:
            same += 1
        else:
            assert wdt != "f32" and margin(om_logits[i]) <= 2 * diff, (
                f"step {i}: token {tok[0]} != oracle {om_tokens[i]} (oracle top-2 margin "
                f"{margin(om_logits[i]):.3g}, logit diff {diff:.3g})")
        prev = int(om_tokens[i])
    return worst, same


CASES = [("f32", "f32"), ("q8_0", "f32"), ("q4_1", "bf16"), ("bf16", "bf16")]


@pytest.mark.parametrize("wdt,kvdt", CASES)
def test_toy_stt_greedy(svl_lib, oracle_lib, wdt, kvdt):
    stt = config.stt_toy(extra_heads_num_heads=2, extra_heads_dim=6)
    cfg = stt.transformer(wdt, kvdt)
    w = synth.stt_weights(stt, cfg)
    frames = 64  # window 12: the ring wraps five times
    audio = synth.audio_tokens(stt, frames)
    om = O.OracleModel(0, cfg, w, stt=stt)
    ref_tok, ref_lg = O.greedy_stt(om, audio, frames)
    gm = LanguageModel(stt, cfg, w)
    worst, same = teacher_forced(gm, ref_tok, ref_lg, stt, audio, wdt)
    print(f"toy {wdt}: worst logit diff {worst:.3g}, {same}/{frames} teacher-forced argmax equal")
    # The device-side token loop (Recognizer::step) equals the host-driven free-running loop
    # exactly (the GPU path is deterministic), and for f32 the oracle's free-running tokens.
    st = gm.init_state(1)
    toks = gm.run_frames(audio[:, None, :], st)[:, 0]
    assert st.position() == frames
    st2 = gm.init_state(1)
    prev, host = stt.text_card, []
    for i in range(frames):
        a = np.full((1, stt.n_q), stt.card, np.uint32) if i == 0 else audio[i][None]
        prev = int(gm.step([prev], a, st2)[0])
        host.append(prev)
    np.testing.assert_array_equal(toks, host)
    if wdt == "f32":
        np.testing.assert_array_equal(toks, ref_tok)


def test_toy_extra_heads(svl_lib, oracle_lib):
    stt = config.stt_toy(extra_heads_num_heads=3, extra_heads_dim=6)
    cfg = stt.transformer("f32")
    w = synth.stt_weights(stt, cfg)
    om = O.OracleModel(0, cfg, w, stt=stt)
    gm = LanguageModel(stt, cfg, w)
    audio = synth.audio_tokens(stt, 8)
    ost, gst = om.init_state(), gm.init_state(1)
    prev = stt.text_card
    for i in range(8):
        tok, _, ex = om.stt_step(prev, audio[i], ost)
        gtok, gex = gm.step([prev], audio[i][None], gst, extra=True)
        assert gtok[0] == tok
        np.testing.assert_allclose(gex[0], ex, atol=1e-5)
        prev = tok


def test_toy_multi_stream_staggered(svl_lib, oracle_lib):
    """Independent streams at different fill levels in one batch equal their own runs."""
    stt = config.stt_toy()
    cfg = stt.transformer("f32")
    w = synth.stt_weights(stt, cfg)
    om = O.OracleModel(0, cfg, w, stt=stt)
    gm = LanguageModel(stt, cfg, w)
    B, frames = 5, 24
    offsets = [0, 3, 11, 12, 17]
    audio = synth.audio_tokens(stt, max(offsets) + frames, seed=1, streams=B)
    big = gm.init_state(B)
    refs = []
    for b in range(B):
        # Pre-roll stream b alone, then move its state into slot b of the batch state.
        one = gm.init_state(1)
        pre = gm.run_frames(audio[: offsets[b], b][:, None, :], one)[:, 0] if offsets[b] else []
        big.copy_from(one, 0, b)
        st = om.init_state()
        toks, _ = O.greedy_stt(om, audio[:, b], offsets[b] + frames, state=st)
        if offsets[b]:
            np.testing.assert_array_equal(pre, toks[: offsets[b]])
        refs.append(toks)
    # The batch continues every stream from its own position; text token = its last argmax.
    got = gm.run_frames(np.stack([audio[offsets[b]: offsets[b] + frames, b] for b in range(B)], 1), big)
    for b in range(B):
        np.testing.assert_array_equal(got[:, b], refs[b][offsets[b]:], err_msg=f"stream {b}")
        assert big.position(b) == offsets[b] + frames


def test_streaming_matches_full_sequence(svl_lib, oracle_lib):
    """nn/transformer.rs:598-628 on the GPU path: chunked prefill (1,3,1,7,1,1,9) equals the
    oracle's full-sequence pass, for a LayerNorm / GELU / layer-scale / GQA backbone with and
    without a window."""
    for context in (None, 5):
        cfg = config.TransformerConfig(
            d_model=128, num_layers=2, num_heads=4, num_kv_heads=2, head_dim=64,
            ffn_kind=config.FFN_PLAIN_GELU_TANH, ffn_hidden=256, norm_kind=config.NORM_LAYER,
            norm_eps=1e-5, layer_scale=True, context=context, max_period=10_000.0)
        specs = synth.transformer_specs(cfg)
        w = synth.materialize(specs, seed=0, std=0.3)
        # Oracle model needs the STT wrapper tensors too; build a tiny STT around the backbone.
        stt = config.SttConfig(card=8, n_q=1, dim=128, text_card=8, num_heads=4, num_layers=2,
                               hidden_scale=1.0, context=context or 0, max_period=10_000.0)
        extra = {"text_emb.weight": np.zeros((9, 128), np.float32),
                 "emb.0.weight": np.zeros((9, 128), np.float32),
                 "out_norm.alpha": np.ones((1, 1, 128), np.float32),
                 "text_linear.weight": np.zeros((8, 128), np.float32)}
        w.update(extra)
        om = O.OracleModel(0, cfg, w, stt=stt)
        gm = LanguageModel(stt, cfg, w)
        xs = np.random.default_rng(5).standard_normal((23, 128)).astype(np.float32)
        full = om.forward(xs, om.init_state())
        st = gm.init_state(1, max_positions=64)
        chunks, start = [], 0
        for n in (1, 3, 1, 7, 1, 1, 9):
            chunks.append(gm.forward(xs[start:start + n], st))
            start += n
        got = np.concatenate(chunks)
        # The reference's own bound is 1e-4 on a d=16 model; here d=128 with values up to ~20,
        # so the bound is taken relative to the output scale.
        err = np.max(np.abs(got - full))
        assert err <= 2e-5 * max(1.0, float(np.max(np.abs(full)))), err


def test_state_export_import_roundtrip(svl_lib, oracle_lib):
    stt = config.stt_toy()
    cfg = stt.transformer("f32")
    w = synth.stt_weights(stt, cfg)
    gm = LanguageModel(stt, cfg, w)
    audio = synth.audio_tokens(stt, 40)
    a = gm.init_state(1)
    gm.run_frames(audio[:20, None, :], a)
    caches = a.layer_caches()
    assert caches[0][0].shape == (cfg.num_kv_heads, cfg.context, cfg.head_dim)
    b = gm.init_state(1)
    b.load_layer_caches(caches, position=20)
    # Both continue from the same text token (the last argmax of `a`).
    last = gm.run_frames(audio[20:21, None, :], a)
    t = gm.step(last[0], audio[21][None], a)
    t2 = gm.step(last[0], audio[21][None], b)
    assert t[0] == t2[0]


def test_invalid_tokens_rejected(svl_lib):
    stt = config.stt_toy()
    cfg = stt.transformer("f32")
    gm = LanguageModel(stt, cfg, synth.stt_weights(stt, cfg))
    st = gm.init_state(1)
    with pytest.raises(SvlError) as e:
        gm.step([stt.text_card + 1], np.zeros((1, stt.n_q), np.uint32), st)
    assert e.value.kind == "INVALID_INPUT"
    with pytest.raises(SvlError) as e:
        gm.step([0], np.full((1, stt.n_q), stt.card + 1, np.uint32), st)
    assert e.value.kind == "INVALID_INPUT"
    assert st.position() == 0
    with pytest.raises(SvlError) as e:
        gm.init_state(0)
    assert e.value.kind == "INVALID_INPUT"


def test_bad_weights_rejected(svl_lib):
    stt = config.stt_toy()
    cfg = stt.transformer("f32")
    w = synth.stt_weights(stt, cfg)
    w["text_linear.weight"] = w["text_linear.weight"][:5]
    with pytest.raises(SvlError) as e:
        LanguageModel(stt, cfg, w)
    assert e.value.kind == "CONFIG"
    del w["text_linear.weight"]
    with pytest.raises(SvlError) as e:
        LanguageModel(stt, cfg, w)
    assert e.value.kind == "CONFIG"


@pytest.mark.slow
@pytest.mark.parametrize("wdt", ["f32", "q8_0"])
def test_stt_1b_256_greedy_steps(svl_lib, oracle_lib, wdt):
    """Configs 1 and 2 in a fast (default) state: STT-1b, batch 1, 256 greedy steps.

    f32: tokens bit-exact (teacher-forced and free-running), logits within 2e-3.
    q8_0: the north-star bars (256/256 tokens, 2e-2 relative logits) are asserted with
    equality on reference-order states (test_gpu_reference_order.py). A fast state sums its
    norms and softmax in parallel and evaluates RoPE with the device's sincosf; the Q8_0
    activation rounding turns those last-bit differences into different activation blocks,
    and the random-init network carries them through 16 layers. This test reports how far the
    fast state lands from the reference (free-running token agreement, first flip, L2-relative
    logit deviation) and bounds it by the oracle's own sensitivity: the oracle against itself
    with the RMS-norm sum reversed, teacher-forced on the same tokens."""
    stt = config.stt_1b()
    cfg = stt.transformer(wdt, "f32")
    w = synth.stt_weights(stt, cfg)
    frames = 256
    audio = synth.audio_tokens(stt, frames)
    om = O.OracleModel(0, cfg, w, stt=stt)
    ref_tok, ref_lg = O.greedy_stt(om, audio, frames)
    env = None
    if wdt != "f32":
        oracle_lib.orc_set_reduction_variant(1)
        try:
            alt_tok, alt_lg = O.greedy_stt(om, audio, frames, teacher=ref_tok)
        finally:
            oracle_lib.orc_set_reduction_variant(0)
        env = np.array([np.linalg.norm(a - r) / np.linalg.norm(r) for a, r in zip(alt_lg, ref_lg)])
        env_same = int(np.sum(alt_tok == ref_tok))
    del om
    gm = LanguageModel(stt, cfg, w)
    del w
    st = gm.init_state(1)
    free = gm.run_frames(audio[:, None, :], st)[:, 0]
    n_free = int(np.sum(free == ref_tok))
    first = int(np.argmax(free != ref_tok)) if n_free < frames else None
    if wdt == "f32":
        worst, same = teacher_forced(gm, ref_tok, ref_lg, stt, audio, wdt)
        np.testing.assert_array_equal(free, ref_tok)
        print(f"STT-1b f32 fast state: worst logit diff {worst:.3g}, {same}/{frames} argmax equal, "
              f"free-running tokens equal for all {frames} steps")
        return
    st = gm.init_state(1)
    prev, rel, same = stt.text_card, [], 0
    for i in range(frames):
        a = np.full((1, stt.n_q), stt.card, np.uint32) if i == 0 else audio[i][None]
        tok, lg = gm.step([prev], a, st, logits=True)
        rel.append(float(np.linalg.norm(lg[0] - ref_lg[i]) / np.linalg.norm(ref_lg[i])))
        same += int(tok[0] == ref_tok[i])
        prev = int(ref_tok[i])
    rel = np.array(rel)
    print(f"STT-1b {wdt} fast state: free-running {n_free}/{frames} tokens equal (first flip at "
          f"step {first}); teacher-forced L2-relative logit deviation median {np.median(rel):.3g} "
          f"max {rel.max():.3g} (north-star bar 2e-2), argmax equal {same}/{frames}; oracle "
          f"self-envelope median {np.median(env):.3g} max {env.max():.3g}, argmax equal "
          f"{env_same}/{frames}")
    assert np.median(rel) <= 2 * np.median(env) + 1e-3
    assert rel.max() <= 2 * env.max() + 1e-3
    assert same >= env_same - frames // 20
