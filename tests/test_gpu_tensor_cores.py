"""The many-streams path: with bf16 weights and at least 16 streams in a step, every weight
product runs on the tcgen05 tensor cores (gemm.cu) instead of the matrix-vector kernel.

Each stream of the batch is checked against the CPU oracle run on that stream alone,
teacher-forced with the oracle's tokens, at the bf16 bar of the north star: logits within
2e-2 relative (||diff||_2 / ||oracle||_2) per stream and step, and an argmax that may differ
from the oracle's only where the oracle's top-2 margin is within twice the logit deviation.

Q8_0 / Q4_1 models run the same kernel on f16 images of their dequantised weights.

The shapes cover the kernel's variants: one to three 128-stream tiles (16 to 260 streams), K
split over thread-block clusters of up to 8 CTAs (the mid-size model's out_proj and
linear_out), ring wrap-around, and staggered stream positions.
"""
import numpy as np
import pytest

import oracle as O
from svl import LanguageModel, config, synth

pytestmark = pytest.mark.gpu

REL_TOL = 2e-2


def mid_model():
    """d 1024, 8 heads x 128, SwiGLU 2816, 2 layers, window 16: out_proj and linear_out have
    8 row tiles, so their K is split over clusters (2 CTAs at 64 streams, 8 at 256)."""
    return config.stt_toy(dim=1024, num_heads=8, num_layers=2, context=16, text_card=1000,
                          card=64, n_q=4)


def run_batch(stt, B, frames, stagger=0, wdt="bf16", kvdt="bf16", strict=True, envelope=None):
    """B streams step together for `frames` frames; stream b first runs b % (stagger + 1)
    frames alone (matrix-vector path, one stream) and is copied into the batch state, so the
    streams sit at different positions. Returns (worst relative diff, argmax flips)."""
    cfg = stt.transformer(wdt, kvdt)
    w = synth.stt_weights(stt, cfg)
    om = O.OracleModel(0, cfg, w, stt=stt)
    gm = LanguageModel(stt, cfg, w)
    offsets = [b % (stagger + 1) for b in range(B)]
    audio = synth.audio_tokens(stt, max(offsets) + frames, seed=1, streams=B)
    initial = np.full(stt.n_q, stt.card, np.uint32)

    def audio_at(b, i):
        return initial if i == 0 else audio[i, b]

    # Oracle: each stream alone from position 0, free-running greedy.
    refs = [O.greedy_stt(om, audio[:, b], offsets[b] + frames) for b in range(B)]
    st = gm.init_state(B)
    for b in range(B):
        if offsets[b]:
            one = gm.init_state(1)
            prev = stt.text_card
            for i in range(offsets[b]):
                gm.step([prev], audio_at(b, i)[None], one)
                prev = int(refs[b][0][i])
            st.copy_from(one, 0, b)
            one.close()
    prev = np.array([stt.text_card if offsets[b] == 0 else refs[b][0][offsets[b] - 1]
                     for b in range(B)], np.uint32)
    worst, flips, rels, env = 0.0, 0, [], []
    if envelope is not None:
        # The oracle against itself with the RMS-norm sum reversed, teacher-forced on its own
        # tokens: how far a 1-ulp reduction-order change moves these logits.
        envelope.orc_set_reduction_variant(1)
        try:
            for b in range(B):
                _, alt = O.greedy_stt(om, audio[:, b], offsets[b] + frames, teacher=refs[b][0])
                env += [float(np.linalg.norm(alt[i] - refs[b][1][i]) / np.linalg.norm(refs[b][1][i]))
                        for i in range(offsets[b], offsets[b] + frames)]
        finally:
            envelope.orc_set_reduction_variant(0)
    for j in range(frames):
        a = np.stack([audio_at(b, offsets[b] + j) for b in range(B)])
        tok, lg = gm.step(prev, a, st, logits=True)
        for b in range(B):
            i = offsets[b] + j
            rt, rl = refs[b]
            rel = float(np.linalg.norm(lg[b] - rl[i]) / np.linalg.norm(rl[i]))
            diff = float(np.max(np.abs(lg[b] - rl[i])))
            worst = max(worst, rel)
            rels.append(rel)
            assert not strict or rel <= REL_TOL, f"stream {b} step {i}: relative logit diff {rel:.3g}"
            if strict and tok[b] != rt[i]:
                s = np.sort(rl[i])
                assert s[-1] - s[-2] <= 2 * diff, (
                    f"stream {b} step {i}: token {tok[b]} != oracle {rt[i]} "
                    f"(margin {s[-1] - s[-2]:.3g}, diff {diff:.3g})")
                flips += 1
            prev[b] = rt[i]
    for b in range(B):
        assert st.position(b) == offsets[b] + frames
    if envelope is not None:
        rels, env = np.array(rels), np.array(env)
        print(f"  GPU vs oracle L2-rel median {np.median(rels):.3g} max {rels.max():.3g}; "
              f"oracle self-envelope median {np.median(env):.3g} max {env.max():.3g}")
        assert np.median(rels) <= 2 * np.median(env) + 1e-3
        assert rels.max() <= 2 * env.max() + 1e-3
    return worst, flips


@pytest.mark.parametrize("B", [16, 100, 260])
def test_toy_bf16_many_streams(svl_lib, oracle_lib, B):
    stt = config.stt_toy()
    worst, flips = run_batch(stt, B, frames=14, stagger=4)  # window 12: every ring wraps
    print(f"toy bf16 B={B}: worst relative logit diff {worst:.3g}, {flips} argmax flips")


@pytest.mark.parametrize("B", [20, 160])
def test_mid_bf16_split_k(svl_lib, oracle_lib, B):
    stt = mid_model()
    worst, flips = run_batch(stt, B, frames=5, stagger=3)
    print(f"mid bf16 B={B}: worst relative logit diff {worst:.3g}, {flips} argmax flips")


@pytest.mark.parametrize("wdt,kvdt", [("q8_0", "f32"), ("q4_1", "bf16")])
def test_quantised_many_streams(svl_lib, oracle_lib, wdt, kvdt):
    """Q8_0 / Q4_1 weights at 16+ streams: the products run on the tensor cores from f16
    images of the dequantised weights, against the f16 values of the activations' Q8 blocks,
    i.e. the values the reference's integer block dots multiply, rounded to 11 bits."""
    worst, flips = run_batch(mid_model(), 40, frames=5, stagger=3, wdt=wdt, kvdt=kvdt)
    print(f"mid {wdt} B=40: worst relative logit diff {worst:.3g}, {flips} argmax flips")


def test_tensor_core_path_is_deterministic(svl_lib):
    """The split-K partial sums are added in a fixed order: two runs give identical tokens,
    and the device token loop equals the host-driven loop."""
    stt = mid_model()
    cfg = stt.transformer("bf16", "bf16")
    gm = LanguageModel(stt, cfg, synth.stt_weights(stt, cfg))
    B, frames = 160, 6
    audio = synth.audio_tokens(stt, frames, seed=3, streams=B)
    a = gm.run_frames(audio, gm.init_state(B))
    b = gm.run_frames(audio, gm.init_state(B))
    np.testing.assert_array_equal(a, b)
    st = gm.init_state(B)
    prev = np.full(B, stt.text_card, np.uint32)
    for i in range(frames):
        au = np.full((B, stt.n_q), stt.card, np.uint32) if i == 0 else audio[i]
        prev = gm.step(prev, au, st)
        np.testing.assert_array_equal(prev, a[i])
