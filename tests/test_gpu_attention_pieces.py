"""The three decode-attention kernels against a float64 reference and against each other.

A batch state of 40 streams has at least 148 (stream, head) units, so its attention runs the
many-stream kernel: the keys of each unit are cut into pieces, warps take pieces in a fixed
round-robin order, and a follow-up kernel merges the partials of units of several pieces. Each
stream is put at its own position with random imported caches (positions past the window wrap
the ring), so units have 1 .. 10 pieces. The same streams in one-stream states run the flat
few-stream kernel (chunks of at most 48 keys, merged by the last CTA of each unit), and the
first 12 of them in one 12-stream state run the cluster-split kernel (4-CTA clusters of 75
keys each). Checked for three consecutive steps (the partial buffers and the flat kernel's
tickets are reused by every launch):
- f32 caches: logits within 2e-3 max-abs of the float64 reference (the reference's step over
  the exported caches);
- bf16 caches: within 2e-2 relative of it (the newest key is rounded to bf16 on the device);
- both: the batch state within 1e-4 max-abs of the one-stream and the 12-stream states (same
  inputs, different attention kernels), and two runs of the batch state bit-identical.
"""
import numpy as np
import pytest

import np_reference as R
from svl import LanguageModel, config, synth

pytestmark = pytest.mark.gpu


def reference_step(stt, cfg, w, caches, position, text, audio):
    """LanguageModel::step logits of one stream at `position` over the given caches, float64."""
    bb = R.Backbone(cfg, w)
    for l, (k, v) in enumerate(caches):
        bb.k[l] = [k[:, i, :].astype(np.float64) for i in range(k.shape[1])]
        bb.v[l] = [v[:, i, :].astype(np.float64) for i in range(v.shape[1])]
    bb.pos = position
    x = w["text_emb.weight"][text].astype(np.float64).copy()
    for c in range(stt.n_q):
        x = x + w[f"emb.{c}.weight"][audio[c]]
    x = bb.forward_token(x)
    ys = x / np.sqrt((x * x).mean() + 1e-8) * w["out_norm.alpha"].reshape(-1)
    return w["text_linear.weight"].astype(np.float64) @ ys


@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("kvdt", ["f32", "bf16"])
def test_many_stream_attention_pieces(svl_lib, head_dim, kvdt):
    heads = 4
    stt = config.stt_toy(dim=heads * head_dim, num_heads=heads, num_layers=2, context=300,
                         text_card=100, card=64, n_q=4, hidden_scale=1.5)
    cfg = stt.transformer("f32", kvdt)
    w = synth.stt_weights(stt, cfg)
    gm = LanguageModel(stt, cfg, w)
    B, steps = 40, 3
    rng = np.random.default_rng(11)
    # Fill levels from 1 key to past the window (ring wrap), a few at the piece edges.
    positions = rng.integers(0, 700, size=B)
    positions[:6] = [0, 1, 31, 32, 299, 300]
    big = gm.init_state(B)
    singles = [gm.init_state(1) for _ in range(B)]
    for b in range(B):
        n = int(min(positions[b], cfg.context))
        caches = [(rng.standard_normal((heads, n, head_dim)).astype(np.float32),
                   rng.standard_normal((heads, n, head_dim)).astype(np.float32))
                  for _ in range(cfg.num_layers)]
        if n:
            singles[b].load_layer_caches(caches, int(positions[b]))
        else:
            singles[b].reset()
        big.copy_from(singles[b], 0, b)
    twin = gm.init_state(B)
    for b in range(B):
        twin.copy_from(singles[b], 0, b)
    M = 12
    mid = gm.init_state(M)
    for b in range(M):
        mid.copy_from(singles[b], 0, b)
    text = rng.integers(0, stt.text_card, size=(steps, B)).astype(np.uint32)
    audio = rng.integers(0, stt.card, size=(steps, B, stt.n_q)).astype(np.uint32)
    for i in range(steps):
        exported = [singles[b].layer_caches() for b in range(B)]
        _, lg = gm.step(text[i], audio[i], big, logits=True)
        _, lg2 = gm.step(text[i], audio[i], twin, logits=True)
        np.testing.assert_array_equal(lg, lg2)
        _, lm = gm.step(text[i][:M], audio[i][:M], mid, logits=True)
        for b in range(M):
            d = float(np.max(np.abs(lg[b] - lm[b])))
            assert d <= 1e-4, f"step {i} stream {b} (position {positions[b] + i}): {d} from the cluster path"
        for b in range(B):
            _, ls = gm.step(text[i][b:b + 1], audio[i][b:b + 1], singles[b], logits=True)
            d = float(np.max(np.abs(lg[b] - ls[0])))
            assert d <= 1e-4, f"step {i} stream {b} (position {positions[b] + i}): {d} from the flat path"
            ref = reference_step(stt, cfg, w, exported[b], int(positions[b]) + i, int(text[i][b]),
                                 audio[i][b])
            if kvdt == "f32":
                d = float(np.max(np.abs(lg[b] - ref)))
                assert d <= 2e-3, f"step {i} stream {b}: {d} max-abs from the reference"
            else:
                r = float(np.linalg.norm(lg[b] - ref) / np.linalg.norm(ref))
                assert r <= 2e-2, f"step {i} stream {b}: {r} relative from the reference"
        for b in range(B):
            assert big.position(b) == positions[b] + i + 1
