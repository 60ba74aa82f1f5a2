"""The batched configurations at their real shapes (4 at 128 streams, 5),
each sampled stream checked against the CPU oracle run on that stream alone.

- Config 3: STT-1b, bf16 weights and KV, 256 streams in one batch (the tcgen05 GEMM path and
  the many-stream attention), streams at staggered positions (ring fills 0..63 before the
  checked frames); 32 of the 256 streams are checked over 64 frames.
- Config 4 at 128 streams: STT-2.6b, q4_1 weights (tensor cores on f16 images of the
  dequantised weights), bf16 KV; 8 of the 128 streams over 24 frames.
- Config 5: Pocket-TTS, bf16, 512 streams, each with its own 64-token text prompt (prefilled in
  one batch), then 16 frames of latent feedback; 16 of the 512 streams checked.

The checked streams are teacher-forced with the oracle's tokens (latents), so each step
compares one step's arithmetic on the oracle's history; every other stream of the batch runs
free and only has to be there. Bars: the north star's bf16 / quantised bar, logits (flow
outputs) within 2e-2 relative, ||diff||_2 / ||oracle||_2 per stream and step; an argmax may
differ from the oracle's only where the oracle's top-2 margin is within twice the logit
deviation.
"""
import numpy as np
import pytest

import oracle as O
from svl import FlowLm, LanguageModel, config, synth

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

REL_TOL = 2e-2


class SampledBatch:
    """B streams of one STT model at staggered positions; the oracle runs of the sampled
    streams (optionally also with the RMS-norm sum reversed: the oracle's own sensitivity to a
    1-ulp reduction-order change, teacher-forced on its tokens)."""

    def __init__(self, stt, wdt, kvdt, B, sample, offsets, frames, envelope_lib=None):
        self.stt, self.B, self.sample, self.offsets, self.frames = stt, B, sample, offsets, frames
        cfg = stt.transformer(wdt, kvdt)
        w = synth.stt_weights(stt, cfg)
        om = O.OracleModel(0, cfg, w, stt=stt)
        self.gm = LanguageModel(stt, cfg, w)
        del w
        self.audio = synth.audio_tokens(stt, max(offsets) + frames, seed=1, streams=B)
        self.refs = {b: O.greedy_stt(om, self.audio[:, b], offsets[b] + frames) for b in sample}
        self.env = None
        if envelope_lib is not None:
            envelope_lib.orc_set_reduction_variant(1)
            try:
                self.env = []
                for b in sample:
                    _, alt = O.greedy_stt(om, self.audio[:, b], offsets[b] + frames, teacher=self.refs[b][0])
                    rl = self.refs[b][1]
                    self.env += [float(np.linalg.norm(alt[i] - rl[i]) / np.linalg.norm(rl[i]))
                                 for i in range(offsets[b], offsets[b] + frames)]
            finally:
                envelope_lib.orc_set_reduction_variant(0)
        del om

    def audio_at(self, b, i):
        return np.full(self.stt.n_q, self.stt.card, np.uint32) if i == 0 else self.audio[i, b]

    def run(self, reference_order=False):
        """The batch on the GPU; returns per sampled step (stream, step, tokens equal, logits, ref)."""
        stt, gm, B, offsets, refs = self.stt, self.gm, self.B, self.offsets, self.refs
        st = gm.init_state(B, reference_order=reference_order)
        for b in range(B):
            if not offsets[b]:
                continue
            one = gm.init_state(1, reference_order=reference_order)
            if b in refs:  # the oracle's history, token for token
                prev = stt.text_card
                for i in range(offsets[b]):
                    gm.step([prev], self.audio_at(b, i)[None], one)
                    prev = int(refs[b][0][i])
            else:
                gm.run_frames(self.audio[: offsets[b], b][:, None, :], one)
            st.copy_from(one, 0, b)
            one.close()
        # A stream's first text token in the batch: text_card at position 0, the oracle's last
        # token for the checked streams; the free-running ones get any valid id.
        prev = np.array([stt.text_card if offsets[b] == 0 else
                         (refs[b][0][offsets[b] - 1] if b in refs else 0) for b in range(B)], np.uint32)
        out = []
        for j in range(self.frames):
            a = np.stack([self.audio_at(b, offsets[b] + j) for b in range(B)])
            tok, lg = gm.step(prev, a, st, logits=True)
            for b in self.sample:
                i = offsets[b] + j
                out.append((b, i, tok[b], lg[b].copy(), refs[b][0][i], refs[b][1][i]))
            prev = tok.copy()
            for b in self.sample:
                prev[b] = refs[b][0][offsets[b] + j]
        for b in range(B):
            assert st.position(b) == offsets[b] + self.frames
        st.close()
        return out


def deviation(steps):
    """(median and max L2-relative logit deviation, argmax differences, steps, differences
    outside the top-2-margin rule)."""
    rels, flips, bad = [], 0, []
    for b, i, tok, lg, rt, rl in steps:
        rel = float(np.linalg.norm(lg - rl) / np.linalg.norm(rl))
        diff = float(np.max(np.abs(lg - rl)))
        rels.append(rel)
        if tok != rt:
            flips += 1
            s = np.sort(rl)
            if s[-1] - s[-2] > 2 * diff:
                bad.append(f"stream {b} step {i}: token {tok} != oracle {rt} "
                           f"(margin {s[-1] - s[-2]:.3g}, diff {diff:.3g})")
    rels = np.array(rels)
    return float(np.median(rels)), float(rels.max()), flips, len(rels), bad


def report(name, nstreams, frames, med, mx, flips, n, bad):
    print(f"{name}: {nstreams} streams x {frames} frames, L2-relative logit diff median {med:.3g} "
          f"max {mx:.3g} (bar 2e-2), {flips}/{n} argmax differences")
    assert mx <= REL_TOL, f"{name}: relative logit diff {mx:.3g} above the 2e-2 bar"
    assert not bad, bad[:5]


def test_config3_stt1b_bf16_256_streams(svl_lib, oracle_lib):
    B, frames = 256, 64
    sample = list(range(0, B, 8))
    offsets = [(b * 37) % 64 for b in range(B)]
    sb = SampledBatch(config.stt_1b(), "bf16", "bf16", B, sample, offsets, frames)
    report("config 3 (STT-1b bf16, 256 streams)", len(sample), frames, *deviation(sb.run()))


def test_config4_stt2b6_q4_1_128_streams(svl_lib, oracle_lib):
    """A reference-order state at 128 streams is the reference's arithmetic bit for bit. A fast
    state runs the products on the tensor cores from f16 images of the dequantised weights: their
    last-bit differences pass through the Q8_1 activation rounding and grow over 24 layers, as
    the oracle's own logits do under a reversed norm sum; that state is reported against the
    2e-2 bar and held to twice the oracle's self-envelope."""
    B, frames = 128, 24
    sample = list(range(0, B, 16))
    offsets = [(b * 23) % 32 for b in range(B)]
    sb = SampledBatch(config.stt_2b6(), "q4_1", "bf16", B, sample, offsets, frames, envelope_lib=oracle_lib)
    exact = sb.run(reference_order=True)
    for b, i, tok, lg, rt, rl in exact:
        assert tok == rt, f"reference order, stream {b} step {i}: token {tok} != {rt}"
        np.testing.assert_array_equal(lg, rl, err_msg=f"reference order, stream {b} step {i}")
    print(f"config 4 (STT-2.6b q4_1, 128 streams), reference-order state: {len(exact)} sampled "
          f"steps bit-exact (logits and tokens)")
    med, mx, flips, n, bad = deviation(sb.run())
    env = np.array(sb.env)
    print(f"config 4 (STT-2.6b q4_1, 128 streams), fast state: L2-relative logit deviation median "
          f"{med:.3g} max {mx:.3g} (north-star bar 2e-2, met by the reference-order state), "
          f"{flips}/{n} argmax differences; oracle self-envelope median {np.median(env):.3g} max "
          f"{env.max():.3g}")
    assert med <= 2 * np.median(env) + 1e-3 and mx <= 2 * env.max() + 1e-3
    assert not bad, bad[:5]


def test_config5_pocket_tts_512_streams(svl_lib, oracle_lib):
    cfg, tts = config.pocket_tts()
    import dataclasses
    cfg = dataclasses.replace(cfg, weight_dtype="bf16", kv_dtype="bf16")
    w = synth.tts_weights(cfg, tts)
    om = O.OracleModel(1, cfg, w, tts=tts)
    gm = FlowLm(cfg, tts, w)
    del w
    B, P, frames = 512, 64, 16
    sample = list(range(0, B, 32))
    tokens = np.stack([np.random.default_rng(3 + b).integers(0, tts.text_bins, size=P, dtype=np.uint32)
                       for b in range(B)])
    noise = np.random.default_rng(4).standard_normal((frames, B, tts.latent_dim)).astype(np.float32)
    osts = {}
    for b in sample:
        osts[b] = om.init_state()
        om.prompt_text(tokens[b], osts[b])
    gst = gm.init_state(B, max_positions=P + frames + 1)
    gm.prompt_text_batch(tokens, gst)
    latent = None
    rels, eos = [], []
    for i in range(frames):
        got_lat, got_eos = gm.step(latent, noise[i], gst)
        nxt = got_lat.copy()
        ref_eos = []
        for b in sample:
            ref_lat, e = om.tts_step(None if latent is None else latent[b], noise[i, b], osts[b])
            fl_got, fl_ref = got_lat[b] - noise[i, b], ref_lat - noise[i, b]
            rels.append(float(np.linalg.norm(fl_got - fl_ref) / np.linalg.norm(fl_ref)))
            ref_eos.append(e)
            nxt[b] = ref_lat  # teacher forcing
        ref_eos = np.array(ref_eos, np.float32)
        eos.append(float(np.linalg.norm(got_eos[sample] - ref_eos) / max(np.linalg.norm(ref_eos), 1e-6)))
        latent = nxt
    rels = np.array(rels)
    print(f"config 5 (Pocket-TTS bf16, 512 streams): {len(sample)} streams x {frames} frames after a "
          f"{P}-token prompt, flow L2-relative diff median {np.median(rels):.3g} max {rels.max():.3g}, "
          f"EOS logits max {max(eos):.3g} (bar 2e-2)")
    assert rels.max() <= REL_TOL and max(eos) <= REL_TOL
