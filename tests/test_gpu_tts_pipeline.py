"""Text to speech end to end on the GPU (svl/tts_pipeline.py): FlowLm steps with latent
feedback on the device, then Tts::decode_latent (emb_std / emb_mean, quantizer.output_proj,
the Pocket-TTS Mimi decoder), against the oracle's chain per stream (tts/mod.rs:441-447, :494).

Bars: the latents as in the f32 TTS tests (2e-3 max-abs, f32 weights); the audio within 1e-3 of
its scale. The decoder is linear in its input up to the ELUs, so the latents' last-bit
differences stay of their size.
"""
import numpy as np
import pytest

import oracle
from svl import FlowLm, codec, config, synth
from svl.tts_pipeline import TtsPipeline

pytestmark = pytest.mark.gpu


def test_text_to_audio(svl_lib):
    import torch
    streams, frames, prompt = 3, 4, 6
    cfg, tts = config.tts_toy()
    w = synth.tts_weights(cfg, tts)
    mcfg = codec.tts_mimi(codec.DECODER)
    mw = synth.mimi_weights(mcfg, latent_dim=tts.latent_dim)
    rng = np.random.default_rng(14)
    emb_std = rng.uniform(0.5, 1.5, tts.latent_dim).astype(np.float32)
    emb_mean = (0.1 * rng.standard_normal(tts.latent_dim)).astype(np.float32)
    tokens = rng.integers(0, tts.text_bins, size=(streams, prompt), dtype=np.uint32)
    noise = rng.standard_normal((frames, streams, tts.latent_dim)).astype(np.float32)

    pipe = TtsPipeline(FlowLm(cfg, tts, w), codec.Mimi(mcfg, mw), emb_std, emb_mean, streams)
    pipe.prompt(tokens)
    pcms, lats = [], []
    for f in range(frames):
        pcm, lat, _ = pipe.step(torch.from_numpy(noise[f]).cuda())
        pipe.stream.synchronize()
        pcms.append(pcm.cpu().numpy())
        lats.append(lat.cpu().numpy())
    pcms, lats = np.concatenate(pcms, 2), np.stack(lats, 1)

    olm = oracle.OracleModel(1, cfg, w, tts=tts)
    om = oracle.OracleMimi(mcfg, mw)
    for s in range(streams):
        st, mst = olm.init_state(), om.init_state()
        olm.prompt_text(tokens[s], st)
        lat, ref_pcm, ref_lat = None, [], []
        for f in range(frames):
            lat, _ = olm.tts_step(lat, noise[f, s], st)
            ref_lat.append(lat)
            ref_pcm.append(om.decode_latent(lat[None], mst, emb_std, emb_mean))
        ref_lat, ref_pcm = np.stack(ref_lat), np.concatenate(ref_pcm, 1)
        assert np.max(np.abs(lats[s] - ref_lat)) <= 2e-3, s
        err = np.max(np.abs(pcms[s] - ref_pcm)) / max(1.0, float(np.abs(ref_pcm).max()))
        assert err <= 1e-3, (s, err)
