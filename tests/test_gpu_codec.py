"""Mimi and the residual vector quantizer on the GPU against the oracle, through the C ABI.

Each stream of a batch is compared with the oracle run on that stream alone. The convolutions
sum in the oracle's order (fixed chunks of FMA chains per output), so they match it; the
transformers between them sum attention in parallel, so the bar is relative: max |gpu - oracle|
<= 1e-4 of the output's scale. The quantizer is compared bit for bit on the same latents; on
latents that went through the encoder, a code may differ only where the oracle's two candidates
are within rounding of each other.
"""
import numpy as np
import pytest

import oracle
from svl import codec, synth

pytestmark = pytest.mark.gpu

REL = 1e-4


def close(gpu, ref):
    scale = max(1.0, float(np.abs(ref).max()))
    return float(np.abs(gpu - ref).max()) <= REL * scale, float(np.abs(gpu - ref).max()) / scale


def run_codec(cfg, streams, calls, seed=7):
    """Encodes (if the config has an encoder) and decodes `calls` (frames per call) on every
    stream at once on the GPU and per stream on the oracle."""
    import torch
    w = synth.mimi_weights(cfg)
    gm, om = codec.Mimi(cfg, w), oracle.OracleMimi(cfg, w)
    fs = gm.frame_size
    assert fs == om.frame_size == cfg.frame_size
    rng = np.random.default_rng(seed)
    total = sum(calls)
    results = {}
    if cfg.parts & codec.ENCODER:
        pcm = (0.3 * rng.standard_normal((streams, cfg.encoder.channels, total * fs))).astype(np.float32)
        gs = gm.init_state(streams, max(calls))
        outs, f0 = [], 0
        for n in calls:
            x = torch.from_numpy(np.ascontiguousarray(pcm[:, :, f0 * fs:(f0 + n) * fs])).cuda()
            outs.append(gm.encode_step(x, gs).cpu().numpy())
            f0 += n
        got = np.concatenate(outs, 2)
        for s in range(streams):
            st, f0, ref = om.init_state(), 0, []
            for n in calls:
                ref.append(om.encode_step(pcm[s, :, f0 * fs:(f0 + n) * fs], st))
                f0 += n
            ok, err = close(got[s], np.concatenate(ref, 1))
            assert ok, ("encode", s, err)
        results["latent"] = got
    if cfg.parts & codec.DECODER:
        lat = rng.standard_normal((streams, cfg.outer_dim, total)).astype(np.float32)
        gs = gm.init_state(streams, max(calls))
        outs, f0 = [], 0
        for n in calls:
            x = torch.from_numpy(np.ascontiguousarray(lat[:, :, f0:f0 + n])).cuda()
            outs.append(gm.decode_step(x, gs).cpu().numpy())
            f0 += n
        got = np.concatenate(outs, 2)
        for s in range(streams):
            st, f0, ref = om.init_state(), 0, []
            for n in calls:
                ref.append(om.decode_step(lat[s, :, f0:f0 + n], st))
                f0 += n
            ok, err = close(got[s], np.concatenate(ref, 1))
            assert ok, ("decode", s, err)
        results["pcm"] = got
    return results


@pytest.mark.parametrize("pad_mode", [0, 1])
def test_toy_mimi_streams(svl_lib, pad_mode):
    """Three streams, frames in calls of 1, 2, 1, 3: the windowed transformer wraps its ring and
    every convolution carries its state across calls."""
    run_codec(codec.toy_mimi(pad_mode=pad_mode), 3, [1, 2, 1, 3])


def test_toy_mimi_many_streams(svl_lib):
    """20 streams: the transformer's products take several launches of streams."""
    run_codec(codec.toy_mimi(), 20, [1, 1])


def test_stt_mimi_encoder(svl_lib):
    """The STT Mimi encoder (moshi's Mimi, stt/model.rs:44-82) at its real shape: 2 streams,
    3 frames."""
    run_codec(codec.stt_mimi(codec.ENCODER), 2, [1, 2])


def test_tts_mimi_decoder(svl_lib):
    """The Pocket-TTS Mimi decoder (depthwise up-sampling by 16, ratios 6 5 4): 2 streams,
    3 frames."""
    run_codec(codec.tts_mimi(codec.DECODER), 2, [2, 1])


def test_mimi_state_reset(svl_lib):
    import torch
    cfg = codec.toy_mimi(codec.ENCODER)
    gm = codec.Mimi(cfg, synth.mimi_weights(cfg))
    pcm = torch.from_numpy((0.3 * np.random.default_rng(8).standard_normal(
        (2, 1, gm.frame_size))).astype(np.float32)).cuda()
    st = gm.init_state(2, 1)
    first = gm.encode_step(pcm, st).cpu().numpy()
    gm.encode_step(pcm, st)
    st.reset(1)
    again = gm.encode_step(pcm, st).cpu().numpy()
    assert np.array_equal(again[1], first[1])
    assert not np.array_equal(again[0], first[0])


def test_mimi_rejects_bad_calls(svl_lib):
    import torch
    from svl._lib import SvlError
    cfg = codec.toy_mimi(codec.ENCODER)
    gm = codec.Mimi(cfg, synth.mimi_weights(cfg))
    st = gm.init_state(2, 1)
    with pytest.raises(SvlError):  # more frames than the state was sized for
        gm.encode_step(torch.zeros((2, 1, 2 * gm.frame_size), device="cuda"), st)
    with pytest.raises(SvlError):  # no decoder loaded
        gm.decode_step(torch.zeros((1, cfg.outer_dim, 1), device="cuda"), st)
    w = synth.mimi_weights(cfg)
    del w["downsample.conv.conv.weight"]
    with pytest.raises(SvlError):
        codec.Mimi(cfg, w)


@pytest.mark.parametrize("n_q,bins,streams,frames",
                         [(32, 2048, 5, 3), (8, 300, 9, 1), (1, 64, 2, 2), (32, 2048, 20, 3), (32, 2048, 40, 3)])
def test_quantizer_bit_exact(svl_lib, n_q, bins, streams, frames):
    """Quantizer::encode on the same latents: codes identical to the oracle's (rows per cluster:
    2 for up to 32 rows, 4 up to 96, 8 above)."""
    import torch
    w = synth.rvq_weights(n_q, bins)
    gq, oq = codec.Quantizer(n_q, bins, w), oracle.OracleQuantizer(n_q, bins, w)
    lat = np.random.default_rng(9).standard_normal((streams, 512, frames)).astype(np.float32)
    got = gq.encode(torch.from_numpy(lat).cuda()).cpu().numpy().astype(np.uint32)
    assert got.shape == (streams, frames, n_q)
    for s in range(streams):
        np.testing.assert_array_equal(got[s], oq.encode(lat[s]))


def test_stt_audio_tokens_from_pcm(svl_lib):
    """Audio to STT tokens on the GPU (Mimi encoder, then the quantizer: stt/mod.rs:532-541)
    against the oracle: codes equal, or, where not, the oracle's distance to the GPU's entry is
    within rounding of its own choice."""
    import torch
    cfg = codec.stt_mimi(codec.ENCODER)
    w = synth.mimi_weights(cfg)
    w.update(synth.rvq_weights(32, 2048))
    gm, gq = codec.Mimi(cfg, w), codec.Quantizer(32, 2048, w)
    om, oq = oracle.OracleMimi(cfg, w), oracle.OracleQuantizer(32, 2048, w)
    pcm = (0.3 * np.random.default_rng(10).standard_normal((2, 1, 2 * gm.frame_size))).astype(np.float32)
    lat = gm.encode_step(torch.from_numpy(pcm).cuda(), gm.init_state(2, 2))
    codes = gq.encode(lat).cpu().numpy().astype(np.uint32)
    flips = 0
    for s in range(2):
        ref_lat = om.encode_step(pcm[s], om.init_state())
        ref = oq.encode(ref_lat)
        flips += int((ref != codes[s]).sum())
    assert flips <= 2, flips  # 128 codes; the latents differ by attention-order rounding
