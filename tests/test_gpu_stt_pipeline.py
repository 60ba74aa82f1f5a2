"""Speech to text end to end on the GPU (svl/stt_pipeline.py): Mimi encoder -> quantizer ->
language model for several streams, frame by frame, against the oracle's chain run per stream
(Stt::encode_frames and Recognizer::step, stt/mod.rs:532-565).

The language model is f32, so its tokens equal the oracle's whenever its audio tokens do. The
audio tokens come from latents whose transformer sums attention in another order than the
oracle. A code may flip only where two codebook entries are within rounding of each other, so
the test compares tokens up to a stream's first code flip and requires flips to be rare.
"""
import numpy as np
import pytest

import oracle
from svl import LanguageModel, codec, config, synth
from svl.stt_pipeline import SttPipeline

pytestmark = pytest.mark.gpu


def test_audio_to_text_tokens(svl_lib):
    import torch
    streams, frames = 3, 6
    stt = config.stt_toy(card=2048, n_q=32)
    cfg = stt.transformer("f32", "f32")
    mcfg = codec.stt_mimi(codec.ENCODER)
    w = synth.mimi_weights(mcfg)
    w.update(synth.rvq_weights(32, 2048))
    lw = synth.stt_weights(stt, cfg)
    mimi, q = codec.Mimi(mcfg, w), codec.Quantizer(32, 2048, w)
    lm = LanguageModel(stt, cfg, lw)
    pipe = SttPipeline(mimi, q, lm, streams)
    fs = mimi.frame_size
    pcm = (0.3 * np.random.default_rng(13).standard_normal((streams, 1, frames * fs))).astype(np.float32)
    toks, codes = [], []
    for f in range(frames):
        t, c = pipe.step(torch.from_numpy(np.ascontiguousarray(pcm[:, :, f * fs:(f + 1) * fs])).cuda())
        pipe.stream.synchronize()
        toks.append(t.cpu().numpy().astype(np.uint32))
        codes.append(c.cpu().numpy().astype(np.uint32))
    toks, codes = np.stack(toks, 1), np.stack(codes, 1)  # [streams][frames], [streams][frames][32]

    om, oq = oracle.OracleMimi(mcfg, w), oracle.OracleQuantizer(32, 2048, w)
    olm = oracle.OracleModel(0, cfg, lw, stt=stt)
    flips = 0
    for s in range(streams):
        ost = om.init_state()
        ref_codes = np.stack([oq.encode(om.encode_step(pcm[s, :, f * fs:(f + 1) * fs], ost))[0]
                              for f in range(frames)])
        diff = np.nonzero((ref_codes != codes[s]).any(1))[0]
        flips += int((ref_codes != codes[s]).sum())
        upto = int(diff[0]) if len(diff) else frames
        ref_toks, _ = oracle.greedy_stt(olm, codes[s], frames)  # the oracle LM on the GPU's codes
        np.testing.assert_array_equal(toks[s], ref_toks)
        own, _ = oracle.greedy_stt(olm, ref_codes, frames)
        np.testing.assert_array_equal(toks[s][:upto], own[:upto])
    assert flips <= 4, flips  # of 576 codes
