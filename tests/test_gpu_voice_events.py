"""Voices (Voice::save / Voice::load, tts/voice.rs:78-149) and the device token loop's
voice-activity output (svl_stt_run_frames_ex), on the GPU.

The voice files are read and written here independently with the safetensors package, in the
layout of upstream Pocket TTS: per layer "transformer.layers.{i}.self_attn/cache" f32
[2, batch, time, kv_heads, head_dim], ".../offset" i64 [1], ".../pad" i64 [1]. The reference's
own check is that a saved voice reloaded reproduces the original generation
(tests/models.rs: saved_voice_reproduces_the_original); it is restated here on the LM step.
"""
import numpy as np
import pytest
from safetensors.numpy import load_file, save_file

import oracle as O
from svl import FlowLm, LanguageModel, config, synth
from svl._lib import SvlError
from svl.events import BatchedRecognizer, VoiceActivity

pytestmark = pytest.mark.gpu


def tts_toy(wdt="f32"):
    cfg, tts = config.tts_toy("lsd", wdt, "bf16" if wdt == "bf16" else "f32")
    return cfg, tts, synth.tts_weights(cfg, tts)


def test_saved_voice_reproduces_the_original(svl_lib, tmp_path):
    cfg, tts, w = tts_toy()
    fm = FlowLm(cfg, tts, w)
    prompt = np.array([3, 1, 4, 1, 5, 9, 2, 6], np.uint32)
    a = fm.init_state(4, max_positions=32)
    fm.prompt_text(prompt, a, stream=0)
    path = tmp_path / "voice.safetensors"
    a.save_voice(path, stream=0)

    # The file: the stream's caches, time-major, with their length and no padding.
    f = load_file(str(path))
    caches = a.layer_caches(0)
    for l, (k, v) in enumerate(caches):
        c = f[f"transformer.layers.{l}.self_attn/cache"]
        assert c.shape == (2, 1, len(prompt), cfg.num_kv_heads, cfg.head_dim) and c.dtype == np.float32
        np.testing.assert_array_equal(c[0, 0], k.transpose(1, 0, 2))
        np.testing.assert_array_equal(c[1, 0], v.transpose(1, 0, 2))
        assert f[f"transformer.layers.{l}.self_attn/offset"].tolist() == [len(prompt)]
        assert f[f"transformer.layers.{l}.self_attn/pad"].tolist() == [0]

    # Loaded into three streams of another state, every stream continues exactly as the
    # original does.
    b = fm.init_state(4, max_positions=32)
    b.load_voice(path, streams=[1, 2, 3])
    for s in (1, 2, 3):
        assert b.position(s) == len(prompt)
    noise = np.random.default_rng(4).standard_normal((3, 4, tts.latent_dim)).astype(np.float32)
    lat_a = lat_b = None
    for i in range(3):
        na = np.repeat(noise[i, :1], 4, 0)
        out_a, eos_a = fm.step(lat_a, na, a)
        out_b, eos_b = fm.step(lat_b, na, b)
        for s in (1, 2, 3):
            np.testing.assert_array_equal(out_b[s], out_a[0])
            np.testing.assert_array_equal(eos_b[s], eos_a[0])
        lat_a, lat_b = out_a, out_b


def test_loaded_voice_steps_like_the_oracle(svl_lib, oracle_lib, tmp_path):
    """A voice written in the upstream layout (here: from the oracle-equal GPU prompt, through
    numpy) and loaded into many streams gives the oracle's steps after prompt_text."""
    cfg, tts, w = tts_toy()
    fm = FlowLm(cfg, tts, w)
    om = O.OracleModel(1, cfg, w, tts=tts)
    prompt = np.array([7, 2, 9, 4, 4, 1], np.uint32)
    src = fm.init_state(1, max_positions=32)
    fm.prompt_text(prompt, src)
    tensors = {}
    for l, (k, v) in enumerate(src.layer_caches(0)):
        # Padded on the time axis beyond the offset, as upstream exports with spare capacity.
        cache = np.zeros((2, 1, len(prompt) + 3, cfg.num_kv_heads, cfg.head_dim), np.float32)
        cache[0, 0, : len(prompt)] = k.transpose(1, 0, 2)
        cache[1, 0, : len(prompt)] = v.transpose(1, 0, 2)
        tensors[f"transformer.layers.{l}.self_attn/cache"] = cache
        tensors[f"transformer.layers.{l}.self_attn/offset"] = np.array([len(prompt)], np.int64)
        tensors[f"transformer.layers.{l}.self_attn/pad"] = np.array([0], np.int64)
    path = tmp_path / "upstream.safetensors"
    save_file(tensors, str(path))
    B = 24
    st = fm.init_state(B, max_positions=32)
    st.load_voice(path, streams=list(range(B)))
    ost = om.init_state()
    om.prompt_text(prompt, ost)
    noise = np.random.default_rng(5).standard_normal((4, tts.latent_dim)).astype(np.float32)
    lat = None
    for i in range(4):
        ref, ref_eos = om.tts_step(None if lat is None else lat[0], noise[i], ost)
        got, eos = fm.step(lat, np.repeat(noise[i][None], B, 0), st)
        assert np.max(np.abs(got - ref[None])) <= 2e-3 and np.max(np.abs(eos - ref_eos)) <= 2e-3
        lat = np.repeat(ref[None], B, 0)


def test_voice_files_that_are_refused(svl_lib, tmp_path):
    cfg, tts, w = tts_toy()
    fm = FlowLm(cfg, tts, w)
    st = fm.init_state(2, max_positions=32)
    good = {}
    for l in range(cfg.num_layers):
        good[f"transformer.layers.{l}.self_attn/cache"] = np.ones((2, 1, 4, cfg.num_kv_heads, cfg.head_dim), np.float32)
        good[f"transformer.layers.{l}.self_attn/offset"] = np.array([4], np.int64)
        good[f"transformer.layers.{l}.self_attn/pad"] = np.array([0], np.int64)

    def refused(tensors, what):
        p = tmp_path / f"{what}.safetensors"
        save_file(tensors, str(p))
        with pytest.raises(SvlError) as e:
            st.load_voice(p, streams=[0])
        assert e.value.kind == "INVALID_INPUT", (what, e.value)

    padded = dict(good)
    padded["transformer.layers.0.self_attn/pad"] = np.array([2], np.int64)
    refused(padded, "padded")
    heads = dict(good)
    heads["transformer.layers.1.self_attn/cache"] = np.ones((2, 1, 4, cfg.num_kv_heads + 1, cfg.head_dim), np.float32)
    refused(heads, "heads")
    missing = {k: v for k, v in good.items() if not k.startswith("transformer.layers.1.")}
    refused(missing, "missing-layer")
    with pytest.raises(SvlError):
        st.load_voice(tmp_path / "no-such-file.safetensors", streams=[0])
    # Older exports: no offset, the length is the shape of current_end; bf16 caches convert.
    older = {}
    for l in range(cfg.num_layers):
        older[f"transformer.layers.{l}.self_attn/cache"] = np.ones((2, 1, 5, cfg.num_kv_heads, cfg.head_dim), np.float32)
        older[f"transformer.layers.{l}.self_attn/current_end"] = np.zeros(3, np.float32)
    p = tmp_path / "older.safetensors"
    save_file(older, str(p))
    st.load_voice(p, streams=[1])
    assert st.position(1) == 3


def test_device_loop_voice_activity_and_events(svl_lib):
    """svl_stt_run_frames_ex returns each frame's extra-head p[0], equal to the host-buffer
    step's; BatchedRecognizer turns the streams' tokens and voice activity into events."""
    stt = config.stt_toy(extra_heads_num_heads=4, extra_heads_dim=6)
    cfg = stt.transformer("q8_0", "f32")
    gm = LanguageModel(stt, cfg, synth.stt_weights(stt, cfg))
    B, frames = 3, 10
    audio = synth.audio_tokens(stt, frames, seed=2, streams=B)
    toks, extra = gm.run_frames(audio, gm.init_state(B), extra=True)
    assert extra.shape == (frames, B, 4)
    st = gm.init_state(B)
    prev = np.full(B, stt.text_card, np.uint32)
    for i in range(frames):
        a = np.full((B, stt.n_q), stt.card, np.uint32) if i == 0 else audio[i]
        tok, ex = gm.step(prev, a, st, extra=True)
        np.testing.assert_array_equal(tok, toks[i])
        np.testing.assert_array_equal(ex, extra[i])
        prev = tok

    class Tok:
        def decode(self, t):
            return " ".join(f"w{x}" for x in t)

        def encode(self, word):
            return [0]

    br = BatchedRecognizer(gm, gm.init_state(B), Tok(), B)
    events = br.feed(audio)
    for b in range(B):
        va = [e for e in events[b] if isinstance(e, VoiceActivity)]
        assert len(va) == frames
        np.testing.assert_allclose([e.pause_probabilities for e in va], extra[:, b], rtol=0, atol=0)
        assert br.recognizers[b].steps == frames
