"""Speech to text on the device for many streams: audio in, text tokens out.

Stt::encode_frames and Recognizer::step's token loop (stt/mod.rs:532-565), batched over
streams. Per 80 ms frame of every stream, Mimi's encoder turns the audio into latents, the
quantizer turns the latents into the 32 audio tokens, and the language model steps with them.
Its first step sees the initial tokens, as in training (stt/mod.rs:551-563), and every later
step feeds back its own argmax. Everything stays on one CUDA stream; only the caller reads
tokens back. Word and voice-activity events are host logic over these tokens (svl/events.py).
"""
from __future__ import annotations

import ctypes

from . import _lib


class SttPipeline:
    def __init__(self, mimi, quantizer, lm, streams: int):
        import torch
        stt = lm.stt
        if quantizer.n_q != stt.n_q or quantizer.bins != stt.card:
            raise ValueError("the quantizer's codebooks must match the language model's audio vocabularies")
        if mimi.cfg.inner_dim != 512:
            raise ValueError("the quantizer takes 512-wide latents (Quantizer::new, stt/model.rs:92)")
        self.mimi, self.quantizer, self.lm, self.streams = mimi, quantizer, lm, streams
        self.stream = torch.cuda.Stream()
        self.mimi_state = mimi.init_state(streams, 1)
        self.lm_state = lm.init_state(streams)
        with torch.cuda.stream(self.stream):
            self.text = torch.full((streams,), stt.text_card, dtype=torch.int32, device="cuda")
            self.initial = torch.full((streams, stt.n_q), stt.card, dtype=torch.int32, device="cuda")
        self.steps = 0

    def step(self, pcm):
        """pcm: CUDA float32 [streams][channels][frame_size], one frame per stream. Returns the
        frame's text tokens and audio codes as CUDA int32 tensors ([streams], [streams][n_q]),
        valid on this pipeline's stream (synchronise it, or wait on it, before reading)."""
        import torch
        s = self.stream
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            latents = self.mimi.encode_step(pcm, self.mimi_state, stream=s)
            codes = self.quantizer.encode(latents, stream=s)[:, 0, :].contiguous()
            audio = self.initial if self.steps == 0 else codes
            out = torch.empty((self.streams,), dtype=torch.int32, device="cuda")
            _lib.check(_lib.lib().svl_stt_step_device(
                self.lm.handle, self.lm_state.handle, self.streams,
                ctypes.c_void_p(self.text.data_ptr()), ctypes.c_void_p(audio.data_ptr()),
                ctypes.c_void_p(out.data_ptr()), None, ctypes.c_void_p(s.cuda_stream)))
        self.text = out
        self.steps += 1
        return out, codes
