"""Text to speech on the device for many streams: prompt in, audio out.

LatentGenerator::advance and Tts::decode_latent (tts/mod.rs:441-447, :494), batched over
streams. Per frame, FlowLm::step produces every stream's next latent from its previous one.
That feedback stays on the device, and the noise is an input, as the reference samples it on
the host. The latent is scaled by the flow LM's emb_std, shifted by emb_mean, projected by
quantizer.output_proj and decoded by Mimi into 80 ms of audio. The reference decodes one frame
behind generation so the two overlap; here both run on one CUDA stream, in order.
"""
from __future__ import annotations

import ctypes

from . import _lib


class TtsPipeline:
    def __init__(self, flow_lm, mimi, emb_std, emb_mean, streams: int, decode_steps: int = 1,
                 max_positions: int = 1024):
        import torch
        if _lib.lib().svl_mimi_latent_dim(mimi.handle) != flow_lm.tts.latent_dim:
            raise ValueError("the codec needs quantizer.output_proj for the flow LM's latent width")
        self.flow_lm, self.mimi, self.streams, self.decode_steps = flow_lm, mimi, streams, decode_steps
        self.stream = torch.cuda.Stream()
        self.lm_state = flow_lm.init_state(streams, max_positions)  # no window: positions bound the cache
        self.mimi_state = mimi.init_state(streams, 1)
        with torch.cuda.stream(self.stream):
            self.emb_std = torch.as_tensor(emb_std, dtype=torch.float32).cuda()
            self.emb_mean = torch.as_tensor(emb_mean, dtype=torch.float32).cuda()
        self.latent = None  # None: the first step starts from BOS

    def prompt(self, tokens):
        """FlowLm::prompt_text for every stream: tokens [streams][n] (host)."""
        self.flow_lm.prompt_text_batch(tokens, self.lm_state)

    def step(self, noise):
        """noise: CUDA float32 [streams][latent_dim]. Returns (pcm [streams][channels][frame_size],
        latent [streams][latent_dim], eos logits [streams]) as CUDA tensors, valid on this
        pipeline's stream."""
        import torch
        s = self.stream
        s.wait_stream(torch.cuda.current_stream())
        lat_dim = self.flow_lm.tts.latent_dim
        with torch.cuda.stream(s):
            out = torch.empty((self.streams, lat_dim), dtype=torch.float32, device="cuda")
            eos = torch.empty((self.streams,), dtype=torch.float32, device="cuda")
            prev = ctypes.c_void_p(self.latent.data_ptr()) if self.latent is not None else None
            _lib.check(_lib.lib().svl_tts_step_device(
                self.flow_lm.handle, self.lm_state.handle, self.streams, prev,
                ctypes.c_void_p(noise.data_ptr()), self.decode_steps, ctypes.c_void_p(out.data_ptr()),
                ctypes.c_void_p(eos.data_ptr()), ctypes.c_void_p(s.cuda_stream)))
            pcm = self.mimi.decode_latent(out.view(self.streams, 1, lat_dim), self.mimi_state,
                                          self.emb_std, self.emb_mean, stream=s)
        self.latent = out
        return pcm, out, eos
