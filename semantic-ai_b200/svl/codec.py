"""Mimi (the codec around the language models) and Kyutai STT's residual vector quantizer.

Configs mirror SeanetConfig (nn/seanet.rs:14-30), ProjectedTransformerConfig (nn/mimi.rs:18-29)
and MimiConfig (nn/mimi.rs:36-51); the presets are the STT Mimi (stt/model.rs:44-82) and the
Pocket-TTS Mimi (configs/tts/english.yaml, CodecConfig::mimi in tts/config.rs:258-281). The
classes drive libsvl_b200.so's codec entry points (include/svl_cuda.h) on device tensors.
Paths are relative to crates/semantic-voice-local/src/ of the reference.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from .model import tensor_views

ENCODER, DECODER = 1, 2


def _call(fn, *args, stream=None):
    """Runs a codec entry point ordered with torch's current stream (or `stream`): a named stream
    is passed through; torch's default stream (handle 0, which the C ABI reads as "the codec's
    own stream") is synchronised around the call."""
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    if s.cuda_stream == 0:
        torch.cuda.synchronize()
        _lib.check(fn(*args, None))
        torch.cuda.synchronize()
    else:
        _lib.check(fn(*args, ctypes.c_void_p(s.cuda_stream)))


class CSeanetConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "dimension", "channels", "n_filters", "n_residual_layers", "kernel_size",
        "residual_kernel_size", "last_kernel_size", "dilation_base", "pad_mode", "compress",
        "n_ratios")] + [("ratios", ctypes.c_int32 * 8), ("_pad", ctypes.c_int32)]


class CProjectedTransformerConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "d_model", "input_dimension", "output_dimension", "num_heads", "num_layers", "context",
        "dim_feedforward", "_pad")] + [("max_period", ctypes.c_double)]


class CMimiConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "sample_rate", "inner_dim", "outer_dim", "exact_gelu", "parts", "_pad")] + [
        ("frame_rate", ctypes.c_double), ("encoder", CSeanetConfig), ("decoder", CSeanetConfig),
        ("encoder_transformer", CProjectedTransformerConfig),
        ("decoder_transformer", CProjectedTransformerConfig)]


@dataclass(frozen=True)
class SeanetConfig:
    dimension: int
    channels: int
    n_filters: int
    n_residual_layers: int
    ratios: tuple
    kernel_size: int
    residual_kernel_size: int
    last_kernel_size: int
    dilation_base: int
    pad_mode: int  # 0 constant, 1 replicate
    compress: int

    @property
    def hop(self) -> int:
        return int(np.prod(self.ratios))

    def to_c(self) -> CSeanetConfig:
        c = CSeanetConfig(self.dimension, self.channels, self.n_filters, self.n_residual_layers,
                          self.kernel_size, self.residual_kernel_size, self.last_kernel_size,
                          self.dilation_base, self.pad_mode, self.compress, len(self.ratios))
        for i, r in enumerate(self.ratios):
            c.ratios[i] = r
        return c


@dataclass(frozen=True)
class ProjectedTransformerConfig:
    d_model: int
    input_dimension: int
    output_dimension: int
    num_heads: int
    num_layers: int
    context: int
    dim_feedforward: int
    max_period: float = 10_000.0

    def to_c(self) -> CProjectedTransformerConfig:
        return CProjectedTransformerConfig(self.d_model, self.input_dimension,
                                           self.output_dimension, self.num_heads,
                                           self.num_layers, self.context, self.dim_feedforward,
                                           0, float(self.max_period))


@dataclass(frozen=True)
class MimiConfig:
    sample_rate: int
    frame_rate: float
    encoder: SeanetConfig
    decoder: SeanetConfig
    encoder_transformer: ProjectedTransformerConfig
    decoder_transformer: ProjectedTransformerConfig
    inner_dim: int
    outer_dim: int
    exact_gelu: bool
    parts: int = ENCODER | DECODER

    @property
    def frame_size(self) -> int:
        return int(round(self.sample_rate / self.frame_rate))

    def resample_stride(self, seanet: SeanetConfig) -> int:
        return int(round(self.sample_rate / seanet.hop / self.frame_rate))

    def to_c(self) -> CMimiConfig:
        return CMimiConfig(self.sample_rate, self.inner_dim, self.outer_dim, int(self.exact_gelu),
                           self.parts, 0, float(self.frame_rate), self.encoder.to_c(),
                           self.decoder.to_c(), self.encoder_transformer.to_c(),
                           self.decoder_transformer.to_c())


def stt_mimi(parts: int = ENCODER | DECODER) -> MimiConfig:
    """mimi_config() of stt/model.rs:44-82 (moshi's Mimi)."""
    s = SeanetConfig(512, 1, 64, 1, (8, 6, 5, 4), 7, 3, 3, 2, 0, 2)
    t = ProjectedTransformerConfig(512, 512, 512, 8, 8, 250, 2048)
    return MimiConfig(24_000, 12.5, s, s, t, t, 512, 512, True, parts)


def tts_mimi(parts: int = ENCODER | DECODER) -> MimiConfig:
    """The Pocket-TTS english Mimi (configs/tts/english.yaml `mimi:`; exact_gelu false,
    tts/config.rs:258-281): SEANet ratios 6, 5, 4 (200 Hz), 2 transformer layers, latents of
    inner_dim 32, decoder input outer_dim 512."""
    s = SeanetConfig(512, 1, 64, 1, (6, 5, 4), 7, 3, 3, 2, 0, 2)
    t = ProjectedTransformerConfig(512, 512, 512, 8, 2, 250, 2048)
    return MimiConfig(24_000, 12.5, s, s, t, t, 32, 512, False, parts)


def toy_mimi(parts: int = ENCODER | DECODER, pad_mode: int = 0) -> MimiConfig:
    """A small Mimi with every feature of the real ones (resnet blocks with dilation, strided
    and transposed convolutions, depthwise up-sampling, a windowed transformer, projections
    in and out of the transformer): 2 kHz, 12.5 Hz frames of 160 samples, 5 transformer
    steps per frame."""
    s = SeanetConfig(64, 1, 8, 2, (4, 2, 4), 5, 3, 3, 2, pad_mode, 2)
    t = ProjectedTransformerConfig(128, 64, 64, 2, 2, 6, 256)
    return MimiConfig(2_000, 12.5, s, s, t, t, 48, 64, True, parts)


class MimiState:
    """MimiEncoder / MimiDecoder states of max_batch streams (nn/mimi.rs:172-178, :253-259)."""

    def __init__(self, mimi: "Mimi", max_batch: int, max_frames: int):
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().svl_mimi_state_create(mimi.handle, max_batch, max_frames,
                                                    ctypes.byref(h)))
        self.handle, self.mimi = h.value, mimi
        self.max_batch, self.max_frames = max_batch, max_frames

    def reset(self, stream: int = -1):
        _lib.check(_lib.lib().svl_mimi_state_reset(self.handle, stream))

    def close(self):
        if self.handle:
            _lib.lib().svl_mimi_state_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Mimi:
    """MimiEncoder and MimiDecoder (nn/mimi.rs:133-272) on the GPU."""

    def __init__(self, cfg: MimiConfig, tensors: dict[str, np.ndarray], device: int = 0):
        self.cfg = cfg
        views, self._keep = tensor_views(tensors)
        h = ctypes.c_void_p()
        c = cfg.to_c()
        _lib.check(_lib.lib().svl_mimi_create(ctypes.byref(c), views, len(tensors), device,
                                              ctypes.byref(h)))
        self.handle = h.value

    @property
    def frame_size(self) -> int:
        return _lib.lib().svl_mimi_frame_size(self.handle)

    def init_state(self, max_batch: int = 1, max_frames: int = 1) -> MimiState:
        return MimiState(self, max_batch, max_frames)

    def encode_step(self, pcm, state: MimiState, stream=None):
        """pcm: a CUDA float32 tensor [batch][channels][frames * frame_size] ->
        latents [batch][inner_dim][frames] (a new CUDA tensor)."""
        import torch
        b, _, n = pcm.shape
        frames = n // self.frame_size
        out = torch.empty((b, self.cfg.inner_dim, frames), dtype=torch.float32, device=pcm.device)
        _call(_lib.lib().svl_mimi_encode_step_device, self.handle, state.handle, b, frames,
              ctypes.c_void_p(pcm.data_ptr()), ctypes.c_void_p(out.data_ptr()), stream=stream)
        return out

    def decode_step(self, latent, state: MimiState, stream=None):
        """latent: a CUDA float32 tensor [batch][outer_dim][frames] -> pcm
        [batch][channels][frames * frame_size]."""
        import torch
        b, _, frames = latent.shape
        out = torch.empty((b, self.cfg.decoder.channels, frames * self.frame_size),
                          dtype=torch.float32, device=latent.device)
        _call(_lib.lib().svl_mimi_decode_step_device, self.handle, state.handle, b, frames,
              ctypes.c_void_p(latent.data_ptr()), ctypes.c_void_p(out.data_ptr()), stream=stream)
        return out

    def decode_latent(self, latent, state: MimiState, emb_std=None, emb_mean=None, stream=None):
        """Tts::decode_latent (tts/mod.rs:441-447): latent, CUDA float32 [batch][frames][latent_dim]
        (FlowLm::step's layout), times emb_std plus emb_mean (CUDA [latent_dim], or None), through
        quantizer.output_proj, then decode_step -> pcm [batch][channels][frames * frame_size]."""
        import torch
        b, frames, _ = latent.shape
        out = torch.empty((b, self.cfg.decoder.channels, frames * self.frame_size),
                          dtype=torch.float32, device=latent.device)
        ptr = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
        _call(_lib.lib().svl_mimi_decode_latent_device, self.handle, state.handle, b, frames,
              ptr(latent), ptr(emb_std), ptr(emb_mean), ptr(out), stream=stream)
        return out

    def close(self):
        if self.handle:
            _lib.lib().svl_mimi_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Quantizer:
    """Quantizer::encode (stt/model.rs:84-170) on the GPU."""

    def __init__(self, n_q: int, bins: int, tensors: dict[str, np.ndarray], device: int = 0):
        self.n_q, self.bins = n_q, bins
        views, self._keep = tensor_views(tensors)
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().svl_rvq_create(n_q, bins, views, len(tensors), device,
                                             ctypes.byref(h)))
        self.handle = h.value

    def encode(self, latent, stream=None):
        """latent: CUDA float32 [batch][512][frames] -> codes uint32 as int32 [batch][frames][n_q]."""
        import torch
        b, _, frames = latent.shape
        out = torch.empty((b, frames, self.n_q), dtype=torch.int32, device=latent.device)
        _call(_lib.lib().svl_rvq_encode_device, self.handle, b, frames,
              ctypes.c_void_p(latent.data_ptr()), ctypes.c_void_p(out.data_ptr()), stream=stream)
        return out

    def close(self):
        if self.handle:
            _lib.lib().svl_rvq_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
