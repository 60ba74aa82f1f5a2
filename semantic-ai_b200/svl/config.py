"""Model configs, mirroring the reference's config structs.

TransformerConfig follows nn/transformer.rs:27-41; SttConfig follows stt/model.rs:17-43 and
LanguageModel::new's derivation of the transformer config (stt/model.rs:196-216);
TtsConfig holds the FlowLmConfig fields the step uses (tts/config.rs:177-219). Paths are
relative to crates/semantic-voice-local/src/ of the reference.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, replace

FFN_PLAIN_GELU_TANH, FFN_PLAIN_GELU_ERF, FFN_GATED_SILU = 0, 1, 2
NORM_LAYER, NORM_RMS = 0, 1
DTYPES = {"f32": 0, "bf16": 1, "q8_0": 2, "q4_1": 3}
FLOW_KINDS = {"lsd": 0, "flow_matching": 1, "drifting": 2, "pointwise": 3}


class CTransformerConfig(ctypes.Structure):
    """svl_transformer_config (include/svl_cuda.h) == orc_tcfg (oracle/svl_oracle.h)."""
    _fields_ = [
        ("d_model", ctypes.c_int32), ("num_layers", ctypes.c_int32),
        ("num_heads", ctypes.c_int32), ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("ffn_kind", ctypes.c_int32),
        ("ffn_hidden", ctypes.c_int32), ("norm_kind", ctypes.c_int32),
        ("norm_eps", ctypes.c_float), ("layer_scale", ctypes.c_int32),
        ("context", ctypes.c_int32), ("weight_dtype", ctypes.c_int32),
        ("kv_dtype", ctypes.c_int32), ("_pad", ctypes.c_int32),
        ("max_period", ctypes.c_double),
    ]


class CSttConfig(ctypes.Structure):
    _fields_ = [("card", ctypes.c_int32), ("n_q", ctypes.c_int32), ("text_card", ctypes.c_int32),
                ("extra_heads_num", ctypes.c_int32), ("extra_heads_dim", ctypes.c_int32),
                ("_pad", ctypes.c_int32)]


class CTtsConfig(ctypes.Structure):
    _fields_ = [("latent_dim", ctypes.c_int32), ("flow_dim", ctypes.c_int32),
                ("flow_depth", ctypes.c_int32), ("flow_kind", ctypes.c_int32),
                ("text_bins", ctypes.c_int32), ("_pad", ctypes.c_int32)]


class CTensorView(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("data", ctypes.c_void_p), ("numel", ctypes.c_int64)]


@dataclass(frozen=True)
class TransformerConfig:
    """nn/transformer.rs:27-41. `quantize` is generalised to weight_dtype."""
    d_model: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    ffn_kind: int
    ffn_hidden: int
    norm_kind: int
    norm_eps: float
    layer_scale: bool = False
    context: int | None = None
    max_period: float = 10_000.0
    weight_dtype: str = "f32"
    kv_dtype: str = "f32"

    def to_c(self) -> CTransformerConfig:
        return CTransformerConfig(
            self.d_model, self.num_layers, self.num_heads, self.num_kv_heads, self.head_dim,
            self.ffn_kind, self.ffn_hidden, self.norm_kind, self.norm_eps,
            int(self.layer_scale), int(self.context or 0), DTYPES[self.weight_dtype],
            DTYPES[self.kv_dtype], 0, float(self.max_period))

    def with_dtypes(self, weight_dtype: str, kv_dtype: str | None = None) -> "TransformerConfig":
        return replace(self, weight_dtype=weight_dtype, kv_dtype=kv_dtype or self.kv_dtype)


@dataclass(frozen=True)
class SttConfig:
    """stt/model.rs:17-43 (the language-model fields)."""
    card: int
    n_q: int
    dim: int
    text_card: int
    num_heads: int
    num_layers: int
    hidden_scale: float
    context: int
    max_period: float
    extra_heads_num_heads: int = 0
    extra_heads_dim: int = 0

    def transformer(self, weight_dtype: str = "f32", kv_dtype: str = "f32") -> TransformerConfig:
        """LanguageModel::new (stt/model.rs:201-216)."""
        feed_forward = int(self.hidden_scale * self.dim)
        return TransformerConfig(
            d_model=self.dim, num_layers=self.num_layers, num_heads=self.num_heads,
            num_kv_heads=self.num_heads, head_dim=self.dim // self.num_heads,
            ffn_kind=FFN_GATED_SILU, ffn_hidden=2 * feed_forward // 3, norm_kind=NORM_RMS,
            norm_eps=1e-8, layer_scale=False, context=self.context, max_period=self.max_period,
            weight_dtype=weight_dtype, kv_dtype=kv_dtype)

    def to_c(self) -> CSttConfig:
        return CSttConfig(self.card, self.n_q, self.text_card, self.extra_heads_num_heads,
                          self.extra_heads_dim, 0)


@dataclass(frozen=True)
class TtsConfig:
    """FlowLmConfig fields used by FlowLm::step (tts/config.rs:177-219)."""
    latent_dim: int
    flow_dim: int
    flow_depth: int
    flow_kind: str
    text_bins: int

    def to_c(self) -> CTtsConfig:
        return CTtsConfig(self.latent_dim, self.flow_dim, self.flow_depth,
                          FLOW_KINDS[self.flow_kind], self.text_bins, 0)


# ------------------------------------------------------------------ presets

def stt_1b(**kw) -> SttConfig:
    """STT-1b: d 2048, 16 layers, 16 heads x 128, SwiGLU 5632, window 750, RoPE 1e5."""
    return SttConfig(card=2048, n_q=32, dim=2048, text_card=8000, num_heads=16, num_layers=16,
                     hidden_scale=4.125, context=750, max_period=100_000.0, **kw)


def stt_2b6(**kw) -> SttConfig:
    """STT-2.6b: d 2560, 24 layers, 20 heads x 128, SwiGLU 10240, window 375, text 4001."""
    return SttConfig(card=2048, n_q=32, dim=2560, text_card=4000, num_heads=20, num_layers=24,
                     hidden_scale=6.0, context=375, max_period=100_000.0, **kw)


def stt_toy(**kw) -> SttConfig:
    """A small STT-shaped model for fast parity runs (head_dim 64 and 128 are the kernel
    shapes; 2 heads x 64 here)."""
    base = dict(card=64, n_q=4, dim=128, text_card=100, num_heads=2, num_layers=2,
                hidden_scale=4.125, context=12, max_period=100_000.0)
    base.update(kw)
    return SttConfig(**base)


def pocket_tts() -> tuple[TransformerConfig, TtsConfig]:
    """Pocket-TTS english (configs/tts/english.yaml; FlowLm::new, tts/flow_lm.rs:56-71):
    d 1024, 6 layers, 16 heads x 64, plain GELU-tanh FFN 4096, LayerNorm, no window."""
    t = TransformerConfig(d_model=1024, num_layers=6, num_heads=16, num_kv_heads=16, head_dim=64,
                          ffn_kind=FFN_PLAIN_GELU_TANH, ffn_hidden=4096, norm_kind=NORM_LAYER,
                          norm_eps=1e-5, layer_scale=False, context=None, max_period=10_000.0)
    return t, TtsConfig(latent_dim=32, flow_dim=512, flow_depth=6, flow_kind="lsd", text_bins=4000)


def tts_toy(flow_kind: str = "lsd", weight_dtype: str = "f32", kv_dtype: str = "f32"):
    """A small Pocket-TTS-shaped model for fast parity runs: d 128, 2 layers, 2 heads x 64,
    GELU-tanh FFN 512, LayerNorm, no window; flow head width 64, depth 2, latent 32."""
    t = TransformerConfig(d_model=128, num_layers=2, num_heads=2, num_kv_heads=2, head_dim=64,
                          ffn_kind=FFN_PLAIN_GELU_TANH, ffn_hidden=512, norm_kind=NORM_LAYER,
                          norm_eps=1e-5, layer_scale=False, context=None, max_period=10_000.0,
                          weight_dtype=weight_dtype, kv_dtype=kv_dtype)
    return t, TtsConfig(latent_dim=32, flow_dim=64, flow_depth=2, flow_kind=flow_kind, text_bins=50)


def kv_bytes_per_stream(cfg: TransformerConfig, fill: int) -> int:
    el = 2 if cfg.kv_dtype == "bf16" else 4
    return cfg.num_layers * 2 * fill * cfg.num_kv_heads * cfg.head_dim * el


def param_count(cfg: TransformerConfig) -> int:
    d, qd = cfg.d_model, cfg.num_heads * cfg.head_dim
    kvd = cfg.num_kv_heads * cfg.head_dim
    ff = 3 * cfg.ffn_hidden * d if cfg.ffn_kind == FFN_GATED_SILU else 2 * cfg.ffn_hidden * d
    return cfg.num_layers * ((qd + 2 * kvd) * d + d * qd + ff)


def inv_freq(cfg: TransformerConfig) -> list[float]:
    half = cfg.head_dim // 2
    return [math.exp(-math.log(cfg.max_period) * 2.0 * i / cfg.head_dim) for i in range(half)]
