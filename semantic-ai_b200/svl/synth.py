"""Deterministic synthetic weights and inputs with the reference's tensor names.

There are no real checkpoints here, so every benchmark and parity run uses random-init
weights: N(0, std) from a per-tensor generator seeded by (seed, crc32(name)), which makes
each tensor independent of the order in which tensors are generated. Norm scales are 1 and
norm biases 0 (a documented choice), biases of linear layers N(0, std). Tensor names follow
stt/model.rs:224-231, nn/transformer.rs:206-218, :305-312, :429-432 and
tts/flow_lm.rs:78-124 of the reference.
"""
from __future__ import annotations

import concurrent.futures as cf
import math
import zlib

import numpy as np

from .config import FFN_GATED_SILU, NORM_RMS, SttConfig, TransformerConfig, TtsConfig


def tensor_rng(seed: int, name: str) -> np.random.Generator:
    return np.random.default_rng([seed, zlib.crc32(name.encode())])


def _normal(seed: int, name: str, shape, std: float) -> np.ndarray:
    a = tensor_rng(seed, name).standard_normal(int(np.prod(shape)), dtype=np.float32)
    a *= np.float32(std)
    return a.reshape(shape)


def transformer_specs(cfg: TransformerConfig, prefix: str = "transformer."):
    """(name, shape, kind) for every transformer tensor; kind is 'w' (random), 'one', 'zero'."""
    d, qd = cfg.d_model, cfg.num_heads * cfg.head_dim
    kvd = cfg.num_kv_heads * cfg.head_dim
    out = []
    for l in range(cfg.num_layers):
        p = f"{prefix}layers.{l}."
        for n in ("norm1", "norm2"):
            if cfg.norm_kind == NORM_RMS:
                out.append((f"{p}{n}.alpha", (1, 1, d), "one"))
            else:
                out.append((f"{p}{n}.weight", (d,), "one"))
                out.append((f"{p}{n}.bias", (d,), "zero"))
        if cfg.layer_scale:
            out.append((f"{p}layer_scale_1.scale", (d,), "w"))
            out.append((f"{p}layer_scale_2.scale", (d,), "w"))
        name = "self_attn.in_proj_weight" if cfg.norm_kind == NORM_RMS else "self_attn.in_proj.weight"
        out.append((p + name, (qd + 2 * kvd, d), "w"))
        out.append((p + "self_attn.out_proj.weight", (d, qd), "w"))
        if cfg.ffn_kind == FFN_GATED_SILU:
            out.append((p + "gating.linear_in.weight", (2 * cfg.ffn_hidden, d), "w"))
            out.append((p + "gating.linear_out.weight", (d, cfg.ffn_hidden), "w"))
        else:
            out.append((p + "linear1.weight", (cfg.ffn_hidden, d), "w"))
            out.append((p + "linear2.weight", (d, cfg.ffn_hidden), "w"))
    return out


def stt_specs(stt: SttConfig, cfg: TransformerConfig):
    d = cfg.d_model
    out = [("text_emb.weight", (stt.text_card + 1, d), "w")]
    out += [(f"emb.{c}.weight", (stt.card + 1, d), "w") for c in range(stt.n_q)]
    out += transformer_specs(cfg)
    out.append(("out_norm.alpha", (1, 1, d), "one"))
    out.append(("text_linear.weight", (stt.text_card, d), "w"))
    for i in range(stt.extra_heads_num_heads):
        out.append((f"extra_heads.{i}.weight", (stt.extra_heads_dim, d), "w"))
    return out


def tts_specs(cfg: TransformerConfig, tts: TtsConfig):
    d, dim, ld = cfg.d_model, tts.flow_dim, tts.latent_dim
    out = [("conditioner.embed.weight", (tts.text_bins + 1, d), "w"),
           ("input_linear.weight", (d, ld), "w")]
    out += transformer_specs(cfg)
    out += [("out_norm.weight", (d,), "one"), ("out_norm.bias", (d,), "zero"),
            ("out_eos.weight", (1, d), "w"), ("out_eos.bias", (1,), "w"),
            ("bos_emb", (ld,), "w"), ("emb_mean", (ld,), "zero"), ("emb_std", (ld,), "one")]
    n_time = {"lsd": 2, "flow_matching": 1}.get(tts.flow_kind, 0)
    for i in range(n_time):
        p = f"flow_net.time_embed.{i}."
        out += [(p + "freqs", (128,), "freqs"),
                (p + "mlp.0.weight", (dim, 256), "w"), (p + "mlp.0.bias", (dim,), "w"),
                (p + "mlp.2.weight", (dim, dim), "w"), (p + "mlp.2.bias", (dim,), "w"),
                (p + "mlp.3.alpha", (dim,), "one")]
    out += [("flow_net.cond_embed.weight", (dim, d), "w"), ("flow_net.cond_embed.bias", (dim,), "w"),
            ("flow_net.input_proj.weight", (dim, ld), "w"), ("flow_net.input_proj.bias", (dim,), "w")]
    for i in range(tts.flow_depth):
        p = f"flow_net.res_blocks.{i}."
        out += [(p + "in_ln.weight", (dim,), "one"), (p + "in_ln.bias", (dim,), "zero"),
                (p + "mlp.0.weight", (dim, dim), "w"), (p + "mlp.0.bias", (dim,), "w"),
                (p + "mlp.2.weight", (dim, dim), "w"), (p + "mlp.2.bias", (dim,), "w"),
                (p + "adaLN_modulation.1.weight", (3 * dim, dim), "w"),
                (p + "adaLN_modulation.1.bias", (3 * dim,), "w")]
    p = "flow_net.final_layer."
    out += [(p + "adaLN_modulation.1.weight", (2 * dim, dim), "w"),
            (p + "adaLN_modulation.1.bias", (2 * dim,), "w"),
            (p + "linear.weight", (ld, dim), "w"), (p + "linear.bias", (ld,), "w")]
    return out


def materialize(specs, seed: int = 0, std: float = 0.02, threads: int = 8) -> dict[str, np.ndarray]:
    """Generates every tensor of `specs` (in parallel; numpy releases the GIL)."""
    def make(spec):
        name, shape, kind = spec
        if kind == "one":
            return name, np.ones(shape, np.float32)
        if kind == "zero":
            return name, np.zeros(shape, np.float32)
        if kind == "freqs":
            # Sinusoidal timestep frequencies exp(-ln(10000) i / 128), i < 128.
            i = np.arange(shape[0], dtype=np.float64)
            return name, np.exp(-math.log(10_000.0) * i / shape[0]).astype(np.float32)
        return name, _normal(seed, name, shape, std)

    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        return dict(ex.map(make, specs))


def stt_weights(stt: SttConfig, cfg: TransformerConfig, seed: int = 0, std: float = 0.02):
    return materialize(stt_specs(stt, cfg), seed, std)


def tts_weights(cfg: TransformerConfig, tts: TtsConfig, seed: int = 0, std: float = 0.02):
    return materialize(tts_specs(cfg, tts), seed, std)


def audio_tokens(stt: SttConfig, frames: int, seed: int = 1, streams: int | None = None) -> np.ndarray:
    """Uniform audio tokens in [0, card): [frames][n_q], or [frames][streams][n_q] with stream
    s drawn from seed + s."""
    if streams is None:
        return np.random.default_rng(seed).integers(0, stt.card, size=(frames, stt.n_q), dtype=np.uint32)
    out = np.empty((frames, streams, stt.n_q), np.uint32)
    for s in range(streams):
        out[:, s] = np.random.default_rng(seed + s).integers(0, stt.card, size=(frames, stt.n_q), dtype=np.uint32)
    return out
