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


# ------------------------------------------------------------------ Mimi and the quantizer

def _conv_spec(prefix: str, cin: int, cout: int, k: int, bias: bool = True):
    out = [(prefix + ".weight", (cout, cin, k), ("fan", cin * k))]
    if bias:
        out.append((prefix + ".bias", (cout,), "w"))
    return out


def _resnet_spec(prefix: str, dim: int, seanet):
    hidden = dim // seanet.compress
    return (_conv_spec(prefix + ".block.1.conv", dim, hidden, seanet.residual_kernel_size)
            + _conv_spec(prefix + ".block.3.conv", hidden, dim, 1))


def _ptrans_spec(prefix: str, p):
    from .config import FFN_PLAIN_GELU_ERF, NORM_LAYER, TransformerConfig
    cfg = TransformerConfig(d_model=p.d_model, num_layers=p.num_layers, num_heads=p.num_heads,
                            num_kv_heads=p.num_heads, head_dim=p.d_model // p.num_heads,
                            ffn_kind=FFN_PLAIN_GELU_ERF, ffn_hidden=p.dim_feedforward,
                            norm_kind=NORM_LAYER, norm_eps=1e-5, layer_scale=True)
    out = [(n.replace(".in_proj.weight", ".in_proj_weight"), s, k)
           for n, s, k in transformer_specs(cfg, prefix + ".transformer.")]
    if p.input_dimension != p.d_model:
        out.append((prefix + ".input_proj.weight", (p.d_model, p.input_dimension, 1), ("fan", p.input_dimension)))
    if p.output_dimension != p.d_model:
        out.append((prefix + ".output_projs.0.weight", (p.output_dimension, p.d_model, 1), ("fan", p.d_model)))
    return out


def mimi_specs(cfg, latent_dim: int | None = None):
    """Tensor names of MimiEncoder::new / MimiDecoder::new (nn/mimi.rs:140-166, :229-251) after
    load_mimi_weights' renaming (nn/mod.rs:26-52). Convolutions are N(0, 1 / fan_in) so that
    activations keep their scale through the SEANet stacks."""
    from .codec import DECODER, ENCODER
    out = []
    if cfg.parts & ENCODER:
        s, li, mult = cfg.encoder, 0, 1
        out += _conv_spec(f"encoder.model.{li}.conv", s.channels, s.n_filters, s.kernel_size)
        li += 1
        for r in reversed(s.ratios):
            dim = mult * s.n_filters
            for _ in range(s.n_residual_layers):
                out += _resnet_spec(f"encoder.model.{li}", dim, s)
                li += 1
            li += 1
            out += _conv_spec(f"encoder.model.{li}.conv", dim, 2 * dim, 2 * r)
            li += 1
            mult *= 2
        li += 1
        out += _conv_spec(f"encoder.model.{li}.conv", mult * s.n_filters, s.dimension, s.last_kernel_size)
        out += _ptrans_spec("encoder_transformer", cfg.encoder_transformer)
        st = cfg.resample_stride(s)
        if st > 1:
            out += _conv_spec("downsample.conv.conv", cfg.encoder_transformer.output_dimension,
                              cfg.inner_dim, 2 * st, bias=False)
    if cfg.parts & DECODER:
        s = cfg.decoder
        st = cfg.resample_stride(s)
        if latent_dim:  # Pocket TTS: the flow LM's latents into the decoder (tts/mod.rs:218-224)
            out.append(("quantizer.output_proj.weight", (cfg.outer_dim, latent_dim, 1), ("fan", latent_dim)))
        if st > 1:
            out.append(("upsample.convtr.convtr.weight", (cfg.outer_dim, 1, 2 * st), ("fan", 2)))
        out += _ptrans_spec("decoder_transformer", cfg.decoder_transformer)
        mult, li = 1 << len(s.ratios), 0
        out += _conv_spec(f"decoder.model.{li}.conv", s.dimension, mult * s.n_filters, s.kernel_size)
        li += 1
        for r in s.ratios:
            dim = mult * s.n_filters
            li += 1
            out += [(f"decoder.model.{li}.convtr.weight", (dim, dim // 2, 2 * r), ("fan", dim * 2)),
                    (f"decoder.model.{li}.convtr.bias", (dim // 2,), "w")]
            li += 1
            for _ in range(s.n_residual_layers):
                out += _resnet_spec(f"decoder.model.{li}", dim // 2, s)
                li += 1
            mult //= 2
        li += 1
        out += _conv_spec(f"decoder.model.{li}.conv", s.n_filters, s.channels, s.last_kernel_size)
    return out


def rvq_specs(n_q: int, bins: int):
    """Quantizer::new's tensors (stt/model.rs:92-157): input projections [256][512][1], and per
    codebook embedding_sum [bins][256] (N(0, 1) times the usage) and cluster_usage [bins] (uniform
    in [0.5, 2], one entry of the first codebook below the 1e-5 floor)."""
    out = [("quantizer.rvq_first.input_proj.weight", (256, 512, 1), ("fan", 512))]
    if n_q > 1:
        out.append(("quantizer.rvq_rest.input_proj.weight", (256, 512, 1), ("fan", 512)))
    for k in range(n_q):
        pre = ("quantizer.rvq_first.vq.layers.0._codebook." if k == 0
               else f"quantizer.rvq_rest.vq.layers.{k - 1}._codebook.")
        out += [(pre + "embedding_sum", (bins, 256), "embsum"), (pre + "cluster_usage", (bins,), "usage")]
    return out


def materialize_codec(specs, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """materialize() with the codec kinds: ("fan", n) is N(0, 1 / n); "usage" uniform in
    [0.5, 2]; "embsum" N(0, 1) scaled by the matching usage row."""
    out = {}
    for name, shape, kind in specs:
        if isinstance(kind, tuple) and kind[0] == "fan":
            out[name] = _normal(seed, name, shape, 1.0 / math.sqrt(kind[1]))
        elif kind == "usage":
            u = tensor_rng(seed, name).uniform(0.5, 2.0, size=shape).astype(np.float32)
            if name.startswith("quantizer.rvq_first"):
                u[3] = 1e-7  # below the floor of Codebook::new
            out[name] = u
        elif kind == "embsum":
            out[name] = _normal(seed, name, shape, 1.0)
        else:
            out.update(materialize([(name, shape, kind)], seed, std, threads=1))
    for name in list(out):
        if name.endswith("embedding_sum"):
            usage = out[name[: -len("embedding_sum")] + "cluster_usage"]
            out[name] = (out[name] * np.maximum(usage, 1e-5)[:, None]).astype(np.float32)
    return out


def mimi_weights(cfg, seed: int = 0, latent_dim: int | None = None):
    return materialize_codec(mimi_specs(cfg, latent_dim), seed)


def rvq_weights(n_q: int, bins: int, seed: int = 0):
    return materialize_codec(rvq_specs(n_q, bins), seed)
