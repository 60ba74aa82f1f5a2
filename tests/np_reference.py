"""An independent float64 numpy restatement of the streaming LM step, used to pin the C oracle.

It follows the reference's structure (crates/semantic-voice-local/src): the embedding sum of
LanguageModel::step (stt/model.rs:246-250), Transformer::forward / Layer::forward
(nn/transformer.rs:139-250) with RMSNorm or LayerNorm, fused QKV, interleaved RoPE
(rope_i, :339-340), windowed causal attention (nn/kernels/attention.rs:81-169), gated SiLU or
plain GELU feed-forward (:418-464) and layer scale, then out_norm and text_linear
(stt/model.rs:252-257). Everything is computed in float64, so the oracle (f32, the
reference's summation order) must agree to f32 rounding.
"""
from __future__ import annotations

import numpy as np


def inv_freq(head_dim: int, max_period: float) -> np.ndarray:
    half = head_dim // 2
    return np.array([np.float32(np.exp(-np.log(max_period) * 2.0 * i / head_dim)) for i in range(half)],
                    np.float64)


class Backbone:
    """Transformer::forward over a growing per-stream cache, float64."""

    def __init__(self, cfg, w: dict[str, np.ndarray]):
        self.cfg = cfg
        self.w = {k: v.astype(np.float64) for k, v in w.items()}
        self.inv = inv_freq(cfg.head_dim, cfg.max_period)
        self.k = [[] for _ in range(cfg.num_layers)]
        self.v = [[] for _ in range(cfg.num_layers)]
        self.pos = 0

    def norm(self, x, prefix):
        c, w = self.cfg, self.w
        if c.norm_kind == 1:  # RMSNorm
            return x / np.sqrt((x * x).mean() + c.norm_eps) * w[prefix + ".alpha"].reshape(-1)
        mu = x.mean()
        var = ((x - mu) ** 2).mean()
        return (x - mu) / np.sqrt(var + c.norm_eps) * w[prefix + ".weight"] + w[prefix + ".bias"]

    def rope(self, a, pos):
        cs, sn = np.cos(pos * self.inv), np.sin(pos * self.inv)
        a0, a1 = a[:, 0::2], a[:, 1::2]
        r = np.empty_like(a)
        r[:, 0::2] = a0 * cs - a1 * sn
        r[:, 1::2] = a0 * sn + a1 * cs
        return r

    def forward_token(self, x: np.ndarray) -> np.ndarray:
        c, w = self.cfg, self.w
        H, kvh, hd = c.num_heads, c.num_kv_heads, c.head_dim
        x = x.astype(np.float64).copy()
        for l in range(c.num_layers):
            p = f"transformer.layers.{l}."
            h = self.norm(x, p + "norm1")
            win = p + "self_attn.in_proj_weight"
            if win not in w:
                win = p + "self_attn.in_proj.weight"
            qkv = w[win] @ h
            q = self.rope(qkv[:H * hd].reshape(H, hd), self.pos)
            k = self.rope(qkv[H * hd:(H + kvh) * hd].reshape(kvh, hd), self.pos)
            v = qkv[(H + kvh) * hd:].reshape(kvh, hd)
            self.k[l].append(k)
            self.v[l].append(v)
            n = len(self.k[l]) if not c.context else min(len(self.k[l]), c.context)
            ks = np.stack(self.k[l][-n:], 1)  # kvh, T, hd
            vs = np.stack(self.v[l][-n:], 1)
            rep = H // kvh
            ks, vs = np.repeat(ks, rep, axis=0), np.repeat(vs, rep, axis=0)
            sc = np.einsum("hd,htd->ht", q, ks) / np.sqrt(hd)
            pr = np.exp(sc - sc.max(1, keepdims=True))
            pr /= pr.sum(1, keepdims=True)
            att = np.einsum("ht,htd->hd", pr, vs).reshape(-1)
            y = w[p + "self_attn.out_proj.weight"] @ att
            if c.layer_scale:
                y = y * w[p + "layer_scale_1.scale"]
            x = x + y
            h = self.norm(x, p + "norm2")
            if c.ffn_kind == 2:  # gated SiLU
                F = c.ffn_hidden
                z = w[p + "gating.linear_in.weight"] @ h
                y = w[p + "gating.linear_out.weight"] @ (z[:F] / (1 + np.exp(-z[:F])) * z[F:])
            else:
                z = w[p + "linear1.weight"] @ h
                if c.ffn_kind == 0:  # GELU tanh
                    g = 0.5 * z * (1 + np.tanh(np.sqrt(2 / np.pi) * (z + 0.044715 * z ** 3)))
                else:
                    from math import erf
                    g = np.array([0.5 * t * (1 + erf(t / np.sqrt(2))) for t in z])
                y = w[p + "linear2.weight"] @ g
            if c.layer_scale:
                y = y * w[p + "layer_scale_2.scale"]
            x = x + y
        self.pos += 1
        return x


def stt_logits(stt, cfg, w, text_tokens, audio_frames) -> np.ndarray:
    """LanguageModel::step logits for the given teacher-forced inputs, float64."""
    bb = Backbone(cfg, w)
    out = []
    for tt, au in zip(text_tokens, audio_frames):
        x = w["text_emb.weight"][tt].astype(np.float64).copy()
        for c in range(stt.n_q):
            x = x + w[f"emb.{c}.weight"][au[c]]
        x = bb.forward_token(x)
        ys = x / np.sqrt((x * x).mean() + 1e-8) * w["out_norm.alpha"].reshape(-1)
        out.append(w["text_linear.weight"].astype(np.float64) @ ys)
    return np.array(out)
