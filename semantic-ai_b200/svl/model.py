"""Python mirror of the reference's model API over the C ABI.

LanguageModel mirrors stt/model.rs:176-277 (new, init_state, step), Transformer::forward
mirrors nn/transformer.rs:139, State mirrors TransformerState (nn/transformer.rs:53-104) for
a batch of independent streams. Everything runs on the GPU through libsvl_b200.so.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from .config import CTensorView, SttConfig, TransformerConfig, TtsConfig


def _u32(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))


def _f32(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def tensor_views(tensors: dict[str, np.ndarray]):
    """An svl_tensor_view array over host f32 tensors (kept alive by the returned list)."""
    keep = []
    views = (CTensorView * len(tensors))()
    for i, (name, arr) in enumerate(tensors.items()):
        a = np.ascontiguousarray(arr, dtype=np.float32)
        nb = name.encode()
        keep += [a, nb]
        views[i] = CTensorView(nb, a.ctypes.data, a.size)
    return views, keep


class State:
    """Per-stream KV rings and positions for up to max_batch streams."""

    handle = None

    def __init__(self, model: "_Model", max_batch: int = 1, max_positions: int = 0,
                 reference_order: bool = False, flags: int = 0):
        h = ctypes.c_void_p()
        flags |= _lib.STATE_REFERENCE_ORDER if reference_order else 0
        _lib.check(_lib.lib().svl_state_create_ex(model.handle, max_batch, max_positions, flags,
                                                  ctypes.byref(h)))
        self.reference_order = reference_order
        self.handle = h
        self.model = model
        self.max_batch = max_batch
        # Bound now: at interpreter exit the module globals may already be gone.
        self._destroy = _lib.lib().svl_state_destroy

    def close(self):
        if self.handle:
            self._destroy(self.handle)
            self.handle = None

    __del__ = close

    def reset(self, stream: int = -1):
        _lib.check(_lib.lib().svl_state_reset(self.handle, stream))

    def position(self, stream: int = 0) -> int:
        p = ctypes.c_int32()
        _lib.check(_lib.lib().svl_state_position(self.handle, stream, ctypes.byref(p)))
        return p.value

    def copy_from(self, other: "State", src: int = 0, dst: int = 0):
        _lib.check(_lib.lib().svl_state_copy(self.handle, dst, other.handle, src))

    def layer_caches(self, stream: int = 0):
        """TransformerState::layer_caches: per layer (k, v) as [kv_heads, len, head_dim]."""
        c = self.model.cfg
        cap = c.context or self.model.max_positions_hint
        out = []
        for l in range(c.num_layers):
            k = np.zeros(c.num_kv_heads * max(cap, 1) * c.head_dim, np.float32)
            v = np.zeros_like(k)
            n = ctypes.c_int32()
            _lib.check(_lib.lib().svl_state_export(self.handle, stream, l, _f32(k), _f32(v),
                                                   ctypes.byref(n), None))
            shape = (c.num_kv_heads, n.value, c.head_dim)
            out.append((k[: np.prod(shape)].reshape(shape), v[: np.prod(shape)].reshape(shape)))
        return out

    def save_voice(self, path, stream: int = 0):
        """Voice::save (tts/voice.rs:78-99): this stream's KV state as a safetensors voice."""
        _lib.check(_lib.lib().svl_voice_save(self.handle, stream, str(path).encode()))

    def load_voice(self, path, streams=(0,)):
        """Voice::load (tts/voice.rs:101-149) into several streams at once."""
        s = np.ascontiguousarray(streams, np.int32)
        _lib.check(_lib.lib().svl_voice_load(self.handle, s.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                             s.size, str(path).encode()))

    def load_layer_caches(self, caches, position: int, stream: int = 0):
        """TransformerState::from_layer_caches for one stream."""
        for l, (k, v) in enumerate(caches):
            k = np.ascontiguousarray(k, np.float32)
            v = np.ascontiguousarray(v, np.float32)
            _lib.check(_lib.lib().svl_state_import(self.handle, stream, l, _f32(k), _f32(v),
                                                   k.shape[1], position))


class _Model:
    handle = None
    max_positions_hint = 0

    _destroy = None

    def close(self):
        if self.handle:
            (self._destroy or _lib.lib().svl_model_destroy)(self.handle)
            self.handle = None

    __del__ = close

    @property
    def weight_bytes(self) -> int:
        return _lib.lib().svl_model_weight_bytes(self.handle)

    def init_state(self, max_batch: int = 1, max_positions: int = 0,
                   reference_order: bool = False, flags: int = 0) -> State:
        """Transformer::init_state for max_batch streams. reference_order: every reduction in
        the reference CPU path's order (svl_state_create_ex, SVL_STATE_REFERENCE_ORDER); flags:
        further svl_state_create_ex options."""
        self.max_positions_hint = max(self.max_positions_hint, max_positions)
        return State(self, max_batch, max_positions, reference_order, flags)

    def forward(self, xs: np.ndarray, state: State, stream: int = 0) -> np.ndarray:
        """Transformer::forward for one stream: xs [t, d_model] -> [t, d_model]."""
        x = np.ascontiguousarray(xs, np.float32).copy()
        _lib.check(_lib.lib().svl_transformer_forward(self.handle, state.handle, stream, _f32(x),
                                                      x.shape[0]))
        return x


class LanguageModel(_Model):
    """LanguageModel (stt/model.rs:176-277) on a B200."""

    def __init__(self, stt: SttConfig, cfg: TransformerConfig, tensors: dict[str, np.ndarray],
                 device: int = 0):
        self.stt, self.cfg = stt, cfg
        views, keep = tensor_views(tensors)
        h = ctypes.c_void_p()
        c, s = cfg.to_c(), stt.to_c()
        _lib.check(_lib.lib().svl_stt_model_create(ctypes.byref(c), ctypes.byref(s), views,
                                                   len(tensors), device, ctypes.byref(h)))
        self.handle = h
        self._destroy = _lib.lib().svl_model_destroy
        del keep

    def step(self, text_tokens, audio_tokens, state: State, logits: bool = False,
             extra: bool = False):
        """LanguageModel::step for streams 0..B-1: text [B], audio [B, n_q] -> tokens [B]
        (and logits [B, text_card], extra-head probabilities [B, n_extra] on request)."""
        t = np.ascontiguousarray(np.atleast_1d(text_tokens), np.uint32)
        b = t.shape[0]
        a = np.ascontiguousarray(audio_tokens, np.uint32).reshape(b, self.stt.n_q)
        out = np.zeros(b, np.uint32)
        lg = np.zeros((b, self.stt.text_card), np.float32) if logits else None
        ex = np.zeros((b, max(self.stt.extra_heads_num_heads, 1)), np.float32) if extra else None
        _lib.check(_lib.lib().svl_stt_step(self.handle, state.handle, b, _u32(t), _u32(a), _u32(out),
                                           _f32(lg) if lg is not None else None,
                                           _f32(ex) if ex is not None else None))
        res = [out]
        if logits:
            res.append(lg)
        if extra:
            res.append(ex)
        return res[0] if len(res) == 1 else tuple(res)

    def run_frames(self, audio: np.ndarray, state: State, extra: bool = False):
        """The Recognizer token loop: audio [frames, B, n_q] -> greedy tokens [frames, B] (and,
        with extra=True, the extra heads' p[0] [frames, B, n_extra])."""
        a = np.ascontiguousarray(audio, np.uint32)
        if a.ndim == 2:
            a = a[:, None, :]
        f, b = a.shape[:2]
        out = np.zeros((f, b), np.uint32)
        if not extra:
            _lib.check(_lib.lib().svl_stt_run_frames(self.handle, state.handle, b, f, _u32(a), _u32(out)))
            return out
        ex = np.zeros((f, b, max(self.stt.extra_heads_num_heads, 1)), np.float32)
        _lib.check(_lib.lib().svl_stt_run_frames_ex(self.handle, state.handle, b, f, _u32(a), _u32(out),
                                                    _f32(ex) if self.stt.extra_heads_num_heads else None))
        return out, ex[:, :, : self.stt.extra_heads_num_heads]


class FlowLm(_Model):
    """FlowLm (tts/flow_lm.rs:24-204) on a B200."""

    def __init__(self, cfg: TransformerConfig, tts: TtsConfig, tensors: dict[str, np.ndarray],
                 device: int = 0):
        self.cfg, self.tts = cfg, tts
        views, keep = tensor_views(tensors)
        h = ctypes.c_void_p()
        c, t = cfg.to_c(), tts.to_c()
        _lib.check(_lib.lib().svl_tts_model_create(ctypes.byref(c), ctypes.byref(t), views,
                                                   len(tensors), device, ctypes.byref(h)))
        self.handle = h
        self._destroy = _lib.lib().svl_model_destroy
        del keep

    def prompt_text(self, tokens, state: State, stream: int = 0):
        """FlowLm::prompt_text for one stream: tokens [n]."""
        t = np.ascontiguousarray(tokens, np.uint32)
        _lib.check(_lib.lib().svl_tts_prompt_text(self.handle, state.handle, stream, _u32(t), t.size))

    def prompt_text_batch(self, tokens, state: State):
        """FlowLm::prompt_text for streams 0..B-1 at once: tokens [B, n]."""
        t = np.ascontiguousarray(tokens, np.uint32)
        _lib.check(_lib.lib().svl_tts_prompt_text_batch(self.handle, state.handle, t.shape[0],
                                                        _u32(t), t.shape[1]))

    def step(self, latent, noise, state: State, decode_steps: int = 1):
        """FlowLm::step for streams 0..B-1: latent [B, latent] (None = BOS), noise [B, latent]
        -> (next latent [B, latent], eos logits [B])."""
        n = np.ascontiguousarray(noise, np.float32)
        b = n.shape[0]
        lat = None if latent is None else np.ascontiguousarray(latent, np.float32)
        out = np.zeros_like(n)
        eos = np.zeros(b, np.float32)
        _lib.check(_lib.lib().svl_tts_step(self.handle, state.handle, b,
                                           _f32(lat) if lat is not None else None, _f32(n),
                                           decode_steps, _f32(out), _f32(eos)))
        return out, eos
