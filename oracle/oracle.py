"""ctypes wrapper of the CPU oracle (oracle/libsvl_oracle.so).

TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and bench.py's CPU legs as
the checker and the timed CPU baseline; the product never imports it. See svl_oracle.h for
the parity status of the restatement.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libsvl_oracle.so"

_lib = None


class _Tensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("data", ctypes.c_void_p), ("numel", ctypes.c_int64)]


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        l = ctypes.CDLL(str(LIB_PATH))
        P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        FP = ctypes.POINTER(ctypes.c_float)
        UP = ctypes.POINTER(ctypes.c_uint32)
        sig = {
            "orc_lm_create": (P, [I, P, P, P, ctypes.POINTER(_Tensor), I]),
            "orc_lm_free": (None, [P]),
            "orc_state_create": (P, [P]),
            "orc_state_duplicate": (P, [P]),
            "orc_state_free": (None, [P]),
            "orc_state_position": (I, [P]),
            "orc_last_error": (ctypes.c_char_p, []),
            "orc_set_threads": (None, [I]),
            "orc_set_reduction_variant": (None, [I]),
            "orc_stt_step": (I, [P, P, ctypes.c_uint32, UP, UP, FP, FP]),
            "orc_transformer_forward": (I, [P, P, FP, I]),
            "orc_tts_step": (I, [P, P, FP, FP, F, FP, FP]),
            "orc_tts_prompt_text": (I, [P, P, UP, I]),
            "orc_dot": (F, [FP, FP, I]),
            "orc_dot_scalar": (F, [FP, FP, I]),
            "orc_exp": (F, [F]),
            "orc_silu": (F, [F]),
            "orc_gelu_tanh": (F, [F]),
            "orc_matvec": (None, [FP, FP, FP, I, I, FP]),
            "orc_attention": (None, [FP, FP, FP, I, I, I, I, I, ctypes.c_int64, ctypes.c_int64,
                                     I, I, I, FP]),
            "orc_rms_norm": (None, [FP, FP, I, F, FP]),
            "orc_layer_norm": (None, [FP, FP, FP, I, F, FP]),
            "orc_quantize_q8_0": (None, [FP, ctypes.c_int64, P]),
            "orc_quantize_q4_1": (None, [FP, ctypes.c_int64, P]),
            "orc_matvec_q8_0": (None, [FP, P, I, I, FP]),
            "orc_matvec_q4_1": (None, [FP, P, I, I, FP]),
            "orc_vec_dot_q8_0": (F, [P, P, I]),
            "orc_vec_dot_q8_0_scalar": (F, [P, P, I]),
            "orc_f32_to_f16": (ctypes.c_uint16, [F]),
            "orc_f16_to_f32": (F, [ctypes.c_uint16]),
            "orc_round_bf16": (F, [F]),
            "orc_elu": (F, [F]),
            "orc_transformer_create": (P, [P, ctypes.c_char_p, ctypes.POINTER(_Tensor), I]),
            "orc_conv1d_stream": (I, [I, I, I, I, I, I, FP, FP, FP, ctypes.POINTER(I), FP, I, I,
                                      FP, FP]),
            "orc_convtr1d_stream": (I, [I, I, I, I, I, FP, FP, FP, FP, I, I, FP]),
            "orc_mimi_create": (P, [P, ctypes.POINTER(_Tensor), I]),
            "orc_mimi_free": (None, [P]),
            "orc_mimi_frame_size": (I, [P]),
            "orc_mimi_state_create": (P, [P]),
            "orc_mimi_state_free": (None, [P]),
            "orc_mimi_encode_step": (I, [P, P, FP, I, FP]),
            "orc_mimi_decode_step": (I, [P, P, FP, I, FP]),
            "orc_mimi_decode_latent": (I, [P, P, FP, I, FP, FP, FP]),
            "orc_rvq_create": (P, [I, I, ctypes.POINTER(_Tensor), I]),
            "orc_rvq_free": (None, [P]),
            "orc_rvq_encode": (I, [P, FP, I, UP]),
            "orc_rvq_distances": (I, [P, I, FP, FP]),
        }
        for name, (res, args) in sig.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def fp(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def up(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))


def set_threads(n: int) -> None:
    lib().orc_set_threads(n)


class OracleModel:
    """An oracle LanguageModel (kind 0) or FlowLm (kind 1) built from named f32 tensors."""

    def __init__(self, kind: int, cfg, tensors: dict[str, np.ndarray], stt=None, tts=None):
        self.kind, self.cfg, self.stt, self.tts = kind, cfg, stt, tts
        keep = []
        arr = (_Tensor * len(tensors))()
        for i, (name, a) in enumerate(tensors.items()):
            a = np.ascontiguousarray(a, np.float32)
            nb = name.encode()
            keep += [a, nb]
            arr[i] = _Tensor(nb, a.ctypes.data, a.size)
        c = cfg.to_c()
        s = stt.to_c() if stt is not None else None
        t = tts.to_c() if tts is not None else None
        h = lib().orc_lm_create(kind, ctypes.byref(c), ctypes.byref(s) if s else None,
                                ctypes.byref(t) if t else None, arr, len(tensors))
        if not h:
            raise ValueError(lib().orc_last_error().decode())
        self.handle = h

    def __del__(self):
        if getattr(self, "handle", None):
            lib().orc_lm_free(self.handle)
            self.handle = None

    def init_state(self) -> "OracleState":
        return OracleState(lib().orc_state_create(self.handle))

    def stt_step(self, text_token: int, audio: np.ndarray, state: "OracleState"):
        a = np.ascontiguousarray(audio, np.uint32)
        out = (ctypes.c_uint32 * 1)()
        logits = np.zeros(self.stt.text_card, np.float32)
        extra = np.zeros(max(self.stt.extra_heads_num_heads, 1), np.float32)
        rc = lib().orc_stt_step(self.handle, state.handle, int(text_token), up(a),
                                ctypes.cast(out, ctypes.POINTER(ctypes.c_uint32)), fp(logits),
                                fp(extra))
        if rc:
            raise ValueError(lib().orc_last_error().decode())
        return int(out[0]), logits, extra[: self.stt.extra_heads_num_heads]

    def forward(self, xs: np.ndarray, state: "OracleState") -> np.ndarray:
        x = np.ascontiguousarray(xs, np.float32).copy()
        lib().orc_transformer_forward(self.handle, state.handle, fp(x), x.shape[0])
        return x

    def tts_step(self, latent, noise: np.ndarray, state: "OracleState", decode_steps: int = 1):
        n = np.ascontiguousarray(noise, np.float32)
        lat = None if latent is None else np.ascontiguousarray(latent, np.float32)
        out = np.zeros_like(n)
        eos = np.zeros(1, np.float32)
        rc = lib().orc_tts_step(self.handle, state.handle, fp(lat) if lat is not None else None,
                                fp(n), float(decode_steps), fp(out), fp(eos))
        if rc:
            raise ValueError(lib().orc_last_error().decode())
        return out, float(eos[0])

    def prompt_text(self, tokens, state: "OracleState"):
        t = np.ascontiguousarray(tokens, np.uint32)
        if lib().orc_tts_prompt_text(self.handle, state.handle, up(t), t.size):
            raise ValueError(lib().orc_last_error().decode())


class OracleState:
    def __init__(self, handle):
        self.handle = handle

    def __del__(self):
        if getattr(self, "handle", None):
            lib().orc_state_free(self.handle)
            self.handle = None

    def duplicate(self) -> "OracleState":
        return OracleState(lib().orc_state_duplicate(self.handle))

    @property
    def position(self) -> int:
        return lib().orc_state_position(self.handle)


def greedy_stt(model: OracleModel, audio: np.ndarray, frames: int, state=None,
               teacher: np.ndarray | None = None):
    """Recognizer::step's loop (stt/mod.rs:551-565) on the oracle: step 0 sees the initial
    tokens; the text token fed back is the previous argmax, or teacher[i-1] when given.
    Returns tokens [frames], logits [frames][text_card]."""
    st = state or model.init_state()
    stt = model.stt
    toks, logits = [], []
    prev = stt.text_card
    for i in range(frames):
        a = np.full(stt.n_q, stt.card, np.uint32) if st.position == 0 else audio[i]
        tok, lg, _ = model.stt_step(prev, a, st)
        toks.append(tok)
        logits.append(lg)
        prev = tok if teacher is None else int(teacher[i])
    return np.array(toks, np.uint32), np.stack(logits)


def _tensor_array(tensors: dict[str, np.ndarray]):
    keep = []
    arr = (_Tensor * len(tensors))()
    for i, (name, a) in enumerate(tensors.items()):
        a = np.ascontiguousarray(a, np.float32)
        nb = name.encode()
        keep += [a, nb]
        arr[i] = _Tensor(nb, a.ctypes.data, a.size)
    return arr, keep


def conv1d_stream(w, bias, prev, started, x, stride=1, dilation=1, replicate=False, elu=False,
                  skip=None):
    """StreamingConv1d::forward of one stream (nn/conv.rs:122-179): returns the output; prev
    ([cin][context]) and started (a one-element int32 array) are updated in place."""
    cout, cin, k = w.shape
    x = np.ascontiguousarray(x, np.float32)
    t = x.shape[1]
    out = np.zeros((cout, t // stride), np.float32)
    w = np.ascontiguousarray(w, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    sk = None if skip is None else np.ascontiguousarray(skip, np.float32)
    rc = lib().orc_conv1d_stream(cin, cout, k, stride, dilation, int(replicate), fp(w),
                                 fp(b) if b is not None else None, fp(prev),
                                 started.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), fp(x), t,
                                 int(elu), fp(sk) if sk is not None else None, fp(out))
    if rc:
        raise ValueError("conv input length is not a positive multiple of the stride")
    return out


def convtr1d_stream(w, bias, partial, x, stride, depthwise=False, elu=False):
    """StreamingConvTranspose1d::forward of one stream (nn/conv.rs:265-335); partial
    ([cout][k - stride]) is updated in place."""
    cin, per, k = w.shape
    cout = cin if depthwise else per
    x = np.ascontiguousarray(x, np.float32)
    t = x.shape[1]
    out = np.zeros((cout, t * stride), np.float32)
    w = np.ascontiguousarray(w, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    rc = lib().orc_convtr1d_stream(cin, cout, k, stride, int(depthwise), fp(w),
                                   fp(b) if b is not None else None, fp(partial), fp(x), t,
                                   int(elu), fp(out))
    if rc:
        raise ValueError("invalid transposed convolution")
    return out


class OracleMimi:
    """MimiEncoder / MimiDecoder (nn/mimi.rs:133-272) for one stream."""

    def __init__(self, cfg, tensors: dict[str, np.ndarray]):
        self.cfg = cfg
        arr, self._keep = _tensor_array(tensors)
        c = cfg.to_c()
        h = lib().orc_mimi_create(ctypes.byref(c), arr, len(tensors))
        if not h:
            raise ValueError("oracle Mimi: missing or mis-shaped tensors")
        self.handle = h
        self.frame_size = lib().orc_mimi_frame_size(h)

    def __del__(self):
        if getattr(self, "handle", None):
            lib().orc_mimi_free(self.handle)
            self.handle = None

    def init_state(self):
        return _MimiState(lib().orc_mimi_state_create(self.handle))

    def encode_step(self, pcm: np.ndarray, state) -> np.ndarray:
        pcm = np.ascontiguousarray(pcm, np.float32)
        frames = pcm.shape[-1] // self.frame_size
        out = np.zeros((self.cfg.inner_dim, frames), np.float32)
        if lib().orc_mimi_encode_step(self.handle, state.handle, fp(pcm), frames, fp(out)):
            raise ValueError("oracle encode failed")
        return out

    def decode_step(self, latent: np.ndarray, state) -> np.ndarray:
        latent = np.ascontiguousarray(latent, np.float32)
        frames = latent.shape[-1]
        out = np.zeros((self.cfg.decoder.channels, frames * self.frame_size), np.float32)
        if lib().orc_mimi_decode_step(self.handle, state.handle, fp(latent), frames, fp(out)):
            raise ValueError("oracle decode failed")
        return out


def _decode_latent(self, latent: np.ndarray, state, emb_std=None, emb_mean=None) -> np.ndarray:
    """Tts::decode_latent: latent [frames][latent_dim] -> pcm [channels][frames * frame_size]."""
    latent = np.ascontiguousarray(latent, np.float32)
    frames = latent.shape[0]
    out = np.zeros((self.cfg.decoder.channels, frames * self.frame_size), np.float32)
    sd = None if emb_std is None else np.ascontiguousarray(emb_std, np.float32)
    mn = None if emb_mean is None else np.ascontiguousarray(emb_mean, np.float32)
    if lib().orc_mimi_decode_latent(self.handle, state.handle, fp(latent), frames,
                                    fp(sd) if sd is not None else None,
                                    fp(mn) if mn is not None else None, fp(out)):
        raise ValueError("oracle decode_latent failed (no quantizer.output_proj.weight?)")
    return out


OracleMimi.decode_latent = _decode_latent


class _MimiState:
    def __init__(self, handle):
        self.handle = handle

    def __del__(self):
        if getattr(self, "handle", None):
            lib().orc_mimi_state_free(self.handle)
            self.handle = None


class OracleQuantizer:
    """Quantizer (stt/model.rs:84-170)."""

    def __init__(self, n_q: int, bins: int, tensors: dict[str, np.ndarray]):
        self.n_q, self.bins = n_q, bins
        arr, keep = _tensor_array(tensors)
        h = lib().orc_rvq_create(n_q, bins, arr, len(tensors))
        if not h:
            raise ValueError("oracle quantizer: missing or mis-shaped tensors")
        self.handle = h

    def __del__(self):
        if getattr(self, "handle", None):
            lib().orc_rvq_free(self.handle)
            self.handle = None

    def encode(self, latent: np.ndarray) -> np.ndarray:
        """latent [512][frames] -> codes [frames][n_q]."""
        latent = np.ascontiguousarray(latent, np.float32)
        frames = latent.shape[1]
        codes = np.zeros((frames, self.n_q), np.uint32)
        lib().orc_rvq_encode(self.handle, fp(latent), frames, up(codes))
        return codes

    def distances(self, codebook: int, residual: np.ndarray) -> np.ndarray:
        r = np.ascontiguousarray(residual, np.float32)
        d = np.zeros(self.bins, np.float32)
        lib().orc_rvq_distances(self.handle, codebook, fp(r), fp(d))
        return d
