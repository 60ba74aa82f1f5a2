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
