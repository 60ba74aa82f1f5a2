"""ctypes binding of libsvl_b200.so (include/svl_cuda.h).

There is no fallback: when the library is missing, or was built without a usable GPU, the
calls raise instead of computing anything on the CPU.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

from .config import CSttConfig, CTensorView, CTransformerConfig, CTtsConfig

LIB_PATH = Path(os.environ.get("SVL_LIB", Path(__file__).resolve().parent.parent / "libsvl_b200.so"))

STATE_REFERENCE_ORDER = 1  # svl_state_create_ex flags (include/svl_cuda.h)
STATE_TEST_WITHHELD_COPY = 2

STATUS = {0: "OK", 1: "CONFIG", 2: "INVALID_INPUT", 3: "CUDA", 4: "OOM", 5: "TIMEOUT",
          6: "UNSUPPORTED"}

# Every symbol of include/svl_cuda.h with its (restype, argtypes).
_P = ctypes.c_void_p
_I = ctypes.c_int32
_U32P = ctypes.POINTER(ctypes.c_uint32)
_F32P = ctypes.POINTER(ctypes.c_float)
SIGNATURES = {
    "svl_stt_model_create": (_I, [ctypes.POINTER(CTransformerConfig), ctypes.POINTER(CSttConfig),
                                  ctypes.POINTER(CTensorView), _I, _I, ctypes.POINTER(_P)]),
    "svl_tts_model_create": (_I, [ctypes.POINTER(CTransformerConfig), ctypes.POINTER(CTtsConfig),
                                  ctypes.POINTER(CTensorView), _I, _I, ctypes.POINTER(_P)]),
    "svl_model_destroy": (None, [_P]),
    "svl_model_weight_bytes": (ctypes.c_int64, [_P]),
    "svl_state_create": (_I, [_P, _I, _I, ctypes.POINTER(_P)]),
    "svl_state_create_ex": (_I, [_P, _I, _I, ctypes.c_uint32, ctypes.POINTER(_P)]),
    "svl_state_destroy": (None, [_P]),
    "svl_state_reset": (_I, [_P, _I]),
    "svl_state_position": (_I, [_P, _I, ctypes.POINTER(_I)]),
    "svl_state_copy": (_I, [_P, _I, _P, _I]),
    "svl_state_export": (_I, [_P, _I, _I, _F32P, _F32P, ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "svl_state_import": (_I, [_P, _I, _I, _F32P, _F32P, _I, _I]),
    "svl_voice_save": (_I, [_P, _I, ctypes.c_char_p]),
    "svl_voice_load": (_I, [_P, ctypes.POINTER(_I), _I, ctypes.c_char_p]),
    "svl_stt_step": (_I, [_P, _P, _I, _U32P, _U32P, _U32P, _F32P, _F32P]),
    "svl_stt_step_device": (_I, [_P, _P, _I, _P, _P, _P, _P, _P]),
    "svl_stt_run_frames": (_I, [_P, _P, _I, _I, _U32P, _U32P]),
    "svl_stt_run_frames_ex": (_I, [_P, _P, _I, _I, _U32P, _U32P, _F32P]),
    "svl_transformer_forward": (_I, [_P, _P, _I, _F32P, _I]),
    "svl_tts_prompt_text": (_I, [_P, _P, _I, _U32P, _I]),
    "svl_tts_prompt_text_batch": (_I, [_P, _P, _I, _U32P, _I]),
    "svl_tts_step": (_I, [_P, _P, _I, _F32P, _F32P, _I, _F32P, _F32P]),
    "svl_tts_step_device": (_I, [_P, _P, _I, _P, _P, _I, _P, _P, _P]),
    "svl_profile_kernels": (_I, [_P, _P, _I, _I, _I, _P, ctypes.POINTER(ctypes.c_int64)]),
    "svl_step_kernel_count": (_I, [_P, _P, _I, ctypes.POINTER(ctypes.c_int32)]),
    "svl_state_error": (_I, [_P]),
    "svl_stt_head_noalloc": (_I, [_P, _I, _P, _P, _P, _P]),
    "svl_mimi_create": (_I, [_P, _P, _I, _I, ctypes.POINTER(_P)]),
    "svl_mimi_destroy": (None, [_P]),
    "svl_mimi_frame_size": (_I, [_P]),
    "svl_mimi_state_create": (_I, [_P, _I, _I, ctypes.POINTER(_P)]),
    "svl_mimi_state_destroy": (None, [_P]),
    "svl_mimi_state_reset": (_I, [_P, _I]),
    "svl_mimi_encode_step_device": (_I, [_P, _P, _I, _I, _P, _P, _P]),
    "svl_mimi_decode_step_device": (_I, [_P, _P, _I, _I, _P, _P, _P]),
    "svl_mimi_decode_latent_device": (_I, [_P, _P, _I, _I, _P, _P, _P, _P, _P]),
    "svl_mimi_latent_dim": (_I, [_P]),
    "svl_rvq_create": (_I, [_I, _I, _P, _I, _I, ctypes.POINTER(_P)]),
    "svl_rvq_destroy": (None, [_P]),
    "svl_rvq_encode_device": (_I, [_P, _I, _I, _P, _P, _P]),
    "svl_last_error": (ctypes.c_char_p, []),
    "svl_version": (ctypes.c_char_p, []),
}

_lib = None


class SvlError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status
        self.kind = STATUS.get(status, str(status))


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with semantic-ai_b200/build.py "
                               "(there is no CPU fallback)")
        l = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def check(status: int) -> None:
    if status != 0:
        raise SvlError(status, lib().svl_last_error().decode())
