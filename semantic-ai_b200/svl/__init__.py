"""semantic-voice-local's streaming LM step on B200 (sm_100a), through the C ABI.

The compute path is libsvl_b200.so (CUDA kernels + C++ host); this package is a thin
Python mirror of the reference's model API for tests, benchmarks and Python callers.
"""
from .config import (SttConfig, TransformerConfig, TtsConfig, pocket_tts, stt_1b, stt_2b6,
                     stt_toy)
from .model import FlowLm, LanguageModel, State

__all__ = ["SttConfig", "TransformerConfig", "TtsConfig", "LanguageModel", "FlowLm", "State",
           "stt_1b", "stt_2b6", "stt_toy", "pocket_tts"]
