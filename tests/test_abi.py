"""The C-ABI library loads and exports every entry point include/svl_cuda.h declares (no GPU
needed), and the ctypes binding covers all of them."""
import ctypes
import re
from pathlib import Path

import pytest

from conftest import ROOT, gpu_available
from svl import _lib, config

HEADER = ROOT / "include" / "svl_cuda.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"SVL_API\s+[\w\s\*]+?\b(svl_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "svl_stt_step" in syms and "svl_last_error" in syms
    assert len(syms) >= 18


def test_library_exports_every_declared_symbol(svl_lib):
    for name in declared_symbols():
        assert hasattr(svl_lib, name), name


def test_binding_covers_header():
    assert set(declared_symbols()) <= set(_lib.SIGNATURES)


def test_version_and_error_without_device(svl_lib):
    assert b"sm_100a" in svl_lib.svl_version()
    assert svl_lib.svl_last_error() is not None


def test_struct_layouts_match_header():
    # svl_transformer_config: 14 x int32/float + 1 double with natural alignment.
    assert ctypes.sizeof(config.CTransformerConfig) == 64
    assert config.CTransformerConfig.max_period.offset == 56
    assert ctypes.sizeof(config.CSttConfig) == 24
    assert ctypes.sizeof(config.CTtsConfig) == 24
    assert ctypes.sizeof(config.CTensorView) == 24


@pytest.mark.skipif(gpu_available(), reason="checks the no-GPU failure path")
def test_no_cpu_fallback(svl_lib):
    """Without a GPU the library fails loudly with SVL_ERR_CUDA instead of computing on the CPU."""
    stt = config.stt_toy()
    cfg = stt.transformer("f32")
    c, s = cfg.to_c(), stt.to_c()
    h = ctypes.c_void_p()
    rc = svl_lib.svl_stt_model_create(ctypes.byref(c), ctypes.byref(s), None, 0, 0, ctypes.byref(h))
    assert rc == 3, rc  # SVL_ERR_CUDA
    assert not h.value
