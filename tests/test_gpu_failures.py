"""Failure paths of the C ABI, made without faulting the GPU (error.rs:2-31 of the reference is
the model for the status codes):

- a device-side bounded wait that runs out: SVL_STATE_TEST_WITHHELD_COPY makes the first weight
  product withhold one staged copy and wait for it only briefly; the step must report
  SVL_ERR_TIMEOUT, through svl_stt_step and through svl_state_error after svl_stt_step_device,
  and a fresh state of the same model must then step exactly as before;
- an out-of-range token on the device path: the embedding flags it, svl_state_error reports
  SVL_ERR_INVALID_INPUT;
- a state larger than the device: svl_state_create reports SVL_ERR_OOM and leaves nothing
  allocated.
"""
import ctypes

import numpy as np
import pytest

from svl import LanguageModel, FlowLm, config, synth
from svl._lib import STATE_TEST_WITHHELD_COPY, SvlError, check, lib

pytestmark = pytest.mark.gpu


def _toy_q8():
    stt = config.stt_toy()
    cfg = stt.transformer("q8_0", "f32")
    w = synth.stt_weights(stt, cfg)
    return stt, cfg, w


def test_bounded_wait_runs_out_and_reports_timeout(svl_lib):
    import torch

    stt, cfg, w = _toy_q8()
    gm = LanguageModel(stt, cfg, w)
    audio = synth.audio_tokens(stt, 6)
    first = np.full((1, stt.n_q), stt.card, np.uint32)

    # The undisturbed run.
    want = gm.run_frames(audio[:, None, :], gm.init_state(1))[:, 0]

    # Host-buffer step: the status comes back from the call itself.
    drill = gm.init_state(1, flags=STATE_TEST_WITHHELD_COPY)
    with pytest.raises(SvlError) as e:
        gm.step([stt.text_card], first, drill)
    assert e.value.kind == "TIMEOUT", e.value

    # Device-buffer step: enqueued without a host synchronisation, so the timeout is read back
    # through svl_state_error, which also clears it.
    d_text = torch.full((1,), stt.text_card, dtype=torch.int32, device="cuda")
    d_audio = torch.from_numpy(first.view(np.int32)).to("cuda")
    d_out = torch.zeros(1, dtype=torch.int32, device="cuda")
    check(lib().svl_stt_step_device(gm.handle, drill.handle, 1, ctypes.c_void_p(d_text.data_ptr()),
                                    ctypes.c_void_p(d_audio.data_ptr()), ctypes.c_void_p(d_out.data_ptr()),
                                    None, None))
    assert lib().svl_state_error(drill.handle) == 5  # SVL_ERR_TIMEOUT
    assert lib().svl_state_error(drill.handle) == 0  # cleared
    drill.close()

    # The model and the context are intact: a fresh state steps exactly as before.
    np.testing.assert_array_equal(gm.run_frames(audio[:, None, :], gm.init_state(1))[:, 0], want)


def test_out_of_range_token_on_the_device_path(svl_lib):
    import torch

    stt, cfg, w = _toy_q8()
    gm = LanguageModel(stt, cfg, w)
    st = gm.init_state(1)
    d_text = torch.full((1,), stt.text_card + 5, dtype=torch.int32, device="cuda")
    d_audio = torch.zeros((1, stt.n_q), dtype=torch.int32, device="cuda")
    d_out = torch.zeros(1, dtype=torch.int32, device="cuda")
    check(lib().svl_stt_step_device(gm.handle, st.handle, 1, ctypes.c_void_p(d_text.data_ptr()),
                                    ctypes.c_void_p(d_audio.data_ptr()), ctypes.c_void_p(d_out.data_ptr()),
                                    None, None))
    assert lib().svl_state_error(st.handle) == 2  # SVL_ERR_INVALID_INPUT
    assert lib().svl_state_error(st.handle) == 0
    # The next (valid) step runs and reports nothing.
    d_text.fill_(stt.text_card)
    check(lib().svl_stt_step_device(gm.handle, st.handle, 1, ctypes.c_void_p(d_text.data_ptr()),
                                    ctypes.c_void_p(d_audio.data_ptr()), ctypes.c_void_p(d_out.data_ptr()),
                                    None, None))
    assert lib().svl_state_error(st.handle) == 0


def test_oversized_state_reports_oom(svl_lib):
    import torch

    cfg, tts = config.tts_toy("lsd")
    fm = FlowLm(cfg, tts, synth.tts_weights(cfg, tts))
    free0 = torch.cuda.mem_get_info()[0]
    h = ctypes.c_void_p()
    # 4096 streams x 2^24 positions of an unwindowed ring: tens of TB.
    rc = lib().svl_state_create(fm.handle, 4096, 1 << 24, ctypes.byref(h))
    assert rc == 4, (rc, lib().svl_last_error())  # SVL_ERR_OOM
    assert not h.value
    assert b"cudaMalloc" in lib().svl_last_error()
    assert torch.cuda.mem_get_info()[0] >= free0 - (64 << 20)
    # The model still works.
    st = fm.init_state(1, max_positions=8)
    fm.step(None, np.zeros((1, tts.latent_dim), np.float32), st)
