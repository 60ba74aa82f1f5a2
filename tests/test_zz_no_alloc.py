"""svl_stt_head_noalloc: the greedy head for callers that cannot allocate device memory.

A host that owns every device allocation of its process (a plugin host's pool, a real-time
audio thread that must never enter the allocator) cannot create a state, so it cannot use
svl_stt_step's head, whose argmax scratch lives in the state. svl_stt_head_noalloc keeps that
scratch in a fixed array inside the library instead. This checks it, through the C ABI,
against the head of svl_stt_step on the same hidden states, on two calls in a row (and one
two-stream call), with the f32 tolerance of the parity tests, for f32 weights and for the
quantised formats, whose head takes the Q8_0 / Q4_1 branch of the product kernel.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F32_TOL = 2e-3


def _embed(w, stt, text, audio):
    """LanguageModel::step's input sum on the host, in the reference's order (f32)."""
    x = w["text_emb.weight"][text].astype(np.float32).copy()
    for c in range(stt.n_q):
        x = x + w[f"emb.{c}.weight"][audio[c]]
    return x


@pytest.mark.parametrize("wdt,kvdt", [("f32", "f32"), ("q8_0", "f32"), ("q4_1", "bf16")])
def test_head_noalloc_matches_step_head(svl_lib, wdt, kvdt):
    import torch

    from svl import LanguageModel, config, synth
    from svl._lib import SvlError, check, lib

    stt = config.stt_toy()
    cfg = stt.transformer(wdt, kvdt)
    w = synth.stt_weights(stt, cfg)
    gm = LanguageModel(stt, cfg, w)
    audio = synth.audio_tokens(stt, 2)
    initial = np.full(stt.n_q, stt.card, np.uint32)

    # The state-based step: tokens and logits of positions 0 and 1.
    st = gm.init_state(1)
    tok0, lg0 = gm.step([stt.text_card], initial[None], st, logits=True)
    tok1, lg1 = gm.step(tok0, audio[1][None], st, logits=True)

    # The same hidden states (transformer output before out_norm) through the prefill path.
    st2 = gm.init_state(1)
    h0 = gm.forward(_embed(w, stt, stt.text_card, initial)[None], st2)[0]
    h1 = gm.forward(_embed(w, stt, int(tok0[0]), audio[1])[None], st2)[0]

    stream = torch.cuda.current_stream()
    d_tok = torch.zeros(2, dtype=torch.int32, device="cuda")
    d_logits = torch.zeros((2, stt.text_card), dtype=torch.float32, device="cuda")

    def head(hidden):
        d_h = torch.from_numpy(np.ascontiguousarray(hidden, np.float32)).to("cuda")
        n = d_h.shape[0]
        check(lib().svl_stt_head_noalloc(gm.handle, n, ctypes.c_void_p(d_h.data_ptr()),
                                         ctypes.c_void_p(d_tok.data_ptr()),
                                         ctypes.c_void_p(d_logits.data_ptr()),
                                         ctypes.c_void_p(stream.cuda_stream)))
        torch.cuda.synchronize()
        return d_tok[:n].cpu().numpy().astype(np.uint32), d_logits[:n].cpu().numpy()

    # Two calls in a row, then both streams in one call.
    for hidden, tok, lg in ((h0, tok0, lg0), (h1, tok1, lg1)):
        t, l = head(hidden[None])
        assert t[0] == tok[0]
        assert np.max(np.abs(l[0] - lg[0])) <= F32_TOL
    t, l = head(np.stack([h0, h1]))
    np.testing.assert_array_equal(t, [tok0[0], tok1[0]])
    assert np.max(np.abs(l - np.stack([lg0[0], lg1[0]]))) <= F32_TOL

    # Beyond the fixed scratch: a clear error, nothing launched.
    big = torch.zeros((9, cfg.d_model), dtype=torch.float32, device="cuda")
    rc = lib().svl_stt_head_noalloc(gm.handle, 9, ctypes.c_void_p(big.data_ptr()),
                                    ctypes.c_void_p(d_tok.data_ptr()), None,
                                    ctypes.c_void_p(stream.cuda_stream))
    assert rc == 2, rc  # SVL_ERR_INVALID_INPUT
    assert b"batch must be 1..8" in lib().svl_last_error()
    with pytest.raises(SvlError):
        check(rc)
