"""The CPU oracle (oracle/svl_oracle.c) pinned before it is trusted.

The reference ships no golden vectors for this path (its parity fixtures are generated
externally and absent), and the Rust crate cannot be built here. These tests hold the oracle
to the reference's own unit tests, restated with their inputs and bounds:

* activations_are_accurate (nn/kernels/activation.rs:88-120): SiLU and GELU-tanh within
  8 eps * max(|f64 value|, 1e-3) of the f64 definitions over [-100, 100] and special values;
* matvec_matches_candle (nn/kernels/matvec.rs:108-128): max |diff| < 1e-5 * k against a
  float64 matmul, with and without bias, for the reference's shapes;
* attention_matches_candle (nn/kernels/attention.rs:177-227): max |diff| < 1e-5 against a
  masked softmax, for the reference's (queries, keys, position, first key, context) cases;
* streaming_matches_full_sequence (nn/transformer.rs:598-628): chunks (1,3,1,7,1,1,9) of a
  23-token sequence equal one full pass within 1e-4, with and without a window;

plus an independent float64 numpy restatement of the whole STT step (tests/np_reference.py),
the ggml block formats' round-trip bounds, AVX vs scalar dot products, and committed golden
fixtures (tests/golden/, made by tests/golden/make_golden.py) that pin the oracle's outputs.
"""
from pathlib import Path

import numpy as np
import pytest

import np_reference as NR
import oracle as O
from svl import config, synth

GOLDEN = Path(__file__).parent / "golden"


def lib():
    return O.lib()


def test_activations_are_accurate(oracle_lib):
    xs = (-100.0 + np.arange(400_000, dtype=np.float64) * 5e-4).astype(np.float32)
    xs = np.concatenate([xs, np.array([0.0, -0.0, 1e-30, -1e-30, -1e-7, 1e-3, -1e-3, 1e4, -1e4,
                                       np.inf, -np.inf], np.float32)])
    sample = xs[::97]  # the oracle's scalar entry points: a dense sample keeps the test fast
    sample = np.concatenate([sample, xs[-11:]])
    x64 = sample.astype(np.float64)
    with np.errstate(over="ignore", invalid="ignore"):
        silu = x64 / (1.0 + np.exp(-x64))
        y = np.sqrt(2.0 / np.pi) * (x64 + 0.044715 * x64 ** 3)
        gelu = x64 / (1.0 + np.exp(-2.0 * y))
    for name, ref in (("orc_silu", silu), ("orc_gelu_tanh", gelu)):
        f = getattr(oracle_lib, name)
        got = np.array([f(float(x)) for x in sample], np.float32)
        exp = ref.astype(np.float32)
        tol = 8 * np.finfo(np.float32).eps * np.maximum(np.abs(exp), 1e-3)
        with np.errstate(invalid="ignore"):
            ok = (got == exp) | (np.abs(got - exp) <= tol) | (np.isnan(got) & np.isnan(exp))
        assert ok.all(), f"{name}: worst at x={sample[~ok][0]}: {got[~ok][0]} vs {exp[~ok][0]}"


def test_exp_is_accurate(oracle_lib):
    xs = np.linspace(-87.0, 88.0, 20001).astype(np.float32)
    got = np.array([oracle_lib.orc_exp(float(x)) for x in xs], np.float64)
    ref = np.exp(xs.astype(np.float64))
    rel = np.abs(got - ref) / ref
    assert rel.max() < 4 * np.finfo(np.float32).eps


@pytest.mark.parametrize("n,k", [(1, 1), (7, 5), (300, 64), (1024, 1000), (3, 4096)])
def test_matvec_matches_matmul(oracle_lib, n, k):
    rng = np.random.default_rng(n * 7 + k)
    w = rng.standard_normal((n, k)).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    x = rng.standard_normal(k).astype(np.float32)
    exp = w.astype(np.float64) @ x.astype(np.float64)
    for bias in (None, b):
        out = np.zeros(n, np.float32)
        oracle_lib.orc_matvec(O.fp(x), O.fp(w), O.fp(bias) if bias is not None else None, n, k, O.fp(out))
        want = exp + (bias if bias is not None else 0)
        assert np.max(np.abs(out - want)) < 1e-5 * k


@pytest.mark.parametrize("t,n,position,first_key,context", [
    (1, 1, 0, 0, None), (1, 9, 8, 0, None), (5, 12, 7, 0, None), (5, 12, 10, 3, 4), (3, 6, 20, 17, 6)])
def test_attention_matches_masked_softmax(oracle_lib, t, n, position, first_key, context):
    heads, kv_heads, d = 4, 2, 8
    rng = np.random.default_rng(t * 100 + n)
    q = rng.standard_normal((heads, t, d)).astype(np.float32)
    # Views into larger buffers, as the caches hand them out: rows 2..2+n of n+5.
    kb = rng.standard_normal((kv_heads, n + 5, d)).astype(np.float32)
    vb = rng.standard_normal((kv_heads, n + 5, d)).astype(np.float32)
    k, v = kb[:, 2:2 + n], vb[:, 2:2 + n]
    out = np.zeros((t, heads, d), np.float32)
    oracle_lib.orc_attention(O.fp(np.ascontiguousarray(q)), O.fp(kb.reshape(-1)[2 * d:]),
                             O.fp(vb.reshape(-1)[2 * d:]), heads, kv_heads, t, n, d,
                             (n + 5) * d, d, position, first_key, context or 0, O.fp(out))
    rep = heads // kv_heads
    kk, vv = np.repeat(k, rep, 0).astype(np.float64), np.repeat(v, rep, 0).astype(np.float64)
    exp = np.zeros((t, heads, d))
    for s in range(t):
        qp = position + s
        keys = np.arange(first_key, first_key + n)
        vis = (keys <= qp) & ((context is None) | (qp - keys < (context or 1 << 30)))
        for h in range(heads):
            sc = kk[h] @ q[h, s].astype(np.float64) / np.sqrt(d)
            sc = np.where(vis, sc, -np.inf)
            p = np.exp(sc - sc.max())
            p /= p.sum()
            exp[s, h] = p @ vv[h]
    assert np.max(np.abs(out - exp)) < 1e-5


@pytest.mark.parametrize("context", [None, 5])
def test_streaming_matches_full_sequence(oracle_lib, context):
    """nn/transformer.rs:579-627: d 16, 2 layers, 4 heads / 2 kv heads of 4, plain GELU-tanh
    FFN 32, LayerNorm 1e-5, layer scale."""
    cfg = config.TransformerConfig(d_model=16, num_layers=2, num_heads=4, num_kv_heads=2, head_dim=4,
                                   ffn_kind=config.FFN_PLAIN_GELU_TANH, ffn_hidden=32,
                                   norm_kind=config.NORM_LAYER, norm_eps=1e-5, layer_scale=True,
                                   context=context, max_period=10_000.0)
    w = synth.materialize(synth.transformer_specs(cfg), seed=0, std=0.3)
    stt = config.SttConfig(card=8, n_q=1, dim=16, text_card=8, num_heads=4, num_layers=2,
                           hidden_scale=1.0, context=context or 0, max_period=10_000.0)
    w.update({"text_emb.weight": np.zeros((9, 16), np.float32), "emb.0.weight": np.zeros((9, 16), np.float32),
              "out_norm.alpha": np.ones((1, 1, 16), np.float32),
              "text_linear.weight": np.zeros((8, 16), np.float32)})
    om = O.OracleModel(0, cfg, w, stt=stt)
    xs = np.random.default_rng(5).standard_normal((23, 16)).astype(np.float32)
    full = om.forward(xs, om.init_state())
    st, parts, start = om.init_state(), [], 0
    for n in (1, 3, 1, 7, 1, 1, 9):
        parts.append(om.forward(xs[start:start + n], st))
        start += n
    assert np.max(np.abs(np.concatenate(parts) - full)) < 1e-4
    # And against the float64 restatement, token by token.
    bb = NR.Backbone(cfg, w)
    ref = np.stack([bb.forward_token(x) for x in xs])
    assert np.max(np.abs(full - ref)) < 1e-4


@pytest.mark.parametrize("shape", ["toy", "mid"])
def test_stt_step_matches_float64_restatement(oracle_lib, shape):
    stt = config.stt_toy() if shape == "toy" else config.stt_toy(dim=256, num_heads=2, num_layers=2, context=6)
    cfg = stt.transformer("f32")
    w = synth.stt_weights(stt, cfg)
    frames = 16
    audio = synth.audio_tokens(stt, frames)
    om = O.OracleModel(0, cfg, w, stt=stt)
    toks, lg = O.greedy_stt(om, audio, frames)
    texts = [stt.text_card] + list(toks[:-1])
    au = [np.full(stt.n_q, stt.card)] + list(audio[1:frames])
    ref = NR.stt_logits(stt, cfg, w, texts, au)
    rel = np.max(np.abs(lg - ref)) / np.max(np.abs(ref))
    assert rel < 1e-5, rel
    np.testing.assert_array_equal(toks, np.argmax(ref, 1))


def test_q8_0_roundtrip(oracle_lib):
    x = np.random.default_rng(1).standard_normal(32 * 64).astype(np.float32) * 3
    blocks = np.zeros(34 * 64, np.uint8)
    oracle_lib.orc_quantize_q8_0(O.fp(x), x.size, blocks.ctypes.data_as(O.ctypes.c_void_p))
    b = blocks.reshape(64, 34)
    d = b[:, :2].copy().view(np.float16).astype(np.float32).reshape(-1)
    q = b[:, 2:].view(np.int8).astype(np.float32)
    deq = (q * d[:, None]).reshape(-1)
    xb = x.reshape(64, 32)
    assert np.allclose(d, np.abs(xb).max(1) / 127, rtol=1e-3)  # f16 of amax / 127
    assert np.all(np.abs(deq - x) <= d.repeat(32) / 2 + 1e-6 + np.abs(x) * 1e-3)


def test_q4_1_roundtrip(oracle_lib):
    x = np.random.default_rng(2).standard_normal(32 * 64).astype(np.float32)
    blocks = np.zeros(20 * 64, np.uint8)
    oracle_lib.orc_quantize_q4_1(O.fp(x), x.size, blocks.ctypes.data_as(O.ctypes.c_void_p))
    b = blocks.reshape(64, 20)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(-1)
    m = b[:, 2:4].copy().view(np.float16).astype(np.float32).reshape(-1)
    lo, hi = b[:, 4:] & 15, b[:, 4:] >> 4
    q = np.concatenate([lo, hi], 1).astype(np.float32)  # element j and j + 16 share byte j
    deq = (q * d[:, None] + m[:, None]).reshape(-1)
    assert np.all(np.abs(deq - x) <= d.repeat(32) / 2 + 2e-3 * (1 + np.abs(x)))


@pytest.mark.parametrize("k", [16, 32, 100, 2048, 5632])
def test_dot_simd_equals_scalar(oracle_lib, k):
    rng = np.random.default_rng(k)
    a, b = rng.standard_normal(k).astype(np.float32), rng.standard_normal(k).astype(np.float32)
    assert oracle_lib.orc_dot(O.fp(a), O.fp(b), k) == oracle_lib.orc_dot_scalar(O.fp(a), O.fp(b), k)
    if k % 32 == 0:
        qa, qb = np.zeros(34 * (k // 32), np.uint8), np.zeros(34 * (k // 32), np.uint8)
        oracle_lib.orc_quantize_q8_0(O.fp(a), k, qa.ctypes.data_as(O.ctypes.c_void_p))
        oracle_lib.orc_quantize_q8_0(O.fp(b), k, qb.ctypes.data_as(O.ctypes.c_void_p))
        pa, pb = qa.ctypes.data_as(O.ctypes.c_void_p), qb.ctypes.data_as(O.ctypes.c_void_p)
        nb = k // 32
        assert oracle_lib.orc_vec_dot_q8_0(pa, pb, nb) == oracle_lib.orc_vec_dot_q8_0_scalar(pa, pb, nb)


def test_golden_fixtures(oracle_lib):
    """The oracle reproduces the committed fixtures bit for bit (tests/golden/make_golden.py)."""
    import sys
    sys.path.insert(0, str(GOLDEN))
    import make_golden as MG
    assert sorted(p.stem for p in GOLDEN.glob("*.npz")) == sorted(MG.CASES)
    for path in sorted(GOLDEN.glob("*.npz")):
        want = np.load(path)
        got = MG.CASES[path.stem]()
        for key in want.files:
            np.testing.assert_array_equal(got[key], want[key], err_msg=f"{path.name}:{key}")
