"""The codec oracle (oracle/svl_codec_oracle.c) against the reference's own tests for the pieces
it restates, and against float64 statements of them.

Restated reference tests (crates/semantic-voice-local/src/): conv_streaming_matches_full,
im2col_conv_matches_candle, transposed_conv_forward_matches_candle,
transposed_conv_streaming_matches_full, depthwise_transposed_conv_matches_candle
(nn/conv.rs:380-566) and activations_are_accurate for ELU (nn/kernels/activation.rs:90-120).
candle's direct convolutions are replaced by float64 numpy statements of the same formulas.
"""
import numpy as np
import pytest

import oracle
from svl import codec, synth


def randn(rng, *shape):
    return rng.standard_normal(shape).astype(np.float32)


def conv_direct(x, w, stride, dilation):
    """An unpadded convolution in float64: out[o][l] = sum_c,j w[o][c][j] x[c][l s + j d]."""
    cout, cin, k = w.shape
    span = (k - 1) * dilation + 1
    n = (x.shape[1] - span) // stride + 1
    out = np.zeros((cout, n))
    for l in range(n):
        taps = x[:, l * stride + np.arange(k) * dilation].astype(np.float64)  # [cin][k]
        out[:, l] = np.einsum("ock,ck->o", w.astype(np.float64), taps)
    return out


def convtr_direct(x, w, stride, groups):
    """conv_transpose1d in float64: input step i, tap j lands on output i stride + j."""
    cin, per, k = w.shape
    cout = per * groups
    t = x.shape[1]
    out = np.zeros((cout, (t - 1) * stride + k))
    for i in range(t):
        for c in range(cin):
            g = c // (cin // groups)
            for o in range(per):
                out[g * per + o, i * stride:i * stride + k] += float(x[c, i]) * w[c, o].astype(np.float64)
    return out


def test_elu_is_accurate(oracle_lib):
    """activations_are_accurate (nn/kernels/activation.rs:90-120), ELU: within 8 ulp of expm1."""
    xs = np.concatenate([-100.0 + np.arange(400_000) * 5e-4,
                         [0.0, -0.0, 1e-30, -1e-30, -1e-7, 1e-3, -1e-3, 1e4, -1e4]]).astype(np.float32)
    ys = np.array([oracle_lib.orc_elu(float(x)) for x in xs[::7]], np.float32)
    x64 = xs[::7].astype(np.float64)
    expected = np.where(x64 > 0, x64, np.expm1(x64)).astype(np.float32)
    tol = 8 * np.finfo(np.float32).eps * np.maximum(np.abs(expected), 1e-3)
    assert np.all((ys == expected) | (np.abs(ys - expected) <= tol))


@pytest.mark.parametrize("replicate", [False, True])
def test_conv_streaming_matches_full(oracle_lib, replicate):
    rng = np.random.default_rng(0)
    w, b, x = randn(rng, 4, 3, 4), randn(rng, 4), randn(rng, 3, 12)
    prev, started = np.zeros((3, 2), np.float32), np.zeros(1, np.int32)
    full = oracle.conv1d_stream(w, b, prev, started, x, stride=2, replicate=replicate)
    prev, started = np.zeros((3, 2), np.float32), np.zeros(1, np.int32)
    chunks = [oracle.conv1d_stream(w, b, prev, started, x[:, 4 * i:4 * i + 4], stride=2,
                                   replicate=replicate) for i in range(3)]
    streamed = np.concatenate(chunks, 1)
    assert full.shape == (4, 6)
    assert np.max(np.abs(full - streamed)) < 1e-5
    # The first outputs see the padding: zeros, or the first sample repeated.
    pad = np.repeat(x[:, :1], 2, 1) if replicate else np.zeros((3, 2), np.float32)
    ref = conv_direct(np.concatenate([pad, x], 1), w, 2, 1) + b[:, None]
    assert np.max(np.abs(full - ref)) < 1e-5


@pytest.mark.parametrize("stride,dilation,kernel", [(1, 1, 7), (1, 2, 3), (4, 1, 8), (2, 1, 4), (1, 1, 1)])
def test_im2col_conv_matches_direct(oracle_lib, stride, dilation, kernel):
    rng = np.random.default_rng(1)
    w = randn(rng, 5, 3, kernel)
    ctx = max(0, (kernel - 1) * dilation + 1 - stride)
    t = (37 - ctx) // stride * stride
    x = randn(rng, 3, ctx + t)
    # A started state whose context is the signal's first samples: the unpadded convolution.
    prev, started = np.ascontiguousarray(x[:, :ctx]), np.ones(1, np.int32)
    if ctx == 0:
        prev = np.zeros((3, 1), np.float32)
    fast = oracle.conv1d_stream(w, None, prev, started, x[:, ctx:], stride=stride, dilation=dilation)
    ref = conv_direct(x, w, stride, dilation)
    assert fast.shape == ref.shape
    assert np.max(np.abs(fast - ref)) < 1e-4


@pytest.mark.parametrize("inp,out,kernel,stride,groups", [(3, 4, 6, 3, 1), (2, 5, 4, 4, 1), (3, 3, 8, 4, 3)])
def test_transposed_conv_forward_matches_direct(oracle_lib, inp, out, kernel, stride, groups):
    rng = np.random.default_rng(2)
    w, b, x = randn(rng, inp, out // groups, kernel), randn(rng, out), randn(rng, inp, 5)
    partial = np.zeros((out, kernel - stride), np.float32)
    fast = oracle.convtr1d_stream(w, b, partial, x, stride, depthwise=groups != 1)
    ref = convtr_direct(x, w, stride, groups) + b[:, None].astype(np.float64)
    assert fast.shape == (out, 5 * stride)
    assert np.max(np.abs(fast - ref[:, :5 * stride])) < 1e-4
    # The tail (no bias) is carried over.
    if kernel > stride:
        assert np.max(np.abs(partial - (ref[:, 5 * stride:] - b[:, None]))) < 1e-4


def test_transposed_conv_streaming_matches_full(oracle_lib):
    rng = np.random.default_rng(3)
    w, b, x = randn(rng, 2, 3, 6), randn(rng, 3), randn(rng, 2, 6)
    full = oracle.convtr1d_stream(w, b, np.zeros((3, 3), np.float32), x, 3)
    partial = np.zeros((3, 3), np.float32)
    streamed = np.concatenate([oracle.convtr1d_stream(w, b, partial, x[:, 2 * i:2 * i + 2], 3)
                               for i in range(3)], 1)
    assert np.max(np.abs(full - streamed)) < 1e-5


def test_conv_rejects_partial_stride(oracle_lib):
    w = np.zeros((2, 2, 4), np.float32)
    with pytest.raises(ValueError):
        oracle.conv1d_stream(w, None, np.zeros((2, 2), np.float32), np.zeros(1, np.int32),
                             np.zeros((2, 5), np.float32), stride=2)


@pytest.mark.parametrize("pad_mode", [0, 1])
def test_mimi_streaming_matches_one_pass(oracle_lib, pad_mode):
    """Encoding / decoding frame by frame equals one call over all frames (nn/conv.rs:1-5:
    "processing a whole signal at once is the same as processing it with a fresh state")."""
    cfg = codec.toy_mimi(pad_mode=pad_mode)
    m = oracle.OracleMimi(cfg, synth.mimi_weights(cfg))
    rng = np.random.default_rng(4)
    pcm = 0.3 * randn(rng, 1, 4 * m.frame_size)
    one = m.encode_step(pcm, m.init_state())
    st = m.init_state()
    steps = np.concatenate([m.encode_step(pcm[:, i * m.frame_size:(i + 1) * m.frame_size], st)
                            for i in range(4)], 1)
    assert one.shape == (cfg.inner_dim, 4)
    assert np.max(np.abs(one - steps)) < 1e-5 * max(1.0, np.abs(one).max())
    lat = randn(rng, cfg.outer_dim, 4)
    one = m.decode_step(lat, m.init_state())
    st = m.init_state()
    steps = np.concatenate([m.decode_step(lat[:, i:i + 1], st) for i in range(4)], 1)
    assert one.shape == (1, 4 * m.frame_size)
    assert np.max(np.abs(one - steps)) < 1e-5 * max(1.0, np.abs(one).max())


def test_quantizer_matches_float64_argmin(oracle_lib):
    """Quantizer::encode (stt/model.rs:100-135) against a float64 statement: every chosen entry
    is the nearest one up to float32 rounding of the distances."""
    n_q, bins = 6, 256
    w = synth.rvq_weights(n_q, bins)
    q = oracle.OracleQuantizer(n_q, bins, w)
    rng = np.random.default_rng(5)
    lat = randn(rng, 512, 7)
    codes = q.encode(lat)
    emb = []
    for k in range(n_q):
        pre = ("quantizer.rvq_first.vq.layers.0._codebook." if k == 0
               else f"quantizer.rvq_rest.vq.layers.{k - 1}._codebook.")
        u = np.maximum(w[pre + "cluster_usage"], np.float32(1e-5))
        emb.append((w[pre + "embedding_sum"] / u[:, None]).astype(np.float64))
    for f in range(lat.shape[1]):
        for part, ks in ((0, [0]), (1, list(range(1, n_q)))):
            proj = w["quantizer.rvq_first.input_proj.weight" if part == 0
                     else "quantizer.rvq_rest.input_proj.weight"][:, :, 0].astype(np.float64)
            r = proj @ lat[:, f].astype(np.float64)
            for k in ks:
                d = 0.5 * (emb[k] ** 2).sum(1) - emb[k] @ r
                c = int(codes[f, k])
                assert d[c] - d.min() <= 1e-4 * max(1.0, np.abs(d).max()), (f, k)
                r = r - emb[k][c]
    # The entry under the usage floor (1e-7 -> 1e-5) is never the nearest.
    assert not np.any(codes[:, 0] == 3)
