"""Host logic of the cached-convolution streaming DAC decoder, on the CPU.

StreamingDacDecoder decides, per chunk, which window of which layer buffer
each launch reads and writes, how many samples it may emit, where the next
layer's input goes and which history each buffer keeps.  These tests run that
bookkeeping on CPU tensors against a fake library whose three entry points
(sn_snake_conv1d_strided, sn_snake_conv_transpose1d_strided, sn_stream_shift)
compute what the CUDA kernels compute, with the float64 oracle, through the
same pointers and strides.  Chunked decoding must equal the one-chunk decode
for every chunk size, and the one-chunk decode must equal the oracle's
one-shot DacDecoder.
"""
import ctypes
import math
import types

import numpy as np
import pytest
import torch

import oracle as O
from sonata_b200 import _lib
from sonata_b200.kernels import dac as D
from sonata_b200.kernels import dac_stream as DS


_ALLOWED = []  # (start, end) byte ranges of the tensors a fake call may touch


def _view(ptr, shape, strides):
    n = 1 + sum((sh - 1) * st for sh, st in zip(shape, strides))
    # a window outside every buffer would be an out-of-bounds access on the GPU
    assert any(a <= ptr and ptr + 4 * n <= b for a, b in _ALLOWED), (ptr, shape, strides)
    base = np.ctypeslib.as_array((ctypes.c_float * n).from_address(ptr))
    return np.lib.stride_tricks.as_strided(base, shape=shape, strides=[4 * s for s in strides])


class FakeLib:
    """The streaming entry points restated on the CPU (float64 math, float32
    results), reading and writing through the raw pointers they are given."""

    def __init__(self):
        self.calls = 0

    def sn_snake_conv1d_strided(self, x, x_bs, x_ld, alpha, W, bias, res, r_bs, r_ld, y, y_bs, y_ld, B, Cin, Cout, T,
                                K, stride, pad, dil, eps, act, post, flags, ws, wsn, st):
        self.calls += 1
        xv = _view(x, (B, Cin, T), (x_bs, x_ld, 1)).astype(np.float64)
        w = _view(W, (Cout, Cin, K), (Cin * K, K, 1))
        b = _view(bias, (Cout,), (1,))
        if act == _lib.SN_ACT_SNAKE:
            a = _view(alpha, (Cin,), (1,))
            out = O.snake_conv1d_ref(xv, a, w, b, stride=stride, padding=pad, dilation=dil, eps=eps.value)
        else:
            out = O.conv1d_ref(xv, w, b, stride=stride, padding=pad, dilation=dil)
        Tout = out.shape[2]
        if res:
            out = out + _view(res, (B, Cout, Tout), (r_bs, r_ld, 1))
        if post == _lib.SN_POST_TANH:
            out = np.tanh(out)
        _view(y, (B, Cout, Tout), (y_bs, y_ld, 1))[...] = out.astype(np.float32)
        return 0

    def sn_snake_conv_transpose1d_strided(self, x, x_bs, x_ld, alpha, W, bias, y, y_bs, y_ld, B, Cin, Cout, T, K, s,
                                          pad, Ty, eps, flags, ws, wsn, st):
        self.calls += 1
        assert 1 <= Ty <= (T - 1) * s - pad + K
        xv = _view(x, (B, Cin, T), (x_bs, x_ld, 1)).astype(np.float64)
        w = _view(W, (Cin, Cout, K), (Cout * K, K, 1))
        a = _view(alpha, (Cin,), (1,))
        full = O.snake_conv_transpose1d_ref(xv, a, w, None, stride=s, padding=0, eps=eps.value)
        out = full[:, :, pad:pad + Ty] + _view(bias, (Cout,), (1,)).reshape(1, -1, 1)
        _view(y, (B, Cout, Ty), (y_bs, y_ld, 1))[...] = out.astype(np.float32)
        return 0

    def sn_stream_shift(self, descs, n, st):
        assert 1 <= n <= _lib.SN_SHIFT_MAX_DESCS
        for i in range(n):
            d = descs[i]
            assert 0 <= d.len <= _lib.SN_SHIFT_MAX_LEN
            v = _view(d.buf, (d.batches, d.rows, d.src + d.len), (d.batch_stride, d.row_stride, 1))
            v[:, :, :d.len] = v[:, :, d.src:d.src + d.len].copy()
        return 0


def _decoder(cfg, seed=0):
    params = {k: v.float().contiguous() for k, v in D.init_decoder_params(cfg, seed=seed).items()}
    dec = types.SimpleNamespace(config=cfg, p=params,
                                packed={k: torch.zeros(16, dtype=torch.uint8) for k in params if k.endswith("weight")})
    dec._a = lambda name: params[name].view(-1)
    return dec


CFG = D.dac_decoder_config(hidden_size=16, decoder_hidden_size=64, upsampling_ratios=(8, 4, 2, 2))


def _new(dec, chunk, batch):
    sd = DS.StreamingDacDecoder(dec, max_chunk_frames=chunk, batch=batch, use_graphs=False, lib=FakeLib())
    _ALLOWED.clear()
    tensors = [sd.out, *dec.p.values()]
    for kind, L in sd.layers:
        tensors += [c.buf for c in (L if kind == "unit" else (L,))]
    _ALLOWED.extend((t.data_ptr(), t.data_ptr() + t.element_size() * t.numel()) for t in tensors)
    return sd


def _stream(dec, latent, chunk):
    sd = _new(dec, chunk, latent.shape[0])
    pieces = []
    for f0 in range(0, latent.shape[2], chunk):
        pieces.append(sd.push(latent[..., f0:f0 + chunk]).clone())
        assert sd.lookahead_samples >= 0
    pieces.append(sd.flush().clone())
    return torch.cat(pieces, dim=-1), sd


@pytest.fixture(scope="module")
def setup():
    dec = _decoder(CFG, seed=3)
    g = torch.Generator().manual_seed(4)
    latent = torch.randn(2, CFG["hidden_size"], 11, generator=g)
    one, sd = _stream(dec, latent, 11)
    return dec, latent, one


def test_one_chunk_equals_oracle_one_shot(setup):
    dec, latent, one = setup
    hop = math.prod(CFG["upsampling_ratios"])
    assert one.shape == (2, 1, 11 * hop)
    p = {k: v.numpy() for k, v in dec.p.items()}
    truth = O.dac_decoder_ref(latent.numpy(), p, CFG["upsampling_ratios"])
    np.testing.assert_allclose(one.numpy(), truth, rtol=0, atol=2e-5)


@pytest.mark.parametrize("chunk", [1, 2, 3, 4, 5, 7])
def test_chunked_equals_one_chunk(setup, chunk):
    dec, latent, one = setup
    got, sd = _stream(dec, latent, chunk)
    assert got.shape == one.shape
    np.testing.assert_allclose(got.numpy(), one.numpy(), rtol=1e-6, atol=1e-6)
    assert sd.lookahead_samples == 0


def test_lookahead_settles_at_the_decoder_bound(setup):
    dec, _, _ = setup
    latent = torch.randn(1, CFG["hidden_size"], 40, generator=torch.Generator().manual_seed(8))
    sd = _new(dec, 2, 1)
    held = []
    for f0 in range(0, 40, 2):
        sd.push(latent[..., f0:f0 + 2])
        held.append(sd.lookahead_samples)
    # every layer holds back its right reach once the stream is past it
    assert held[-1] == held[-2] == held[-5] == sd.lookahead_bound() > 0, held


def test_push_validation(setup):
    dec, latent, _ = setup
    sd = _new(dec, 4, 2)
    with pytest.raises(ValueError):
        sd.push(latent[..., :5])
    with pytest.raises(ValueError):
        sd.push(latent[:1, :, :2])
    sd.push(latent[..., :2])
    sd.flush()
    with pytest.raises(RuntimeError):
        sd.push(latent[..., :2])
