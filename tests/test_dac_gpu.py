"""GPU parity of the DAC decoder edges beyond config 5 (transformers' DacDecoder).

Tolerances (the north-star Snake-conv gate): cosine >= 0.9999 and
max |err| <= 2e-3 against the float64 oracle / the frozen transformers
outputs; the split-bf16 products are far inside it (~1e-5 relative).
"""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def S(cuda_lib):
    from sonata_b200.kernels import fused_snake_conv
    return fused_snake_conv


def _check(out, truth, atol=2e-3):
    out = out.detach().cpu().double().numpy()
    assert out.shape == truth.shape
    assert O.cosine(out, truth) >= 0.9999
    err = np.abs(out - truth).max()
    assert err <= atol * max(1.0, np.abs(truth).max()), err


@pytest.mark.parametrize("n", range(4))
def test_conv_transpose_matches_torch_golden(S, golden, n):
    g = golden("dac")
    s, K, p = g[f"convt_{n}__meta"].tolist()
    t = lambda k: torch.from_numpy(g[f"convt_{n}__{k}"]).cuda()
    y = S.fused_snake_conv_transpose1d(t("x"), t("alpha"), t("w"), t("b"), stride=s, padding=p)
    torch.cuda.synchronize()
    _check(y, g[f"convt_{n}__y"].astype(np.float64), atol=1e-4)


@pytest.mark.parametrize("Cin,Cout,T,s,K,p,B", [
    (1536, 768, 40, 8, 16, 4, 1),   # DAC block 0 (tensor cores: Cout * s = 6144 GEMM columns)
    (768, 384, 33, 8, 16, 4, 2),    # block 1, two streams
    (384, 192, 70, 4, 8, 2, 1),     # block 2
    (192, 96, 300, 2, 4, 1, 1),     # block 3
    (48, 20, 9, 3, 5, 1, 2),        # K not a multiple of stride: per-output fallback
    (20, 6, 11, 2, 4, 1, 1),        # Cin not a multiple of 16: fallback
])
def test_conv_transpose_shapes(S, Cin, Cout, T, s, K, p, B):
    g = torch.Generator().manual_seed(Cin + T)
    x = torch.randn(B, Cin, T, generator=g)
    a = torch.rand(Cin, generator=g) + 0.5
    w = torch.randn(Cin, Cout, K, generator=g) / np.sqrt(Cin * K / s)
    b = torch.randn(Cout, generator=g) * 0.1
    y = S.fused_snake_conv_transpose1d(x.cuda(), a.cuda(), w.cuda(), b.cuda(), stride=s, padding=p)
    torch.cuda.synchronize()
    truth = O.snake_conv_transpose1d_ref(x.numpy(), a.numpy(), w.numpy(), b.numpy(), stride=s, padding=p)
    _check(y, truth)


@pytest.mark.parametrize("C,T,d,B", [(96, 500, 1, 1), (192, 300, 3, 2), (768, 129, 9, 1), (40, 77, 3, 1)])
def test_residual_unit(C, T, d, B):
    from sonata_b200.kernels.dac import dac_residual_unit
    g = torch.Generator().manual_seed(C * T)
    x = torch.randn(B, C, T, generator=g)
    a1, a2 = torch.rand(C, generator=g) + 0.5, torch.rand(C, generator=g) + 0.5
    w1 = torch.randn(C, C, 7, generator=g) / np.sqrt(7 * C)
    w2 = torch.randn(C, C, 1, generator=g) / np.sqrt(C)
    b1, b2 = torch.randn(C, generator=g) * 0.1, torch.randn(C, generator=g) * 0.1
    y = dac_residual_unit(x.cuda(), a1.cuda(), w1.cuda(), b1.cuda(), a2.cuda(), w2.cuda(), b2.cuda(), d)
    torch.cuda.synchronize()
    p = {"u.snake1.alpha": a1.numpy(), "u.conv1.weight": w1.numpy(), "u.conv1.bias": b1.numpy(),
         "u.snake2.alpha": a2.numpy(), "u.conv2.weight": w2.numpy(), "u.conv2.bias": b2.numpy()}
    _check(y, O.dac_residual_unit_ref(x.numpy(), p, "u", d))


@pytest.mark.parametrize("Cin,Cout,T,act,post", [(1024, 1536, 20, "none", None), (96, 1, 333, "snake", "tanh"),
                                                 (64, 32, 200, "none", "tanh"), (30, 16, 50, "none", None),
                                                 (32, 20, 300, "snake", None)])
def test_activation_and_post_variants(S, Cin, Cout, T, act, post):
    g = torch.Generator().manual_seed(Cin + Cout)
    x = torch.randn(1, Cin, T, generator=g)
    a = torch.rand(Cin, generator=g) + 0.5
    w = torch.randn(Cout, Cin, 7, generator=g) / np.sqrt(7 * Cin)
    b = torch.randn(Cout, generator=g) * 0.1
    y = S.fused_snake_conv1d(x.cuda(), a.cuda() if act == "snake" else None, w.cuda(), b.cuda(), padding=3,
                             activation=act, post=post)
    torch.cuda.synchronize()
    if act == "snake":
        truth = O.snake_conv1d_ref(x.numpy(), a.numpy(), w.numpy(), b.numpy(), padding=3)
    else:
        truth = O.conv1d_ref(x.numpy(), w.numpy(), b.numpy(), padding=3)
    if post == "tanh":
        truth = np.tanh(truth)
    _check(y, truth)


@pytest.mark.parametrize("Cin,Cout,T,K", [(32, 20, 300, 1), (64, 40, 129, 7), (96, 96, 1000, 1)])
def test_residual_epilogue(S, Cin, Cout, T, K):
    # GEMM widths padded past Cout (20, 40) and the DAC 1x1 case
    g = torch.Generator().manual_seed(Cin * Cout + T)
    x = torch.randn(2, Cin, T, generator=g)
    a = torch.rand(Cin, generator=g) + 0.5
    w = torch.randn(Cout, Cin, K, generator=g) / np.sqrt(K * Cin)
    b = torch.randn(Cout, generator=g) * 0.1
    r = torch.randn(2, Cout, T, generator=g)
    y = S.fused_snake_conv1d(x.cuda(), a.cuda(), w.cuda(), b.cuda(), padding=(K - 1) // 2, residual=r.cuda())
    torch.cuda.synchronize()
    truth = O.snake_conv1d_ref(x.numpy(), a.numpy(), w.numpy(), b.numpy(), padding=(K - 1) // 2) + r.numpy()
    _check(y, truth)


def test_residual_rejects_alias_and_shape(S):
    x = torch.randn(1, 32, 40, device="cuda")
    a = torch.rand(32, device="cuda") + 0.5
    w = torch.randn(32, 32, 1, device="cuda")
    out = torch.empty(1, 32, 40, device="cuda")
    with pytest.raises(ValueError):
        S.fused_snake_conv1d(x, a, w, None, out=out, residual=out)
    with pytest.raises(ValueError):
        S.fused_snake_conv1d(x, a, w, None, residual=torch.zeros(1, 32, 39, device="cuda"))
    with pytest.raises(ValueError):
        S.fused_snake_conv1d(x, a, w, None, activation="relu")


def test_decoder_matches_transformers_golden(cuda_lib, golden):
    from sonata_b200.kernels.dac import DacDecoder, init_decoder_params
    g = golden("dac")
    cfg = {"hidden_size": 32, "decoder_hidden_size": 256, "upsampling_ratios": (8, 8, 4, 2)}
    dec = DacDecoder(init_decoder_params(cfg, seed=int(g["decoder__param_seed"])), cfg)
    audio = dec(torch.from_numpy(g["decoder__latent"]).cuda())
    torch.cuda.synchronize()
    _check(audio, g["decoder__audio"].astype(np.float64))


def test_decoder_full_size_short_latent(cuda_lib):
    """The 44.1 kHz model's shapes (channels 1536 .. 96, every edge on its
    production kernel) on 2 latent frames against the float64 oracle."""
    from sonata_b200.kernels.dac import DacDecoder, dac_decoder_config, init_decoder_params
    cfg = dac_decoder_config()
    params = init_decoder_params(cfg, seed=3)
    dec = DacDecoder(params, cfg)
    latent = torch.randn(1, 1024, 2, generator=torch.Generator().manual_seed(4))
    audio = dec(latent.cuda())
    torch.cuda.synchronize()
    assert audio.shape == (1, 1, 1024)
    truth = O.dac_decoder_ref(latent.numpy(), {k: v.numpy() for k, v in params.items()}, cfg["upsampling_ratios"])
    _check(audio, truth)


def test_prepacked_weights_give_identical_results(S):
    g = torch.Generator().manual_seed(21)
    x = torch.randn(1, 64, 300, generator=g).cuda()
    a = (torch.rand(64, generator=g) + 0.5).cuda()
    for cout, k, pad in [(64, 7, 9), (20, 1, 0)]:  # plain and padded GEMM width
        w = (torch.randn(cout, 64, k, generator=g) / np.sqrt(64 * k)).cuda()
        b = torch.randn(cout, generator=g).cuda()
        packed = S.pack_conv1d_weight(w)
        ref = S.fused_snake_conv1d(x, a, w, b, padding=pad, dilation=3 if k == 7 else 1)
        got = S.fused_snake_conv1d(x, a, w, b, padding=pad, dilation=3 if k == 7 else 1, packed=packed)
        torch.cuda.synchronize()
        assert torch.equal(ref, got)
    wt = (torch.randn(64, 24, 8, generator=g) / np.sqrt(128)).cuda()
    bt = torch.randn(24, generator=g).cuda()
    pt = S.pack_conv_transpose1d_weight(wt, 4)
    ref = S.fused_snake_conv_transpose1d(x, a, wt, bt, stride=4, padding=2)
    got = S.fused_snake_conv_transpose1d(x, a, wt, bt, stride=4, padding=2, packed=pt)
    torch.cuda.synchronize()
    assert torch.equal(ref, got)
    assert S.pack_conv_transpose1d_weight(torch.randn(16, 16, 5, device="cuda"), 2) is None
    with pytest.raises(ValueError):
        S.fused_snake_conv1d(x, a, w, b, packed=packed[:10])
