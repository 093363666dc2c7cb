"""GPU parity of the Mamba2 decode-step ops against the reference's frozen goldens.

The kernels compute in fp32 and round once to bf16, as causal_conv1d /
mamba_ssm do, so they land on the golden bf16 outputs up to one rounding
step; the gates are the reference harness's own tolerances
(scripts/validation_harness.py:177-210) plus a 1-ulp-of-bf16 agreement
check; state updates that are pure data movement must be bit-exact.
"""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def M(cuda_lib):
    from sonata_b200.kernels import mamba_step
    return mamba_step


def _t(g, key):
    return torch.from_numpy(g[key].view(np.int16)).view(torch.bfloat16).cuda()


def _f(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def _gate(out, ref_bits, max_abs, mean_abs):
    ref = O.bf16_bits_to_f32(ref_bits).astype(np.float64)
    got = _f(out).reshape(ref.shape)
    d = np.abs(got - ref)
    assert d.max() <= max_abs and d.mean() <= mean_abs, (d.max(), d.mean())
    # within one bf16 rounding step of the golden (2^-8 relative, 1e-6 absolute floor)
    assert (d <= np.maximum(np.abs(ref) * 2.0 ** -7, 1e-6)).mean() >= 0.999


def test_causal_conv1d_update_golden(M, golden):
    g = golden("mamba_step")
    n = "causal_conv1d_update"
    st = _t(g, f"{n}__in__conv_state").clone()
    y = M.causal_conv1d_update(_t(g, f"{n}__in__x"), st, _t(g, f"{n}__in__weight"), _t(g, f"{n}__in__bias"), "silu")
    torch.cuda.synchronize()
    _gate(y, g[f"{n}__out0"], 9e-2, 4e-3)
    np.testing.assert_array_equal(st.cpu().view(torch.int16).numpy().view(np.uint16), g[f"{n}__out1"])


def test_rmsnorm_gated_golden(M, golden):
    g = golden("mamba_step")
    n = "rmsnorm_gated"
    y = M.rmsnorm_fn(_t(g, f"{n}__in__x"), _t(g, f"{n}__in__weight"), None, z=_t(g, f"{n}__in__z"),
                     eps=float(g[f"{n}__in__eps"]), group_size=int(g[f"{n}__in__group_size"]),
                     norm_before_gate=bool(g[f"{n}__in__norm_before_gate"]))
    torch.cuda.synchronize()
    _gate(y, g[f"{n}__out0"], 9e-2, 2e-3)


def test_layer_norm_fn_golden(M, golden):
    g = golden("mamba_step")
    n = "layer_norm_fn"
    out, res = M.layer_norm_fn(_t(g, f"{n}__in__x"), _t(g, f"{n}__in__weight"), _t(g, f"{n}__in__bias"),
                               residual=_t(g, f"{n}__in__residual"), eps=float(g[f"{n}__in__eps"]), prenorm=True)
    torch.cuda.synchronize()
    _gate(out, g[f"{n}__out0"], 5e-2, 5e-3)
    np.testing.assert_array_equal(res.cpu().view(torch.int16).numpy().view(np.uint16), g[f"{n}__out1"])
    n = "layer_norm_fn_exit"
    out = M.layer_norm_fn(_t(g, f"{n}__in__x"), _t(g, f"{n}__in__weight"), _t(g, f"{n}__in__bias"),
                          residual=_t(g, f"{n}__in__residual"), eps=float(g[f"{n}__in__eps"]))
    torch.cuda.synchronize()
    _gate(out, g[f"{n}__out0"], 5e-2, 5e-3)


def _ssu_inputs(seed, batch=2, nh=64, hd=64, ds=128, ng=1):
    """The harness's selective_state_update fixture (validation_harness.py:69-88):
    negative A = -exp(randn) per head, bf16 randn tensors."""
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g)
    a_head = -torch.exp(r(nh))
    return {"state": r(batch, nh, hd, ds).to(torch.bfloat16), "x": r(batch, nh, hd).to(torch.bfloat16),
            "dt": r(batch, nh, hd).to(torch.bfloat16), "A": a_head[:, None, None].expand(nh, hd, ds).contiguous(),
            "B": r(batch, ng, ds).to(torch.bfloat16), "C": r(batch, ng, ds).to(torch.bfloat16),
            "D": r(nh)[:, None].expand(nh, hd).contiguous().to(torch.bfloat16),
            "dt_bias": r(nh)[:, None].expand(nh, hd).contiguous().to(torch.bfloat16),
            "z": r(batch, nh, hd).to(torch.bfloat16)}


@pytest.mark.parametrize("use_z,ng,ds,nh,hd", [(False, 1, 128, 64, 64), (True, 1, 128, 64, 64), (True, 4, 128, 64, 64),
                                               (True, 2, 256, 8, 64), (True, 3, 128, 3, 5), (False, 1, 256, 1, 7),
                                               (True, 1, 64, 8, 64), (False, 2, 100, 6, 64), (True, 1, 16, 4, 64)])
def test_selective_state_update_oracle(M, use_z, ng, ds, nh, hd):
    """d_state 128 / 256 take the vector kernel (16 lanes a row, odd row
    counts included), 16 / 64 / 100 the strided one."""
    inp = _ssu_inputs(7 + ng + ds + hd, batch=1 if hd < 8 else 2, nh=nh, hd=hd, ds=ds, ng=ng)  # 15, 7 rows: odd
    st = inp["state"].cuda()
    y = M.selective_state_update(st, inp["x"].cuda(), inp["dt"].cuda(), inp["A"].cuda(), inp["B"].cuda(),
                                 inp["C"].cuda(), D=inp["D"].cuda(), z=inp["z"].cuda() if use_z else None,
                                 dt_bias=inp["dt_bias"].cuda(), dt_softplus=True)
    torch.cuda.synchronize()
    f = lambda t: t.float().numpy().astype(np.float64)
    y_ref, st_ref = O.selective_state_update_ref(f(inp["state"]), f(inp["x"]), f(inp["dt"]), f(inp["A"]), f(inp["B"]),
                                                 f(inp["C"]), D=f(inp["D"]), z=f(inp["z"]) if use_z else None,
                                                 dt_bias=f(inp["dt_bias"]), dt_softplus=True)
    # bf16 rounding of y and of the stored state (half an ulp is 2^-9 of the
    # value; 2^-8 leaves room for fp32 summation order), and the harness's
    # mean tolerances (validation_harness.py:186-190; its max-abs bounds were
    # set for its own seed's output magnitudes, ~10, and scale with them)
    dy = np.abs(_f(y) - y_ref)
    assert (dy <= np.abs(y_ref) * 2.0 ** -8 + 1e-3).all(), dy.max()
    assert dy.mean() <= 3e-2
    ds = np.abs(_f(st) - st_ref)
    assert (ds <= np.abs(st_ref) * 2.0 ** -8 + 1e-6).all(), ds.max()
    assert ds.mean() <= 4e-3


def test_selective_state_update_unaligned_state(M):
    """A state view 2 bytes off an 8-byte boundary takes the strided kernel
    and gives the same result as an aligned copy on the vector kernel."""
    inp = _ssu_inputs(31, nh=8, ds=128)
    buf = torch.empty(inp["state"].numel() + 1, dtype=torch.bfloat16, device="cuda")
    st_u = buf[1:].view(inp["state"].shape)
    st_u.copy_(inp["state"].cuda())
    st_a = inp["state"].cuda()
    args = [inp[k].cuda() for k in ("x", "dt", "A", "B", "C")]
    kw = dict(D=inp["D"].cuda(), z=inp["z"].cuda(), dt_bias=inp["dt_bias"].cuda(), dt_softplus=True)
    y_u = M.selective_state_update(st_u, *args, **kw)
    y_a = M.selective_state_update(st_a, *args, **kw)
    torch.cuda.synchronize()
    assert torch.equal(st_u, st_a)
    # the two kernels sum d_state in different orders: y agrees to fp32 order
    assert (_f(y_u) - _f(y_a)).__abs__().max() <= 2.0 ** -7 * np.abs(_f(y_a)).max()


@pytest.mark.parametrize("N,G,nbg,bias", [(4096, 4096, False, False), (4096, 1024, True, True), (1000, 500, False, True),
                                          (8192, 8192, True, True), (24, 8, False, False)])
def test_rmsnorm_gated_variants(M, N, G, nbg, bias):
    g = torch.Generator().manual_seed(N + G)
    x = torch.randn(3, N, generator=g).to(torch.bfloat16)
    w = torch.randn(N, generator=g).to(torch.bfloat16)
    b = torch.randn(N, generator=g).to(torch.bfloat16) if bias else None
    z = torch.randn(3, N, generator=g).to(torch.bfloat16)
    y = M.rmsnorm_fn(x.cuda(), w.cuda(), b.cuda() if bias else None, z=z.cuda(), eps=1e-5, group_size=G,
                     norm_before_gate=nbg)
    torch.cuda.synchronize()
    f = lambda t: t.float().numpy().astype(np.float64)
    ref = O.rmsnorm_gated_ref(f(x), f(w), f(b) if bias else None, f(z), 1e-5, G, nbg)
    d = np.abs(_f(y) - ref)
    assert (d <= np.abs(ref) * 2.0 ** -7 + 1e-6).mean() >= 0.999 and d.max() <= 9e-2


@pytest.mark.parametrize("N,rms,rf32,shift", [(2048, False, False, 0.0), (2048, True, True, 0.0),
                                              (777, False, True, 0.0), (8192, False, False, 0.0),
                                              (3, False, False, 0.0), (4096, False, False, 60.0),
                                              (1000, True, False, 0.0)])
def test_layer_norm_variants(M, N, rms, rf32, shift):
    """Row lengths over every cluster size (1, 2, 4, 8 CTAs), rows shorter
    than a CTA, and a mean far from zero (the merged mean / M2 reduction)."""
    g = torch.Generator().manual_seed(N)
    x = (torch.randn(4, N, generator=g) + shift).to(torch.bfloat16)
    r = torch.randn(4, N, generator=g).to(torch.bfloat16)
    w = torch.randn(N, generator=g).to(torch.bfloat16)
    b = torch.randn(N, generator=g).to(torch.bfloat16)
    out, res = M.layer_norm_fn(x.cuda(), w.cuda(), b.cuda(), residual=r.cuda(), eps=1e-5, prenorm=True,
                               residual_in_fp32=rf32, is_rms_norm=rms)
    torch.cuda.synchronize()
    f = lambda t: t.float().numpy().astype(np.float64)
    ref, h = O.layer_norm_fn_ref(f(x), f(w), f(b), f(r), 1e-5, is_rms_norm=rms)
    assert res.dtype == (torch.float32 if rf32 else torch.bfloat16)
    # fp32 residual_out is exact; bf16 is rounded once (half an ulp: 2^-8 of |h|)
    assert (np.abs(_f(res) - h) <= (0 if rf32 else np.abs(h) * 2.0 ** -8)).all()
    d = np.abs(_f(out) - ref)
    assert (d <= np.abs(ref) * 2.0 ** -7 + 1e-6).mean() >= 0.999 and d.max() <= 5e-2


def test_causal_conv1d_update_widths(M):
    for W, act in [(2, None), (4, "silu"), (8, "swish")]:
        g = torch.Generator().manual_seed(W)
        x = torch.randn(3, 300, generator=g).to(torch.bfloat16)
        st = torch.randn(3, 300, W, generator=g).to(torch.bfloat16)
        w = torch.randn(300, W, generator=g).to(torch.bfloat16)
        b = torch.randn(300, generator=g).to(torch.bfloat16)
        sd = st.cuda()
        y = M.causal_conv1d_update(x.cuda(), sd, w.cuda(), b.cuda(), act)
        torch.cuda.synchronize()
        f = lambda t: t.float().numpy().astype(np.float64)
        yr, sr = O.causal_conv1d_update_ref(f(x), f(st), f(w), f(b), act)
        np.testing.assert_array_equal(_f(sd), sr)
        d = np.abs(_f(y) - yr)
        assert (d <= np.abs(yr) * 2.0 ** -7 + 1e-6).mean() >= 0.999
    with pytest.raises(NotImplementedError):
        M.causal_conv1d_update(x.cuda(), sd, w.cuda(), b.cuda(), "relu")
