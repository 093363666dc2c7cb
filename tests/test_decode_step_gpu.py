"""A Zonos-hybrid decode step through the patched Linears, against the oracle.

SyntheticZonos has the Zonos backbone's module names and shapes; after
``patch_zonos_projections(model, include_attn=True)`` (the reference's
drop-in call) one token runs the repository's GEMV, Mamba2-op and codebook
head kernels with the attention, rotary and SwiGLU torch ops between them.
The logits are compared with the float64 op restatements chained on the CPU
(oracle.zonos_decode_step_ref, bf16 rounding wherever the model stores bf16);
the CUDA-graph replay of the step must equal the eager step bit for bit and
must recompute when the input changes (the reference's empty-graph tripwire,
kernels/bench_decode.py:114-121).
"""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def _model(n_layer=6, attn=(0, 4), batch=2, seed=5):
    from sonata_b200.kernels import decode_step as DS
    cfg = DS.ZonosBackboneConfig(n_layer=n_layer, attn_layer_idx=list(attn))
    m = DS.SyntheticZonos(cfg, batch=batch, context=40, max_seqlen=64, seed=seed)
    g = torch.Generator(device="cuda").manual_seed(seed + 100)
    for blk in m.backbone.layers:  # non-trivial recurrent state
        if not blk.is_attn:
            blk.mixer.conv_state.copy_(torch.randn(blk.mixer.conv_state.shape, device="cuda", generator=g))
            blk.mixer.ssm_state.copy_(0.5 * torch.randn(blk.mixer.ssm_state.shape, device="cuda", generator=g))
    return m


def _snapshot(m):
    p, st = {}, {}
    for i, blk in enumerate(m.backbone.layers):
        pre = f"L{i}."
        p[pre + "norm_w"], p[pre + "norm_b"] = _np(blk.norm_w), _np(blk.norm_b)
        p[pre + "in_proj"], p[pre + "out_proj"] = _np(blk.mixer.in_proj.weight), _np(blk.mixer.out_proj.weight)
        if blk.is_attn:
            p[pre + "norm2_w"], p[pre + "norm2_b"] = _np(blk.norm2_w), _np(blk.norm2_b)
            p[pre + "fc1"], p[pre + "fc2"] = _np(blk.mlp.fc1.weight), _np(blk.mlp.fc2.weight)
            p[pre + "k_cache"], p[pre + "v_cache"] = _np(blk.mixer.k_cache), _np(blk.mixer.v_cache)
            st[i] = (blk.mixer.k_cache.clone(), blk.mixer.v_cache.clone())
        else:
            mx = blk.mixer
            p[pre + "conv_w"], p[pre + "conv_b"] = _np(mx.conv_w), _np(mx.conv_b)
            p[pre + "conv_state"], p[pre + "ssm_state"] = _np(mx.conv_state), _np(mx.ssm_state)
            p[pre + "A"], p[pre + "D_e"], p[pre + "dt_bias_e"] = _np(mx.A), _np(mx.D_e), _np(mx.dt_bias_e)
            p[pre + "norm_mix_w"] = _np(mx.norm_w)
            st[i] = (mx.conv_state.clone(), mx.ssm_state.clone())
    p["norm_f_w"], p["norm_f_b"] = _np(m.backbone.norm_f_w), _np(m.backbone.norm_f_b)
    p["head_W"] = _np(m.head_W)
    return p, st


def _restore(m, st):
    for i, blk in enumerate(m.backbone.layers):
        a, b = st[i]
        if blk.is_attn:
            blk.mixer.k_cache.copy_(a)
            blk.mixer.v_cache.copy_(b)
        else:
            blk.mixer.conv_state.copy_(a)
            blk.mixer.ssm_state.copy_(b)


def _cfg(m):
    c = m.cfg
    return {"d_inner": c.d_inner, "d_state": c.d_state, "nheads": c.nheads, "headdim": c.headdim,
            "conv_dim": c.d_inner + 2 * c.ngroups * c.d_state, "num_heads": c.num_heads,
            "num_heads_kv": c.num_heads_kv, "head_dim": c.head_dim, "attn_layer_idx": list(c.attn_layer_idx),
            "n_layer": c.n_layer, "pos": m.pos, "eps": c.norm_epsilon}


@pytest.fixture(scope="module")
def patched():
    from sonata_b200.kernels.patch import patch_zonos_projections
    m = _model()
    p, st = _snapshot(m)
    n = patch_zonos_projections(m, include_attn=True)
    assert n == 2 * 6 + 2 * 2
    x = torch.randn(2, 2048, device="cuda", generator=torch.Generator(device="cuda").manual_seed(9)).to(torch.bfloat16)
    return m, p, st, x


@pytest.mark.parametrize("fused_glue,fused_norms", [(True, True), (True, False), (False, False)])
def test_step_matches_oracle_chain(patched, fused_glue, fused_norms):
    m, p, st, x = patched
    _restore(m, st)
    m.fused_glue, m.fused_norms = fused_glue, fused_norms
    with torch.no_grad():
        logits = m.step(x)
    m.fused_glue, m.fused_norms = True, False
    torch.cuda.synchronize()
    truth = O.zonos_decode_step_ref(p, _np(x), _cfg(m))
    got = logits.cpu().numpy()
    assert np.isfinite(got).all()
    assert O.rel_err_inf(got, truth) <= 5e-2, O.rel_err_inf(got, truth)
    assert O.cosine(got, truth) >= 0.999


def test_graph_replay_equals_eager_and_recomputes(patched):
    m, p, st, x = patched
    _restore(m, st)
    with torch.no_grad():
        eager = m.step(x).clone()
    _restore(m, st)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.no_grad(), torch.cuda.stream(s):
        m.step(x)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    _restore(m, st)
    with torch.no_grad(), torch.cuda.graph(g):
        out = m.step(x)
    _restore(m, st)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    before = out.clone()
    _restore(m, st)
    x2 = x.clone()
    x.mul_(-1)
    g.replay()
    torch.cuda.synchronize()
    x.copy_(x2)
    assert not torch.equal(out, before)
    del g


def test_full_46_layer_step_runs_in_a_graph(cuda_lib):
    from sonata_b200.kernels import decode_step as DS
    r = DS.bench_decode_step(steps=3, warmup=1)
    assert r["patched_linears"] == 34 * 2 + 12 * 4
    assert r["value"] > 0 and r["us_cublas_linear"] > 0
    assert cuda_lib.sn_device_status(1, None) == 0


def test_glue_kernels_match_torch_glue():
    """The fused glue kernels against the torch ops they replace: the split +
    conv and the rotary bit for bit, SwiGLU within one bf16 rounding."""
    from sonata_b200.kernels import decode_step as DS
    from sonata_b200.kernels import mamba_step as MS
    g = torch.Generator(device="cuda").manual_seed(3)
    b, di, ds, nh, W = 2, 4096, 128, 64, 4
    cd = di + 2 * ds
    zx = torch.randn(b, 2 * di + 2 * ds + nh, device="cuda", generator=g).to(torch.bfloat16)
    st = torch.randn(b, cd, W, device="cuda", generator=g).to(torch.bfloat16)
    w = torch.randn(cd, W, device="cuda", generator=g).to(torch.bfloat16)
    bias = torch.randn(cd, device="cuda", generator=g).to(torch.bfloat16)
    st2 = st.clone()
    z, x, Bm, Cm, dt = MS.mamba2_split_conv(zx, st, w, bias, di, 1, ds, nh)
    xbc = MS.causal_conv1d_update(zx[:, di:di + cd].contiguous(), st2, w, bias, "silu")
    assert torch.equal(st, st2)
    assert torch.equal(z, zx[:, :di]) and torch.equal(x.view(b, di), xbc[:, :di])
    assert torch.equal(Bm.view(b, ds), xbc[:, di:di + ds]) and torch.equal(Cm.view(b, ds), xbc[:, di + ds:])
    assert torch.equal(dt, zx[:, di + cd:, None].expand(b, nh, di // nh))

    hq, hk, hd, S, pos = 16, 4, 128, 64, 37
    qkv = torch.randn(b, (hq + 2 * hk) * hd, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(b, hk, S, hd, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(b, hk, S, hd, device="cuda", generator=g).to(torch.bfloat16)
    kc2, vc2 = kc.clone(), vc.clone()
    cos, sin = DS.rotary_cos_sin(pos, hd, "cuda")
    q = MS.rotary_kv_append(qkv, kc, vc, cos, sin, hq, pos)
    q_ref = DS.apply_rotary(qkv[:, :hq * hd].view(b, hq, 1, hd), cos, sin)
    kc2[:, :, pos:pos + 1] = DS.apply_rotary(qkv[:, hq * hd:(hq + hk) * hd].view(b, hk, 1, hd), cos, sin)
    vc2[:, :, pos:pos + 1] = qkv[:, (hq + hk) * hd:].view(b, hk, 1, hd)
    assert torch.equal(q, q_ref) and torch.equal(kc, kc2) and torch.equal(vc, vc2)

    h = torch.randn(b, 2 * 8192, device="cuda", generator=g).to(torch.bfloat16)
    y = MS.swiglu(h)
    ref = h[:, :8192] * torch.nn.functional.silu(h[:, 8192:])
    ulp = (ref.float().abs() * 2.0 ** -7).clamp_min(1e-30)
    assert ((y.float() - ref.float()).abs() <= ulp).all()


@pytest.mark.parametrize("b,di,ng,ds,nh,W", [(2, 4096, 1, 128, 64, 4), (1, 4096, 1, 128, 64, 4),
                                               (3, 2048, 2, 256, 32, 4), (2, 1024, 4, 128, 32, 3)])
def test_conv_ssu_equals_split_conv_then_ssu(b, di, ng, ds, nh, W):
    """sn_mamba2_conv_ssu against mamba2_split_conv + selective_state_update
    (per-head A / D / dt_bias broadcast for the latter): z, y and both
    states bit for bit, over three calls in a row (its group counters must
    come back to zero), and the counters are zero afterwards."""
    from sonata_b200.kernels import mamba_step as MS
    g = torch.Generator(device="cuda").manual_seed(11 + b + ng)
    hd = di // nh
    cd = di + 2 * ng * ds
    r = lambda *s: torch.randn(*s, device="cuda", generator=g)
    w = (0.5 * r(cd, W)).to(torch.bfloat16)
    bias = (0.1 * r(cd)).to(torch.bfloat16)
    A_h = -torch.exp(torch.log(torch.rand(nh, device="cuda", generator=g) * 15 + 1))
    D = (1 + 0.1 * r(nh)).to(torch.bfloat16)
    dtb = (torch.rand(nh, device="cuda", generator=g) * 2 - 4).to(torch.bfloat16)
    A_e = A_h[:, None, None].expand(nh, hd, ds).contiguous()
    D_e, dtb_e = D[:, None].expand(nh, hd).contiguous(), dtb[:, None].expand(nh, hd).contiguous()
    cs1 = r(b, cd, W).to(torch.bfloat16)
    ss1 = (0.5 * r(b, nh, hd, ds)).to(torch.bfloat16)
    cs2, ss2 = cs1.clone(), ss1.clone()
    sync = torch.zeros(b * ng, device="cuda", dtype=torch.int32)
    for _ in range(3):
        zx = r(b, 2 * di + 2 * ng * ds + nh).to(torch.bfloat16)
        z1, y1 = MS.mamba2_conv_ssu(zx, cs1, w, bias, ss1, A_h, D, dtb, di, ng, ds, nh, sync)
        z2, x, Bm, Cm, dt = MS.mamba2_split_conv(zx, cs2, w, bias, di, ng, ds, nh)
        y2 = MS.selective_state_update(ss2, x, dt, A_e, Bm, Cm, D=D_e, z=None, dt_bias=dtb_e, dt_softplus=True)
        torch.cuda.synchronize()
        assert torch.equal(z1, z2) and torch.equal(y1, y2)
        assert torch.equal(cs1, cs2) and torch.equal(ss1, ss2)
    assert int(sync.abs().sum()) == 0
    from sonata_b200 import _lib
    assert _lib.lib().sn_device_status(1, None) == 0


@pytest.mark.parametrize("M", [1, 2])
def test_norm_fused_gemv_matches_norm_then_gemv(M):
    """The norms fused into the GEMV's x staging against the standalone norm
    kernel followed by the GEMV: the residual sum bit for bit, the outputs
    within the decode-step tolerance (the row sums run in another order, so
    x' may differ by one bf16 rounding)."""
    from sonata_b200.kernels import gemv as G
    from sonata_b200.kernels import mamba_step as MS
    g = torch.Generator(device="cuda").manual_seed(30 + M)
    r = lambda *s, sc=1.0: (torch.randn(*s, device="cuda", generator=g) * sc).to(torch.bfloat16)
    # gated RMSNorm -> out_proj (K = 4096)
    y, z, w = r(M, 4096), r(M, 4096), r(4096, sc=0.5)
    W = r(2048, 4096, sc=0.02)
    got = G.gemv_rmsnorm_gated(y, z, w, W, 1e-5)
    ref = G.gemv(MS.rmsnorm_fn(y, w, None, z=z, eps=1e-5, group_size=4096, norm_before_gate=False), W)
    torch.cuda.synchronize()
    err = (got.float() - ref.float()).abs().max().item()
    assert err <= 2e-2 * ref.float().abs().max().item(), err
    # add + LayerNorm -> in_proj (K = 2048), with and without a residual
    for with_res in (True, False):
        h, res, w2, b2 = r(M, 2048), r(M, 2048), r(2048, sc=0.5), r(2048, sc=0.1)
        W2 = r(8512, 2048, sc=0.02)
        got, rout = G.gemv_add_layernorm(h, res if with_res else None, w2, b2, W2, 1e-5)
        xn, rref = MS.layer_norm_fn(h, w2, b2, residual=res if with_res else None, eps=1e-5, prenorm=True)
        ref = G.gemv(xn, W2)
        torch.cuda.synchronize()
        assert torch.equal(rout, rref)
        err = (got.float() - ref.float()).abs().max().item()
        assert err <= 2e-2 * ref.float().abs().max().item(), (with_res, err)
