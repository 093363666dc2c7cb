"""Mamba2 decode-step ops on B200: the element ops between the decode GEMVs.

Same call signatures and semantics as the library functions the reference's
Mamba2.step() uses and its frozen goldens were made with
(scripts/validation_harness.py:39, 117-171): causal_conv1d's
``causal_conv1d_update`` and mamba_ssm's ``selective_state_update``,
``rmsnorm_fn`` (ops/triton/layernorm_gated) and ``layer_norm_fn``
(ops/triton/layer_norm), restricted to the decode path (bf16 tensors, no
dropout / second input / rowscale).  Each runs one sm_100a kernel through the
C ABI (``sn_causal_conv1d_update``, ``sn_selective_state_update``,
``sn_rmsnorm_gated``, ``sn_layer_norm_fused``); in-place state updates are
in place, as in those libraries.
"""
from __future__ import annotations

import torch

from .. import _lib
from ._common import call, require_cuda, stream_handle

_BF16 = torch.bfloat16


def _ptr(t):
    return t.data_ptr() if t is not None else None


def _bf16(name, t, shape=None):
    require_cuda(name, t, _BF16)
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")


def causal_conv1d_update(x: torch.Tensor, conv_state: torch.Tensor, weight: torch.Tensor,
                         bias: torch.Tensor | None = None, activation: str | None = None, stream=None) -> torch.Tensor:
    """x [B, D]; conv_state [B, D, W] (updated in place); weight [D, W];
    bias [D] or None; activation None | "silu" | "swish".  Returns y [B, D]."""
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("activation must be None, silu, or swish")
    Bn, D = x.shape
    W = conv_state.shape[-1]
    _bf16("x", x)
    _bf16("conv_state", conv_state, (Bn, D, W))
    _bf16("weight", weight, (D, W))
    if bias is not None:
        _bf16("bias", bias, (D,))
    y = torch.empty_like(x)
    act = _lib.SN_ACT_NONE if activation is None else _lib.SN_ACT_SILU
    call("sn_causal_conv1d_update", x.data_ptr(), conv_state.data_ptr(), weight.data_ptr(), _ptr(bias), y.data_ptr(),
         Bn, D, W, act, stream_handle(stream))
    return y


def selective_state_update(state: torch.Tensor, x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor,
                           B: torch.Tensor, C: torch.Tensor, D: torch.Tensor | None = None,
                           z: torch.Tensor | None = None, dt_bias: torch.Tensor | None = None,
                           dt_softplus: bool = False, stream=None) -> torch.Tensor:
    """state [batch, nheads, headdim, dstate] (updated in place); x, dt, z
    [batch, nheads, headdim]; A fp32 [nheads, headdim, dstate]; B, C [batch,
    ngroups, dstate]; D, dt_bias [nheads, headdim].  Returns y like x."""
    batch, nh, hd, ds = state.shape
    ng = B.shape[1]
    _bf16("state", state)
    for name, t in (("x", x), ("dt", dt)):
        _bf16(name, t, (batch, nh, hd))
    if z is not None:
        _bf16("z", z, (batch, nh, hd))
    require_cuda("A", A, torch.float32)
    if tuple(A.shape) != (nh, hd, ds) or not A.is_contiguous():
        raise ValueError(f"A must be a contiguous fp32 [{nh}, {hd}, {ds}] tensor")
    _bf16("B", B, (batch, ng, ds))
    _bf16("C", C, (batch, ng, ds))
    for name, t in (("D", D), ("dt_bias", dt_bias)):
        if t is not None:
            _bf16(name, t, (nh, hd))
    y = torch.empty_like(x)
    call("sn_selective_state_update", state.data_ptr(), x.data_ptr(), dt.data_ptr(), A.data_ptr(), B.data_ptr(),
         C.data_ptr(), _ptr(D), _ptr(z), _ptr(dt_bias), y.data_ptr(), batch, nh, hd, ds, ng, int(bool(dt_softplus)),
         stream_handle(stream))
    return y


def rmsnorm_fn(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, z: torch.Tensor | None = None,
               eps: float = 1e-6, group_size: int | None = None, norm_before_gate: bool = True,
               stream=None) -> torch.Tensor:
    """Gated RMSNorm over the last dimension in groups of group_size (None:
    the whole row); returns a new tensor like x."""
    N = x.shape[-1]
    g = N if group_size is None else int(group_size)
    _bf16("x", x)
    _bf16("weight", weight, (N,))
    if bias is not None:
        _bf16("bias", bias, (N,))
    if z is not None:
        _bf16("z", z, tuple(x.shape))
    y = torch.empty_like(x)
    call("sn_rmsnorm_gated", x.data_ptr(), weight.data_ptr(), _ptr(bias), _ptr(z), y.data_ptr(), x.numel() // N, N, g,
         float(eps), int(bool(norm_before_gate)), stream_handle(stream))
    return y


def layer_norm_fn(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, residual=None,
                  eps: float = 1e-6, prenorm: bool = False, residual_in_fp32: bool = False,
                  is_rms_norm: bool = False, stream=None):
    """Fused residual add + LayerNorm / RMSNorm over the last dimension.
    Returns out, or (out, residual_out) with prenorm; residual_out is x +
    residual in x's dtype (fp32 with residual_in_fp32)."""
    N = x.shape[-1]
    _bf16("x", x)
    _bf16("weight", weight, (N,))
    if bias is not None:
        _bf16("bias", bias, (N,))
    res_f32 = 0
    if residual is not None:
        require_cuda("residual", residual, None)
        if tuple(residual.shape) != tuple(x.shape) or not residual.is_contiguous():
            raise ValueError("residual must be contiguous with x's shape")
        if residual.dtype not in (_BF16, torch.float32):
            raise TypeError("residual must be bf16 or fp32")
        res_f32 = int(residual.dtype == torch.float32)
    out = torch.empty_like(x)
    rout = None
    if prenorm:
        rout = torch.empty(x.shape, device=x.device, dtype=torch.float32 if residual_in_fp32 else x.dtype)
    call("sn_layer_norm_fused", x.data_ptr(), _ptr(residual), res_f32, weight.data_ptr(), _ptr(bias), out.data_ptr(),
         _ptr(rout), int(rout is not None and rout.dtype == torch.float32), x.numel() // N, N, float(eps),
         int(bool(is_rms_norm)), stream_handle(stream))
    return (out, rout) if prenorm else out


def mamba2_split_conv(zxbcdt: torch.Tensor, conv_state: torch.Tensor, weight: torch.Tensor, bias, d_inner: int,
                      ngroups: int, d_state: int, nheads: int, stream=None):
    """The Mamba2 step between in_proj and selective_state_update in one
    launch: zxbcdt [b, >= width] (row stride taken from the tensor) ->
    (z [b, d_inner], x [b, nheads, headdim], B [b, ngroups, d_state],
    C [b, ngroups, d_state], dt [b, nheads, headdim]); conv_state updated in
    place (causal_conv1d_update with SiLU on xBC)."""
    require_cuda("zxbcdt", zxbcdt, _BF16, 2)
    if zxbcdt.stride(1) != 1:
        raise ValueError("zxbcdt must be contiguous along its last dimension")
    b = zxbcdt.shape[0]
    hd = d_inner // nheads
    conv_dim = d_inner + 2 * ngroups * d_state
    _bf16("conv_state", conv_state, (b, conv_dim, conv_state.shape[-1]))
    _bf16("weight", weight, (conv_dim, conv_state.shape[-1]))
    if bias is not None:
        _bf16("bias", bias, (conv_dim,))
    dev = zxbcdt.device
    z = torch.empty(b, d_inner, device=dev, dtype=_BF16)
    x = torch.empty(b, nheads, hd, device=dev, dtype=_BF16)
    Bm = torch.empty(b, ngroups, d_state, device=dev, dtype=_BF16)
    Cm = torch.empty(b, ngroups, d_state, device=dev, dtype=_BF16)
    dt = torch.empty(b, nheads, hd, device=dev, dtype=_BF16)
    call("sn_mamba2_split_conv", zxbcdt.data_ptr(), zxbcdt.stride(0) if b > 1 else zxbcdt.shape[1],
         conv_state.data_ptr(), weight.data_ptr(), _ptr(bias), z.data_ptr(), x.data_ptr(), Bm.data_ptr(),
         Cm.data_ptr(), dt.data_ptr(), b, d_inner, ngroups, d_state, nheads, hd, conv_state.shape[-1],
         stream_handle(stream))
    return z, x, Bm, Cm, dt


def mamba2_conv_ssu(zxbcdt: torch.Tensor, conv_state: torch.Tensor, weight: torch.Tensor, bias,
                    ssm_state: torch.Tensor, A: torch.Tensor, D, dt_bias, d_inner: int, ngroups: int,
                    d_state: int, nheads: int, sync: torch.Tensor, stream=None):
    """``mamba2_split_conv`` then ``selective_state_update`` (dt softplus,
    z applied later by the gated norm) in one launch: zxbcdt [b, >= width],
    conv_state and ssm_state [b, nheads, headdim, d_state] updated in place,
    A fp32 [nheads], D / dt_bias bf16 [nheads] or None (per head).  Returns
    (z [b, d_inner], y [b, nheads, headdim]), equal bit for bit to the
    two-launch path.  ``sync``: int32 [b * ngroups] zeros (the kernel leaves
    them zero); calls sharing it must not overlap."""
    require_cuda("zxbcdt", zxbcdt, _BF16, 2)
    if zxbcdt.stride(1) != 1:
        raise ValueError("zxbcdt must be contiguous along its last dimension")
    b = zxbcdt.shape[0]
    hd = d_inner // nheads
    conv_dim = d_inner + 2 * ngroups * d_state
    _bf16("conv_state", conv_state, (b, conv_dim, conv_state.shape[-1]))
    _bf16("weight", weight, (conv_dim, conv_state.shape[-1]))
    if bias is not None:
        _bf16("bias", bias, (conv_dim,))
    _bf16("ssm_state", ssm_state, (b, nheads, hd, d_state))
    require_cuda("A", A, torch.float32, 1)
    if tuple(A.shape) != (nheads,) or not A.is_contiguous():
        raise ValueError(f"A must be a contiguous fp32 [{nheads}] tensor")
    for name, t in (("D", D), ("dt_bias", dt_bias)):
        if t is not None:
            _bf16(name, t, (nheads,))
    require_cuda("sync", sync, torch.int32, 1)
    if sync.numel() < b * ngroups or not sync.is_contiguous():
        raise ValueError(f"sync must hold {b * ngroups} contiguous int32 counters")
    dev = zxbcdt.device
    z = torch.empty(b, d_inner, device=dev, dtype=_BF16)
    y = torch.empty(b, nheads, hd, device=dev, dtype=_BF16)
    call("sn_mamba2_conv_ssu", zxbcdt.data_ptr(), zxbcdt.stride(0) if b > 1 else zxbcdt.shape[1],
         conv_state.data_ptr(), weight.data_ptr(), _ptr(bias), ssm_state.data_ptr(), A.data_ptr(), _ptr(D),
         _ptr(dt_bias), z.data_ptr(), y.data_ptr(), sync.data_ptr(), b, d_inner, ngroups, d_state, nheads, hd,
         conv_state.shape[-1], stream_handle(stream))
    return z, y


def rotary_kv_append(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, cos: torch.Tensor,
                     sin: torch.Tensor, nheads: int, pos: int, stream=None) -> torch.Tensor:
    """q with rotary [b, nheads, 1, head_dim]; k (rotated) and v written at
    position pos of the caches [b, nheads_kv, max_seqlen, head_dim]."""
    _bf16("qkv", qkv)
    b, hk, S, hd = k_cache.shape
    _bf16("k_cache", k_cache)
    _bf16("v_cache", v_cache, (b, hk, S, hd))
    require_cuda("cos", cos, torch.float32)
    require_cuda("sin", sin, torch.float32)
    q = torch.empty(b, nheads, 1, hd, device=qkv.device, dtype=_BF16)
    call("sn_rotary_kv_append", qkv.data_ptr(), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), cos.data_ptr(),
         sin.data_ptr(), b, nheads, hk, hd, S, pos, stream_handle(stream))
    return q


def swiglu(h: torch.Tensor, stream=None) -> torch.Tensor:
    """h [b, 2d] -> h[:, :d] * SiLU(h[:, d:])."""
    _bf16("h", h)
    b, d2 = h.shape
    y = torch.empty(b, d2 // 2, device=h.device, dtype=_BF16)
    call("sn_swiglu", h.data_ptr(), y.data_ptr(), b, d2 // 2, stream_handle(stream))
    return y


def bench_step_ops(reps: int = 10, calls: int = 20, seed: int = 0) -> dict:
    """Microseconds per call of the four decode-step ops at the Zonos shapes of
    the reference's goldens (validation_harness.py:18-36: batch 2, d_inner
    4096, conv width 4 over 4352 channels, 64 heads x 64 x d_state 128,
    d_model 2048), each timed as `calls` back-to-back launches captured in a
    CUDA graph (CUDA events around `reps` replays), on device-resident
    synthetic inputs.  Bytes are the ops' algorithmic reads + writes."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    r = lambda *s: torch.randn(*s, device="cuda", generator=g)
    bf = _BF16
    x = r(2, 4352).to(bf); st = r(2, 4352, 4).to(bf); w = r(4352, 4).to(bf); b = r(4352).to(bf)
    state = r(2, 64, 64, 128).to(bf); xs = r(2, 64, 64).to(bf); dt = r(2, 64, 64).to(bf)
    A = (-torch.exp(r(64)))[:, None, None].expand(64, 64, 128).contiguous()
    Bm = r(2, 1, 128).to(bf); Cm = r(2, 1, 128).to(bf); D = r(64, 64).to(bf); dtb = r(64, 64).to(bf)
    xr = r(2, 4096).to(bf); wr = r(4096).to(bf); z = r(2, 4096).to(bf)
    xl = r(2, 1, 2048).to(bf); rl = r(2, 1, 2048).to(bf); wl = r(2048).to(bf); bl = r(2048).to(bf)
    ops = {
        "causal_conv1d_update": (lambda: causal_conv1d_update(x, st, w, b, "silu"),
                                 2 * 4352 * 2 * 2 + 2 * 4352 * 4 * 2 * 2 + 4352 * 5 * 2),
        "selective_state_update": (lambda: selective_state_update(state, xs, dt, A, Bm, Cm, D=D, dt_bias=dtb,
                                                                  dt_softplus=True),
                                   2 * 64 * 64 * 128 * 2 * 2 + 64 * 64 * 128 * 4 + 2 * 64 * 64 * 2 * 3),
        "rmsnorm_gated": (lambda: rmsnorm_fn(xr, wr, None, z=z, eps=1e-5, group_size=4096, norm_before_gate=False),
                          2 * 4096 * 2 * 3 + 4096 * 2),
        "layer_norm_fn_prenorm": (lambda: layer_norm_fn(xl, wl, bl, residual=rl, eps=1e-5, prenorm=True),
                                  2 * 2048 * 2 * 4 + 2048 * 4),
    }
    out = {}
    for name, (fn, nbytes) in ops.items():
        for _ in range(3):
            fn()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(calls):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            graph.replay()
        e.record()
        torch.cuda.synchronize()
        us = a.elapsed_time(e) * 1e3 / (reps * calls)
        out[name] = {"us_per_call": round(us, 2), "bytes": nbytes, "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}
    return {"metric": "Mamba2 decode-step ops µs per call (CUDA graph)", "unit": "us", "ops": out,
            "note": "latency-bound at decode shapes: each op moves 41 KB - 6.3 MB; the 20 calls of a replay reuse "
                    "one set of tensors, so operands are L2 hits after the first call (in a decode step the SSU "
                    "state would come from HBM)"}
