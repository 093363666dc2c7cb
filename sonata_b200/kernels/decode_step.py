"""A Zonos-hybrid decode step on the B200 kernels, with synthetic weights.

The reference's production path is the patched ``nn.Linear`` inside Zonos's
graph-captured ``_decode_one_token`` (kernels/bench_decode.py:56-121,
kernels/patch.py:79-98).  The Zonos source and checkpoint are not available
offline, so this module builds a module tree of the same shape and names from
the backbone config the reference documents (docs/architecture.md:5-30,
138-170: d_model 2048, 46 layers, attention at layers 0, 4, ..., 44 with 16
query / 4 KV heads of 128 and rotary over the whole head, a gated MLP of
8192 after each attention mixer, Mamba2 mixers with d_inner 4096, 64 heads of
64, d_state 128, conv width 4, LayerNorm between blocks, eps 1e-5) and runs
one decode token through it:

* every block: fused residual add + LayerNorm (``layer_norm_fn``, prenorm);
* Mamba2 block (``Mamba2.step``, docs/architecture.md:212-236): ``in_proj``
  GEMV, split [z, xBC, dt], ``causal_conv1d_update`` with SiLU,
  ``selective_state_update`` (softplus(dt + dt_bias), D, no z), gated
  RMSNorm with SiLU(z), ``out_proj`` GEMV;
* attention block: ``in_proj`` (qkv) GEMV, rotary, one query over a KV cache
  (torch scaled_dot_product_attention), ``out_proj`` GEMV, add + LayerNorm,
  ``fc1`` GEMV, SwiGLU, ``fc2`` GEMV;
* final add + LayerNorm and the 9 codebook heads (the codebook-head kernel).

``patch_zonos_projections(model, include_attn=True)`` -- the reference's
drop-in call -- routes every projection through the GEMV kernel, so a step
runs the repository's GEMV, Mamba2-op and head kernels with the attention,
rotary and SwiGLU torch ops between them, as a real decode step does.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import gemv as G
from . import mamba_step as MS
from .bmm import CodebookHead

_BF16 = torch.bfloat16


@dataclass
class ZonosBackboneConfig:
    """The Zonos-v0.1-hybrid backbone config (docs/architecture.md:5-30)."""
    d_model: int = 2048
    n_layer: int = 46
    attn_layer_idx: list = field(default_factory=lambda: list(range(0, 46, 4)))
    attn_mlp_d_intermediate: int = 8192
    num_heads: int = 16
    num_heads_kv: int = 4
    head_dim: int = 128
    d_state: int = 128
    d_conv: int = 4
    headdim: int = 64
    expand: int = 2
    ngroups: int = 1
    norm_epsilon: float = 1e-5
    n_codebooks: int = 9
    vocab: int = 1025

    @property
    def d_inner(self):
        return self.expand * self.d_model

    @property
    def nheads(self):
        return self.d_inner // self.headdim


class Mamba2Mixer(torch.nn.Module):
    def __init__(self, cfg: ZonosBackboneConfig, device, g: torch.Generator):
        super().__init__()
        self.cfg = cfg
        di, ds, nh = cfg.d_inner, cfg.d_state, cfg.nheads
        self.conv_dim = di + 2 * cfg.ngroups * ds
        self.in_proj = torch.nn.Linear(cfg.d_model, 2 * di + 2 * cfg.ngroups * ds + nh, bias=False, device=device,
                                       dtype=_BF16)
        self.out_proj = torch.nn.Linear(di, cfg.d_model, bias=False, device=device, dtype=_BF16)
        r = lambda *s, sc=1.0: (torch.randn(*s, device=device, generator=g) * sc)
        with torch.no_grad():
            self.in_proj.weight.copy_(r(*self.in_proj.weight.shape, sc=0.02))
            self.out_proj.weight.copy_(r(*self.out_proj.weight.shape, sc=0.02))
        self.conv_w = r(self.conv_dim, cfg.d_conv, sc=0.5).to(_BF16)
        self.conv_b = r(self.conv_dim, sc=0.1).to(_BF16)
        self.A_log = torch.log(torch.rand(nh, device=device, generator=g) * 15 + 1)
        self.D = torch.ones(nh, device=device).to(_BF16)
        self.dt_bias = (torch.rand(nh, device=device, generator=g) * 2 - 4).to(_BF16)
        self.norm_w = (1 + 0.1 * r(di)).to(_BF16)
        # decode-time expansions (constant): A fp32 [nh, headdim, d_state], D / dt_bias [nh, headdim]
        self.A = (-torch.exp(self.A_log.float()))[:, None, None].expand(nh, cfg.headdim, ds).contiguous()
        self.D_e = self.D[:, None].expand(nh, cfg.headdim).contiguous()
        self.dt_bias_e = self.dt_bias[:, None].expand(nh, cfg.headdim).contiguous()
        self.A_h = (-torch.exp(self.A_log.float())).contiguous()  # per head, for the fused conv + SSU
        # split + conv and selective_state_update as one launch (sn_mamba2_conv_ssu) in the fused-norm step:
        # off by default, since in a CUDA graph with programmatic dependent launch the two launches measured as
        # fast or faster; it saves the launch outside a graph
        self.conv_ssu_supported = ds in (128, 256) and cfg.headdim % 16 == 0
        self.fused_conv_ssu = False

    def alloc_state(self, batch):
        cfg = self.cfg
        dev = self.conv_w.device
        self.conv_state = torch.zeros(batch, self.conv_dim, cfg.d_conv, device=dev, dtype=_BF16)
        self.ssm_state = torch.zeros(batch, cfg.nheads, cfg.headdim, cfg.d_state, device=dev, dtype=_BF16)
        self.sync = torch.zeros(batch * cfg.ngroups, device=dev, dtype=torch.int32)  # the fused kernel's counters

    def step_fused_norms(self, h: torch.Tensor, residual, norm_w, norm_b):
        """The block's add + LayerNorm fused into in_proj and the gated RMSNorm
        fused into out_proj (sn_gemv_bf16_norm): returns (out, residual)."""
        cfg = self.cfg
        b = h.shape[0]
        di, ds, nh = cfg.d_inner, cfg.d_state, cfg.nheads
        zxbcdt, residual = G.gemv_add_layernorm(h, residual, norm_w, norm_b, self.in_proj.weight,
                                                cfg.norm_epsilon, link=self.in_proj)
        if self.fused_conv_ssu:
            z, y = MS.mamba2_conv_ssu(zxbcdt, self.conv_state, self.conv_w, self.conv_b, self.ssm_state, self.A_h,
                                      self.D, self.dt_bias, di, cfg.ngroups, ds, nh, self.sync)
        else:
            z, x, Bm, Cm, dt_e = MS.mamba2_split_conv(zxbcdt, self.conv_state, self.conv_w, self.conv_b, di,
                                                      cfg.ngroups, ds, nh)
            y = MS.selective_state_update(self.ssm_state, x, dt_e, self.A, Bm, Cm, D=self.D_e, z=None,
                                          dt_bias=self.dt_bias_e, dt_softplus=True)
        out = G.gemv_rmsnorm_gated(y.view(b, di), z, self.norm_w, self.out_proj.weight, cfg.norm_epsilon,
                                   link=self.out_proj)
        return out, residual

    def step(self, u: torch.Tensor, fused_glue: bool = True) -> torch.Tensor:
        cfg = self.cfg
        b = u.shape[0]
        di, ds, nh = cfg.d_inner, cfg.d_state, cfg.nheads
        zxbcdt = self.in_proj(u)
        if fused_glue:
            z, x, Bm, Cm, dt_e = MS.mamba2_split_conv(zxbcdt, self.conv_state, self.conv_w, self.conv_b, di,
                                                      cfg.ngroups, ds, nh)
            y = MS.selective_state_update(self.ssm_state, x, dt_e, self.A, Bm, Cm, D=self.D_e, z=None,
                                          dt_bias=self.dt_bias_e, dt_softplus=True)
            y = MS.rmsnorm_fn(y.view(b, di), self.norm_w, None, z=z, eps=cfg.norm_epsilon,
                              group_size=di // cfg.ngroups, norm_before_gate=False)
            return self.out_proj(y)
        z = zxbcdt[:, :di].contiguous()
        xBC = zxbcdt[:, di:di + self.conv_dim].contiguous()
        dt = zxbcdt[:, di + self.conv_dim:]
        xBC = MS.causal_conv1d_update(xBC, self.conv_state, self.conv_w, self.conv_b, "silu")
        x = xBC[:, :di].view(b, nh, cfg.headdim)
        Bm = xBC[:, di:di + cfg.ngroups * ds].view(b, cfg.ngroups, ds)
        Cm = xBC[:, di + cfg.ngroups * ds:].view(b, cfg.ngroups, ds)
        dt_e = dt[:, :, None].expand(b, nh, cfg.headdim).contiguous()
        y = MS.selective_state_update(self.ssm_state, x.contiguous(), dt_e, self.A, Bm.contiguous(), Cm.contiguous(),
                                      D=self.D_e, z=None, dt_bias=self.dt_bias_e, dt_softplus=True)
        y = MS.rmsnorm_fn(y.view(b, di), self.norm_w, None, z=z, eps=cfg.norm_epsilon, group_size=di // cfg.ngroups,
                          norm_before_gate=False)
        return self.out_proj(y)


def rotary_cos_sin(pos: int, dim: int, device, base: float = 10000.0):
    inv = 1.0 / (base ** (torch.arange(0, dim, 2, device=device, dtype=torch.float32) / dim))
    ang = pos * inv
    return torch.cos(ang), torch.sin(ang)


def apply_rotary(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Non-interleaved rotary on the last dimension (the halves rotate): x
    [..., D] bf16, cos / sin [D/2] fp32; fp32 arithmetic, bf16 result."""
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h].float(), x[..., h:].float()
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)


class AttnMixer(torch.nn.Module):
    def __init__(self, cfg: ZonosBackboneConfig, device, g: torch.Generator):
        super().__init__()
        self.cfg = cfg
        qkv = (cfg.num_heads + 2 * cfg.num_heads_kv) * cfg.head_dim
        self.in_proj = torch.nn.Linear(cfg.d_model, qkv, bias=False, device=device, dtype=_BF16)
        self.out_proj = torch.nn.Linear(cfg.num_heads * cfg.head_dim, cfg.d_model, bias=False, device=device,
                                        dtype=_BF16)
        with torch.no_grad():
            self.in_proj.weight.copy_(torch.randn(*self.in_proj.weight.shape, device=device, generator=g) * 0.02)
            self.out_proj.weight.copy_(torch.randn(*self.out_proj.weight.shape, device=device, generator=g) * 0.02)

    def alloc_state(self, batch, max_seqlen, device, g: torch.Generator, prefix: int):
        """KV cache [batch, kv heads, max_seqlen, head_dim] with `prefix`
        positions already filled (a synthetic context)."""
        cfg = self.cfg
        shape = (batch, cfg.num_heads_kv, max_seqlen, cfg.head_dim)
        self.k_cache = torch.zeros(shape, device=device, dtype=_BF16)
        self.v_cache = torch.zeros(shape, device=device, dtype=_BF16)
        self.k_cache[:, :, :prefix] = torch.randn(batch, cfg.num_heads_kv, prefix, cfg.head_dim, device=device,
                                                  generator=g).to(_BF16)
        self.v_cache[:, :, :prefix] = torch.randn(batch, cfg.num_heads_kv, prefix, cfg.head_dim, device=device,
                                                  generator=g).to(_BF16)

    def step_fused_norms(self, h, residual, norm_w, norm_b, pos: int, cos, sin):
        """add + LayerNorm fused into the qkv projection; returns (out, residual)."""
        cfg = self.cfg
        b = h.shape[0]
        hq, hd = cfg.num_heads, cfg.head_dim
        qkv, residual = G.gemv_add_layernorm(h, residual, norm_w, norm_b, self.in_proj.weight, cfg.norm_epsilon,
                                             link=self.in_proj)
        q = MS.rotary_kv_append(qkv, self.k_cache, self.v_cache, cos, sin, hq, pos)
        o = F.scaled_dot_product_attention(q, self.k_cache[:, :, :pos + 1], self.v_cache[:, :, :pos + 1],
                                           enable_gqa=True)
        return self.out_proj(o.reshape(b, hq * hd)), residual

    def step(self, u: torch.Tensor, pos: int, cos, sin, fused_glue: bool = True) -> torch.Tensor:
        cfg = self.cfg
        b = u.shape[0]
        hq, hk, hd = cfg.num_heads, cfg.num_heads_kv, cfg.head_dim
        qkv = self.in_proj(u)
        if fused_glue:
            q = MS.rotary_kv_append(qkv, self.k_cache, self.v_cache, cos, sin, hq, pos)
            o = F.scaled_dot_product_attention(q, self.k_cache[:, :, :pos + 1], self.v_cache[:, :, :pos + 1],
                                               enable_gqa=True)
            return self.out_proj(o.reshape(b, hq * hd))
        q = apply_rotary(qkv[:, :hq * hd].view(b, hq, 1, hd), cos, sin)
        k = apply_rotary(qkv[:, hq * hd:(hq + hk) * hd].view(b, hk, 1, hd), cos, sin)
        v = qkv[:, (hq + hk) * hd:].view(b, hk, 1, hd)
        self.k_cache[:, :, pos:pos + 1] = k
        self.v_cache[:, :, pos:pos + 1] = v
        o = F.scaled_dot_product_attention(q, self.k_cache[:, :, :pos + 1], self.v_cache[:, :, :pos + 1],
                                           enable_gqa=True)
        return self.out_proj(o.reshape(b, hq * hd))


class GatedMLP(torch.nn.Module):
    def __init__(self, cfg: ZonosBackboneConfig, device, g: torch.Generator):
        super().__init__()
        d = cfg.attn_mlp_d_intermediate
        self.fc1 = torch.nn.Linear(cfg.d_model, 2 * d, bias=False, device=device, dtype=_BF16)
        self.fc2 = torch.nn.Linear(d, cfg.d_model, bias=False, device=device, dtype=_BF16)
        with torch.no_grad():
            self.fc1.weight.copy_(torch.randn(*self.fc1.weight.shape, device=device, generator=g) * 0.02)
            self.fc2.weight.copy_(torch.randn(*self.fc2.weight.shape, device=device, generator=g) * 0.02)

    def forward_fused_norm(self, h, residual, norm_w, norm_b, eps):
        """add + LayerNorm fused into fc1; returns (out, residual)."""
        y, residual = G.gemv_add_layernorm(h, residual, norm_w, norm_b, self.fc1.weight, eps, link=self.fc1)
        return self.fc2(MS.swiglu(y)), residual

    def forward(self, u, fused_glue: bool = True):
        if fused_glue:
            return self.fc2(MS.swiglu(self.fc1(u)))
        y, gate = self.fc1(u).chunk(2, dim=-1)
        return self.fc2(y * F.silu(gate))


class Block(torch.nn.Module):
    def __init__(self, cfg, idx, device, g):
        super().__init__()
        self.is_attn = idx in cfg.attn_layer_idx
        d = cfg.d_model
        self.norm_w = (1 + 0.1 * torch.randn(d, device=device, generator=g)).to(_BF16)
        self.norm_b = (0.02 * torch.randn(d, device=device, generator=g)).to(_BF16)
        self.mixer = AttnMixer(cfg, device, g) if self.is_attn else Mamba2Mixer(cfg, device, g)
        if self.is_attn:
            self.norm2_w = (1 + 0.1 * torch.randn(d, device=device, generator=g)).to(_BF16)
            self.norm2_b = (0.02 * torch.randn(d, device=device, generator=g)).to(_BF16)
            self.mlp = GatedMLP(cfg, device, g)


class _Backbone(torch.nn.Module):
    def __init__(self, cfg, device, g):
        super().__init__()
        self.config = cfg
        self.layers = torch.nn.ModuleList([Block(cfg, i, device, g) for i in range(cfg.n_layer)])
        d = cfg.d_model
        self.norm_f_w = (1 + 0.1 * torch.randn(d, device=device, generator=g)).to(_BF16)
        self.norm_f_b = (0.02 * torch.randn(d, device=device, generator=g)).to(_BF16)


class SyntheticZonos(torch.nn.Module):
    """Zonos-hybrid-shaped model (``model.backbone.layers[i].mixer.in_proj``
    ... the names ``patch_zonos_projections`` walks) with seeded synthetic
    weights, decode state for ``batch`` streams and a KV cache with
    ``context`` filled positions."""

    def __init__(self, cfg: ZonosBackboneConfig | None = None, batch: int = 1, context: int = 256,
                 max_seqlen: int = 1024, device="cuda", seed: int = 0):
        super().__init__()
        self.cfg = cfg or ZonosBackboneConfig()
        self.fused_glue = True  # False: the glue between the kernels as plain torch ops
        # norms fused into the next GEMV's x staging (needs fused_glue and
        # patched projections: patch_zonos_projections)
        self.fused_norms = False
        g = torch.Generator(device=device).manual_seed(seed)
        self.backbone = _Backbone(self.cfg, device, g)
        self.batch = batch
        self.pos = context
        for blk in self.backbone.layers:
            if blk.is_attn:
                blk.mixer.alloc_state(batch, max_seqlen, device, g, context)
            else:
                blk.mixer.alloc_state(batch)
        c = self.cfg
        self.head_W = (torch.randn(c.n_codebooks, c.d_model, c.vocab, device=device, generator=g) * 0.02).to(_BF16)
        self.head = CodebookHead(self.head_W)
        self.cos, self.sin = rotary_cos_sin(self.pos, self.cfg.head_dim, device)

    def weight_bytes(self) -> int:
        n = sum(m.weight.numel() for m in self.modules() if isinstance(m, torch.nn.Linear))
        return 2 * (n + self.head_W.numel())

    def projections(self):
        """The decode step's projection Linears in call order."""
        out = []
        for blk in self.backbone.layers:
            out += [blk.mixer.in_proj, blk.mixer.out_proj]
            if blk.is_attn:
                out += [blk.mlp.fc1, blk.mlp.fc2]
        return out

    def step(self, hidden: torch.Tensor) -> torch.Tensor:
        """One decode token: hidden [batch, d_model] bf16 -> logits fp32
        [n_codebooks, batch, vocab].  Updates the conv / SSM states and writes
        the KV cache at the current position (the position itself is fixed:
        repeated steps model a decoder at a constant context length)."""
        cfg = self.cfg
        eps = cfg.norm_epsilon
        residual = None
        h = hidden
        fg = self.fused_glue
        if fg and self.fused_norms:
            for blk in self.backbone.layers:
                if blk.is_attn:
                    h, residual = blk.mixer.step_fused_norms(h, residual, blk.norm_w, blk.norm_b, self.pos, self.cos,
                                                             self.sin)
                    h, residual = blk.mlp.forward_fused_norm(h, residual, blk.norm2_w, blk.norm2_b, eps)
                else:
                    h, residual = blk.mixer.step_fused_norms(h, residual, blk.norm_w, blk.norm_b)
            h = MS.layer_norm_fn(h, self.backbone.norm_f_w, self.backbone.norm_f_b, residual=residual, eps=eps)
            hid = h.unsqueeze(0).expand(cfg.n_codebooks, *h.shape).contiguous()
            return self.head(hid, pdl=True)
        for blk in self.backbone.layers:
            h, residual = MS.layer_norm_fn(h, blk.norm_w, blk.norm_b, residual=residual, eps=eps, prenorm=True)
            if blk.is_attn:
                h = blk.mixer.step(h, self.pos, self.cos, self.sin, fused_glue=fg)
                h, residual = MS.layer_norm_fn(h, blk.norm2_w, blk.norm2_b, residual=residual, eps=eps, prenorm=True)
                h = blk.mlp(h, fused_glue=fg)
            else:
                h = blk.mixer.step(h, fused_glue=fg)
        h = MS.layer_norm_fn(h, self.backbone.norm_f_w, self.backbone.norm_f_b, residual=residual, eps=eps)
        hid = h.unsqueeze(0).expand(cfg.n_codebooks, *h.shape).contiguous()
        return self.head(hid, pdl=True)


def bench_decode_step(steps: int = 20, warmup: int = 3, batch: int = 1, seed: int = 0) -> dict:
    """Microseconds per decode step of the 46-layer synthetic Zonos hybrid,
    each step one replay of a CUDA graph of the whole step (the reference's
    measure_cg, kernels/bench_decode.py:56-96), in three variants of the same
    model: the GEMV kernel with programmatic dependent launch and the
    next-weight L2 prefetch (``patch_zonos_projections(include_attn=True)``),
    the GEMV kernel without the prefetch chain, and the unpatched nn.Linear
    (cuBLAS); and the first variant with the glue between the kernels as
    plain torch ops (slices made contiguous, rotary, SwiGLU) instead of the
    fused glue kernels, and with split + conv and selective_state_update as one
    launch (sn_mamba2_conv_ssu) instead of two.  A replay after changing the input
    must change the logits (the empty-graph tripwire of
    bench_decode.py:114-121)."""
    from .patch import patch_zonos_projections, unpatch_linear
    model = SyntheticZonos(batch=batch, seed=seed)
    x = torch.randn(batch, model.cfg.d_model, device="cuda",
                    generator=torch.Generator(device="cuda").manual_seed(seed + 1)).to(_BF16)
    wbytes = model.weight_bytes()

    def capture():
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.no_grad(), torch.cuda.stream(s):
            for _ in range(2):
                model.step(x)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(g):
            out = model.step(x)
        return g, out

    def timed(g):
        for _ in range(warmup):
            g.replay()
        torch.cuda.synchronize()
        a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            g.replay()
        e.record()
        torch.cuda.synchronize()
        return a.elapsed_time(e) * 1e3 / steps

    res = {}
    n = patch_zonos_projections(model, include_attn=True, prefetch_chain=True)
    model.fused_glue = False
    g, out = capture()
    res["torch_glue"] = timed(g)
    del g
    model.fused_glue = True
    g, out = capture()
    res["gemv_unfused_norms"] = timed(g)
    del g
    model.fused_norms = True
    g, out = capture()
    res["gemv_pdl_prefetch"] = timed(g)
    before = out.clone()
    x.mul_(-1.0)
    g.replay()
    torch.cuda.synchronize()
    if torch.equal(before, out) or not torch.isfinite(out).all():
        raise RuntimeError("decode-step graph replay did not recompute (tripwire)")
    x.mul_(-1.0)
    del g
    mixers = [blk.mixer for blk in model.backbone.layers if not blk.is_attn]
    fused_cs = [mx.fused_conv_ssu for mx in mixers]
    for mx in mixers:  # split + conv and selective_state_update as one launch where supported
        mx.fused_conv_ssu = mx.conv_ssu_supported
    g, out = capture()
    res["one_launch_conv_ssu"] = timed(g)
    del g
    for mx, f in zip(mixers, fused_cs):
        mx.fused_conv_ssu = f
    for m in model.projections():
        if hasattr(m, "_gemv_next"):
            m._gemv_next = None
    g, out = capture()
    res["gemv_pdl"] = timed(g)
    model.fused_norms = False
    del g
    for m in model.projections():
        unpatch_linear(m)
    g, out = capture()
    res["cublas"] = timed(g)
    del g
    us = res["gemv_pdl_prefetch"]
    cfg = model.cfg
    n_attn = len(cfg.attn_layer_idx)
    # with the fused glue and norms: per Mamba2 block the fused conv + SSU
    # (or split+conv and SSU); per attention block rotary+cache, SDPA and
    # SwiGLU; then the final norm and the head's input copy
    launches_other = sum(1 if f else 2 for f in fused_cs) + n_attn * 3 + 2
    return {
        "metric": "synthetic Zonos-hybrid decode step µs (46 layers, CUDA graph)",
        "value": round(us, 1),
        "unit": "us per step",
        "batch": batch,
        "weight_bytes": wbytes,
        "weight_gbs": round(wbytes / (us * 1e-6) / 1e9, 1),
        "us_gemv_without_prefetch_chain": round(res["gemv_pdl"], 1),
        "us_torch_glue": round(res["torch_glue"], 1),
        "us_norms_as_kernels": round(res["gemv_unfused_norms"], 1),
        "us_conv_ssu_one_launch": round(res["one_launch_conv_ssu"], 1),
        "us_cublas_linear": round(res["cublas"], 1),
        "patched_linears": n,
        "tokens_per_s": round(1e6 / us, 1),
        "frame_budget_frac": round(us / 11610.0, 4),
        "workload": f"46 layers ({cfg.n_layer - n_attn} Mamba2, {n_attn} attention + gated MLP), d_model 2048, batch "
                    f"{batch}, KV context {model.pos}, synthetic weights; per token: add+LayerNorm, Mamba2 step "
                    "(in_proj GEMV, split + causal_conv1d_update, selective_state_update, gated RMSNorm, out_proj "
                    "GEMV) or attention (qkv GEMV, rotary + KV append, SDPA over the cache, o_proj GEMV, "
                    "add+LayerNorm, fc1 GEMV, SwiGLU, fc2 GEMV), final norm, 9 codebook heads",
        "non_gemv_launches_approx": launches_other,
    }
