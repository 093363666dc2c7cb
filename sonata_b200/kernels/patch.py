"""Swap decode-shaped projection ``nn.Linear``s to the B200 GEMV.

Drop-in for the reference's kernels/patch.py (42-98), same names and
semantics:

* ``patch_linear(lin, batches=(1, 2))`` asserts the Linear has no bias
  (patch.py:44), binds the weight once, pins one output buffer per M and
  replaces ``lin.forward``.  2-D ``(M, K)`` inputs (Mamba2 ``step``) and 3-D
  ``(M, 1, K)`` inputs (attention / MLP at decode) with ``M in batches`` go to
  the GEMV; every other call (prefill, other M) falls back to the original
  forward (patch.py:54-66).  The returned tensor is the pinned buffer, reused
  by the next call, so the caller consumes it first (patch.py:49,65).  The
  launch goes to torch's current stream with no allocation or sync, so the
  patched forward can be captured inside a CUDA graph.
* ``unpatch_linear(lin)`` restores the original forward (patch.py:73-76).
* ``patch_zonos_projections(model, include_attn=False, verbose=False)``
  patches bias-free ``in_proj`` / ``out_proj`` / ``fc1`` / ``fc2`` Linears of
  ``model.backbone``, skipping attention layers unless ``include_attn``
  (patch.py:79-98).  Returns the number patched.

B200 additions:

* ``weight_format="int8" | "e4m3"`` quantises the weight once per output
  channel on the device and routes decode calls through the fused-dequant
  GEMV (bf16 output, as the Linear would produce); prefill keeps the original
  bf16 forward.
* Patched GEMVs are launched with programmatic dependent launch, which is
  valid because a frozen Linear weight is never written by the kernel before
  it in the decode step.
* ``link_decode_chain(linears)`` tells each patched Linear which one the
  decode step calls next; its GEMV then prefetches the start of that weight
  into L2 while it drains (a hint: a wrong order costs bandwidth, never
  results).  ``patch_zonos_projections(..., prefetch_chain=True)`` links the
  patched Linears in module order, which is the order Zonos' blocks call them.
"""
from __future__ import annotations

import torch

from .. import _lib
from ._common import require_cuda, stream_handle
from .gemv import MAX_M, QuantizedWeight, quantize_weight

_TARGETS = ("in_proj", "out_proj", "fc1", "fc2")


def _make_launch(W: torch.Tensor, qw: QuantizedWeight | None, lin: torch.nn.Linear):
    """Bind the weight once; return launch(x_contig, y, M).  The next-weight
    hint is read from ``lin._gemv_next`` at every call (set by
    link_decode_chain)."""
    N, K = W.shape
    lib = _lib.lib()
    flags = _lib.SN_FLAG_PDL
    ex = lib.sn_gemv_ex
    if qw is None:
        fn = lib.sn_gemv_bf16
        kind, w_ptr, s_ptr = _lib.SN_WEIGHT_BF16, W.data_ptr(), None

        def plain(xc, y, M):
            return fn(w_ptr, K, xc.data_ptr(), K, y.data_ptr(), N, M, N, K, _lib.SN_DTYPE_BF16, flags,
                      stream_handle())
    else:
        fn = lib.sn_gemv_int8 if qw.kind == "int8" else lib.sn_gemv_fp8e4m3
        kind = _lib.SN_WEIGHT_INT8 if qw.kind == "int8" else _lib.SN_WEIGHT_E4M3
        w_ptr, s_ptr = qw.q.data_ptr(), qw.scale.data_ptr()

        def plain(xc, y, M):
            return fn(w_ptr, K, s_ptr, xc.data_ptr(), K, y.data_ptr(), N, M, N, K, _lib.SN_DTYPE_BF16, flags,
                      stream_handle())

    def launch(xc: torch.Tensor, y: torch.Tensor, M: int) -> None:
        nxt = getattr(lin, "_gemv_next", None)
        if nxt is None:
            _lib.check("sn_gemv", plain(xc, y, M))
        else:
            _lib.check("sn_gemv_ex", ex(kind, w_ptr, K, s_ptr, xc.data_ptr(), K, y.data_ptr(), N, M, N, K,
                                        _lib.SN_DTYPE_BF16, flags, stream_handle(), *nxt[0]))
    return launch


def patch_linear(lin: torch.nn.Linear, batches=(1, 2), weight_format: str = "bf16"):
    """Route decode-shaped (M in `batches`) calls of `lin` through the GEMV kernel."""
    assert lin.bias is None, "GEMV kernel has no bias path"
    W = lin.weight.detach()
    require_cuda("lin.weight", W, torch.bfloat16, 2)
    if not W.is_contiguous():
        W = W.contiguous()
    N, K = W.shape
    batches = tuple(int(m) for m in batches)
    if any(not 1 <= m <= MAX_M for m in batches):
        raise ValueError(f"batches must lie in [1, {MAX_M}], got {batches}")
    if weight_format == "bf16":
        qw = None
    elif weight_format in ("int8", "e4m3"):
        qw = quantize_weight(W, weight_format)
    else:
        raise ValueError(f"weight_format must be bf16 | int8 | e4m3, got {weight_format!r}")
    launch = _make_launch(W, qw, lin)
    ybuf = {M: torch.empty(M, N, device=W.device, dtype=torch.bfloat16) for M in batches}
    orig = lin.forward

    def fwd(x):
        three_d = x.dim() == 3 and x.shape[1] == 1
        if x.dim() == 2 or three_d:
            x2 = x.squeeze(1) if three_d else x
            M = int(x2.shape[0])
            if M in ybuf and x2.shape[1] == K and x2.dtype == torch.bfloat16 and x2.device == W.device:
                xc = x2.detach().contiguous()
                launch(xc, ybuf[M], M)
                return ybuf[M].unsqueeze(1) if three_d else ybuf[M]
        return orig(x)  # prefill / unsupported -> original forward

    lin.forward = fwd
    lin._gemv_orig = orig
    lin._gemv_keepalive = (W, qw, ybuf)
    return lin


def unpatch_linear(lin: torch.nn.Linear):
    if hasattr(lin, "_gemv_orig"):
        lin.forward = lin._gemv_orig
        del lin._gemv_orig
        for attr in ("_gemv_keepalive", "_gemv_next"):
            if hasattr(lin, attr):
                delattr(lin, attr)


def link_decode_chain(linears, cyclic: bool = False) -> None:
    """Give each patched Linear of ``linears`` (in decode-step call order) the
    weight of the one after it as an L2 prefetch hint (sn_gemv_ex).  The last
    one gets none unless ``cyclic``.  Only patched Linears are linked; a
    Linear's hint is replaced by a later call and cleared by unpatch_linear.
    Launches already captured in a CUDA graph keep the hint they were
    captured with."""
    mods = [m for m in linears if hasattr(m, "_gemv_keepalive")]
    for i, m in enumerate(mods):
        j = i + 1
        if j == len(mods):
            if not cyclic or len(mods) < 2:
                m._gemv_next = None
                continue
            j = 0
        W, qw, _ = mods[j]._gemv_keepalive
        t = W if qw is None else qw.q
        kind = (_lib.SN_WEIGHT_BF16 if qw is None else
                _lib.SN_WEIGHT_INT8 if qw.kind == "int8" else _lib.SN_WEIGHT_E4M3)
        # (sn_gemv_ex's trailing arguments, the tensor they point into)
        m._gemv_next = ((kind, t.data_ptr(), t.stride(0), int(t.shape[0]), int(t.shape[1])), t)


def zonos_patch_targets(model, include_attn: bool = False):
    """(name, module) pairs patch_zonos_projections would patch (patch.py:82-92)."""
    attn = set(model.backbone.config.attn_layer_idx)
    out = []
    for name, mod in model.backbone.named_modules():
        if not (isinstance(mod, torch.nn.Linear) and name.endswith(_TARGETS)):
            continue
        if mod.bias is not None:  # GEMV has no bias path
            continue
        idx = next((int(p) for p in name.split(".") if p.isdigit()), None)
        if (idx in attn) and not include_attn:
            continue
        out.append((name, mod))
    return out


def patch_zonos_projections(model, include_attn=False, verbose=False, weight_format: str = "bf16",
                            prefetch_chain: bool = True) -> int:
    """Patch decode-shaped, bias-free projection Linears across the backbone:
    Mamba2 in_proj/out_proj always; attention qkv/out_proj and MLP fc1/fc2 when
    include_attn=True.  With ``prefetch_chain`` the patched Linears are linked
    in module order (link_decode_chain).  Returns the number patched."""
    n = 0
    mods = []
    for name, mod in zonos_patch_targets(model, include_attn):
        patch_linear(mod, weight_format=weight_format)
        mods.append(mod)
        n += 1
        if verbose:
            print(f"  patched {name}: {tuple(mod.weight.shape)}")
    if prefetch_chain:
        link_decode_chain(mods)
    return n
