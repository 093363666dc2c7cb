"""Decode GEMV: y[M, N] = x[M, K] . W[N, K]^T, bf16 in, fp32 accumulate.

Drop-in for the reference's kernels/gemv.py:

* ``candidate_cute``, ``candidate_cute_coalesced``, ``candidate_cute_splitk``
  (gemv.py:215-219): functional ``(x[M, K], W[N, K]) -> y[M, N]`` bf16 on x's
  device, allocating ``y`` on every call like ``_run`` (gemv.py:199-212).
* ``skinny_gemv``, ``skinny_gemv_coalesced``, ``skinny_gemv_splitk_m1``,
  ``skinny_gemv_splitk_m2`` (gemv.py:38-54, 169-193): launchers with the
  reference's ``(y, x, W, M, N, K, stream)`` argument order that write into a
  caller-owned ``y`` on ``stream`` without allocating, so they can be captured
  in a CUDA graph.

The reference's four launchers are four kernel *variants* of one contract; on
B200 they all run the same tuned sm_100a kernel (``sn_gemv_bf16``), which
streams W once with 16-byte non-allocating loads, accumulates in fp32 and
rounds to bf16 once in the epilogue.  Unlike ``_skinny_gemv_splitk_m2_kernel``
(gemv.py:135), K need not be a multiple of 8: the tail is summed, not dropped.

Additions: ``gemv`` (fp32 or bf16 output, optional programmatic dependent
launch), and the fused-dequant weight-only GEMVs ``gemv_int8`` /
``gemv_fp8e4m3`` with ``quantize_weight`` (the real kernels behind
scripts/fake_quant.py's simulation).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from .. import _lib
from ._common import call, require_cuda, row_major, stream_handle

_BF16 = torch.bfloat16
MAX_M = 4


def _check_gemv(x: torch.Tensor, W: torch.Tensor):
    require_cuda("x", x, _BF16, 2)
    require_cuda("W", W, _BF16, 2)
    M, K = x.shape
    N, K2 = W.shape
    if K2 != K:
        raise ValueError(f"x has K={K} but W has K={K2}")
    if not 1 <= M <= MAX_M:
        raise ValueError(f"M={M}: the decode GEMV supports 1 <= M <= {MAX_M}")
    if x.device != W.device:
        raise ValueError("x and W must be on the same device")
    return M, N, K


def _next_args(next_weight, device) -> tuple:
    """(kind, pointer, row stride, N, K) of sn_gemv_ex's next-weight hint."""
    if next_weight is None:
        return (_lib.SN_WEIGHT_BF16, None, 0, 0, 0)
    if isinstance(next_weight, QuantizedWeight):
        t = next_weight.q
        kind = _lib.SN_WEIGHT_INT8 if next_weight.kind == "int8" else _lib.SN_WEIGHT_E4M3
    else:
        t = next_weight
        require_cuda("next_weight", t, _BF16, 2)
        kind = _lib.SN_WEIGHT_BF16
    if t.dim() != 2 or t.device != device:
        raise ValueError("next_weight must be a 2-D weight on the GEMV's device")
    return (kind, t.data_ptr(), row_major("next_weight", t), int(t.shape[0]), int(t.shape[1]))


def gemv(x: torch.Tensor, W: torch.Tensor, out: torch.Tensor | None = None, out_dtype=_BF16,
         pdl: bool = False, stream=None, next_weight=None) -> torch.Tensor:
    """y = x @ W.T with fp32 accumulation; y is bf16 (RNE) or fp32.

    ``pdl=True`` lets the kernel overlap the previous kernel on the stream;
    only use it when that kernel does not write W.  ``next_weight`` (a bf16
    weight or a ``QuantizedWeight``) names the weight of the GEMV launched
    next on the stream: its first bytes are prefetched into L2 while this one
    drains.  It changes no result.
    """
    M, N, K = _check_gemv(x, W)
    if out is None:
        out = torch.empty(M, N, device=x.device, dtype=out_dtype)
    require_cuda("out", out, None, 2)
    if out.shape != (M, N) or out.dtype not in (_BF16, torch.float32):
        raise ValueError(f"out must be [{M}, {N}] bf16 or fp32")
    y_dtype = _lib.SN_DTYPE_F32 if out.dtype == torch.float32 else _lib.SN_DTYPE_BF16
    flags = _lib.SN_FLAG_PDL if pdl else 0
    if next_weight is None:
        call("sn_gemv_bf16", W.data_ptr(), row_major("W", W), x.data_ptr(), row_major("x", x), out.data_ptr(),
             row_major("out", out), M, N, K, y_dtype, flags, stream_handle(stream))
    else:
        call("sn_gemv_ex", _lib.SN_WEIGHT_BF16, W.data_ptr(), row_major("W", W), None, x.data_ptr(),
             row_major("x", x), out.data_ptr(), row_major("out", out), M, N, K, y_dtype, flags,
             stream_handle(stream), *_next_args(next_weight, x.device))
    return out


class GemvChain:
    """A list of decode GEMVs ``y_j = x_j @ W_j.T`` run by ONE persistent
    launch (``sn_gemv_chain_*``), e.g. the per-token projection set of a
    decode step.  Each CTA streams the jobs' weights in order through one
    ring, so HBM reads the next job's weights while the current one finishes;
    a job's x waits, inside the kernel, for the job named in ``deps``.

    jobs: ``(W, x [M, K] bf16, y [M, N] bf16 or fp32)`` triples, M (1 or 2)
    common to all; W is a bf16 [N, K] weight or, for every job alike, a
    ``QuantizedWeight`` of one kind (the fused-dequant int8 / e4m3 GEMV).
    deps: ``"serial"`` (job j waits for job j-1: the order of back-to-back
    launches on one stream), ``"none"`` (every x is ready when the launch
    starts) or a list of earlier job indices (-1: none).  The plan is
    validated and uploaded once; ``__call__`` only launches (CUDA graph
    capturable).  bf16 and int8 results equal ``gemv`` / ``gemv_quantized``
    on each job bit for bit; e4m3 within fp32 summation order.
    """

    def __init__(self, jobs, deps="serial", device=None):
        if not jobs:
            raise ValueError("GemvChain needs at least one job")
        n = len(jobs)
        if deps == "serial":
            deps = [j - 1 for j in range(n)]
        elif deps == "none":
            deps = [-1] * n
        deps = [int(d) for d in deps]
        if len(deps) != n:
            raise ValueError("deps must name one dependency per job")
        kinds = {(w.kind if isinstance(w, QuantizedWeight) else "bf16") for (w, _, _) in jobs}
        if len(kinds) != 1:
            raise ValueError(f"every job of a chain has the same weight kind, got {sorted(kinds)}")
        kind = kinds.pop()
        w_kind = {"bf16": _lib.SN_WEIGHT_BF16, "int8": _lib.SN_WEIGHT_INT8, "e4m3": _lib.SN_WEIGHT_E4M3}[kind]
        arr = (_lib.GemvJob * n)()
        M = None
        self._keep = []
        for j, (W, x, y) in enumerate(jobs):
            if kind == "bf16":
                Mj, N, K = _check_gemv(x, W)
                codes, scale = W, None
            else:
                require_cuda("x", x, _BF16, 2)
                codes, scale = W.q, W.scale
                Mj, K = x.shape
                N = codes.shape[0]
                if codes.shape[1] != K or scale.shape != (N,) or scale.dtype != torch.float32:
                    raise ValueError(f"job {j}: quantised weight does not match x")
            require_cuda("y", y, None, 2)
            if y.shape != (Mj, N) or y.dtype not in (_BF16, torch.float32):
                raise ValueError(f"job {j}: y must be [{Mj}, {N}] bf16 or fp32")
            if M is None:
                M = Mj
            elif Mj != M:
                raise ValueError("every job of a chain has the same M")
            arr[j] = _lib.GemvJob(codes.data_ptr(), x.data_ptr(), y.data_ptr(),
                                  scale.data_ptr() if scale is not None else None, row_major("W", codes),
                                  row_major("x", x), row_major("y", y), N, K, deps[j],
                                  _lib.SN_DTYPE_F32 if y.dtype == torch.float32 else _lib.SN_DTYPE_BF16)
            self._keep += [codes, x, y] + ([scale] if scale is not None else [])
        if not 1 <= M <= 2:
            raise ValueError("a GEMV chain takes M <= 2")
        dev = device if device is not None else jobs[0][1].device
        nbytes = _lib.lib().sn_gemv_chain_workspace_size(n)
        if nbytes == 0:
            raise ValueError(f"{n} jobs: outside the chain's limits")
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.info = _lib.GemvChainInfo()
        call("sn_gemv_chain_plan", w_kind, ctypes.addressof(arr), n, M, self.workspace.data_ptr(), nbytes,
             ctypes.byref(self.info), stream_handle(None))
        self.njobs, self.M, self.deps, self.kind = n, M, deps, kind
        self.outputs = [y for (_, _, y) in jobs]

    def __call__(self, pdl: bool = False, stream=None):
        call("sn_gemv_chain_launch", ctypes.byref(self.info), self.workspace.data_ptr(),
             _lib.SN_FLAG_PDL if pdl else 0, stream_handle(stream))
        return self.outputs


def _linear_next(lin) -> tuple:
    """sn_gemv_ex's next-weight arguments from a patched Linear's chain link
    (kernels.patch.link_decode_chain), or none."""
    nxt = getattr(lin, "_gemv_next", None) if lin is not None else None
    return nxt[0] if nxt is not None else (_lib.SN_WEIGHT_BF16, None, 0, 0, 0)


def _gemv_norm(kind, x, aux, norm_w, norm_b, W, eps, residual_out, out, pdl, stream, link):
    M, N, K = _check_gemv(x, W)
    for name, t in (("aux", aux), ("residual_out", residual_out)):
        if t is not None:
            require_cuda(name, t, _BF16, 2)
            if tuple(t.shape) != (M, K) or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous bf16 [{M}, {K}] tensor")
    for name, t in (("norm_w", norm_w), ("norm_b", norm_b)):
        if t is not None:
            require_cuda(name, t, _BF16)
            if t.numel() != K or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous bf16 [{K}] tensor")
    if not x.is_contiguous():
        raise ValueError("x must be contiguous")
    if out is None:
        out = torch.empty(M, N, device=x.device, dtype=_BF16)
    call("sn_gemv_bf16_norm", kind, W.data_ptr(), row_major("W", W), x.data_ptr(),
         aux.data_ptr() if aux is not None else None, norm_w.data_ptr(),
         norm_b.data_ptr() if norm_b is not None else None,
         residual_out.data_ptr() if residual_out is not None else None, float(eps), out.data_ptr(), N, M, N, K,
         _lib.SN_DTYPE_BF16, _lib.SN_FLAG_PDL if pdl else 0, stream_handle(stream), *_linear_next(link))
    return out


def gemv_rmsnorm_gated(x: torch.Tensor, z: torch.Tensor | None, norm_w: torch.Tensor, W: torch.Tensor,
                       eps: float = 1e-5, out=None, pdl: bool = True, stream=None, link=None) -> torch.Tensor:
    """``rmsnorm_fn(x, norm_w, None, z, eps, norm_before_gate=False)`` (one
    group over the row) followed by ``x' @ W.T``, the norm done inside the
    GEMV's x staging (``sn_gemv_bf16_norm``): one launch for the Mamba2 step's
    gated RMSNorm -> out_proj.  ``link``: a patched Linear whose next-weight
    hint to use."""
    return _gemv_norm(_lib.SN_NORM_RMS_GATED, x, z, norm_w, None, W, eps, None, out, pdl, stream, link)


def gemv_add_layernorm(x: torch.Tensor, residual: torch.Tensor | None, norm_w: torch.Tensor,
                       norm_b: torch.Tensor | None, W: torch.Tensor, eps: float = 1e-5, out=None,
                       pdl: bool = True, stream=None, link=None):
    """``layer_norm_fn(x, norm_w, norm_b, residual, eps, prenorm=True)``
    followed by ``x' @ W.T`` in one launch: returns (y, residual_out) with
    residual_out = x + residual (bf16), as the block entry of a Zonos decode
    step feeds in_proj / qkv / fc1."""
    M, K = x.shape
    rout = torch.empty(M, K, device=x.device, dtype=_BF16)
    y = _gemv_norm(_lib.SN_NORM_ADD_LAYER, x, residual, norm_w, norm_b, W, eps, rout, out, pdl, stream, link)
    return y, rout


def _launcher(y, x, W, M, N, K, stream):
    if tuple(x.shape) != (M, K) or tuple(W.shape) != (N, K) or tuple(y.shape) != (M, N):
        raise ValueError("shapes of y, x, W disagree with M, N, K")
    gemv(x, W, out=y, stream=stream)


def skinny_gemv(y, x, W, M, N, K, stream=None):
    """Launcher with the signature of kernels/gemv.py:38-54."""
    _launcher(y, x, W, M, N, K, stream)


def skinny_gemv_coalesced(y, x, W, M, N, K, stream=None):
    """Launcher with the signature of kernels/gemv.py:169-175."""
    _launcher(y, x, W, M, N, K, stream)


def skinny_gemv_splitk_m1(y, x, W, M, N, K, stream=None):
    """Launcher with the signature of kernels/gemv.py:179-185 (M == 1)."""
    _launcher(y, x, W, M, N, K, stream)


def skinny_gemv_splitk_m2(y, x, W, M, N, K, stream=None):
    """Launcher with the signature of kernels/gemv.py:187-193 (M == 2)."""
    _launcher(y, x, W, M, N, K, stream)


def candidate_cute(x, W):
    return gemv(x, W)


def candidate_cute_coalesced(x, W):
    return gemv(x, W)


def candidate_cute_splitk(x, W):
    return gemv(x, W)


# ---------------------------------------------------------------------------
# weight-only quantised GEMV
# ---------------------------------------------------------------------------

@dataclass
class QuantizedWeight:
    """Per-output-channel quantised weight: codes [N, K] + fp32 scale [N]."""
    q: torch.Tensor       # int8 (kind "int8") or uint8 e4m3 bit patterns (kind "e4m3")
    scale: torch.Tensor   # fp32 [N]
    kind: str

    @property
    def shape(self):
        return tuple(self.q.shape)

    def dequantize(self) -> torch.Tensor:
        """fp32 ``q * scale`` (scripts/fake_quant.py:41 before its dtype cast)."""
        if self.kind == "int8":
            c = self.q.float()
        else:
            c = self.q.view(torch.float8_e4m3fn).float()
        return c * self.scale[:, None]


def quantize_weight(W: torch.Tensor, kind: str = "int8", stream=None) -> QuantizedWeight:
    """Quantise a bf16 [N, K] weight per output channel on the device.

    int8: scale = max(amax_row, 1e-8) / 127, q = round-half-even(w / scale),
    identical to scripts/fake_quant.py:16-42 (bits=8, group_size=None).
    e4m3: scale = max(amax_row, 1e-8) / 448, q = e4m3_rn(w / scale).
    """
    require_cuda("W", W, _BF16, 2)
    N, K = W.shape
    if kind == "int8":
        q = torch.empty(N, K, device=W.device, dtype=torch.int8)
        fn = "sn_quantize_rows_int8"
    elif kind == "e4m3":
        q = torch.empty(N, K, device=W.device, dtype=torch.uint8)
        fn = "sn_quantize_rows_fp8e4m3"
    else:
        raise ValueError(f"unknown quantisation kind {kind!r} (int8 | e4m3)")
    scale = torch.empty(N, device=W.device, dtype=torch.float32)
    call(fn, W.data_ptr(), row_major("W", W), N, K, q.data_ptr(), K, scale.data_ptr(), stream_handle(stream))
    return QuantizedWeight(q, scale, kind)


def gemv_quantized(x: torch.Tensor, qw: QuantizedWeight, out: torch.Tensor | None = None,
                   out_dtype=torch.float32, pdl: bool = False, stream=None, next_weight=None) -> torch.Tensor:
    """y[m, n] = scale[n] * sum_k x[m, k] * q[n, k] with the dequant fused in-kernel.

    ``pdl`` and ``next_weight`` as for ``gemv``."""
    require_cuda("x", x, _BF16, 2)
    q, scale = qw.q, qw.scale
    require_cuda("q", q, None, 2)
    require_cuda("scale", scale, torch.float32, 1)
    M, K = x.shape
    N = q.shape[0]
    if q.shape[1] != K or scale.numel() != N or not scale.is_contiguous():
        raise ValueError("x, q and scale shapes disagree")
    if not 1 <= M <= MAX_M:
        raise ValueError(f"M={M}: the decode GEMV supports 1 <= M <= {MAX_M}")
    if out is None:
        out = torch.empty(M, N, device=x.device, dtype=out_dtype)
    if out.shape != (M, N) or out.dtype not in (_BF16, torch.float32):
        raise ValueError(f"out must be [{M}, {N}] bf16 or fp32")
    y_dtype = _lib.SN_DTYPE_F32 if out.dtype == torch.float32 else _lib.SN_DTYPE_BF16
    flags = _lib.SN_FLAG_PDL if pdl else 0
    if next_weight is None:
        fn = {"int8": "sn_gemv_int8", "e4m3": "sn_gemv_fp8e4m3"}[qw.kind]
        call(fn, q.data_ptr(), row_major("q", q), scale.data_ptr(), x.data_ptr(), row_major("x", x),
             out.data_ptr(), row_major("out", out), M, N, K, y_dtype, flags, stream_handle(stream))
    else:
        kind = _lib.SN_WEIGHT_INT8 if qw.kind == "int8" else _lib.SN_WEIGHT_E4M3
        call("sn_gemv_ex", kind, q.data_ptr(), row_major("q", q), scale.data_ptr(), x.data_ptr(),
             row_major("x", x), out.data_ptr(), row_major("out", out), M, N, K, y_dtype, flags,
             stream_handle(stream), *_next_args(next_weight, x.device))
    return out


def gemv_int8(x, qw: QuantizedWeight, **kw):
    if qw.kind != "int8":
        raise ValueError("gemv_int8 needs an int8 QuantizedWeight")
    return gemv_quantized(x, qw, **kw)


def gemv_fp8e4m3(x, qw: QuantizedWeight, **kw):
    if qw.kind != "e4m3":
        raise ValueError("gemv_fp8e4m3 needs an e4m3 QuantizedWeight")
    return gemv_quantized(x, qw, **kw)
