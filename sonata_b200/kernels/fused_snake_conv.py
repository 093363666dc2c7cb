"""Fused Snake + Conv1d (the DAC decoder's residual-unit front half) on B200.

Drop-in for the reference's kernels/fused_snake_conv.py:

* ``conv1d_output_length`` (fused_snake_conv.py:13-26);
* ``fused_snake_conv1d(x, alpha, weight, bias, stride=1, padding=0,
  dilation=1, eps=1e-9)`` (:134-199): same validation (ValueError for
  groups != 1, alpha or bias of the wrong size), returns a new output of x's
  dtype (fp32), computed by the sm_100a kernel ``sn_snake_conv1d``;
* ``explicit_snake_conv1d`` / ``reference_snake_conv1d`` (:201-286): the
  reference's two torch formulations, kept for users' own checks -- the fused
  path never calls them;
* ``test_snake_conv1d`` / ``test_fused_kernel`` (:288-355): its self-tests.

``bench_dac_stream()`` times BASELINE config 5: the 12 Snake+Conv1d units
(4 decoder stages x dilations 1, 3, 9, kernel 7, 'same' padding) of 10 s of
44.1 kHz audio, and reports microseconds per second of audio.
"""
from __future__ import annotations

import math
import time

import torch
import torch.nn.functional as F

from .. import _lib
from ._common import require_cuda, stream_handle

_WORKSPACE: dict = {}


def conv1d_output_length(input_length: int, kernel_size: int, stride: int, padding: int, dilation: int) -> int:
    """Calculate PyTorch Conv1d's output length."""
    return (input_length + 2 * padding - dilation * (kernel_size - 1) - 1) // stride + 1


def _workspace(device, nbytes: int) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device())
    buf = _WORKSPACE.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1), device=device, dtype=torch.uint8)
        _WORKSPACE[key] = buf
    return buf


_ACTS = {"snake": _lib.SN_ACT_SNAKE, "none": _lib.SN_ACT_NONE}
_POSTS = {None: _lib.SN_POST_NONE, "tanh": _lib.SN_POST_TANH}


def fused_snake_conv1d(x: torch.Tensor, alpha: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
                       stride: int = 1, padding: int = 0, dilation: int = 1, eps: float = 1e-9,
                       out: torch.Tensor | None = None, stream=None, *, residual: torch.Tensor | None = None,
                       activation: str = "snake", post: str | None = None,
                       packed: torch.Tensor | None = None) -> torch.Tensor:
    """Validate inputs and run the fused Snake -> Conv1d kernel.

    Keyword-only additions for the rest of the DAC decoder: ``residual``
    (fp32, the output's shape) is added after the bias, ``activation="none"``
    skips the Snake (alpha may then be None), ``post="tanh"`` applies tanh
    last, ``packed`` (from ``pack_conv1d_weight(weight)``) skips the per-call
    weight pack."""
    batch_size, input_channels, input_length = x.shape
    output_channels, weight_channels, kernel_size = weight.shape
    if activation not in _ACTS:
        raise ValueError(f"activation must be one of {sorted(_ACTS)}, got {activation!r}")
    if post not in _POSTS:
        raise ValueError(f"post must be None or 'tanh', got {post!r}")
    snake = activation == "snake"
    if weight_channels != input_channels:
        raise ValueError("Only groups=1 is currently supported.")
    if snake and alpha.numel() != input_channels:
        raise ValueError("alpha must contain one value per input channel.")
    if bias is not None and bias.numel() != output_channels:
        raise ValueError("bias must contain one value per output channel.")
    require_cuda("x", x, torch.float32, 3)
    if snake:
        require_cuda("alpha", alpha, torch.float32)
    require_cuda("weight", weight, torch.float32, 3)
    if bias is not None:
        require_cuda("bias", bias, torch.float32)
    output_length = conv1d_output_length(input_length, kernel_size, stride, padding, dilation)
    if output_length < 1:
        raise ValueError("the convolution has no output positions")
    x = x.contiguous()
    weight = weight.contiguous()
    alpha_c = alpha.contiguous().view(-1) if snake else None
    bias_c = bias.contiguous().view(-1) if bias is not None else None
    if out is None:
        out = torch.empty((batch_size, output_channels, output_length), device=x.device, dtype=x.dtype)
    elif tuple(out.shape) != (batch_size, output_channels, output_length) or not out.is_contiguous():
        raise ValueError("out has the wrong shape or is not contiguous")
    res_c = None
    if residual is not None:
        require_cuda("residual", residual, torch.float32, 3)
        if tuple(residual.shape) != tuple(out.shape):
            raise ValueError(f"residual must have the output's shape {tuple(out.shape)}")
        res_c = residual.contiguous()
        if res_c.data_ptr() == out.data_ptr():
            raise ValueError("residual must not alias out")
    lib = _lib.lib()
    ws_bytes = lib.sn_snake_conv1d_workspace_size(input_channels, output_channels, kernel_size)
    flags = 0
    if packed is not None:
        _check_packed(packed, ws_bytes, x.device)
        ws, flags = packed, _lib.SN_FLAG_PREPACKED
    else:
        ws = _workspace(x.device, ws_bytes)
    if res_c is None and snake and post is None and not flags:
        _lib.check("sn_snake_conv1d", lib.sn_snake_conv1d(
            x.data_ptr(), alpha_c.data_ptr(), weight.data_ptr(), bias_c.data_ptr() if bias_c is not None else None,
            out.data_ptr(), batch_size, input_channels, output_channels, input_length, kernel_size, stride, padding,
            dilation, float(eps), ws.data_ptr(), ws.numel(), stream_handle(stream)))
    else:
        _lib.check("sn_snake_conv1d_ex", lib.sn_snake_conv1d_ex(
            x.data_ptr(), alpha_c.data_ptr() if alpha_c is not None else None, weight.data_ptr(),
            bias_c.data_ptr() if bias_c is not None else None, res_c.data_ptr() if res_c is not None else None,
            out.data_ptr(), batch_size, input_channels, output_channels, input_length, kernel_size, stride, padding,
            dilation, float(eps), _ACTS[activation], _POSTS[post], flags, ws.data_ptr(), ws.numel(),
            stream_handle(stream)))
    return out


def _check_packed(packed: torch.Tensor, nbytes: int, device) -> None:
    if not isinstance(packed, torch.Tensor) or packed.dtype != torch.uint8 or packed.device != device:
        raise ValueError("packed must be a uint8 tensor from pack_conv1d_weight / pack_conv_transpose1d_weight "
                         "on the input's device")
    if packed.numel() < nbytes or not packed.is_contiguous():
        raise ValueError("packed is too small for this weight shape")


def pack_conv1d_weight(weight: torch.Tensor, stream=None) -> torch.Tensor:
    """Pack a Conv1d weight [Cout, Cin, K] once for ``fused_snake_conv1d(...,
    packed=)`` (sn_snake_conv1d_pack): the bf16 hi/lo tensor-core planes."""
    require_cuda("weight", weight, torch.float32, 3)
    weight = weight.contiguous()
    cout, cin, k = weight.shape
    lib = _lib.lib()
    buf = torch.empty(lib.sn_snake_conv1d_workspace_size(cin, cout, k), device=weight.device, dtype=torch.uint8)
    _lib.check("sn_snake_conv1d_pack", lib.sn_snake_conv1d_pack(weight.data_ptr(), cin, cout, k, buf.data_ptr(),
                                                                buf.numel(), stream_handle(stream)))
    return buf


def pack_conv_transpose1d_weight(weight: torch.Tensor, stride: int, stream=None) -> torch.Tensor | None:
    """Pack a ConvTranspose1d weight [Cin, Cout, K] once into the polyphase
    planes for ``fused_snake_conv_transpose1d(..., packed=)``; None when K is
    not a multiple of stride (that shape has no polyphase GEMM to pack for)."""
    require_cuda("weight", weight, torch.float32, 3)
    weight = weight.contiguous()
    cin, cout, k = weight.shape
    if k % stride:
        return None
    lib = _lib.lib()
    buf = torch.empty(lib.sn_snake_conv1d_workspace_size(cin, cout, k), device=weight.device, dtype=torch.uint8)
    _lib.check("sn_snake_conv_transpose1d_pack", lib.sn_snake_conv_transpose1d_pack(
        weight.data_ptr(), cin, cout, k, stride, buf.data_ptr(), buf.numel(), stream_handle(stream)))
    return buf


def conv_transpose1d_output_length(input_length: int, kernel_size: int, stride: int, padding: int) -> int:
    """PyTorch ConvTranspose1d's output length (dilation 1, output_padding 0)."""
    return (input_length - 1) * stride - 2 * padding + kernel_size


def fused_snake_conv_transpose1d(x: torch.Tensor, alpha: torch.Tensor, weight: torch.Tensor,
                                 bias: torch.Tensor | None = None, stride: int = 1, padding: int = 0,
                                 eps: float = 1e-9, out: torch.Tensor | None = None, stream=None, *,
                                 packed: torch.Tensor | None = None) -> torch.Tensor:
    """Snake -> ConvTranspose1d (the DacDecoderBlock's snake1 -> conv_t1):
    ``conv_transpose1d(snake(x), weight, bias, stride, padding)`` with weight
    in torch's [Cin, Cout, K] layout; runs ``sn_snake_conv_transpose1d``.
    ``packed``: from ``pack_conv_transpose1d_weight(weight, stride)``."""
    batch_size, input_channels, input_length = x.shape
    weight_channels, output_channels, kernel_size = weight.shape
    if weight_channels != input_channels:
        raise ValueError("Only groups=1 is currently supported.")
    if alpha.numel() != input_channels:
        raise ValueError("alpha must contain one value per input channel.")
    if bias is not None and bias.numel() != output_channels:
        raise ValueError("bias must contain one value per output channel.")
    require_cuda("x", x, torch.float32, 3)
    require_cuda("alpha", alpha, torch.float32)
    require_cuda("weight", weight, torch.float32, 3)
    if bias is not None:
        require_cuda("bias", bias, torch.float32)
    output_length = conv_transpose1d_output_length(input_length, kernel_size, stride, padding)
    if output_length < 1:
        raise ValueError("the transposed convolution has no output positions")
    x = x.contiguous()
    weight = weight.contiguous()
    alpha = alpha.contiguous().view(-1)
    bias_c = bias.contiguous().view(-1) if bias is not None else None
    if out is None:
        out = torch.empty((batch_size, output_channels, output_length), device=x.device, dtype=x.dtype)
    elif tuple(out.shape) != (batch_size, output_channels, output_length) or not out.is_contiguous():
        raise ValueError("out has the wrong shape or is not contiguous")
    lib = _lib.lib()
    ws_bytes = lib.sn_snake_conv1d_workspace_size(input_channels, output_channels, kernel_size)
    flags = 0
    if packed is not None:
        _check_packed(packed, ws_bytes, x.device)
        ws, flags = packed, _lib.SN_FLAG_PREPACKED
    else:
        ws = _workspace(x.device, ws_bytes)
    _lib.check("sn_snake_conv_transpose1d", lib.sn_snake_conv_transpose1d(
        x.data_ptr(), alpha.data_ptr(), weight.data_ptr(), bias_c.data_ptr() if bias_c is not None else None,
        out.data_ptr(), batch_size, input_channels, output_channels, input_length, kernel_size, stride, padding,
        float(eps), flags, ws.data_ptr(), ws.numel(), stream_handle(stream)))
    return out


def snake1d(x: torch.Tensor, alpha: torch.Tensor, eps: float = 1e-9, out: torch.Tensor | None = None,
            stream=None) -> torch.Tensor:
    """Snake on its own, ``x + sin(alpha * x)**2 / (alpha + eps)`` per channel of
    x [B, C, T] (fp32): the Snake of ``reference_snake_conv1d`` and of
    transformers' ``Snake1d``, computed by ``sn_snake1d`` with the same device
    arithmetic the fused kernels' producers use.  ``out`` may be ``x``."""
    require_cuda("x", x, torch.float32, 3)
    require_cuda("alpha", alpha, torch.float32)
    batch_size, channels, length = x.shape
    if alpha.numel() != channels:
        raise ValueError("alpha must contain one value per input channel.")
    x = x.contiguous()
    alpha = alpha.contiguous().view(-1)
    if out is None:
        out = torch.empty_like(x)
    elif tuple(out.shape) != tuple(x.shape) or not out.is_contiguous() or out.dtype != torch.float32:
        raise ValueError("out has the wrong shape, dtype or is not contiguous")
    _lib.check("sn_snake1d", _lib.lib().sn_snake1d(x.data_ptr(), alpha.data_ptr(), out.data_ptr(), batch_size,
                                                   channels, length, float(eps), stream_handle(stream)))
    return out


def explicit_snake_conv1d(x, alpha, weight, bias=None, stride=1, padding=0, dilation=1, eps=1e-9):
    """Unfold + einsum formulation (fused_snake_conv.py:201-262)."""
    _, input_channels, _ = x.shape
    output_channels, weight_channels, kernel_size = weight.shape
    if weight_channels != input_channels:
        raise ValueError("This oracle supports ungrouped Conv1d only.")
    if alpha.numel() != input_channels:
        raise ValueError("alpha must contain one value per input channel.")
    if bias is not None and bias.numel() != output_channels:
        raise ValueError("bias must contain one value per output channel.")
    padded = F.pad(x, (padding, padding))
    receptive_field = dilation * (kernel_size - 1) + 1
    windows = padded.unfold(dimension=2, size=receptive_field, step=stride)[..., ::dilation]
    a = alpha.reshape(1, input_channels, 1, 1)
    activated = windows + torch.sin(a * windows).square() / (a + eps)
    output = torch.einsum("bctk, ock -> bot", activated, weight)
    if bias is not None:
        output = output + bias.reshape(1, -1, 1)
    return output


def reference_snake_conv1d(x, alpha, weight, bias=None, stride=1, padding=0, dilation=1, eps=1e-9):
    """Snake then F.conv1d (fused_snake_conv.py:264-286)."""
    a = alpha.reshape(1, -1, 1)
    activated = x + torch.sin(a * x).square() / (a + eps)
    return F.conv1d(activated, weight, bias, stride=stride, padding=padding, dilation=dilation)


def test_snake_conv1d():
    torch.manual_seed(42)
    x = torch.randn(2, 4, 8)
    alpha = torch.rand(4) * 2 + 0.3
    weight = torch.randn(3, 4, 3)
    bias = torch.randn(3)
    y_e = explicit_snake_conv1d(x, alpha, weight, bias, stride=1, padding=1, dilation=1)
    y_r = reference_snake_conv1d(x, alpha, weight, bias, stride=1, padding=1, dilation=1)
    d = (y_e - y_r).abs().max().item()
    print(f"Max abs difference: {d:.6g}")
    assert d < 1e-5, "explicit and reference formulations diverge"


def test_fused_kernel():
    """Runs the B200 kernel on the reference's self-test case (needs CUDA)."""
    if not torch.cuda.is_available():
        print("SKIP: test_fused_kernel requires CUDA, none available.")
        return
    torch.manual_seed(42)
    dev = "cuda"
    x = torch.randn(2, 4, 8, device=dev)
    alpha = torch.rand(4, device=dev) * 2 + 0.3
    weight = torch.randn(3, 4, 3, device=dev)
    bias = torch.randn(3, device=dev)
    y_k = fused_snake_conv1d(x, alpha, weight, bias, stride=1, padding=1, dilation=1)
    torch.cuda.synchronize()
    y_r = reference_snake_conv1d(x, alpha, weight, bias, stride=1, padding=1, dilation=1)
    d = (y_k - y_r).abs().max().item()
    print(f"Max abs difference: {d:.6g}")
    assert d < 1e-2, "fused kernel diverges from reference"


# ---------------------------------------------------------------------------
# 10 s of audio through the 12 Snake+Conv1d units
# ---------------------------------------------------------------------------
DAC_STAGES = ((768, 6896), (384, 55168), (192, 220672), (96, 441344))  # (channels, samples) at T0 = 862
DAC_DILATIONS = (1, 3, 9)
SAMPLE_RATE = 44100
AUDIO_SECONDS = DAC_STAGES[-1][1] / SAMPLE_RATE  # 10.008 s


def dac_stage_inputs(C, T, streams=1, seed=0, device="cuda"):
    """x ~ N(0,1) fp32, alpha ~ U(0.5,1.5), W ~ N(0, 1/sqrt(7C)), bias ~ N(0,1)."""
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(streams, C, T, device=device, generator=g)
    alpha = torch.rand(C, device=device, generator=g) + 0.5
    W = torch.randn(C, C, 7, device=device, generator=g) / math.sqrt(7 * C)
    b = torch.randn(C, device=device, generator=g)
    return x, alpha, W, b


def stream_flops(streams=1):
    return sum(2 * C * C * 7 * T * len(DAC_DILATIONS) for C, T in DAC_STAGES) * streams


def stream_bytes(streams=1):
    """Algorithmic HBM bytes of the 12 units: fp32 x read and y written per
    stream, fp32 weights read once per unit."""
    return sum((8 * C * T * streams + 4 * 7 * C * C) * len(DAC_DILATIONS) for C, T in DAC_STAGES)


def bench_snake_then_cudnn(warmup=1, reps=2, streams=1):
    """The baseline the reference judged its fused kernel against
    (kernels/bench_snake_conv.py:27-58): Snake as torch elementwise ops, then
    cuDNN fp32 Conv1d (reference_snake_conv1d on the GPU), TF32 off, over the
    same 12 units; microseconds per second of audio."""
    units = []
    for si, (C, T) in enumerate(DAC_STAGES):
        units.append(dac_stage_inputs(C, T, streams=streams, seed=si))
    prev = (torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32)
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        def one_pass():
            for x, alpha, W, b in units:
                for d in DAC_DILATIONS:
                    reference_snake_conv1d(x, alpha, W, b, padding=3 * d, dilation=d)

        for _ in range(warmup):
            one_pass()
        torch.cuda.synchronize()
        a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            one_pass()
        e.record()
        torch.cuda.synchronize()
    finally:
        torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32 = prev
    us = a.elapsed_time(e) * 1e3 / reps
    return {"us_per_audio_second": round(us / (AUDIO_SECONDS * streams), 2), "us_per_pass": round(us, 1),
            "useful_tflops": round(stream_flops(streams) / (us * 1e-6) / 1e12, 1),
            "what": "Snake as torch ops then cuDNN fp32 Conv1d (TF32 off), the reference's own GPU baseline "
                    "(kernels/bench_snake_conv.py), same 12 units"}


def bench_dac_stream(warmup=2, reps=3, streams=1):
    """Microseconds per second of audio for `streams` independent streams.

    Each rep runs the 12 units (4 stages x 3 dilations) on device-resident
    inputs; time is measured with CUDA events around all reps."""
    units = []
    for si, (C, T) in enumerate(DAC_STAGES):
        x, alpha, W, b = dac_stage_inputs(C, T, streams=streams, seed=si)
        y = torch.empty_like(x)
        units.append((x, alpha, W, b, y))

    def one_pass():
        for x, alpha, W, b, y in units:
            for d in DAC_DILATIONS:
                fused_snake_conv1d(x, alpha, W, b, padding=3 * d, dilation=d, out=y)

    for _ in range(warmup):
        one_pass()
    torch.cuda.synchronize()
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        one_pass()
    e.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(e) * 1e3 / reps
    flops = stream_flops(streams)
    return {
        "metric": "DAC snake-conv µs per audio-sec",
        "value": round(us / (AUDIO_SECONDS * streams), 2),
        "unit": "us per audio-second",
        "streams": streams,
        "us_per_pass": round(us, 1),
        "realtime_factor": round(AUDIO_SECONDS * streams / (us * 1e-6), 1),
        "useful_tflops": round(flops / (us * 1e-6) / 1e12, 1),
        "mma_tflops": round(3 * flops / (us * 1e-6) / 1e12, 1),
        "bytes": stream_bytes(streams),
        "gbs": round(stream_bytes(streams) / (us * 1e-6) / 1e9, 1),
        "workload": "BASELINE config 5: stages (768,6896) (384,55168) (192,220672) (96,441344) x dilations 1,3,9, "
                    "k=7 'same', fp32 in/out, bf16x3 split-precision tcgen05",
        "launches_per_pass": 2 * len(DAC_STAGES) * len(DAC_DILATIONS),
    }
