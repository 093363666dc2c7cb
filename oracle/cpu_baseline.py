"""The reference's CPU path for each hot path, timed as the CPU baseline.

TEST / BENCHMARK INFRASTRUCTURE ONLY: ``bench.py`` runs these on the GPU box's
host cores for its ``cpu_baseline`` field and for ``--impl reference``; the
product never calls them.

The reference (Vishal-Padia/Sonata) is Python whose CPU-side oracle for every
path is plain torch:

* decode GEMV: ``torch.nn.functional.linear`` in bf16 (
  kernels/bench_gemv.py:18-19 ``candidate_torch``);
* codebook-head BMM: ``torch.bmm`` in bf16 (the survey's CPU probe);
* Snake + Conv1d: ``reference_snake_conv1d`` (kernels/fused_snake_conv.py:
  264-286): snake then ``F.conv1d`` in fp32.

These are restated here (the reference modules import cutlass at top level
and cannot travel to the GPU box).
"""
from __future__ import annotations

import os
import time

import torch
import torch.nn.functional as F


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def gemv_layer_set(shapes: dict, seed: int = 0, layers: int = 1):
    """bf16 weights N(0, 0.02) and activations N(0, 1) for `layers` layers."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(layers):
        out.append({n: ((torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16),
                        torch.randn(1, K, generator=g).to(torch.bfloat16)) for n, (N, K) in shapes.items()})
    return out


def run_gemv_layers(layer_set) -> None:
    for layer in layer_set:
        for W, x in layer.values():
            F.linear(x, W)


def time_gemv(shapes: dict, threads: int, min_seconds: float = 10.0, layers: int = 2):
    """Time the reference CPU GEMV path; returns (GB/s, seconds, iterations)."""
    torch.set_num_threads(threads)
    ls = gemv_layer_set(shapes, layers=layers)
    per_pass = sum((N * K + K + N) * 2 for (N, K) in shapes.values()) * layers
    run_gemv_layers(ls)  # warm-up
    t0 = time.perf_counter()
    it = 0
    while True:
        run_gemv_layers(ls)
        it += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    return per_pass * it / el / 1e9, el, it


def reference_snake_conv1d(x, alpha, weight, bias=None, stride=1, padding=0, dilation=1, eps=1e-9):
    """kernels/fused_snake_conv.py:264-286, restated."""
    a = alpha.reshape(1, -1, 1)
    activated = x + torch.sin(a * x).square() / (a + eps)
    return F.conv1d(activated, weight, bias, stride=stride, padding=padding, dilation=dilation)


def _time(fn, min_seconds: float):
    fn()  # warm-up
    t0 = time.perf_counter()
    it = 0
    while True:
        fn()
        it += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            return el / it, it


def time_quant_gemv(N: int, K: int, kind: str, threads: int, min_seconds: float = 2.0):
    """BASELINE config 3's CPU reference: dequantise the per-row codes to fp32,
    then matmul in fp32 (the fake-quant probe path, scripts/fake_quant.py:41
    before its dtype cast).  Returns seconds per GEMV."""
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    W = torch.randn(N, K, generator=g) * 0.02
    x = torch.randn(1, K, generator=g).to(torch.bfloat16)
    amax = W.abs().amax(dim=1, keepdim=True).clamp_min(1e-8)
    if kind == "int8":
        scale = amax / 127
        q = torch.round(W / scale).clamp(-127, 127).to(torch.int8)
        fn = lambda: F.linear(x.float(), q.float() * scale)
    else:
        scale = amax / 448
        q = (W / scale).to(torch.float8_e4m3fn)
        fn = lambda: F.linear(x.float(), q.float() * scale)
    return _time(fn, min_seconds)[0]


def time_head_bmm(B: int, threads: int, min_seconds: float = 2.0):
    """BASELINE config 4's CPU reference: torch.bmm in bf16 over the 9 heads.
    Returns seconds per call."""
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    h = torch.randn(9, B, 2048, generator=g).to(torch.bfloat16)
    W = (torch.randn(9, 2048, 1025, generator=g) * 0.02).to(torch.bfloat16)
    return _time(lambda: torch.bmm(h, W), min_seconds)[0]


def time_snake_stream(stages, dilations, threads: int, frames_fraction: float = 1.0):
    """BASELINE config 5's CPU reference: reference_snake_conv1d in fp32 over
    the 12 units of one stream, each stage's time axis cut to
    `frames_fraction` of its length (a bounded sample).  Returns seconds for
    that sample."""
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    total = 0.0
    for C, T in stages:
        t = max(64, int(T * frames_fraction))
        x = torch.randn(1, C, t, generator=g)
        a = torch.rand(C, generator=g) + 0.5
        W = torch.randn(C, C, 7, generator=g) / (7 * C) ** 0.5
        b = torch.randn(C, generator=g)
        for d in dilations:
            t0 = time.perf_counter()
            reference_snake_conv1d(x, a, W, b, padding=3 * d, dilation=d)
            total += time.perf_counter() - t0
    return total
