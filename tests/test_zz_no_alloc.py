"""The allocation-free Snake + Conv1d entry point, called through the C ABI.

sn_snake_conv1d_noalloc exists for callers that cannot allocate device
memory -- a real-time audio thread that must never block in cudaMalloc, or a
host runtime that loads the library over the C ABI without a CUDA allocator.
It keeps its packed-weight scratch in a static device array instead of a
caller workspace.  These tests check that it agrees with the regular entry
point (the workspace-taking sn_snake_conv1d behind fused_snake_conv1d) within
the same tolerance the other Snake+Conv1d tests use, on two calls in a row
with different weights -- the shared array must carry the second call's
weights, not the first's -- that a call leaves the device's free memory
unchanged, that shapes which need no scratch (they run the per-output
kernel) are served whatever their size, and that oversized problems are
refused.

This file is collected last on purpose (tests/test_zz_*): a failure here does
not hide any other test in a run that stops at the first failure.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

COS_MIN = 0.9999
MAX_ABS = 2e-3


def _case(C, T, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(1, C, T, device="cuda", generator=g)
    alpha = torch.rand(C, device="cuda", generator=g) + 0.5
    W = torch.randn(C, C, 7, device="cuda", generator=g) / math.sqrt(7 * C)
    b = torch.randn(C, device="cuda", generator=g)
    return x, alpha, W, b


def _noalloc(lib, x, alpha, W, b, y, d, stride=1):
    B, Cin, T = x.shape
    Cout, _, K = W.shape
    return lib.sn_snake_conv1d_noalloc(x.data_ptr(), alpha.data_ptr(), W.data_ptr(), b.data_ptr(), y.data_ptr(), B,
                                       Cin, Cout, T, K, stride, 3 * d, d, ctypes.c_float(1e-9),
                                       torch.cuda.current_stream().cuda_stream)


def _close(y, ref):
    err = (y - ref).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(y.flatten().double(), ref.flatten().double(), dim=0).item()
    return err <= MAX_ABS and cos >= COS_MIN, (err, cos)


def test_noalloc_matches_regular_entry_point_twice(cuda_lib):
    from sonata_b200.kernels import fused_snake_conv as S
    for call, (C, T, d) in enumerate([(768, 1500, 3), (384, 2200, 9)]):
        x, alpha, W, b = _case(C, T, seed=100 + call)
        y = torch.full_like(x, float("nan"))
        assert _noalloc(cuda_lib, x, alpha, W, b, y, d) == 0
        ref = S.fused_snake_conv1d(x, alpha, W, b, padding=3 * d, dilation=d)
        torch.cuda.synchronize()
        assert torch.isfinite(y).all()
        ok, info = _close(y, ref)
        assert ok, (call, info)
    assert cuda_lib.sn_device_status(1, None) == 0


def test_noalloc_leaves_device_memory_unchanged(cuda_lib):
    # every buffer exists before the measurement; a warm-up call first (the
    # first call into the library on a device may load its device code)
    x, alpha, W, b = _case(768, 3000, seed=7)
    y = torch.empty_like(x)
    assert _noalloc(cuda_lib, x, alpha, W, b, y, 1) == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for d in (3, 9):
        assert _noalloc(cuda_lib, x, alpha, W, b, y, d) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)


def test_noalloc_serves_shapes_without_scratch(cuda_lib):
    # stride 2 runs the per-output kernel, which reads W itself: 1024 x 1024 x 7
    # is beyond the static array but needs none of it
    from sonata_b200.kernels import fused_snake_conv as S
    x, alpha, W, b = _case(1024, 96, seed=11)
    Tout = S.conv1d_output_length(96, 7, stride=2, padding=3, dilation=1)
    y = torch.full((1, 1024, Tout), float("nan"), device="cuda")
    assert _noalloc(cuda_lib, x, alpha, W, b, y, 1, stride=2) == 0
    ref = S.fused_snake_conv1d(x, alpha, W, b, stride=2, padding=3, dilation=1)
    torch.cuda.synchronize()
    ok, info = _close(y, ref)
    assert ok, info


def test_noalloc_refuses_problems_beyond_its_scratch(cuda_lib):
    # 1024 x 1024 x 7 packed weights need 28 MiB > the 16 MiB static array;
    # refused on the host before any device work
    p = ctypes.c_void_p(16)
    rc = cuda_lib.sn_snake_conv1d_noalloc(p, p, p, p, p, 1, 1024, 1024, 128, 7, 1, 3, 1, ctypes.c_float(1e-9), None)
    assert rc == -7
    assert b"scratch" in cuda_lib.sn_status_string(rc)
