"""The C-ABI library: it loads without a GPU, exports every declared symbol, and
its host-side argument checks reject bad calls before touching the device."""
import ctypes

import pytest

from sonata_b200 import _lib


@pytest.fixture(scope="module")
def L():
    from sonata_b200 import build
    build.build()
    return _lib.lib()


def test_every_header_symbol_is_exported(L):
    declared = _lib.header_symbols()
    assert declared, "no sn_* declarations found in include/sonata_b200.h"
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, f"declared but not exported: {missing}"
    # and every declared symbol has a ctypes signature in the binding
    assert set(declared) <= set(_lib.SIGNATURES), set(declared) - set(_lib.SIGNATURES)


def test_version_and_status_strings(L):
    assert L.sn_version() >= 100
    for code in (0, -1, -2, -3, -4, -5, -6):
        assert L.sn_status_string(code)
    assert b"unknown" in L.sn_status_string(12345)


def test_gemv_rejects_bad_arguments_on_host(L):
    # null pointers
    assert L.sn_gemv_bf16(None, 8, None, 8, None, 8, 1, 8, 8, 0, 0, None) == _lib.SN_OK - 1
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    # M out of range
    assert L.sn_gemv_bf16(p, 8, p, 8, p, 8, 5, 8, 8, 0, 0, None) == -1
    assert L.sn_gemv_bf16(p, 8, p, 8, p, 8, 0, 8, 8, 0, 0, None) == -1
    # stride smaller than K
    assert L.sn_gemv_bf16(p, 4, p, 8, p, 8, 1, 8, 8, 0, 0, None) == -1
    # bad output dtype
    assert L.sn_gemv_bf16(p, 8, p, 8, p, 8, 1, 8, 8, 7, 0, None) == -1
    # quantised GEMV without a scale
    assert L.sn_gemv_int8(p, 8, None, p, 8, p, 8, 1, 8, 8, 0, 0, None) == -1
    # sn_gemv_ex: weight kind, and the next-weight hint's kind / shape / stride
    assert L.sn_gemv_ex(3, p, 8, None, p, 8, p, 8, 1, 8, 8, 0, 0, None, 0, None, 0, 0, 0) == -1
    assert L.sn_gemv_ex(1, p, 8, None, p, 8, p, 8, 1, 8, 8, 0, 0, None, 0, None, 0, 0, 0) == -1
    assert L.sn_gemv_ex(0, p, 8, None, p, 8, p, 8, 1, 8, 8, 0, 0, None, 5, p, 8, 8, 8) == -1
    assert L.sn_gemv_ex(0, p, 8, None, p, 8, p, 8, 1, 8, 8, 0, 0, None, 0, p, 4, 8, 8) == -1
    assert L.sn_gemv_ex(0, p, 8, None, p, 8, p, 8, 1, 8, 8, 0, 0, None, 0, p, 8, 0, 8) == -1
    # Snake conv variants: unknown flags / activation / post-op, null pack buffers
    assert L.sn_snake_conv1d_ex(p, p, p, None, None, p, 1, 16, 16, 8, 1, 1, 0, 1, 1e-9, 0, 0, 4, p, 1 << 20,
                                None) == -1
    assert L.sn_snake_conv1d_ex(p, p, p, None, None, p, 1, 16, 16, 8, 1, 1, 0, 1, 1e-9, 7, 0, 0, p, 1 << 20,
                                None) == -1
    assert L.sn_snake_conv1d_ex(p, p, p, None, None, p, 1, 16, 16, 8, 1, 1, 0, 1, 1e-9, 0, 9, 0, p, 1 << 20,
                                None) == -1
    assert L.sn_snake_conv_transpose1d(p, p, p, None, p, 1, 16, 16, 8, 4, 2, 1, 1e-9, 8, p, 1 << 20, None) == -1
    assert L.sn_snake_conv1d_pack(None, 16, 16, 7, p, 1 << 20, None) == -1
    assert L.sn_snake_conv1d_pack(p, 16, 16, 7, p, 16, None) == -1
    assert L.sn_snake_conv_transpose1d_pack(p, 16, 16, 5, 2, p, 1 << 20, None) == -3
    assert L.sn_snake_conv_transpose1d_output_length(10, 16, 8, 4) == 80
    # channel / stream counts whose round-up to the GEMM tile would overflow int
    imax = 2**31 - 1
    assert L.sn_snake_conv1d_noalloc(p, p, p, None, p, 1, 16, imax, 8, 1, 1, 0, 1, 1e-9, None) == -1
    assert L.sn_codebook_head_bmm(p, p, p, 9, imax, 2048, 1025, 0, None) == -1
    # Mamba2 decode-step ops
    assert L.sn_causal_conv1d_update(None, p, p, None, p, 1, 8, 4, 2, None) == -1
    assert L.sn_causal_conv1d_update(p, p, p, None, p, 1, 8, 9, 2, None) == -1   # W > 8
    assert L.sn_causal_conv1d_update(p, p, p, None, p, 1, 8, 4, 0, None) == -1   # snake is not a conv1d act
    assert L.sn_selective_state_update(p, p, p, p, p, p, None, None, None, p, 1, 6, 4, 8, 4, 1, None) == -1
    assert L.sn_selective_state_update(p, p, p, p, p, p, None, None, None, p, 1, 4, 4, 512, 1, 1, None) == -1
    assert L.sn_rmsnorm_gated(p, p, None, None, p, 2, 100, 30, 1e-5, 0, None) == -1
    assert L.sn_rmsnorm_gated(p, p, None, None, p, 2, 16384, 16384, 1e-5, 0, None) == -3
    assert L.sn_layer_norm_fused(None, None, 0, p, None, p, None, 0, 2, 64, 1e-5, 0, None) == -1
    assert L.sn_layer_norm_fused(p, None, 0, p, None, p, None, 0, 2, 9000, 1e-5, 0, None) == -3
    # fused Mamba2 conv + SSU: the counters are required; d_state 64 is the two-launch path's
    assert L.sn_mamba2_conv_ssu(p, 8512, p, p, None, p, p, None, None, p, p, None, 1, 4096, 1, 128, 64, 64, 4,
                                None) == -1
    assert L.sn_mamba2_conv_ssu(p, 8512, p, p, None, p, p, None, None, p, p, p, 1, 4096, 1, 64, 64, 64, 4,
                                None) == -3
    assert L.sn_quantize_rows_int8(None, 8, 8, 8, p, 8, p, None) == -1
    assert L.sn_quantize_rows_fp8e4m3(p, 4, 8, 8, p, 8, p, None) == -1


def test_product_raises_without_library(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "missing.so")
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.lib()


def _job(W, x, y, N=64, K=256, dep=-1, ldw=None, ldx=None, ldy=None, y_dtype=0, scale=None):
    return _lib.GemvJob(W, x, y, scale, ldw or K, ldx or K, ldy or N, N, K, dep, y_dtype)


def test_gemv_chain_plan_rejects_bad_jobs_on_host(L):
    """sn_gemv_chain_plan validates every job (shapes, alignment, dependency
    order, buffer overlaps) before it touches the device: fake, never
    dereferenced addresses are enough."""
    assert L.sn_gemv_chain_workspace_size(0) == 0
    assert L.sn_gemv_chain_workspace_size(4097) == 0
    n = L.sn_gemv_chain_workspace_size(3)
    assert n >= 3 * 64 + 4 * 128
    ws = 1 << 40
    info = _lib.GemvChainInfo()
    W0, W1, X, Y0, Y1 = 1 << 30, 2 << 30, 3 << 30, 4 << 30, 5 << 30

    def plan(jobs, M=1, wsb=n, kind=0):
        arr = (_lib.GemvJob * len(jobs))(*jobs)
        return L.sn_gemv_chain_plan(kind, ctypes.addressof(arr), len(jobs), M, ctypes.c_void_p(ws), wsb,
                                    ctypes.byref(info), None)

    good = [_job(W0, X, Y0), _job(W1, Y0, Y1, dep=0)]
    assert plan(good, M=3) == -1                                    # M outside 1..2
    assert plan(good, kind=3) == -1                                 # weight kind
    assert plan(good, kind=1) == -1                                 # 8-bit codes without row scales
    assert plan(good, wsb=L.sn_gemv_chain_workspace_size(2) - 1) == -1  # workspace too small
    assert plan([_job(W0, X, Y0), _job(W1, X, Y1, dep=1)]) == -1    # dep must name an earlier job
    assert plan([_job(W0, X, Y0, y_dtype=5)]) == -1                 # output dtype
    assert plan([_job(W0, X, Y0, ldw=128)]) == -1                   # row stride below K
    assert plan([_job(W0 + 8, X, Y0)]) == -2                        # W not 16-byte aligned
    assert plan([_job(W0, X, Y0, K=104)]) == -3                     # K outside the tensor-core rules
    assert plan([_job(W0, X, Y0), _job(W1, Y0, Y1)]) == -1          # x written by a job it does not wait for
    assert plan([_job(W0, X, Y0), _job(W1, X, Y0, dep=0)]) == -1    # two jobs writing one buffer
    assert plan([_job(W0, X, W0 + 256)]) == -1                      # an output over a weight
    assert plan([_job(W0, X, X)]) == -1                             # x and y of one job overlap
    # a transitive dependency is enough: job 2 reads job 0's output through 1
    chain3 = [_job(W0, X, Y0), _job(W1, X, Y1, dep=0), _job(W1 + (1 << 20), Y0, 6 << 30, dep=1)]
    import torch
    if not torch.cuda.is_available():  # valid jobs reach the device copy, which fails without a GPU
        assert plan(chain3, wsb=L.sn_gemv_chain_workspace_size(3)) == -4
    launch_info = _lib.GemvChainInfo(0, 1, 0, 2, 4096, 8192, 512, 8, 16, 0, 0)
    assert L.sn_gemv_chain_launch(ctypes.byref(launch_info), ctypes.c_void_p(ws), 0, None) == -1
