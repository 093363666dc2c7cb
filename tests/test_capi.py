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
    assert L.sn_quantize_rows_int8(None, 8, 8, 8, p, 8, p, None) == -1
    assert L.sn_quantize_rows_fp8e4m3(p, 4, 8, 8, p, 8, p, None) == -1


def test_product_raises_without_library(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "missing.so")
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.lib()
