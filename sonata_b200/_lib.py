"""ctypes binding of libsonata_b200.so (the C ABI declared in include/sonata_b200.h).

The library is built in-tree by ``sonata_b200.build``; there is no CPU or
eager fallback: if the library cannot be loaded, every kernel entry point
raises ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libsonata_b200.so"
HEADER = _PKG.parent / "include" / "sonata_b200.h"

SN_OK = 0
SN_DTYPE_BF16 = 0
SN_DTYPE_F32 = 1
SN_FLAG_PDL = 1
SN_FLAG_PREPACKED = 2
SN_WEIGHT_BF16 = 0
SN_WEIGHT_INT8 = 1
SN_WEIGHT_E4M3 = 2
SN_NORM_RMS_GATED = 1
SN_NORM_ADD_LAYER = 2
SN_ACT_SNAKE = 0
SN_ACT_NONE = 1
SN_ACT_SILU = 2
SN_POST_NONE = 0
SN_POST_TANH = 1

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_U = ctypes.c_uint

# argtypes of every exported symbol; must match include/sonata_b200.h
SIGNATURES: dict[str, tuple[list, object]] = {
    "sn_version": ([], _I),
    "sn_status_string": ([_I], ctypes.c_char_p),
    "sn_gemv_bf16": ([_P, _I64, _P, _I64, _P, _I64, _I, _I, _I, _I, _U, _P], _I),
    "sn_gemv_int8": ([_P, _I64, _P, _P, _I64, _P, _I64, _I, _I, _I, _I, _U, _P], _I),
    "sn_gemv_fp8e4m3": ([_P, _I64, _P, _P, _I64, _P, _I64, _I, _I, _I, _I, _U, _P], _I),
    "sn_gemv_ex": ([_I, _P, _I64, _P, _P, _I64, _P, _I64, _I, _I, _I, _I, _U, _P, _I, _P, _I64, _I, _I], _I),
    "sn_gemv_bf16_norm": ([_I, _P, _I64, _P, _P, _P, _P, _P, ctypes.c_float, _P, _I64, _I, _I, _I, _I, _U, _P, _I, _P,
                           _I64, _I, _I], _I),
    "sn_quantize_rows_int8": ([_P, _I64, _I, _I, _P, _I64, _P, _P], _I),
    "sn_quantize_rows_fp8e4m3": ([_P, _I64, _I, _I, _P, _I64, _P, _P], _I),
    "sn_device_status": ([_I, _P], _I),
    "sn_codebook_head_pack": ([_P, _I, _I, _I, _P, _P], _I),
    "sn_codebook_head_bmm": ([_P, _P, _P, _I, _I, _I, _I, _U, _P], _I),
    "sn_ssd_chunk_bmm": ([_P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I, _I, _I, _I, _I, _I, _P, _P], _I),
    "sn_snake_conv1d_output_length": ([_I64, _I, _I, _I, _I], _I64),
    "sn_snake_conv1d_workspace_size": ([_I, _I, _I], ctypes.c_size_t),
    "sn_snake_conv1d": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, ctypes.c_float, _P, ctypes.c_size_t,
                         _P], _I),
    "sn_snake_conv1d_noalloc": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, ctypes.c_float, _P], _I),
    "sn_snake_conv1d_ex": ([_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, ctypes.c_float, _I, _I, _U,
                            _P, ctypes.c_size_t, _P], _I),
    "sn_snake_conv1d_pack": ([_P, _I, _I, _I, _P, ctypes.c_size_t, _P], _I),
    "sn_causal_conv1d_update": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _P], _I),
    "sn_selective_state_update": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P], _I),
    "sn_rmsnorm_gated": ([_P, _P, _P, _P, _P, _I, _I, _I, ctypes.c_float, _I, _P], _I),
    "sn_layer_norm_fused": ([_P, _P, _I, _P, _P, _P, _P, _I, _I, _I, ctypes.c_float, _I, _P], _I),
    "sn_snake_conv1d_strided": ([_P, _I64, _I64, _P, _P, _P, _P, _I64, _I64, _P, _I64, _I64, _I, _I, _I, _I, _I, _I,
                                 _I, _I, ctypes.c_float, _I, _I, _U, _P, ctypes.c_size_t, _P], _I),
    "sn_snake_conv_transpose1d_strided": ([_P, _I64, _I64, _P, _P, _P, _P, _I64, _I64, _I, _I, _I, _I, _I, _I, _I,
                                           _I, ctypes.c_float, _U, _P, ctypes.c_size_t, _P], _I),
    "sn_stream_shift": ([_P, _I, _P], _I),
    "sn_mamba2_split_conv": ([_P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P], _I),
    "sn_mamba2_conv_ssu": ([_P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P], _I),
    "sn_rotary_kv_append": ([_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P], _I),
    "sn_swiglu": ([_P, _P, _I, _I, _P], _I),
    "sn_snake1d": ([_P, _P, _P, _I, _I, _I64, ctypes.c_float, _P], _I),
    "sn_diag_bounded_wait": ([ctypes.c_uint64, _P], _I),
    "sn_snake_conv_transpose1d_pack": ([_P, _I, _I, _I, _I, _P, ctypes.c_size_t, _P], _I),
    "sn_snake_conv_transpose1d_output_length": ([_I64, _I, _I, _I], _I64),
    "sn_gemv_chain_workspace_size": ([_I], ctypes.c_size_t),
    "sn_gemv_chain_plan": ([_I, _P, _I, _I, _P, ctypes.c_size_t, _P, _P], _I),
    "sn_gemv_chain_launch": ([_P, _P, _U, _P], _I),
    "sn_snake_conv_transpose1d": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, ctypes.c_float, _U, _P,
                                   ctypes.c_size_t, _P], _I),
}



class ShiftDesc(ctypes.Structure):
    """sn_shift_desc of include/sonata_b200.h."""
    _fields_ = [("buf", ctypes.c_void_p), ("batch_stride", ctypes.c_int64), ("row_stride", ctypes.c_int64),
                ("batches", ctypes.c_int), ("rows", ctypes.c_int), ("src", ctypes.c_int), ("len", ctypes.c_int)]


class GemvJob(ctypes.Structure):
    """sn_gemv_job of include/sonata_b200.h."""
    _fields_ = [("W", ctypes.c_void_p), ("x", ctypes.c_void_p), ("y", ctypes.c_void_p), ("scale", ctypes.c_void_p),
                ("ldw", ctypes.c_int64), ("ldx", ctypes.c_int64), ("ldy", ctypes.c_int64), ("N", ctypes.c_int),
                ("K", ctypes.c_int), ("dep", ctypes.c_int), ("y_dtype", ctypes.c_int)]


class GemvChainInfo(ctypes.Structure):
    """sn_gemv_chain_info of include/sonata_b200.h."""
    _fields_ = [("njobs", ctypes.c_int), ("M", ctypes.c_int), ("w_kind", ctypes.c_int), ("x_buffers", ctypes.c_int),
                ("tile_bytes_max", ctypes.c_uint32), ("ring_bytes", ctypes.c_uint32), ("xbuf_bytes", ctypes.c_uint32),
                ("accumulators", ctypes.c_uint32), ("accumulator_cols", ctypes.c_uint32), ("grid", ctypes.c_uint32),
                ("workspace_bytes", ctypes.c_uint64)]


SN_SHIFT_MAX_DESCS = 48
SN_SHIFT_MAX_LEN = 64

_lib = None


class SonataError(RuntimeError):
    def __init__(self, fn: str, status: int):
        msg = lib().sn_status_string(status).decode() if _lib is not None else str(status)
        super().__init__(f"{fn} failed with status {status}: {msg}")
        self.status = status


def header_symbols() -> list[str]:
    """Every sn_* function declared in include/sonata_b200.h."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(sn_[a-z0-9_]+)\s*\(", text)))


def lib() -> ctypes.CDLL:
    """Load (once) and return the CUDA library; raise if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m sonata_b200.build` "
                "(sonata_b200 has no CPU fallback)")
        l = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in SIGNATURES.items():
            f = getattr(l, name)
            f.argtypes = args
            f.restype = res
        _lib = l
    return _lib


def check(fn: str, status: int) -> None:
    if status != SN_OK:
        raise SonataError(fn, status)


def call(fn: str, *args) -> None:
    check(fn, getattr(lib(), fn)(*args))
