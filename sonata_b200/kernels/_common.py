"""Tensor / stream plumbing shared by the kernel wrappers."""
from __future__ import annotations

import torch

from .. import _lib


def stream_handle(stream=None) -> int:
    """Raw cudaStream_t for `stream` (None -> torch's current stream)."""
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    if isinstance(stream, int):
        return stream
    h = getattr(stream, "cuda_stream", None)
    if h is not None:
        return int(h)
    raise TypeError(f"cannot interpret {type(stream).__name__} as a CUDA stream")


def require_cuda(name: str, t: torch.Tensor, dtype=None, dim=None) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (sonata_b200 has no CPU path)")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if dim is not None and t.dim() != dim:
        raise ValueError(f"{name} must be {dim}-D, got shape {tuple(t.shape)}")


def row_major(name: str, t: torch.Tensor) -> int:
    """Row stride of a 2-D tensor whose last dim is contiguous."""
    if t.stride(-1) != 1:
        raise ValueError(f"{name} must have a contiguous last dimension")
    return t.stride(0) if t.size(0) > 1 else max(t.stride(0), t.size(1))


def call(fn: str, *args) -> None:
    _lib.call(fn, *args)
