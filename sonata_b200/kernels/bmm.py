"""Batched products on B200: the SSD chunk product and the codebook head.

Drop-in for the reference's kernels/bmm.py:

* ``launch_bmm(C, B, BATCH, SEQLEN, NGROUPS, DSTATE, CHUNK, NCHUNKS, CB_out,
  stream)`` (bmm.py:96-117) writes
  ``CB[b, c, g, i, j] = sum_d C[b, c*CHUNK+i, g, d] * B[b, c*CHUNK+j, g, d]``
  into ``CB_out`` (fp32 [BATCH, NCHUNKS, NGROUPS, CHUNK, CHUNK]).  Unlike the
  reference kernel, positions at or beyond ``SEQLEN`` are masked to zero
  (the semantics bmm.py:205-212 asks for), so a ragged last chunk is exact:
  pass the true sequence length as ``SEQLEN`` and ``NCHUNKS = ceil(SEQLEN /
  CHUNK)``; C and B may be padded buffers with more rows.  The strides of C
  and B are taken from the tensors.
* ``test_bmm()`` / ``test_bmm_ragged()``: the reference's two self-tests
  (bmm.py:119-240), same shapes, seeds and tolerance (atol 1e-3, rtol 1e-2);
  the ragged one passes here.

Addition (no reference kernel): the multi-codebook logit
head ``logits[cb, b, n] = sum_k hidden[cb, b, k] * W[cb, k, n]`` --
``CodebookHead(W)`` packs the [ncb, K, N] weight once, ``head(hidden, pdl=...)`` or
``codebook_head_bmm(hidden, W)`` returns fp32 [ncb, B, N].
"""
from __future__ import annotations

import math

import torch

from .. import _lib
from ._common import call, require_cuda, stream_handle

_BF16 = torch.bfloat16


def launch_bmm(C, B, BATCH, SEQLEN, NGROUPS, DSTATE, CHUNK, NCHUNKS, CB_out, stream=None):
    """SSD chunk product C.B^T per (batch, chunk, group), masked past SEQLEN."""
    require_cuda("C", C, _BF16, 4)
    require_cuda("B", B, _BF16, 4)
    require_cuda("CB_out", CB_out, torch.float32, 5)
    for name, t in (("C", C), ("B", B)):
        if t.shape[0] != BATCH or t.shape[2] != NGROUPS or t.shape[3] != DSTATE or t.shape[1] < SEQLEN:
            raise ValueError(f"{name} must be [BATCH, >=SEQLEN, NGROUPS, DSTATE], got {tuple(t.shape)}")
        if t.stride(3) != 1:
            raise ValueError(f"{name} must be contiguous along DSTATE")
    if tuple(CB_out.shape) != (BATCH, NCHUNKS, NGROUPS, CHUNK, CHUNK) or not CB_out.is_contiguous():
        raise ValueError("CB_out must be a contiguous fp32 [BATCH, NCHUNKS, NGROUPS, CHUNK, CHUNK] tensor")
    if NCHUNKS * CHUNK < SEQLEN:
        raise ValueError("NCHUNKS * CHUNK must cover SEQLEN")
    call("sn_ssd_chunk_bmm", C.data_ptr(), B.data_ptr(), C.stride(0), C.stride(1), C.stride(2), B.stride(0),
         B.stride(1), B.stride(2), BATCH, SEQLEN, NGROUPS, DSTATE, CHUNK, NCHUNKS, CB_out.data_ptr(),
         stream_handle(stream))
    return CB_out


def ssd_chunk_bmm(C, B, chunk, seqlen=None, out=None):
    """Functional form: CB [BATCH, ceil(seqlen/chunk), NGROUPS, chunk, chunk]."""
    BATCH, L, NG, DS = C.shape
    seqlen = L if seqlen is None else seqlen
    nch = math.ceil(seqlen / chunk)
    if out is None:
        out = torch.empty(BATCH, nch, NG, chunk, chunk, device=C.device, dtype=torch.float32)
    return launch_bmm(C, B, BATCH, seqlen, NG, DS, chunk, nch, out)


# ---------------------------------------------------------------------------
# multi-codebook logit head
# ---------------------------------------------------------------------------
class CodebookHead:
    """The 9 DAC-codebook logit heads of one decode step, packed for B200.

    W: bf16 [ncb, K, N] (``hidden @ W[cb]`` layout).  It is transposed once on
    the device into [ncb, N, K] so every output logit is a contiguous K-row.
    """

    def __init__(self, W: torch.Tensor, stream=None):
        require_cuda("W", W, _BF16, 3)
        W = W.contiguous()
        self.ncb, self.K, self.N = W.shape
        self.Wt = torch.empty(self.ncb, self.N, self.K, device=W.device, dtype=_BF16)
        call("sn_codebook_head_pack", W.data_ptr(), self.ncb, self.K, self.N, self.Wt.data_ptr(),
             stream_handle(stream))

    def __call__(self, hidden: torch.Tensor, out: torch.Tensor | None = None, pdl: bool = False, stream=None):
        require_cuda("hidden", hidden, _BF16, 3)
        if hidden.shape[0] != self.ncb or hidden.shape[2] != self.K:
            raise ValueError(f"hidden must be [{self.ncb}, B, {self.K}], got {tuple(hidden.shape)}")
        hidden = hidden.contiguous()
        Bn = hidden.shape[1]
        if out is None:
            out = torch.empty(self.ncb, Bn, self.N, device=hidden.device, dtype=torch.float32)
        if tuple(out.shape) != (self.ncb, Bn, self.N) or out.dtype != torch.float32 or not out.is_contiguous():
            raise ValueError("out must be a contiguous fp32 [ncb, B, N] tensor")
        call("sn_codebook_head_bmm", hidden.data_ptr(), self.Wt.data_ptr(), out.data_ptr(), self.ncb, Bn, self.K,
             self.N, _lib.SN_FLAG_PDL if pdl else 0, stream_handle(stream))
        return out


def codebook_head_bmm(hidden: torch.Tensor, W, out=None):
    """logits[cb, b, n] = sum_k hidden[cb, b, k] * W[cb, k, n] (fp32).

    `W` is a ``CodebookHead`` (packed once, the fast path) or a raw bf16
    [ncb, K, N] tensor (packed on every call).
    """
    head = W if isinstance(W, CodebookHead) else CodebookHead(W)
    return head(hidden, out=out)


# ---------------------------------------------------------------------------
# the reference's self-tests (kernels/bmm.py:119-240), run on the B200 kernel
# ---------------------------------------------------------------------------
def test_bmm():
    BATCH, SEQLEN, NGROUPS, DSTATE, CHUNK = 1, 512, 2, 128, 256
    NCHUNKS = SEQLEN // CHUNK
    g = torch.Generator(device="cuda").manual_seed(0)
    C = torch.randn(BATCH, SEQLEN, NGROUPS, DSTATE, device="cuda", dtype=_BF16, generator=g)
    B = torch.randn(BATCH, SEQLEN, NGROUPS, DSTATE, device="cuda", dtype=_BF16, generator=g)
    CB_out = torch.empty(BATCH, NCHUNKS, NGROUPS, CHUNK, CHUNK, dtype=torch.float32, device="cuda")
    Cc = C.reshape(BATCH, NCHUNKS, CHUNK, NGROUPS, DSTATE)
    Bc = B.reshape(BATCH, NCHUNKS, CHUNK, NGROUPS, DSTATE)
    CB_ref = torch.einsum("bcigd,bcjgd->bcgij", Cc.float(), Bc.float())
    launch_bmm(C, B, BATCH, SEQLEN, NGROUPS, DSTATE, CHUNK, NCHUNKS, CB_out)
    torch.cuda.synchronize()
    max_abs = (CB_out - CB_ref).abs().max().item()
    assert torch.allclose(CB_out, CB_ref, atol=1e-3, rtol=1e-2), f"kernel mismatch: max_abs={max_abs}"
    print(f"[kernel] max_abs={max_abs:.6f}  (tol: atol=1e-3 rtol=1e-2)")


def test_bmm_ragged():
    BATCH, NGROUPS, DSTATE, CHUNK = 1, 2, 128, 256
    SEQLEN = 300
    NCHUNKS = math.ceil(SEQLEN / CHUNK)
    PADDED = NCHUNKS * CHUNK
    g = torch.Generator(device="cuda").manual_seed(0)
    C = torch.randn(BATCH, PADDED, NGROUPS, DSTATE, device="cuda", dtype=_BF16, generator=g)
    B = torch.randn(BATCH, PADDED, NGROUPS, DSTATE, device="cuda", dtype=_BF16, generator=g)
    C[:, SEQLEN:] = 7.0
    B[:, SEQLEN:] = 7.0
    CB_out = torch.empty(BATCH, NCHUNKS, NGROUPS, CHUNK, CHUNK, dtype=torch.float32, device="cuda")
    Cm, Bm = C.clone(), B.clone()
    Cm[:, SEQLEN:] = 0
    Bm[:, SEQLEN:] = 0
    CB_ref = torch.einsum("bcigd,bcjgd->bcgij", Cm.reshape(BATCH, NCHUNKS, CHUNK, NGROUPS, DSTATE).float(),
                          Bm.reshape(BATCH, NCHUNKS, CHUNK, NGROUPS, DSTATE).float())
    # the true length goes in SEQLEN; the buffers stay padded and poisoned
    launch_bmm(C, B, BATCH, SEQLEN, NGROUPS, DSTATE, CHUNK, NCHUNKS, CB_out)
    torch.cuda.synchronize()
    max_abs = (CB_out - CB_ref).abs().max().item()
    assert torch.allclose(CB_out, CB_ref, atol=1e-3, rtol=1e-2), f"ragged mismatch: max_abs={max_abs}"
    print(f"[ragged] max_abs={max_abs:.6f}  PASS")


if __name__ == "__main__":
    test_bmm()
    test_bmm_ragged()
