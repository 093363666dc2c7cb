"""GPU parity of the SSD chunk product and the multi-codebook head.

Tolerance (north star): max|err| <= 1e-2 * ||y||_inf for the bf16 BMMs; the
reference's own self-tests use allclose(atol=1e-3, rtol=1e-2).
"""
import math

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def bits(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.fixture(scope="module")
def Bm(cuda_lib):
    from sonata_b200.kernels import bmm
    return bmm


def test_reference_selftests(Bm):
    Bm.test_bmm()
    Bm.test_bmm_ragged()  # RED in the reference (no masking), GREEN here


def test_ssd_against_golden(Bm, golden):
    b = golden("bmm")
    BATCH, SEQLEN, NG, DS, CH, SEQ_R = b["dims"].tolist()
    C = torch.from_numpy(b["C"].view(np.int16)).view(torch.bfloat16).cuda()
    B = torch.from_numpy(b["B"].view(np.int16)).view(torch.bfloat16).cuda()
    # CHUNK=32 / DSTATE=32 is outside the tensor-core shapes: the masked fallback runs
    out = Bm.ssd_chunk_bmm(C, B, CH)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), b["CB"], rtol=1e-5, atol=1e-4)
    Cr = torch.from_numpy(b["C_ragged"].view(np.int16)).view(torch.bfloat16).cuda()
    Br = torch.from_numpy(b["B_ragged"].view(np.int16)).view(torch.bfloat16).cuda()
    outr = Bm.ssd_chunk_bmm(Cr, Br, CH, seqlen=SEQ_R)
    torch.cuda.synchronize()
    np.testing.assert_allclose(outr.cpu().numpy(), b["CB_ragged"], rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("batch,seqlen,ng,ds,ch", [
    (1, 512, 2, 128, 256),      # the reference's test shape
    (2, 300, 1, 128, 256),      # ragged, batch stride != seqlen stride
    (1, 4096, 1, 128, 256),     # Zonos prefill-sized
    (3, 200, 2, 64, 128),       # CHUNK 128, DSTATE 64
    (1, 257, 4, 256, 128),      # DSTATE 256, one row into the last chunk
    (1, 100, 2, 48, 64),        # fallback shapes
])
def test_ssd_shapes_vs_oracle(Bm, batch, seqlen, ng, ds, ch):
    g = torch.Generator().manual_seed(seqlen + ds)
    L = math.ceil(seqlen / ch) * ch + 7  # padded, poisoned buffers
    C = torch.randn(batch, L, ng, ds, generator=g).to(torch.bfloat16)
    B = torch.randn(batch, L, ng, ds, generator=g).to(torch.bfloat16)
    C[:, seqlen:] = 7.0
    B[:, seqlen:] = -3.0
    out = Bm.ssd_chunk_bmm(C.cuda(), B.cuda(), ch, seqlen=seqlen)
    torch.cuda.synchronize()
    truth = O.ssd_chunk_bmm_ref(bits(C), bits(B), seqlen, ch)
    assert out.shape == truth.shape
    got = out.cpu().numpy()
    assert O.rel_err_inf(got, truth) <= 1e-5 or np.abs(got - truth).max() <= 1e-3


def test_ssd_noncontiguous_group_view(Bm):
    # C and B as views into a fused projection buffer (strided rows)
    g = torch.Generator().manual_seed(5)
    big = torch.randn(1, 512, 2 * 2 * 128 + 64, generator=g).to(torch.bfloat16).cuda()
    C = big[..., :256].view(1, 512, 2, 128)
    B = big[..., 256:512].view(1, 512, 2, 128)
    out = Bm.ssd_chunk_bmm(C, B, 256)
    torch.cuda.synchronize()
    truth = O.ssd_chunk_bmm_ref(bits(C.contiguous()), bits(B.contiguous()), 512, 256)
    assert np.abs(out.cpu().numpy() - truth).max() <= 1e-3


@pytest.mark.parametrize("B", [1, 2, 4, 5, 8, 64, 256, 300])
def test_codebook_head(Bm, B):
    g = torch.Generator().manual_seed(B)
    ncb, K, N = 9, 2048, 1025
    hidden = torch.randn(ncb, B, K, generator=g).to(torch.bfloat16)
    W = (torch.randn(ncb, K, N, generator=g) * 0.02).to(torch.bfloat16)
    head = Bm.CodebookHead(W.cuda())
    out = torch.full((ncb, B, N), float("nan"), device="cuda")
    head(hidden.cuda(), out=out)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    truth = O.codebook_head_ref(bits(hidden), bits(W))
    assert O.rel_err_inf(out.cpu().numpy(), truth) <= 1e-2
    # fp32 accumulation: far inside the bf16 tolerance
    assert O.rel_err_inf(out.cpu().numpy(), truth) <= 1e-4


@pytest.mark.parametrize("ncb,B,K,N", [(9, 8, 2048, 300), (9, 64, 1024, 100), (2, 5, 512, 129),
                                        (4, 16, 2048, 256), (3, 40, 2048, 1025), (9, 33, 4096, 1025),
                                        (2, 7, 192, 300), (2, 3, 100, 130), (1, 2, 64, 128)])
def test_codebook_head_shapes(Bm, ncb, B, K, N):
    # row counts with and without a remainder past the last 128-row tile, K
    # halves of 256..2048, stream tiles that do not fill the MMA N, N < 128
    # (no full tile: CUDA cores only), K = 192 (a multiple of 64, not of 128:
    # the single-CTA tensor-core kernel plus the remainder-row kernel), K = 100
    # (K-major packing: the decode GEMV) and K = 64 with one exact tile
    g = torch.Generator().manual_seed(ncb * 1000 + B + N)
    hidden = torch.randn(ncb, B, K, generator=g).to(torch.bfloat16)
    W = (torch.randn(ncb, K, N, generator=g) * 0.02).to(torch.bfloat16)
    head = Bm.CodebookHead(W.cuda())
    out = torch.full((ncb, B, N), float("nan"), device="cuda")
    head(hidden.cuda(), out=out)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    truth = O.codebook_head_ref(bits(hidden), bits(W))
    assert O.rel_err_inf(out.cpu().numpy(), truth) <= 1e-4


def test_codebook_head_unaligned_hidden(Bm):
    # hidden 2 bytes past a 16-byte boundary (the C ABI takes any bf16
    # pointer): no TMA, every logit on the CUDA cores
    from sonata_b200 import _lib
    g = torch.Generator().manual_seed(11)
    ncb, B, K, N = 3, 6, 256, 200
    hidden = torch.randn(ncb, B, K, generator=g).to(torch.bfloat16)
    W = (torch.randn(ncb, K, N, generator=g) * 0.02).to(torch.bfloat16)
    head = Bm.CodebookHead(W.cuda())
    buf = torch.zeros(ncb * B * K + 8, dtype=torch.bfloat16, device="cuda")
    buf[1:1 + ncb * B * K] = hidden.reshape(-1).cuda()
    out = torch.full((ncb, B, N), float("nan"), device="cuda")
    rc = _lib.lib().sn_codebook_head_bmm(buf.data_ptr() + 2, head.Wt.data_ptr(), out.data_ptr(), ncb, B, K, N, 0,
                                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0
    truth = O.codebook_head_ref(bits(hidden), bits(W))
    assert O.rel_err_inf(out.cpu().numpy(), truth) <= 1e-4


def test_codebook_head_functional_raw_weight(Bm):
    g = torch.Generator().manual_seed(3)
    hidden = torch.randn(3, 16, 256, generator=g).to(torch.bfloat16).cuda()
    W = (torch.randn(3, 256, 77, generator=g) * 0.02).to(torch.bfloat16).cuda()
    out = Bm.codebook_head_bmm(hidden, W)
    torch.cuda.synchronize()
    truth = O.codebook_head_ref(bits(hidden), bits(W))
    assert O.rel_err_inf(out.cpu().numpy(), truth) <= 1e-4


def test_no_device_timeouts(cuda_lib):
    from sonata_b200 import _lib
    assert _lib.lib().sn_device_status(1, None) == 0
