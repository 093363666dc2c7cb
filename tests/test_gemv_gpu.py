"""GPU parity of the decode GEMV (bf16, int8, e4m3) against the CPU oracle.

Tolerances:
* bf16 GEMV: max|err| <= 1e-2 * ||y||_inf and, at the
  check_gemv shapes with M=2, rel-RMS < 3e-3 (scripts/validation_harness.py:346).
* quantised GEMV, fp32 output: max|err| <= 1e-3 * ||y||_inf against
  dequantise-to-fp32-then-matmul; the quantisation codes themselves are
  bit-exact against the C oracle.
"""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

SHAPES = {  # (N, K) of BASELINE configs 1-2 plus the real Zonos attention MLP
    "in_proj": (8512, 2048), "out_proj": (2048, 4096), "qkv": (3072, 2048), "o_proj": (2048, 2048),
    "fc1": (11264, 2048), "fc2": (2048, 5632), "zonos_fc1": (16384, 2048), "zonos_fc2": (2048, 8192),
}


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def make(N, K, M, seed=0, dev="cuda"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    W = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    return x.to(dev), W.to(dev)


@pytest.fixture(scope="module")
def G(cuda_lib):
    from sonata_b200.kernels import gemv
    return gemv


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("M", [1, 2])
def test_bf16_gemv_decode_shapes(G, name, M):
    N, K = SHAPES[name]
    x, W = make(N, K, M)
    y = G.candidate_cute_splitk(x, W)
    torch.cuda.synchronize()
    assert y.dtype == torch.bfloat16 and y.shape == (M, N)
    truth = O.gemv_ref(bits(x), bits(W))
    out = y.float().cpu().numpy()
    assert O.rel_err_inf(out, truth) <= 1e-2
    if M == 2:
        assert O.rel_rms(out, truth) < 3e-3
    # fp32 output: only summation-order differences remain
    y32 = G.gemv(x, W, out_dtype=torch.float32)
    assert O.rel_err_inf(y32.cpu().numpy(), truth) <= 1e-5


@pytest.mark.parametrize("N,K,M", [(1, 8, 1), (7, 24, 3), (1025, 2048, 4), (300, 1280, 3), (33, 1000, 2), (300, 12, 1),
                                   (96, 6152, 2), (130, 16384, 1)])
def test_bf16_gemv_odd_shapes(G, N, K, M):
    x, W = make(N, K, M, seed=N + K)
    y = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float32)
    G.gemv(x, W, out=y)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all(), "unwritten output elements"
    truth = O.gemv_ref(bits(x), bits(W))
    assert O.rel_err_inf(y.cpu().numpy(), truth) <= 1e-5


def test_bf16_gemv_k_not_multiple_of_8(G):
    # rows of 2050 bf16 are not 16-byte aligned: the kernel must still sum
    # every element (the reference's m2 kernel drops the tail, gemv.py:135)
    x, W = make(257, 2050, 2, seed=5)
    y = G.gemv(x, W, out_dtype=torch.float32)
    torch.cuda.synchronize()
    truth = O.gemv_ref(bits(x), bits(W))
    assert O.rel_err_inf(y.cpu().numpy(), truth) <= 1e-5


def test_bf16_gemv_strided_and_misaligned(G):
    x, Wfull = make(512, 2056, 2, seed=9)
    W = Wfull[:, :2048]                      # aligned row stride 2056 > K
    xs = torch.randn(2, 2049, device="cuda").to(torch.bfloat16)[:, 1:]  # x misaligned by 2 bytes
    y = G.gemv(xs, W, out_dtype=torch.float32)
    torch.cuda.synchronize()
    truth = O.gemv_ref(bits(xs), bits(W))
    assert O.rel_err_inf(y.cpu().numpy(), truth) <= 1e-5
    # aligned rows (stride 1032) with a K tail of one element
    x2, W2full = make(300, 1032, 2, seed=10)
    W2, x2 = W2full[:, :1025], x2[:, :1025]
    y2 = G.gemv(x2, W2, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert O.rel_err_inf(y2.cpu().numpy(), O.gemv_ref(bits(x2), bits(W2))) <= 1e-5


def test_launchers_write_in_place_and_capture_in_graph(G):
    N, K = 2048, 4096
    x, W = make(N, K, 2)
    y = torch.empty(2, N, device="cuda", dtype=torch.bfloat16)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        G.skinny_gemv_splitk_m2(y, x, W, 2, N, K, torch.cuda.current_stream())
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        G.skinny_gemv_splitk_m2(y, x, W, 2, N, K, None)
    y.zero_()
    x.copy_(torch.randn(2, K, device="cuda").to(torch.bfloat16))
    g.replay()
    torch.cuda.synchronize()
    # empty-graph tripwire: the replay must have recomputed y from the new x
    truth = O.gemv_ref(bits(x), bits(W))
    assert O.rel_err_inf(y.float().cpu().numpy(), truth) <= 1e-2


def test_rejects_bad_inputs(G):
    x, W = make(16, 32, 1)
    with pytest.raises(ValueError):
        G.gemv(torch.randn(5, 32, device="cuda").to(torch.bfloat16), W)
    with pytest.raises(TypeError):
        G.gemv(x.float(), W)
    with pytest.raises(ValueError):
        G.gemv(x.cpu(), W)


# ---------------- quantised ----------------

@pytest.mark.parametrize("kind", ["int8", "e4m3"])
def test_quantize_codes_bit_exact(G, kind):
    x, W = make(8512, 2048, 1, seed=3)
    W[5] = 0  # dead row
    qw = G.quantize_weight(W, kind)
    torch.cuda.synchronize()
    if kind == "int8":
        q_ref, s_ref = O.quant_int_rows(bits(W), 8)
        q = qw.q.cpu().numpy()
    else:
        q_ref, s_ref = O.quant_e4m3_rows(bits(W))
        q = qw.q.cpu().numpy()
    assert np.array_equal(q, q_ref)
    assert np.array_equal(qw.scale.cpu().numpy().view(np.uint32), s_ref.reshape(-1).view(np.uint32))


@pytest.mark.parametrize("kind", ["int8", "e4m3"])
@pytest.mark.parametrize("M", [1, 2, 4])
@pytest.mark.parametrize("NK", [(8512, 2048), (2048, 4096), (512, 5632), (777, 1280), (1000, 1040), (64, 24)])
def test_quantized_gemv_matches_dequant_oracle(G, kind, M, NK):
    N, K = NK
    x, W = make(N, K, M, seed=11)
    qw = G.quantize_weight(W, kind)
    y = G.gemv_quantized(x, qw)  # fp32 output
    torch.cuda.synchronize()
    truth = O.dequant_gemv_ref(bits(x), qw.q.cpu().numpy(), qw.scale.cpu().numpy(), kind)
    assert O.rel_err_inf(y.cpu().numpy(), truth) <= 1e-3
    # bf16 output is the same value rounded once
    yb = G.gemv_quantized(x, qw, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert O.rel_err_inf(yb.float().cpu().numpy(), truth) <= 1e-2


@pytest.mark.parametrize("kind", ["int8", "e4m3"])
def test_quantized_gemv_extreme_activations(G, kind):
    # The tensor-core path stages x as f16 times a power of two per x row:
    # activations far outside f16's range must come through unchanged.
    x, W = make(1024, 2048, 2, seed=17)
    x = x.float()
    x[0] *= 3.0e6      # beyond f16's largest finite value
    x[1] *= 1.0e-30    # far below f16's smallest subnormal
    x = x.to(torch.bfloat16)
    qw = G.quantize_weight(W, kind)
    y = G.gemv_quantized(x, qw)
    torch.cuda.synchronize()
    truth = O.dequant_gemv_ref(bits(x), qw.q.cpu().numpy(), qw.scale.cpu().numpy(), kind)
    out = y.cpu().numpy()
    for m in range(2):
        t = np.asarray(truth[m], np.float64)
        assert np.isfinite(out[m]).all() and np.abs(t).max() > 0
        assert np.abs(out[m] - t).max() / np.abs(t).max() <= 1e-3


def test_quantized_gemv_unaligned_rows(G):
    # K = 1001: int8 rows are not 16-byte aligned -> element-load path
    x, W = make(77, 1001, 2, seed=13)
    for kind in ("int8", "e4m3"):
        qw = G.quantize_weight(W, kind)
        y = G.gemv_quantized(x, qw)
        torch.cuda.synchronize()
        truth = O.dequant_gemv_ref(bits(x), qw.q.cpu().numpy(), qw.scale.cpu().numpy(), kind)
        assert O.rel_err_inf(y.cpu().numpy(), truth) <= 1e-3


# ---------------- next-weight L2 prefetch hint (sn_gemv_ex) ----------------

@pytest.mark.parametrize("M", [1, 2, 4])
def test_next_weight_hint_is_result_neutral(G, M):
    x, W = make(8512, 2048, M, seed=3)
    base = G.gemv(x, W, out_dtype=torch.float32)
    wide = (torch.randn(3072, 2056, device="cuda") * 0.02).to(torch.bfloat16)
    nexts = [
        make(2048, 4096, 1, seed=4)[1],                          # bf16, contiguous rows
        wide[:, :2048],                                          # rows 4112 bytes apart: one prefetch per row
        G.quantize_weight(make(1025, 2048, 1, seed=5)[1], "int8"),
        G.quantize_weight(make(777, 1280, 1, seed=6)[1], "e4m3"),
        make(5, 7, 1, seed=7)[1],                                # 14-byte rows: not prefetchable, skipped
        W,                                                       # itself
    ]
    for nw in nexts:
        y = G.gemv(x, W, out_dtype=torch.float32, next_weight=nw)
        torch.cuda.synchronize()
        assert torch.equal(y, base)
        assert torch.equal(G.gemv(x, W, next_weight=nw), G.gemv(x, W))
    for kind in ("int8", "e4m3"):
        qw = G.quantize_weight(W, kind)
        yq = G.gemv_quantized(x, qw)
        for nw in (nexts[0], nexts[2]):
            assert torch.equal(G.gemv_quantized(x, qw, next_weight=nw), yq)
    with pytest.raises(ValueError):
        G.gemv(x, W, next_weight=torch.zeros(4, 8, 8, device="cuda", dtype=torch.bfloat16).view(4, 64)[:, ::2])


def test_next_weight_chain_in_graph_with_pdl(G):
    """The config-2 call pattern: a PDL chain in one CUDA graph, every GEMV
    hinting the next one's weight, equals the same chain without hints."""
    shapes = [(8512, 2048), (2048, 4096), (3072, 2048), (2048, 2048), (11264, 2048), (2048, 5632)] * 2
    Ws = [make(N, K, 1, seed=20 + i)[1] for i, (N, K) in enumerate(shapes)]
    xs = [make(N, K, 1, seed=40 + i)[0] for i, (N, K) in enumerate(shapes)]
    ys = [torch.empty(1, N, device="cuda", dtype=torch.bfloat16) for (N, K) in shapes]
    ref = [G.gemv(x, W) for x, W in zip(xs, Ws)]

    def chain():
        for i in range(len(Ws)):
            G.gemv(xs[i], Ws[i], out=ys[i], pdl=True, next_weight=Ws[i + 1] if i + 1 < len(Ws) else None)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        chain()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        chain()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for y, r in zip(ys, ref):
        assert torch.equal(y, r)


# ---------------- nn.Linear patch ----------------

def test_patch_linear_on_gpu_and_in_graph(cuda_lib):
    from sonata_b200.kernels.patch import patch_linear, unpatch_linear
    torch.manual_seed(0)
    lin = torch.nn.Linear(2048, 8512, bias=False, device="cuda", dtype=torch.bfloat16)
    ref = lin.weight.detach().float()
    patch_linear(lin)
    x = torch.randn(2, 2048, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        y = lin(x)
        torch.cuda.synchronize()
        truth = (x.float() @ ref.t()).cpu().numpy()
        assert O.rel_err_inf(y.float().cpu().numpy(), truth) <= 1e-2
        y3 = lin(x[:1].unsqueeze(1))
        assert y3.shape == (1, 1, 8512)
        # prefill falls back to the original forward
        xp = torch.randn(1, 9, 2048, device="cuda", dtype=torch.bfloat16)
        torch.testing.assert_close(lin(xp), torch.nn.functional.linear(xp, lin.weight))
        # graph capture of the patched forward (Zonos captures its decode step)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            lin(x)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            yg = lin(x)
        x.copy_(torch.randn_like(x))
        g.replay()
        torch.cuda.synchronize()
        truth = (x.float() @ ref.t()).cpu().numpy()
        assert O.rel_err_inf(yg.float().cpu().numpy(), truth) <= 1e-2
    unpatch_linear(lin)


@pytest.mark.parametrize("fmt", ["int8", "e4m3"])
def test_patch_linear_quantized(cuda_lib, fmt):
    from sonata_b200.kernels.patch import patch_linear
    torch.manual_seed(1)
    lin = torch.nn.Linear(2048, 4096, bias=False, device="cuda", dtype=torch.bfloat16)
    patch_linear(lin, weight_format=fmt)
    qw = lin._gemv_keepalive[1]
    x = torch.randn(2, 2048, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        y = lin(x)
    torch.cuda.synchronize()
    truth = O.dequant_gemv_ref(bits(x), qw.q.cpu().numpy(), qw.scale.cpu().numpy(), fmt)
    assert O.rel_err_inf(y.float().cpu().numpy(), truth) <= 1e-2


def test_patch_linear_decode_chain(cuda_lib):
    """link_decode_chain: bf16 and quantised patched Linears hinting each
    other give the outputs they give unlinked."""
    from sonata_b200.kernels.patch import link_decode_chain, patch_linear
    torch.manual_seed(2)
    lins = [torch.nn.Linear(K, N, bias=False, device="cuda", dtype=torch.bfloat16)
            for (N, K) in [(8512, 2048), (2048, 4096), (3072, 2048)]]
    for lin, fmt in zip(lins, ["bf16", "int8", "e4m3"]):
        patch_linear(lin, batches=(1, 2), weight_format=fmt)
    xs = [torch.randn(2, lin.in_features, device="cuda", dtype=torch.bfloat16) for lin in lins]
    with torch.no_grad():
        ref = [lin(x).clone() for lin, x in zip(lins, xs)]
        link_decode_chain(lins, cyclic=True)
        out = [lin(x).clone() for lin, x in zip(lins, xs)]
    torch.cuda.synchronize()
    for a, b in zip(out, ref):
        assert torch.equal(a, b)
