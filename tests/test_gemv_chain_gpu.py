"""GPU parity of the GEMV chain (one persistent launch over a list of decode
GEMVs, sn_gemv_chain_*) against the per-call GEMV and the CPU oracle.

The chain runs the same tensor-core partition and summation order per row as
sn_gemv_bf16, so its outputs must equal the per-call kernel's bit for bit;
against the float64 oracle the per-call bound applies (max|err| <=
1e-2 * ||y||_inf for bf16 outputs, 1e-5 for fp32 outputs).  Dependencies are
exercised with real data flow: job j + 1 reads job j's output as its x.
"""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

CONFIG2 = [("in_proj", 8512, 2048), ("out_proj", 2048, 4096), ("qkv", 3072, 2048), ("o_proj", 2048, 2048),
           ("fc1", 11264, 2048), ("fc2", 2048, 5632)]


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.fixture(scope="module")
def G(cuda_lib):
    from sonata_b200.kernels import gemv
    return gemv


def _weights(shapes, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [(torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16) for (N, K) in shapes]


@pytest.mark.parametrize("M", [1, 2])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_independent_jobs_match_per_call_and_oracle(G, cuda_lib, M, out_dtype):
    shapes = [(N, K) for (_, N, K) in CONFIG2] * 2
    Ws = _weights(shapes, 3 + M)
    g = torch.Generator(device="cuda").manual_seed(7)
    xs = [torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16) for (N, K) in shapes]
    ys = [torch.full((M, N), float("nan"), device="cuda", dtype=out_dtype) for (N, K) in shapes]
    chain = G.GemvChain(list(zip(Ws, xs, ys)), deps="none")
    chain()
    torch.cuda.synchronize()
    assert cuda_lib.sn_device_status(1, None) == 0
    for W, x, y in zip(Ws, xs, ys):
        ref = G.gemv(x, W, out_dtype=out_dtype)
        torch.cuda.synchronize()
        assert torch.equal(y, ref)
    for j in (0, 1, 5):  # the oracle on a few jobs (float64 on the CPU)
        truth = O.gemv_ref(bits(xs[j]), bits(Ws[j]))
        tol = 1e-2 if out_dtype == torch.bfloat16 else 1e-5
        assert O.rel_err_inf(ys[j].float().cpu().numpy(), truth) <= tol


def _dependent_chain(G, M, seed):
    """Six jobs, each reading the previous job's output as its x (a view of
    it when the next K is shorter): in_proj-, out_proj-, fc2-like shapes."""
    plan = [(4096, 2048), (8512, 4096), (2048, 8192), (5632, 2048), (2048, 5632), (3072, 2048)]
    Ws = _weights(plan, seed)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    x0 = torch.randn(M, plan[0][1], device="cuda", generator=g).to(torch.bfloat16)
    ys = [torch.empty(M, N, device="cuda", dtype=torch.bfloat16) for (N, K) in plan]
    xs = [x0] + [ys[j][:, :plan[j + 1][1]] for j in range(len(plan) - 1)]
    return Ws, xs, ys


@pytest.mark.parametrize("M", [1, 2])
def test_dependent_jobs_read_their_producers_output(G, cuda_lib, M):
    Ws, xs, ys = _dependent_chain(G, M, 11 + M)
    chain = G.GemvChain(list(zip(Ws, xs, ys)), deps="serial")
    chain()
    torch.cuda.synchronize()
    assert cuda_lib.sn_device_status(1, None) == 0
    got = [y.clone() for y in ys]
    # the same data flow as per-call launches on one stream
    for y in ys:
        y.fill_(float("nan"))
    for W, x, y in zip(Ws, xs, ys):
        G.gemv(x, W, out=y)
    torch.cuda.synchronize()
    for a, b in zip(got, ys):
        assert torch.equal(a, b)
    # and the last output against the oracle chained on the CPU
    x = bits(xs[0])
    for j, W in enumerate(Ws):
        t = O.gemv_ref(x, bits(W))
        tb = torch.from_numpy(t.astype(np.float32)).to(torch.bfloat16)  # the chain stores bf16
        x = bits(tb[:, :Ws[j + 1].shape[1]]) if j + 1 < len(Ws) else None
    assert O.rel_err_inf(got[-1].float().cpu().numpy(), t) <= 1e-2


def test_chain_in_a_graph_replays_and_recomputes(G, cuda_lib):
    Ws, xs, ys = _dependent_chain(G, 1, 21)
    chain = G.GemvChain(list(zip(Ws, xs, ys)))
    chain()
    torch.cuda.synchronize()
    eager = [y.clone() for y in ys]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        chain()
    for y in ys:
        y.zero_()
    for _ in range(3):  # the counters reset themselves between launches
        graph.replay()
    torch.cuda.synchronize()
    for a, b in zip(eager, ys):
        assert torch.equal(a, b)
    xs[0].mul_(-1)
    graph.replay()
    torch.cuda.synchronize()
    assert not torch.equal(ys[-1], eager[-1])
    assert cuda_lib.sn_device_status(1, None) == 0
    del graph


def test_config2_chain_matches_per_call(G, cuda_lib):
    """The bench's workload: 26 layers x 6 GEMVs, serial order, one launch."""
    shapes = [(N, K) for _ in range(26) for (_, N, K) in CONFIG2]
    Ws = _weights(shapes, 31)
    g = torch.Generator(device="cuda").manual_seed(32)
    x_flat = torch.randn(sum(K for _, K in shapes), device="cuda", generator=g).to(torch.bfloat16)
    y_flat = torch.empty(sum(N for N, _ in shapes), device="cuda", dtype=torch.bfloat16)
    xs, ys, ox, oy = [], [], 0, 0
    for N, K in shapes:
        xs.append(x_flat[ox:ox + K].view(1, K))
        ys.append(y_flat[oy:oy + N].view(1, N))
        ox, oy = ox + K, oy + N
    chain = G.GemvChain(list(zip(Ws, xs, ys)))
    for _ in range(2):
        chain(pdl=True)
    torch.cuda.synchronize()
    assert cuda_lib.sn_device_status(1, None) == 0
    for j in range(0, len(shapes), 7):
        assert torch.equal(ys[j], G.gemv(xs[j], Ws[j]))


def test_plan_rejects_unordered_buffers(G):
    from sonata_b200._lib import SonataError
    Ws, xs, ys = _dependent_chain(G, 1, 41)
    jobs = list(zip(Ws, xs, ys))
    with pytest.raises(SonataError):  # x of job j+1 is job j's y, but nothing orders them
        G.GemvChain(jobs, deps="none")
    with pytest.raises(SonataError):  # two jobs writing one buffer
        G.GemvChain([(Ws[0], xs[0], ys[0]), (Ws[0], xs[0], ys[0])], deps="serial")
    with pytest.raises(SonataError):  # an output over one of the chain's weights
        G.GemvChain([(Ws[0], xs[0], Ws[0].view(-1)[:4096].view(1, 4096))], deps="none")


@pytest.mark.parametrize("kind", ["int8", "e4m3"])
@pytest.mark.parametrize("M", [1, 2])
def test_quantized_chain_matches_per_call(G, cuda_lib, kind, M):
    """8-bit weights (fused dequant): the chain takes whole rows as one
    segment (32 KB tiles); int8 equals gemv_quantized bit for bit (exact
    integer sums), e4m3 within fp32 summation order (1e-5 of ||y||_inf); both
    the dequantise-then-matmul oracle within 1e-3."""
    shapes = [(N, K) for (_, N, K) in CONFIG2]
    Ws = _weights(shapes, 51 + M)
    qws = [G.quantize_weight(W, kind) for W in Ws]
    g = torch.Generator(device="cuda").manual_seed(52)
    xs = [torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16) for (N, K) in shapes]
    xs[1][0, 5] = 300.0  # one large activation
    ys = [torch.full((M, N), float("nan"), device="cuda", dtype=torch.float32) for (N, K) in shapes]
    chain = G.GemvChain(list(zip(qws, xs, ys)), deps="none")
    chain()
    torch.cuda.synchronize()
    assert cuda_lib.sn_device_status(1, None) == 0
    for qw, x, y in zip(qws, xs, ys):
        ref = G.gemv_quantized(x, qw, out_dtype=torch.float32)
        if kind == "int8":  # exact integer sums either way
            assert torch.equal(y, ref)
        else:  # one fp32 accumulator per row here, two segment partials per call
            assert (y - ref).abs().max().item() <= 1e-5 * ref.abs().max().item()
    for j in (0, 1, 5):
        truth = O.dequant_gemv_ref(bits(xs[j]), qws[j].q.cpu().numpy(), qws[j].scale.cpu().numpy(), kind)
        assert O.rel_err_inf(ys[j].cpu().numpy(), truth) <= 1e-3


@pytest.mark.parametrize("kind", ["int8", "e4m3"])
def test_quantized_dependent_chain_and_nonfinite_rows(G, cuda_lib, kind):
    Ws, xs, ys = _dependent_chain(G, 2, 61)
    qws = [G.quantize_weight(W, kind) for W in Ws]
    with torch.no_grad():
        xs[0][1, 3] = float("inf")  # row 1 of the first x is non-finite: NaN outputs on that row
    chain = G.GemvChain(list(zip(qws, xs, ys)), deps="serial")
    chain()
    torch.cuda.synchronize()
    assert cuda_lib.sn_device_status(1, None) == 0
    got = [y.clone() for y in ys]
    for y in ys:
        y.zero_()
    for qw, x, y in zip(qws, xs, ys):
        G.gemv_quantized(x, qw, out=y)
    torch.cuda.synchronize()
    for a, b in zip(got, ys):
        assert (torch.isnan(a) == torch.isnan(b)).all()
        fa, fb = torch.nan_to_num(a).float(), torch.nan_to_num(b).float()
        if kind == "int8":
            assert torch.equal(fa, fb)
        else:  # fp32 summation order, then one bf16 rounding per job
            assert (fa - fb).abs().max().item() <= 2e-2 * fb.abs().max().item()
    assert torch.isnan(got[0][1]).all() and torch.isfinite(got[0][0]).all()
