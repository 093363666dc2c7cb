"""Host logic of the nn.Linear patch (kernels/patch.py semantics), on the CPU.

The CUDA launch is replaced by a recorder so the routing rules can be checked
without a GPU: 2-D (M, K) and 3-D (M, 1, K) decode shapes with M in batches go
to the kernel and return the pinned buffer; everything else falls back to the
original forward.
"""
import types

import pytest
import torch

from sonata_b200.kernels import patch as P


@pytest.fixture
def cpu_patch(monkeypatch):
    calls = []

    def fake_make_launch(W, qw, lin):
        def launch(xc, y, M):
            nxt = getattr(lin, "_gemv_next", None)
            calls.append((tuple(xc.shape), M, y.data_ptr(), None if nxt is None else nxt[0]))
            y.copy_((xc.float() @ W.float().t()).to(y.dtype))
        return launch

    monkeypatch.setattr(P, "_make_launch", fake_make_launch)
    monkeypatch.setattr(P, "require_cuda", lambda *a, **k: None)
    return calls


def _lin(N=16, K=32, bias=False):
    torch.manual_seed(0)
    lin = torch.nn.Linear(K, N, bias=bias).to(torch.bfloat16)
    return lin


def test_routes_decode_shapes_and_pins_buffers(cpu_patch):
    lin = _lin()
    ref_w = lin.weight.detach().float()
    P.patch_linear(lin, batches=(1, 2))
    x2 = torch.randn(2, 32).to(torch.bfloat16)
    y = lin(x2)
    assert cpu_patch[-1][:2] == ((2, 32), 2)
    torch.testing.assert_close(y.float(), (x2.float() @ ref_w.t()).to(torch.bfloat16).float())
    y_again = lin(torch.randn(2, 32).to(torch.bfloat16))
    assert y_again.data_ptr() == y.data_ptr()  # pinned, reused buffer
    x3 = torch.randn(1, 1, 32).to(torch.bfloat16)
    y3 = lin(x3)
    assert y3.shape == (1, 1, 16) and cpu_patch[-1][:2] == ((1, 32), 1)


def test_falls_back_for_prefill_and_other_m(cpu_patch):
    lin = _lin()
    P.patch_linear(lin, batches=(1, 2))
    n = len(cpu_patch)
    lin(torch.randn(3, 32).to(torch.bfloat16))          # M not in batches
    lin(torch.randn(1, 7, 32).to(torch.bfloat16))       # prefill seqlen 7
    lin(torch.randn(2, 5, 32).to(torch.bfloat16))
    assert len(cpu_patch) == n


def test_bias_is_rejected_and_unpatch_restores(cpu_patch):
    with pytest.raises(AssertionError):
        P.patch_linear(_lin(bias=True))
    lin = _lin()
    orig = lin.forward
    P.patch_linear(lin)
    assert lin.forward is not orig and hasattr(lin, "_gemv_orig")
    P.unpatch_linear(lin)
    assert not hasattr(lin, "_gemv_orig")
    n = len(cpu_patch)
    lin(torch.randn(1, 32).to(torch.bfloat16))
    assert len(cpu_patch) == n


def test_batches_limited_to_kernel_m(cpu_patch):
    with pytest.raises(ValueError):
        P.patch_linear(_lin(), batches=(1, 8))


class _Layer(torch.nn.Module):
    def __init__(self, attn: bool):
        super().__init__()
        if attn:
            self.mixer = torch.nn.Module()
            self.mixer.in_proj = torch.nn.Linear(8, 24, bias=False)
            self.mixer.out_proj = torch.nn.Linear(8, 8, bias=False)
            self.mlp = torch.nn.Module()
            self.mlp.fc1 = torch.nn.Linear(8, 16, bias=False)
            self.mlp.fc2 = torch.nn.Linear(16, 8, bias=True)   # bias -> skipped
        else:
            self.mixer = torch.nn.Module()
            self.mixer.in_proj = torch.nn.Linear(8, 32, bias=False)
            self.mixer.out_proj = torch.nn.Linear(16, 8, bias=False)
            self.mixer.dt_proj = torch.nn.Linear(8, 8, bias=False)  # not a target


def _model():
    m = torch.nn.Module()
    m.backbone = torch.nn.Module()
    m.backbone.layers = torch.nn.ModuleList([_Layer(i == 1) for i in range(3)])
    m.backbone.config = types.SimpleNamespace(attn_layer_idx=[1])
    return m


def test_zonos_target_selection():
    m = _model()
    names = [n for n, _ in P.zonos_patch_targets(m)]
    assert names == ["layers.0.mixer.in_proj", "layers.0.mixer.out_proj",
                     "layers.2.mixer.in_proj", "layers.2.mixer.out_proj"]
    names_attn = [n for n, _ in P.zonos_patch_targets(m, include_attn=True)]
    assert "layers.1.mlp.fc1" in names_attn and "layers.1.mlp.fc2" not in names_attn
    assert len(names_attn) == 7


def test_patch_zonos_projections_counts(cpu_patch):
    m = _model()
    for p in m.parameters():
        p.data = p.data.to(torch.bfloat16)
    assert P.patch_zonos_projections(m) == 4
    m2 = _model()
    for p in m2.parameters():
        p.data = p.data.to(torch.bfloat16)
    assert P.patch_zonos_projections(m2, include_attn=True) == 7


def test_link_decode_chain_hints_the_next_weight(cpu_patch):
    lins = [_lin(N=16 * (i + 1), K=32) for i in range(3)]
    for lin in lins:
        P.patch_linear(lin, batches=(1,))
    plain = torch.nn.Linear(32, 8, bias=False)  # not patched: skipped by the chain
    P.link_decode_chain([lins[0], plain, lins[1], lins[2]])
    x = torch.randn(1, 32).to(torch.bfloat16)
    for lin in lins:
        lin(x)
    hints = [c[3] for c in cpu_patch[-3:]]
    for i in range(2):
        W1 = lins[i + 1]._gemv_keepalive[0]
        assert hints[i] == (0, W1.data_ptr(), 32, W1.shape[0], 32)
    assert hints[2] is None  # the last one has no successor
    P.link_decode_chain(lins, cyclic=True)
    lins[2](x)
    assert cpu_patch[-1][3][1] == lins[0]._gemv_keepalive[0].data_ptr()
    # outputs do not depend on the hint
    y_hint = lins[0](x).clone()
    P.unpatch_linear(lins[1])
    assert not hasattr(lins[1], "_gemv_next")
    lins[0]._gemv_next = None
    torch.testing.assert_close(lins[0](x), y_hint)


def test_patch_zonos_projections_links_in_module_order(cpu_patch):
    m = _model()
    for p in m.parameters():
        p.data = p.data.to(torch.bfloat16)
    P.patch_zonos_projections(m)
    mods = [mod for _, mod in P.zonos_patch_targets(m)]
    for a, b in zip(mods, mods[1:]):
        assert a._gemv_next[0][1] == b._gemv_keepalive[0].data_ptr()
    assert mods[-1]._gemv_next is None
    m2 = _model()
    for p in m2.parameters():
        p.data = p.data.to(torch.bfloat16)
    P.patch_zonos_projections(m2, prefetch_chain=False)
    assert all(getattr(mod, "_gemv_next", None) is None for _, mod in P.zonos_patch_targets(m2))
