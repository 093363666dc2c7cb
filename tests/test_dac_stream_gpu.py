"""GPU parity of the cached-convolution streaming DAC decoder.

Chunked decoding through StreamingDacDecoder must give the one-shot
DacDecoder's audio: every output sample is the same sequence of tensor-core
products and additions, only the launch windows differ, so the comparison is
bit-for-bit.  Full 44.1 kHz decoder layout (channels 1536 ... 96, strides 8,
8, 4, 2), synthetic weights, chunk sizes from one latent frame up, with and
without the CUDA-graph replay of steady-state chunks, one and two streams.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dec(cuda_lib):
    from sonata_b200.kernels import dac as D
    cfg = D.dac_decoder_config()
    return D.DacDecoder(D.init_decoder_params(cfg, seed=11), cfg)


@pytest.fixture(scope="module")
def latents():
    g = torch.Generator(device="cuda").manual_seed(12)
    return {b: torch.randn(b, 1024, 23, device="cuda", generator=g) for b in (1, 2)}


@pytest.mark.parametrize("batch,chunk,graphs", [(1, 1, False), (1, 5, True), (1, 8, False), (1, 23, False),
                                                (2, 3, True), (2, 7, False)])
def test_streaming_equals_one_shot(dec, latents, batch, chunk, graphs):
    from sonata_b200.kernels import dac_stream as DS
    latent = latents[batch]
    ref = dec(latent)
    got = DS.decode_streaming(dec, latent, chunk, use_graphs=graphs)
    torch.cuda.synchronize()
    assert got.shape == ref.shape
    assert torch.isfinite(got).all()
    diff = (got - ref).abs().max().item()
    assert torch.equal(got, ref), (diff, (got != ref).float().mean().item())


def test_streaming_graph_replays_match_eager(dec, latents):
    from sonata_b200.kernels import dac_stream as DS
    latent = latents[1]
    outs = []
    for graphs in (False, True):
        sd = DS.StreamingDacDecoder(dec, max_chunk_frames=4, use_graphs=graphs)
        pieces = [sd.push(latent[..., f0:f0 + 4]).clone() for f0 in range(0, 20, 4)]
        pieces.append(sd.flush().clone())
        outs.append(torch.cat(pieces, dim=-1))
        if graphs:
            assert len(sd._graphs) >= 1
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


def test_no_device_timeouts(cuda_lib):
    assert cuda_lib.sn_device_status(1, None) == 0
