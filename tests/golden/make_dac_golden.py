"""Freeze transformers' DAC decoder outputs on seeded inputs as tests/golden/dac.npz.

The vocoder the reference decodes with (requirements.txt: transformers
>= 4.48.1; the reference's dumped config says 5.10.2,
docs/dac_architecture.md:27) is a third-party package, not part of the
reference checkout.  This script runs in the build container, where
transformers 5.5.0 is installed:

    python tests/golden/make_dac_golden.py

* ``decoder``: transformers' own ``DacDecoder`` (modeling_dac.py) with a small
  config (hidden 32, decoder hidden 256 -> channels 128 / 64 / 32 / 16,
  upsampling 8, 8, 4, 2), weights from ``sonata_b200.kernels.dac.
  init_decoder_params(config, seed=7)`` loaded into it, on a seeded latent
  [2, 32, 3]: audio [2, 1, 1536].
* ``convt_*``: torch ``F.conv_transpose1d`` of transformers' ``Snake1d`` output
  for the four DacDecoderBlock stride / kernel / padding triples
  (modeling_dac.py DacDecoderBlock.__init__).

It also checks the oracle's float64 restatement (oracle.dac_decoder_ref,
oracle.snake_conv_transpose1d_ref) against both before saving.  The GPU box
never runs this script.
"""
from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIG = {"hidden_size": 32, "decoder_hidden_size": 256, "upsampling_ratios": (8, 8, 4, 2)}
PARAM_SEED = 7
LATENT_SEED = 8
CONVT_CASES = [(8, 16, 4, 32, 16, 5), (8, 16, 4, 16, 32, 4), (4, 8, 2, 32, 16, 6), (2, 4, 1, 16, 16, 7)]  # s, K, p, Cin, Cout, T


def main() -> int:
    from transformers import DacConfig
    from transformers.models.dac.modeling_dac import DacDecoder, Snake1d

    import oracle as O
    from sonata_b200.kernels.dac import init_decoder_params

    out = {}
    cfg = DacConfig(hidden_size=CONFIG["hidden_size"], decoder_hidden_size=CONFIG["decoder_hidden_size"],
                    upsampling_ratios=list(CONFIG["upsampling_ratios"]))
    dec = DacDecoder(cfg).eval()
    params = init_decoder_params(CONFIG, seed=PARAM_SEED)
    dec.load_state_dict(params, strict=True)
    latent = torch.randn(2, CONFIG["hidden_size"], 3, generator=torch.Generator().manual_seed(LATENT_SEED))
    with torch.no_grad():
        audio = dec(latent)
    ref = O.dac_decoder_ref(latent.numpy(), {k: v.numpy() for k, v in params.items()},
                            CONFIG["upsampling_ratios"])
    err = np.abs(ref - audio.numpy()).max()
    print(f"decoder: audio {tuple(audio.shape)}, |oracle - transformers| = {err:.2e}")
    assert err < 1e-4, err
    out["decoder__latent"] = latent.numpy()
    out["decoder__audio"] = audio.numpy()
    out["decoder__param_seed"] = np.array(PARAM_SEED)
    out["decoder__param_sum"] = np.array(sum(float(v.double().sum()) for v in params.values()))

    g = torch.Generator().manual_seed(11)
    for n, (s, K, p, cin, cout, T) in enumerate(CONVT_CASES):
        x = torch.randn(1, cin, T, generator=g)
        snake = Snake1d(cin)
        with torch.no_grad():
            snake.alpha.copy_(torch.rand(1, cin, 1, generator=g) + 0.5)
        w = torch.randn(cin, cout, K, generator=g) / math.sqrt(cin * K / s)
        b = torch.randn(cout, generator=g) * 0.1
        with torch.no_grad():
            y = F.conv_transpose1d(snake(x), w, b, stride=s, padding=p)
        yo = O.snake_conv_transpose1d_ref(x.numpy(), snake.alpha.detach().numpy().reshape(-1), w.numpy(), b.numpy(),
                                          stride=s, padding=p)
        e = np.abs(yo - y.numpy()).max()
        print(f"convt {n}: s={s} K={K} p={p} -> {tuple(y.shape)}, |oracle - torch| = {e:.2e}")
        assert e < 1e-5, e
        key = f"convt_{n}"
        out[f"{key}__x"] = x.numpy()
        out[f"{key}__alpha"] = snake.alpha.detach().numpy().reshape(-1)
        out[f"{key}__w"] = w.numpy()
        out[f"{key}__b"] = b.numpy()
        out[f"{key}__y"] = y.numpy()
        out[f"{key}__meta"] = np.array([s, K, p])
    np.savez_compressed(OUT / "dac.npz", **out)
    print("wrote", OUT / "dac.npz")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
