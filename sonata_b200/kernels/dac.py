"""The DAC decoder on the fused Snake kernels: all 29 Snake -> conv edges.

The vocoder the reference decodes with is transformers' ``DacModel``
(modeling_dac.py: ``DacDecoder``, ``DacDecoderBlock``, ``DacResidualUnit``,
``Snake1d``); its module list and the 29 fuse edges are in the reference's
docs/dac_architecture.md:37-133, 306-314.  Each edge is one kernel launch:

* stem ``conv1`` (k 7, pad 3, no Snake): ``fused_snake_conv1d(...,
  activation="none")``;
* per block, ``snake1 -> conv_t1`` (ConvTranspose1d, kernel 2 s, stride s,
  padding ceil(s / 2)): ``fused_snake_conv_transpose1d`` -- a polyphase GEMM
  on the tensor cores;
* per residual unit (dilations 1, 3, 9), ``snake1 -> conv1`` (k 7) and
  ``snake2 -> conv2`` (k 1) with the unit's ``hidden_state + ...`` fused into
  the second launch's epilogue (``residual=``);
* ``snake1 -> conv2 -> tanh``, the tanh fused (``post="tanh"``).

Weights are a state dict with the transformers names (``conv1.weight``,
``block.0.conv_t1.weight``, ``block.0.res_unit1.snake1.alpha`` ...), the
effective weights of a checkpoint (weight norm folded in), packed once into
the tensor-core layout when the decoder is built.  No checkpoint is
available offline; ``init_decoder_params`` draws seeded synthetic ones.
"""
from __future__ import annotations

import math

import torch

from .fused_snake_conv import (fused_snake_conv1d, fused_snake_conv_transpose1d, pack_conv1d_weight,
                               pack_conv_transpose1d_weight)

DILATIONS = (1, 3, 9)


def dac_decoder_config(hidden_size: int = 1024, decoder_hidden_size: int = 1536,
                       upsampling_ratios=(8, 8, 4, 2)) -> dict:
    """The decoder half of transformers' DacConfig (defaults: the 44.1 kHz
    model of docs/dac_architecture.md:5-34)."""
    return {"hidden_size": int(hidden_size), "decoder_hidden_size": int(decoder_hidden_size),
            "upsampling_ratios": tuple(int(s) for s in upsampling_ratios)}


def decoder_shapes(config: dict) -> dict:
    """Parameter name -> shape, in the transformers DacDecoder layout."""
    C = config["decoder_hidden_size"]
    shapes = {"conv1.weight": (C, config["hidden_size"], 7), "conv1.bias": (C,)}
    for i, s in enumerate(config["upsampling_ratios"]):
        cin, cout = C // 2 ** i, C // 2 ** (i + 1)
        b = f"block.{i}"
        shapes[f"{b}.snake1.alpha"] = (1, cin, 1)
        shapes[f"{b}.conv_t1.weight"] = (cin, cout, 2 * s)
        shapes[f"{b}.conv_t1.bias"] = (cout,)
        for j in range(3):
            r = f"{b}.res_unit{j + 1}"
            shapes[f"{r}.snake1.alpha"] = (1, cout, 1)
            shapes[f"{r}.conv1.weight"] = (cout, cout, 7)
            shapes[f"{r}.conv1.bias"] = (cout,)
            shapes[f"{r}.snake2.alpha"] = (1, cout, 1)
            shapes[f"{r}.conv2.weight"] = (cout, cout, 1)
            shapes[f"{r}.conv2.bias"] = (cout,)
    cl = C // 2 ** len(config["upsampling_ratios"])
    shapes["snake1.alpha"] = (1, cl, 1)
    shapes["conv2.weight"] = (1, cl, 7)
    shapes["conv2.bias"] = (1,)
    return shapes


def init_decoder_params(config: dict, seed: int = 0) -> dict:
    """Seeded synthetic decoder weights (CPU fp32, drawn in ``decoder_shapes``
    order from one torch.Generator): alpha ~ U(0.5, 1.5); conv weights
    ~ N(0, 1 / fan_in) (fan_in = Cin * K, Cin * K / s for a transposed conv),
    the residual units' 1x1 convs and the output conv scaled by 1/2 so the
    residual stack and the tanh stay in range; biases ~ N(0, 0.05^2)."""
    g = torch.Generator().manual_seed(seed)
    p = {}
    strides = dict(enumerate(config["upsampling_ratios"]))
    for name, shape in decoder_shapes(config).items():
        if name.endswith("alpha"):
            p[name] = torch.rand(shape, generator=g) + 0.5
        elif name.endswith("bias"):
            p[name] = torch.randn(shape, generator=g) * 0.05
        else:
            if "conv_t1" in name:
                s = strides[int(name.split(".")[1])]
                fan_in = shape[0] * shape[2] / s
            else:
                fan_in = shape[1] * shape[2]
            scale = 0.5 if (name.endswith("conv2.weight")) else 1.0
            p[name] = torch.randn(shape, generator=g) * (scale / math.sqrt(fan_in))
    return p


class DacDecoder:
    """Latent [B, hidden_size, T0] -> audio [B, 1, T0 * prod(strides)] on the
    B200 kernels; same function as transformers' DacDecoder.forward."""

    def __init__(self, params: dict, config: dict, device="cuda"):
        self.config = config
        self.p = {k: v.detach().to(device=device, dtype=torch.float32).contiguous() for k, v in params.items()}
        missing = set(decoder_shapes(config)) - set(self.p)
        if missing:
            raise ValueError(f"missing decoder parameters: {sorted(missing)[:4]} ...")
        # every conv weight packed once into the tensor-core layout
        self.packed = {}
        for name, w in self.p.items():
            if not name.endswith("weight"):
                continue
            if "conv_t1" in name:
                s = self.config["upsampling_ratios"][int(name.split(".")[1])]
                self.packed[name] = pack_conv_transpose1d_weight(w, s)
            else:
                self.packed[name] = pack_conv1d_weight(w)

    def _a(self, name: str) -> torch.Tensor:
        return self.p[name].view(-1)

    def __call__(self, latent: torch.Tensor, stream=None) -> torch.Tensor:
        p = self.p
        k = self.packed
        h = fused_snake_conv1d(latent, None, p["conv1.weight"], p["conv1.bias"], padding=3, stream=stream,
                               activation="none", packed=k["conv1.weight"])
        for i, s in enumerate(self.config["upsampling_ratios"]):
            b = f"block.{i}"
            h = fused_snake_conv_transpose1d(h, self._a(f"{b}.snake1.alpha"), p[f"{b}.conv_t1.weight"],
                                             p[f"{b}.conv_t1.bias"], stride=s, padding=(s + 1) // 2, stream=stream,
                                             packed=k[f"{b}.conv_t1.weight"])
            for j, d in enumerate(DILATIONS):
                r = f"{b}.res_unit{j + 1}"
                y = fused_snake_conv1d(h, self._a(f"{r}.snake1.alpha"), p[f"{r}.conv1.weight"], p[f"{r}.conv1.bias"],
                                       padding=3 * d, dilation=d, stream=stream, packed=k[f"{r}.conv1.weight"])
                h = fused_snake_conv1d(y, self._a(f"{r}.snake2.alpha"), p[f"{r}.conv2.weight"], p[f"{r}.conv2.bias"],
                                       stream=stream, residual=h, packed=k[f"{r}.conv2.weight"])
        return fused_snake_conv1d(h, self._a("snake1.alpha"), p["conv2.weight"], p["conv2.bias"], padding=3,
                                  stream=stream, post="tanh", packed=k["conv2.weight"])

    def flops(self, T0: int, batch: int = 1) -> int:
        """Multiply-add flops (2 per MAC) of one forward over T0 latent frames."""
        cfg = self.config
        C = cfg["decoder_hidden_size"]
        T = T0
        f = 2 * cfg["hidden_size"] * C * 7 * T
        for i, s in enumerate(cfg["upsampling_ratios"]):
            cin, cout = C // 2 ** i, C // 2 ** (i + 1)
            T = T * s
            f += 2 * cin * cout * 2 * T  # two taps per output (kernel 2 s, stride s)
            f += 3 * (2 * cout * cout * 7 * T + 2 * cout * cout * T)
        f += 2 * (C // 2 ** len(cfg["upsampling_ratios"])) * 7 * T
        return f * batch


def decoder_bytes(dec: "DacDecoder", T0: int, batch: int = 1) -> int:
    """Algorithmic HBM bytes of one forward: every launch reads its fp32
    input (and residual) and writes its fp32 output once, and reads its
    packed weights (bf16 hi + lo, 4 bytes per weight) once."""
    cfg = dec.config
    C = cfg["decoder_hidden_size"]
    T = T0
    elems = cfg["hidden_size"] * T + C * T  # stem in, out
    for i, s in enumerate(cfg["upsampling_ratios"]):
        cin, cout = C // 2 ** i, C // 2 ** (i + 1)
        elems += cin * T + cout * T * s  # ConvTranspose in, out
        T *= s
        elems += 3 * 5 * cout * T  # per unit: k7 in, out; k1 in, residual, out
    elems += (C // 2 ** len(cfg["upsampling_ratios"])) * T + T  # output conv in, out
    weights = sum(v.numel() for k, v in dec.p.items() if k.endswith("weight"))
    return 4 * batch * elems + 4 * weights


def dac_residual_unit(x: torch.Tensor, alpha1, w1, b1, alpha2, w2, b2, dilation: int, stream=None) -> torch.Tensor:
    """x + conv2(snake2(conv1(snake1(x)))) (transformers DacResidualUnit):
    two launches, the residual add fused into the second's epilogue."""
    k = w1.shape[-1]
    y = fused_snake_conv1d(x, alpha1, w1, b1, padding=(k - 1) * dilation // 2, dilation=dilation, stream=stream)
    return fused_snake_conv1d(y, alpha2, w2, b2, stream=stream, residual=x)


def bench_dac_decoder(warmup: int = 2, reps: int = 3, frames: int = 862, seed: int = 0) -> dict:
    """Microseconds per second of audio for the whole 44.1 kHz decoder (one
    stream, `frames` latent frames = 10.0 s at 862), on device-resident
    synthetic weights and latent; CUDA events around `reps` forwards."""
    cfg = dac_decoder_config()
    dec = DacDecoder(init_decoder_params(cfg, seed=seed), cfg)
    latent = torch.randn(1, cfg["hidden_size"], frames, device="cuda",
                         generator=torch.Generator(device="cuda").manual_seed(seed + 1))
    for _ in range(warmup):
        audio = dec(latent)
    torch.cuda.synchronize()
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        audio = dec(latent)
    e.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(e) * 1e3 / reps
    hop = math.prod(cfg["upsampling_ratios"])
    seconds = frames * hop / 44100.0
    flops = dec.flops(frames)
    nbytes = decoder_bytes(dec, frames)
    if not torch.isfinite(audio).all():
        raise RuntimeError("DAC decoder produced non-finite audio")
    return {
        "metric": "DAC decoder µs per audio-sec",
        "value": round(us / seconds, 2),
        "unit": "us per audio-second",
        "us_per_pass": round(us, 1),
        "audio_seconds": round(seconds, 3),
        "realtime_factor": round(seconds / (us * 1e-6), 1),
        "useful_tflops": round(flops / (us * 1e-6) / 1e12, 1),
        "mma_tflops": round(3 * flops / (us * 1e-6) / 1e12, 1),
        "bytes": nbytes,
        "gbs": round(nbytes / (us * 1e-6) / 1e9, 1),
        "workload": "full 44.1 kHz DAC decoder (transformers DacDecoder layout): stem conv 1024->1536 k7, 4 blocks of "
                    "Snake+ConvTranspose1d (strides 8,8,4,2) and 3 residual units (Snake+Conv1d k7 d=1,3,9, "
                    "Snake+Conv1d k1 + residual), Snake+Conv1d 96->1 k7 + tanh; synthetic weights, fp32 in/out",
        "launches_per_pass": 2 + 4 + 24,
    }
