"""Copy the reference's frozen Mamba2 decode-step goldens into tests/golden/mamba_step.npz.

The reference checkout holds torch.save'd goldens for the decode-step ops
(tests/goldens/kernels/*.pt, sha256 in MANIFEST.json), made by
scripts/validation_harness.py against causal_conv1d 1.6.2.post1 and mamba_ssm
2.3.2.post1 on CUDA.  This script runs in the build container, checks each
file's sha256 against the manifest, loads it with torch.load(weights_only=True)
and stores every bf16 tensor as its uint16 bit pattern:

    python tests/golden/make_mamba_step_golden.py --reference PATH   (or SONATA_REFERENCE=PATH)

selective_state_update is listed in the manifest but its file is absent from
the checkout, so it has no golden here.  The GPU box never runs this script.
"""
from __future__ import annotations

import argparse
import os
import hashlib
import json
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent
OPS = ["causal_conv1d_update", "rmsnorm_gated", "layer_norm_fn", "layer_norm_fn_exit"]


def bits(t: torch.Tensor) -> np.ndarray:
    assert t.dtype == torch.bfloat16, t.dtype
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SONATA_REFERENCE"), required="SONATA_REFERENCE" not in os.environ,
                    help="path of the reference checkout (or set SONATA_REFERENCE)")
    args = ap.parse_args()
    gdir = Path(args.reference) / "tests" / "goldens" / "kernels"
    manifest = json.loads((gdir / "MANIFEST.json").read_text())
    out = {}
    for name in OPS:
        path = gdir / manifest[name]["file"]
        assert hashlib.sha256(path.read_bytes()).hexdigest() == manifest[name]["sha256"], name
        blob = torch.load(path, weights_only=True)
        for k, v in blob["inputs"].items():
            if torch.is_tensor(v):
                out[f"{name}__in__{k}"] = bits(v)
            elif v is not None:
                out[f"{name}__in__{k}"] = np.array(v)
        outs = blob["outputs"]
        for i, v in enumerate(outs if isinstance(outs, (list, tuple)) else [outs]):
            out[f"{name}__out{i}"] = bits(v)
        print(name, {k.split("__")[-1]: out[k].shape for k in out if k.startswith(name + "__")})
    np.savez_compressed(OUT / "mamba_step.npz", **out)
    print("wrote", OUT / "mamba_step.npz")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
