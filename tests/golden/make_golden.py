"""Freeze the reference's own outputs on seeded inputs as small .npz fixtures.

Run in the build container, where the reference checkout is importable:

    python tests/golden/make_golden.py --reference PATH   (or SONATA_REFERENCE=PATH)

It imports the reference's Python modules directly --
``kernels/fused_snake_conv.py`` (reference_snake_conv1d, explicit_snake_conv1d,
conv1d_output_length), ``scripts/fake_quant.py`` (fake_quantize_weights) and
``kernels/gemv.py`` / ``kernels/bmm.py`` for their module-level contracts --
and runs their torch CPU paths.  The BMM oracle is the einsum that
kernels/bmm.py:134-136 and :205-212 evaluate inline inside test_bmm /
test_bmm_ragged; it is re-evaluated here with the same expression.  The GPU box
never runs this script: it only reads the committed fixtures.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

OUT = Path(__file__).resolve().parent


def bits(t: torch.Tensor) -> np.ndarray:
    assert t.dtype == torch.bfloat16
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SONATA_REFERENCE"), required="SONATA_REFERENCE" not in os.environ,
                    help="path of the reference checkout (or set SONATA_REFERENCE)")
    args = ap.parse_args()
    ref = Path(args.reference)
    sys.path.insert(0, str(ref / "kernels"))
    sys.path.insert(0, str(ref / "scripts"))
    import fake_quant  # scripts/fake_quant.py
    import fused_snake_conv as fsc  # kernels/fused_snake_conv.py

    torch.set_num_threads(4)

    # ---------------- fake-quant (scripts/fake_quant.py:16-42) ----------------
    g = torch.Generator().manual_seed(0)
    W = (torch.randn(48, 256, generator=g) * 0.02).to(torch.bfloat16)
    W[5] = 0                                    # dead row -> clamp_min(1e-8) path
    W[7, :8] = torch.tensor([3.0, -3.0, 1.5, -0.75, 2.99, 0.0117, -0.0117, 0.5])
    W[9] = (torch.randn(256, generator=g) * 40).to(torch.bfloat16)   # wide row
    fq = {
        "w": bits(W),
        "int8_rows_bf16": bits(fake_quant.fake_quantize_weights(W, 8, None)),
        "int8_rows_f32": fake_quant.fake_quantize_weights(W.float(), 8, None).numpy(),
        "int8_g64_f32": fake_quant.fake_quantize_weights(W.float(), 8, 64).numpy(),
        "int4_rows_f32": fake_quant.fake_quantize_weights(W.float(), 4, None).numpy(),
        "int4_g64_f32": fake_quant.fake_quantize_weights(W.float(), 4, 64).numpy(),
    }
    # e4m3 per-row (torch's float8_e4m3fn conversion)
    wf = W.float()
    amax = wf.abs().amax(dim=-1, keepdim=True).clamp_min(1e-8)
    s8 = amax / 448.0
    q8 = (wf / s8).to(torch.float8_e4m3fn)
    fq["e4m3_codes"] = q8.view(torch.uint8).numpy().copy()
    fq["e4m3_scale"] = s8.squeeze(1).numpy().copy()
    fq["e4m3_dequant_f32"] = (q8.float() * s8).numpy()
    sweep = torch.cat([
        torch.linspace(-500, 500, 4001),
        torch.tensor([448.0, 449.0, 463.99, 464.0, 464.01, 480.0, -464.0, 2.0 ** -6, 2.0 ** -7,
                      2.0 ** -9, 2.0 ** -10, 2.0 ** -10 * 1.0001, 3 * 2.0 ** -10, 1e-3,
                      0.0, -0.0, 1e-30, 17.0, 18.0, 19.0, 0.9375, 0.96875]),
        torch.randn(2000, generator=g) * 4,
    ])
    fq["e4m3_sweep_in"] = sweep.numpy()
    fq["e4m3_sweep_codes"] = sweep.to(torch.float8_e4m3fn).view(torch.uint8).numpy().copy()
    np.savez_compressed(OUT / "fake_quant.npz", **fq)

    # ---------------- GEMV (F.linear; kernels/bench_gemv.py:48-55) ----------------
    g = torch.Generator().manual_seed(0)
    Wg = (torch.randn(96, 512, generator=g) * 0.02).to(torch.bfloat16)
    xg = torch.randn(2, 512, generator=g).to(torch.bfloat16)
    np.savez_compressed(
        OUT / "gemv.npz", w=bits(Wg), x=bits(xg),
        y_linear_bf16=bits(F.linear(xg, Wg)),
        y_truth_f32=(xg.float() @ Wg.float().t()).numpy())

    # ---------------- SSD chunk BMM (kernels/bmm.py:119-240) ----------------
    g = torch.Generator().manual_seed(0)
    BATCH, SEQLEN, NG, DS, CH = 2, 96, 2, 32, 32
    NCH = SEQLEN // CH
    C = torch.randn(BATCH, SEQLEN, NG, DS, generator=g).to(torch.bfloat16)
    B = torch.randn(BATCH, SEQLEN, NG, DS, generator=g).to(torch.bfloat16)
    CB = torch.einsum("bcigd,bcjgd->bcgij",
                      C.reshape(BATCH, NCH, CH, NG, DS).float(), B.reshape(BATCH, NCH, CH, NG, DS).float())
    # ragged: valid length 70 inside a padded, poisoned 96-row buffer (bmm.py:186-212)
    SEQ_R = 70
    Cr, Br = C.clone(), B.clone()
    Cr[:, SEQ_R:] = 7.0
    Br[:, SEQ_R:] = 7.0
    Cm, Bm = Cr.clone(), Br.clone()
    Cm[:, SEQ_R:] = 0
    Bm[:, SEQ_R:] = 0
    CBr = torch.einsum("bcigd,bcjgd->bcgij",
                       Cm.reshape(BATCH, NCH, CH, NG, DS).float(), Bm.reshape(BATCH, NCH, CH, NG, DS).float())
    np.savez_compressed(OUT / "bmm.npz", C=bits(C), B=bits(B), CB=CB.numpy(),
                        C_ragged=bits(Cr), B_ragged=bits(Br), CB_ragged=CBr.numpy(),
                        dims=np.array([BATCH, SEQLEN, NG, DS, CH, SEQ_R]))

    # ---------------- Snake + Conv1d (kernels/fused_snake_conv.py) ----------------
    cases = {}
    # the reference's own self-test case (fused_snake_conv.py:288-305)
    torch.manual_seed(42)
    x = torch.randn(2, 4, 8)
    alpha = torch.rand(4) * 2 + 0.3
    w = torch.randn(3, 4, 3)
    b = torch.randn(3)
    cases["selftest"] = (x, alpha, w, b, 1, 1, 1)
    g = torch.Generator().manual_seed(0)
    for d in (1, 3, 9):
        C_ = 16
        x = torch.randn(1, C_, 100, generator=g)
        alpha = torch.rand(C_, generator=g) + 0.5
        w = torch.randn(C_, C_, 7, generator=g) / (7 * C_) ** 0.5
        b = torch.randn(C_, generator=g)
        cases[f"same_d{d}"] = (x, alpha, w, b, 1, 3 * d, d)
    x = torch.randn(2, 8, 37, generator=g)
    alpha = torch.rand(8, generator=g) * 2 + 0.3
    w = torch.randn(5, 8, 4, generator=g)
    b = torch.randn(5, generator=g)
    cases["stride2_pad1_d2"] = (x, alpha, w, b, 2, 1, 2)
    x = torch.randn(1, 6, 50, generator=g) * 8      # large |alpha x|: sin precision
    alpha = torch.rand(6, generator=g) * 2 + 0.3
    w = torch.randn(6, 6, 7, generator=g) / 6.5
    b = torch.randn(6, generator=g)
    cases["large_x"] = (x, alpha, w, b, 1, 3, 1)
    sc = {}
    for name, (x, alpha, w, b, s, p, d) in cases.items():
        sc[f"{name}__x"] = x.numpy()
        sc[f"{name}__alpha"] = alpha.numpy()
        sc[f"{name}__w"] = w.numpy()
        sc[f"{name}__b"] = b.numpy()
        sc[f"{name}__spd"] = np.array([s, p, d])
        sc[f"{name}__y_reference"] = fsc.reference_snake_conv1d(x, alpha, w, b, stride=s, padding=p,
                                                                 dilation=d).numpy()
        sc[f"{name}__y_explicit"] = fsc.explicit_snake_conv1d(x, alpha, w, b, stride=s, padding=p,
                                                               dilation=d).numpy()
    ol = []
    for (L, K, s, p, d) in [(100, 7, 1, 3, 1), (100, 7, 1, 27, 9), (37, 4, 2, 1, 2), (8, 3, 1, 1, 1),
                            (5, 7, 1, 0, 1), (441344, 7, 1, 9, 3), (10, 3, 3, 0, 1)]:
        ol.append([L, K, s, p, d, fsc.conv1d_output_length(L, K, s, p, d)])
    sc["output_length_cases"] = np.array(ol)
    np.savez_compressed(OUT / "snake_conv.npz", **sc)

    for f in sorted(OUT.glob("*.npz")):
        print(f"{f.name}: {f.stat().st_size} bytes")
    return 0


if __name__ == "__main__":
    sys.exit(main())
