"""CPU restatements of the reference's hot-path algorithms (test infrastructure).

Every function cites the reference file:line it restates.  Floating-point
paths are numpy in float64 (inputs are the exact fp32 / bf16 values the kernels
see); the quantisation codes come from the plain-C restatement in
``quant_ref.c`` (bit-exact byte work), loaded through ctypes.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liboracle.so"
_lib = None


def build_c_oracle(force: bool = False) -> Path:
    """Compile quant_ref.c into oracle/_build/liboracle.so (gcc, IEEE fp32)."""
    src = _HERE / "quant_ref.c"
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        _LIB_PATH.parent.mkdir(parents=True, exist_ok=True)
        tmp = _LIB_PATH.with_suffix(f".{os.getpid()}.tmp")
        subprocess.check_call(["gcc", "-O2", "-fPIC", "-shared", "-std=c11",
                               "-fno-fast-math", "-ffp-contract=off", str(src), "-o", str(tmp), "-lm"])
        os.replace(tmp, _LIB_PATH)
    return _LIB_PATH


def _c():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(build_c_oracle()))
        P, L, I = ctypes.c_void_p, ctypes.c_long, ctypes.c_int
        lib.oracle_quant_int_rows.argtypes = [P, L, I, I, I, I, P, P]
        lib.oracle_quant_int_rows.restype = I
        lib.oracle_quant_e4m3_rows.argtypes = [P, L, I, I, P, P]
        lib.oracle_quant_e4m3_rows.restype = I
        lib.oracle_dequant_gemv.argtypes = [P, P, P, I, I, I, I, P]
        lib.oracle_gemv_bf16.argtypes = [P, L, P, I, I, I, P]
        lib.oracle_f32_to_e4m3.argtypes = [ctypes.c_float]
        lib.oracle_f32_to_e4m3.restype = ctypes.c_uint8
        lib.oracle_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        lib.oracle_e4m3_to_f32.restype = ctypes.c_float
        lib.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        lib.oracle_f32_to_bf16.restype = ctypes.c_uint16
        _lib = lib
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


# --------------------------------------------------------------------------
# bf16 helpers (bit patterns carried as uint16)
# --------------------------------------------------------------------------

def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(f: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 (torch's ``.to(torch.bfloat16)``)."""
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(f, dtype=np.float32))
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


# --------------------------------------------------------------------------
# GEMV (kernels/gemv.py, kernels/bench_gemv.py:48-55, validation_harness.py:356)
# --------------------------------------------------------------------------

def gemv_ref(x_bits: np.ndarray, w_bits: np.ndarray) -> np.ndarray:
    """y[M, N] = x[M, K] . W[N, K]^T accumulated in float64.

    Restates the fp32 ground truth ``x.float() @ W.float().t()`` of
    kernels/bench_gemv.py:49 and scripts/validation_harness.py:356, which every
    reference GEMV candidate (kernels/gemv.py:215-219) is gated against.
    """
    x = bf16_bits_to_f32(x_bits).astype(np.float64)
    w = bf16_bits_to_f32(w_bits).astype(np.float64)
    return x @ w.T


def rel_err_inf(out: np.ndarray, truth: np.ndarray) -> float:
    """max|out - truth| / max|truth| (kernels/bench_gemv.py:48-55)."""
    truth = np.asarray(truth, dtype=np.float64)
    return float(np.abs(np.asarray(out, np.float64) - truth).max() / max(np.abs(truth).max(), 1e-12))


def rel_rms(out: np.ndarray, truth: np.ndarray) -> float:
    """rel-RMS error of scripts/validation_harness.py:351,357."""
    truth = np.asarray(truth, dtype=np.float64)
    d = np.asarray(out, np.float64) - truth
    return float(np.sqrt((d ** 2).mean()) / np.sqrt((truth ** 2).mean()))


# --------------------------------------------------------------------------
# Weight-only quantisation (scripts/fake_quant.py:16-42)
# --------------------------------------------------------------------------

def quant_int_rows(w_bits: np.ndarray, bits: int = 8, group_size: int | None = None):
    """Codes and scales of ``fake_quantize_weights(w, bits, group_size)``.

    Returns (q int8 [N, K], scale fp32 [N, K // group]).  The dequantised
    weight of scripts/fake_quant.py:41 is ``q * scale`` in fp32 (see
    ``dequant_int``).
    """
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    N, K = w.shape
    g = K if group_size is None else int(group_size)
    q = np.empty((N, K), dtype=np.int8)
    s = np.empty((N, K // g), dtype=np.float32)
    rc = _c().oracle_quant_int_rows(_ptr(w), K, N, K, g, bits, _ptr(q), _ptr(s))
    if rc != 0:
        raise ValueError("group_size must divide K and bits must be in [2, 8]")
    return q, s


def dequant_int(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """fp32 ``q * scale`` (scripts/fake_quant.py:41), before the dtype cast."""
    N, K = q.shape
    G = scale.shape[1]
    return (q.astype(np.float32).reshape(N, G, K // G) * scale[:, :, None]).reshape(N, K)


def quant_e4m3_rows(w_bits: np.ndarray):
    """Per-row e4m3 codes + fp32 scales (scale = amax/448)."""
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    N, K = w.shape
    q = np.empty((N, K), dtype=np.uint8)
    s = np.empty((N,), dtype=np.float32)
    _c().oracle_quant_e4m3_rows(_ptr(w), K, N, K, _ptr(q), _ptr(s))
    return q, s


_E4M3_TABLE = None


def e4m3_decode(q: np.ndarray) -> np.ndarray:
    global _E4M3_TABLE
    if _E4M3_TABLE is None:
        _E4M3_TABLE = np.array([_c().oracle_e4m3_to_f32(i) for i in range(256)], dtype=np.float32)
    return _E4M3_TABLE[np.asarray(q, dtype=np.uint8)]


def f32_to_e4m3(v: np.ndarray) -> np.ndarray:
    f = _c().oracle_f32_to_e4m3
    flat = np.asarray(v, dtype=np.float32).ravel()
    return np.array([f(float(a)) for a in flat], dtype=np.uint8).reshape(np.shape(v))


def dequant_gemv_ref(x_bits: np.ndarray, q: np.ndarray, scale: np.ndarray, kind: str) -> np.ndarray:
    """Dequantise to fp32 then matmul (float64 accumulation): BASELINE config 3's oracle."""
    if kind == "int8":
        wdq = dequant_int(q, scale.reshape(q.shape[0], -1))
    elif kind == "e4m3":
        wdq = e4m3_decode(q) * scale.reshape(-1, 1).astype(np.float32)
    else:
        raise ValueError(kind)
    x = bf16_bits_to_f32(x_bits).astype(np.float64)
    return x @ wdq.astype(np.float64).T


# --------------------------------------------------------------------------
# BMM (kernels/bmm.py)
# --------------------------------------------------------------------------

def ssd_chunk_bmm_ref(C_bits: np.ndarray, B_bits: np.ndarray, seqlen: int, chunk: int) -> np.ndarray:
    """CB[b, c, g, i, j] = sum_d C[b, c*CH+i, g, d] * B[b, c*CH+j, g, d].

    Restates kernels/bmm.py:134-136 (einsum "bcigd,bcjgd->bcgij") with the
    masked semantics of kernels/bmm.py:205-212: rows at positions >= seqlen
    (the padded tail of a ragged last chunk) contribute zeros.  C, B are bf16
    bit patterns [BATCH, L, NGROUPS, DSTATE] with L >= seqlen.
    """
    BATCH, L, G, D = C_bits.shape
    nchunks = -(-seqlen // chunk)
    Cf = np.zeros((BATCH, nchunks * chunk, G, D), np.float64)
    Bf = np.zeros_like(Cf)
    Cf[:, :seqlen] = bf16_bits_to_f32(C_bits[:, :seqlen])
    Bf[:, :seqlen] = bf16_bits_to_f32(B_bits[:, :seqlen])
    Cc = Cf.reshape(BATCH, nchunks, chunk, G, D)
    Bc = Bf.reshape(BATCH, nchunks, chunk, G, D)
    return np.einsum("bcigd,bcjgd->bcgij", Cc, Bc)


def codebook_head_ref(hidden_bits: np.ndarray, w_bits: np.ndarray) -> np.ndarray:
    """logits[cb, b, n] = sum_k hidden[cb, b, k] * W[cb, k, n]  (float64).

    The multi-codebook logit head of BASELINE config 4 (no reference kernel;
    it is the per-codebook ``torch.bmm`` the survey's CPU probe times).
    hidden: [NCB, B, K] bf16 bits, W: [NCB, K, N] bf16 bits.
    """
    h = bf16_bits_to_f32(hidden_bits).astype(np.float64)
    w = bf16_bits_to_f32(w_bits).astype(np.float64)
    return np.matmul(h, w)


# --------------------------------------------------------------------------
# Snake + Conv1d (kernels/fused_snake_conv.py)
# --------------------------------------------------------------------------

def conv1d_output_length(input_length: int, kernel_size: int, stride: int, padding: int,
                         dilation: int) -> int:
    """kernels/fused_snake_conv.py:13-26 (PyTorch Conv1d output length)."""
    return (input_length + 2 * padding - dilation * (kernel_size - 1) - 1) // stride + 1


def snake_ref(x: np.ndarray, alpha: np.ndarray, eps: float = 1e-9) -> np.ndarray:
    """snake(v) = v + sin(alpha v)^2 / (alpha + eps), per input channel, float64.

    kernels/fused_snake_conv.py:275-277 (reference_snake_conv1d's activation).
    x: [B, C, T]; alpha: [C].
    """
    x = np.asarray(x, np.float64)
    a = np.asarray(alpha, np.float64).reshape(1, -1, 1)
    return x + np.sin(a * x) ** 2 / (a + eps)


def snake_conv1d_ref(x: np.ndarray, alpha: np.ndarray, weight: np.ndarray, bias: np.ndarray | None,
                     stride: int = 1, padding: int = 0, dilation: int = 1,
                     eps: float = 1e-9) -> np.ndarray:
    """Snake then Conv1d in float64 (kernels/fused_snake_conv.py:264-286).

    Zero padding is applied to the *activated* signal (F.conv1d's padding),
    which equals padding x because snake(0) == 0 (fused_snake_conv.py:240).
    weight: [Cout, Cin, K]; returns [B, Cout, Tout].
    """
    act = snake_ref(x, alpha, eps)
    Bn, Cin, T = act.shape
    Cout, Cw, K = weight.shape
    if Cw != Cin:
        raise ValueError("Only groups=1 is supported.")
    Tout = conv1d_output_length(T, K, stride, padding, dilation)
    padded = np.zeros((Bn, Cin, T + 2 * padding), np.float64)
    padded[:, :, padding:padding + T] = act
    w = np.asarray(weight, np.float64)
    y = np.zeros((Bn, Cout, Tout), np.float64)
    span = (Tout - 1) * stride + 1
    for k in range(K):
        seg = padded[:, :, k * dilation:k * dilation + span:stride]  # [B, Cin, Tout]
        y += np.einsum("oi,bit->bot", w[:, :, k], seg, optimize=True)
    if bias is not None:
        y += np.asarray(bias, np.float64).reshape(1, -1, 1)
    return y


def conv1d_ref(x: np.ndarray, weight: np.ndarray, bias: np.ndarray | None, stride: int = 1, padding: int = 0,
               dilation: int = 1) -> np.ndarray:
    """Plain Conv1d in float64 (F.conv1d semantics; the DAC decoder's stem
    conv1 has no Snake in front, transformers modeling_dac.py DacDecoder)."""
    x = np.asarray(x, np.float64)
    Bn, Cin, T = x.shape
    Cout, Cw, K = weight.shape
    if Cw != Cin:
        raise ValueError("Only groups=1 is supported.")
    Tout = conv1d_output_length(T, K, stride, padding, dilation)
    padded = np.zeros((Bn, Cin, T + 2 * padding), np.float64)
    padded[:, :, padding:padding + T] = x
    w = np.asarray(weight, np.float64)
    y = np.zeros((Bn, Cout, Tout), np.float64)
    span = (Tout - 1) * stride + 1
    for k in range(K):
        y += np.einsum("oi,bit->bot", w[:, :, k], padded[:, :, k * dilation:k * dilation + span:stride],
                       optimize=True)
    if bias is not None:
        y += np.asarray(bias, np.float64).reshape(1, -1, 1)
    return y


def conv_transpose1d_output_length(T: int, K: int, stride: int, padding: int) -> int:
    """torch ConvTranspose1d output length (dilation 1, output_padding 0)."""
    return (T - 1) * stride - 2 * padding + K


def snake_conv_transpose1d_ref(x: np.ndarray, alpha: np.ndarray, weight: np.ndarray, bias: np.ndarray | None,
                               stride: int, padding: int, eps: float = 1e-9) -> np.ndarray:
    """Snake then ConvTranspose1d in float64, by its definition: input j, tap
    k lands on output j * stride - padding + k (torch ConvTranspose1d,
    weight [Cin, Cout, K]; the DacDecoderBlock's snake1 -> conv_t1,
    transformers modeling_dac.py DacDecoderBlock.forward)."""
    act = snake_ref(x, alpha, eps)
    Bn, Cin, T = act.shape
    Cw, Cout, K = weight.shape
    if Cw != Cin:
        raise ValueError("Only groups=1 is supported.")
    Ty = conv_transpose1d_output_length(T, K, stride, padding)
    full = np.zeros((Bn, Cout, (T - 1) * stride + K), np.float64)
    w = np.asarray(weight, np.float64)
    for k in range(K):
        contrib = np.einsum("io,bit->bot", w[:, :, k], act, optimize=True)  # [B, Cout, T]
        full[:, :, k:k + (T - 1) * stride + 1:stride] += contrib
    y = full[:, :, padding:padding + Ty]
    if bias is not None:
        y = y + np.asarray(bias, np.float64).reshape(1, -1, 1)
    return y


def dac_residual_unit_ref(x: np.ndarray, p: dict, prefix: str, dilation: int, eps: float = 1e-9) -> np.ndarray:
    """x + conv2(snake2(conv1(snake1(x)))) (transformers modeling_dac.py
    DacResidualUnit.forward; conv1 k = 7 with padding 3 * dilation, conv2 k = 1,
    so the crop of its residual is 0).  p: the decoder's state dict (numpy)."""
    a1 = np.asarray(p[f"{prefix}.snake1.alpha"]).reshape(-1)
    a2 = np.asarray(p[f"{prefix}.snake2.alpha"]).reshape(-1)
    y = snake_conv1d_ref(x, a1, p[f"{prefix}.conv1.weight"], p[f"{prefix}.conv1.bias"], padding=3 * dilation,
                         dilation=dilation, eps=eps)
    y = snake_conv1d_ref(y, a2, p[f"{prefix}.conv2.weight"], p[f"{prefix}.conv2.bias"], eps=eps)
    return np.asarray(x, np.float64) + y


def dac_decoder_ref(latent: np.ndarray, p: dict, upsampling_ratios, eps: float = 1e-9) -> np.ndarray:
    """The DAC decoder (transformers modeling_dac.py DacDecoder.forward, the
    module layout of docs/dac_architecture.md:37-133): stem conv1 (k 7, pad 3),
    per block snake1 -> ConvTranspose1d (kernel 2 s, stride s, padding
    ceil(s / 2)) -> residual units with dilations 1, 3, 9, then snake1 ->
    conv2 (k 7, pad 3) -> tanh.  float64; p holds the state dict (numpy)."""
    h = conv1d_ref(latent, p["conv1.weight"], p["conv1.bias"], padding=3)
    for i, s in enumerate(upsampling_ratios):
        b = f"block.{i}"
        h = snake_conv_transpose1d_ref(h, np.asarray(p[f"{b}.snake1.alpha"]).reshape(-1), p[f"{b}.conv_t1.weight"],
                                       p[f"{b}.conv_t1.bias"], stride=s, padding=(s + 1) // 2, eps=eps)
        for j, d in enumerate((1, 3, 9)):
            h = dac_residual_unit_ref(h, p, f"{b}.res_unit{j + 1}", d, eps)
    h = snake_conv1d_ref(h, np.asarray(p["snake1.alpha"]).reshape(-1), p["conv2.weight"], p["conv2.bias"],
                         padding=3, eps=eps)
    return np.tanh(h)


# --------------------------------------------------------------------------
# Mamba2 decode-step ops (the reference's frozen goldens,
# tests/goldens/kernels/*.pt, made by scripts/validation_harness.py:58-115,
# 140-171 against causal_conv1d 1.6.2.post1 and mamba_ssm 2.3.2.post1,
# validation_harness.py:39).  float64 restatements of those libraries'
# published algorithms; bf16 inputs are given as float arrays.
# --------------------------------------------------------------------------

def _silu(v):
    return v / (1.0 + np.exp(-v))


def causal_conv1d_update_ref(x, conv_state, weight, bias, activation="silu"):
    """causal_conv1d_update (validation_harness.py:58-66,140-143): the state
    [B, D, W] shifts left by one step and takes x [B, D] as its newest column;
    y = sum_w state[:, :, w] * weight[:, w] + bias, then SiLU.  Returns
    (y, new_state)."""
    st = np.concatenate([np.asarray(conv_state, np.float64)[:, :, 1:],
                         np.asarray(x, np.float64)[:, :, None]], axis=2)
    y = np.einsum("bdw,dw->bd", st, np.asarray(weight, np.float64))
    if bias is not None:
        y = y + np.asarray(bias, np.float64)[None, :]
    if activation in ("silu", "swish"):
        y = _silu(y)
    return y, st


def rmsnorm_gated_ref(x, weight, bias, z, eps, group_size, norm_before_gate=False):
    """mamba_ssm rmsnorm_fn (validation_harness.py:91-101,153-156): with
    norm_before_gate False, x * SiLU(z) is RMS-normalised over groups of
    group_size, times weight (+ bias); with it True the gate follows the norm."""
    x = np.asarray(x, np.float64)
    zz = np.asarray(z, np.float64) if z is not None else None
    if zz is not None and not norm_before_gate:
        x = x * _silu(zz)
    shp = x.shape
    g = x.reshape(shp[:-1] + (shp[-1] // group_size, group_size))
    r = 1.0 / np.sqrt((g * g).mean(axis=-1, keepdims=True) + eps)
    y = (g * r).reshape(shp) * np.asarray(weight, np.float64)
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    if zz is not None and norm_before_gate:
        y = y * _silu(zz)
    return y


def layer_norm_fn_ref(x, weight, bias, residual=None, eps=1e-5, is_rms_norm=False):
    """mamba_ssm layer_norm_fn (validation_harness.py:104-114,159-171): the
    residual add happens first (its output is what prenorm returns), the norm
    runs on the unrounded sum.  Returns (out, residual_out)."""
    h = np.asarray(x, np.float64)
    if residual is not None:
        h = h + np.asarray(residual, np.float64)
    if is_rms_norm:
        y = h / np.sqrt((h * h).mean(axis=-1, keepdims=True) + eps)
    else:
        mu = h.mean(axis=-1, keepdims=True)
        y = (h - mu) / np.sqrt(((h - mu) ** 2).mean(axis=-1, keepdims=True) + eps)
    y = y * np.asarray(weight, np.float64)
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    return y, h


def selective_state_update_ref(state, x, dt, A, B, C, D=None, z=None, dt_bias=None, dt_softplus=False):
    """mamba_ssm selective_state_update (validation_harness.py:69-88,146-150):
    dt (+ dt_bias, softplus) per (head, dim); state = state * exp(dt * A) +
    dt * B * x; y = sum over d_state of state * C (+ D * x) (* SiLU(z)).  B, C
    [batch, ngroups, dstate] shared by nheads / ngroups heads.  Returns
    (y, new_state)."""
    st = np.asarray(state, np.float64)
    xx = np.asarray(x, np.float64)
    d = np.asarray(dt, np.float64)
    if dt_bias is not None:
        d = d + np.asarray(dt_bias, np.float64)
    if dt_softplus:
        d = np.where(d <= 20.0, np.log1p(np.exp(np.minimum(d, 20.0))), d)
    nh = st.shape[1]
    ng = np.asarray(B).shape[1]
    hg = nh // ng
    Bh = np.repeat(np.asarray(B, np.float64), hg, axis=1)  # [batch, nh, ds]
    Ch = np.repeat(np.asarray(C, np.float64), hg, axis=1)
    dA = np.exp(d[..., None] * np.asarray(A, np.float64)[None])
    st = st * dA + (d * xx)[..., None] * Bh[:, :, None, :]
    y = (st * Ch[:, :, None, :]).sum(axis=-1)
    if D is not None:
        y = y + xx * np.asarray(D, np.float64)
    if z is not None:
        y = y * _silu(np.asarray(z, np.float64))
    return y, st


def bf16_round(v) -> np.ndarray:
    """Round to the nearest bf16 value (ties to even), returned as float64."""
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(v, np.float32))).astype(np.float64)


def rotary_ref(x, pos: int, base: float = 10000.0):
    """Non-interleaved rotary embedding over the last dimension (the halves
    rotate by angle pos / base**(2i / D)), mamba_ssm MHA's decode rotary."""
    x = np.asarray(x, np.float64)
    D = x.shape[-1]
    inv = 1.0 / (base ** (np.arange(0, D, 2, dtype=np.float64) / D))
    c, s = np.cos(pos * inv), np.sin(pos * inv)
    x1, x2 = x[..., :D // 2], x[..., D // 2:]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)


def gqa_attention_ref(q, k, v):
    """One query per head over a cache: q [b, hq, d], k / v [b, hk, L, d],
    query head h reads KV head h // (hq / hk); softmax(q.k / sqrt(d)).v."""
    q, k, v = (np.asarray(t, np.float64) for t in (q, k, v))
    hq, hk = q.shape[1], k.shape[1]
    k = np.repeat(k, hq // hk, axis=1)
    v = np.repeat(v, hq // hk, axis=1)
    sc = np.einsum("bhd,bhld->bhl", q, k) / np.sqrt(q.shape[-1])
    sc = np.exp(sc - sc.max(axis=-1, keepdims=True))
    sc /= sc.sum(axis=-1, keepdims=True)
    return np.einsum("bhl,bhld->bhd", sc, v)


def zonos_decode_step_ref(p: dict, hidden, cfg: dict) -> np.ndarray:
    """One Zonos-hybrid decode token (mamba_ssm Block / Mamba2.step / MHA
    decode / GatedMLP, the layout of the reference's docs/architecture.md:
    5-30, 138-236) restated with the float64 op restatements above, rounding
    to bf16 wherever the bf16 model stores a tensor.  p: per-layer numpy
    arrays and states (``L{i}.*``), ``norm_f_w`` / ``norm_f_b``, ``head_W``
    [ncb, d, vocab]; cfg: d_inner, d_state, nheads, headdim, conv_dim,
    num_heads, num_heads_kv, head_dim, attn_layer_idx, n_layer, pos, eps.
    Returns fp64 logits [ncb, batch, vocab]; states in p are not modified."""
    r = bf16_round
    eps = cfg["eps"]
    h = r(hidden)
    res = None
    b = h.shape[0]
    di, ds, nh, hdim = cfg["d_inner"], cfg["d_state"], cfg["nheads"], cfg["headdim"]
    for i in range(cfg["n_layer"]):
        L = lambda k: p[f"L{i}.{k}"]
        out, hres = layer_norm_fn_ref(h, L("norm_w"), L("norm_b"), res, eps)
        h, res = r(out), r(hres)
        if i in cfg["attn_layer_idx"]:
            hq, hk, hd = cfg["num_heads"], cfg["num_heads_kv"], cfg["head_dim"]
            qkv = r(h @ L("in_proj").T)
            q = r(rotary_ref(qkv[:, :hq * hd].reshape(b, hq, hd), cfg["pos"]))
            k = r(rotary_ref(qkv[:, hq * hd:(hq + hk) * hd].reshape(b, hk, hd), cfg["pos"]))
            v = qkv[:, (hq + hk) * hd:].reshape(b, hk, hd)
            pos = cfg["pos"]
            kc = L("k_cache")[:, :, :pos + 1].copy()
            vc = L("v_cache")[:, :, :pos + 1].copy()
            kc[:, :, pos] = k
            vc[:, :, pos] = v
            o = r(gqa_attention_ref(q, kc, vc)).reshape(b, hq * hd)
            h = r(o @ L("out_proj").T)
            out, hres = layer_norm_fn_ref(h, L("norm2_w"), L("norm2_b"), res, eps)
            h, res = r(out), r(hres)
            f = r(h @ L("fc1").T)
            d = f.shape[1] // 2
            y = r(f[:, :d] * r(_silu(f[:, d:])))
            h = r(y @ L("fc2").T)
        else:
            zx = r(h @ L("in_proj").T)
            cd = cfg["conv_dim"]
            z, xBC, dt = zx[:, :di], zx[:, di:di + cd], zx[:, di + cd:]
            y, _ = causal_conv1d_update_ref(xBC, L("conv_state"), L("conv_w"), L("conv_b"), "silu")
            xBC = r(y)
            x = xBC[:, :di].reshape(b, nh, hdim)
            Bm = xBC[:, di:di + ds].reshape(b, 1, ds)
            Cm = xBC[:, di + ds:].reshape(b, 1, ds)
            dt_e = np.repeat(dt[:, :, None], hdim, axis=2)
            y, _ = selective_state_update_ref(L("ssm_state"), x, dt_e, L("A"), Bm, Cm, D=L("D_e"), z=None,
                                              dt_bias=L("dt_bias_e"), dt_softplus=True)
            y = r(y).reshape(b, di)
            y = r(rmsnorm_gated_ref(y, L("norm_mix_w"), None, z, eps, di, norm_before_gate=False))
            h = r(y @ L("out_proj").T)
    out, _ = layer_norm_fn_ref(h, p["norm_f_w"], p["norm_f_b"], res, eps)
    hf = r(out)
    return np.einsum("bk,ckn->cbn", hf, np.asarray(p["head_W"], np.float64))


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300))


__all__ = [n for n in dir() if not n.startswith("_")]
