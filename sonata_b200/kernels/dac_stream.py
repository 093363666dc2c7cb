"""Cached-convolution streaming DAC decoder: sample-exact chunked vocoding.

The reference vocodes a stream by overlap-save: every chunk re-decodes
CONTEXT latent frames it has already decoded and holds back a TAIL of
samples (scripts/streaming.py:191-238), which costs a 6x re-decode and is
only approximately equal to one-shot decoding.  Its documented fix
(docs/dac_profile.md:42,86) is a left-history cache per convolution; this
module is that fix on the fused B200 kernels.

Each convolution with a temporal kernel keeps an input buffer
[B, Cin, capacity] whose first ``h`` samples are the history it still needs
and whose next samples are the chunk's new input, written there directly by
the previous layer (the strided entry points take row and batch strides, so
no concatenation copy is made):

* a stride-1 convolution (kernel K, dilation d, padding p) holds input
  samples from ``n_out - p`` on (zeros before 0, which is the left padding);
  a 'valid' convolution over [history | new] yields exactly the outputs whose
  inputs have all arrived, ``(K-1)*d - p`` samples behind the input;
* the residual unit's k1 convolution adds the unit's input, read from its k7
  convolution's buffer ``p`` samples in;
* a ConvTranspose1d (kernel 2s, stride s, padding p) keeps the last input
  frame; over [last frame | new frames] with padding s it yields exactly the
  s samples of every new frame (the first chunk uses padding p and drops
  nothing else; the flush adds the final p samples);
* ``flush()`` appends each layer's right zero padding in turn.

Every output sample is the same dot product, in the same order, as in the
one-shot ``DacDecoder``, so the concatenated chunks equal the one-shot audio.
At the end of each chunk one launch (``sn_stream_shift``) moves every
buffer's kept samples to its front.  A chunk whose layer geometry repeats
(every chunk after the first few, for a fixed chunk size) replays a CUDA
graph of its launches.
"""
from __future__ import annotations

import ctypes
import math

import torch

from .. import _lib
from .dac import DILATIONS, DacDecoder


class _Conv:
    """One stride-1 convolution with a history buffer (or none for K == 1)."""

    def __init__(self, name, cin, cout, k, dil, pad, act, post, alpha, w, b, packed):
        self.name, self.cin, self.cout, self.k, self.dil, self.pad = name, cin, cout, k, dil, pad
        self.reach = (k - 1) * dil  # input samples beyond the first one an output needs
        self.act, self.post = act, post
        self.alpha, self.w, self.b, self.packed = alpha, w, b, packed
        self.buf = None
        self.h = 0


class _ConvT:
    def __init__(self, name, cin, cout, stride, alpha, w, b, packed):
        self.name, self.cin, self.cout, self.s = name, cin, cout, stride
        self.k = 2 * stride
        self.pad = (stride + 1) // 2
        self.alpha, self.w, self.b, self.packed = alpha, w, b, packed
        self.buf = None
        self.h = 0
        self.started = False


class StreamingDacDecoder:
    """Chunked, sample-exact version of ``DacDecoder`` for ``batch`` lockstep
    streams, on torch's current stream.  ``push(latent[B, hidden, n])`` returns the audio samples whose
    inputs have all arrived ([B, 1, m], a view of an internal buffer that the
    next call overwrites); ``flush()`` returns the rest.  Concatenated, the
    pieces equal ``decoder(latent)`` for the whole sequence.  At most
    ``max_chunk_frames`` latent frames per push."""

    def __init__(self, decoder: DacDecoder, max_chunk_frames: int = 64, batch: int = 1, use_graphs: bool = True,
                 lib=None):
        self.dec = decoder
        self.lib = lib if lib is not None else _lib.lib()
        self.B = int(batch)
        self.max_frames = int(max_chunk_frames)
        self.use_graphs = use_graphs
        p, k = decoder.p, decoder.packed
        cfg = decoder.config
        C = cfg["decoder_hidden_size"]
        a = decoder._a
        self.layers = []
        # stem: no Snake
        self.layers.append(("conv", _Conv("conv1", cfg["hidden_size"], C, 7, 1, 3, _lib.SN_ACT_NONE, _lib.SN_POST_NONE,
                                          None, p["conv1.weight"], p["conv1.bias"], k["conv1.weight"])))
        for i, s in enumerate(cfg["upsampling_ratios"]):
            cin, cout = C // 2 ** i, C // 2 ** (i + 1)
            bn = f"block.{i}"
            self.layers.append(("convt", _ConvT(f"{bn}.conv_t1", cin, cout, s, a(f"{bn}.snake1.alpha"),
                                                p[f"{bn}.conv_t1.weight"], p[f"{bn}.conv_t1.bias"],
                                                k[f"{bn}.conv_t1.weight"])))
            for j, d in enumerate(DILATIONS):
                r = f"{bn}.res_unit{j + 1}"
                c1 = _Conv(f"{r}.conv1", cout, cout, 7, d, 3 * d, _lib.SN_ACT_SNAKE, _lib.SN_POST_NONE,
                           a(f"{r}.snake1.alpha"), p[f"{r}.conv1.weight"], p[f"{r}.conv1.bias"], k[f"{r}.conv1.weight"])
                c2 = _Conv(f"{r}.conv2", cout, cout, 1, 1, 0, _lib.SN_ACT_SNAKE, _lib.SN_POST_NONE,
                           a(f"{r}.snake2.alpha"), p[f"{r}.conv2.weight"], p[f"{r}.conv2.bias"], k[f"{r}.conv2.weight"])
                self.layers.append(("unit", (c1, c2)))
        cl = C // 2 ** len(cfg["upsampling_ratios"])
        self.layers.append(("conv", _Conv("conv2", cl, 1, 7, 1, 3, _lib.SN_ACT_SNAKE, _lib.SN_POST_TANH,
                                          a("snake1.alpha"), p["conv2.weight"], p["conv2.bias"], k["conv2.weight"])))
        self.hop = math.prod(cfg["upsampling_ratios"])
        self._alloc()
        self._graphs = {}
        self._seen = set()
        self.reset()

    # -- buffers -----------------------------------------------------------
    def _alloc(self):
        dev = self.dec.p["conv1.weight"].device
        # new input samples a layer can receive in one call, at its own rate:
        # a push brings at most max_frames frames, and a flush releases every
        # layer's held-back samples on top, at most the decoder's whole
        # lookahead, counted here in latent frames
        n = self.max_frames + -(-self.lookahead_bound() // self.hop) + 2
        for kind, L in self.layers:
            if kind == "conv":
                L.cap = L.reach + n + L.reach + 8
                L.buf = torch.zeros(self.B, L.cin, L.cap, device=dev)
            elif kind == "convt":
                L.cap = 1 + n + 1
                L.buf = torch.zeros(self.B, L.cin, L.cap, device=dev)
                n = n * L.s
            else:
                c1, c2 = L
                c1.cap = c1.reach + n + c1.reach + 8
                c1.buf = torch.zeros(self.B, c1.cin, c1.cap, device=dev)
                c2.buf = torch.empty(self.B, c2.cin, n + c1.reach + 8, device=dev)  # conv1's output
        self.out = torch.empty(self.B, 1, n + 64, device=dev)

    def lookahead_bound(self) -> int:
        """Output samples the decoder can hold back: each layer's right reach
        (the samples after an output that it needs), scaled to the output
        rate, summed from the last layer back to the stem."""
        la, f = 0, 1
        for kind, L in reversed(self.layers):
            if kind == "conv":
                la += (L.reach - L.pad) * f
            elif kind == "unit":
                la += (L[0].reach - L[0].pad) * f
            else:
                la += L.pad * f
                f *= L.s
        return la

    def reset(self):
        """Start new streams: every history is the zero left padding."""
        for kind, L in self.layers:
            if kind == "conv":
                L.buf.zero_()
                L.h = L.pad
            elif kind == "convt":
                L.buf.zero_()
                L.h = 0
                L.started = False
            else:
                L[0].buf.zero_()
                L[0].h = L[0].pad
        self.frames_in = 0
        self.samples_out = 0
        self.finished = False

    @property
    def lookahead_samples(self) -> int:
        """Audio samples held back after any push: frames pushed * hop - samples returned."""
        return self.frames_in * self.hop - self.samples_out

    # -- launches ------------------------------------------------------------
    def _ws_args(self, L):
        return L.packed.data_ptr(), L.packed.numel()

    def _conv(self, L, x_len, dst, dst_off, dst_ld, dst_bs, residual=None, st=0):
        """'Valid' convolution over L.buf[..., :x_len] into dst (+ dst_off)."""
        out_len = x_len - L.reach
        if out_len <= 0:
            return 0
        buf = L.buf
        ws, wsn = self._ws_args(L)
        rptr, rbs, rld = 0, 0, 0
        if residual is not None:
            rbuf, roff = residual
            rptr = rbuf.data_ptr() + 4 * roff
            rbs, rld = rbuf.stride(0), rbuf.stride(1)
        _lib.check("sn_snake_conv1d_strided", self.lib.sn_snake_conv1d_strided(
            buf.data_ptr(), buf.stride(0), buf.stride(1), L.alpha.data_ptr() if L.alpha is not None else None,
            L.w.data_ptr(), L.b.data_ptr(), rptr or None, rbs, rld, dst.data_ptr() + 4 * dst_off, dst_bs, dst_ld,
            self.B, L.cin, L.cout, x_len, L.k, 1, 0, L.dil, ctypes.c_float(1e-9), L.act, L.post,
            _lib.SN_FLAG_PREPACKED, ws, wsn, st))
        return out_len

    def _convt(self, L, x_len, final, dst, dst_off, st=0):
        if not L.started:
            pad, ty = L.pad, x_len * L.s - (0 if final else L.pad)
        else:
            pad, ty = L.s, (x_len - 1) * L.s + (L.pad if final else 0)
        if ty <= 0 or x_len <= 0:
            return 0
        buf = L.buf
        ws, wsn = self._ws_args(L)
        _lib.check("sn_snake_conv_transpose1d_strided", self.lib.sn_snake_conv_transpose1d_strided(
            buf.data_ptr(), buf.stride(0), buf.stride(1), L.alpha.data_ptr(), L.w.data_ptr(), L.b.data_ptr(),
            dst.data_ptr() + 4 * dst_off, dst.stride(0), dst.stride(1), self.B, L.cin, L.cout, x_len, L.k, L.s, pad,
            ty, ctypes.c_float(1e-9), _lib.SN_FLAG_PREPACKED, ws, wsn, st))
        return ty

    def _run(self, n_new: int, final: bool, st: int):
        """Every layer once over the new input already in the stem's buffer;
        returns (samples written to self.out, shift table, new histories)."""
        shifts, new_h = [], []
        layers = self.layers
        n = n_new
        for li, (kind, L) in enumerate(layers):
            nxt = layers[li + 1] if li + 1 < len(layers) else None
            if nxt is None:
                dst, doff = self.out, 0
            else:
                nk, NL = nxt
                D = NL[0] if nk == "unit" else NL
                dst, doff = D.buf, D.h
            if kind == "conv":
                avail = L.h + n
                x_len = avail
                if final:
                    L.buf[..., avail:avail + L.reach - L.pad].zero_()
                    x_len = avail + L.reach - L.pad
                produced = self._conv(L, x_len, dst, doff, dst.stride(1), dst.stride(0), st=st)
                self._keep(L, avail, produced, shifts, new_h)
            elif kind == "convt":
                avail = L.h + n
                produced = self._convt(L, avail, final, dst, doff, st=st)
                if produced > 0 or avail > 0:
                    new_h.append((L, 1, True))
                    if avail > 1:
                        shifts.append((L.buf, avail - 1, 1))
            else:
                c1, c2 = L
                avail = c1.h + n
                x_len = avail
                if final:
                    c1.buf[..., avail:avail + c1.reach - c1.pad].zero_()
                    x_len = avail + c1.reach - c1.pad
                y = c2.buf
                produced = self._conv(c1, x_len, y, 0, y.stride(1), y.stride(0), st=st)
                if produced > 0:
                    self._conv(c2, produced, dst, doff, dst.stride(1), dst.stride(0), residual=(c1.buf, c1.pad), st=st)
                self._keep(c1, avail, produced, shifts, new_h)
            n = produced
        return n, shifts, new_h

    @staticmethod
    def _keep(L, avail, produced, shifts, new_h):
        keep = avail - produced
        new_h.append((L, keep, False))
        if produced > 0 and keep > 0:
            shifts.append((L.buf, produced, keep))

    def _shift(self, shifts, st):
        if not shifts:
            return
        arr = (_lib.ShiftDesc * len(shifts))()
        for i, (buf, src, ln) in enumerate(shifts):
            if ln > _lib.SN_SHIFT_MAX_LEN:
                raise RuntimeError(f"history of {ln} samples exceeds {_lib.SN_SHIFT_MAX_LEN}")
            arr[i] = _lib.ShiftDesc(buf.data_ptr(), buf.stride(0), buf.stride(1), buf.size(0), buf.size(1), src, ln)
        _lib.check("sn_stream_shift", self.lib.sn_stream_shift(arr, len(shifts), st))

    def _geometry(self, n_new, final):
        hs = []
        for kind, L in self.layers:
            if kind == "unit":
                hs.append(L[0].h)
            elif kind == "convt":
                hs.append((L.h, L.started))
            else:
                hs.append(L.h)
        return (n_new, final, tuple(hs))

    def _commit(self, new_h):
        for L, h, is_t in new_h:
            L.h = h
            if is_t:
                L.started = True

    def _stream(self) -> int:
        return torch.cuda.current_stream().cuda_stream if self.out.is_cuda else 0

    # -- public --------------------------------------------------------------
    def push(self, latent: torch.Tensor) -> torch.Tensor:
        if self.finished:
            raise RuntimeError("flush() was called; reset() before pushing more frames")
        if latent.dim() != 3 or latent.size(0) != self.B or latent.size(1) != self.layers[0][1].cin:
            raise ValueError(f"latent must be [{self.B}, {self.layers[0][1].cin}, n]")
        n = latent.size(2)
        if not 1 <= n <= self.max_frames:
            raise ValueError(f"1 <= frames per push <= {self.max_frames}, got {n}")
        st = self._stream()
        stem = self.layers[0][1]
        stem.buf[..., stem.h:stem.h + n].copy_(latent)
        key = self._geometry(n, False)
        if self.use_graphs and key in self._graphs:
            g, produced, new_h = self._graphs[key]
            g.replay()
        elif self.use_graphs and key in self._seen:
            # second time this geometry comes: capture it, then replay
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    produced, shifts, new_h = self._run(n, False, s.cuda_stream)
                    self._shift(shifts, s.cuda_stream)
            torch.cuda.current_stream().wait_stream(s)
            self._graphs[key] = (g, produced, new_h)
            g.replay()
        else:
            self._seen.add(key)
            produced, shifts, new_h = self._run(n, False, st)
            self._shift(shifts, st)
        self._commit(new_h)
        self.frames_in += n
        self.samples_out += produced
        return self.out[..., :produced]

    def flush(self) -> torch.Tensor:
        """Right-pad every layer in turn and return the remaining samples."""
        if self.finished:
            raise RuntimeError("flush() was already called")
        st = self._stream()
        produced, shifts, new_h = self._run(0, True, st)
        self._commit(new_h)
        self.finished = True
        self.samples_out += produced
        return self.out[..., :produced]


def decode_streaming(decoder: DacDecoder, latent: torch.Tensor, chunk_frames: int,
                     use_graphs: bool = True) -> torch.Tensor:
    """Decode latent [B, hidden, T0] in chunks of ``chunk_frames`` through a
    ``StreamingDacDecoder`` and concatenate the pieces (equals
    ``decoder(latent)``)."""
    sd = StreamingDacDecoder(decoder, max_chunk_frames=chunk_frames, batch=latent.size(0), use_graphs=use_graphs)
    pieces = []
    for f0 in range(0, latent.size(2), chunk_frames):
        pieces.append(sd.push(latent[..., f0:f0 + chunk_frames]).clone())
    pieces.append(sd.flush().clone())
    return torch.cat(pieces, dim=-1)
