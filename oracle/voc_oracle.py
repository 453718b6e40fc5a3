"""CPU oracle for the vocoder -- TEST INFRASTRUCTURE ONLY.

Only tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
use this module, and only as the checker or the timed CPU baseline.  The
product path (``nanovllm_dots_b200``) never imports it.

It restates, in torch on the CPU (float64 by default), the decode path of the
reference's BigVGAN ``AudioVAE`` (``nanovllm_dots/models/dots/native/vocoder/
bigvgan.py``), both the one-shot ``inference_from_latents(do_sample=False)``
(``bigvgan.py:800-813``) and the strict streaming decode (``bigvgan.py:
815-1065``):

* the front (``_decode_stream_latents``, ``bigvgan.py:858-873``): the 1x1
  ``post_proj`` conv, ``dec_mi_layer`` = Linear(L, 4L), a skip-connected LSTM
  of ``mi_num_layers`` layers (``SLSTM``, ``bigvgan.py:120-214``; gate order
  i, f, g, o; the stream carries (h, c) per layer), Linear(4L, L);
* the decoder (``Decoder.forward``, ``bigvgan.py:614-640``): ``conv_pre`` (a
  non-causal conv of 2*lookahead+1 taps), per stage a causal transposed conv
  (kernel 2u, stride u; ``layers.py:54-75``) and the mean of the stage's
  AMP resblocks (``bigvgan.py:329-540``), each a chain of alias-free SnakeBeta
  activations (``alias_free_act.py:12-48``, ``alias_free_resample.py``: x2
  upsampling by a 12-tap transposed conv scaled by 2 and trimmed causally,
  the activation ``x + 1/(exp(beta) + 1e-9) sin^2(exp(alpha) x)``, x2
  downsampling by a 12-tap filter after 11 samples of replicate padding on the
  left) and causal dilated convs with residual adds; then
  ``activation_post``, the causal 7-tap ``conv_post`` to one channel, tanh;
* the stream (``bigvgan.py:875-1065``): a fixed window of
  chunk + lookahead + left-context frames (the left context summed over the
  decoder's layers, ``bigvgan.py:700-760``), the new chunk appended after the
  valid frames or the window slid left, the decoder re-run over the whole
  window, and the samples of the frames that became stable emitted.

Convolutions are written as sums over taps of [T, Cin] x [Cin, Cout] products
on frames-first (channels-last) data, the formulation the CUDA kernels use.

Parity pin: ``tests/golden/make_golden_voc.py`` runs the reference's own
``AudioVAE`` (one-shot and streaming) on seeded weights and latents;
``tests/test_voc_oracle.py`` checks this module against those fixtures.
"""
from __future__ import annotations

import dataclasses
import math
from fractions import Fraction

import torch

EPS_SNAKE = 1e-9


# --------------------------------------------------------------------------- #
# Layers (frames-first: x is [B, T, C])                                        #
# --------------------------------------------------------------------------- #
def conv_taps(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None,
              offsets: list[int]) -> torch.Tensor:
    """y[t] = b + sum_j W[:, :, j] x[t + offsets[j]], x zero outside [0, T).
    ``w`` is the torch Conv1d layout [Cout, Cin, k]."""
    B, T, _ = x.shape
    y = torch.zeros(B, T, w.shape[0], dtype=x.dtype)
    for j, off in enumerate(offsets):
        lo, hi = max(0, -off), min(T, T - off)
        if lo >= hi:
            continue
        y[:, lo:hi] += x[:, lo + off:hi + off] @ w[:, :, j].t().to(x.dtype)
    if b is not None:
        y += b.to(x.dtype)
    return y


def conv_causal(x, w, b, dil: int = 1):
    """Causal conv: left padding dil*(k-1) (``layers.py:31-51``)."""
    k = w.shape[2]
    return conv_taps(x, w, b, [(j - (k - 1)) * dil for j in range(k)])


def conv_centered(x, w, b):
    """Non-causal conv with symmetric zero padding (k-1)/2 (conv_pre)."""
    k = w.shape[2]
    return conv_taps(x, w, b, [j - (k - 1) // 2 for j in range(k)])


def conv_transpose_causal(x, w, b, u: int):
    """Causal transposed conv, kernel 2u, stride u, the last u outputs trimmed
    (``layers.py:54-75``): y[t*u + r] = b + W[:, :, r]^T x[t] + W[:, :, r+u]^T
    x[t-1].  ``w`` is the torch ConvTranspose1d layout [Cin, Cout, 2u]."""
    B, T, _ = x.shape
    cout = w.shape[1]
    w = w.to(x.dtype)
    xprev = torch.cat([torch.zeros_like(x[:, :1]), x[:, :-1]], dim=1)
    y = torch.empty(B, T, u, cout, dtype=x.dtype)
    for r in range(u):
        y[:, :, r] = x @ w[:, :, r] + xprev @ w[:, :, r + u]
    y = y.reshape(B, T * u, cout)
    return y + b.to(x.dtype)


def snake_coeffs(alpha: torch.Tensor, beta: torch.Tensor | None):
    """(a, 1/(b + eps)) per channel in fp32, as the reference computes them on
    its log-scale parameters (``alias_free_act.py:96-101,158-163``); plain
    Snake passes beta=None and uses alpha for both."""
    a = torch.exp(alpha.float())
    bb = torch.exp(beta.float()) if beta is not None else a
    return a, 1.0 / (bb + EPS_SNAKE)


def alias_free_act(x, a, inv_b, f_up, f_down):
    """Anti-aliased (Snake)Beta: x2 upsample, activation, x2 downsample, all
    causal.  ``f_up``/``f_down`` are [12] (shared) or [C, 12] (per channel).

    up:   u[2m+p] = 2 sum_{q<6} x[m-q] f_up[2q+p]      (x[<0] = 0)
    act:  y = u + inv_b * sin(a u)^2
    down: out[m] = sum_{j<12} f_down[j] y[max(2m+j-11, 0)]
    """
    B, T, C = x.shape
    dt = x.dtype
    fu = f_up.reshape(-1, 12).to(dt).expand(C, 12)
    fd = f_down.reshape(-1, 12).to(dt).expand(C, 12)
    xp = torch.cat([torch.zeros(B, 5, C, dtype=dt), x], dim=1)      # xp[m+5] = x[m]
    u = torch.zeros(B, T, 2, C, dtype=dt)
    for p in range(2):
        for q in range(6):
            u[:, :, p] += xp[:, 5 - q:5 - q + T] * fu[:, 2 * q + p]
    u = 2.0 * u.reshape(B, 2 * T, C)
    y = u + inv_b.to(dt) * torch.sin(u * a.to(dt)) ** 2
    yp = torch.cat([y[:, :1].expand(B, 11, C), y], dim=1)          # yp[q+11] = y[q]
    out = torch.zeros(B, T, C, dtype=dt)
    for j in range(12):
        out += yp[:, j:j + 2 * T:2] * fd[:, j]
    return out


# --------------------------------------------------------------------------- #
# Model                                                                        #
# --------------------------------------------------------------------------- #
class VocOracle:
    """The decode path of one vocoder: ``w`` is its state dict (reference
    names), ``cfg`` a ``synthetic.VocConfig``."""

    def __init__(self, w: dict[str, torch.Tensor], cfg, dtype=torch.float64):
        self.w, self.cfg, self.dt = w, cfg, dtype
        self.nk = len(cfg.resblock_kernel_sizes)

    def _act(self, x, name):
        w = self.w
        a, ib = snake_coeffs(w[f"{name}.act.alpha"], w.get(f"{name}.act.beta"))
        return alias_free_act(x, a, ib, w[f"{name}.upsample.filter"],
                              w[f"{name}.downsample.lowpass.filter"])

    # ---- front: post_proj + Linear + LSTM + Linear
    def front(self, lat: torch.Tensor, h=None, c=None):
        """lat [B, F, L] -> (decoder input [B, F, L], h, c); h, c are
        [layers, B, 4L] (zeros when None)."""
        w, dt = self.w, self.dt
        x = lat.to(dt)
        x = x @ w["post_proj.weight"][:, :, 0].t().to(dt) + w["post_proj.bias"].to(dt)
        x = x @ w["dec_mi_layer.0.weight"].t().to(dt) + w["dec_mi_layer.0.bias"].to(dt)
        B, F, Hm = x.shape
        nl = self.cfg.mi_layers
        h = torch.zeros(nl, B, Hm, dtype=dt) if h is None else h.to(dt).clone()
        c = torch.zeros(nl, B, Hm, dtype=dt) if c is None else c.to(dt).clone()
        res = x
        for l in range(nl):
            wih = w[f"dec_mi_layer.1.lstm.weight_ih_l{l}"].to(dt)
            whh = w[f"dec_mi_layer.1.lstm.weight_hh_l{l}"].to(dt)
            bih = w[f"dec_mi_layer.1.lstm.bias_ih_l{l}"].to(dt)
            bhh = w[f"dec_mi_layer.1.lstm.bias_hh_l{l}"].to(dt)
            gx = x @ wih.t() + bih
            outs = []
            hl, cl = h[l], c[l]
            for f in range(F):
                gts = gx[:, f] + hl @ whh.t() + bhh
                i_, f_, g_, o_ = gts.chunk(4, dim=-1)
                cl = torch.sigmoid(f_) * cl + torch.sigmoid(i_) * torch.tanh(g_)
                hl = torch.sigmoid(o_) * torch.tanh(cl)
                outs.append(hl)
            h[l], c[l] = hl, cl
            x = torch.stack(outs, dim=1)
        x = x + res
        x = x @ w["dec_mi_layer.2.weight"].t().to(dt) + w["dec_mi_layer.2.bias"].to(dt)
        return x, h, c

    # ---- decoder
    def decode(self, z: torch.Tensor) -> torch.Tensor:
        """z [B, T, L] -> audio [B, T * hop]."""
        w, cfg, dt = self.w, self.cfg, self.dt
        x = conv_centered(z.to(dt), w["decoder.conv_pre.weight"], w["decoder.conv_pre.bias"])
        for i, u in enumerate(cfg.upsample_rates):
            x = conv_transpose_causal(x, w[f"decoder.ups.{i}.0.weight"],
                                      w[f"decoder.ups.{i}.0.bias"], u)
            xs = None
            for j, (ks, dil) in enumerate(zip(cfg.resblock_kernel_sizes, cfg.resblock_dilations)):
                r = f"decoder.resblocks.{i * self.nk + j}"
                h = x
                if cfg.resblock == "1":
                    for l, d in enumerate(dil):
                        t = self._act(h, f"{r}.activations.{2 * l}")
                        t = conv_causal(t, w[f"{r}.convs1.{l}.weight"], w[f"{r}.convs1.{l}.bias"], d)
                        t = self._act(t, f"{r}.activations.{2 * l + 1}")
                        t = conv_causal(t, w[f"{r}.convs2.{l}.weight"], w[f"{r}.convs2.{l}.bias"], 1)
                        h = t + h
                else:
                    for l, d in enumerate(dil[:2]):
                        t = self._act(h, f"{r}.activations.{l}")
                        t = conv_causal(t, w[f"{r}.convs.{l}.weight"], w[f"{r}.convs.{l}.bias"], d)
                        h = t + h
                xs = h if xs is None else xs + h
            x = xs / self.nk
        x = self._act(x, "decoder.activation_post")
        x = conv_causal(x, w["decoder.conv_post.weight"], w.get("decoder.conv_post.bias"), 1)
        x = torch.tanh(x) if cfg.use_tanh else x.clamp(-1.0, 1.0)
        return x[..., 0]

    def inference(self, lat: torch.Tensor) -> torch.Tensor:
        """One-shot: latents [B, T, L] -> audio [B, T * hop]
        (``inference_from_latents(do_sample=False)``)."""
        z, _, _ = self.front(lat)
        return self.decode(z)


# --------------------------------------------------------------------------- #
# Streaming                                                                    #
# --------------------------------------------------------------------------- #
def stream_left_context(cfg) -> int:
    """Frames of left context the decoder's causal layers need
    (``Decoder._stream_left_context``, ``bigvgan.py:700-722``), summed exactly
    in fractions of a frame and rounded up."""
    act = (12 - 1 + 12 - 1 + 2 - 1) // 2                   # one alias-free activation
    left = Fraction((2 * cfg.lookahead + 1 - 1) // 2)      # conv_pre's padding
    scale = Fraction(1)
    for u in cfg.upsample_rates:
        left += scale * 1                                  # causal transposed conv
        scale /= u
        stage = 0
        for ks, dil in zip(cfg.resblock_kernel_sizes, cfg.resblock_dilations):
            if cfg.resblock == "1":
                ctx = sum(act + d * (ks - 1) + act + (ks - 1) for d in dil)
            else:
                ctx = sum(act + d * (ks - 1) for d in dil[:2])
            stage = max(stage, ctx)
        left += scale * stage
    left += scale * act + scale * 6                        # activation_post, conv_post
    return math.ceil(left)


def stream_window(cfg, chunk: int) -> int:
    """``Decoder.stream_window_size`` (``bigvgan.py:724-733``)."""
    if chunk < 1:
        raise ValueError(f"chunk_size must be >= 1, got {chunk}.")
    return chunk + cfg.lookahead + stream_left_context(cfg)


@dataclasses.dataclass
class OracleStream:
    """One request's stream: LSTM state, decoder window [W, L], frame counts."""
    h: torch.Tensor
    c: torch.Tensor
    window: torch.Tensor
    chunk: int
    total: int = 0
    emitted: int = 0


def stream_init(voc: VocOracle, chunk: int) -> OracleStream:
    cfg, dt = voc.cfg, voc.dt
    Hm = 4 * cfg.latent_dim
    W = stream_window(cfg, chunk)
    z = torch.zeros(cfg.mi_layers, 1, Hm, dtype=dt)
    return OracleStream(z.clone(), z.clone(), torch.zeros(W, cfg.latent_dim, dtype=dt), chunk)


def window_append(window: torch.Tensor, valid: int, new: torch.Tensor) -> torch.Tensor:
    """``_append_stream_decoder_input_tensor`` (``bigvgan.py:887-928``): the
    chunk goes after the ``valid`` frames; the window keeps its last W frames;
    positions past the valid count are zero."""
    W, F = window.shape[0], new.shape[0]
    if F >= W:
        raise ValueError(f"decoder window size {W} must be larger than chunk_size {F}.")
    valid = min(max(valid, 0), W)
    seq = torch.cat([window[:valid], new.to(window.dtype)], dim=0)
    seq = seq[-W:]
    out = torch.zeros_like(window)
    out[:seq.shape[0]] = seq
    return out


def _slice(voc: VocOracle, st: OracleStream, audio: torch.Tensor, final: bool) -> torch.Tensor:
    """``_slice_stream_audio_window`` (``bigvgan.py:1005-1035``)."""
    hop = voc.cfg.hop
    stable = st.total if final else max(0, st.total - voc.cfg.lookahead)
    if stable <= st.emitted:
        return audio[:0]
    W = st.window.shape[0]
    start = st.total - min(st.total, W)
    if st.emitted < start:
        raise RuntimeError("Decoder stream window is too short for fixed-graph decoding.")
    a, b = (st.emitted - start) * hop, (stable - start) * hop
    st.emitted = stable
    return audio[a:b]


def stream_step(voc: VocOracle, st: OracleStream, lat: torch.Tensor) -> torch.Tensor:
    """One chunk lat [F, L] -> the newly stable samples (``stream_step``,
    ``bigvgan.py:1037-1046``)."""
    if lat.shape[0] != st.chunk:
        raise ValueError(f"Streaming chunk_size must stay fixed at {st.chunk}, got {lat.shape[0]}.")
    z, st.h, st.c = voc.front(lat[None], st.h, st.c)
    st.window = window_append(st.window, min(st.total, st.window.shape[0]), z[0])
    st.total += st.chunk
    audio = voc.decode(st.window[None])[0]
    return _slice(voc, st, audio, final=False)


def stream_flush(voc: VocOracle, st: OracleStream) -> torch.Tensor:
    """``stream_flush`` (``bigvgan.py:1048-1050``)."""
    audio = voc.decode(st.window[None])[0]
    return _slice(voc, st, audio, final=True)
