"""B200 vocoder: the decode path of the dots.tts BigVGAN ``AudioVAE``
(``nanovllm_dots/models/dots/native/vocoder/bigvgan.py``) on sm_100a, for
many requests per call.

``B200Vocoder`` has the methods of ``AudioVAE`` that the engine calls through
``DotsModel`` (``native/model.py:204-218``): ``inference_from_latents`` (one
shot), ``init_stream_state``, ``stream_step`` and ``stream_flush`` (strict
streaming), plus ``hop_size`` and ``sample_rate``.  Assigning one to
``engine.dots.vocoder`` (``install_vocoder``) routes the engine's
``vocode``/``_vocode_stream_step``/``_vocode_flush`` (``engine.py:825-852``)
through the CUDA path, and replaces ``step_stream`` with
``batched_step_stream``, which gives the step's vocoder work to the batched
calls.  The batched forms, ``decode_batch`` and
``stream_step_many``/``stream_flush_many``, serve every request of a tick in
one call: the reference runs one request at a time.

Every call goes through the C ABI (``include/dvoc.h``): the front (post_proj,
Linear, LSTM, Linear) in fp32, every decoder convolution on the tcgen05 tensor
cores with fp16 operands (the 10-bit mantissa of tf32) and fp32 accumulation,
activations, conv_post and tanh in fp32.  There is no other path: without the library every call raises.
"""
from __future__ import annotations

import ctypes
import dataclasses

import torch

from . import _lib
from .synthetic import VocConfig


def _pad32(c: int) -> int:
    return (c + 31) // 32 * 32


def dvoc_config(cfg: VocConfig, max_batch: int, max_frames: int) -> _lib.DvocConfig:
    c = _lib.DvocConfig()
    c.latent_dim = cfg.latent_dim
    c.initial_channels = cfg.initial_channels
    c.num_stages = len(cfg.upsample_rates)
    for i, u in enumerate(cfg.upsample_rates):
        c.upsample_rates[i] = u
    c.num_kernels = len(cfg.resblock_kernel_sizes)
    for j, (k, d) in enumerate(zip(cfg.resblock_kernel_sizes, cfg.resblock_dilations)):
        c.resblock_kernel_sizes[j] = k
        for l in range(3):
            c.resblock_dilations[j][l] = d[l] if l < len(d) else 1
    c.resblock_type = int(cfg.resblock)
    c.mi_layers = cfg.mi_layers
    c.lookahead = cfg.lookahead
    c.use_tanh = int(cfg.use_tanh)
    c.max_batch = max_batch
    c.max_frames = max_frames
    return c


def _act_block(sd: dict, name: str, c: int, activation: str) -> torch.Tensor:
    """[26 * Cp]: exp(alpha), 1/(exp(beta)+1e-9), up filter [Cp][12], down filter
    [Cp][12] of one alias-free activation (``alias_free_act.py:90-163``)."""
    cp = _pad32(c)
    a = torch.exp(sd[f"{name}.act.alpha"].float())
    bsrc = sd[f"{name}.act.beta"] if activation == "snakebeta" else sd[f"{name}.act.alpha"]
    ib = 1.0 / (torch.exp(bsrc.float()) + 1e-9)
    out = torch.zeros(26, cp)
    out[0, :c] = a
    out[1, :c] = ib
    fu = sd[f"{name}.upsample.filter"].float().reshape(-1, 12).expand(c, 12)
    fd = sd[f"{name}.downsample.lowpass.filter"].float().reshape(-1, 12).expand(c, 12)
    flat = out.reshape(-1)
    flat[2 * cp:2 * cp + 12 * c] = fu.reshape(-1)
    flat[14 * cp:14 * cp + 12 * c] = fd.reshape(-1)
    return flat


def pack_voc_weights(sd: dict, cfg: VocConfig, device=None) -> dict[str, torch.Tensor]:
    """The reference state dict (after ``remove_weight_norm``) in the layouts of
    ``DvocWeights`` (``include/dvoc.h``), as fp32 tensors on ``device``."""
    L, Hm = cfg.latent_dim, 4 * cfg.latent_dim
    Lp = _pad32(L)
    f = lambda k: sd[k].detach().float().cpu()
    w: dict[str, torch.Tensor] = {
        "post_w": f("post_proj.weight")[:, :, 0].contiguous(),
        "post_b": f("post_proj.bias"),
        "mi_in_w": f("dec_mi_layer.0.weight"), "mi_in_b": f("dec_mi_layer.0.bias"),
        "mi_out_w": f("dec_mi_layer.2.weight"), "mi_out_b": f("dec_mi_layer.2.bias"),
    }
    for kind in ("w_ih", "w_hh", "b_ih", "b_hh"):
        w[f"lstm_{kind}"] = torch.stack([
            f(f"dec_mi_layer.1.lstm.{'weight' if kind[0] == 'w' else 'bias'}_{kind[2:]}_l{l}")
            for l in range(cfg.mi_layers)])
    convs, biases = [], []

    def conv(name: str, cin: int):
        wt = f(f"{name}.weight")                   # [Cout, Cin, k]
        cout, _, k = wt.shape
        cp, cinp = _pad32(cout), _pad32(cin)
        dst = torch.zeros(cp, k, cinp)
        dst[:cout, :, :cin] = wt.permute(0, 2, 1)
        convs.append(dst.reshape(-1))
        b = torch.zeros(cp)
        b[:cout] = f(f"{name}.bias")
        biases.append(b)

    conv("decoder.conv_pre", L)
    nk = len(cfg.resblock_kernel_sizes)
    for i, u in enumerate(cfg.upsample_rates):
        cin, cout = cfg.stage_channels(i - 1), cfg.stage_channels(i)
        cinp, cp = _pad32(cin), _pad32(cout)
        wt = f(f"decoder.ups.{i}.0.weight")        # [Cin, Cout, 2u]
        dst = torch.zeros(u, cp, 2, cinp)
        for r in range(u):
            dst[r, :cout, 0, :cin] = wt[:, :, r + u].t()   # tap 0: frame t-1
            dst[r, :cout, 1, :cin] = wt[:, :, r].t()       # tap 1: frame t
        convs.append(dst.reshape(-1))
        b = torch.zeros(u, cp)
        b[:, :cout] = f(f"decoder.ups.{i}.0.bias")
        biases.append(b.reshape(-1))
        for j, dil in enumerate(cfg.resblock_dilations):
            r = f"decoder.resblocks.{i * nk + j}"
            if cfg.resblock == "1":
                for l in range(len(dil)):
                    conv(f"{r}.convs1.{l}", cout)
                    conv(f"{r}.convs2.{l}", cout)
            else:
                for l in range(2):
                    conv(f"{r}.convs.{l}", cout)
    acts = []
    per = 6 if cfg.resblock == "1" else 2
    for i in range(len(cfg.upsample_rates)):
        for j in range(nk):
            for a in range(per):
                acts.append(_act_block(sd, f"decoder.resblocks.{i * nk + j}.activations.{a}",
                                       cfg.stage_channels(i), cfg.activation))
    cl = cfg.stage_channels(len(cfg.upsample_rates) - 1)
    acts.append(_act_block(sd, "decoder.activation_post", cl, cfg.activation))
    w["conv_w"] = torch.cat(convs).to(torch.float16)
    w["conv_b"] = torch.cat(biases)
    w["act"] = torch.cat(acts)
    pw = torch.zeros(7, _pad32(cl))
    pw[:, :cl] = f("decoder.conv_post.weight")[0].t()
    w["post_conv_w"] = pw
    if cfg.use_bias_at_final:
        w["post_conv_b"] = f("decoder.conv_post.bias").reshape(1)
    dev = torch.device("cuda") if device is None else torch.device(device)
    return {k: v.contiguous().to(dev) for k, v in w.items()}


@dataclasses.dataclass
class B200StreamState:
    """One request's stream (``BigVGANStreamState``, ``bigvgan.py:20-31``): the
    LSTM state [mi_layers, 4L] (h, c), the decoder window [W, L] and the
    frame counts."""
    h: torch.Tensor
    c: torch.Tensor
    window: torch.Tensor
    chunk: int
    total: int = 0
    emitted: int = 0


class B200Vocoder:
    """AudioVAE decode on the B200 (see the module docstring).

    sd          the vocoder state dict (reference names, after remove_weight_norm)
    cfg         its shape (``synthetic.VocConfig``)
    max_batch   most requests per call
    max_frames  most latent frames per call (an utterance, or a stream window)
    """

    def __init__(self, sd: dict, cfg: VocConfig, max_batch: int = 64, max_frames: int = 64,
                 device=None):
        self.cfg = cfg
        self.device = torch.device("cuda") if device is None else torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("B200Vocoder needs a CUDA device")
        self.max_batch, self.max_frames = max_batch, max_frames
        self.hop_size = cfg.hop
        self.sample_rate = cfg.sample_rate
        self.lookahead = cfg.lookahead
        self.L, self.Hm = cfg.latent_dim, 4 * cfg.latent_dim
        L = _lib.lib()
        self._cfg = dvoc_config(cfg, max_batch, max_frames)
        with torch.cuda.device(self.device):
            self.w = pack_voc_weights(sd, cfg, self.device)
            sizes = {"conv_w": L.dvoc_conv_floats(ctypes.byref(self._cfg)),
                     "conv_b": L.dvoc_bias_floats(ctypes.byref(self._cfg)),
                     "act": L.dvoc_act_floats(ctypes.byref(self._cfg))}
            for k, n in sizes.items():
                if n == 0:
                    raise ValueError(f"unsupported vocoder configuration: {cfg}")
                if self.w[k].numel() != n:
                    raise RuntimeError(f"packed {k} has {self.w[k].numel()} floats, the library expects {n}")
            wt = _lib.DvocWeights()
            for f in _lib.VOC_WEIGHT_FIELDS:
                setattr(wt, f, _lib.ptr(self.w.get(f)))
            self._wt = wt
            h = ctypes.c_void_p()
            _lib.check(L.dvoc_create(ctypes.byref(self._cfg), ctypes.byref(wt), ctypes.byref(h)),
                       "dvoc_create")
            self._h = h
            self.ws = torch.zeros(L.dvoc_workspace_size(h), dtype=torch.uint8, device=self.device)
        self.left_context = L.dvoc_stream_left_context(ctypes.byref(self._cfg))

    # ------------------------------------------------------------------ core call
    def batch(self, n: int, frames: int, window: int, audio: torch.Tensor, latents=None,
              lengths=None, h=None, c=None, windows=None, valid=None) -> _lib.DvocBatch:
        """The ``DvocBatch`` of one call over caller-owned device tensors."""
        b = _lib.DvocBatch()
        b.n, b.frames, b.window = n, frames, window
        b.latents, b.lengths = _lib.ptr(latents), _lib.ptr(lengths)
        b.lstm_h, b.lstm_c = _lib.ptr(h), _lib.ptr(c)
        b.windows, b.valid = _lib.ptr(windows), _lib.ptr(valid)
        b.audio = audio.data_ptr()
        return b

    def launch(self, b: _lib.DvocBatch, conv: int | None = None) -> None:
        """``dvoc_decode`` on the current stream (or, with ``conv``, only that
        decoder convolution: ``dvoc_conv_launch``, for profiling)."""
        s = torch.cuda.current_stream(self.device).cuda_stream
        L = _lib.lib()
        if conv is None:
            _lib.check(L.dvoc_decode(self._h, ctypes.byref(b), self.ws.data_ptr(), self.ws.numel(), s),
                       "dvoc_decode")
        else:
            _lib.check(L.dvoc_conv_launch(self._h, ctypes.byref(b), self.ws.data_ptr(), self.ws.numel(),
                                          conv, s), "dvoc_conv_launch")

    @property
    def num_convs(self) -> int:
        return _lib.lib().dvoc_num_convs(self._h)

    def _call(self, n: int, frames: int, window: int, **tensors) -> torch.Tensor:
        T = window if window else frames
        audio = torch.empty(n, T * self.hop_size, dtype=torch.float32, device=self.device)
        self.launch(self.batch(n, frames, window, audio, **tensors))
        return audio

    def check_errors(self) -> None:
        err = ctypes.c_uint32(0)
        s = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(_lib.lib().dvoc_read_error(self._h, self.ws.data_ptr(), s, ctypes.byref(err)),
                   "dvoc_read_error")
        if err.value:
            raise RuntimeError(f"vocoder device error bits {err.value:#x}")

    def _state_zeros(self, n: int):
        z = torch.zeros(self.cfg.mi_layers, n, self.Hm, dtype=torch.float32, device=self.device)
        return z, z.clone()

    # ------------------------------------------------------------------ one shot
    def decode_batch(self, latents) -> list[torch.Tensor]:
        """One-shot decode of several utterances in one call: ``latents`` is a
        list of [T_i, L] tensors (or one [n, T, L]); returns the audio of each,
        [T_i * hop] fp32 on the device (``inference_from_latents``)."""
        if isinstance(latents, torch.Tensor):
            latents = list(latents)
        out: list[torch.Tensor] = []
        for s in range(0, len(latents), self.max_batch):
            part = latents[s:s + self.max_batch]
            lens = [int(x.shape[0]) for x in part]
            T = max(lens)
            if T > self.max_frames:
                raise ValueError(f"utterance of {T} frames exceeds max_frames={self.max_frames}")
            if min(lens) < 1:
                raise ValueError("empty utterance")
            n = len(part)
            x = torch.zeros(n, T, self.L, dtype=torch.float32, device=self.device)
            for i, lat in enumerate(part):
                if lat.shape[-1] != self.L:
                    raise ValueError(f"latent_dim must be {self.L}, got {lat.shape[-1]}")
                x[i, :lens[i]] = lat.to(self.device, torch.float32)
            ln = torch.tensor(lens, dtype=torch.int32).to(self.device)
            h, c = self._state_zeros(n)
            audio = self._call(n, T, 0, latents=x, lengths=ln, h=h, c=c)
            out += [audio[i, :lens[i] * self.hop_size] for i in range(n)]
        return out

    @torch.no_grad()
    def inference_from_latents(self, x: torch.Tensor, do_sample: bool = True,
                               noise_scale: float = 1.0) -> torch.Tensor:
        """``AudioVAE.inference_from_latents`` (``bigvgan.py:800-813``): x is
        [B, D, T] (D = 2L with do_sample: mean and log-scale, sampled here);
        returns [B, 1, T * hop]."""
        if do_sample:
            if x.size(1) != 2 * self.L:
                raise ValueError(f"Input must be like [B, D, H], got {tuple(x.shape)}")
            m, logs = torch.split(x, self.L, dim=1)
            x = m + torch.randn_like(m) * torch.exp(logs) * noise_scale
        elif x.size(1) != self.L:
            raise ValueError(f"Input must be like [B, D, H], got {tuple(x.shape)}")
        audio = self.decode_batch(list(x.transpose(1, 2).float()))
        return torch.stack(audio)[:, None]

    # ------------------------------------------------------------------ streaming
    def stream_window_size(self, chunk_size: int) -> int:
        """``Decoder.stream_window_size`` (``bigvgan.py:724-733``)."""
        if chunk_size < 1:
            raise ValueError(f"chunk_size must be >= 1, got {chunk_size}.")
        return chunk_size + self.lookahead + self.left_context

    def init_stream_state(self, batch_size: int = 1, chunk_size: int = 8) -> B200StreamState:
        """``AudioVAE.init_stream_state`` (``bigvgan.py:835-856``) for one request."""
        if batch_size != 1:
            raise ValueError("B200Vocoder streams one request per state (batch them with stream_step_many)")
        W = self.stream_window_size(chunk_size)
        if W > self.max_frames:
            raise ValueError(f"stream window {W} exceeds max_frames={self.max_frames}")
        z = torch.zeros(self.cfg.mi_layers, self.Hm, dtype=torch.float32, device=self.device)
        win = torch.zeros(W, self.L, dtype=torch.float32, device=self.device)
        return B200StreamState(z, z.clone(), win, int(chunk_size))

    def _slice(self, st: B200StreamState, audio: torch.Tensor, final: bool) -> torch.Tensor:
        """``_slice_stream_audio_window`` (``bigvgan.py:1005-1035``)."""
        stable = st.total if final else max(0, st.total - self.lookahead)
        if stable <= st.emitted:
            return audio[:0]
        W = st.window.shape[0]
        start = st.total - min(st.total, W)
        if st.emitted < start:
            raise RuntimeError("Decoder stream window is too short for fixed-graph decoding.")
        a, b = (st.emitted - start) * self.hop_size, (stable - start) * self.hop_size
        st.emitted = stable
        return audio[a:b]

    def _gather(self, states: list[B200StreamState]):
        W = states[0].window.shape[0]
        if any(s.window.shape[0] != W for s in states):
            raise ValueError("states of one call must share the chunk size")
        h = torch.stack([s.h for s in states], dim=1).contiguous()
        c = torch.stack([s.c for s in states], dim=1).contiguous()
        win = torch.stack([s.window for s in states]).contiguous()
        valid = torch.tensor([min(s.total, W) for s in states], dtype=torch.int32).to(self.device)
        return W, h, c, win, valid

    def stream_step_many(self, states: list[B200StreamState], latents: torch.Tensor) -> list[torch.Tensor]:
        """One chunk for each of n requests in one call: ``latents`` is [n, chunk,
        L] (frames-first); returns each request's newly stable samples."""
        n = len(states)
        if latents.dim() != 3 or latents.shape[0] != n or latents.shape[2] != self.L:
            raise ValueError(f"latents must be [{n}, chunk, {self.L}], got {tuple(latents.shape)}")
        chunk = latents.shape[1]
        for s in states:
            if chunk != s.chunk:
                raise ValueError(f"Streaming chunk_size must stay fixed at {s.chunk}, got {chunk}.")
        out: list[torch.Tensor] = []
        for p in range(0, n, self.max_batch):
            part = states[p:p + self.max_batch]
            W, h, c, win, valid = self._gather(part)
            lat = latents[p:p + len(part)].to(self.device, torch.float32).contiguous()
            audio = self._call(len(part), chunk, W, latents=lat, h=h, c=c, windows=win, valid=valid)
            for i, s in enumerate(part):
                s.h.copy_(h[:, i])
                s.c.copy_(c[:, i])
                s.window.copy_(win[i])
                s.total += chunk
                out.append(self._slice(s, audio[i], final=False))
        return out

    def stream_flush_many(self, states: list[B200StreamState]) -> list[torch.Tensor]:
        """``stream_flush`` for n requests in one call."""
        out: list[torch.Tensor] = []
        for p in range(0, len(states), self.max_batch):
            part = states[p:p + self.max_batch]
            W, h, c, win, valid = self._gather(part)
            audio = self._call(len(part), 0, W, windows=win, valid=valid)
            out += [self._slice(s, audio[i], final=True) for i, s in enumerate(part)]
        return out

    @torch.no_grad()
    def stream_step(self, latents: torch.Tensor, state: B200StreamState) -> torch.Tensor:
        """``AudioVAE.stream_step``: latents [1, L, chunk] -> [1, 1, samples]."""
        if latents.ndim != 3 or latents.size(1) != self.L:
            raise ValueError("Streaming latents must have shape [batch, latent_dim, frames], "
                             f"got {tuple(latents.shape)}.")
        return self.stream_step_many([state], latents.transpose(1, 2))[0].view(1, 1, -1)

    @torch.no_grad()
    def stream_flush(self, state: B200StreamState) -> torch.Tensor:
        """``AudioVAE.stream_flush``: -> [1, 1, samples]."""
        return self.stream_flush_many([state])[0].view(1, 1, -1)

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            _lib.lib().dvoc_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@torch.no_grad()
def batched_step_stream(engine, *, vocode: bool = True) -> list:
    """``DotsBatchEngine.step_stream`` (``engine.py:855-893``) with the vocoder
    work of the step batched: every streaming request's pending patches in one
    ``stream_step_many`` call per round (usually one round: one patch per
    request per step), every finished stream in one ``stream_flush_many``, every
    finished one-shot request in one ``decode_batch``, and the audio read back
    in one copy.  Events, their order and the per-request bookkeeping
    (``vocoded``, lazy stream state, the silent chunks of ``vocode=False``) are
    the reference's; each request's audio is what its own per-request calls
    would give (requests are decoded independently)."""
    hop = engine.dots.hop_size * engine.core.latent_patch_size
    seqs = engine.step()
    if not seqs and not engine.scheduler.is_finished():
        raise RuntimeError("scheduler made no progress with pending requests "
                           "(KV exhaustion / preemption livelock).")
    voc = engine.dots.vocoder
    pieces: dict[int, list] = {}
    if vocode:
        work = []
        for i, seq in enumerate(seqs):
            st = seq.custom_payload
            if st.stream and st.vocoded < len(st.latents):
                if st.vocoder_state is None:
                    st.vocoder_state = engine.dots._init_vocoder_stream_state()
                work.append((i, st))
                pieces[i] = []
        r = 0
        while True:
            batch = [(i, st) for i, st in work if st.vocoded + r < len(st.latents)]
            if not batch:
                break
            lat = torch.cat([st.latents[st.vocoded + r] for _, st in batch], dim=0)
            outs = voc.stream_step_many([st.vocoder_state for _, st in batch], lat)
            for (i, _), o in zip(batch, outs):
                pieces[i].append(o)
            r += 1
    flush = [(i, seq.custom_payload) for i, seq in enumerate(seqs)
             if seq.custom_payload.stream and seq.stoped and seq.custom_payload.vocoder_state is not None]
    finals = dict(zip((i for i, _ in flush),
                      voc.stream_flush_many([st.vocoder_state for _, st in flush]))) if flush else {}
    oneshot = [(i, seq.custom_payload) for i, seq in enumerate(seqs)
               if vocode and not seq.custom_payload.stream and seq.stoped and seq.custom_payload.latents]
    wavs = dict(zip((i for i, _ in oneshot),
                    voc.decode_batch([torch.cat(st.latents, dim=1)[0] for _, st in oneshot]))) if oneshot else {}
    # one device -> host copy of every piece of audio of the step
    dev = [t.reshape(-1).float() for lst in pieces.values() for t in lst]
    dev += [t.reshape(-1).float() for t in finals.values()] + [t.reshape(-1).float() for t in wavs.values()]
    host = iter(torch.cat(dev).cpu().split([t.numel() for t in dev])) if dev else iter(())
    host_pieces = {i: [next(host) for _ in lst] for i, lst in pieces.items()}
    host_finals = {i: next(host) for i in finals}
    host_wavs = {i: next(host) for i in wavs}
    events: list = []
    for i, seq in enumerate(seqs):
        st = seq.custom_payload
        if st.stream:
            k = 0
            while st.vocoded < len(st.latents):
                chunk = host_pieces[i][k] if vocode else torch.zeros(hop)
                k += 1
                st.vocoded += 1
                if chunk.numel():
                    events.append((seq.seq_id, "audio", chunk))
            if seq.stoped:
                final = host_finals.get(i, torch.zeros(0))
                if final.numel():
                    events.append((seq.seq_id, "audio", final))
                events.append((seq.seq_id, "done", None))
        elif seq.stoped:
            if vocode:
                wav = host_wavs.get(i, torch.zeros(0))
            else:
                wav = torch.zeros(hop * len(st.latents))
            if wav.numel():
                events.append((seq.seq_id, "audio", wav))
            events.append((seq.seq_id, "done", None))
    return events


def install_vocoder(engine, voc: B200Vocoder, batch_streams: bool = True) -> None:
    """Route the engine's vocoder calls (``engine.py:825-852`` through
    ``DotsModel``, ``native/model.py:204-218``) to ``voc``; with
    ``batch_streams`` the engine's ``step_stream`` also batches the step's
    vocoder work across requests (``batched_step_stream``)."""
    engine.dots.vocoder = voc
    engine.dots.hop_size = voc.hop_size
    if batch_streams:
        engine.step_stream = lambda *, vocode=True: batched_step_stream(engine, vocode=vocode)
