"""``fm_accel="b200"``: the engine-side drop-in for the reference's FM dispatch.

The reference engine calls ``DotsBatchEngine._batched_fm(payloads)`` once per
tick (``nanovllm_dots/models/dots/engine.py:539,615-633``).  For MeanFlow it
pads every request's full FM history and re-runs the DiT over all of it at each
solver step (``_pack_fm_inputs`` + ``batched_meanflow``, ``engine.py:635-709``).
``B200FMDispatch`` keeps the same call signature and return value
([N, latent_patch, latent_dim], normalised latents) but runs the O(P) paged
cache path: per request only the history rows that graduated since its last
tick go through the DiT (and into the cache), plus the 17 active rows.

Payloads are duck-typed like the reference's ``DotsSeqState``
(``engine.py:48-77``): ``gen_state.fm_sequence`` [1, cap, H] holds the
projected FM history (``model.py:101-120``), ``gen_state.fm_seq_len`` its length,
``g_cond`` / ``gen_state.fm_null_g_cond`` the speaker condition and
``num_steps`` the NFE.

Usage with the reference engine:

    engine = DotsBatchEngine(runtime, paged_llm, model_dir=..., fm_accel="none")
    install(engine, B200FMHead(weights, cfg, num_pages=..., ...))
"""
from __future__ import annotations

import contextlib
import weakref

import torch

from . import _lib
from .fm_head import B200FMHead, FMRequest


class B200FMDispatch:
    """Batched FM dispatch over one ``B200FMHead`` (one per GPU/process).

    ``noise_fn(n)``, when set, supplies the tick's solver noise (bf16 [n, lp,
    ld] on the head's device) instead of the reference's own draw; tests use it
    to feed the noise a golden run used."""

    def __init__(self, head: B200FMHead, noise_fn=None):
        self.head = head
        self.cfg = head.cfg
        self.noise_fn = noise_fn
        self._cached: dict[int, int] = {}     # rid -> history rows already in the cache
        self._g_dev: dict[int, tuple[int, torch.Tensor]] = {}   # rid -> (source id, device g_cond)

    def _rid(self, payload) -> int:
        rid = id(payload)
        if rid not in self._cached:
            self._cached[rid] = 0
            weakref.finalize(payload, self._forget, rid)
        return rid

    def _forget(self, rid: int) -> None:
        self._cached.pop(rid, None)
        self._g_dev.pop(rid, None)
        self.head.release(rid)

    def plan(self, payloads):
        """Per request: (rid, graduating row range, active row index).  The
        history rows [cached, L-1) graduate; row L-1 is the active hidden row
        (``cached_fm.py:264-277`` reads the same ranges)."""
        c = self.cfg
        plans = []
        for p in payloads:
            st = p.gen_state
            L = int(st.fm_seq_len)
            if L <= 0:
                raise RuntimeError("FM sequence length must be positive before decode.")
            if int(getattr(p, "num_steps", c.nfe)) != c.nfe:
                raise RuntimeError(f"fm_accel='b200' is built for num_steps={c.nfe}; got "
                                   f"{p.num_steps} (batched FM requires uniform decode params)")
            rid = self._rid(p)
            s = self._cached[rid]
            e = L - c.hidden_patch
            if e < s:
                raise RuntimeError("FM history shrank below the cached prefix")
            plans.append((rid, s, e))
        return plans

    @staticmethod
    def _g_cond(p):
        return p.g_cond if p.g_cond is not None else getattr(p.gen_state, "fm_null_g_cond", None)

    def _prime_backlog(self, payloads, plans):
        """Requests with more history rows pending than one tick graduates
        (a voice-clone prompt, a request switched in mid-stream) get all but
        the last ``stride`` of them bulk-prefilled first (``B200FMHead.prime``)."""
        c, head = self.cfg, self.head
        rids, rows, gs, out = [], [], [], []
        for p, (rid, s, e) in zip(payloads, plans):
            if e - s > c.stride:
                cut = e - c.stride
                rids.append(rid)
                rows.append(p.gen_state.fm_sequence[0, s:cut])
                gc = self._g_cond(p)
                gs.append(torch.zeros(c.hidden) if gc is None else gc.float().reshape(-1).cpu())
                self._cached[rid] = cut
                out.append((rid, cut, e))
            else:
                out.append((rid, s, e))
        if rids:
            for rid in rids:
                head.requests.setdefault(rid, FMRequest(rid))
            head.prime(rids, rows, g_cond=torch.stack(gs).to(torch.bfloat16))
        return out

    def _g_row(self, rid: int, p) -> int:
        """Device address of the request's bf16 g_cond row (0 = none).  A
        condition held elsewhere (host memory, another dtype) is copied to the
        device once per request and reused while the payload keeps it."""
        gc = self._g_cond(p)
        if gc is None:
            return 0
        c, dev = self.cfg, self.head.device
        if (gc.device == dev and gc.dtype == torch.bfloat16 and gc.is_contiguous()
                and gc.numel() == c.hidden):
            return gc.data_ptr()
        have = self._g_dev.get(rid)
        if have is None or have[0] != id(gc):
            have = (id(gc), gc.reshape(-1).to(dev, torch.bfloat16).contiguous())
            self._g_dev[rid] = have
        return have[1].data_ptr()

    def pack(self, payloads, plans):
        """This tick's device inputs: the active hidden rows act [n, H], the
        graduating rows ext [n, stride, H] (zero past each request's count) and
        g_cond [n, H], gathered from every request's ``fm_sequence`` by one
        kernel from a table of row addresses (one host-to-device copy)."""
        c, head = self.cfg, self.head
        dev, H, n = head.device, c.hidden, len(payloads)
        table = []
        for p, (rid, s, e) in zip(payloads, plans):
            seq = p.gen_state.fm_sequence
            if (seq.device != dev or seq.dtype != torch.bfloat16 or seq.stride(-1) != 1
                    or seq.stride(-2) != H or seq.shape[-1] != H or seq.shape[-2] <= e):
                raise RuntimeError("fm_sequence: expected bf16 rows of width "
                                   f"{H} on {dev} covering the active row")
            table.append((seq[0].data_ptr(), s, e - s, self._g_row(rid, p)))
        tab = torch.tensor(table, dtype=torch.int64).pin_memory().to(dev, non_blocking=True)
        act = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
        ext = torch.empty(n, c.stride, H, dtype=torch.bfloat16, device=dev)
        g = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
        s = torch.cuda.current_stream(dev)
        _lib.check(head.L.dfm_gather_rows(tab.data_ptr(), n, H, c.stride, act.data_ptr(),
                                          ext.data_ptr(), g.data_ptr(),
                                          _lib.c_void_p(s.cuda_stream)), "dfm_gather_rows")
        return act, ext, g

    @torch.no_grad()
    def __call__(self, payloads) -> torch.Tensor:
        c, head = self.cfg, self.head
        dev = head.device
        plans = self._prime_backlog(payloads, self.plan(payloads))
        n = len(payloads)
        # the head's device is current for the gather and the tick (a head on
        # cuda:1 works while cuda:0 is the caller's current device)
        with torch.cuda.device(dev) if dev.type == "cuda" else contextlib.nullcontext():
            act, ext, g = self.pack(payloads, plans)
            # same draw as batched_meanflow (batched_fm.py:110-111) so seeded runs line up
            if self.noise_fn is not None:
                noise = self.noise_fn(n)
            else:
                noise = torch.randn((n, c.latent_patch, c.latent_dim), device=dev,
                                    dtype=torch.bfloat16)
            rids = [r for r, _, _ in plans]
            for rid, s, _ in plans:
                req = head.requests.get(rid)
                if req is not None and req.cache_len != s:
                    raise RuntimeError("FM cache out of step with the request history")
            out = head.tick(rids, noise=noise, act_row=act, ext_rows=ext,
                            n_extend=[e - s for _, s, e in plans], g_cond=g)
        for rid, _, e in plans:
            self._cached[rid] = e
        return out


def install(engine, head: B200FMHead) -> B200FMDispatch:
    """Route ``engine._batched_fm`` through the B200 head (``fm_accel="b200"``)."""
    dispatch = B200FMDispatch(head)
    engine.fm_accel = "b200"
    engine._batched_fm = dispatch
    return dispatch


def install_patch_encoder(engine, pe) -> None:
    """Route the engine's batched patch encoder through ``B200PatchEncoder``.

    The reference engine (``flash_pe=True``, ``engine.py:197-222``) keeps a
    ``FlashPatchEncoder`` in ``engine._flash_pe`` and a free list of its cache
    rows in ``engine._pe_free``; it calls ``reset_rows(rows)`` when a request
    claims a row, ``prefill(prompt_latents, row)`` for a voice-clone prompt
    (``engine.py:392-405``) and ``decode_patch(patches, rows)`` once per tick
    for every request that emitted a patch (``engine.py:743-765``).
    ``B200PatchEncoder`` has the same three methods with the same arguments and
    results, so installing it is an attribute swap.  Install before the first
    request is admitted: the free list is rebuilt over the encoder's rows.
    """
    for name in ("decode_patch", "prefill", "reset_rows"):
        if not callable(getattr(pe, name, None)):
            raise TypeError(f"patch encoder lacks {name}()")
    engine.flash_pe = True
    engine._flash_pe = pe
    engine._pe_max_batch = pe.max_rows
    engine._pe_free = list(range(pe.max_rows))
