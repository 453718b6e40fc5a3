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

import weakref

import torch

from .fm_head import B200FMHead, FMRequest


class B200FMDispatch:
    """Batched FM dispatch over one ``B200FMHead`` (one per GPU/process)."""

    def __init__(self, head: B200FMHead):
        self.head = head
        self.cfg = head.cfg
        self._cached: dict[int, int] = {}     # rid -> history rows already in the cache

    def _rid(self, payload) -> int:
        rid = id(payload)
        if rid not in self._cached:
            self._cached[rid] = 0
            weakref.finalize(payload, self._forget, rid)
        return rid

    def _forget(self, rid: int) -> None:
        self._cached.pop(rid, None)
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

    @torch.no_grad()
    def __call__(self, payloads) -> torch.Tensor:
        c, head = self.cfg, self.head
        dev = head.device
        plans = self._prime_backlog(payloads, self.plan(payloads))
        n = len(payloads)
        H = c.hidden
        act = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
        ext = torch.zeros(n, c.stride, H, dtype=torch.bfloat16, device=dev)
        g = torch.zeros(n, H, dtype=torch.bfloat16, device=dev)
        n_ext = []
        for i, (p, (rid, s, e)) in enumerate(zip(payloads, plans)):
            seq = p.gen_state.fm_sequence
            act[i] = seq[0, e]
            if e > s:
                ext[i, : e - s] = seq[0, s:e]
            n_ext.append(e - s)
            gc = self._g_cond(p)
            if gc is not None:
                g[i] = gc.to(dev, torch.bfloat16).reshape(-1)
        # same draw as batched_meanflow (batched_fm.py:110-111) so seeded runs line up
        noise = torch.randn((n, c.latent_patch, c.latent_dim), device=dev, dtype=torch.bfloat16)
        rids = [r for r, _, _ in plans]
        for rid, s, _ in plans:
            req = head.requests.get(rid)
            if req is not None and req.cache_len != s:
                raise RuntimeError("FM cache out of step with the request history")
        out = head.tick(rids, noise=noise, act_row=act, ext_rows=ext, n_extend=n_ext, g_cond=g)
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
