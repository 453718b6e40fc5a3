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
from .fm_head import B200FMHead, FMRequest, TickGraph


class B200FMDispatch:
    """Batched FM dispatch over one ``B200FMHead`` (one per GPU/process).

    ``noise_fn(n)``, when set, supplies the tick's solver noise (bf16 [n, lp,
    ld] on the head's device) instead of the reference's own draw; tests use it
    to feed the noise a golden run used.  With ``use_graphs`` each batch size's
    tick is captured once as a CUDA graph and replayed (its first tick pays the
    capture); otherwise every tick launches its kernels eagerly."""

    def __init__(self, head: B200FMHead, noise_fn=None, use_graphs: bool = True):
        self.head = head
        self.cfg = head.cfg
        self.noise_fn = noise_fn
        self.use_graphs = use_graphs
        self._cached: dict[int, int] = {}     # rid -> history rows already in the cache
        self._g_dev: dict[int, tuple[int, torch.Tensor]] = {}   # rid -> (source id, device g_cond)
        self._graphs: dict[int, TickGraph] = {}   # batch size -> captured tick
        self._seq_ok: dict[int, tuple] = {}   # rid -> (checked history buffer, row 0 address, rows)

    def _rid(self, payload) -> int:
        rid = id(payload)
        if rid not in self._cached:
            self._cached[rid] = 0
            weakref.finalize(payload, self._forget, rid)
        return rid

    def _forget(self, rid: int) -> None:
        self._cached.pop(rid, None)
        self._g_dev.pop(rid, None)
        self._seq_ok.pop(rid, None)
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

    def pack(self, payloads, plans, out=None):
        """This tick's device inputs: the active hidden rows act [n, H], the
        graduating rows ext [n, stride, H] (zero past each request's count) and
        g_cond [n, H], gathered from every request's ``fm_sequence`` by one
        kernel from a table of row addresses (one host-to-device copy), into
        ``out`` = (act, ext, g) when given."""
        c, head = self.cfg, self.head
        dev, H, n = head.device, c.hidden, len(payloads)
        table = []
        for p, (rid, s, e) in zip(payloads, plans):
            seq = p.gen_state.fm_sequence
            # a request's history buffer is checked once (the engine allocates it
            # at admission and appends in place); its row count every tick
            ok = self._seq_ok.get(rid)
            if ok is None or ok[0] is not seq:
                if (seq.device != dev or seq.dtype != torch.bfloat16 or seq.stride(-1) != 1
                        or seq.stride(-2) != H or seq.shape[-1] != H):
                    raise RuntimeError("fm_sequence: expected bf16 rows of width "
                                       f"{H} on {dev}")
                ok = self._seq_ok[rid] = (seq, seq[0].data_ptr(), seq.shape[-2])
            if ok[2] <= e:
                raise RuntimeError("fm_sequence does not hold the active row")
            table.append((ok[1], s, e - s, self._g_row(rid, p)))
        tab = torch.tensor(table, dtype=torch.int64).pin_memory().to(dev, non_blocking=True)
        if out is None:
            act = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
            ext = torch.empty(n, c.stride, H, dtype=torch.bfloat16, device=dev)
            g = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
        else:
            act, ext, g = out
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
            rids = [r for r, _, _ in plans]
            for rid, s, _ in plans:
                req = head.requests.get(rid)
                if req is not None and req.cache_len != s:
                    raise RuntimeError("FM cache out of step with the request history")
            n_ext = [e - s for _, s, e in plans]
            # same draw as batched_meanflow (batched_fm.py:110-111) so seeded runs line up
            if self.noise_fn is not None:
                noise = self.noise_fn(n)
            else:
                noise = torch.randn((n, c.latent_patch, c.latent_dim), device=dev,
                                    dtype=torch.bfloat16)
            if self.use_graphs and dev.type == "cuda":
                # one captured tick per batch size (the reference captures its
                # decode per batch size too, batched_llm.py:177-296): the rows,
                # the noise and the page table go into the graph's buffers
                tg = self._graphs.get(n)
                if tg is None:
                    tg = self._graphs[n] = head.graph(n, raw_inputs=False, with_g=True)
                t = tg.inputs
                self.pack(payloads, plans, out=(t["act_row"], t["ext_rows"], t["g_cond"]))
                t["noise"].copy_(noise)
                out = head.replay_tick(tg, rids, n_ext).clone()
            else:
                act, ext, g = self.pack(payloads, plans)
                out = head.tick(rids, noise=noise, act_row=act, ext_rows=ext, n_extend=n_ext,
                                g_cond=g)
        for rid, _, e in plans:
            self._cached[rid] = e
        return out


def install(engine, head: B200FMHead, batch_host_syncs: bool = True) -> B200FMDispatch:
    """Route ``engine._batched_fm`` through the B200 head (``fm_accel="b200"``).

    With ``batch_host_syncs`` (and the engine's batched patch encoder,
    ``flash_pe``) the two per-request host synchronisations of every tick go
    too: the end-of-speech check becomes a device flag instead of an
    ``.item()`` per request (``native/model.py:197-201``), and the emitted
    patches and those flags come to the host in one read per tick instead of
    a ``.cpu()`` per request (``engine.py:761-774``); see ``BatchedFinish``."""
    dispatch = B200FMDispatch(head)
    engine.fm_accel = "b200"
    engine._batched_fm = dispatch
    if batch_host_syncs and getattr(engine, "flash_pe", False):
        fin = BatchedFinish(engine)
        engine.dots._should_stop_after_current_audio = fin.deferred_stop
        engine._finish_patches_flash = fin
    return dispatch


class BatchedFinish:
    """The engine's post-FM step for the batched patch encoder
    (``DotsBatchEngine._finish_patches_flash`` + ``_emit_patch``,
    ``engine.py:743-778``) with one host synchronisation per tick.

    The reference reads each request's end-of-speech probability with
    ``.item()`` before the FM call (``model.py:197-201``) and copies each
    emitted patch to the host with ``.cpu()`` after it (``engine.py:761``):
    2N waits per tick for the GPU, each stalling the launch of the next
    work.  Here the end-of-speech check returns the device flag
    (``deferred_stop``); after the FM head and the patch encoder have been
    queued, the patches and every flag come to the host in one pinned copy,
    and each request's record is then updated exactly as ``_emit_patch``
    does: the patch encoder's embedding as the next LLM input, the
    denormalised patch appended to the results and to the sequence, the
    counters advanced, and the stop rule (end of speech, schedule exhausted
    or patch cap)."""

    def __init__(self, engine):
        self.engine = engine

    def deferred_stop(self, state, *, eos_threshold):
        """``_should_stop_after_current_audio`` without the host read: False
        before the first hidden, True after an explicit end, else the device
        flag ``eos_prob > eos_threshold`` (``model.py:197-201``)."""
        if state.llm_hiddens is None:
            return False
        if state.end_flag:
            return True
        eos = self.engine.core.eos_proj(state.llm_hiddens).softmax(dim=-1)[:, -1, 1]
        return (eos > eos_threshold).reshape(())

    def __call__(self, seqs, latents, stops) -> None:
        eng = self.engine
        core, dots, dev = eng.core, eng.dots, latents.device
        rows, claim = [], []
        for seq, latent in zip(seqs, latents):
            st = seq.custom_payload
            dots._append_history_chunk(st.gen_state, latent.unsqueeze(0))  # normalized
            if st.pe_row is None:                       # lazily claim a cache row
                if not eng._pe_free:
                    raise RuntimeError(
                        f"flash_pe: row pool exhausted ({eng._pe_max_batch} rows); "
                        f"more sequences are generating concurrently. Increase "
                        f"pe_max_batch or cap concurrency (max_num_seqs).")
                st.pe_row = eng._pe_free.pop()
                claim.append(st.pe_row)
            rows.append(st.pe_row)
        cuda = dev.type == "cuda"
        pinned = (lambda t: t.pin_memory()) if cuda else (lambda t: t)
        to_dev = lambda v: pinned(torch.tensor(v, dtype=torch.int32)).to(dev, non_blocking=True)
        if claim:
            eng._flash_pe.reset_rows(to_dev(claim))
        patches = core.io_helper.denormalize(latents)              # [N, ps, ld]
        embeds = eng._flash_pe.decode_patch(patches, to_dev(rows))  # [N, 1, H]
        n = len(seqs)
        flags = torch.stack([s.to(dev, torch.float32).reshape(()) if torch.is_tensor(s)
                             else torch.tensor(float(bool(s)), device=dev) for s in stops])
        # the one host synchronisation of the tick: every patch and stop flag
        host = pinned(torch.empty(patches.numel() + n, dtype=torch.float32))
        host.copy_(torch.cat([patches.detach().float().reshape(-1), flags]), non_blocking=cuda)
        if cuda:
            torch.cuda.current_stream(dev).synchronize()
        lat = host[:patches.numel()].view(patches.shape)
        stop_h = host[patches.numel():]
        for i, (seq, emb) in enumerate(zip(seqs, embeds)):
            st = seq.custom_payload
            st.next_embed = emb
            latent_cpu = lat[i:i + 1].clone()
            st.latents.append(latent_cpu)
            st.patches_emitted += 1
            st.position += 1
            seq.append_token(latent_cpu.reshape(-1).numpy().tobytes())
            schedule_exhausted = st.position >= st.schedule.size(1)
            cap = st.span_count if st.max_patches is None else min(st.span_count, st.max_patches)
            if bool(stop_h[i] > 0.5) or schedule_exhausted or st.patches_emitted >= cap:
                seq.stoped = True


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
