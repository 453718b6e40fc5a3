"""Host-side mirror of the reference's FM-head interface, over the C ABI.

``B200FMHead`` is the batched counterpart of the reference's per-request KV
cache heads (``CachedFMHead`` / ``FlashCachedFMHead``,
``nanovllm_dots/models/dots/cached_fm.py:200-309``,
``flash_cached_fm.py:81-360``): it owns the packed weights, the paged K/V
pool and every request's page list, and one ``tick`` call decodes the next
latent patch of every in-flight request (``decode_patch`` of each head, for all
of them at once).  Errors raise ``RuntimeError``, as the reference engine does
(``engine.py:487-506,661-666``).

PyTorch is used only for device memory and streams; all arithmetic runs in the
CUDA library.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np
import torch

from . import _lib
from .synthetic import BASE, FMConfig


# --------------------------------------------------------------------------- #
# Weights                                                                      #
# --------------------------------------------------------------------------- #
PRECISIONS = {"bf16": 0, "fp8": 1}   # DFM_PRECISION_BF16 / DFM_PRECISION_FP8


def quantize_rows_e4m3(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Rowwise e4m3 quantisation of the last dimension: returns (bytes uint8,
    fp32 scale per row) with w ~= e4m3(bytes) * scale, scale = row absmax / 448
    (1 for an all-zero row).  The FP8 counterpart of the reference's
    Int8DynamicLinear weight quantisation (``int8_dit.py:34-65``)."""
    wf = w.float()
    amax = wf.abs().amax(dim=-1)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q = (wf / scale.unsqueeze(-1)).to(torch.float8_e4m3fn)
    return q.view(torch.uint8), scale


def pack_weights(sd: dict[str, torch.Tensor], cfg: FMConfig, device,
                 precision: str = "bf16") -> dict[str, torch.Tensor]:
    """Pack reference-named weights into the C-ABI layout (bf16 matrices, fp32
    vectors) on ``device``.  Keys follow the reference state dict
    (``native/dit.py`` module names plus ``coordinate_proj``, ``hidden_proj``,
    ``latent_proj``).  ``precision="fp8"`` adds the e4m3 QKV and fc1 matrices
    with their per-row scales (quantised from the bf16 weights)."""
    L = cfg.layers
    bf = lambda t: t.detach().to(device=device, dtype=torch.bfloat16).contiguous()
    f32 = lambda t: t.detach().to(device=device, dtype=torch.float32).contiguous()
    blk = lambda l, n: sd[f"blocks.{l}.{n}"]
    out = {
        "input_w": bf(sd["input_layer.weight"]), "input_b": f32(sd["input_layer.bias"]),
        "temb_w1": bf(sd["time_embedder.mlp.0.weight"]), "temb_b1": f32(sd["time_embedder.mlp.0.bias"]),
        "temb_w2": bf(sd["time_embedder.mlp.2.weight"]), "temb_b2": f32(sd["time_embedder.mlp.2.bias"]),
        "demb_w1": bf(sd["duration_embedder.mlp.0.weight"]),
        "demb_b1": f32(sd["duration_embedder.mlp.0.bias"]),
        "demb_w2": bf(sd["duration_embedder.mlp.2.weight"]),
        "demb_b2": f32(sd["duration_embedder.mlp.2.bias"]),
        "ada_w": bf(torch.cat([blk(l, "adaLN_modulation.1.weight") for l in range(L)]
                              + [sd["output_layer.adaLN_modulation.1.weight"]])),
        "ada_b": f32(torch.cat([blk(l, "adaLN_modulation.1.bias") for l in range(L)]
                               + [sd["output_layer.adaLN_modulation.1.bias"]])),
        "qkv_w": bf(torch.stack([torch.cat([blk(l, "attn.q_proj.weight"), blk(l, "attn.k_proj.weight"),
                                            blk(l, "attn.v_proj.weight")]) for l in range(L)])),
        "qk_norm": f32(torch.stack([torch.stack([blk(l, "attn.q_norm.weight"), blk(l, "attn.q_norm.bias"),
                                                 blk(l, "attn.k_norm.weight"), blk(l, "attn.k_norm.bias")])
                                    for l in range(L)])),
        "o_w": bf(torch.stack([blk(l, "attn.o_proj.weight") for l in range(L)])),
        "o_b": f32(torch.stack([blk(l, "attn.o_proj.bias") for l in range(L)])),
        "fc1_w": bf(torch.stack([blk(l, "ffn.fc1.weight") for l in range(L)])),
        "fc1_b": f32(torch.stack([blk(l, "ffn.fc1.bias") for l in range(L)])),
        "fc2_w": bf(torch.stack([blk(l, "ffn.fc2.weight") for l in range(L)])),
        "fc2_b": f32(torch.stack([blk(l, "ffn.fc2.bias") for l in range(L)])),
        "final_w": bf(sd["output_layer.linear.weight"]), "final_b": f32(sd["output_layer.linear.bias"]),
        "coord_w": bf(sd["coordinate_proj.weight"]), "coord_b": f32(sd["coordinate_proj.bias"]),
        "hidden_w": bf(sd["hidden_proj.weight"]), "hidden_b": f32(sd["hidden_proj.bias"]),
        "latent_w": bf(sd["latent_proj.weight"]), "latent_b": f32(sd["latent_proj.bias"]),
    }
    # RotaryEmbedding.inv_freq exactly as the reference builds it (layers.py:105-110)
    dh = cfg.head_dim
    out["rope_inv_freq"] = f32(1.0 / (cfg.rotary_theta ** (torch.arange(0, dh, 2).float() / dh)))
    if precision not in PRECISIONS:
        raise ValueError(f"precision must be one of {sorted(PRECISIONS)}, got {precision!r}")
    if precision == "fp8":
        for name in ("qkv", "fc1"):
            q, s = quantize_rows_e4m3(out[f"{name}_w"])
            out[f"{name}_w8"] = q.contiguous()
            out[f"{name}_ws"] = s.contiguous()
    return out


def abi_config(cfg: FMConfig, num_pages: int, max_pages_per_req: int, max_requests: int,
               precision: str = "bf16"):
    return _lib.DfmConfig(cfg.layers, cfg.hidden, cfg.heads, cfg.head_dim, cfg.ffn, cfg.latent_dim,
                          cfg.latent_patch, cfg.hidden_patch, cfg.cond_dim, cfg.nfe, cfg.page_rows,
                          num_pages, max_pages_per_req, max_requests, cfg.ln_eps,
                          PRECISIONS[precision])


# --------------------------------------------------------------------------- #
# Pages                                                                        #
# --------------------------------------------------------------------------- #
class PageAllocator:
    """Free list of K/V pool pages and each request's page list (host side).

    A page holds ``page_rows`` consecutive cache positions of one request for
    every (layer, step, K|V) plane.  This is the FM counterpart of the LLM
    engine's block manager (``nanovllm_dots/engine/block_manager.py:90``)
    without prefix sharing (FM cache contents depend on the request's g_cond).
    Each request's pages are also kept as a block-table row (int32, -1 past
    its pages), so a tick's block table is one row copy per request.
    """

    def __init__(self, num_pages: int, page_rows: int, max_pages_per_req: int):
        self.num_pages = num_pages
        self.page_rows = page_rows
        self.max_pages_per_req = max_pages_per_req
        self.free = list(range(num_pages - 1, -1, -1))
        self.pages: dict[object, list[int]] = {}
        self.rows: dict[object, np.ndarray] = {}

    def ensure(self, rid, rows: int) -> list[int]:
        """Grow request rid's page list to cover ``rows`` positions."""
        need = -(-rows // self.page_rows)
        have = self.pages.get(rid)
        if have is not None and len(have) >= need:
            return have
        if need > self.max_pages_per_req:
            raise RuntimeError(f"request {rid!r}: {rows} FM cache rows exceed the block-table "
                               f"capacity ({self.max_pages_per_req} pages of {self.page_rows})")
        if have is None:
            have = self.pages[rid] = []
            self.rows[rid] = np.full(self.max_pages_per_req, -1, dtype=np.int32)
        row = self.rows[rid]
        while len(have) < need:
            if not self.free:
                raise RuntimeError("FM K/V pool exhausted: no free pages "
                                   f"({self.num_pages} pages total)")
            row[len(have)] = self.free[-1]
            have.append(self.free.pop())
        return have

    def row(self, rid) -> np.ndarray:
        """Request rid's block-table row (after ``ensure``)."""
        return self.rows[rid]

    def release(self, rid) -> None:
        self.rows.pop(rid, None)
        for p in self.pages.pop(rid, []):
            self.free.append(p)

    def used(self) -> int:
        return self.num_pages - len(self.free)


@dataclasses.dataclass
class FMRequest:
    """Per-request FM state kept by the head: rows already cached."""
    rid: object
    cache_len: int = 0


# --------------------------------------------------------------------------- #
# Head                                                                         #
# --------------------------------------------------------------------------- #
class B200FMHead:
    """Batched MeanFlow FM head over the paged per-(layer, step) K/V cache.

    ``tick`` is one engine step for all in-flight requests: it extends each
    request's cache by the rows that graduated since its previous tick and runs
    the NFE solver steps on the active rows (hidden row + latent patch),
    returning the next latent patch of every request.
    """

    def __init__(self, weights: dict[str, torch.Tensor], cfg: FMConfig = BASE, *,
                 num_pages: int, max_pages_per_req: int, max_requests: int,
                 device: torch.device | str = "cuda", precision: str = "bf16"):
        self.cfg = cfg
        self.precision = precision
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("B200FMHead runs on a CUDA device only (no CPU path)")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.L = _lib.lib()
        self.w = pack_weights(weights, cfg, self.device, precision)
        self.acfg = abi_config(cfg, num_pages, max_pages_per_req, max_requests, precision)
        wstruct = _lib.DfmWeights(*[_lib.ptr(self.w.get(f)) for f in _lib.WEIGHT_FIELDS])
        h = _lib.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(self.L.dfm_create(self.acfg, wstruct, h), "dfm_create")
        self.handle = h
        self.ws_bytes = int(self.L.dfm_workspace_size(h))
        self.workspace = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=self.device)
        pool_bytes = int(self.L.dfm_pool_bytes(self.acfg))
        self.pool = torch.zeros(pool_bytes // 2, dtype=torch.bfloat16, device=self.device)
        if num_pages < 2:
            raise RuntimeError("the K/V pool needs at least 2 pages")
        # The last page is never handed to a request: graph warm-up writes there.
        self.scratch_page = num_pages - 1
        self.pages = PageAllocator(num_pages - 1, cfg.page_rows, max_pages_per_req)
        self.max_requests = max_requests
        self.max_pages_per_req = max_pages_per_req
        self.requests: dict[object, FMRequest] = {}

    # ------------------------------------------------------------- pool views
    def pool_view(self) -> torch.Tensor:
        """The pool as [layers, nfe, 2, pages, heads, page_rows, head_dim]."""
        c = self.cfg
        return self.pool.view(c.layers, c.nfe, 2, self.acfg.num_pages, c.heads, c.page_rows,
                              c.head_dim)

    def write_prefix(self, rid, kv: torch.Tensor) -> None:
        """Install a request's cached prefix K/V (bf16 [nfe, layers, 2, P, heads,
        head_dim]) into its pages; the request's cache_len becomes P.  This is
        the bulk-prefill entry (``flash_cached_fm.py:279-313`` builds the same
        state by running the prefix through the DiT)."""
        c = self.cfg
        P = kv.shape[3]
        req = self.requests.setdefault(rid, FMRequest(rid))
        pages = self.pages.ensure(rid, P)
        if P:
            npg = math.ceil(P / c.page_rows)
            planes = c.layers * c.nfe * 2
            kvd = kv.to(self.device, torch.bfloat16).permute(1, 0, 2, 3, 4, 5)  # [L, nfe, 2, P, h, d]
            kvd = kvd.reshape(planes, P, c.heads, c.head_dim)
            if npg * c.page_rows != P:
                kvd = torch.cat([kvd, kvd.new_zeros(planes, npg * c.page_rows - P, c.heads,
                                                    c.head_dim)], dim=1)
            blocks = kvd.view(planes, npg, c.page_rows, c.heads, c.head_dim).transpose(2, 3)
            view = self.pool.view(planes, self.acfg.num_pages, c.heads, c.page_rows, c.head_dim)
            idx = torch.tensor(pages[:npg], dtype=torch.long, device=self.device)
            view[:, idx] = blocks
        req.cache_len = P

    def release(self, rid) -> None:
        """Free a finished request's pages and state (``engine.py:460-473``
        cancel/finish)."""
        self.pages.release(rid)
        self.requests.pop(rid, None)

    # ------------------------------------------------------------- ticks
    def prepare(self, rids, n_extend, dst: torch.Tensor | None = None
                ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Host bookkeeping for one tick: allocate pages for the graduating and
        active rows, build (cache_len, n_extend, block_table) device tensors
        (packed in one buffer: one host-to-device copy, into ``dst`` when
        given: an int32 device buffer of 2n + n * max_pages_per_req)."""
        c = self.cfg
        n = len(rids)
        if not 1 <= n <= self.max_requests:
            raise RuntimeError(f"tick with {n} requests (max {self.max_requests})")
        W = self.max_pages_per_req
        buf = np.empty(2 * n + n * W, dtype=np.int32)
        cl, ne, bt = buf[:n], buf[n:2 * n], buf[2 * n:].reshape(n, W)
        for i, (rid, e) in enumerate(zip(rids, n_extend)):
            if not 0 <= e <= c.stride:
                raise RuntimeError(f"request {rid!r}: n_extend={e} outside [0, {c.stride}]")
            req = self.requests.get(rid)
            if req is None:
                req = self.requests[rid] = FMRequest(rid)
            self.pages.ensure(rid, req.cache_len + e + c.stride)
            bt[i] = self.pages.row(rid)
            cl[i] = req.cache_len
            ne[i] = e
        if dst is None:
            d = torch.from_numpy(buf).pin_memory().to(self.device, non_blocking=True)
        else:
            d = dst
            d.copy_(torch.from_numpy(buf).pin_memory(), non_blocking=True)
        return d[:n], d[n:2 * n], d[2 * n:].view(n, W)

    def _batch(self, *, noise, cache_len, n_extend, block_table, out, act_hidden=None,
               act_row=None, ext_hidden=None, ext_latent=None, ext_rows=None, g_cond=None):
        for name, t in (("noise", noise), ("out", out), ("act_hidden", act_hidden),
                        ("act_row", act_row), ("ext_hidden", ext_hidden),
                        ("ext_latent", ext_latent), ("ext_rows", ext_rows), ("g_cond", g_cond)):
            if t is not None:
                if t.dtype != torch.bfloat16 or t.device != self.device or not t.is_contiguous():
                    raise RuntimeError(f"{name}: expected a contiguous bf16 tensor on {self.device}")
        for name, t in (("cache_len", cache_len), ("n_extend", n_extend),
                        ("block_table", block_table)):
            if t.dtype != torch.int32 or t.device != self.device or not t.is_contiguous():
                raise RuntimeError(f"{name}: expected a contiguous int32 tensor on {self.device}")
        n = noise.shape[0]
        if block_table.shape != (n, self.max_pages_per_req):
            raise RuntimeError(f"block_table must be [n, {self.max_pages_per_req}]")
        return _lib.DfmBatch(n, _lib.ptr(noise), _lib.ptr(act_hidden), _lib.ptr(act_row),
                             _lib.ptr(ext_hidden), _lib.ptr(ext_latent), _lib.ptr(ext_rows),
                             _lib.ptr(g_cond), _lib.ptr(cache_len), _lib.ptr(n_extend),
                             _lib.ptr(block_table), _lib.ptr(self.pool), _lib.ptr(out))

    def launch(self, *, stream=None, **tensors) -> None:
        """One ``dfm_step`` on device tensors (no host bookkeeping); keyword
        tensors as ``DfmBatch`` names them (noise, cache_len, n_extend,
        block_table, out, and the row inputs)."""
        b = self._batch(**tensors)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        _lib.check(self.L.dfm_step(self.handle, b, _lib.ptr(self.workspace), self.ws_bytes,
                                   _lib.c_void_p(s.cuda_stream)), "dfm_step")

    def launch_kernel(self, kernel: str, step: int, layer: int, *, stream=None, **tensors) -> None:
        """One per-layer launch of the tick (``_lib.TICK_KERNELS`` names it) with
        the tick's own arguments, on the workspace a ``launch`` with the same
        tensors filled (for timing the tick's kernels one at a time)."""
        b = self._batch(**tensors)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        _lib.check(self.L.dfm_tick_launch(self.handle, b, _lib.ptr(self.workspace), self.ws_bytes,
                                          _lib.TICK_KERNELS.index(kernel), step, layer,
                                          _lib.c_void_p(s.cuda_stream)), "dfm_tick_launch")

    def tick(self, rids, *, noise, act_hidden=None, act_row=None, ext_hidden=None,
             ext_latent=None, ext_rows=None, n_extend=None, g_cond=None) -> torch.Tensor:
        """Decode the next latent patch of every request in ``rids``.

        Inputs are device tensors with one leading row per request.  Each
        request graduates ``n_extend[i]`` rows (default: stride, or 0 when no
        graduating inputs are given) into its cache.  Returns bf16
        [n, latent_patch, latent_dim]."""
        c = self.cfg
        n = len(rids)
        if n_extend is None:
            has_ext = ext_hidden is not None or ext_rows is not None
            n_extend = [c.stride if has_ext else 0] * n
        cl, ne, bt = self.prepare(rids, n_extend)
        out = torch.empty(n, c.latent_patch, c.latent_dim, dtype=torch.bfloat16, device=self.device)
        self.launch(noise=noise, cache_len=cl, n_extend=ne, block_table=bt, out=out,
                    act_hidden=act_hidden, act_row=act_row, ext_hidden=ext_hidden,
                    ext_latent=ext_latent, ext_rows=ext_rows, g_cond=g_cond)
        for rid, e in zip(rids, n_extend):
            self.requests[rid].cache_len += int(e)
        return out

    def replay_tick(self, tg: "TickGraph", rids, n_extend) -> torch.Tensor:
        """``tick`` through a captured graph: the caller has written this
        tick's row inputs and noise into ``tg.inputs``; this does the page
        bookkeeping (straight into the graph's block-table buffer) and replays.
        Returns ``tg.out`` (overwritten by the next replay)."""
        if len(rids) != tg.n:
            raise RuntimeError(f"graph for {tg.n} requests replayed with {len(rids)}")
        self.prepare(rids, n_extend, dst=tg.ints)
        out = tg.replay()
        for rid, e in zip(rids, n_extend):
            self.requests[rid].cache_len += int(e)
        return out

    @torch.no_grad()
    def prime(self, rids, rows, g_cond=None) -> None:
        """Bulk prefill of the caches (``prime_to``, ``flash_cached_fm.py:279-313``,
        used for voice-clone prompts and late switch-in, ``engine.py:440-458``):
        graduate request ``rids[i]``'s projected history rows ``rows[i]``
        (bf16 [P_i, hidden] device tensor; lengths may differ) into its cache
        after the rows it already holds.  Attention over the cache is causal by
        position, so this equals graduating the rows tick by tick; it runs
        ticks of up to ``stride`` graduating rows per request, all requests in
        the same ticks, and discards their latents.  ``g_cond`` [n, hidden]
        (or None) is each request's speaker condition, which the cached K/V
        depend on."""
        c = self.cfg
        H = c.hidden
        rows = [r.to(self.device, torch.bfloat16) for r in rows]
        done = [0] * len(rids)
        while True:
            live = [i for i in range(len(rids)) if done[i] < rows[i].shape[0]]
            if not live:
                return
            live = live[: self.max_requests]
            n = len(live)
            ext = torch.zeros(n, c.stride, H, dtype=torch.bfloat16, device=self.device)
            n_ext = []
            for j, i in enumerate(live):
                take = min(c.stride, rows[i].shape[0] - done[i])
                ext[j, :take] = rows[i][done[i]:done[i] + take]
                n_ext.append(take)
                done[i] += take
            act = torch.zeros(n, H, dtype=torch.bfloat16, device=self.device)
            noise = torch.zeros(n, c.latent_patch, c.latent_dim, dtype=torch.bfloat16,
                                device=self.device)
            g = None if g_cond is None else g_cond[live].to(self.device, torch.bfloat16)
            self.tick([rids[i] for i in live], noise=noise, act_row=act, ext_rows=ext,
                      n_extend=n_ext, g_cond=g)

    def graph(self, n: int, *, raw_inputs: bool = True, with_g: bool = False) -> "TickGraph":
        """A CUDA graph of one ``dfm_step`` for n requests over static buffers
        (the capture pattern of ``GraphedFlashCachedFMHead``,
        ``flash_cached_fm.py:191-360``): copy a tick's inputs into
        ``TickGraph.inputs``, ``replay()``, read ``TickGraph.out``."""
        return TickGraph(self, n, raw_inputs=raw_inputs, with_g=with_g)

    def check_errors(self) -> None:
        """Synchronise and raise if any kernel reported a device-side error."""
        v = _lib.c_uint32(0)
        s = torch.cuda.current_stream(self.device)
        _lib.check(self.L.dfm_read_error(self.handle, _lib.ptr(self.workspace),
                                         _lib.c_void_p(s.cuda_stream), v), "dfm_read_error")
        if v.value:
            names = [nm for bit, nm in _lib.DEVERR_BITS.items() if v.value & bit]
            raise RuntimeError(f"FM head device error: {', '.join(names)} (0x{v.value:x})")

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.L.dfm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TickGraph:
    """One captured FM-head tick over static device buffers.

    ``inputs`` holds noise, the active-row inputs (raw ``act_hidden`` or
    projected ``act_row``), the graduating-row inputs, g_cond (optional) and the
    per-request (cache_len, n_extend, block_table); ``out`` receives the next
    latent patch.  Every kernel of the tick replays from one graph launch, so
    the tick costs no per-kernel host work.
    """

    def __init__(self, head: B200FMHead, n: int, *, raw_inputs: bool = True, with_g: bool = False):
        c, dev = head.cfg, head.device
        self.head, self.n = head, n
        bf = dict(dtype=torch.bfloat16, device=dev)
        W = head.max_pages_per_req
        # cache_len, n_extend and block_table in one buffer (prepare's layout)
        self.ints = torch.zeros(2 * n + n * W, dtype=torch.int32, device=dev)
        t = {"noise": torch.zeros(n, c.latent_patch, c.latent_dim, **bf),
             "cache_len": self.ints[:n], "n_extend": self.ints[n:2 * n],
             "block_table": self.ints[2 * n:].view(n, W)}
        if raw_inputs:
            t["act_hidden"] = torch.zeros(n, c.cond_dim, **bf)
            t["ext_hidden"] = torch.zeros(n, c.cond_dim, **bf)
            t["ext_latent"] = torch.zeros(n, c.latent_patch, c.latent_dim, **bf)
        else:
            t["act_row"] = torch.zeros(n, c.hidden, **bf)
            t["ext_rows"] = torch.zeros(n, c.stride, c.hidden, **bf)
        if with_g:
            t["g_cond"] = torch.zeros(n, c.hidden, **bf)
        self.inputs = t
        self.out = torch.zeros(n, c.latent_patch, c.latent_dim, **bf)
        # Warm-up and capture point every request at the head's scratch page, so
        # the warm-up's K/V writes touch no request's cache.
        t["block_table"].fill_(head.scratch_page)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            head.launch(out=self.out, stream=side, **t)     # warm-up: plans, attributes
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            head.launch(out=self.out, stream=torch.cuda.current_stream(dev), **t)
        torch.cuda.synchronize(dev)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.out
