"""Batched patch encoder on the B200 kernels: the drop-in for the reference's
``FlashPatchEncoder`` (``nanovllm_dots/models/dots/flash_patch_encoder.py:33-139``).

The reference turns each emitted latent patch into the LLM's next input
embedding with one ``flash_attn_with_kvcache`` call per encoder layer over a
persistent cache row per request (``decode_patch``), plus a whole-prompt pass
for voice-clone prompts (``prefill``).  ``B200PatchEncoder`` keeps the same
interface and state (cache rows, per-row ``seqlens``, per-row conv tail) and
runs each call as ONE ``dpe_decode`` of ``libdfm.so`` (``include/dpe.h``): the
conv, in_proj, every encoder layer (tcgen05 GEMMs with fused epilogues, the
paged attention kernel over the rows' own histories) and out_proj, on the
current stream without host synchronisation.  There is no CPU path.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from .synthetic import PE_BASE, PEConfig


def pack_pe_weights(sd: dict[str, torch.Tensor], cfg: PEConfig, device) -> dict[str, torch.Tensor]:
    """Reference state dict (``VAESemanticEncoder``) -> the layout ``DpeWeights``
    describes: bf16 [out, in] matrices, fp32 vectors; q/k/v stacked per layer;
    the conv kernel [out, in, 2] as [out, 2*in] (tap 0 | tap 1)."""
    L = cfg.layers
    bf = lambda t: t.to(device=device, dtype=torch.bfloat16).contiguous()
    f32 = lambda t: t.to(device=device, dtype=torch.float32).contiguous()
    blk = lambda l, k: sd[f"encoder.layers.{l}.{k}"]
    wc = sd["ds_proj.weight"]
    return {
        "conv_w": bf(torch.cat([wc[:, :, 0], wc[:, :, 1]], dim=1)),
        "conv_b": f32(sd["ds_proj.bias"]),
        "in_w": bf(sd["in_proj.weight"]), "in_b": f32(sd["in_proj.bias"]),
        "attn_norm": f32(torch.stack([torch.stack([blk(l, "attn_norm.weight"), blk(l, "attn_norm.bias")])
                                      for l in range(L)])),
        "ffn_norm": f32(torch.stack([torch.stack([blk(l, "ffn_norm.weight"), blk(l, "ffn_norm.bias")])
                                     for l in range(L)])),
        "qkv_w": bf(torch.stack([torch.cat([blk(l, "attn.q_proj.weight"), blk(l, "attn.k_proj.weight"),
                                            blk(l, "attn.v_proj.weight")]) for l in range(L)])),
        "o_w": bf(torch.stack([blk(l, "attn.o_proj.weight") for l in range(L)])),
        "o_b": f32(torch.stack([blk(l, "attn.o_proj.bias") for l in range(L)])),
        "fc1_w": bf(torch.stack([blk(l, "ffn.fc1.weight") for l in range(L)])),
        "fc1_b": f32(torch.stack([blk(l, "ffn.fc1.bias") for l in range(L)])),
        "fc2_w": bf(torch.stack([blk(l, "ffn.fc2.weight") for l in range(L)])),
        "fc2_b": f32(torch.stack([blk(l, "ffn.fc2.bias") for l in range(L)])),
        "out_w": bf(sd["out_proj.weight"]), "out_b": f32(sd["out_proj.bias"]),
    }


def pe_abi_config(cfg: PEConfig, max_rows: int, max_pages_per_row: int, max_batch: int):
    return _lib.DpeConfig(cfg.layers, cfg.hidden, cfg.heads, cfg.head_dim, cfg.ffn,
                          cfg.latent_dim, cfg.patch, cfg.out_dim, max_rows, max_pages_per_row,
                          max_batch, cfg.ln_eps)


class B200PatchEncoder:
    """Flash-equivalent, batched, length-generic patch encoder.

    ``max_batch`` cache rows (a persistent row per generating request, as the
    engine claims them, ``engine.py:750-760``), each holding up to
    ``max_seq_len`` encoder positions (``pe_max_patches * out_ds_rate``).
    """

    def __init__(self, weights: dict[str, torch.Tensor], cfg: PEConfig = PE_BASE, *,
                 max_batch: int, max_seq_len: int, device: torch.device | str = "cuda",
                 max_rows: int | None = None):
        self.cfg = cfg
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("B200PatchEncoder runs on a CUDA device only (no CPU path)")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.out_ds_rate = cfg.rows
        self.max_batch = max_batch
        self.max_rows = max_batch if max_rows is None else max_rows
        self.pages_per_row = math.ceil(max_seq_len / cfg.page_rows)
        self.cap = self.pages_per_row * cfg.page_rows
        self.L = _lib.lib()
        self.w = pack_pe_weights(weights, cfg, self.device)
        self.acfg = pe_abi_config(cfg, self.max_rows, self.pages_per_row, max_batch)
        wstruct = _lib.DpeWeights(*[_lib.ptr(self.w[f]) for f in _lib.PE_WEIGHT_FIELDS])
        h = _lib.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(self.L.dpe_create(self.acfg, wstruct, h), "dpe_create")
        self.handle = h
        self.ws_bytes = int(self.L.dpe_workspace_size(h))
        self.workspace = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=self.device)
        pool_bytes = int(self.L.dpe_pool_bytes(self.acfg))
        self.pool = torch.zeros(pool_bytes // 2, dtype=torch.bfloat16, device=self.device)
        self.seqlens = torch.zeros(self.max_rows, dtype=torch.int32, device=self.device)
        self.conv_tail = torch.zeros(self.max_rows, cfg.latent_dim, dtype=torch.bfloat16,
                                     device=self.device)

    # ------------------------------------------------------------- state
    def reset_rows(self, rows) -> None:
        """Zero the length and conv tail of the given cache rows, on
        (re)assignment (``flash_patch_encoder.py:71-76``).  Their stale K/V are
        never read: attention stops at each row's length."""
        rows = torch.as_tensor(rows, dtype=torch.long, device=self.device)
        self.seqlens[rows] = 0
        self.conv_tail[rows] = 0

    def pool_view(self) -> torch.Tensor:
        """The K/V pool as [layers, 2, rows, pages_per_row, heads, 16, head_dim]."""
        c = self.cfg
        return self.pool.view(c.layers, 2, self.max_rows, self.pages_per_row, c.heads,
                              c.page_rows, c.head_dim)

    # ------------------------------------------------------------- calls
    def launch(self, patches: torch.Tensor, rows: torch.Tensor, out: torch.Tensor,
               stream=None) -> None:
        """One ``dpe_decode`` on device tensors: patches bf16 [n, patch, ld],
        rows int32 [n] (distinct), out bf16 [n, out_dim]."""
        for name, t, dt in (("patches", patches, torch.bfloat16), ("rows", rows, torch.int32),
                            ("out", out, torch.bfloat16)):
            if t.dtype != dt or t.device != self.device or not t.is_contiguous():
                raise RuntimeError(f"{name}: expected a contiguous {dt} tensor on {self.device}")
        n = patches.shape[0]
        if not 1 <= n <= self.max_batch:
            raise RuntimeError(f"decode with {n} requests (max {self.max_batch})")
        if tuple(patches.shape[1:]) != (self.cfg.patch, self.cfg.latent_dim) or rows.numel() != n \
                or tuple(out.shape) != (n, self.cfg.out_dim):
            raise RuntimeError("patch encoder: inconsistent shapes")
        b = _lib.DpeBatch(n, _lib.ptr(patches), _lib.ptr(rows), _lib.ptr(self.seqlens),
                          _lib.ptr(self.conv_tail), _lib.ptr(self.pool), _lib.ptr(out))
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        _lib.check(self.L.dpe_decode(self.handle, b, _lib.ptr(self.workspace), self.ws_bytes,
                                     _lib.c_void_p(s.cuda_stream)), "dpe_decode")

    @torch.no_grad()
    def decode_patch(self, latent_patches: torch.Tensor, rows) -> torch.Tensor:
        """latent_patches [n, patch, latent_dim] (denormalised; cast to bf16 as
        the reference does), rows [n] cache rows -> embeddings [n, 1, out_dim];
        each row's cache advances by ``out_ds_rate``
        (``flash_patch_encoder.py:104-139``)."""
        patches = latent_patches.to(self.device, torch.bfloat16).contiguous()
        rows = torch.as_tensor(rows, dtype=torch.int32).to(self.device).contiguous()
        out = torch.empty(patches.shape[0], self.cfg.out_dim, dtype=torch.bfloat16,
                          device=self.device)
        self.launch(patches, rows, out)
        return out.unsqueeze(1)

    @torch.no_grad()
    def prime(self, rows: list[int], prompts: list[torch.Tensor]) -> list[torch.Tensor]:
        """Seed cache rows with whole prompts (``prefill`` for many rows): row
        ``rows[i]`` is reset and prompt ``prompts[i]`` ([frames, latent_dim],
        frames a multiple of the patch) is encoded into it.  The encoder is
        causal by position and the conv's zero pad is a reset row's tail, so
        this equals the reference's one-pass prefill; it runs decode calls of
        one patch per row, all rows in the same calls.  Returns each prompt's
        patch embeddings [frames / patch, out_dim]."""
        c = self.cfg
        chunks = []
        for r, p in zip(rows, prompts):
            p = p.reshape(-1, c.latent_dim)
            if p.shape[0] % c.patch:
                raise ValueError(f"prompt latent length {p.shape[0]} must be divisible by "
                                 f"patch_size={c.patch}")
            if p.shape[0] // c.patch * self.out_ds_rate > self.cap:
                raise RuntimeError(f"prompt encoder tokens {p.shape[0] // c.patch * self.out_ds_rate} "
                                   f"exceed capacity {self.cap}")
            chunks.append(p.to(self.device, torch.bfloat16).reshape(-1, c.patch, c.latent_dim))
        self.reset_rows(list(rows))
        outs = [[] for _ in rows]
        step = 0
        while True:
            live = [i for i in range(len(rows)) if step < chunks[i].shape[0]]
            if not live:
                break
            for k in range(0, len(live), self.max_batch):
                part = live[k:k + self.max_batch]
                emb = self.decode_patch(torch.stack([chunks[i][step] for i in part]),
                                        [rows[i] for i in part])
                for j, i in enumerate(part):
                    outs[i].append(emb[j, 0])
            step += 1
        return [torch.stack(o) if o else torch.zeros(0, c.out_dim, dtype=torch.bfloat16,
                                                     device=self.device) for o in outs]

    @torch.no_grad()
    def prefill(self, prompt_latents: torch.Tensor, row: int) -> torch.Tensor:
        """Seed cache ``row`` with a whole prompt [1, frames, latent_dim] and
        return its patch embeddings [1, P, out_dim]
        (``flash_patch_encoder.py:78-102``)."""
        return self.prime([row], [prompt_latents.reshape(-1, self.cfg.latent_dim)])[0].unsqueeze(0)

    def graph(self, n: int) -> "DecodeGraph":
        """A CUDA graph of one ``dpe_decode`` for n requests over static
        buffers: copy patches and rows into ``DecodeGraph.inputs``,
        ``replay()``, read ``DecodeGraph.out``."""
        return DecodeGraph(self, n)

    def check_errors(self) -> None:
        """Synchronise and raise if any kernel reported a device-side error."""
        v = _lib.c_uint32(0)
        s = torch.cuda.current_stream(self.device)
        _lib.check(self.L.dpe_read_error(self.handle, _lib.ptr(self.workspace),
                                         _lib.c_void_p(s.cuda_stream), v), "dpe_read_error")
        if v.value:
            names = [nm for bit, nm in _lib.DEVERR_BITS.items() if v.value & bit]
            raise RuntimeError(f"patch encoder device error: {', '.join(names)} (0x{v.value:x})")

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.L.dpe_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DecodeGraph:
    """One captured ``dpe_decode`` over static device buffers (``inputs``:
    patches [n, patch, ld] bf16 and rows [n] int32; ``out`` [n, out_dim]).
    The warm-up call that plans the workspace runs on rows 0..n-1, whose
    lengths and conv tails are restored afterwards; the K/V it wrote lie past
    those lengths and are never read."""

    def __init__(self, pe: B200PatchEncoder, n: int):
        c, dev = pe.cfg, pe.device
        if not 1 <= n <= min(pe.max_batch, pe.max_rows):
            raise RuntimeError(f"graph for {n} requests (max {min(pe.max_batch, pe.max_rows)})")
        self.pe, self.n = pe, n
        self.inputs = {"patches": torch.zeros(n, c.patch, c.latent_dim, dtype=torch.bfloat16, device=dev),
                       "rows": torch.arange(n, dtype=torch.int32, device=dev)}
        self.out = torch.zeros(n, c.out_dim, dtype=torch.bfloat16, device=dev)
        saved = (pe.seqlens.clone(), pe.conv_tail.clone())
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            pe.launch(self.inputs["patches"], self.inputs["rows"], self.out, stream=side)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        pe.seqlens.copy_(saved[0])
        pe.conv_tail.copy_(saved[1])
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            pe.launch(self.inputs["patches"], self.inputs["rows"], self.out,
                      stream=torch.cuda.current_stream(dev))
        torch.cuda.synchronize(dev)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.out
