"""Paged decode attention of the LLM backbone on the B200 kernels (``include/dllm.h``).

The reference's ``Attention`` layer (``nanovllm_dots/layers/attention.py:50-97``)
stores each step's K/V with a Triton kernel and attends with flash-attn's
``flash_attn_with_kvcache`` (sm_80 FA2).  ``B200DecodeAttention.decode`` is that
decode branch as one ``dllm_decode_attention`` call on the caller's stream;
``install_decode_attention`` routes a reference ``Attention`` module's decode
steps through it (prefill keeps the module's own path).  There is no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib


class B200DecodeAttention:
    """Decode attention for one model: GQA shape, cache geometry and a
    workspace sized for ``max_batch`` sequences of ``max_blocks`` blocks."""

    def __init__(self, num_heads: int, head_dim: int, scale: float, num_kv_heads: int, *,
                 max_batch: int, max_blocks: int, block_size: int = 256,
                 device: torch.device | str = "cuda"):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("B200DecodeAttention runs on a CUDA device only (no CPU path)")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.num_heads, self.head_dim, self.scale = num_heads, head_dim, float(scale)
        self.num_kv_heads = num_kv_heads
        self.max_batch, self.max_blocks, self.block_size = max_batch, max_blocks, block_size
        self.L = _lib.lib()
        ws = int(self.L.dllm_decode_workspace_size(max_batch, num_heads, head_dim, max_blocks,
                                                   block_size))
        if ws == 0:
            raise RuntimeError("unsupported decode-attention shape")
        self.ws_bytes = ws
        self.workspace = torch.zeros(ws, dtype=torch.uint8, device=self.device)

    def decode(self, q, k, v, k_cache, v_cache, slot_mapping, context_lens, block_tables,
               out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """q [n, H, D] (after rotary), k / v [n, KVH, D] (or None with
        slot_mapping None), caches [num_blocks, block_size, KVH, D], int32
        slot_mapping [n], context_lens [n], block_tables [n, width <=
        max_blocks] -> [n, H, D] bf16."""
        n = q.shape[0]
        if not 1 <= n <= self.max_batch:
            raise RuntimeError(f"decode with {n} sequences (max {self.max_batch})")
        if block_tables.shape[1] > self.max_blocks:
            raise RuntimeError(f"block table width {block_tables.shape[1]} > {self.max_blocks}")
        for name, t, dt in (("q", q, torch.bfloat16), ("k", k, torch.bfloat16),
                            ("v", v, torch.bfloat16), ("k_cache", k_cache, torch.bfloat16),
                            ("v_cache", v_cache, torch.bfloat16),
                            ("slot_mapping", slot_mapping, torch.int32),
                            ("context_lens", context_lens, torch.int32),
                            ("block_tables", block_tables, torch.int32)):
            if t is not None and (t.dtype != dt or t.device != self.device or not t.is_contiguous()):
                raise RuntimeError(f"{name}: expected a contiguous {dt} tensor on {self.device}")
        if tuple(k_cache.shape[1:]) != (self.block_size, self.num_kv_heads, self.head_dim):
            raise RuntimeError("k_cache shape does not match the decode-attention geometry")
        if out is None:
            out = torch.empty(n, self.num_heads, self.head_dim, dtype=torch.bfloat16,
                              device=self.device)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        _lib.check(self.L.dllm_decode_attention(
            _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(k_cache), _lib.ptr(v_cache),
            _lib.ptr(slot_mapping), _lib.ptr(context_lens), _lib.ptr(block_tables), n,
            self.num_heads, self.num_kv_heads, self.head_dim, k_cache.shape[0], self.block_size,
            block_tables.shape[1], self.scale, _lib.ptr(out), _lib.ptr(self.workspace),
            self.ws_bytes, _lib.c_void_p(s.cuda_stream)), "dllm_decode_attention")
        return out

    def check_errors(self) -> None:
        """Synchronise and raise if a kernel reported a device-side error."""
        v = _lib.c_uint32(0)
        s = torch.cuda.current_stream(self.device)
        _lib.check(self.L.dllm_read_error(_lib.ptr(self.workspace), _lib.c_void_p(s.cuda_stream), v),
                   "dllm_read_error")
        if v.value:
            names = [nm for bit, nm in _lib.DEVERR_BITS.items() if v.value & bit]
            raise RuntimeError(f"decode attention device error: {', '.join(names)} (0x{v.value:x})")


def install_decode_attention(module, get_context, dec: B200DecodeAttention) -> None:
    """Route a reference ``Attention`` module's decode steps through ``dec``.

    ``get_context`` is the reference's ``nanovllm_dots.utils.context.get_context``
    (passed in, so this package does not import the reference).  When the
    context is a decode step (``is_prefill`` false) the module's forward becomes
    ``dec.decode`` over its ``k_cache`` / ``v_cache`` with the context's
    ``slot_mapping``, ``context_lens`` and ``block_tables``
    (``attention.py:66-97``); prefill and non-causal calls keep the original
    forward."""
    original = module.forward

    def forward(q, k, v):
        ctx = get_context()
        if not getattr(module, "is_causal", True) or ctx.is_prefill or not module.k_cache.numel():
            return original(q, k, v)
        qh = q.view(-1, module.num_heads, module.head_dim)
        kh = k.view(-1, module.num_kv_heads, module.head_dim)
        vh = v.view(-1, module.num_kv_heads, module.head_dim)
        return dec.decode(qh, kh, vh, module.k_cache, module.v_cache, ctx.slot_mapping,
                          ctx.context_lens, ctx.block_tables)

    module.forward = forward
