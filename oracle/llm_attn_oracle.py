"""CPU oracle for the LLM backbone's paged decode attention -- TEST
INFRASTRUCTURE ONLY.

Only tests and ``bench.py``'s CPU-baseline leg use this module, and only as the
checker or the timed CPU baseline.  The product path never imports it.

It restates, in fp32 torch on the CPU, the decode branch of the reference's
``Attention.forward`` (``nanovllm_dots/layers/attention.py:60-97``):

* ``store_kvcache`` (``attention.py:10-47``): row i of this step's k / v goes to
  cache slot ``slot_mapping[i]`` of the flattened [num_blocks * block_size,
  kv_heads * head_dim] cache, and slot -1 skips the row;
* ``flash_attn_with_kvcache(q.unsqueeze(1), k_cache, v_cache,
  cache_seqlens=context_lens, block_table=block_tables, softmax_scale,
  causal=True)`` (flash-attn 2.8.3, pinned at ``uv.lock:167-168`` of the
  reference; its published semantics): the single query of sequence i sits at
  the last of its ``context_lens[i]`` positions, so causality lets it see every
  cached position; position p is row ``p % block_size`` of block
  ``block_table[i][p // block_size]``; query head h reads kv head
  ``h // (num_heads / num_kv_heads)`` (GQA); softmax(q k^T * scale) v.

Parity note: flash-attn needs a GPU, so the reference's decode path cannot
run in this container; the oracle is pinned to the published definition and
to the reference's own consistency test for this path
(``tests/test_llm.py::test_paged_incremental_append_matches_oneshot``: paged
decode == one-shot attention), which ``tests/test_llm_attn_oracle.py``
restates at the layer level.  No golden vectors of executed reference output
exist for it ("parity unpinned" against executed reference code).
"""
from __future__ import annotations

import torch


def store_kvcache(k, v, k_cache, v_cache, slot_mapping) -> None:
    """In place: cache.view(-1, kv_heads * D)[slot] = row (``attention.py:10-47``)."""
    kc = k_cache.view(-1, k_cache.shape[-2] * k_cache.shape[-1])
    vc = v_cache.view(-1, v_cache.shape[-2] * v_cache.shape[-1])
    for i, slot in enumerate(slot_mapping.tolist()):
        if slot == -1:
            continue
        kc[slot] = k[i].reshape(-1).to(kc.dtype)
        vc[slot] = v[i].reshape(-1).to(vc.dtype)


def gather(cache, block_table_row, n_pos: int) -> torch.Tensor:
    """Positions [0, n_pos) of one sequence: [n_pos, kv_heads, D]."""
    bs = cache.shape[1]
    idx = torch.arange(n_pos)
    blocks = torch.as_tensor(block_table_row)[idx // bs]
    return cache[blocks, idx % bs].float()


def decode_attention(q, k_cache, v_cache, context_lens, block_table, scale: float) -> torch.Tensor:
    """q [n, H, D] -> out [n, H, D] (fp32)."""
    n, H, D = q.shape
    KVH = k_cache.shape[2]
    G = H // KVH
    out = torch.zeros(n, H, D)
    for i in range(n):
        L = int(context_lens[i])
        K = gather(k_cache, block_table[i], L)          # [L, KVH, D]
        V = gather(v_cache, block_table[i], L)
        for h in range(H):
            s = (K[:, h // G] @ q[i, h].float()) * scale
            out[i, h] = torch.softmax(s, dim=0) @ V[:, h // G]
    return out


def decode_step(q, k, v, k_cache, v_cache, slot_mapping, context_lens, block_table,
                scale: float) -> torch.Tensor:
    """The whole decode branch: store, then attend (the stored token included)."""
    store_kvcache(k, v, k_cache, v_cache, slot_mapping)
    return decode_attention(q, k_cache, v_cache, context_lens, block_table, scale)
