"""The LLM decode-attention oracle (``oracle/llm_attn_oracle.py``) against the
reference's own consistency pin for this path (``tests/test_llm.py::
test_paged_incremental_append_matches_oneshot`` of the reference: tokens
appended one by one through the paged cache == one-shot attention), restated
at the layer level with GQA 12/2, head_dim 128 and 256-position blocks."""
from __future__ import annotations

import torch

from oracle import llm_attn_oracle as LO


def _oneshot_last(qs, ks, vs, scale, G):
    """Causal attention of the last query over the contiguous K/V."""
    L, H, D = qs.shape
    out = torch.zeros(H, D)
    for h in range(H):
        s = (ks[:, h // G] @ qs[-1, h]) * scale
        out[h] = torch.softmax(s, 0) @ vs[:, h // G]
    return out


def test_paged_token_by_token_equals_oneshot():
    g = torch.Generator().manual_seed(0)
    H, KVH, D, bs, L = 12, 2, 128, 256, 600
    scale = D ** -0.5
    qs = torch.randn(L, H, D, generator=g)
    ks = torch.randn(L, KVH, D, generator=g)
    vs = torch.randn(L, KVH, D, generator=g)
    kc = torch.full((6, bs, KVH, D), float("nan"))     # stale rows must never be read
    vc = torch.full((6, bs, KVH, D), float("nan"))
    table = [4, 1, 3]                                   # shuffled physical blocks
    for p in range(L):
        slot = torch.tensor([table[p // bs] * bs + p % bs], dtype=torch.int32)
        out = LO.decode_step(qs[p:p + 1], ks[p:p + 1], vs[p:p + 1], kc, vc, slot,
                             torch.tensor([p + 1]), [table], scale)
        if p in (0, 255, 256, L - 1):
            ref = _oneshot_last(qs[:p + 1], ks[:p + 1], vs[:p + 1], scale, H // KVH)
            assert torch.allclose(out[0], ref, atol=1e-5), p


def test_store_skips_minus_one_slots():
    kc = torch.zeros(2, 256, 2, 64)
    vc = torch.zeros(2, 256, 2, 64)
    k = torch.ones(2, 2, 64)
    LO.store_kvcache(k, 2 * k, kc, vc, torch.tensor([300, -1], dtype=torch.int32))
    assert kc[1, 44].eq(1).all() and vc[1, 44].eq(2).all()
    assert kc.sum() == 128 and vc.sum() == 256
