"""LLM paged decode attention (``dllm_decode_attention`` through
``B200DecodeAttention``) against the CPU oracle, in the shapes of the dots.tts
Qwen2 backbone (GQA 12 query / 2 kv heads, head_dim 128, 256-position blocks).

Tolerance (bf16 q/k/v, fp32 scores and accumulation, bf16 output): per
(sequence, head) cosine >= 0.9999 and max-abs <= 1e-2 against fp32."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from nanovllm_dots_b200.llm_attention import B200DecodeAttention
from oracle import llm_attn_oracle as LO

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _case(ctx, H=12, KVH=2, D=128, bs=256, seed=0, extra_blocks=3):
    g = torch.Generator().manual_seed(seed)
    n = len(ctx)
    nblk = [(c + bs - 1) // bs for c in ctx]
    num_blocks = sum(nblk) + extra_blocks
    perm = torch.randperm(num_blocks, generator=g).tolist()
    width = max(nblk)
    table = torch.full((n, width), -1, dtype=torch.int32)
    o = 0
    for i, b in enumerate(nblk):
        table[i, :b] = torch.tensor(perm[o:o + b], dtype=torch.int32)
        o += b
    # unused cache rows hold NaN, as an uninitialised cache may
    kc = torch.full((num_blocks, bs, KVH, D), float("nan")).to(torch.bfloat16)
    vc = torch.full((num_blocks, bs, KVH, D), float("nan")).to(torch.bfloat16)
    for i, c in enumerate(ctx):
        for p in range(c - 1):              # the history; the last token is this step's
            b = int(table[i, p // bs])
            kc[b, p % bs] = torch.randn(KVH, D, generator=g).to(torch.bfloat16)
            vc[b, p % bs] = torch.randn(KVH, D, generator=g).to(torch.bfloat16)
    q = torch.randn(n, H, D, generator=g).to(torch.bfloat16)
    k = torch.randn(n, KVH, D, generator=g).to(torch.bfloat16)
    v = torch.randn(n, KVH, D, generator=g).to(torch.bfloat16)
    slot = torch.tensor([int(table[i, (c - 1) // bs]) * bs + (c - 1) % bs for i, c in enumerate(ctx)],
                        dtype=torch.int32)
    return q, k, v, kc, vc, slot, torch.tensor(ctx, dtype=torch.int32), table


def _run(case, H=12, KVH=2, D=128, bs=256, max_batch=8):
    q, k, v, kc, vc, slot, cl, table = case
    dec = B200DecodeAttention(H, D, D ** -0.5, KVH, max_batch=max_batch, max_blocks=table.shape[1],
                              block_size=bs, device=DEV)
    d = lambda t: t.to(DEV).contiguous()
    kcd, vcd = d(kc), d(vc)
    out = dec.decode(d(q), d(k), d(v), kcd, vcd, d(slot), d(cl), d(table))
    dec.check_errors()
    return out.float().cpu(), kcd.cpu(), vcd.cpu(), dec


def _check(got, ref, label):
    got, ref = got.reshape(-1, got.shape[-1]), ref.reshape(-1, ref.shape[-1])
    c = F.cosine_similarity(got, ref, dim=-1).min().item()
    e = (got - ref).abs().max().item()
    assert c >= 0.9999 and e <= 1e-2, f"{label}: cos_min={c:.6f} max_abs={e:.4g}"


def test_ragged_batch_matches_oracle():
    """Lengths across sub-tile, block and split-key chunk boundaries, shuffled
    physical blocks, NaN in every unused cache row."""
    ctx = [1, 63, 64, 257, 700, 1300]
    case = _case(ctx)
    q, k, v, kc, vc, slot, cl, table = case
    got, kcd, vcd, _ = _run(case)
    kr, vr = kc.clone(), vc.clone()
    ref = LO.decode_step(q, k, v, kr, vr, slot, cl, table.tolist(), 128 ** -0.5)
    _check(got, ref, "ragged")
    # the store wrote exactly this step's rows
    for i, s in enumerate(slot.tolist()):
        b, r = divmod(s, 256)
        assert torch.equal(kcd[b, r], k[i]) and torch.equal(vcd[b, r], v[i])


def test_head_dim_64_four_heads_per_group():
    ctx = [5, 130, 513]
    case = _case(ctx, H=8, KVH=2, D=64, bs=128, seed=3)
    q, k, v, kc, vc, slot, cl, table = case
    got, *_ = _run(case, H=8, KVH=2, D=64, bs=128)
    ref = LO.decode_step(q, k, v, kc.clone(), vc.clone(), slot, cl, table.tolist(), 64 ** -0.5)
    _check(got, ref, "d64")


def test_graph_replay_equals_eager():
    case = _case([300, 1000, 17], seed=5)
    q, k, v, kc, vc, slot, cl, table = case
    dec = B200DecodeAttention(12, 128, 128 ** -0.5, 2, max_batch=4, max_blocks=table.shape[1],
                              device=DEV)
    d = lambda t: t.to(DEV).contiguous()
    qd, kd, vd, sd, cld, td = d(q), d(k), d(v), d(slot), d(cl), d(table)
    kcd, vcd = d(kc), d(vc)
    eager = dec.decode(qd, kd, vd, kcd, vcd, sd, cld, td).clone()
    out = torch.empty_like(eager)
    dec.decode(qd, kd, vd, kcd, vcd, sd, cld, td, out=out)      # warm-up outside capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        dec.decode(qd, kd, vd, kcd, vcd, sd, cld, td, out=out, stream=torch.cuda.current_stream())
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    dec.check_errors()


def test_bad_block_id_is_reported():
    case = _case([40, 300], seed=7)
    q, k, v, kc, vc, slot, cl, table = case
    table = table.clone()
    table[1, 1] = 10_000                         # past the cache
    dec = B200DecodeAttention(12, 128, 128 ** -0.5, 2, max_batch=2, max_blocks=table.shape[1],
                              device=DEV)
    d = lambda t: t.to(DEV).contiguous()
    dec.decode(d(q), None, None, d(kc), d(vc), None, d(cl), d(table))
    with pytest.raises(RuntimeError, match="page"):
        dec.check_errors()
