"""The LLM backbone decode step (``dllm_decode_step`` through
``B200QwenDecoder``) against the fp32 oracle (``oracle/llm_oracle.py``, pinned to
HuggingFace transformers' Qwen2), at the dots.tts backbone's width (1536, GQA
12/2 x 128, MLP 8960, 256-position blocks) with two layers.

Tolerance (bf16 operands, fp32 accumulation and residual stream, bf16 output;
a CPU emulation of the bf16 operands gives cos 0.99999, max-abs 0.014 at |x|
~ 4): per-sequence cosine >= 0.9999 and max-abs <= 5e-2."""
from __future__ import annotations

import functools

import pytest
import torch
import torch.nn.functional as F

from nanovllm_dots_b200 import synthetic as syn
from nanovllm_dots_b200.llm_decode import B200QwenDecoder
from oracle import llm_oracle as LLO

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
CFG = syn.LLMConfig(layers=2)
BS = CFG.block_size


@functools.lru_cache(maxsize=1)
def _weights():
    return syn.make_llm_weights(CFG)


def _setup(ctx, seed=0, width=3):
    g = torch.Generator().manual_seed(seed)
    n = len(ctx)
    nb = sum((x + BS - 1) // BS for x in ctx) + 2
    perm = torch.randperm(nb, generator=g)
    table = torch.full((n, width), -1, dtype=torch.int32)
    o = 0
    for i, x in enumerate(ctx):
        b = (x + BS - 1) // BS
        table[i, :b] = perm[o:o + b].to(torch.int32)
        o += b
    mk = lambda: (torch.randn(nb, BS, CFG.kv_heads, CFG.head_dim, generator=g)).to(torch.bfloat16)
    kc = [mk() for _ in range(CFG.layers)]
    vc = [mk() for _ in range(CFG.layers)]
    return table, kc, vc


def _inputs(ctx, table, seed):
    g = torch.Generator().manual_seed(seed)
    emb = torch.randn(len(ctx), CFG.hidden, generator=g).to(torch.bfloat16)
    pos = torch.tensor([x - 1 for x in ctx], dtype=torch.int32)
    slot = torch.tensor([int(table[i, (x - 1) // BS]) * BS + (x - 1) % BS for i, x in enumerate(ctx)],
                        dtype=torch.int32)
    return emb, pos, slot, torch.tensor(ctx, dtype=torch.int32)


def _check(got, ref, label):
    got = got.float().cpu()
    c = F.cosine_similarity(got, ref, dim=-1).min().item()
    e = (got - ref).abs().max().item()
    assert c >= 0.9999 and e <= 5e-2, f"{label}: cos_min={c:.6f} max_abs={e:.4g}"


def test_decode_steps_match_oracle():
    """Three consecutive decode steps of four sequences (contexts 1 .. 513,
    across block and chunk boundaries); the caches written by each step feed
    the next."""
    w = _weights()
    ctx = [1, 70, 255, 511]
    table, kc, vc = _setup([x + 2 for x in ctx])     # blocks for the last step's lengths
    dec = B200QwenDecoder(w, CFG, max_batch=8, max_blocks=table.shape[1], device=DEV)
    d = lambda t: t.to(DEV).contiguous()
    kd, vd = [d(t) for t in kc], [d(t) for t in vc]
    kr, vr = [t.float() for t in kc], [t.float() for t in vc]
    td = d(table)
    try:
        for step in range(3):
            cur = [x + step for x in ctx]
            emb, pos, slot, cl = _inputs(cur, table, seed=10 + step)
            got = dec.step(d(emb), d(pos), d(slot), d(cl), td, kd, vd)
            dec.check_errors()
            ref = LLO.decode_step(w, CFG, emb, pos.long(), kr, vr, slot, cl, table.tolist())
            _check(got, ref, f"step {step}")
    finally:
        dec.close()


def test_graph_replay_equals_eager():
    w = _weights()
    ctx = [40, 300]
    table, kc, vc = _setup(ctx, seed=2)
    dec = B200QwenDecoder(w, CFG, max_batch=2, max_blocks=table.shape[1], device=DEV)
    d = lambda t: t.to(DEV).contiguous()
    emb, pos, slot, cl = [d(t) for t in _inputs(ctx, table, seed=3)]
    td = d(table)
    try:
        kd, vd = [d(t) for t in kc], [d(t) for t in vc]
        eager = dec.step(emb, pos, slot, cl, td, kd, vd).clone()
        out = torch.empty_like(eager)
        kd, vd = [d(t) for t in kc], [d(t) for t in vc]
        dec.step(emb, pos, slot, cl, td, kd, vd, out=out)      # encodes the cache descriptors
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            dec.step(emb, pos, slot, cl, td, kd, vd, out=out, stream=torch.cuda.current_stream())
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
        dec.check_errors()
    finally:
        dec.close()
