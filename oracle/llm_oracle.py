"""CPU oracle for one decode step of the LLM backbone -- TEST INFRASTRUCTURE ONLY.

Only tests and ``bench.py``'s CPU-baseline leg use this module, as the checker
or the timed CPU baseline; the product path never imports it.

It restates, in fp32 torch on the CPU, ``QwenLLM.forward`` as driven one token
per sequence by ``BatchedPagedLLM._decode_batch``
(``nanovllm_dots/models/dots/model_llm.py:113-171``, ``batched_llm.py:177-236``):

* per layer ``QwenDecoderLayer.forward`` (``model_llm.py:138-147``):
  ``h = h + o_proj(attn(rope(qkv_proj(rms(h)))))``, then
  ``h = h + down(silu(gate(rms(h))) * up(rms(h)))``;
* ``RMSNorm`` (``layers/layernorm.py:17-26``): x * rsqrt(mean(x^2) + eps) * w;
* q/k/v with bias, o_proj / gate / up / down without (``model_llm.py:57-70, 98-111``);
* NeoX rotary at the token's position, inv_freq = base^(-2i/D)
  (``layers/rotary_embedding.py:6-47``);
* the paged decode attention of ``oracle/llm_attn_oracle.py`` (store the
  token's K/V at its slot, attend over ``context_lens`` positions);
* the final ``norm`` (``model_llm.py:165-171``).

Pin: ``tests/golden/make_golden_llm.py`` runs HuggingFace transformers'
``Qwen2Model`` (the reference's own ground truth for this backbone,
``tests/test_llm.py::test_qwen_backbone_matches_huggingface``) one-shot over a
sequence; ``tests/test_llm_oracle.py`` decodes the same sequence token by token
through this oracle's paged cache and matches every position.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from nanovllm_dots_b200.synthetic import LLM_BASE, LLMConfig
from oracle import llm_attn_oracle as LO


def rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def rope(x, pos, cfg: LLMConfig):
    """x [n, heads, D], pos [n] -> NeoX rotary in fp32."""
    D = cfg.head_dim
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, D, 2, dtype=torch.float) / D))
    f = pos.float()[:, None] * inv[None]                  # [n, D/2]
    c, s = f.cos()[:, None], f.sin()[:, None]
    x1, x2 = x[..., : D // 2], x[..., D // 2:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def decode_step(w, cfg: LLMConfig, embeds, positions, k_caches, v_caches, slot_mapping,
                context_lens, block_table) -> torch.Tensor:
    """embeds [n, hidden] -> hidden states [n, hidden] (after the final norm);
    k_caches / v_caches: per-layer [num_blocks, block_size, kv_heads, D] tensors,
    updated in place with this step's K/V."""
    n = embeds.shape[0]
    H, D = cfg.heads, cfg.head_dim
    h = embeds.float()
    for l in range(cfg.layers):
        p = f"layers.{l}"
        x = rms(h, w[f"{p}.input_layernorm.weight"], cfg.rms_eps)
        q = x @ w[f"{p}.self_attn.q_proj.weight"].t() + w[f"{p}.self_attn.q_proj.bias"]
        k = x @ w[f"{p}.self_attn.k_proj.weight"].t() + w[f"{p}.self_attn.k_proj.bias"]
        v = x @ w[f"{p}.self_attn.v_proj.weight"].t() + w[f"{p}.self_attn.v_proj.bias"]
        q = rope(q.view(n, H, D), positions, cfg)
        k = rope(k.view(n, cfg.kv_heads, D), positions, cfg)
        v = v.view(n, cfg.kv_heads, D)
        o = LO.decode_step(q, k, v, k_caches[l], v_caches[l], slot_mapping, context_lens,
                           block_table, D ** -0.5)
        h = h + o.reshape(n, H * D) @ w[f"{p}.self_attn.o_proj.weight"].t()
        x = rms(h, w[f"{p}.post_attention_layernorm.weight"], cfg.rms_eps)
        a = F.silu(x @ w[f"{p}.mlp.gate_proj.weight"].t()) * (x @ w[f"{p}.mlp.up_proj.weight"].t())
        h = h + a @ w[f"{p}.mlp.down_proj.weight"].t()
    return rms(h, w["norm.weight"], cfg.rms_eps)
