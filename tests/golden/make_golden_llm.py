"""Generate the golden LLM-backbone fixture with HuggingFace transformers' Qwen2.

The reference checks its Qwen2 backbone against ``transformers``'
``Qwen2ForCausalLM`` (``tests/test_llm.py::test_qwen_backbone_matches_huggingface``
of the reference) and its paged decode against a one-shot forward
(``test_paged_incremental_append_matches_oneshot``).  This script runs
``transformers.Qwen2Model`` one-shot (fp32, eager attention, CPU) over a short
sequence of input embeddings with the seeded weights of
``nanovllm_dots_b200.synthetic.make_llm_weights`` and records the final hidden
state of every position; ``tests/test_llm_oracle.py`` decodes the same sequence
token by token through the oracle's paged cache.

    python tests/golden/make_golden_llm.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from nanovllm_dots_b200 import synthetic as syn  # noqa: E402

SMALL = syn.LLMConfig(layers=2, hidden=256, heads=2, kv_heads=1, head_dim=128, inter=512)
T = 40


def main():
    import transformers
    from transformers import Qwen2Config, Qwen2Model

    c = SMALL
    cfg = Qwen2Config(vocab_size=32, hidden_size=c.hidden, intermediate_size=c.inter,
                      num_hidden_layers=c.layers, num_attention_heads=c.heads,
                      num_key_value_heads=c.kv_heads, max_position_embeddings=256,
                      rms_norm_eps=c.rms_eps, attn_implementation="eager")
    if hasattr(cfg, "rope_parameters"):
        cfg.rope_parameters = {"rope_type": "default", "rope_theta": c.rope_theta}
    else:
        cfg.rope_theta = c.rope_theta
    torch.manual_seed(0)
    model = Qwen2Model(cfg).eval()
    w = syn.make_llm_weights(c)
    sd = dict(w)
    sd["embed_tokens.weight"] = model.embed_tokens.weight.detach()
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected and all("rotary" in m for m in missing), (missing, unexpected)
    g = torch.Generator().manual_seed(1)
    embeds = torch.randn(1, T, c.hidden, generator=g).to(torch.bfloat16).float()
    with torch.no_grad():
        out = model(inputs_embeds=embeds, use_cache=False).last_hidden_state[0]
    np.savez_compressed(os.path.join(HERE, "llm_golden.npz"), embeds=embeds[0].numpy(),
                        out=out.numpy())
    with open(os.path.join(HERE, "llm_manifest.json"), "w") as f:
        json.dump({"transformers": transformers.__version__, "T": T,
                   "weights_sha256": syn.weights_digest(w),
                   "config": {"layers": c.layers, "hidden": c.hidden, "heads": c.heads,
                              "kv_heads": c.kv_heads, "head_dim": c.head_dim, "inter": c.inter,
                              "rms_eps": c.rms_eps, "rope_theta": c.rope_theta}}, f, indent=1)
    print("wrote", out.shape)


if __name__ == "__main__":
    main()
