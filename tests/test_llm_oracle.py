"""Pins the LLM decode-step oracle (``oracle/llm_oracle.py``) against the golden
fixture written by ``tests/golden/make_golden_llm.py`` (HuggingFace
transformers' ``Qwen2Model`` one-shot over 40 positions): the same sequence
decoded one token per step through the oracle's paged cache (shuffled 16-position
blocks) must reproduce every position's final hidden state."""
from __future__ import annotations

import json
import os

import numpy as np
import torch

from nanovllm_dots_b200 import synthetic as syn
from oracle import llm_oracle as LLO

HERE = os.path.dirname(os.path.abspath(__file__))


def test_paged_decode_matches_hf_qwen2_oneshot():
    with open(os.path.join(HERE, "golden", "llm_manifest.json")) as f:
        man = json.load(f)
    c = syn.LLMConfig(**{k: man["config"][k] for k in
                         ("layers", "hidden", "heads", "kv_heads", "head_dim", "inter", "rms_eps",
                          "rope_theta")}, block_size=16)
    w = syn.make_llm_weights(c)
    assert syn.weights_digest(w) == man["weights_sha256"]
    g = np.load(os.path.join(HERE, "golden", "llm_golden.npz"))
    embeds, ref = torch.from_numpy(g["embeds"]), torch.from_numpy(g["out"])
    T = embeds.shape[0]
    table = [3, 0, 2]                                 # 48 positions in shuffled blocks
    kc = [torch.full((4, 16, c.kv_heads, c.head_dim), float("nan")) for _ in range(c.layers)]
    vc = [torch.full((4, 16, c.kv_heads, c.head_dim), float("nan")) for _ in range(c.layers)]
    for p in range(T):
        slot = torch.tensor([table[p // 16] * 16 + p % 16], dtype=torch.int32)
        out = LLO.decode_step(w, c, embeds[p:p + 1], torch.tensor([p]), kc, vc, slot,
                              torch.tensor([p + 1]), [table])
        err = (out[0] - ref[p]).abs().max().item()
        assert err <= 1e-4 * max(1.0, ref[p].abs().max().item()), (p, err)
