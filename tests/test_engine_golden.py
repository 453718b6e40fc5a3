"""The oracle against golden vectors made by the reference's own engine code
(``tests/golden/make_golden_engine.py``: ``DotsBatchEngine._pack_fm_inputs`` +
``batched_meanflow`` over histories built by ``DotsModel._append_hidden_chunk``
/ ``_append_history_chunk``): a request's tick computed through the paged
cache formulation from its history rows equals the reference's padded full
path, for a request with no prompt, one with a voice-clone prompt, and one
with a speaker condition that joins late."""
from __future__ import annotations

import json
import os

import numpy as np
import torch

from conftest import GOLDEN
from nanovllm_dots_b200 import synthetic as syn
from oracle import dit_oracle as O


def load_engine_golden():
    """(manifest, arrays) with bf16 fields decoded to bf16 tensors."""
    with open(os.path.join(GOLDEN, "engine_manifest.json")) as f:
        man = json.load(f)
    raw = dict(np.load(os.path.join(GOLDEN, "engine_golden.npz")))
    arr = {}
    for k, v in raw.items():
        t = torch.from_numpy(v)
        arr[k] = t.view(torch.bfloat16) if t.dtype == torch.int16 else t
    return man, arr


def test_oracle_matches_reference_engine_ticks(weights):
    man, arr = load_engine_golden()
    assert man["weights_sha256"] == syn.weights_digest(weights)
    cfg = syn.BASE
    for t, tk in enumerate(man["ticks"]):
        for j, (name, L) in enumerate(zip(tk["requests"], tk["fm_seq_len"])):
            rows = arr[f"{name}_fm_sequence"][:L]
            g = arr.get(f"{name}_g_cond")
            z = O.history_tick(weights, cfg, rows, arr[f"tick{t}_noise"][j].float(),
                               None if g is None else g.float())
            err = (z - arr[f"tick{t}_z"][j]).abs().max().item()
            assert err < 1e-4, (t, name, err)
