"""Pins the patch-encoder oracle (``oracle/pe_oracle.py``) against the golden
fixtures written by ``tests/golden/make_golden_pe.py`` from the reference's own
``VAESemanticEncoder.decode_patch`` / ``prefill``."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from nanovllm_dots_b200 import synthetic as syn
from oracle import pe_oracle as PO

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden", "pe_golden.npz")
SMALL = syn.PEConfig(layers=2, hidden=128, heads=2, ffn=256, out_dim=192)


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


@pytest.fixture(scope="module")
def manifest():
    with open(os.path.join(HERE, "golden", "pe_manifest.json")) as f:
        return json.load(f)


def _close(a, b, tol=1e-4):
    a, b = torch.as_tensor(a).float(), torch.as_tensor(b).float()
    assert a.shape == b.shape
    err = (a - b).abs().max().item()
    scale = b.abs().max().item()
    assert err <= tol * max(1.0, scale), f"max abs err {err:.3g} (scale {scale:.3g})"


def test_weights_match_fixture(manifest):
    assert syn.weights_digest(syn.make_pe_weights(SMALL)) == manifest["small_weights_sha256"]


def test_small_decode(gold):
    w = syn.make_pe_weights(SMALL)
    patches = torch.from_numpy(gold["small_decode_patches"])
    P, n = patches.shape[:2]
    states = [PO.PEState(SMALL) for _ in range(n)]
    for p in range(P):
        got = PO.decode_batch(w, SMALL, states, patches[p])
        _close(got, gold["small_decode_out"][p])
    assert states[0].seq_len == P * SMALL.rows


def test_small_prefill_then_decode(gold):
    w = syn.make_pe_weights(SMALL)
    st = PO.PEState(SMALL)
    _close(PO.prefill(w, SMALL, st, torch.from_numpy(gold["small_prefill_prompt"])),
           gold["small_prefill_out"])
    tail = torch.from_numpy(gold["small_prefill_tail"])
    for p in range(tail.shape[0]):
        _close(PO.decode_patch(w, SMALL, st, tail[p]), gold["small_prefill_dec"][p])


def test_prefill_equals_patch_by_patch_decode(gold):
    """The whole-prompt causal pass equals decoding the prompt one patch at a
    time from an empty state (the zero conv pad is the empty state's tail)."""
    w = syn.make_pe_weights(SMALL)
    prompt = torch.from_numpy(gold["small_prefill_prompt"])
    a, b = PO.PEState(SMALL), PO.PEState(SMALL)
    pre = PO.prefill(w, SMALL, a, prompt)
    dec = torch.stack([PO.decode_patch(w, SMALL, b, prompt[16 * p:16 * (p + 1)])
                       for p in range(prompt.shape[0] // 16)])
    _close(dec, pre)
    for l in range(SMALL.layers):
        _close(a.k[l], b.k[l])
        _close(a.v[l], b.v[l])


def test_full_decode(gold, manifest):
    w = syn.make_pe_weights(syn.PE_BASE)
    assert syn.weights_digest(w) == manifest["full_weights_sha256"]
    patches = torch.from_numpy(gold["full_decode_patches"])
    states = [PO.PEState(syn.PE_BASE) for _ in range(patches.shape[1])]
    for p in range(patches.shape[0]):
        _close(PO.decode_batch(w, syn.PE_BASE, states, patches[p]), gold["full_decode_out"][p])
