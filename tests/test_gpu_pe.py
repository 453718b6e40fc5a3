"""Patch-encoder parity: ``dpe_decode`` through the C ABI (``B200PatchEncoder``)
against the golden vectors made by the reference's ``VAESemanticEncoder`` and
against the CPU oracle (``oracle/pe_oracle.py``), in the reference tests'
patterns (``tests/test_patch_encoder.py`` of the reference: rows advanced in a
reversed permutation at different history lengths; prefill then decode).

Tolerance (bf16 operands, fp32 accumulation and residual stream, bf16 output):
per-request embedding cosine >= 0.9999 and max-abs <= 3e-2 against the fp32
reference (embeddings reach |x| ~ 2, where one bf16 step is 1.6e-2)."""
from __future__ import annotations

import functools
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from nanovllm_dots_b200 import synthetic as syn
from nanovllm_dots_b200.patch_encoder import B200PatchEncoder
from oracle import pe_oracle as PO

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
COS, MAXABS = 0.9999, 3e-2
CFG = syn.PE_BASE
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "pe_golden.npz")


@functools.lru_cache(maxsize=1)
def _weights():
    return syn.make_pe_weights(CFG)


@pytest.fixture(scope="module")
def pe():
    enc = B200PatchEncoder(_weights(), CFG, max_batch=8, max_seq_len=2048, device=DEV)
    yield enc
    enc.close()


def _check(got, ref, label):
    got, ref = got.float().cpu().reshape(ref.shape[0], -1), ref.float().reshape(ref.shape[0], -1)
    c = F.cosine_similarity(got, ref, dim=-1).min().item()
    e = (got - ref).abs().max().item()
    assert c >= COS and e <= MAXABS, f"{label}: cos_min={c:.6f} max_abs={e:.4g}"


def test_full_decode_golden(pe):
    """Two requests, two patches each, against the reference's own decode_patch."""
    g = np.load(GOLD)
    patches = torch.from_numpy(g["full_decode_patches"]).to(torch.bfloat16)
    pe.reset_rows([0, 1])
    for p in range(patches.shape[0]):
        out = pe.decode_patch(patches[p], [0, 1])
        pe.check_errors()
        _check(out[:, 0], torch.from_numpy(g["full_decode_out"][p]), f"golden patch {p}")


def test_decode_reversed_rows_different_lengths(pe):
    """Five requests in cache rows 4..0, started at different ticks so their
    histories differ in length; every call checked against the oracle."""
    w = _weights()
    n, P = 5, 6
    rows = list(reversed(range(n)))
    pe.reset_rows(rows)
    states = [PO.PEState(CFG) for _ in range(n)]
    patches = syn.make_pe_patches(n, P, seed=21)
    for p in range(P):
        live = [i for i in range(n) if p >= i // 2]          # request i joins at tick i // 2
        got = pe.decode_patch(patches[p, live], [rows[i] for i in live])
        pe.check_errors()
        ref = torch.stack([PO.decode_patch(w, CFG, states[i], patches[p, i]) for i in live])
        _check(got[:, 0], ref, f"tick {p}")
    assert pe.seqlens[rows[0]].item() == P * CFG.rows


def test_prefill_then_decode(pe):
    """A 22-patch prompt through prefill, then decode steps that continue it
    (the reference's ``test_flash_pe_prefill_matches_reference`` sizes)."""
    w = _weights()
    prompt = syn.make_pe_patches(1, 22, seed=22)[:, 0].reshape(-1, CFG.latent_dim)
    st = PO.PEState(CFG)
    ref = PO.prefill(w, CFG, st, prompt)
    got = pe.prefill(prompt.unsqueeze(0), 6)
    pe.check_errors()
    assert got.shape == (1, 22, CFG.out_dim)
    _check(got[0], ref, "prefill")
    tail = syn.make_pe_patches(1, 4, seed=23)[:, 0]
    for p in range(tail.shape[0]):
        out = pe.decode_patch(tail[p:p + 1], [6])
        pe.check_errors()
        _check(out[:, 0], PO.decode_patch(w, CFG, st, tail[p]).unsqueeze(0), f"post-prefill {p}")


def test_long_histories_batched_prime(pe):
    """Rows primed with histories of 240 and 90 patches (1920 and 720
    positions, up to the 2048-position capacity) next to a fresh row, then one
    batched decode."""
    w = _weights()
    lens = [240, 90]
    prompts = [syn.make_pe_patches(1, L, seed=30 + i)[:, 0].reshape(-1, CFG.latent_dim)
               for i, L in enumerate(lens)]
    outs = pe.prime([2, 3], prompts)
    pe.check_errors()
    states = []
    for i, pr in enumerate(prompts):
        st = PO.PEState(CFG)
        ref = PO.prefill(w, CFG, st, pr)
        _check(outs[i][-4:], ref[-4:], f"prime row {i}")
        states.append(st)
    pe.reset_rows([5])
    states.append(PO.PEState(CFG))
    patches = syn.make_pe_patches(3, 1, seed=33)[0]
    got = pe.decode_patch(patches, [2, 3, 5])
    pe.check_errors()
    ref = torch.stack([PO.decode_patch(w, CFG, states[i], patches[i]) for i in range(3)])
    _check(got[:, 0], ref, "after prime")


def test_graph_replay_equals_eager(pe):
    """The captured decode equals eager calls on the same state."""
    n = 4
    patches = syn.make_pe_patches(n, 3, seed=40).to(DEV)
    pe.reset_rows(range(n))
    eager = [pe.decode_patch(patches[p], list(range(n)))[:, 0].clone() for p in range(3)]
    pe.reset_rows(range(n))
    g = pe.graph(n)
    for p in range(3):
        g.inputs["patches"].copy_(patches[p])
        out = g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager[p]), f"graph replay differs at patch {p}"
    pe.check_errors()


def test_full_row_reports_length_error(pe):
    """A row already at capacity: the call reports DFM_DEVERR_LEN and writes
    no K/V (host-visible error, no fault)."""
    pe.reset_rows([7])
    pe.seqlens[7] = pe.cap
    pe.decode_patch(torch.zeros(1, CFG.patch, CFG.latent_dim), [7])
    with pytest.raises(RuntimeError, match="len"):
        pe.check_errors()
    pe.reset_rows([7])


def test_large_batch_wide_tiles():
    """136 requests in one call (1088 encoder rows, past the small-call
    threshold): the layer GEMMs take the 256 x 256 tiles with two split-K
    partials; rows in a shuffled order."""
    w = _weights()
    n = 136
    enc = B200PatchEncoder(w, CFG, max_batch=n, max_seq_len=256, device=DEV)
    try:
        rows = torch.randperm(n, generator=torch.Generator().manual_seed(3)).tolist()
        states = [PO.PEState(CFG) for _ in range(n)]
        patches = syn.make_pe_patches(n, 2, seed=50)
        for p in range(2):
            got = enc.decode_patch(patches[p], rows)
            enc.check_errors()
            ref = PO.decode_batch(w, CFG, states, patches[p])
            _check(got[:, 0], ref, f"wide patch {p}")
    finally:
        enc.close()
