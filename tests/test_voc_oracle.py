"""The vocoder oracle (``oracle/voc_oracle.py``) against golden vectors made
by the reference's own ``AudioVAE`` (``tests/golden/make_golden_voc.py``):
one-shot decode of two utterances and two strict streams (one long enough
for the decoder window to slide), every emitted piece compared.  The
reference ran in fp32, the oracle in float64: max-abs <= 2e-5 on audio in
[-1, 1]."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from nanovllm_dots_b200 import synthetic as syn
from oracle import voc_oracle as vo

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TOL = 2e-5


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLDEN, "voc_manifest.json")) as f:
        man = json.load(f)
    arr = dict(np.load(os.path.join(GOLDEN, "voc_golden.npz")))
    return man, arr


@pytest.fixture(scope="module")
def voc():
    w = syn.make_voc_weights(syn.VOC_SMALL, seed=0)
    return vo.VocOracle(w, syn.VOC_SMALL)


def test_weights_match_fixture(golden):
    man, _ = golden
    w = syn.make_voc_weights(syn.VOC_SMALL, seed=0)
    assert syn.weights_digest(w) == man["weights_sha256"]
    assert man["config"] == syn.VOC_SMALL.reference_dict()


def test_window_size(golden):
    man, _ = golden
    for s in man["streams"].values():
        assert vo.stream_window(syn.VOC_SMALL, man["chunk"]) == s["window"]


def test_oneshot(golden, voc):
    man, arr = golden
    for i, T in enumerate(man["oneshot_frames"]):
        lat = torch.from_numpy(arr[f"oneshot{i}_latents"])[None]
        got = voc.inference(lat)[0].numpy()
        ref = arr[f"oneshot{i}_audio"]
        assert got.shape == ref.shape == (T * syn.VOC_SMALL.hop,)
        assert np.abs(got - ref).max() <= TOL


def test_streams(golden, voc):
    man, arr = golden
    chunk = man["chunk"]
    for name, s in man["streams"].items():
        lat = torch.from_numpy(arr[f"stream{name}_latents"])
        st = vo.stream_init(voc, chunk)
        pieces = [vo.stream_step(voc, st, lat[k * chunk:(k + 1) * chunk]) for k in range(s["chunks"])]
        pieces.append(vo.stream_flush(voc, st))
        assert [p.numel() for p in pieces] == s["piece_samples"]
        for k, p in enumerate(pieces):
            ref = arr[f"stream{name}_piece{k}"]
            assert np.abs(p.numpy() - ref).max() <= TOL, (name, k)


def test_stream_errors(voc):
    st = vo.stream_init(voc, 8)
    with pytest.raises(ValueError, match="chunk_size must stay fixed"):
        vo.stream_step(voc, st, torch.zeros(4, syn.VOC_SMALL.latent_dim))
    with pytest.raises(ValueError):
        vo.stream_window(syn.VOC_SMALL, 0)
