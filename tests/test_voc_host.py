"""Host-side checks of the vocoder (no GPU): the C ABI's layer tables and the
Python packer agree, and the library's stream left context matches the
reference's rule (restated in ``oracle/voc_oracle.py``, pinned by the golden
window sizes) on several shapes."""
from __future__ import annotations

import ctypes
import dataclasses

import pytest

from nanovllm_dots_b200 import _lib
from nanovllm_dots_b200 import synthetic as syn
from nanovllm_dots_b200.vocoder import dvoc_config, pack_voc_weights
from oracle import voc_oracle as vo

SHAPES = [
    syn.VOC_SMALL,
    syn.VOC_BASE,
    dataclasses.replace(syn.VOC_SMALL, resblock="2", resblock_dilations=((1, 3, 1), (1, 3, 1), (1, 3, 1))),
    dataclasses.replace(syn.VOC_SMALL, resblock_kernel_sizes=(3, 5), resblock_dilations=((1, 2, 4), (1, 3, 9)),
                        lookahead=0, upsample_rates=(5, 3)),
    dataclasses.replace(syn.VOC_SMALL, activation="snake", latent_dim=48, initial_channels=96),
]


@pytest.mark.parametrize("cfg", SHAPES, ids=range(len(SHAPES)))
def test_tables_match_packer(cfg):
    L = _lib.lib()
    c = dvoc_config(cfg, 4, 64)
    w = pack_voc_weights(syn.make_voc_weights(cfg, seed=3), cfg, device="cpu")
    assert w["conv_w"].numel() == L.dvoc_conv_floats(ctypes.byref(c))
    assert w["conv_b"].numel() == L.dvoc_bias_floats(ctypes.byref(c))
    assert w["act"].numel() == L.dvoc_act_floats(ctypes.byref(c))
    assert L.dvoc_hop(ctypes.byref(c)) == cfg.hop
    assert L.dvoc_stream_left_context(ctypes.byref(c)) == vo.stream_left_context(cfg)


def test_unsupported_shapes():
    L = _lib.lib()
    bad = [dataclasses.replace(syn.VOC_SMALL, latent_dim=33),
           dataclasses.replace(syn.VOC_SMALL, latent_dim=1024)]
    for cfg in bad:
        assert L.dvoc_conv_floats(ctypes.byref(dvoc_config(cfg, 4, 64))) == 0
    c = dvoc_config(syn.VOC_SMALL, 4, 64)
    c.resblock_type = 3
    assert L.dvoc_act_floats(ctypes.byref(c)) == 0
    h = ctypes.c_void_p()
    assert L.dvoc_create(ctypes.byref(c), ctypes.byref(_lib.DvocWeights()), ctypes.byref(h)) != 0
