"""The C-ABI library builds, loads without a GPU and exports every entry point
``include/dfm.h``, ``include/dpe.h``, ``include/dllm.h`` and ``include/dvoc.h``
declare; host-side
bookkeeping that needs no GPU."""
from __future__ import annotations

import ctypes
import os
import pathlib
import re

import pytest
import torch

from nanovllm_dots_b200 import _lib, build
from nanovllm_dots_b200.fm_head import PageAllocator, abi_config, pack_weights
from nanovllm_dots_b200.patch_encoder import pack_pe_weights, pe_abi_config
from nanovllm_dots_b200.synthetic import BASE, PE_BASE, PEConfig, make_pe_weights

INCLUDE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
HEADER = os.path.join(INCLUDE, "dfm.h")
PE_HEADER = os.path.join(INCLUDE, "dpe.h")
LLM_HEADER = os.path.join(INCLUDE, "dllm.h")
VOC_HEADER = os.path.join(INCLUDE, "dvoc.h")


def declared_functions():
    names = set()
    for path, prefix in ((HEADER, "dfm_"), (PE_HEADER, "dpe_"), (LLM_HEADER, "dllm_"),
                         (VOC_HEADER, "dvoc_")):
        src = pathlib.Path(path).read_text()
        found = re.findall(rf"^\s*(?:int|int32_t|size_t|const char\*)\s+({prefix}\w+)\s*\(", src, re.M)
        assert found, f"no declarations parsed from {path}"
        names |= set(found)
    return sorted(names)


def test_library_builds_and_exports_every_declared_symbol():
    path = build.build()
    L = ctypes.CDLL(path)
    decl = declared_functions()
    for name in decl:
        assert hasattr(L, name), f"{name} declared in include/ but not exported"
    assert set(decl) == set(_lib.EXPORTS)


def test_struct_layouts_match_header():
    src = pathlib.Path(HEADER).read_text()
    body = src[src.index("typedef struct DfmWeights"):src.index("} DfmWeights;")]
    n_ptr = len(re.findall(r"const (?:void|float)\*\s+\w+", body))
    assert n_ptr == len(_lib.WEIGHT_FIELDS)
    assert ctypes.sizeof(_lib.DfmConfig) == 16 * 4
    assert ctypes.sizeof(_lib.DfmBatch) == 8 + 12 * 8


def test_pool_bytes_and_error_strings():
    L = _lib.lib()
    cfg = abi_config(BASE, num_pages=10, max_pages_per_req=4, max_requests=2)
    assert L.dfm_pool_bytes(cfg) == 12 * 4 * 2 * 10 * 16 * 16 * 64 * 2
    assert L.dfm_error_string(0) == b"ok"
    assert L.dfm_error_string(4) == b"workspace too small"


def test_create_rejects_bad_configs_without_a_gpu():
    L = _lib.lib()
    w = _lib.DfmWeights()
    h = ctypes.c_void_p()
    bad = abi_config(BASE, num_pages=10, max_pages_per_req=4, max_requests=2)
    bad.hidden = 768
    assert L.dfm_create(bad, w, h) == 2          # unsupported width
    good = abi_config(BASE, num_pages=10, max_pages_per_req=4, max_requests=2)
    assert L.dfm_create(good, w, h) == 1         # null weight pointers
    assert L.dfm_step(None, None, None, 0, None) == 1
    assert L.dfm_linear(None, 64, 1, 64, None, 64, 64, None, None, 0, 0, None) == 1


def test_page_allocator():
    pa = PageAllocator(num_pages=5, page_rows=16, max_pages_per_req=3)
    assert pa.ensure("a", 17) == [0, 1]
    assert pa.ensure("b", 1) == [2]
    assert pa.ensure("a", 48) == [0, 1, 3]
    with pytest.raises(RuntimeError, match="block-table"):
        pa.ensure("a", 49)
    with pytest.raises(RuntimeError, match="exhausted"):
        pa.ensure("b", 48)
    pa.release("a")
    assert pa.used() == 2 and sorted(pa.free) == [0, 1, 3]


def test_pack_weights_layout(weights):
    p = pack_weights(weights, BASE, "cpu")
    H, L, F = BASE.hidden, BASE.layers, BASE.ffn
    assert p["ada_w"].shape == (L * 6 * H + 2 * H, H) and p["ada_w"].dtype == torch.bfloat16
    assert p["qkv_w"].shape == (L, 3 * H, H)
    assert torch.equal(p["qkv_w"][3, H:2 * H].float(), weights["blocks.3.attn.k_proj.weight"])
    assert torch.equal(p["ada_w"][L * 6 * H:].float(), weights["output_layer.adaLN_modulation.1.weight"])
    assert p["qk_norm"].shape == (L, 4, 64)
    assert p["fc2_w"].shape == (L, H, F)
    assert p["rope_inv_freq"].shape == (32,)
    fp8_only = {"qkv_w8", "qkv_ws", "fc1_w8", "fc1_ws"}
    for f in _lib.WEIGHT_FIELDS:
        assert (f in p) == (f not in fp8_only)


def test_pack_weights_fp8_rowwise(weights):
    """The e4m3 copies of the QKV and fc1 matrices dequantise to the bf16
    weights within e4m3 rounding (half a unit in the last place, 3 mantissa
    bits: at most 1/16 of each value) with one scale per output row."""
    p = pack_weights(weights, BASE, "cpu", "fp8")
    H, L, F = BASE.hidden, BASE.layers, BASE.ffn
    assert p["qkv_w8"].shape == (L, 3 * H, H) and p["qkv_w8"].dtype == torch.uint8
    assert p["fc1_w8"].shape == (L, F, H) and p["fc1_ws"].shape == (L, F)
    for name in ("qkv", "fc1"):
        w = p[f"{name}_w"][:2].float()
        deq = p[f"{name}_w8"][:2].view(torch.float8_e4m3fn).float() * p[f"{name}_ws"][:2, :, None]
        assert (deq - w).abs().le(w.abs() / 16 + p[f"{name}_ws"][:2, :, None] * 2 ** -9).all()
        # the row absmax maps to 448 exactly
        assert torch.allclose(deq.abs().amax(-1), w.abs().amax(-1), rtol=1e-6)
    with pytest.raises(ValueError):
        pack_weights(weights, BASE, "cpu", "int4")


def test_pe_struct_layouts_and_pool_bytes():
    src = pathlib.Path(PE_HEADER).read_text()
    body = src[src.index("typedef struct DpeWeights"):src.index("} DpeWeights;")]
    assert len(re.findall(r"const (?:void|float)\*\s+\w+", body)) == len(_lib.PE_WEIGHT_FIELDS)
    assert ctypes.sizeof(_lib.DpeConfig) == 12 * 4
    assert ctypes.sizeof(_lib.DpeBatch) == 8 + 6 * 8
    L = _lib.lib()
    cfg = pe_abi_config(PE_BASE, max_rows=3, max_pages_per_row=4, max_batch=2)
    assert L.dpe_pool_bytes(cfg) == 6 * 2 * (3 * 4) * 16 * 16 * 64 * 2
    w = _lib.DpeWeights()
    h = ctypes.c_void_p()
    assert L.dpe_create(cfg, w, h) == 1            # null weight pointers
    cfg.hidden = 768
    assert L.dpe_create(cfg, w, h) == 2            # unsupported width
    assert L.dpe_pool_bytes(cfg) == 0
    assert L.dpe_decode(None, None, None, 0, None) == 1


def test_pack_pe_weights_layout():
    cfg = PEConfig(layers=2, hidden=128, heads=2, ffn=256, out_dim=192)
    sd = make_pe_weights(cfg)
    p = pack_pe_weights(sd, cfg, "cpu")
    assert set(p) == set(_lib.PE_WEIGHT_FIELDS)
    assert p["conv_w"].shape == (64, 128) and p["conv_w"].dtype == torch.bfloat16
    assert torch.equal(p["conv_w"][:, 64:].float(), sd["ds_proj.weight"][:, :, 1])
    assert p["qkv_w"].shape == (2, 3 * 128, 128)
    assert torch.equal(p["qkv_w"][1, 256:].float(), sd["encoder.layers.1.attn.v_proj.weight"])
    assert p["attn_norm"].shape == (2, 2, 128)
    assert torch.equal(p["ffn_norm"][0, 1], sd["encoder.layers.0.ffn_norm.bias"])
    assert p["out_w"].shape == (192, 8 * 128)


def test_llm_decode_attention_rejects_bad_arguments_without_a_gpu():
    L = _lib.lib()
    assert L.dllm_decode_workspace_size(4, 12, 128, 8, 256) > 0
    assert L.dllm_decode_workspace_size(4, 12, 96, 8, 256) == 0        # head_dim
    args = [None] * 8 + [1, 12, 2, 128, 4, 256, 4, 0.088, None, None, 0, None]
    assert L.dllm_decode_attention(*args) == 1                           # null pointers
    x = ctypes.c_void_p(256)   # never dereferenced: validation fails first
    bad_g = [x, None, None, x, x, None, x, x, 1, 18, 2, 128, 4, 256, 4, 0.088, x, x, 1 << 20, None]
    assert L.dllm_decode_attention(*bad_g) == 2                          # 9 query heads per kv head
    bad_bs = [x, None, None, x, x, None, x, x, 1, 12, 2, 128, 4, 100, 4, 0.088, x, x, 1 << 20, None]
    assert L.dllm_decode_attention(*bad_bs) == 2                         # block_size not a multiple of 64
    small = [x, None, None, x, x, None, x, x, 1, 12, 2, 128, 4, 256, 4, 0.088, x, x, 16, None]
    assert L.dllm_decode_attention(*small) == 4                          # workspace too small


def test_llm_decode_step_rejects_bad_configs_without_a_gpu():
    L = _lib.lib()
    assert ctypes.sizeof(_lib.DllmConfig) == 10 * 4
    w = _lib.DllmWeights()
    h = ctypes.c_void_p()
    good = _lib.DllmConfig(2, 1536, 12, 2, 128, 8960, 1e-6, 256, 4, 8)
    assert L.dllm_create(good, w, h) == 1              # null weight pointers
    bad = _lib.DllmConfig(2, 1600, 12, 2, 128, 8960, 1e-6, 256, 4, 8)
    assert L.dllm_create(bad, w, h) == 2               # width
    bad = _lib.DllmConfig(2, 1536, 12, 2, 64, 8960, 1e-6, 256, 4, 8)
    assert L.dllm_create(bad, w, h) == 2               # head_dim
    assert L.dllm_decode_step(None, None, None, 0, None) == 1


def test_pack_llm_weights_accepts_hf_and_packed_names():
    from nanovllm_dots_b200.llm_decode import pack_llm_weights
    from nanovllm_dots_b200.synthetic import LLMConfig, make_llm_weights
    c = LLMConfig(layers=2, hidden=256, heads=2, kv_heads=1, inter=512)
    hf = make_llm_weights(c)
    packed = {}
    for k, v in hf.items():
        packed["model." + k] = v
    for l in range(2):
        a, m = f"model.layers.{l}.self_attn.", f"model.layers.{l}.mlp."
        packed[a + "qkv_proj.weight"] = torch.cat([packed.pop(a + f"{x}_proj.weight") for x in "qkv"])
        packed[a + "qkv_proj.bias"] = torch.cat([packed.pop(a + f"{x}_proj.bias") for x in "qkv"])
        packed[m + "gate_up_proj.weight"] = torch.cat([packed.pop(m + "gate_proj.weight"),
                                                       packed.pop(m + "up_proj.weight")])
    p1, p2 = pack_llm_weights(hf, c, "cpu"), pack_llm_weights(packed, c, "cpu")
    assert set(p1) == set(_lib.LLM_WEIGHT_FIELDS)
    for k in p1:
        assert torch.equal(p1[k], p2[k]), k
    assert p1["qkv_w"].shape == (2, 512, 256) and p1["gate_up_w"].shape == (2, 1024, 256)
    assert torch.equal(p1["qkv_w"][1, 384:].float(), hf["layers.1.self_attn.v_proj.weight"])
