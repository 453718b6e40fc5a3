"""ctypes binding of ``libdfm.so`` (declarations in ``include/dfm.h`` for the FM
head, ``include/dpe.h`` for the patch encoder, ``include/dllm.h`` for the LLM
decode attention and ``include/dvoc.h`` for the vocoder).

The library is built in-tree by ``nanovllm_dots_b200.build``.  There is no
fallback: if the shared object is missing or fails to load, every entry point
raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int32, c_int64, c_size_t, c_uint32, c_void_p

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libdfm.so")

DFM_OK = 0
TICK_KERNELS = ("ln_attn", "qkv", "attention", "o_proj", "ln_mlp", "fc1", "fc2")  # DFM_TICK_* order
DEVERR_TIMEOUT, DEVERR_PAGE, DEVERR_LEN = 1, 2, 4    # DFM_DEVERR_* bits of the error word
DEVERR_BITS = {DEVERR_TIMEOUT: "timeout", DEVERR_PAGE: "page", DEVERR_LEN: "len"}

EXPORTS = ("dfm_create", "dfm_workspace_size", "dfm_pool_bytes", "dfm_step", "dfm_read_error",
           "dfm_destroy", "dfm_error_string", "dfm_linear", "dfm_attention_workspace_size",
           "dfm_paged_attention", "dfm_paged_attention_noalloc", "dfm_gather_rows", "dfm_tick_launch",
           "dpe_create", "dpe_workspace_size", "dpe_pool_bytes", "dpe_decode", "dpe_read_error",
           "dpe_destroy", "dllm_decode_workspace_size", "dllm_decode_attention", "dllm_read_error",
           "dllm_create", "dllm_step_workspace_size", "dllm_decode_step", "dllm_destroy",
           "dvoc_create", "dvoc_destroy", "dvoc_conv_floats", "dvoc_bias_floats", "dvoc_act_floats",
           "dvoc_hop", "dvoc_stream_left_context", "dvoc_workspace_size", "dvoc_decode",
           "dvoc_read_error", "dvoc_num_convs", "dvoc_conv_launch")


class DfmConfig(ctypes.Structure):
    _fields_ = [("layers", c_int32), ("hidden", c_int32), ("heads", c_int32),
                ("head_dim", c_int32), ("ffn", c_int32), ("latent_dim", c_int32),
                ("latent_patch", c_int32), ("hidden_patch", c_int32), ("cond_dim", c_int32),
                ("nfe", c_int32), ("page_rows", c_int32), ("num_pages", c_int32),
                ("max_pages_per_req", c_int32), ("max_requests", c_int32), ("ln_eps", c_float),
                ("precision", c_int32)]


WEIGHT_FIELDS = ("input_w", "input_b", "temb_w1", "temb_b1", "temb_w2", "temb_b2", "demb_w1",
                 "demb_b1", "demb_w2", "demb_b2", "ada_w", "ada_b", "qkv_w", "qk_norm", "o_w",
                 "o_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b", "final_w", "final_b", "coord_w",
                 "coord_b", "hidden_w", "hidden_b", "latent_w", "latent_b", "rope_inv_freq",
                 "qkv_w8", "qkv_ws", "fc1_w8", "fc1_ws")


class DfmWeights(ctypes.Structure):
    _fields_ = [(f, c_void_p) for f in WEIGHT_FIELDS]


class DfmBatch(ctypes.Structure):
    _fields_ = [("n", c_int32), ("noise", c_void_p), ("act_hidden", c_void_p),
                ("act_row", c_void_p), ("ext_hidden", c_void_p), ("ext_latent", c_void_p),
                ("ext_rows", c_void_p), ("g_cond", c_void_p), ("cache_len", c_void_p),
                ("n_extend", c_void_p), ("block_table", c_void_p), ("kv_pool", c_void_p),
                ("out", c_void_p)]


class DpeConfig(ctypes.Structure):
    _fields_ = [("layers", c_int32), ("hidden", c_int32), ("heads", c_int32),
                ("head_dim", c_int32), ("ffn", c_int32), ("latent_dim", c_int32),
                ("patch", c_int32), ("out_dim", c_int32), ("max_rows", c_int32),
                ("max_pages_per_row", c_int32), ("max_batch", c_int32), ("ln_eps", c_float)]


PE_WEIGHT_FIELDS = ("conv_w", "conv_b", "in_w", "in_b", "attn_norm", "ffn_norm", "qkv_w", "o_w",
                    "o_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b", "out_w", "out_b")


class DpeWeights(ctypes.Structure):
    _fields_ = [(f, c_void_p) for f in PE_WEIGHT_FIELDS]


class DpeBatch(ctypes.Structure):
    _fields_ = [("n", c_int32), ("patches", c_void_p), ("rows", c_void_p), ("seqlens", c_void_p),
                ("conv_tail", c_void_p), ("kv_pool", c_void_p), ("out", c_void_p)]


class DllmConfig(ctypes.Structure):
    _fields_ = [("layers", c_int32), ("hidden", c_int32), ("heads", c_int32),
                ("kv_heads", c_int32), ("head_dim", c_int32), ("inter", c_int32),
                ("rms_eps", c_float), ("block_size", c_int32), ("max_blocks", c_int32),
                ("max_batch", c_int32)]


LLM_WEIGHT_FIELDS = ("in_norm", "qkv_w", "qkv_b", "o_w", "post_norm", "gate_up_w", "down_w",
                     "final_norm", "inv_freq")


class DllmWeights(ctypes.Structure):
    _fields_ = [(f, c_void_p) for f in LLM_WEIGHT_FIELDS]


class DllmStep(ctypes.Structure):
    _fields_ = [("n", c_int32), ("embeds", c_void_p), ("positions", c_void_p),
                ("slot_mapping", c_void_p), ("context_lens", c_void_p), ("block_table", c_void_p),
                ("k_caches", POINTER(c_void_p)), ("v_caches", POINTER(c_void_p)),
                ("num_blocks", c_int32), ("out", c_void_p)]


DVOC_MAX_STAGES, DVOC_MAX_KERNELS = 8, 4


class DvocConfig(ctypes.Structure):
    _fields_ = [("latent_dim", c_int32), ("initial_channels", c_int32), ("num_stages", c_int32),
                ("upsample_rates", c_int32 * DVOC_MAX_STAGES), ("num_kernels", c_int32),
                ("resblock_kernel_sizes", c_int32 * DVOC_MAX_KERNELS),
                ("resblock_dilations", (c_int32 * 3) * DVOC_MAX_KERNELS),
                ("resblock_type", c_int32), ("mi_layers", c_int32), ("lookahead", c_int32),
                ("use_tanh", c_int32), ("max_batch", c_int32), ("max_frames", c_int32)]


VOC_WEIGHT_FIELDS = ("post_w", "post_b", "mi_in_w", "mi_in_b", "lstm_w_ih", "lstm_w_hh",
                     "lstm_b_ih", "lstm_b_hh", "mi_out_w", "mi_out_b", "conv_w", "conv_b", "act",
                     "post_conv_w", "post_conv_b")


class DvocWeights(ctypes.Structure):
    _fields_ = [(f, c_void_p) for f in VOC_WEIGHT_FIELDS]


class DvocBatch(ctypes.Structure):
    _fields_ = [("n", c_int32), ("frames", c_int32), ("window", c_int32), ("latents", c_void_p),
                ("lengths", c_void_p), ("lstm_h", c_void_p), ("lstm_c", c_void_p),
                ("windows", c_void_p), ("valid", c_void_p), ("audio", c_void_p)]


_lib = None


def lib() -> ctypes.CDLL:
    """Load (once) and return the FM-head library; raise if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"FM-head CUDA library not built: {LIB_PATH} is missing "
                           "(run `python -m nanovllm_dots_b200.build`)")
    L = ctypes.CDLL(LIB_PATH)
    L.dfm_create.argtypes = [POINTER(DfmConfig), POINTER(DfmWeights), POINTER(c_void_p)]
    L.dfm_create.restype = c_int32
    L.dfm_workspace_size.argtypes = [c_void_p]
    L.dfm_workspace_size.restype = c_size_t
    L.dfm_pool_bytes.argtypes = [POINTER(DfmConfig)]
    L.dfm_pool_bytes.restype = c_size_t
    L.dfm_step.argtypes = [c_void_p, POINTER(DfmBatch), c_void_p, c_size_t, c_void_p]
    L.dfm_step.restype = c_int32
    L.dfm_read_error.argtypes = [c_void_p, c_void_p, c_void_p, POINTER(c_uint32)]
    L.dfm_read_error.restype = c_int32
    L.dfm_destroy.argtypes = [c_void_p]
    L.dfm_destroy.restype = c_int32
    L.dfm_error_string.argtypes = [c_int32]
    L.dfm_error_string.restype = ctypes.c_char_p
    L.dfm_linear.argtypes = [c_void_p, c_int64, c_int32, c_int32, c_void_p, c_int64, c_int32,
                             c_void_p, c_void_p, c_int32, c_int32, c_void_p]
    L.dfm_linear.restype = c_int32
    L.dfm_attention_workspace_size.argtypes = [c_int32, c_int32, c_int32]
    L.dfm_attention_workspace_size.restype = c_size_t
    L.dfm_paged_attention.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                      c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_int32,
                                      c_int32, c_void_p, c_size_t, c_void_p]
    L.dfm_paged_attention.restype = c_int32
    L.dfm_paged_attention_noalloc.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                                              c_int32, c_int32, c_int32, c_void_p, c_void_p,
                                              c_void_p, c_int32, c_int32, c_void_p, c_void_p]
    L.dfm_paged_attention_noalloc.restype = c_int32
    L.dfm_gather_rows.argtypes = [c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p,
                                  c_void_p, c_void_p]
    L.dfm_gather_rows.restype = c_int32
    L.dfm_tick_launch.argtypes = [c_void_p, POINTER(DfmBatch), c_void_p, c_size_t, c_int32,
                                  c_int32, c_int32, c_void_p]
    L.dfm_tick_launch.restype = c_int32
    L.dpe_create.argtypes = [POINTER(DpeConfig), POINTER(DpeWeights), POINTER(c_void_p)]
    L.dpe_create.restype = c_int32
    L.dpe_workspace_size.argtypes = [c_void_p]
    L.dpe_workspace_size.restype = c_size_t
    L.dpe_pool_bytes.argtypes = [POINTER(DpeConfig)]
    L.dpe_pool_bytes.restype = c_size_t
    L.dpe_decode.argtypes = [c_void_p, POINTER(DpeBatch), c_void_p, c_size_t, c_void_p]
    L.dpe_decode.restype = c_int32
    L.dpe_read_error.argtypes = [c_void_p, c_void_p, c_void_p, POINTER(c_uint32)]
    L.dpe_read_error.restype = c_int32
    L.dpe_destroy.argtypes = [c_void_p]
    L.dpe_destroy.restype = c_int32
    L.dllm_decode_workspace_size.argtypes = [c_int32] * 5
    L.dllm_decode_workspace_size.restype = c_size_t
    L.dllm_decode_attention.argtypes = ([c_void_p] * 8 + [c_int32] * 7
                                        + [c_float, c_void_p, c_void_p, c_size_t, c_void_p])
    L.dllm_decode_attention.restype = c_int32
    L.dllm_read_error.argtypes = [c_void_p, c_void_p, POINTER(c_uint32)]
    L.dllm_read_error.restype = c_int32
    L.dllm_create.argtypes = [POINTER(DllmConfig), POINTER(DllmWeights), POINTER(c_void_p)]
    L.dllm_create.restype = c_int32
    L.dllm_step_workspace_size.argtypes = [c_void_p]
    L.dllm_step_workspace_size.restype = c_size_t
    L.dllm_decode_step.argtypes = [c_void_p, POINTER(DllmStep), c_void_p, c_size_t, c_void_p]
    L.dllm_decode_step.restype = c_int32
    L.dllm_destroy.argtypes = [c_void_p]
    L.dllm_destroy.restype = c_int32
    L.dvoc_create.argtypes = [POINTER(DvocConfig), POINTER(DvocWeights), POINTER(c_void_p)]
    L.dvoc_create.restype = c_int32
    L.dvoc_destroy.argtypes = [c_void_p]
    L.dvoc_destroy.restype = c_int32
    for name in ("dvoc_conv_floats", "dvoc_bias_floats", "dvoc_act_floats"):
        getattr(L, name).argtypes = [POINTER(DvocConfig)]
        getattr(L, name).restype = c_size_t
    L.dvoc_hop.argtypes = [POINTER(DvocConfig)]
    L.dvoc_hop.restype = c_int32
    L.dvoc_stream_left_context.argtypes = [POINTER(DvocConfig)]
    L.dvoc_stream_left_context.restype = c_int32
    L.dvoc_workspace_size.argtypes = [c_void_p]
    L.dvoc_workspace_size.restype = c_size_t
    L.dvoc_decode.argtypes = [c_void_p, POINTER(DvocBatch), c_void_p, c_size_t, c_void_p]
    L.dvoc_decode.restype = c_int32
    L.dvoc_read_error.argtypes = [c_void_p, c_void_p, c_void_p, POINTER(c_uint32)]
    L.dvoc_read_error.restype = c_int32
    L.dvoc_num_convs.argtypes = [c_void_p]
    L.dvoc_num_convs.restype = c_int32
    L.dvoc_conv_launch.argtypes = [c_void_p, POINTER(DvocBatch), c_void_p, c_size_t, c_int32, c_void_p]
    L.dvoc_conv_launch.restype = c_int32
    _lib = L
    return L


def check(rc: int, what: str) -> None:
    if rc != DFM_OK:
        msg = lib().dfm_error_string(rc).decode()
        raise RuntimeError(f"{what} failed: {msg} (code {rc})")


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None for None)."""
    return None if t is None else t.data_ptr()
