"""The LLM backbone's decode step on the B200 kernels (``dllm_decode_step``,
``include/dllm.h``).

The reference advances every generating sequence by one token per engine
step through ``BatchedPagedLLM._decode_batch`` (``batched_llm.py:177-236``):
``QwenLLM.forward`` (``model_llm.py:113-171``) over torch linears, a Triton
K/V store and flash-attn's paged decode.  ``B200QwenDecoder.step`` is that
forward as one C call: per layer RMSNorm, the QKV / O / gate-up / down
projections on a swapped-operand tcgen05 GEMM (SiLU-and-mul in the gate-up
epilogue), rotary with the K/V cache write, the paged decode attention and
the residual adds, on the caller's stream.  The caches stay
the engine's (``BatchedPagedLLM`` allocates one K and one V tensor per layer,
``batched_llm.py:57-66``).  There is no CPU path.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .synthetic import LLM_BASE, LLMConfig


def pack_llm_weights(sd: dict[str, torch.Tensor], cfg: LLMConfig, device) -> dict[str, torch.Tensor]:
    """A Qwen2 state dict (HuggingFace names ``self_attn.q_proj`` ... or the
    reference's packed ``self_attn.qkv_proj`` / ``mlp.gate_up_proj``, with or
    without a ``model.`` / ``llm.`` prefix) -> the stacked layout of
    ``DllmWeights``."""
    def get(name):
        for pre in ("", "model.", "llm.", "llm.model."):
            if pre + name in sd:
                return sd[pre + name]
        raise KeyError(name)

    def has(name):
        try:
            get(name)
            return True
        except KeyError:
            return False

    bf = lambda t: t.to(device=device, dtype=torch.bfloat16).contiguous()
    f32 = lambda t: t.to(device=device, dtype=torch.float32).contiguous()
    L = cfg.layers
    qkv_w, qkv_b, gu = [], [], []
    for l in range(L):
        a = f"layers.{l}.self_attn."
        if has(a + "qkv_proj.weight"):
            qkv_w.append(get(a + "qkv_proj.weight"))
            qkv_b.append(get(a + "qkv_proj.bias"))
        else:
            qkv_w.append(torch.cat([get(a + f"{x}_proj.weight") for x in "qkv"]))
            qkv_b.append(torch.cat([get(a + f"{x}_proj.bias") for x in "qkv"]))
        m = f"layers.{l}.mlp."
        gu.append(get(m + "gate_up_proj.weight") if has(m + "gate_up_proj.weight") else
                  torch.cat([get(m + "gate_proj.weight"), get(m + "up_proj.weight")]))
    D = cfg.head_dim
    return {
        "in_norm": f32(torch.stack([get(f"layers.{l}.input_layernorm.weight") for l in range(L)])),
        "qkv_w": bf(torch.stack(qkv_w)), "qkv_b": f32(torch.stack(qkv_b)),
        "o_w": bf(torch.stack([get(f"layers.{l}.self_attn.o_proj.weight") for l in range(L)])),
        "post_norm": f32(torch.stack([get(f"layers.{l}.post_attention_layernorm.weight")
                                      for l in range(L)])),
        "gate_up_w": bf(torch.stack(gu)),
        "down_w": bf(torch.stack([get(f"layers.{l}.mlp.down_proj.weight") for l in range(L)])),
        "final_norm": f32(get("norm.weight")),
        # RotaryEmbedding.inv_freq as the reference builds it (rotary_embedding.py:26-27)
        "inv_freq": f32(1.0 / (cfg.rope_theta ** (torch.arange(0, D, 2, dtype=torch.float) / D))),
    }


class B200QwenDecoder:
    """The backbone decode step for up to ``max_batch`` sequences whose block
    tables are at most ``max_blocks`` wide."""

    def __init__(self, weights: dict[str, torch.Tensor], cfg: LLMConfig = LLM_BASE, *,
                 max_batch: int, max_blocks: int, device: torch.device | str = "cuda"):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("B200QwenDecoder runs on a CUDA device only (no CPU path)")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.cfg, self.max_batch, self.max_blocks = cfg, max_batch, max_blocks
        self.L = _lib.lib()
        self.w = pack_llm_weights(weights, cfg, self.device)
        self.acfg = _lib.DllmConfig(cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim,
                                    cfg.inter, cfg.rms_eps, cfg.block_size, max_blocks, max_batch)
        ws = _lib.DllmWeights(*[_lib.ptr(self.w[f]) for f in _lib.LLM_WEIGHT_FIELDS])
        h = _lib.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(self.L.dllm_create(self.acfg, ws, h), "dllm_create")
        self.handle = h
        self.ws_bytes = int(self.L.dllm_step_workspace_size(h))
        self.workspace = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=self.device)

    def alloc_caches(self, num_blocks: int):
        """Per-layer K and V caches in the reference's layout (zeroed)."""
        c = self.cfg
        shape = (num_blocks, c.block_size, c.kv_heads, c.head_dim)
        return ([torch.zeros(shape, dtype=torch.bfloat16, device=self.device) for _ in range(c.layers)],
                [torch.zeros(shape, dtype=torch.bfloat16, device=self.device) for _ in range(c.layers)])

    def step(self, embeds, positions, slot_mapping, context_lens, block_tables, k_caches, v_caches,
             out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """embeds bf16 [n, hidden]; int32 positions, slot_mapping, context_lens [n]
        and block_tables [n, max_blocks]; per-layer cache lists -> bf16 [n, hidden]."""
        c = self.cfg
        n = embeds.shape[0]
        if not 1 <= n <= self.max_batch:
            raise RuntimeError(f"decode step with {n} sequences (max {self.max_batch})")
        if block_tables.shape != (n, self.max_blocks):
            raise RuntimeError(f"block_tables must be [n, {self.max_blocks}]")
        for name, t, dt in (("embeds", embeds, torch.bfloat16), ("positions", positions, torch.int32),
                            ("slot_mapping", slot_mapping, torch.int32),
                            ("context_lens", context_lens, torch.int32),
                            ("block_tables", block_tables, torch.int32)):
            if t.dtype != dt or t.device != self.device or not t.is_contiguous():
                raise RuntimeError(f"{name}: expected a contiguous {dt} tensor on {self.device}")
        if len(k_caches) != c.layers or len(v_caches) != c.layers:
            raise RuntimeError(f"expected {c.layers} K and V caches")
        # every layer's cache must have the first one's block count: the kernels
        # bound slot_mapping and the block table by it
        shape = (k_caches[0].shape[0], c.block_size, c.kv_heads, c.head_dim)
        for name, caches in (("k_caches", k_caches), ("v_caches", v_caches)):
            for l, t in enumerate(caches):
                if (t.dtype != torch.bfloat16 or t.device != self.device or not t.is_contiguous()
                        or tuple(t.shape) != shape):
                    raise RuntimeError(f"{name}[{l}]: expected a contiguous bf16 tensor of shape "
                                       f"{shape} on {self.device}")
        if out is None:
            out = torch.empty(n, c.hidden, dtype=torch.bfloat16, device=self.device)
        kp = (ctypes.c_void_p * c.layers)(*[t.data_ptr() for t in k_caches])
        vp = (ctypes.c_void_p * c.layers)(*[t.data_ptr() for t in v_caches])
        st = _lib.DllmStep(n, _lib.ptr(embeds), _lib.ptr(positions), _lib.ptr(slot_mapping),
                           _lib.ptr(context_lens), _lib.ptr(block_tables), kp, vp,
                           k_caches[0].shape[0], _lib.ptr(out))
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        with torch.cuda.device(self.device):
            _lib.check(self.L.dllm_decode_step(self.handle, st, _lib.ptr(self.workspace),
                                               self.ws_bytes, _lib.c_void_p(s.cuda_stream)),
                       "dllm_decode_step")
        return out

    def check_errors(self) -> None:
        v = _lib.c_uint32(0)
        s = torch.cuda.current_stream(self.device)
        with torch.cuda.device(self.device):
            _lib.check(self.L.dllm_read_error(_lib.ptr(self.workspace),
                                              _lib.c_void_p(s.cuda_stream), v), "dllm_read_error")
        if v.value:
            names = [nm for bit, nm in _lib.DEVERR_BITS.items() if v.value & bit]
            raise RuntimeError(f"LLM decode device error: {', '.join(names)} (0x{v.value:x})")

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.L.dllm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
