"""Seeded synthetic FM-head model and inputs (the BASELINE.json configs).

The reference publishes no checkpoint for the synthetic DiT, so weights are a
seeded random init with torch's default ``nn.Linear`` initialisation, created in
the same module order as the reference constructor
(``nanovllm_dots/models/dots/native/dit.py:113-133``: input_layer,
time_embedder, duration_embedder, then per block q/k/v/o, fc1, fc2, adaLN, then
the final layer's adaLN and linear) followed by the core projections
(``native/core.py:66-68``: coordinate_proj, hidden_proj, latent_proj).  The
draw happens in fp32 on the CPU; every weight is then rounded to bf16, which
is the precision the head computes with.  The oracle and the CUDA path both use
these bf16-valued weights, so parity is about arithmetic, not weight rounding.

All per-request inputs come from explicit ``torch.Generator`` seeds so that the
test box regenerates exactly what the golden fixtures were made from.
"""
from __future__ import annotations

import dataclasses
import hashlib

import numpy as np
import torch
import torch.nn as nn


@dataclasses.dataclass(frozen=True)
class FMConfig:
    """Shape of the FM head.  Defaults are BASELINE.json's synthetic DiT."""
    layers: int = 12
    hidden: int = 1024
    heads: int = 16
    head_dim: int = 64
    ffn: int = 4096
    latent_dim: int = 64
    latent_patch: int = 16
    hidden_patch: int = 1
    cond_dim: int = 1536
    nfe: int = 4
    page_rows: int = 16
    freq_dim: int = 256
    rotary_theta: float = 50000.0
    ln_eps: float = 1e-5

    @property
    def stride(self) -> int:
        """Rows one patch adds to the FM history (hidden row + latent rows)."""
        return self.hidden_patch + self.latent_patch

    @property
    def mod_width(self) -> int:
        """Columns of the concatenated adaLN output: 6H per block + 2H final."""
        return self.layers * 6 * self.hidden + 2 * self.hidden


BASE = FMConfig()

# Order of the per-block parameters in the packed dict.
BLOCK_KEYS = ("q", "k", "v", "q_norm_w", "q_norm_b", "k_norm_w", "k_norm_b",
              "o_w", "o_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b", "ada_w", "ada_b")


def _lin(i: int, o: int, bias: bool = True) -> nn.Linear:
    return nn.Linear(i, o, bias=bias)


def make_weights(cfg: FMConfig = BASE, seed: int = 0) -> dict[str, torch.Tensor]:
    """Seeded weights as a flat dict of fp32 CPU tensors holding bf16 values.

    Keys follow the reference state-dict names (``blocks.{l}.attn.q_proj.weight``
    and so on, plus ``coordinate_proj.*``, ``hidden_proj.*``, ``latent_proj.*``)
    so a real checkpoint maps onto the same packer.
    """
    H, F = cfg.hidden, cfg.ffn
    torch.manual_seed(seed)
    sd: dict[str, torch.Tensor] = {}

    def put(prefix: str, mod: nn.Module) -> None:
        for n, p in mod.named_parameters():
            sd[f"{prefix}.{n}"] = p.detach()

    with torch.no_grad():
        put("input_layer", _lin(H, H))
        for emb in ("time_embedder", "duration_embedder"):
            put(f"{emb}.mlp.0", _lin(cfg.freq_dim, H))
            put(f"{emb}.mlp.2", _lin(H, H))
        for l in range(cfg.layers):
            b = f"blocks.{l}"
            put(f"{b}.attn.q_proj", _lin(H, H, bias=False))
            put(f"{b}.attn.k_proj", _lin(H, H, bias=False))
            put(f"{b}.attn.v_proj", _lin(H, H, bias=False))
            put(f"{b}.attn.q_norm", nn.LayerNorm(cfg.head_dim))
            put(f"{b}.attn.k_norm", nn.LayerNorm(cfg.head_dim))
            put(f"{b}.attn.o_proj", _lin(H, H))
            put(f"{b}.ffn.fc1", _lin(H, F))
            put(f"{b}.ffn.fc2", _lin(F, H))
            put(f"{b}.adaLN_modulation.1", _lin(H, 6 * H))
        put("output_layer.adaLN_modulation.1", _lin(H, 2 * H))
        put("output_layer.linear", _lin(H, cfg.latent_dim))
        put("coordinate_proj", _lin(cfg.latent_dim, H))
        put("hidden_proj", _lin(cfg.cond_dim, H))
        put("latent_proj", _lin(cfg.latent_dim, H))
    return {k: v.to(torch.bfloat16).float() for k, v in sd.items()}


def weights_digest(w: dict[str, torch.Tensor]) -> str:
    """Order-independent sha256 over every weight's bf16 bytes."""
    h = hashlib.sha256()
    for k in sorted(w):
        h.update(k.encode())
        h.update(w[k].to(torch.bfloat16).view(torch.int16).numpy().tobytes())
    return h.hexdigest()


def tensor_digest(t: torch.Tensor) -> str:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


# --------------------------------------------------------------------------- #
# Per-request inputs                                                           #
# --------------------------------------------------------------------------- #
@dataclasses.dataclass
class RequestBatch:
    """Host-side inputs of one tick for n requests (CPU tensors).

    noise        bf16 [n, lp, ld]   the solver's starting point
    cond         bf16 [n, cond_dim] this tick's LLM hidden (the active hidden row)
    prev_hidden  bf16 [n, cond_dim] previous tick's LLM hidden (graduating row)
    prev_latent  bf16 [n, lp, ld]   previous patch (graduating rows)
    g_cond       bf16 [n, H] or None
    prefix_rows  int  [n]           cached prefix rows P_i before this tick
    n_extend     int  [n]           graduating rows this tick (0 or stride)
    kv_seed      int                base seed of the cached K/V draws
    """
    noise: torch.Tensor
    cond: torch.Tensor
    prev_hidden: torch.Tensor
    prev_latent: torch.Tensor
    g_cond: torch.Tensor | None
    prefix_rows: list[int]
    n_extend: list[int]
    kv_seed: int
    kv_std: float = 0.5

    @property
    def n(self) -> int:
        return len(self.prefix_rows)


def make_batch(n: int, prefix_patches: list[int], seed: int, cfg: FMConfig = BASE,
               n_extend: list[int] | None = None, with_g: bool = False) -> RequestBatch:
    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    noise = torch.randn(n, cfg.latent_patch, cfg.latent_dim, generator=g).to(bf)
    cond = torch.randn(n, cfg.cond_dim, generator=g).to(bf)
    prev_hidden = torch.randn(n, cfg.cond_dim, generator=g).to(bf)
    prev_latent = torch.randn(n, cfg.latent_patch, cfg.latent_dim, generator=g).to(bf)
    gc = torch.randn(n, cfg.hidden, generator=g).to(bf) * 0.5 if with_g else None
    if n_extend is None:
        n_extend = [cfg.stride] * n
    return RequestBatch(noise, cond, prev_hidden, prev_latent, gc,
                        [cfg.stride * p for p in prefix_patches], list(n_extend), seed)


def config_batch(name: str, cfg: FMConfig = BASE) -> RequestBatch:
    """The request mix of a BASELINE.json config ("cfg1", "cfg2", "cfg4")."""
    if name == "cfg1":
        g = torch.Generator().manual_seed(1)
        pp = torch.randint(0, 33, (8,), generator=g).tolist()
        return make_batch(8, pp, seed=1, cfg=cfg)
    if name == "cfg2":
        g = torch.Generator().manual_seed(2)
        pp = torch.randint(0, 121, (64,), generator=g).tolist()
        return make_batch(64, pp, seed=2, cfg=cfg)
    if name == "cfg4":
        g = torch.Generator().manual_seed(4)
        long_ = torch.rand(64, generator=g) < 0.25
        short_p = torch.randint(0, 61, (64,), generator=g)
        long_p = torch.randint(200, 321, (64,), generator=g)
        pp = torch.where(long_, long_p, short_p).tolist()
        return make_batch(64, pp, seed=4, cfg=cfg)
    raise ValueError(f"unknown config {name!r}")


def request_kv(batch: RequestBatch, i: int, cfg: FMConfig = BASE) -> torch.Tensor:
    """Cached K/V of request i: bf16 [nfe, layers, 2, P_i, heads, head_dim].

    Each (step, layer) slice is N(0, kv_std^2), drawn from a generator seeded
    by (kv_seed, i) so any request can be regenerated on its own.
    """
    P = batch.prefix_rows[i]
    g = torch.Generator().manual_seed(batch.kv_seed * 1_000_003 + 7919 * i + 17)
    shape = (cfg.nfe, cfg.layers, 2, P, cfg.heads, cfg.head_dim)
    return (torch.randn(shape, generator=g) * batch.kv_std).to(torch.bfloat16)


def time_grid(nfe: int) -> tuple[list[float], list[float]]:
    """The MeanFlow grid the reference DiT sees: timesteps t_k = k/nfe and
    durations dt_k = t_{k+1} - t_k (``batched_fm.py:113-116``).  For nfe=4 all
    values are exact in bf16, so the bf16 ``linspace`` of the reference and
    this fp32 grid agree bit for bit."""
    ts = np.linspace(0.0, 1.0, nfe + 1, dtype=np.float32)
    ts = torch.tensor(ts).to(torch.bfloat16).float().tolist()
    return ts[:-1], [ts[k + 1] - ts[k] for k in range(nfe)]


# --------------------------------------------------------------------------- #
# Patch encoder (the step after the FM head)                                   #
# --------------------------------------------------------------------------- #
@dataclasses.dataclass(frozen=True)
class PEConfig:
    """Shape of the patch encoder (``VAESemanticEncoder``,
    ``nanovllm_dots/models/dots/native/patch_encoder.py:139-150``).

    The reference reads these from the checkpoint's config.json, which is not
    published; the defaults are synthetic choices consistent with the FM head
    above: the 16-frame latent patch of 64 channels, the causal stride-2
    downsampling conv (so 8 encoder rows per patch), a 1024-wide encoder with
    16 heads of 64, FFN 4096, the ``SuperviseEncoder`` default of 6 layers
    (``patch_encoder.py:99``), and the LLM hidden size 1536 (the FM head's
    ``cond_dim``) as the output width (``native/loader.py:85-87``).
    """
    layers: int = 6
    hidden: int = 1024
    heads: int = 16
    head_dim: int = 64
    ffn: int = 4096
    latent_dim: int = 64
    patch: int = 16
    in_ds: int = 2
    out_dim: int = 1536
    page_rows: int = 16
    ln_eps: float = 1e-5

    @property
    def rows(self) -> int:
        """Encoder rows one patch adds (``out_ds_rate``, ``patch_encoder.py:148``)."""
        return self.patch // self.in_ds


PE_BASE = PEConfig()


def make_pe_weights(cfg: PEConfig = PE_BASE, seed: int = 0,
                    ln_jitter: float = 0.1) -> dict[str, torch.Tensor]:
    """Seeded patch-encoder weights (fp32 CPU tensors holding bf16 values).

    Modules are created in the reference constructor's order
    (``patch_encoder.py:142-150``: ds_proj, in_proj, the encoder layers with
    ``attn`` {q,k,v,o}_proj, ``attn_norm``, ``ffn`` fc1/fc2, ``ffn_norm``
    (``patch_encoder.py:28-38``, ``layers.py:146-161``), then out_proj) with
    torch's default initialisation, so the reference module built under the
    same seed holds the same values.  LayerNorm weights and biases default to
    1 and 0; they are then jittered (seed + 1) so the affine path is exercised.
    Keys are the reference state-dict names.
    """
    H, F = cfg.hidden, cfg.ffn
    torch.manual_seed(seed)
    sd: dict[str, torch.Tensor] = {}

    def put(prefix: str, mod: nn.Module) -> None:
        for n, p in mod.named_parameters():
            sd[f"{prefix}.{n}"] = p.detach()

    with torch.no_grad():
        put("ds_proj", nn.Conv1d(cfg.latent_dim, cfg.latent_dim, cfg.in_ds, stride=cfg.in_ds))
        put("in_proj", _lin(cfg.latent_dim, H))
        for l in range(cfg.layers):
            b = f"encoder.layers.{l}"
            put(f"{b}.attn.q_proj", _lin(H, H, bias=False))
            put(f"{b}.attn.k_proj", _lin(H, H, bias=False))
            put(f"{b}.attn.v_proj", _lin(H, H, bias=False))
            put(f"{b}.attn.o_proj", _lin(H, H))
            put(f"{b}.attn_norm", nn.LayerNorm(H))
            put(f"{b}.ffn.fc1", _lin(H, F))
            put(f"{b}.ffn.fc2", _lin(F, H))
            put(f"{b}.ffn_norm", nn.LayerNorm(H))
        put("out_proj", _lin(H * cfg.rows, cfg.out_dim))
        g = torch.Generator().manual_seed(seed + 1)
        for k in sorted(sd):
            if "_norm." in k:
                base = 1.0 if k.endswith("weight") else 0.0
                sd[k] = base + ln_jitter * torch.randn(sd[k].shape, generator=g)
    return {k: v.to(torch.bfloat16).float() for k, v in sd.items()}


def make_pe_patches(n: int, count: int, seed: int, cfg: PEConfig = PE_BASE) -> torch.Tensor:
    """``count`` successive latent patches for n requests: bf16 [count, n, patch,
    latent_dim], N(0, 1) (the engine feeds denormalised latents,
    ``engine.py:750-752``)."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(count, n, cfg.patch, cfg.latent_dim, generator=g).to(torch.bfloat16)


# --------------------------------------------------------------------------- #
# LLM backbone (the step before the FM head)                                   #
# --------------------------------------------------------------------------- #
@dataclasses.dataclass(frozen=True)
class LLMConfig:
    """Shape of the dots.tts LLM backbone: Qwen2 with GQA 12 query / 2 kv heads
    and head_dim 128 (``nanovllm_dots/models/dots/model_llm.py:1-12``), width
    1536 (the FM head's ``cond_dim``), paged K/V in 256-position blocks
    (``batched_llm.py:32-45``).  Depth, MLP width, RMSNorm eps and rope base are
    the Qwen2-1.5B values (the checkpoint's llm_config.json is unpublished)."""
    layers: int = 28
    hidden: int = 1536
    heads: int = 12
    kv_heads: int = 2
    head_dim: int = 128
    inter: int = 8960
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    block_size: int = 256

    @property
    def qkv_width(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim


LLM_BASE = LLMConfig()


def make_llm_weights(cfg: LLMConfig = LLM_BASE, seed: int = 0, device="cpu",
                     std: float = 0.02) -> dict[str, torch.Tensor]:
    """Seeded Qwen2 decoder weights (fp32 tensors holding bf16 values) under the
    HuggingFace ``Qwen2Model`` state-dict names (``layers.{l}.self_attn.q_proj``,
    ..., ``norm.weight``).  Linear weights N(0, std^2) (HF's initializer_range),
    q/k/v biases N(0, 0.1^2) and RMSNorm weights 1 + N(0, 0.1^2), so every term
    of the layer is exercised."""
    g = torch.Generator(device=device).manual_seed(seed)
    H, D, I = cfg.hidden, cfg.head_dim, cfg.inter
    sd: dict[str, torch.Tensor] = {}

    def rn(*shape, s=std, base=0.0):
        t = torch.randn(*shape, generator=g, device=device) * s + base
        return t.to(torch.bfloat16).float()

    for l in range(cfg.layers):
        p = f"layers.{l}"
        sd[f"{p}.input_layernorm.weight"] = rn(H, s=0.1, base=1.0)
        sd[f"{p}.self_attn.q_proj.weight"] = rn(cfg.heads * D, H)
        sd[f"{p}.self_attn.q_proj.bias"] = rn(cfg.heads * D, s=0.1)
        sd[f"{p}.self_attn.k_proj.weight"] = rn(cfg.kv_heads * D, H)
        sd[f"{p}.self_attn.k_proj.bias"] = rn(cfg.kv_heads * D, s=0.1)
        sd[f"{p}.self_attn.v_proj.weight"] = rn(cfg.kv_heads * D, H)
        sd[f"{p}.self_attn.v_proj.bias"] = rn(cfg.kv_heads * D, s=0.1)
        sd[f"{p}.self_attn.o_proj.weight"] = rn(H, cfg.heads * D)
        sd[f"{p}.post_attention_layernorm.weight"] = rn(H, s=0.1, base=1.0)
        sd[f"{p}.mlp.gate_proj.weight"] = rn(I, H)
        sd[f"{p}.mlp.up_proj.weight"] = rn(I, H)
        sd[f"{p}.mlp.down_proj.weight"] = rn(H, I)
    sd["norm.weight"] = rn(H, s=0.1, base=1.0)
    return sd
