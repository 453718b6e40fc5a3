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
import math

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


# --------------------------------------------------------------------------- #
# Vocoder (BigVGAN AudioVAE decoder, the step after the patch encoder)         #
# --------------------------------------------------------------------------- #
@dataclasses.dataclass(frozen=True)
class VocConfig:
    """Shape of the vocoder's decode path (``AudioVAE``,
    ``nanovllm_dots/models/dots/native/vocoder/bigvgan.py:751-788`` and
    ``Decoder``, ``bigvgan.py:542-640``; keys of ``vocoder/config.py``).

    The checkpoint's config.json is not published.  The defaults are synthetic
    choices consistent with the rest of this package: 64-channel latents (the
    FM head's ``latent_dim``, so FM patches feed it directly), 25 latent frames
    per second and 48 kHz audio (the reference's golden manifests: 1920 samples
    per frame), the config default of 1536 initial channels, six causal
    transposed-conv upsamplers whose rates multiply to 1920, three AMPBlock1
    resblocks per stage with kernels 3/7/11 and dilations 1/3/5, SnakeBeta on a
    log scale, a 4-layer LSTM front (``mi_num_layers``) and 2 lookahead frames.
    """
    latent_dim: int = 64
    initial_channels: int = 1536
    upsample_rates: tuple = (8, 5, 4, 3, 2, 2)
    resblock_kernel_sizes: tuple = (3, 7, 11)
    resblock_dilations: tuple = ((1, 3, 5), (1, 3, 5), (1, 3, 5))
    resblock: str = "1"
    activation: str = "snakebeta"
    mi_layers: int = 4
    lookahead: int = 2
    use_tanh: bool = True
    use_bias_at_final: bool = True
    sample_rate: int = 48000

    @property
    def hop(self) -> int:
        """Audio samples per latent frame (the product of the upsample rates)."""
        return int(np.prod(self.upsample_rates))

    @property
    def upsample_kernel_sizes(self) -> tuple:
        """Causal transposed convs need kernel = 2 * stride (``layers.py:61-64``)."""
        return tuple(2 * u for u in self.upsample_rates)

    def stage_channels(self, i: int) -> int:
        """Output channels of stage i (``bigvgan.py:572-583``); -1 is conv_pre's."""
        return self.initial_channels // (2 ** (i + 1))

    def reference_dict(self) -> dict:
        """The ``vocoder`` section of config.json that builds this shape with the
        reference's ``AudioVAEConfig``."""
        return {
            "sample_rate": self.sample_rate, "upsample_rates": list(self.upsample_rates),
            "upsample_kernel_sizes": list(self.upsample_kernel_sizes),
            "upsample_initial_channel": self.initial_channels, "resblock": self.resblock,
            "resblock_kernel_sizes": list(self.resblock_kernel_sizes),
            "resblock_dilation_sizes": [list(d) for d in self.resblock_dilations],
            "downsample_rates": list(self.upsample_rates),
            "downsample_channels": [8] * (len(self.upsample_rates) + 1),
            "activation": self.activation, "snake_logscale": True,
            "latent_dim": self.latent_dim, "causal": True, "mi_num_layers": self.mi_layers,
            "causal_encoder": True, "use_bias_at_final": self.use_bias_at_final,
            "use_tanh_at_final": self.use_tanh, "num_decoder_lookahead": self.lookahead,
        }


VOC_BASE = VocConfig()
# A small shape for golden fixtures and fast parity tests: three stages, the
# last one narrower than 32 channels (exercises the channel padding).
VOC_SMALL = VocConfig(latent_dim=32, initial_channels=128, upsample_rates=(4, 3, 2), mi_layers=2)


def kaiser_sinc(cutoff: float, half_width: float, kernel_size: int) -> np.ndarray:
    """Kaiser-windowed sinc low-pass filter normalised to unit sum (Kaiser's
    window with his published beta rule; the filter the reference builds in
    ``alias_free_filter.py:28-60``).  float64 [kernel_size]."""
    half = kernel_size // 2
    delta_f = 4.0 * half_width
    att = 2.285 * (half - 1) * math.pi * delta_f + 7.95
    if att > 50.0:
        beta = 0.1102 * (att - 8.7)
    elif att >= 21.0:
        beta = 0.5842 * (att - 21.0) ** 0.4 + 0.07886 * (att - 21.0)
    else:
        beta = 0.0
    window = np.kaiser(kernel_size, beta)
    time = np.arange(-half, half) + 0.5 if kernel_size % 2 == 0 else np.arange(kernel_size) - half
    filt = 2.0 * cutoff * window * np.sinc(2.0 * cutoff * time)
    return filt / filt.sum()


def voc_filter(kernel_size: int = 12) -> torch.Tensor:
    """The fixed filter of the ratio-2 up- and down-samplers (cutoff 0.25, half
    width 0.3), fp32.  Computed here in float64 and rounded once; a real
    checkpoint carries the reference's own fp32 buffers, which are used then."""
    return torch.tensor(kaiser_sinc(0.25, 0.3, kernel_size), dtype=torch.float32)


def voc_act_names(cfg: VocConfig) -> list[str]:
    """State-dict prefixes of every alias-free activation of the decoder in
    execution order: per resblock its 6 (AMPBlock1) or 2 (AMPBlock2)
    activations, then ``activation_post``."""
    per = 6 if cfg.resblock == "1" else 2
    names = []
    for r in range(len(cfg.upsample_rates) * len(cfg.resblock_kernel_sizes)):
        names += [f"decoder.resblocks.{r}.activations.{a}" for a in range(per)]
    return names + ["decoder.activation_post"]


def make_voc_weights(cfg: VocConfig = VOC_SMALL, seed: int = 0) -> dict[str, torch.Tensor]:
    """Seeded fp32 weights of the vocoder's decode path under the reference's
    state-dict names (after ``remove_weight_norm``, ``loader.py:94-110``).

    Convolutions are N(0, (g / sqrt(fan_in))^2) with gains that keep the
    residual stream O(1) through every stage (the reference's N(0, 0.01^2)
    init would leave the audio near zero), biases N(0, 0.05^2), log-alpha and
    log-beta N(0, 0.3^2), the LSTM uniform(+-1/sqrt(hidden)) as torch
    initialises it.  The resblock activations carry the fixed filter (a
    buffer); ``activation_post``'s learnable per-channel filters are that
    filter jittered per channel, as a trained checkpoint's would differ.
    """
    g = torch.Generator().manual_seed(seed)
    L, Hm = cfg.latent_dim, 4 * cfg.latent_dim
    sd: dict[str, torch.Tensor] = {}

    def rn(*shape, s=1.0):
        return torch.randn(*shape, generator=g) * s

    def conv(name, cout, cin, k, gain=1.0, bias=True):
        sd[f"{name}.weight"] = rn(cout, cin, k, s=gain / math.sqrt(cin * k))
        if bias:
            sd[f"{name}.bias"] = rn(cout, s=0.05)

    conv("post_proj", L, L, 1)
    sd["dec_mi_layer.0.weight"] = rn(Hm, L, s=1.0 / math.sqrt(L))
    sd["dec_mi_layer.0.bias"] = rn(Hm, s=0.05)
    bound = 1.0 / math.sqrt(Hm)
    for l in range(cfg.mi_layers):
        for kind in ("ih", "hh"):
            sd[f"dec_mi_layer.1.lstm.weight_{kind}_l{l}"] = (torch.rand(4 * Hm, Hm, generator=g) * 2 - 1) * bound
            sd[f"dec_mi_layer.1.lstm.bias_{kind}_l{l}"] = (torch.rand(4 * Hm, generator=g) * 2 - 1) * bound
    sd["dec_mi_layer.2.weight"] = rn(L, Hm, s=1.0 / math.sqrt(Hm))
    sd["dec_mi_layer.2.bias"] = rn(L, s=0.05)
    conv("decoder.conv_pre", cfg.initial_channels, L, 2 * cfg.lookahead + 1)
    filt = voc_filter()
    nk = len(cfg.resblock_kernel_sizes)
    for i, (u, k) in enumerate(zip(cfg.upsample_rates, cfg.upsample_kernel_sizes)):
        cin, cout = cfg.stage_channels(i - 1), cfg.stage_channels(i)
        sd[f"decoder.ups.{i}.0.weight"] = rn(cin, cout, k, s=1.0 / math.sqrt(cin * 2))
        sd[f"decoder.ups.{i}.0.bias"] = rn(cout, s=0.05)
        for j, (ks, dil) in enumerate(zip(cfg.resblock_kernel_sizes, cfg.resblock_dilations)):
            r = i * nk + j
            if cfg.resblock == "1":
                for cname in ("convs1", "convs2"):
                    for l in range(len(dil)):
                        conv(f"decoder.resblocks.{r}.{cname}.{l}", cout, cout, ks, gain=0.4)
            else:
                for l in range(2):
                    conv(f"decoder.resblocks.{r}.convs.{l}", cout, cout, ks, gain=0.4)
    C = cfg.stage_channels(len(cfg.upsample_rates) - 1)
    for name in voc_act_names(cfg):
        post = name.endswith("post")
        ch = C if post else cfg.stage_channels(int(name.split(".")[2]) // nk)
        sd[f"{name}.act.alpha"] = rn(ch, s=0.3)
        if cfg.activation == "snakebeta":
            sd[f"{name}.act.beta"] = rn(ch, s=0.3)
        for part in ("upsample.filter", "downsample.lowpass.filter"):
            if post:
                sd[f"{name}.{part}"] = filt.view(1, 1, 12) * (1.0 + 0.05 * rn(ch, 1, 12))
            else:
                sd[f"{name}.{part}"] = filt.view(1, 1, 12).clone()
    conv("decoder.conv_post", 1, C, 7, bias=cfg.use_bias_at_final)
    return {k: v.float().contiguous() for k, v in sd.items()}


def make_voc_latents(n: int, frames: int, seed: int, cfg: VocConfig = VOC_SMALL) -> torch.Tensor:
    """Latent frames for n requests: fp32 [n, frames, latent_dim], N(0, 1),
    frames-first (the layout the engine stores them in, ``engine.py:835-845``)."""
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(n, frames, cfg.latent_dim, generator=gen)
