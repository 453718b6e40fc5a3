"""CPU oracle for the patch encoder -- TEST INFRASTRUCTURE ONLY.

Only tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
use this module, and only as the checker or the timed CPU baseline.  The
product path (``nanovllm_dots_b200``) never imports it.

It restates, in plain fp32 torch on the CPU, the reference's streaming decode
of the patch encoder (``VAESemanticEncoder``,
``nanovllm_dots/models/dots/native/patch_encoder.py``), which turns each newly
generated latent patch into the LLM's next input embedding:

* the causal stride-2 downsampling conv (``patch_encoder.py:225-235``,
  ``native/layers.py:31-50``): the patch's 16 frames, preceded by the last
  frame of the previous patch (the "conv tail", zero for the first patch),
  give 8 rows ``x_t = b + W0 f_{2t-1} + W1 f_{2t}``; the patch's last frame
  becomes the next tail;
* ``in_proj`` (``patch_encoder.py:234``);
* per encoder layer ``TransformerEncoderLayer.decode_step``
  (``patch_encoder.py:78-87``): pre-LayerNorm with affine, q/k/v projections
  without bias, qk-norm and rotary (the encoder builds its attention with
  neither, ``patch_encoder.py:31-32``, ``layers.py:140-165``), the new K/V
  appended to the per-layer cache at positions ``S..S+7``, causal attention
  over the cache (``layers.py:210-245``: query at position p sees keys
  ``0..p``), softmax(QK^T/8)V, ``o_proj`` with bias, residual; then the SiLU
  MLP (``patch_encoder.py:36``, ``layers.py:78-92``) on the ``ffn_norm``
  output, residual;
* ``_project_embeddings`` (``patch_encoder.py:218-221``): the 8 rows of the
  patch concatenated row-major into one ``8 * hidden`` vector, then
  ``out_proj``.

``prefill`` restates ``VAESemanticEncoder.prefill`` (``patch_encoder.py:170-200``):
the whole prompt through the conv and one causal pass.  The batched flash
variant (``flash_patch_encoder.py:81-139``) computes the same function per
cache row.

Parity pin: ``tests/golden/make_golden_pe.py`` runs the reference's own
``VAESemanticEncoder.decode_patch`` and ``prefill`` on seeded inputs;
``tests/test_pe_oracle.py`` checks this module against those fixtures.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from nanovllm_dots_b200.synthetic import PE_BASE, PEConfig


class PEState:
    """One request's decode state: conv tail [latent_dim] and per-layer K/V
    caches [S, heads, head_dim] (``patch_encoder.py:21-25``)."""

    def __init__(self, cfg: PEConfig = PE_BASE):
        self.cfg = cfg
        self.tail = torch.zeros(cfg.latent_dim)
        z = torch.zeros(0, cfg.heads, cfg.head_dim)
        self.k = [z.clone() for _ in range(cfg.layers)]
        self.v = [z.clone() for _ in range(cfg.layers)]

    @property
    def seq_len(self) -> int:
        return self.k[0].shape[0]


def _lin(x, w, name, bias=True):
    y = x @ w[f"{name}.weight"].t()
    return y + w[f"{name}.bias"] if bias else y


def downsample(w, frames: torch.Tensor, tail: torch.Tensor) -> torch.Tensor:
    """Causal conv over [tail | frames] (frames [T, ld], T even) -> [T/2, ld]."""
    inp = torch.cat([tail.reshape(1, -1), frames], dim=0)     # T + 1 frames
    wc = w["ds_proj.weight"]                                   # [out, in, 2]
    n = frames.shape[0] // 2
    x0, x1 = inp[0:2 * n:2], inp[1:2 * n:2]
    return x0 @ wc[:, :, 0].t() + x1 @ wc[:, :, 1].t() + w["ds_proj.bias"]


def encoder_rows(w, cfg: PEConfig, st: PEState, x: torch.Tensor) -> torch.Tensor:
    """The encoder layers on T new rows [T, hidden] at positions S..S+T-1,
    appending their K/V to ``st``; returns the rows after the last layer."""
    T, H, nh, dh = x.shape[0], cfg.hidden, cfg.heads, cfg.head_dim
    S = st.seq_len
    qpos = torch.arange(S, S + T)
    kpos = torch.arange(S + T)
    mask = kpos[None, :] <= qpos[:, None]                      # [T, S+T]
    for l in range(cfg.layers):
        p = f"encoder.layers.{l}"
        h = F.layer_norm(x, (H,), w[f"{p}.attn_norm.weight"], w[f"{p}.attn_norm.bias"], cfg.ln_eps)
        q = _lin(h, w, f"{p}.attn.q_proj", bias=False).reshape(T, nh, dh)
        k = _lin(h, w, f"{p}.attn.k_proj", bias=False).reshape(T, nh, dh)
        v = _lin(h, w, f"{p}.attn.v_proj", bias=False).reshape(T, nh, dh)
        st.k[l] = torch.cat([st.k[l], k], dim=0)
        st.v[l] = torch.cat([st.v[l], v], dim=0)
        s = torch.einsum("qhd,khd->hqk", q, st.k[l]) / dh ** 0.5
        s = s.masked_fill(~mask[None], float("-inf"))
        o = torch.einsum("hqk,khd->qhd", torch.softmax(s, dim=-1), st.v[l]).reshape(T, H)
        x = x + _lin(o, w, f"{p}.attn.o_proj")
        h = F.layer_norm(x, (H,), w[f"{p}.ffn_norm.weight"], w[f"{p}.ffn_norm.bias"], cfg.ln_eps)
        x = x + _lin(F.silu(_lin(h, w, f"{p}.ffn.fc1")), w, f"{p}.ffn.fc2")
    return x


def project(w, cfg: PEConfig, x: torch.Tensor) -> torch.Tensor:
    """[T, hidden] rows (T a multiple of 8) -> [T/8, out_dim] embeddings."""
    return _lin(x.reshape(-1, cfg.rows * cfg.hidden), w, "out_proj")


def decode_patch(w, cfg: PEConfig, st: PEState, patch: torch.Tensor) -> torch.Tensor:
    """One latent patch [patch, ld] -> embedding [out_dim]; advances ``st``."""
    frames = patch.float()
    x = _lin(downsample(w, frames, st.tail), w, "in_proj")
    st.tail = frames[-1].clone()
    return project(w, cfg, encoder_rows(w, cfg, st, x))[0]


def decode_batch(w, cfg: PEConfig, states: list[PEState], patches: torch.Tensor) -> torch.Tensor:
    """patches [n, patch, ld] for n requests -> [n, out_dim]."""
    return torch.stack([decode_patch(w, cfg, st, patches[i]) for i, st in enumerate(states)])


def prefill(w, cfg: PEConfig, st: PEState, prompt: torch.Tensor) -> torch.Tensor:
    """A whole prompt [frames, ld] (frames a multiple of the patch) through the
    conv and one causal pass -> [frames / patch, out_dim]; leaves ``st`` ready
    for the next ``decode_patch``.  As in the reference, the conv pads the
    prompt with a zero frame (``layers.py:48-50``), whatever tail ``st`` holds."""
    frames = prompt.float()
    if frames.shape[0] % cfg.patch:
        raise ValueError("prompt length must be a multiple of the patch size")
    if frames.shape[0] == 0:
        return torch.zeros(0, cfg.out_dim)
    x = _lin(downsample(w, frames, torch.zeros(cfg.latent_dim)), w, "in_proj")
    st.tail = frames[-1].clone()
    return project(w, cfg, encoder_rows(w, cfg, st, x))
