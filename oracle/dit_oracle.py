"""CPU oracle for the MeanFlow FM head -- TEST INFRASTRUCTURE ONLY.

Only tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
use this module, and only as the checker or the timed CPU baseline.  The
product path (``nanovllm_dots_b200``) never imports it.

It restates, in plain fp32 torch on the CPU, the reference's per-timestep
prefix-cache formulation of the MeanFlow DiT head:

* condition ``c = time_embedder(t) + duration_embedder(dt) + g_cond``
  (``nanovllm_dots/models/dots/native/dit.py:135-143``), with the sinusoidal
  embedding of ``dit.py:33-42`` and the MLP of ``dit.py:26-30,44-47``;
* ``DiTBlock.forward`` with adaLN modulation (``dit.py:81-108``, chunk order
  shift_a, scale_a, gate_a, shift_f, scale_f, gate_f at ``dit.py:86-87``),
  LayerNorm without affine (``dit.py:70-71``), ``modulate`` (``dit.py:19-20``);
* attention projections with per-head LayerNorm and NeoX rotary
  (``native/layers.py:95-134,181-198``), softmax(QK^T/sqrt(dh))V
  (``layers.py:204-206``) and the GELU(tanh) MLP (``layers.py:78-92``);
* the prefix cache semantics of ``cached_fm.py:124-197``: graduating rows are
  causal among themselves and see the whole cached prefix; active rows (the
  hidden row plus the latent patch) see the prefix, the graduating rows and
  each other; graduating K/V persist, active K/V do not;
* the solver ``z <- z + v * dt`` over ``t_k = k/nfe`` (``batched_fm.py:110-126``)
  with ``coordinate_proj`` feeding the latent rows (``batched_fm.py:117-119``);
* the final layer (``dit.py:50-63``), whose hidden-row output is dropped
  (``cached_fm.py:290``).

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own
``DiT.forward``/``batched_meanflow`` and ``cached_fm.extend_cache``/
``active_forward`` on the same seeded inputs; ``tests/test_oracle_golden.py``
checks this module against those fixtures.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from nanovllm_dots_b200.synthetic import BASE, FMConfig, time_grid


# --------------------------------------------------------------------------- #
# Building blocks                                                              #
# --------------------------------------------------------------------------- #
def timestep_embedding(t: torch.Tensor, dim: int = 256, max_period: float = 10000.0):
    """[cos(t*f) | sin(t*f)], f_i = exp(-ln(max_period) * i / (dim/2))
    (``dit.py:33-42``)."""
    half = dim // 2
    freqs = torch.exp(-math.log(max_period)
                      * torch.arange(half, dtype=torch.float32) / half)
    args = t.reshape(-1, 1).float() * freqs[None]
    return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)


def linear(x, w, name, bias=True):
    y = x @ w[f"{name}.weight"].t()
    if bias:
        y = y + w[f"{name}.bias"]
    return y


def embedder(w, name, t):
    """TimestepEmbedder.forward: Linear -> SiLU -> Linear (``dit.py:26-30,44-47``)."""
    h = linear(timestep_embedding(t), w, f"{name}.mlp.0")
    return linear(F.silu(h), w, f"{name}.mlp.2")


def condition(w, t: float, dt: float, g_cond: torch.Tensor | None, n: int):
    """c = temb(t) + demb(dt) (+ g_cond), one row per request (``dit.py:137-143``)."""
    tt = torch.full((n,), t, dtype=torch.float32)
    dd = torch.full((n,), dt, dtype=torch.float32)
    c = embedder(w, "time_embedder", tt) + embedder(w, "duration_embedder", dd)
    if g_cond is not None:
        c = c + g_cond.float()
    return c


def layer_norm(x, eps=1e-5):
    return F.layer_norm(x, (x.shape[-1],), eps=eps)


def modulate(x, shift, scale):
    """``dit.py:19-20``; shift/scale broadcast over rows."""
    return x * (1 + scale) + shift


def rotary(pos: torch.Tensor, dh: int, theta: float):
    """NeoX rotary angles cat(freqs, freqs) with inv_freq = theta^(-2i/dh)
    (``layers.py:95-134``).  pos: [m] -> [m, dh]."""
    inv = 1.0 / (theta ** (torch.arange(0, dh, 2).float() / dh))
    f = pos.float()[:, None] * inv[None]
    return torch.cat([f, f], dim=-1)


def apply_rotary(x, ang):
    """x*cos + rotate_half(x)*sin (``layers.py:95-100``); x [m, heads, dh]."""
    x1, x2 = x.chunk(2, dim=-1)
    rot = torch.cat([-x2, x1], dim=-1)
    return x * ang.cos()[:, None] + rot * ang.sin()[:, None]


# --------------------------------------------------------------------------- #
# One request, one tick                                                        #
# --------------------------------------------------------------------------- #
def _block_rows(w, l, cfg, h, c, pos, kv_layer, n_ext, lims):
    """One DiT block over the rows of one request.

    h      [m, H] rows (n_ext graduating rows first, then active rows)
    kv_layer (K, V) cached prefix [P, heads, dh] (fp32)
    lims   [m] number of keys (prefix + new rows) each row may attend to
    Returns (h_out, K_new, V_new) where K_new/V_new are the graduating rows' K/V.
    """
    H, nh, dh = cfg.hidden, cfg.heads, cfg.head_dim
    b = f"blocks.{l}"
    mod = linear(F.silu(c), w, f"{b}.adaLN_modulation.1")
    sa, sca, ga, sf, scf, gf = mod.chunk(6, dim=-1)
    m = h.shape[0]
    x = modulate(layer_norm(h, cfg.ln_eps), sa, sca)
    q = linear(x, w, f"{b}.attn.q_proj", bias=False).view(m, nh, dh)
    k = linear(x, w, f"{b}.attn.k_proj", bias=False).view(m, nh, dh)
    v = linear(x, w, f"{b}.attn.v_proj", bias=False).view(m, nh, dh)
    q = F.layer_norm(q, (dh,), w[f"{b}.attn.q_norm.weight"], w[f"{b}.attn.q_norm.bias"], cfg.ln_eps)
    k = F.layer_norm(k, (dh,), w[f"{b}.attn.k_norm.weight"], w[f"{b}.attn.k_norm.bias"], cfg.ln_eps)
    ang = rotary(pos, dh, cfg.rotary_theta)
    q, k = apply_rotary(q, ang), apply_rotary(k, ang)
    K = torch.cat([kv_layer[0], k], dim=0)          # [P+m, heads, dh]
    V = torch.cat([kv_layer[1], v], dim=0)
    T = K.shape[0]
    s = torch.einsum("mhd,thd->hmt", q, K) / math.sqrt(dh)
    keep = torch.arange(T)[None, :] < lims[:, None]  # [m, T]
    s = s.masked_fill(~keep[None], float("-inf"))
    o = torch.einsum("hmt,thd->mhd", torch.softmax(s, dim=-1), V).reshape(m, H)
    h = h + ga * linear(o, w, f"{b}.attn.o_proj")
    x = modulate(layer_norm(h, cfg.ln_eps), sf, scf)
    u = F.gelu(linear(x, w, f"{b}.ffn.fc1"), approximate="tanh")
    h = h + gf * linear(u, w, f"{b}.ffn.fc2")
    return h, k[:n_ext], v[:n_ext]


def tick_request(w, cfg: FMConfig, *, noise, act_row, ext_rows, kv, g_cond=None):
    """Run one FM-head tick for ONE request.

    noise    [lp, ld]          starting z
    act_row  [H]               active hidden row in DiT input space
                               (``hidden_proj`` output, ``model.py:101-110``)
    ext_rows [n_ext, H]        graduating rows in DiT input space, or None
    kv       fp32 [nfe, layers, 2, P, heads, dh] cached prefix K/V
    g_cond   [H] or None
    Returns (z_out [lp, ld], new_kv [nfe, layers, 2, n_ext, heads, dh]).
    """
    H, lp = cfg.hidden, cfg.latent_patch
    P = kv.shape[3]
    n_ext = 0 if ext_rows is None else ext_rows.shape[0]
    m = n_ext + cfg.hidden_patch + lp
    pos = torch.arange(P, P + m, dtype=torch.float32)
    lims = torch.full((m,), P + m, dtype=torch.long)
    lims[:n_ext] = P + torch.arange(1, n_ext + 1)
    ts, dts = time_grid(cfg.nfe)
    z = noise.float().clone()
    g = None if g_cond is None else g_cond.reshape(1, H).float()
    new_kv = torch.zeros(cfg.nfe, cfg.layers, 2, n_ext, cfg.heads, cfg.head_dim)
    for k in range(cfg.nfe):
        c = condition(w, ts[k], dts[k], g, 1)                       # [1, H]
        zp = linear(z, w, "coordinate_proj")                  # [lp, H]
        parts = ([ext_rows.float()] if n_ext else []) + [act_row.reshape(1, H).float(), zp]
        h = linear(torch.cat(parts, dim=0), w, "input_layer")
        for l in range(cfg.layers):
            h, kn, vn = _block_rows(w, l, cfg, h, c, pos, (kv[k, l, 0], kv[k, l, 1]), n_ext, lims)
            new_kv[k, l, 0], new_kv[k, l, 1] = kn, vn
        mod = linear(F.silu(c), w, "output_layer.adaLN_modulation.1")
        sh, sc = mod.chunk(2, dim=-1)
        lat = h[n_ext + cfg.hidden_patch:]
        vel = linear(modulate(layer_norm(lat, cfg.ln_eps), sh, sc), w, "output_layer.linear")
        z = z + vel * dts[k]
    return z, new_kv


def project_rows(w, cfg: FMConfig, *, cond, prev_hidden, prev_latent, n_extend):
    """DiT-input-space rows of one request: the active hidden row
    ``hidden_proj(cond)`` and the graduating rows
    ``[hidden_proj(prev_hidden), latent_proj(prev_latent)]`` (``model.py:101-120``)."""
    act = linear(cond.float().reshape(1, -1), w, "hidden_proj")[0]
    if n_extend == 0:
        return act, None
    eh = linear(prev_hidden.float().reshape(1, -1), w, "hidden_proj")
    el = linear(prev_latent.float(), w, "latent_proj")
    rows = torch.cat([eh, el], dim=0)
    return act, rows[:n_extend]


def dit_forward_full(w, cfg: FMConfig, x, t: float, dt: float, g_cond=None, fm_seq_len=1):
    """The reference's full (uncached) DiT forward on ONE padded-free sequence
    with the FM mask of ``model.py:57-75`` and positions of ``model.py:77-87``
    (history of ``fm_seq_len`` rows followed by the latent slot).  Used for
    config 0 (empty prefix) and to pin the cache path.  x: [L, H] -> [L, ld]."""
    L = x.shape[0]
    lp = cfg.latent_patch
    hist = fm_seq_len
    assert L == hist + lp
    block_start = hist - cfg.hidden_patch
    lims = torch.full((L,), L, dtype=torch.long)
    lims[:block_start] = torch.arange(1, block_start + 1)
    pos = torch.arange(L, dtype=torch.float32)
    empty = torch.zeros(0, cfg.heads, cfg.head_dim)
    c = condition(w, t, dt, None if g_cond is None else g_cond.reshape(1, -1), 1)
    h = linear(x.float(), w, "input_layer")
    for l in range(cfg.layers):
        h, _, _ = _block_rows(w, l, cfg, h, c, pos, (empty, empty), 0, lims)
    mod = linear(F.silu(c), w, "output_layer.adaLN_modulation.1")
    sh, sc = mod.chunk(2, dim=-1)
    return linear(modulate(layer_norm(h, cfg.ln_eps), sh, sc), w, "output_layer.linear")


def tick_batch(w, batch, cfg: FMConfig = BASE, kv_fn=None, indices=None):
    """Oracle tick for every request of a ``synthetic.RequestBatch``.
    ``kv_fn(i)`` returns request i's cached K/V (bf16 or fp32); defaults to the
    seeded draw.  Returns z_out [len(indices), lp, ld] fp32."""
    from nanovllm_dots_b200.synthetic import request_kv
    if kv_fn is None:
        kv_fn = lambda i: request_kv(batch, i, cfg)
    idx = range(batch.n) if indices is None else indices
    outs = []
    for i in idx:
        act, ext = project_rows(w, cfg, cond=batch.cond[i], prev_hidden=batch.prev_hidden[i],
                                prev_latent=batch.prev_latent[i], n_extend=batch.n_extend[i])
        g = None if batch.g_cond is None else batch.g_cond[i]
        z, _ = tick_request(w, cfg, noise=batch.noise[i], act_row=act, ext_rows=ext,
                            kv=kv_fn(i).float(), g_cond=g)
        outs.append(z)
    return torch.stack(outs, 0)


def history_tick(w, cfg: FMConfig, rows: torch.Tensor, noise, g_cond=None):
    """One engine tick of ONE request from its whole FM history, the way the
    reference engine feeds ``_pack_fm_inputs`` + ``batched_meanflow``
    (``engine.py:635-709``): ``rows`` [L, H] are the projected history rows
    (``gen_state.fm_sequence[0, :fm_seq_len]``, ``model.py:101-120``), the last
    one being the active hidden row.  The prefix rows [0, L-1) are causal
    among themselves (``model.py:57-75``), so their K/V are built here by
    graduating them through the cache path in chunks of at most ``stride``
    rows (any chunking gives the same cache), then the active rows run against
    it.  Returns z [lp, ld]."""
    L = rows.shape[0]
    kv = torch.zeros(cfg.nfe, cfg.layers, 2, 0, cfg.heads, cfg.head_dim)
    dummy_noise = torch.zeros(cfg.latent_patch, cfg.latent_dim)
    for s in range(0, L - 1, cfg.stride):
        e = min(L - 1, s + cfg.stride)
        _, new = tick_request(w, cfg, noise=dummy_noise, act_row=torch.zeros(cfg.hidden),
                              ext_rows=rows[s:e].float(), kv=kv, g_cond=g_cond)
        kv = torch.cat([kv, new], dim=3)
    z, _ = tick_request(w, cfg, noise=noise, act_row=rows[L - 1].float(), ext_rows=None, kv=kv,
                        g_cond=g_cond)
    return z
