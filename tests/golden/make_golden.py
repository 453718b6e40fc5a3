"""Generate the golden FM-head fixtures by running the REFERENCE's own code.

Run in a container where the reference checkout is importable (it is not on
the GPU test box; the fixtures it writes are committed):

    python tests/golden/make_golden.py --reference /path/to/nanovllm_dots

The reference modules used are
``nanovllm_dots/models/dots/native/dit.py`` (``DiT``),
``nanovllm_dots/models/dots/native/model.py`` (``_build_fm_attn_mask``,
``_build_fm_pos_ids``), ``nanovllm_dots/models/dots/batched_fm.py``
(``batched_meanflow``) and ``nanovllm_dots/models/dots/cached_fm.py``
(``FMCache``, ``extend_cache``, ``active_forward``).  ``torchdiffeq`` is only
imported by those modules, never called on the MeanFlow path, so a stub
stands in for it.  Everything runs in fp32 on the CPU with the seeded bf16
weights of ``nanovllm_dots_b200.synthetic``.

Cases (all outputs fp32):
  cfg0       one DiT forward, 1 request, empty prefix, timesteps=0, duration=.25
             full-forward path -> v [16, 64]; plus the
             4-step ``batched_meanflow`` solve -> z [16, 64]
  cfg1       8 requests, prefixes of 17*U{0..32} rows with N(0, .5^2) cached
             K/V, 17 graduating rows each, 4 steps via the cache path
  long       2 requests with 17*120 and 17*45 cached rows (config-2 sizes)
  gcond      3 requests with a non-zero g_cond and one request with no
             graduating rows (first patch)
  traj       2 requests decoded for 3 and 2 ticks from an empty history with the
             full O(P^2) ``batched_meanflow`` path; each tick's output latent
             becomes the next tick's graduating patch
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from nanovllm_dots_b200 import synthetic as syn  # noqa: E402


def load_reference(path):
    sys.modules.setdefault("torchdiffeq", types.SimpleNamespace(odeint=None))
    sys.path.insert(0, path)
    from nanovllm_dots.models.dots.native.dit import DiT
    from nanovllm_dots.models.dots.native.config import TransformerConfig
    from nanovllm_dots.models.dots.native import model as nmodel
    from nanovllm_dots.models.dots import batched_fm, cached_fm
    return DiT, TransformerConfig, nmodel, batched_fm, cached_fm


def build(ref, cfg, w):
    DiT, TransformerConfig, *_ = ref
    tc = TransformerConfig(dict(hidden_size=cfg.hidden, num_layers=cfg.layers,
                                num_heads=cfg.heads, ffn_hidden_size=cfg.ffn,
                                modulation=True, qk_norm=True, rotary_bias=True,
                                rotary_theta=cfg.rotary_theta))
    torch.manual_seed(0)
    dit = DiT(in_dim=cfg.hidden, out_dim=cfg.latent_dim, transformer_config=tc,
              mode="meanflow").eval()
    projs = {n: torch.nn.Linear(i, cfg.hidden) for n, i in
             (("coordinate_proj", cfg.latent_dim), ("hidden_proj", cfg.cond_dim),
              ("latent_proj", cfg.latent_dim))}
    # The seeded init of the reference constructor must equal the factory's.
    ref_sd = {k: v.detach().to(torch.bfloat16).float() for k, v in dit.state_dict().items()
              if not k.endswith("inv_freq")}
    for n, m in projs.items():
        for k, v in m.state_dict().items():
            ref_sd[f"{n}.{k}"] = v.detach().to(torch.bfloat16).float()
    assert set(ref_sd) == set(w), sorted(set(ref_sd) ^ set(w))[:8]
    for k in w:
        assert torch.equal(ref_sd[k], w[k]), k
    with torch.no_grad():
        dit.load_state_dict({k: w[k] for k in dit.state_dict() if not k.endswith("inv_freq")},
                            strict=False)
        for n, m in projs.items():
            m.weight.copy_(w[f"{n}.weight"])
            m.bias.copy_(w[f"{n}.bias"])
    core = types.SimpleNamespace(
        latent_patch_size=cfg.latent_patch, hidden_patch_size=cfg.hidden_patch,
        latent_dim=cfg.latent_dim, fm_hidden_size=cfg.hidden,
        velocity_field_predictor=dit, **projs)
    return dit, core


def full_inputs(ref, cfg, core, hist):
    """Padded-free full-path inputs for one request: history [L, H]."""
    nmodel = ref[2]
    L = hist.shape[0]
    total = L + cfg.latent_patch
    inp = torch.zeros(1, total, cfg.hidden)
    inp[0, :L] = hist
    mask = torch.zeros(1, total, total, dtype=torch.bool)
    pos = torch.zeros(1, total, dtype=torch.float32)
    st = types.SimpleNamespace(fm_seq_len=L)
    owner = types.SimpleNamespace(core=core)
    nmodel.DotsModel._build_fm_attn_mask(owner, state=st, attn_mask=mask)
    nmodel.DotsModel._build_fm_pos_ids(owner, state=st, pos_ids=pos)
    return inp, mask, pos


def cache_tick(ref, cfg, dit, core, kv, act_row, ext_rows, noise, g_cond):
    """One tick through the reference's cache path for one request."""
    cached_fm = ref[4]
    ts, dts = syn.time_grid(cfg.nfe)
    P = kv.shape[3]
    cache = cached_fm.FMCache(cfg.nfe, cfg.layers)
    for k in range(cfg.nfe):
        for l in range(cfg.layers):
            if P:
                K = kv[k, l, 0].float().permute(1, 0, 2).unsqueeze(0).contiguous()
                V = kv[k, l, 1].float().permute(1, 0, 2).unsqueeze(0).contiguous()
                cache.kv[k][l] = (K, V)
    g = torch.zeros(1, cfg.hidden) if g_cond is None else g_cond.float().reshape(1, -1)
    n_ext = 0 if ext_rows is None else ext_rows.shape[0]
    with torch.no_grad():
        gks = []
        for k in range(cfg.nfe):
            # MeanFlow conditioning through the FM-era helper: duration folded
            # into g (cached_fm._build_c adds only time_embedder(t) + g).
            gk = dit.duration_embedder(torch.tensor([dts[k]])) + g
            gks.append(gk)
            if n_ext:
                pos_new = torch.arange(P, P + n_ext, dtype=torch.float32).reshape(1, -1)
                cached_fm.extend_cache(dit, cache, ext_rows.float().unsqueeze(0), pos_new,
                                       torch.tensor(ts[k]), gk, k)
        Pn = P + n_ext
        pos_act = torch.arange(Pn, Pn + cfg.stride, dtype=torch.float32).reshape(1, -1)
        z = noise.float().reshape(1, cfg.latent_patch, cfg.latent_dim).clone()
        for k in range(cfg.nfe):
            zp = core.coordinate_proj(z)
            x = torch.cat([act_row.float().reshape(1, 1, -1), zp], dim=1)
            v = cached_fm.active_forward(dit, cache, x, pos_act, torch.tensor(ts[k]), gks[k], k)
            z = z + v[:, cfg.hidden_patch:] * dts[k]
    return z[0]


def rows_of(core, cond, prev_hidden, prev_latent, n_ext):
    with torch.no_grad():
        act = core.hidden_proj(cond.float().reshape(1, -1))[0]
        if n_ext == 0:
            return act, None
        eh = core.hidden_proj(prev_hidden.float().reshape(1, -1))
        el = core.latent_proj(prev_latent.float())
        return act, torch.cat([eh, el], 0)[:n_ext]


def run_cache_case(ref, cfg, dit, core, batch):
    outs = []
    for i in range(batch.n):
        act, ext = rows_of(core, batch.cond[i], batch.prev_hidden[i], batch.prev_latent[i],
                           batch.n_extend[i])
        g = None if batch.g_cond is None else batch.g_cond[i]
        outs.append(cache_tick(ref, cfg, dit, core, syn.request_kv(batch, i, cfg), act, ext,
                               batch.noise[i], g))
    return torch.stack(outs, 0)


def batch_digests(batch, cfg):
    d = {"noise": syn.tensor_digest(batch.noise), "cond": syn.tensor_digest(batch.cond),
         "prev_hidden": syn.tensor_digest(batch.prev_hidden),
         "prev_latent": syn.tensor_digest(batch.prev_latent),
         "kv0": syn.tensor_digest(syn.request_kv(batch, 0, cfg))}
    if batch.g_cond is not None:
        d["g_cond"] = syn.tensor_digest(batch.g_cond)
    return d


def traj_inputs(cfg, seed, ticks):
    g = torch.Generator().manual_seed(seed)
    conds = torch.randn(ticks, cfg.cond_dim, generator=g).to(torch.bfloat16)
    noises = torch.randn(ticks, cfg.latent_patch, cfg.latent_dim, generator=g).to(torch.bfloat16)
    return conds, noises


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DFM_REFERENCE"),
                    required=os.environ.get("DFM_REFERENCE") is None,
                    help="reference checkout (or set DFM_REFERENCE)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = syn.BASE
    ref = load_reference(args.reference)
    w = syn.make_weights(cfg, seed=0)
    dit, core = build(ref, cfg, w)
    batched_fm = ref[3]
    arrays, manifest = {}, {"weights_sha256": syn.weights_digest(w), "cases": {}}
    ts, dts = syn.time_grid(cfg.nfe)

    # ---- cfg0: one full DiT forward + the 4-step full solve -------------------
    b0 = syn.make_batch(1, [0], seed=0, cfg=cfg, n_extend=[0])
    with torch.no_grad():
        act, _ = rows_of(core, b0.cond[0], None, None, 0)
        zp = core.coordinate_proj(b0.noise[0].float())
        inp, mask, pos = full_inputs(ref, cfg, core, act.reshape(1, -1))
        inp[0, 1:] = zp
        v0 = dit(x=inp, timesteps=torch.tensor([ts[0]]), duration=torch.tensor([dts[0]]),
                 attn_mask=mask, pos_ids=pos, g_cond=torch.zeros(1, cfg.hidden))[0, 1:]
        inp[0, 1:] = 0
        z0 = batched_fm.batched_meanflow(core, input_sequence=inp, attn_mask=mask, pos_ids=pos,
                                         g_cond=torch.zeros(1, cfg.hidden), num_steps=cfg.nfe,
                                         noise=b0.noise.float(), vfp=dit)[0]
    arrays["cfg0_v"] = v0.numpy()
    arrays["cfg0_z"] = z0.numpy()
    manifest["cases"]["cfg0"] = {"seed": 0, "prefix_patches": [0], "n_extend": [0],
                                 "inputs": batch_digests(b0, cfg)}
    print("cfg0 done", float(v0.abs().max()), float(z0.abs().max()))

    # ---- cfg1 -------------------------------------------------------------------
    b1 = syn.config_batch("cfg1", cfg)
    z1 = run_cache_case(ref, cfg, dit, core, b1)
    arrays["cfg1_z"] = z1.numpy()
    manifest["cases"]["cfg1"] = {"prefix_rows": b1.prefix_rows, "n_extend": b1.n_extend,
                                 "inputs": batch_digests(b1, cfg)}
    print("cfg1 done", b1.prefix_rows)

    # ---- long -------------------------------------------------------------------
    bl = syn.make_batch(2, [120, 45], seed=11, cfg=cfg)
    zl = run_cache_case(ref, cfg, dit, core, bl)
    arrays["long_z"] = zl.numpy()
    manifest["cases"]["long"] = {"seed": 11, "prefix_patches": [120, 45],
                                 "prefix_rows": bl.prefix_rows, "n_extend": bl.n_extend,
                                 "inputs": batch_digests(bl, cfg)}
    print("long done")

    # ---- gcond + a first-patch request ----------------------------------------
    bg = syn.make_batch(3, [3, 0, 7], seed=21, cfg=cfg, n_extend=[17, 0, 17], with_g=True)
    zg = run_cache_case(ref, cfg, dit, core, bg)
    arrays["gcond_z"] = zg.numpy()
    manifest["cases"]["gcond"] = {"seed": 21, "prefix_patches": [3, 0, 7], "n_extend": [17, 0, 17],
                                  "with_g": True, "prefix_rows": bg.prefix_rows,
                                  "inputs": batch_digests(bg, cfg)}
    print("gcond done")

    # ---- traj: full O(P^2) path over real histories -----------------------------
    traj = {}
    for r, (seed, ticks) in enumerate(((31, 3), (32, 2))):
        conds, noises = traj_inputs(cfg, seed, ticks)
        hist = torch.zeros(0, cfg.hidden)
        zs = []
        with torch.no_grad():
            for t in range(ticks):
                hrow = core.hidden_proj(conds[t].float().reshape(1, -1))
                hist = torch.cat([hist, hrow], 0)
                inp, mask, pos = full_inputs(ref, cfg, core, hist)
                z = batched_fm.batched_meanflow(core, input_sequence=inp, attn_mask=mask,
                                                pos_ids=pos, g_cond=torch.zeros(1, cfg.hidden),
                                                num_steps=cfg.nfe, noise=noises[t:t + 1].float(),
                                                vfp=dit)[0]
                zs.append(z)
                hist = torch.cat([hist, core.latent_proj(z)], 0)
        arrays[f"traj{r}_z"] = torch.stack(zs, 0).numpy()
        traj[f"traj{r}"] = {"seed": seed, "ticks": ticks,
                            "conds": syn.tensor_digest(conds), "noises": syn.tensor_digest(noises)}
        print(f"traj{r} done")
    manifest["cases"]["traj"] = traj

    np.savez_compressed(os.path.join(args.out, "fm_golden.npz"), **arrays)
    with open(os.path.join(args.out, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    print("wrote", os.path.join(args.out, "fm_golden.npz"))


if __name__ == "__main__":
    main()
