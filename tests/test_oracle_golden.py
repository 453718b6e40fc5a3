"""The CPU oracle against the golden vectors made by the reference's own code
(``tests/golden/make_golden.py``).  This pins the oracle before any CUDA result
is compared with it."""
from __future__ import annotations

import torch

from nanovllm_dots_b200 import synthetic as syn
from oracle import dit_oracle as O

TOL = 2e-5   # fp32 vs fp32, different summation order only


def test_weights_match_reference_construction(weights, golden):
    man, _ = golden
    assert syn.weights_digest(weights) == man["weights_sha256"]


def _check_inputs(batch, case):
    d = case["inputs"]
    assert syn.tensor_digest(batch.noise) == d["noise"]
    assert syn.tensor_digest(batch.cond) == d["cond"]
    assert syn.tensor_digest(batch.prev_latent) == d["prev_latent"]
    assert syn.tensor_digest(syn.request_kv(batch, 0)) == d["kv0"]


def test_cfg0_single_forward(weights, golden):
    man, arr = golden
    cfg = syn.BASE
    b = syn.make_batch(1, [0], seed=0, n_extend=[0])
    _check_inputs(b, man["cases"]["cfg0"])
    act, _ = O.project_rows(weights, cfg, cond=b.cond[0], prev_hidden=None, prev_latent=None,
                            n_extend=0)
    x = torch.cat([act.reshape(1, -1), O.linear(b.noise[0].float(), weights, "coordinate_proj")])
    ts, dts = syn.time_grid(cfg.nfe)
    v = O.dit_forward_full(weights, cfg, x, ts[0], dts[0])[1:]
    assert (v - arr["cfg0_v"]).abs().max().item() < TOL
    z = O.tick_batch(weights, b, cfg)[0]
    assert (z - arr["cfg0_z"]).abs().max().item() < TOL


def test_cfg1_cache_path(weights, golden):
    man, arr = golden
    b = syn.config_batch("cfg1")
    _check_inputs(b, man["cases"]["cfg1"])
    assert b.prefix_rows == man["cases"]["cfg1"]["prefix_rows"]
    z = O.tick_batch(weights, b)
    assert (z - arr["cfg1_z"]).abs().max().item() < TOL


def test_gcond_and_first_patch(weights, golden):
    man, arr = golden
    c = man["cases"]["gcond"]
    b = syn.make_batch(3, c["prefix_patches"], seed=c["seed"], n_extend=c["n_extend"], with_g=True)
    assert syn.tensor_digest(b.g_cond) == c["inputs"]["g_cond"]
    z = O.tick_batch(weights, b)
    assert (z - arr["gcond_z"]).abs().max().item() < TOL


def test_trajectory_cache_equals_full_path(weights, golden):
    """Ticks built from real rows through the cache formulation reproduce the
    reference's full O(P^2) ``batched_meanflow`` outputs."""
    man, arr = golden
    cfg = syn.BASE
    for r in range(2):
        t = man["cases"]["traj"][f"traj{r}"]
        g = torch.Generator().manual_seed(t["seed"])
        conds = torch.randn(t["ticks"], cfg.cond_dim, generator=g).to(torch.bfloat16)
        noises = torch.randn(t["ticks"], cfg.latent_patch, cfg.latent_dim,
                             generator=g).to(torch.bfloat16)
        gold = arr[f"traj{r}_z"]
        kv = torch.zeros(cfg.nfe, cfg.layers, 2, 0, cfg.heads, cfg.head_dim)
        for tick in range(t["ticks"]):
            act = O.linear(conds[tick].float().reshape(1, -1), weights, "hidden_proj")[0]
            ext = None
            if tick > 0:
                ext = torch.cat([O.linear(conds[tick - 1].float().reshape(1, -1), weights,
                                          "hidden_proj"),
                                 O.linear(gold[tick - 1].float(), weights, "latent_proj")])
            z, new = O.tick_request(weights, cfg, noise=noises[tick], act_row=act, ext_rows=ext,
                                    kv=kv)
            kv = torch.cat([kv, new], dim=3)
            assert (z - gold[tick]).abs().max().item() < 1e-4, (r, tick)


def test_time_grid_matches_bf16_linspace():
    ts, dts = syn.time_grid(4)
    ref = torch.linspace(0.0, 1.0, 5, dtype=torch.bfloat16).float()
    assert ts == ref[:-1].tolist()
    assert dts == (ref[1:] - ref[:-1]).tolist()
