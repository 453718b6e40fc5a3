"""FP8 path (precision="fp8", config 3): QKV and fc1 on e4m3 operands through
the C ABI.  Tolerance (north_star): per-frame cosine >= 0.999 against the bf16
path on the same inputs, and against the fp32 oracle."""
from __future__ import annotations

import pytest
import torch

from conftest import cos_min
from nanovllm_dots_b200 import synthetic as syn
from nanovllm_dots_b200.fm_head import B200FMHead
from oracle import dit_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
FP8_COS = 0.999


def _run(head, batch, rids):
    for rid in list(head.requests):
        head.release(rid)
    for i, rid in enumerate(rids):
        head.write_prefix(rid, syn.request_kv(batch, i))
    d = lambda t: None if t is None else t.to(DEV).contiguous()
    out = head.tick(rids, noise=d(batch.noise), act_hidden=d(batch.cond),
                    ext_hidden=d(batch.prev_hidden), ext_latent=d(batch.prev_latent),
                    g_cond=d(batch.g_cond), n_extend=batch.n_extend)
    head.check_errors()
    return out.float().cpu()


def test_fp8_matches_bf16_and_oracle(weights):
    b = syn.make_batch(6, [0, 3, 17, 40, 64, 120], seed=21)
    rids = [f"f{i}" for i in range(b.n)]
    outs = {}
    for prec in ("bf16", "fp8"):
        h = B200FMHead(weights, syn.BASE, num_pages=800, max_pages_per_req=140, max_requests=8,
                       device=DEV, precision=prec)
        try:
            outs[prec] = _run(h, b, rids)
        finally:
            h.close()
    ref = O.tick_batch(weights, b, syn.BASE)
    assert torch.isfinite(outs["fp8"]).all()
    c_bf, c_or = cos_min(outs["fp8"], outs["bf16"]), cos_min(outs["fp8"], ref)
    assert c_bf >= FP8_COS, f"fp8 vs bf16 cos_min={c_bf:.6f}"
    assert c_or >= FP8_COS, f"fp8 vs oracle cos_min={c_or:.6f}"
    # the two paths are not the same computation
    assert not torch.equal(outs["fp8"], outs["bf16"])


def test_fp8_cfg3_full_tick_against_bf16(weights):
    """the config-2 workload (64 requests, prefixes of
    17*U{0..120} rows) on the FP8 path, compared with the bf16 path on the
    same inputs over all 64 requests (cos >= 0.999), and with the fp32 oracle
    on four requests."""
    cfg = syn.BASE
    b = syn.config_batch("cfg2")
    pages = sum(-(-(p + 2 * cfg.stride) // cfg.page_rows) for p in b.prefix_rows) + 8
    width = max(-(-(p + 2 * cfg.stride) // cfg.page_rows) for p in b.prefix_rows)
    heads = {prec: B200FMHead(weights, cfg, num_pages=pages, max_pages_per_req=width,
                              max_requests=64, device=DEV, precision=prec)
             for prec in ("bf16", "fp8")}
    rids = [f"c3_{i}" for i in range(b.n)]
    check = sorted({0, 17, max(range(b.n), key=lambda i: b.prefix_rows[i]), 40})
    refs = {}
    try:
        for i, rid in enumerate(rids):
            kv = syn.request_kv(b, i)
            for h in heads.values():
                h.write_prefix(rid, kv)
            if i in check:
                refs[i] = O.tick_batch(weights, b, cfg, kv_fn=lambda _i, kv=kv: kv,
                                       indices=[i])[0]
        d = lambda t: None if t is None else t.to(DEV).contiguous()
        outs = {}
        for prec, h in heads.items():
            o = h.tick(rids, noise=d(b.noise), act_hidden=d(b.cond), ext_hidden=d(b.prev_hidden),
                       ext_latent=d(b.prev_latent), n_extend=b.n_extend)
            h.check_errors()
            outs[prec] = o.float().cpu()
    finally:
        for h in heads.values():
            h.close()
    assert torch.isfinite(outs["fp8"]).all()
    c_bf = cos_min(outs["fp8"], outs["bf16"])
    c_or = cos_min(outs["fp8"][check], torch.stack([refs[i] for i in check]))
    assert c_bf >= FP8_COS, f"cfg3 fp8 vs bf16 cos_min={c_bf:.6f}"
    assert c_or >= FP8_COS, f"cfg3 fp8 vs oracle cos_min={c_or:.6f}"
