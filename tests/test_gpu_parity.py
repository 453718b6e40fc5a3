"""End-to-end FM-head parity: one ``dfm_step`` tick through the C ABI against
the golden vectors made by the reference code and against the CPU oracle.

Tolerance (bf16 path, after 4 NFE): per-frame cosine >= 0.9999 and
max-abs <= 2e-2 against the fp32 reference."""
from __future__ import annotations

import pytest
import torch

from conftest import cos_min
from nanovllm_dots_b200 import synthetic as syn
from nanovllm_dots_b200.fm_head import B200FMHead
from oracle import dit_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
COS, MAXABS = 0.9999, 2e-2


@pytest.fixture(scope="module")
def head(weights):
    h = B200FMHead(weights, syn.BASE, num_pages=4800, max_pages_per_req=140, max_requests=64,
                   device=DEV)
    yield h
    h.close()


def _run(head, batch, rids, n_extend=None):
    for rid in list(head.requests):
        head.release(rid)
    for i, rid in enumerate(rids):
        head.write_prefix(rid, syn.request_kv(batch, i))
    d = lambda t: None if t is None else t.to(DEV).contiguous()
    ne = batch.n_extend if n_extend is None else n_extend
    out = head.tick(rids, noise=d(batch.noise), act_hidden=d(batch.cond),
                    ext_hidden=d(batch.prev_hidden), ext_latent=d(batch.prev_latent),
                    g_cond=d(batch.g_cond), n_extend=ne)
    head.check_errors()
    return out.float().cpu()


def _assert_close(out, ref, label):
    c = cos_min(out, ref)
    e = (out - ref).abs().max().item()
    assert c >= COS and e <= MAXABS, f"{label}: cos_min={c:.6f} max_abs={e:.4g}"


def test_cfg0_first_patch(head, golden):
    _, arr = golden
    b = syn.make_batch(1, [0], seed=0, n_extend=[0])
    out = _run(head, b, ["c0"])
    _assert_close(out[0], arr["cfg0_z"], "cfg0")


def test_cfg1_golden(head, golden):
    _, arr = golden
    b = syn.config_batch("cfg1")
    out = _run(head, b, [f"c1_{i}" for i in range(b.n)])
    _assert_close(out, arr["cfg1_z"], "cfg1")


def test_long_prefix_golden(head, golden):
    man, arr = golden
    c = man["cases"]["long"]
    b = syn.make_batch(2, c["prefix_patches"], seed=c["seed"])
    out = _run(head, b, ["l0", "l1"])
    _assert_close(out, arr["long_z"], "long")


def test_gcond_and_first_patch_golden(head, golden):
    man, arr = golden
    c = man["cases"]["gcond"]
    b = syn.make_batch(3, c["prefix_patches"], seed=c["seed"], n_extend=c["n_extend"], with_g=True)
    out = _run(head, b, ["g0", "g1", "g2"])
    _assert_close(out, arr["gcond_z"], "gcond")


def test_trajectory_matches_full_path(head, weights, golden):
    """Requests decoded tick by tick from an empty history (the cache built by
    the kernels' own graduating-row writes) reproduce the reference's full
    O(P^2) batched_meanflow outputs; both requests share each tick."""
    man, arr = golden
    cfg = syn.BASE
    conds, noises, gold = [], [], []
    for r in range(2):
        t = man["cases"]["traj"][f"traj{r}"]
        g = torch.Generator().manual_seed(t["seed"])
        conds.append(torch.randn(t["ticks"], cfg.cond_dim, generator=g).to(torch.bfloat16))
        noises.append(torch.randn(t["ticks"], cfg.latent_patch, cfg.latent_dim,
                                  generator=g).to(torch.bfloat16))
        gold.append(arr[f"traj{r}_z"])
    rids = ["t0", "t1"]
    for rid in rids:
        head.release(rid)
    for tick in range(3):
        live = [r for r in range(2) if tick < gold[r].shape[0]]
        noise = torch.stack([noises[r][tick] for r in live]).to(DEV)
        act = torch.stack([conds[r][tick] for r in live]).to(DEV)
        if tick == 0:
            out = head.tick([rids[r] for r in live], noise=noise, act_hidden=act)
        else:
            eh = torch.stack([conds[r][tick - 1] for r in live]).to(DEV)
            el = torch.stack([gold[r][tick - 1] for r in live]).to(torch.bfloat16).to(DEV)
            out = head.tick([rids[r] for r in live], noise=noise, act_hidden=act,
                            ext_hidden=eh, ext_latent=el)
        head.check_errors()
        for j, r in enumerate(live):
            _assert_close(out[j].float().cpu(), gold[r][tick], f"traj{r} tick{tick}")


def _run_checked(head, weights, batch, rids, check):
    """One tick of every request of ``batch`` (cached prefixes installed
    first), and the oracle's result for the requests in ``check``; each
    request's cached K/V is drawn once and used by both."""
    cfg = syn.BASE
    for rid in list(head.requests):
        head.release(rid)
    refs = {}
    for i, rid in enumerate(rids):
        kv = syn.request_kv(batch, i)
        head.write_prefix(rid, kv)
        if i in check:
            act, ext = O.project_rows(weights, cfg, cond=batch.cond[i],
                                      prev_hidden=batch.prev_hidden[i],
                                      prev_latent=batch.prev_latent[i],
                                      n_extend=batch.n_extend[i])
            g = None if batch.g_cond is None else batch.g_cond[i]
            refs[i], _ = O.tick_request(weights, cfg, noise=batch.noise[i], act_row=act,
                                        ext_rows=ext, kv=kv.float(), g_cond=g)
        del kv
    d = lambda t: None if t is None else t.to(DEV).contiguous()
    out = head.tick(rids, noise=d(batch.noise), act_hidden=d(batch.cond),
                    ext_hidden=d(batch.prev_hidden), ext_latent=d(batch.prev_latent),
                    g_cond=d(batch.g_cond), n_extend=batch.n_extend)
    head.check_errors()
    return out.float().cpu(), refs


def test_cfg2_full_tick_against_oracle(head, weights):
    """BASELINE config 2 at full size: 64 requests with prefixes of 17*U{0..120}
    rows in one tick; every request is checked against the oracle."""
    b = syn.config_batch("cfg2")
    out, refs = _run_checked(head, weights, b, [f"c2_{i}" for i in range(b.n)], set(range(b.n)))
    ref = torch.stack([refs[i] for i in range(b.n)])
    _assert_close(out, ref, "cfg2 (64 requests)")


def test_cfg4_mix_against_oracle(weights):
    """BASELINE config 4's per-GPU batch: 64 requests, 75% short prefixes
    (U{0..60} patches) and 25% long ones (U{200..320} patches, 3400-5440
    rows, each split over two attention work units).  Every long request and
    eight short ones are checked against the oracle."""
    cfg = syn.BASE
    b = syn.config_batch("cfg4")
    pages = sum(-(-(p + 2 * cfg.stride) // cfg.page_rows) for p in b.prefix_rows) + 8
    width = max(-(-(p + 2 * cfg.stride) // cfg.page_rows) for p in b.prefix_rows)
    h = B200FMHead(weights, cfg, num_pages=pages, max_pages_per_req=width, max_requests=64,
                   device=DEV)
    long_ = [i for i in range(b.n) if b.prefix_rows[i] >= 200 * cfg.stride]
    short = [i for i in range(b.n) if b.prefix_rows[i] < 200 * cfg.stride][:8]
    assert len(long_) >= 8 and max(b.prefix_rows) > 4096
    try:
        out, refs = _run_checked(h, weights, b, [f"c4_{i}" for i in range(b.n)], set(long_ + short))
    finally:
        h.close()
    pick = sorted(refs)
    _assert_close(out[pick], torch.stack([refs[i] for i in pick]), "cfg4 mix")


def test_graduating_rows_persist_in_cache(head, weights):
    """The K/V the tick writes for graduating rows equal the oracle's."""
    cfg = syn.BASE
    b = syn.make_batch(1, [2], seed=77)
    _run(head, b, ["kv0"])
    P = b.prefix_rows[0]
    act, ext = O.project_rows(weights, cfg, cond=b.cond[0], prev_hidden=b.prev_hidden[0],
                              prev_latent=b.prev_latent[0], n_extend=17)
    _, new = O.tick_request(weights, cfg, noise=b.noise[0], act_row=act, ext_rows=ext,
                            kv=syn.request_kv(b, 0).float())
    pages = head.pages.pages["kv0"]
    view = head.pool_view()
    got = torch.stack([view[:, :, :, pages[(P + j) // 16], :, (P + j) % 16] for j in range(17)], 3)
    got = got.permute(1, 0, 2, 3, 4, 5).float().cpu()          # [nfe, L, 2, 17, heads, dh]
    assert head.requests["kv0"].cache_len == P + 17
    err = (got - new).abs().max().item()
    assert err < 5e-2, err
    assert cos_min(got, new) > 0.9999


def test_batch_invariance_and_determinism(head):
    """Same inputs give the same bits; a request's result does not depend on
    the batch it shares a tick with."""
    b = syn.make_batch(5, [0, 3, 9, 30, 1], seed=91)
    out_all = _run(head, b, [f"bi{i}" for i in range(5)])
    again = _run(head, b, [f"bi{i}" for i in range(5)])
    assert torch.equal(out_all, again)
    head.release("solo")
    head.write_prefix("solo", syn.request_kv(b, 3))
    d = lambda t: t[3:4].to(DEV).contiguous()
    one = head.tick(["solo"], noise=d(b.noise), act_hidden=d(b.cond), ext_hidden=d(b.prev_hidden),
                    ext_latent=d(b.prev_latent), n_extend=[17])
    assert torch.equal(one.float().cpu()[0], out_all[3])


def test_graph_replay_matches_eager(head):
    """The captured tick (static buffers, one graph launch) equals the eager call."""
    cfg = syn.BASE
    b = syn.make_batch(4, [5, 0, 20, 2], seed=61, n_extend=[17, 0, 17, 17])
    for rid in list(head.requests):
        head.release(rid)
    rids = [f"gr{i}" for i in range(4)]
    for i, rid in enumerate(rids):
        head.write_prefix(rid, syn.request_kv(b, i))
    cl, ne, bt = head.prepare(rids, b.n_extend)
    d = lambda t: t.to(DEV).contiguous()
    eager = torch.empty(4, cfg.latent_patch, cfg.latent_dim, dtype=torch.bfloat16, device=DEV)
    head.launch(noise=d(b.noise), act_hidden=d(b.cond), ext_hidden=d(b.prev_hidden),
                ext_latent=d(b.prev_latent), cache_len=cl, n_extend=ne, block_table=bt, out=eager)
    tg = head.graph(4)
    for k, v in (("noise", b.noise), ("act_hidden", b.cond), ("ext_hidden", b.prev_hidden),
                 ("ext_latent", b.prev_latent), ("cache_len", cl), ("n_extend", ne),
                 ("block_table", bt)):
        tg.inputs[k].copy_(v)
    out = tg.replay().clone()
    out2 = tg.replay().clone()
    head.check_errors()
    assert torch.equal(out, eager) and torch.equal(out2, eager)


def test_device_error_on_bad_block_table(head):
    """A block table pointing outside the pool is reported, not a fault."""
    cfg = syn.BASE
    noise = torch.zeros(1, cfg.latent_patch, cfg.latent_dim, dtype=torch.bfloat16, device=DEV)
    act = torch.zeros(1, cfg.cond_dim, dtype=torch.bfloat16, device=DEV)
    cl = torch.zeros(1, dtype=torch.int32, device=DEV)
    ne = torch.zeros(1, dtype=torch.int32, device=DEV)
    bt = torch.full((1, head.max_pages_per_req), 10 ** 6, dtype=torch.int32, device=DEV)
    out = torch.empty_like(noise)
    head.launch(noise=noise, act_hidden=act, cache_len=cl, n_extend=ne, block_table=bt, out=out)
    with pytest.raises(RuntimeError, match="page"):
        head.check_errors()
    head.check_errors()   # cleared


def test_device_error_on_cache_longer_than_the_block_table(head):
    """A cache length the block table cannot hold is reported as a length
    error (no K/V write, no attention over it), and the next good tick runs."""
    cfg = syn.BASE
    noise = torch.zeros(1, cfg.latent_patch, cfg.latent_dim, dtype=torch.bfloat16, device=DEV)
    act = torch.zeros(1, cfg.cond_dim, dtype=torch.bfloat16, device=DEV)
    cl = torch.full((1,), head.max_pages_per_req * cfg.page_rows, dtype=torch.int32, device=DEV)
    ne = torch.zeros(1, dtype=torch.int32, device=DEV)
    bt = torch.zeros((1, head.max_pages_per_req), dtype=torch.int32, device=DEV)
    out = torch.empty_like(noise)
    head.launch(noise=noise, act_hidden=act, cache_len=cl, n_extend=ne, block_table=bt, out=out)
    with pytest.raises(RuntimeError, match="len"):
        head.check_errors()
    b = syn.make_batch(1, [1], seed=8)
    good = _run(head, b, ["after_len_error"])
    assert torch.isfinite(good).all()


def test_prime_equals_tick_by_tick(head):
    """Bulk prefill (``prime``) of three patches of history rows leaves the
    same cache as graduating them over three ticks: the next tick's latents
    are identical."""
    cfg = syn.BASE
    g = torch.Generator().manual_seed(5)
    rows = (torch.randn(51, cfg.hidden, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    act = (torch.randn(1, cfg.hidden, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    noise = torch.randn(1, cfg.latent_patch, cfg.latent_dim, generator=g).to(torch.bfloat16).to(DEV)
    for rid in ("pr", "tt"):
        head.release(rid)
    head.prime(["pr"], [rows])
    zero_noise = torch.zeros(1, cfg.latent_patch, cfg.latent_dim, dtype=torch.bfloat16, device=DEV)
    zero_act = torch.zeros(1, cfg.hidden, dtype=torch.bfloat16, device=DEV)
    for t in range(3):
        head.tick(["tt"], noise=zero_noise, act_row=zero_act,
                  ext_rows=rows[17 * t:17 * t + 17].unsqueeze(0), n_extend=[17])
    assert head.requests["pr"].cache_len == head.requests["tt"].cache_len == 51
    a = head.tick(["pr"], noise=noise, act_row=act)
    b = head.tick(["tt"], noise=noise, act_row=act)
    head.check_errors()
    assert torch.isfinite(a.float()).all()
    assert torch.equal(a, b)


def test_long_requests_split_over_attention_units(weights):
    """Config-4 lengths: a request longer than one attention work unit (4096
    keys) is split over two units whose partials are merged, next to short
    requests in the same tick; checked against the oracle."""
    b = syn.make_batch(3, [247, 2, 60], seed=44)         # 4199, 34 and 1020 cached rows
    h = B200FMHead(weights, syn.BASE, num_pages=400, max_pages_per_req=270, max_requests=4,
                   device=DEV)
    try:
        out = _run(h, b, ["L0", "L1", "L2"])
    finally:
        h.close()
    ref = O.tick_batch(weights, b, syn.BASE)
    _assert_close(out, ref, "long split")
