#!/usr/bin/env python
"""FM-head benchmark: latent xRT of one engine tick, 64 concurrent requests per GPU.

    python bench.py [--gpus N --steps K --warmup W] [--impl b200|reference] [--workload cfg2]

A step is one FM-head tick for every request on the GPU: each request graduates
its previous patch's 17 rows into its paged per-(layer, step) K/V cache and
runs the 4 MeanFlow solver steps (prefixes of 17*U{0..120}
rows, 16-row pages, seeded synthetic DiT).  xRT = requests * 16 frames * 0.04 s
per tick / tick time (``scripts/bench_engine.py:25-27,133-143`` of the reference).
Cache lengths are held fixed across timed ticks so every tick does the same
work.  The K/V pool (~15 GB) and the weights (~465 MB) exceed the 126 MB L2, so
no flush is needed between ticks.

Multi-GPU (torchrun): one process per GPU, each with its own head and 64
requests (weak scaling, no collective on the data path); time = max over ranks.

``--impl reference`` times the reference's algorithm on the host CPU (the oracle
restatement of the reference's cache path; the reference itself is Python with
no GPU MeanFlow cache head) on a bounded sample of the same workload.

Other rows of the build, each with its own metric line (not the headline):
``--workload pe`` (the patch encoder: one batched decode_patch of 64 requests),
``--workload llmattn`` (the LLM backbone's paged decode attention, one layer),
``--workload llmdecode`` (the whole 28-layer backbone decode step) and
``--workload voc`` / ``voc1`` (the vocoder: strict streaming / one-shot).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

AUDIO_S_PER_PATCH = 16 * 0.04
METRIC = "FM-head latent xRT (audio-s/s) at conc 64 per GPU"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="cfg2",
                    choices=["cfg1", "cfg2", "cfg3", "cfg4", "prof", "gemm64", "gemm64fp8", "pe", "llmattn",
                             "llmdecode", "engine", "voc", "voc1", "vocprof"],
                    help="cfg3 = cfg2 on the FP8 path (QKV and fc1 on e4m3 operands); "
                         "prof = the first 16 requests of cfg2 (a few GB, for ncu captures); "
                         "gemm64 = 64 requests with empty prefixes (config-2 GEMM shapes, tiny pool); "
                         "gemm64fp8 = gemm64 on the FP8 path; "
                         "pe = the patch encoder (the step after the FM head): one batched "
                         "decode_patch for 64 requests with cfg2's history lengths; "
                         "llmattn = the LLM backbone's paged decode attention (one layer, 64 "
                         "sequences, Qwen2 GQA 12/2 x 128); llmdecode = the whole backbone "
                         "decode step (28 layers, 64 sequences); engine = the engine drop-in "
                         "(fm_accel='b200' dispatch over engine-style histories) against dfm_step "
                         "alone; voc = the vocoder streaming 16-frame chunks for 64 requests; "
                         "voc1 = the vocoder decoding 64 10-second utterances one-shot; vocprof = voc "
                         "with 16 requests (a small case for ncu captures)")
    ap.add_argument("--cpu-sample", type=int, default=64,
                    help="requests in the CPU baseline sample (64 = one whole tick)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-tick", action="store_true",
                    help="run one eager tick inside cudaProfilerStart/Stop (for ncu "
                         "--profile-from-start off) and exit")
    return ap.parse_args()


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def population(name: str, world: int) -> list[int]:
    """Prefix patches of every request on the box (64 per GPU).

    cfg2 / cfg3 (the default, also what the driver's 1/2/4/8-GPU runs use):
    ``world`` copies of config 2's seeded 64-request draw, so the per-GPU work
    is config 2's at every N (weak scaling).  cfg4: BASELINE config 4's mix (75%
    U{0..60}, 25% U{200..320} patches) drawn once for the whole 8-GPU box (512
    requests, seed 4); N GPUs serve its first 64*N."""
    from nanovllm_dots_b200 import synthetic as syn
    cfg = syn.BASE
    if name in ("cfg1", "cfg2", "cfg3"):
        base = syn.config_batch("cfg1" if name == "cfg1" else "cfg2")
        return [p // cfg.stride for p in base.prefix_rows] * world
    if name == "cfg4":
        g = torch.Generator().manual_seed(4)
        long_ = torch.rand(512, generator=g) < 0.25
        short_p = torch.randint(0, 61, (512,), generator=g)
        long_p = torch.randint(200, 321, (512,), generator=g)
        pp = torch.where(long_, long_p, short_p).tolist()
        if world > 8:
            raise ValueError("cfg4 is an 8-GPU box workload")
        return pp[: 64 * world]
    raise ValueError(name)


def placement(pp: list[int], world: int):
    """Place the box's requests on ranks with ``LeastLoadedSharder`` (each
    request for its life on the rank with the fewest K/V rows to stream,
    longest request first, at most the per-GPU request count per rank).
    Returns (per-rank prefix-patch lists, per-rank loads in rows)."""
    from nanovllm_dots_b200 import synthetic as syn
    from nanovllm_dots_b200.sharding import LeastLoadedSharder
    cfg = syn.BASE
    per = len(pp) // world
    sh = LeastLoadedSharder(world, stride=cfg.stride, max_per_rank=per)
    for rid in sorted(range(len(pp)), key=lambda i: (-pp[i], i)):
        sh.assign(rid, cfg.stride * pp[rid])
    shards = [[pp[r] for r in sorted(ids)] for ids in sh.by_rank(range(len(pp)))]
    return shards, list(sh.load)


def workload_batch(name: str, rank: int, world: int = 1):
    """(this rank's RequestBatch, placement summary)."""
    from nanovllm_dots_b200 import synthetic as syn
    if name in ("gemm64", "gemm64fp8"):
        return syn.make_batch(64, [0] * 64, seed=2), None
    if name == "prof":
        full = syn.config_batch("cfg2")
        return syn.make_batch(16, [p // 17 for p in full.prefix_rows[:16]], seed=2), None
    if world == 1 and name in ("cfg1", "cfg2", "cfg3"):
        return syn.config_batch("cfg1" if name == "cfg1" else "cfg2"), None
    shards, loads = placement(population(name, world), world)
    mine = shards[rank]
    seed = {"cfg1": 1, "cfg4": 4}.get(name, 2)
    b = syn.make_batch(len(mine), mine, seed=seed if rank == 0 else 1000 * seed + rank)
    summary = {"requests_total": sum(len(x) for x in shards), "rows_per_rank": loads,
               "load_max_over_mean": round(max(loads) / (sum(loads) / len(loads)), 4),
               "placement": "LeastLoadedSharder (K/V rows), longest request first"}
    return b, summary


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.out = self.proc.communicate(timeout=5)[0]
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out = ""

    def summary(self):
        if not self.proc or not getattr(self, "out", ""):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 6:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for nm, v in zip(names, parts[2:6]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------- #
# CPU baseline (the oracle restatement of the reference cache path)            #
# --------------------------------------------------------------------------- #
def cpu_tick_seconds(weights, batch, idx):
    from nanovllm_dots_b200 import synthetic as syn
    from oracle import dit_oracle as O
    cfg = syn.BASE
    kvs = {}
    for i in idx:
        g = torch.Generator().manual_seed(99 + i)
        P = batch.prefix_rows[i]
        kvs[i] = torch.randn(cfg.nfe, cfg.layers, 2, P, cfg.heads, cfg.head_dim, generator=g) * 0.5
    t0 = time.perf_counter()
    O.tick_batch(weights, batch, kv_fn=lambda i: kvs[i], indices=idx)
    return time.perf_counter() - t0


def cpu_full_path_seconds(weights, batch, idx):
    """The reference's shipping MeanFlow path on the host: per request, 4 DiT
    forwards over the whole padded-free history plus the latent slot with the
    FM mask (``_pack_fm_inputs`` + ``batched_meanflow``, ``engine.py:635-709``,
    ``batched_fm.py:82-126``; O(P^2) attention, every history row recomputed
    at every step).  History rows are N(0,1) rows of the cached length."""
    from nanovllm_dots_b200 import synthetic as syn
    from oracle import dit_oracle as O
    cfg = syn.BASE
    ts, dts = syn.time_grid(cfg.nfe)
    hists = {}
    for i in idx:
        g = torch.Generator().manual_seed(55 + i)
        hists[i] = torch.randn(batch.prefix_rows[i] + cfg.stride + 1, cfg.hidden, generator=g)
    t0 = time.perf_counter()
    with torch.no_grad():
        for i in idx:
            x = hists[i]
            z = batch.noise[i].float()
            for k in range(cfg.nfe):
                inp = torch.cat([x, O.linear(z, weights, "coordinate_proj")], dim=0)
                v = O.dit_forward_full(weights, cfg, inp, ts[k], dts[k], fm_seq_len=x.shape[0])
                z = z + v[x.shape[0]:] * dts[k]
    return time.perf_counter() - t0


def cpu_baseline(weights, batch, n_sample):
    idx = list(range(min(n_sample, batch.n)))
    secs = cpu_tick_seconds(weights, batch, idx)
    mean_p = sum(batch.prefix_rows[i] for i in idx) / len(idx)
    # the O(P^2) full path on two requests near the median length
    order = sorted(range(batch.n), key=lambda i: batch.prefix_rows[i])
    fidx = [order[batch.n // 2 - 1], order[batch.n // 2]]
    fsecs = cpu_full_path_seconds(weights, batch, fidx)
    return {"value": round(len(idx) * AUDIO_S_PER_PATCH / secs, 4), "unit": "audio-s/s",
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{len(idx)} request-ticks of the same workload (mean prefix {mean_p:.0f} "
                      f"rows) through the reference's cache path (extend + active rows), "
                      f"fp32 eager torch on the host, {secs:.1f} s",
            "full_path": {"value": round(len(fidx) * AUDIO_S_PER_PATCH / fsecs, 4),
                          "unit": "audio-s/s",
                          "sample": f"{len(fidx)} request-ticks (prefixes "
                                    f"{[batch.prefix_rows[i] for i in fidx]} rows) through the "
                                    f"reference's shipping full O(P^2) MeanFlow path, fp32 eager, "
                                    f"{fsecs:.1f} s"}}


def run_reference(args, rank):
    if rank != 0:
        return
    from nanovllm_dots_b200 import synthetic as syn
    torch.set_num_threads(os.cpu_count() or 1)
    w = syn.make_weights(syn.BASE)
    b, _ = workload_batch(args.workload, 0)
    per_step = 2
    times = []
    for s in range(args.warmup + args.steps):
        idx = [(s * per_step + j) % b.n for j in range(per_step)]
        t = cpu_tick_seconds(w, b, idx)
        if s >= args.warmup:
            times.append(t)
    tot = sum(times)
    val = args.steps * per_step * AUDIO_S_PER_PATCH / tot
    line = {"metric": METRIC, "value": round(val, 4), "unit": "audio-s/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1000 * tot / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": args.workload, "requests_per_step": per_step,
                       "note": "host-CPU run of the reference algorithm (cache path), bounded "
                               "sample of the workload's requests per step"},
            "cpu_baseline": {"value": round(val, 4), "unit": "audio-s/s",
                             "cores": torch.get_num_threads(), "kind": "port",
                             "sample": f"{per_step} request-ticks per step"},
            "e2e": {"value": round(val, 4), "unit": "audio-s/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- #
# GPU arm                                                                      #
# --------------------------------------------------------------------------- #
def launches_per_tick(cfg, raw_ext=True):
    # per step: coordinate_proj, input_layer, 7 per block (LayerNorm, QKV, attention,
    # O-projection, LayerNorm, fc1, fc2), the final LayerNorm and GEMM
    per_step = 2 + cfg.layers * 7 + 2
    return 3 + 1 + 1 + (2 if raw_ext else 0) + cfg.nfe * per_step


def run_b200(args, rank, world):
    from nanovllm_dots_b200 import _lib
    from nanovllm_dots_b200 import synthetic as syn
    from nanovllm_dots_b200.fm_head import B200FMHead, FMRequest

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    cfg = syn.BASE
    b, place = workload_batch(args.workload, rank, world)
    n = b.n
    max_pages = max(math.ceil((p + 2 * cfg.stride) / cfg.page_rows) for p in b.prefix_rows)
    num_pages = sum(math.ceil((p + 2 * cfg.stride) / cfg.page_rows) for p in b.prefix_rows) + 8
    weights = syn.make_weights(cfg)
    precision = "fp8" if args.workload in ("cfg3", "gemm64fp8") else "bf16"
    head = B200FMHead(weights, cfg, num_pages=num_pages, max_pages_per_req=max_pages,
                      max_requests=n, device=dev, precision=precision)
    # cached prefixes: N(0, 0.5^2) K/V drawn on the device straight into the pool
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    chunk = 1 << 28
    flat = head.pool
    for s in range(0, flat.numel(), chunk):
        e = min(flat.numel(), s + chunk)
        flat[s:e] = (torch.randn(e - s, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    rids = list(range(n))
    for i in rids:
        head.pages.ensure(i, b.prefix_rows[i])
        head.requests[i] = FMRequest(i, b.prefix_rows[i])
    cl, ne, bt = head.prepare(rids, [cfg.stride] * n)
    d = lambda t: t.to(dev).contiguous()
    noise, cond, ph, pl = d(b.noise), d(b.cond), d(b.prev_hidden), d(b.prev_latent)
    out = torch.empty(n, cfg.latent_patch, cfg.latent_dim, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)

    def eager_tick():
        head.launch(noise=noise, act_hidden=cond, ext_hidden=ph, ext_latent=pl, cache_len=cl,
                    n_extend=ne, block_table=bt, out=out)

    for _ in range(2):
        eager_tick()
    torch.cuda.synchronize()
    head.check_errors()
    if args.profile_tick:
        torch.cuda.cudart().cudaProfilerStart()
        eager_tick()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        head.check_errors()
        if rank == 0:
            print(json.dumps({"profile_tick": True, "workload": args.workload, "requests": n,
                              "launches": launches_per_tick(cfg)}), flush=True)
        head.close()
        return
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(3):
        eager_tick()
    ev1.record(stream)
    ev1.synchronize()
    eager_ms = ev0.elapsed_time(ev1) / 3

    # the tick as one CUDA graph over static buffers (the serving configuration)
    tg = head.graph(n, raw_inputs=True)
    for k, v in (("noise", noise), ("act_hidden", cond), ("ext_hidden", ph), ("ext_latent", pl),
                 ("cache_len", cl), ("n_extend", ne), ("block_table", bt)):
        tg.inputs[k].copy_(v)
    torch.cuda.synchronize()

    def tick():
        tg.replay()

    for _ in range(args.warmup):
        tick()
    torch.cuda.synchronize()
    head.check_errors()

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def all_ranks(x):
        if world == 1:
            return [round(x, 4)]
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        parts = [torch.empty_like(t) for _ in range(world)]
        torch.distributed.all_gather(parts, t)
        return [round(float(p.item()), 4) for p in parts]

    # ---- device-resident timing
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            tick()
        e1.record(stream)
        e1.synchronize()
    barrier()
    my_ms = e0.elapsed_time(e1) / args.steps
    ms = max_over_ranks(my_ms)
    per_rank_ms = all_ranks(my_ms)
    head.check_errors()

    # ---- end to end through the C ABI with host buffers (pinned), per-tick copies
    pin = lambda t: t.contiguous().pin_memory()
    h_noise, h_cond, h_ph, h_pl = pin(b.noise), pin(b.cond), pin(b.prev_hidden), pin(b.prev_latent)
    h_cl, h_ne, h_bt = pin(cl.cpu()), pin(ne.cpu()), pin(bt.cpu())
    h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    h2d = sum(x.numel() * x.element_size() for x in (h_noise, h_cond, h_ph, h_pl, h_cl, h_ne, h_bt))
    d2h = h_out.numel() * h_out.element_size()
    pairs = [(tg.inputs[k], v) for k, v in (("noise", h_noise), ("act_hidden", h_cond),
                                             ("ext_hidden", h_ph), ("ext_latent", h_pl),
                                             ("cache_len", h_cl), ("n_extend", h_ne),
                                             ("block_table", h_bt))]

    def e2e_tick():
        for dst, src in pairs:
            dst.copy_(src, non_blocking=True)
        tg.replay()
        h_out.copy_(tg.out, non_blocking=True)
        stream.synchronize()

    for _ in range(2):
        e2e_tick()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        e2e_tick()
    f1.record(stream)
    f1.synchronize()
    barrier()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1) / args.steps)

    # ---- the tick's own kernels, one at a time (dfm_tick_launch: same kernel,
    # tiles, epilogue and workspace as inside the tick), layers cycled so the
    # weights stream from HBM as they do in the tick
    hbm, tflops, peak_kind = load_peaks()
    R = 2 * cfg.stride * n
    H, F_ = cfg.hidden, cfg.ffn
    tensors = dict(noise=noise, act_hidden=cond, ext_hidden=ph, ext_latent=pl, cache_len=cl,
                   n_extend=ne, block_table=bt, out=out)
    eager_tick()                                 # workspace state of a full tick
    torch.cuda.synchronize()
    keys = sum(p + 2 * cfg.stride for p in b.prefix_rows)
    ln_bytes = R * H * (4 + 2 * 4 + 4 + 2) + n * 3 * H * 4
    kinds = {
        "ln_attn": {"bytes": ln_bytes, "bound": "hbm"},
        "qkv": {"flops": 2.0 * R * 3 * H * H, "bound": "tensor"},
        "attention": {"bytes": keys * cfg.heads * cfg.head_dim * 2 * 2 + 2 * R * H * 2,
                      "bound": "hbm"},
        "o_proj": {"flops": 2.0 * R * H * H, "bound": "tensor"},
        "ln_mlp": {"bytes": ln_bytes, "bound": "hbm"},
        "fc1": {"flops": 2.0 * R * F_ * H, "bound": "tensor"},
        "fc2": {"flops": 2.0 * R * H * F_, "bound": "tensor"},
    }
    reps = 4
    for nm, k in kinds.items():
        def run(nm=nm):
            for l in range(cfg.layers):
                head.launch_kernel(nm, 0, l, stream=stream, **tensors)
        run()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(reps):
            run()
        s1.record(stream)
        s1.synchronize()
        k["us"] = s0.elapsed_time(s1) * 1000 / (reps * cfg.layers)
    head.check_errors()
    eager_tick()                                 # leave the workspace as a tick leaves it
    torch.cuda.synchronize()
    per_tick = cfg.layers * cfg.nfe
    summary = {}
    for nm, k in kinds.items():
        if k["bound"] == "hbm":
            ach, peak, unit = k["bytes"] / (k["us"] * 1e-6) / 1e9, hbm, "GB/s"
        else:
            ach, peak, unit = k["flops"] / (k["us"] * 1e-6) / 1e12, tflops, "TFLOP/s"
        summary[nm] = {"us": round(k["us"], 2), "achieved": round(ach, 1), "unit": unit,
                       "frac": round(ach / peak, 4),
                       "tick_share_est": round(k["us"] * per_tick / (ms * 1000), 4)}
    gemm_us = sum(kinds[g]["us"] for g in ("qkv", "o_proj", "fc1", "fc2"))
    gemm_fl = sum(kinds[g]["flops"] for g in ("qkv", "o_proj", "fc1", "fc2"))
    summary["per_layer_gemms"] = {"us": round(gemm_us, 2),
                                  "achieved": round(gemm_fl / (gemm_us * 1e-6) / 1e12, 1),
                                  "unit": "TFLOP/s",
                                  "frac": round(gemm_fl / (gemm_us * 1e-6) / 1e12 / tflops, 4),
                                  "note": "QKV + O-proj + fc1 + fc2, FLOP-weighted"}
    summary["sum_of_shares"] = round(sum(v["tick_share_est"] for kk, v in summary.items()
                                         if kk in kinds), 4)
    dom = max(kinds, key=lambda x: summary[x]["tick_share_est"])
    traffic = None
    tp = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            traffic = json.load(f).get(dom)
    dk = kinds[dom]
    roof = {"kernel": dom, "bound": dk["bound"], "achieved": summary[dom]["achieved"],
            "peak": hbm if dk["bound"] == "hbm" else tflops, "unit": summary[dom]["unit"],
            "frac": summary[dom]["frac"], "traffic": traffic,
            "algorithmic_per_launch": dk.get("bytes", dk.get("flops")),
            "peak_source": f"{peak_kind} ({'hbm_gbs' if dk['bound'] == 'hbm' else 'bf16_tflops'})",
            "timing": "the tick's own launch (dfm_tick_launch), CUDA events, 12 layers x "
                      f"{reps} on the tick's stream"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(weights, b, args.cpu_sample)

    total_req = n * world
    value = total_req * AUDIO_S_PER_PATCH / (ms / 1000)
    e2e_val = total_req * AUDIO_S_PER_PATCH / (e2e_ms / 1000)
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": "audio-s/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16" if args.workload != "cfg3" else "fp8-e4m3 (QKV, fc1) + bf16",
                "data": "synthetic (seeded random-init DiT, N(0,1) inputs, N(0,0.5^2) cached K/V)",
                "config": {"workload": args.workload, "requests_per_gpu": n,
                           "mean_prefix_rows": round(sum(b.prefix_rows) / n, 1),
                           "nfe": cfg.nfe, "layers": cfg.layers, "page_rows": cfg.page_rows,
                           "l2": "inputs larger than L2 (K/V pool and weights), no flush",
                           "parallelism": f"request-sharded x{world}",
                           "precision": precision,
                           "per_rank_ms": per_rank_ms,
                           "rank_ms_max_over_mean": round(max(per_rank_ms)
                                                          / (sum(per_rank_ms) / world), 4),
                           **({"placement": place} if place else {})},
                "e2e": {"value": round(e2e_val, 2), "unit": "audio-s/s",
                        "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                        "ms_per_step": round(e2e_ms, 4)},
                "eager_ms_per_step": round(eager_ms, 4),
                "gpu_launches": launches_per_tick(cfg) * args.steps,
                "roofline": roof, "kernels": summary, "clocks": clk.summary(),
                "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)
    head.close()


# --------------------------------------------------------------------------- #
# Patch encoder (``--workload pe``)                                            #
# --------------------------------------------------------------------------- #
PE_METRIC = "patch-encoder xRT (audio-s/s) at conc 64 per GPU"


def pe_histories(rank: int) -> list[int]:
    """History patches per request: cfg2's draw (U{0..120} patches, the same
    count the FM head's prefix holds), an independent draw per rank."""
    g = torch.Generator().manual_seed(2 if rank == 0 else 1000 + rank)
    return torch.randint(0, 121, (64,), generator=g).tolist()


def pe_cpu_seconds(w, cfg, hist, idx, patches):
    from oracle import pe_oracle as PO
    states = []
    for i in idx:
        st = PO.PEState(cfg)
        g = torch.Generator().manual_seed(77 + i)
        S = hist[i] * cfg.rows
        for l in range(cfg.layers):
            st.k[l] = torch.randn(S, cfg.heads, cfg.head_dim, generator=g) * 0.5
            st.v[l] = torch.randn(S, cfg.heads, cfg.head_dim, generator=g) * 0.5
        states.append(st)
    t0 = time.perf_counter()
    for j, i in enumerate(idx):
        PO.decode_patch(w, cfg, states[j], patches[i])
    return time.perf_counter() - t0


def run_pe(args, rank, world):
    from nanovllm_dots_b200 import synthetic as syn
    from nanovllm_dots_b200.patch_encoder import B200PatchEncoder

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    cfg = syn.PE_BASE
    hist = pe_histories(rank)
    n = len(hist)
    w = syn.make_pe_weights(cfg)
    pe = B200PatchEncoder(w, cfg, max_batch=n, max_seq_len=256 * cfg.rows, device=dev)
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    chunk = 1 << 28
    for s0 in range(0, pe.pool.numel(), chunk):
        e = min(pe.pool.numel(), s0 + chunk)
        pe.pool[s0:e] = (torch.randn(e - s0, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    seq0 = torch.tensor([h * cfg.rows for h in hist], dtype=torch.int32, device=dev)
    patches = syn.make_pe_patches(n, 1, seed=5 + rank)[0]
    stream = torch.cuda.current_stream(dev)
    if args.profile_tick:
        rows = torch.arange(n, dtype=torch.int32, device=dev)
        out = torch.empty(n, cfg.out_dim, dtype=torch.bfloat16, device=dev)
        p_dev = patches.to(dev).contiguous()
        for prof in (False, True):
            pe.seqlens.copy_(seq0)
            if prof:
                torch.cuda.cudart().cudaProfilerStart()
            pe.launch(p_dev, rows, out)
            torch.cuda.synchronize()
            if prof:
                torch.cuda.cudart().cudaProfilerStop()
        pe.check_errors()
        if rank == 0:
            print(json.dumps({"profile_tick": True, "workload": "pe", "requests": n,
                              "launches": 6 + 7 * cfg.layers}), flush=True)
        pe.close()
        return
    dg = pe.graph(n)
    dg.inputs["patches"].copy_(patches.to(dev))
    pe.seqlens.copy_(seq0)

    def step():
        pe.seqlens.copy_(seq0)      # every step decodes at the same history lengths
        dg.replay()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    pe.check_errors()

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        e1.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    pe.check_errors()

    # end to end: pinned host patches and rows in, embeddings out, every step
    h_patches = patches.contiguous().pin_memory()
    h_rows = torch.arange(n, dtype=torch.int32).pin_memory()
    h_out = torch.empty(n, cfg.out_dim, dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        dg.inputs["patches"].copy_(h_patches, non_blocking=True)
        dg.inputs["rows"].copy_(h_rows, non_blocking=True)
        step()
        h_out.copy_(dg.out, non_blocking=True)
        stream.synchronize()

    for _ in range(2):
        e2e_step()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    f1.record(stream)
    f1.synchronize()
    barrier()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1) / args.steps)
    pe.check_errors()

    hbm, tflops, peak_kind = load_peaks()
    H, F_, Lyr = cfg.hidden, cfg.ffn, cfg.layers
    kv_bytes = sum((h * cfg.rows + cfg.rows) for h in hist) * Lyr * 2 * H * 2
    w_bytes = 2 * (Lyr * (4 * H * H + 2 * H * F_) + cfg.out_dim * cfg.rows * H
                   + H * cfg.latent_dim + 2 * cfg.latent_dim * cfg.latent_dim)
    flops = 2.0 * n * cfg.rows * Lyr * (4 * H * H + 2 * H * F_) + 2.0 * n * cfg.rows * H * cfg.out_dim
    achieved = (kv_bytes + w_bytes) / (ms * 1e-3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        idx = list(range(min(8, n)))
        secs = pe_cpu_seconds(w, cfg, hist, idx, patches)
        cpu = {"value": round(len(idx) * AUDIO_S_PER_PATCH / secs, 4), "unit": "audio-s/s",
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{len(idx)} request decode_patch calls of the same workload, fp32 "
                         f"eager torch on the host, {secs:.2f} s"}
    value = n * world * AUDIO_S_PER_PATCH / (ms / 1000)
    if rank == 0:
        line = {"metric": PE_METRIC, "value": round(value, 2), "unit": "audio-s/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded random-init encoder, N(0,1) patches, N(0,0.5^2) cached K/V)",
                "config": {"workload": "pe", "requests_per_gpu": n,
                           "mean_history_positions": round(sum(hist) * cfg.rows / n, 1),
                           "layers": Lyr, "capacity_positions": pe.cap,
                           "l2": "K/V read per step (~0.8 GB) larger than L2, no flush",
                           "parallelism": f"request-sharded x{world}"},
                "e2e": {"value": round(n * world * AUDIO_S_PER_PATCH / (e2e_ms / 1000), 2),
                        "unit": "audio-s/s",
                        "h2d_bytes_per_step": h_patches.numel() * 2 + h_rows.numel() * 4,
                        "d2h_bytes_per_step": h_out.numel() * 2, "ms_per_step": round(e2e_ms, 4)},
                "gpu_launches": (6 + 7 * Lyr) * args.steps,
                "roofline": {"kernel": "whole decode call (K/V + weights streamed once)",
                             "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                             "unit": "GB/s", "frac": round(achieved / hbm, 4), "traffic": None,
                             "algorithmic_per_launch": kv_bytes + w_bytes,
                             "gemm_tflops": round(flops / (ms * 1e-3) / 1e12, 1),
                             "peak_source": f"{peak_kind} (hbm_gbs)"},
                "clocks": clk.summary(), "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)
    pe.close()


# --------------------------------------------------------------------------- #
# LLM decode attention (``--workload llmattn``)                                #
# --------------------------------------------------------------------------- #
LLM_METRIC = "LLM paged decode attention: layer-steps/s (64 sequences)"


def run_llmattn(args, rank, world):
    from nanovllm_dots_b200.llm_attention import B200DecodeAttention

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    H, KVH, D, bs = 12, 2, 128, 256
    g = torch.Generator().manual_seed(11 + rank)
    n = 64
    # contexts: text prompt (~U{100..300} tokens) + one token per generated patch
    # (cfg2's U{0..120} history patches)
    ctx = (torch.randint(100, 301, (n,), generator=g) + torch.randint(0, 121, (n,), generator=g)
           + 1).tolist()
    nblk = [(c + bs - 1) // bs for c in ctx]
    width = max(nblk)
    num_blocks = sum(nblk)
    table = torch.full((n, width), -1, dtype=torch.int32)
    perm = torch.randperm(num_blocks, generator=g)
    o = 0
    for i, b in enumerate(nblk):
        table[i, :b] = perm[o:o + b].to(torch.int32)
        o += b
    kc = (torch.randn(num_blocks, bs, KVH, D, device=dev) * 0.5).to(torch.bfloat16)
    vc = (torch.randn(num_blocks, bs, KVH, D, device=dev) * 0.5).to(torch.bfloat16)
    q = torch.randn(n, H, D, device=dev).to(torch.bfloat16)
    k = torch.randn(n, KVH, D, device=dev).to(torch.bfloat16)
    v = torch.randn(n, KVH, D, device=dev).to(torch.bfloat16)
    slot = torch.tensor([int(table[i, (c - 1) // bs]) * bs + (c - 1) % bs for i, c in enumerate(ctx)],
                        dtype=torch.int32, device=dev)
    cl = torch.tensor(ctx, dtype=torch.int32, device=dev)
    td = table.to(dev)
    dec = B200DecodeAttention(H, D, D ** -0.5, KVH, max_batch=n, max_blocks=width, device=dev)
    out = torch.empty(n, H, D, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)
    # the per-layer caches of a 28-layer backbone do not fit in L2; cycle over
    # enough copies of the pool that every call reads from HBM
    copies = max(2, math.ceil(4 * 126e6 / (kc.numel() * 4)))
    pools = [(kc, vc)] + [(kc.clone(), vc.clone()) for _ in range(copies - 1)]

    # one CUDA graph holds a decode call per cache copy (the layers of a decode
    # step, as the reference's graph-captured decode replays them); a step is
    # one layer's call, timed as graph time / calls
    for j in range(copies):
        a, b = pools[j]
        dec.decode(q, k, v, a, b, slot, cl, td, out=out)
    torch.cuda.synchronize()
    dec.check_errors()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for j in range(copies):
            a, b = pools[j]
            dec.decode(q, k, v, a, b, slot, cl, td, out=out, stream=torch.cuda.current_stream(dev))
    reps = max(1, args.steps // copies)
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        e1.synchronize()
    ms = e0.elapsed_time(e1) / (reps * copies)
    dec.check_errors()
    # the same calls issued eagerly from Python, for the host-side cost
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for j in range(reps * copies):
        a, b = pools[j % copies]
        dec.decode(q, k, v, a, b, slot, cl, td, out=out)
    f1.record(stream)
    f1.synchronize()
    eager_ms = f0.elapsed_time(f1) / (reps * copies)
    hbm, _, peak_kind = load_peaks()
    kv_bytes = sum(ctx) * KVH * D * 2 * 2
    achieved = kv_bytes / (ms * 1e-3) / 1e9
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import llm_attn_oracle as LO
        idx = list(range(8))
        kcc, vcc = kc.cpu(), vc.cpu()
        t0 = time.perf_counter()
        LO.decode_attention(q[idx].cpu(), kcc, vcc, cl[idx].cpu(), table[idx].tolist(), D ** -0.5)
        secs = time.perf_counter() - t0
        cpu = {"value": round(len(idx) / n / secs, 3), "unit": "layer-steps/s",
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{len(idx)} of the {n} sequences, fp32 eager torch, {secs:.3f} s"}
    if rank == 0:
        line = {"metric": LLM_METRIC, "value": round(1000.0 / ms, 1), "unit": "layer-steps/s",
                "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(ms, 5), "eager_ms_per_step": round(eager_ms, 5),
                "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic (N(0,1) q, N(0,0.5^2) cache)",
                "config": {"workload": "llmattn", "sequences": n, "heads": H, "kv_heads": KVH,
                           "head_dim": D, "block_size": bs,
                           "mean_context": round(sum(ctx) / n, 1),
                           "l2": f"{copies} cache copies cycled (each call reads from HBM)",
                           "timing": f"CUDA graph of {copies} calls replayed {reps} times"},
                "gpu_launches": 3 * reps * copies,
                "roofline": {"kernel": "llm_decode_attn_kernel + store + combine", "bound": "hbm",
                             "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                             "frac": round(achieved / hbm, 4), "traffic": None,
                             "algorithmic_per_launch": kv_bytes,
                             "peak_source": f"{peak_kind} (hbm_gbs)"},
                "clocks": clk.summary(), "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- #
# LLM backbone decode step (``--workload llmdecode``)                          #
# --------------------------------------------------------------------------- #
LLMDEC_METRIC = "LLM backbone decode tokens/s (64 sequences, 28 layers)"


def llm_contexts(rank: int, n: int = 64) -> list[int]:
    """Prompt tokens U{100..300} + one token per generated patch (cfg2's
    U{0..120} history), + the step's own token."""
    g = torch.Generator().manual_seed(11 + rank)
    return (torch.randint(100, 301, (n,), generator=g) + torch.randint(0, 121, (n,), generator=g)
            + 1).tolist()


def run_llmdecode(args, rank, world):
    from nanovllm_dots_b200 import synthetic as syn
    from nanovllm_dots_b200.llm_decode import B200QwenDecoder

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    cfg = syn.LLM_BASE
    ctx = llm_contexts(rank)
    n, bs = len(ctx), cfg.block_size
    nblk = [(c + bs - 1) // bs for c in ctx]
    width, num_blocks = max(nblk), sum(nblk)
    g = torch.Generator().manual_seed(5 + rank)
    perm = torch.randperm(num_blocks, generator=g)
    table = torch.full((n, width), -1, dtype=torch.int32)
    o = 0
    for i, b in enumerate(nblk):
        table[i, :b] = perm[o:o + b].to(torch.int32)
        o += b
    w = syn.make_llm_weights(cfg, device=dev)          # drawn on the device: 1.3 B parameters
    dec = B200QwenDecoder(w, cfg, max_batch=n, max_blocks=width, device=dev)
    del w
    torch.cuda.empty_cache()
    kc, vc = dec.alloc_caches(num_blocks)
    gd = torch.Generator(device=dev).manual_seed(7)
    for t in kc + vc:
        t.copy_((torch.randn(t.shape, device=dev, generator=gd) * 0.5).to(torch.bfloat16))
    emb = torch.randn(n, cfg.hidden, device=dev, generator=gd).to(torch.bfloat16)
    pos = torch.tensor([c - 1 for c in ctx], dtype=torch.int32, device=dev)
    slot = torch.tensor([int(table[i, (c - 1) // bs]) * bs + (c - 1) % bs for i, c in enumerate(ctx)],
                        dtype=torch.int32, device=dev)
    cl = torch.tensor(ctx, dtype=torch.int32, device=dev)
    td = table.to(dev)
    out = torch.empty(n, cfg.hidden, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)
    dec.step(emb, pos, slot, cl, td, kc, vc, out=out)     # plans the workspace and cache maps
    torch.cuda.synchronize()
    dec.check_errors()
    if args.profile_tick:
        torch.cuda.cudart().cudaProfilerStart()
        dec.step(emb, pos, slot, cl, td, kc, vc, out=out)
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        dec.check_errors()
        if rank == 0:
            print(json.dumps({"profile_tick": True, "workload": "llmdecode", "sequences": n,
                              "launches": 1 + 11 * cfg.layers}), flush=True)
        dec.close()
        return
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        dec.step(emb, pos, slot, cl, td, kc, vc, out=out, stream=torch.cuda.current_stream(dev))
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
        e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    dec.check_errors()
    # end to end: pinned-host embeddings in, hidden states out, every step
    h_emb = emb.cpu().pin_memory()
    h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        emb.copy_(h_emb, non_blocking=True)
        graph.replay()
        h_out.copy_(out, non_blocking=True)
        stream.synchronize()
    f1.record(stream)
    f1.synchronize()
    e2e_ms = f0.elapsed_time(f1) / args.steps
    hbm, tflops, peak_kind = load_peaks()
    per_layer_w = (cfg.qkv_width * cfg.hidden + cfg.hidden * cfg.heads * cfg.head_dim
                   + 3 * cfg.inter * cfg.hidden) * 2
    kv_bytes = sum(ctx) * cfg.kv_heads * cfg.head_dim * 2 * 2 * cfg.layers
    bytes_step = per_layer_w * cfg.layers + kv_bytes
    achieved = bytes_step / (ms * 1e-3) / 1e9
    if rank == 0:
        line = {"metric": LLMDEC_METRIC, "value": round(n * 1000.0 / ms, 1), "unit": "tokens/s",
                "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded Qwen2-shaped weights, N(0,1) embeddings, N(0,0.5^2) caches)",
                "config": {"workload": "llmdecode", "sequences": n, "layers": cfg.layers,
                           "hidden": cfg.hidden, "heads": cfg.heads, "kv_heads": cfg.kv_heads,
                           "inter": cfg.inter, "mean_context": round(sum(ctx) / n, 1),
                           "l2": "weights (2.6 GB) and caches larger than L2, no flush",
                           "timing": "CUDA graph of one decode step"},
                "e2e": {"value": round(n * 1000.0 / e2e_ms, 1), "unit": "tokens/s",
                        "h2d_bytes_per_step": h_emb.numel() * 2, "d2h_bytes_per_step": h_out.numel() * 2,
                        "ms_per_step": round(e2e_ms, 4)},
                "gpu_launches": (1 + 9 * cfg.layers) * args.steps,
                "roofline": {"kernel": "whole decode step (weights + K/V streamed once)",
                             "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                             "unit": "GB/s", "frac": round(achieved / hbm, 4), "traffic": None,
                             "algorithmic_per_launch": bytes_step,
                             "peak_source": f"{peak_kind} (hbm_gbs)"},
                "clocks": clk.summary(), "cpu_baseline": None}
        print(json.dumps(line), flush=True)
    dec.close()


# --------------------------------------------------------------------------- #
# Engine drop-in (``--workload engine``)                                       #
# --------------------------------------------------------------------------- #
ENGINE_METRIC = "FM engine-tick xRT through the fm_accel='b200' dispatch (conc 64 per GPU)"


class _EnginePayload:
    """The fields of the reference's DotsSeqState the FM dispatch reads
    (``engine.py:48-77``): gen_state.fm_sequence [1, cap, H] bf16 on the GPU,
    fm_seq_len, g_cond, num_steps."""

    def __init__(self, rows, cap, dev, nfe):
        buf = torch.zeros(1, cap, rows.shape[1], dtype=torch.bfloat16, device=dev)
        buf[0, :rows.shape[0]] = rows.to(dev)
        from types import SimpleNamespace
        self.gen_state = SimpleNamespace(fm_sequence=buf, fm_seq_len=rows.shape[0],
                                         fm_null_g_cond=None)
        self.g_cond = None
        self.num_steps = nfe


def run_engine(args, rank, world):
    from nanovllm_dots_b200 import synthetic as syn
    from nanovllm_dots_b200.engine_mode import B200FMDispatch
    from nanovllm_dots_b200.fm_head import B200FMHead

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    cfg = syn.BASE
    b, _ = workload_batch("cfg2", rank, world)
    n = b.n
    ticks = max(args.warmup, 3) + args.steps + 1
    hist = [p + cfg.hidden_patch for p in b.prefix_rows]     # history rows before the first tick
    cap = [h + cfg.stride * (ticks + 2) for h in hist]
    max_pages = max(math.ceil((c + 2 * cfg.stride) / cfg.page_rows) for c in cap)
    num_pages = sum(math.ceil((c + 2 * cfg.stride) / cfg.page_rows) for c in cap) + 8
    head = B200FMHead(syn.make_weights(cfg), cfg, num_pages=num_pages, max_pages_per_req=max_pages,
                      max_requests=n, device=dev)
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    rows = lambda m: (torch.randn(m, cfg.hidden, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    pay = [_EnginePayload(rows(cap[i]), cap[i], dev, cfg.nfe) for i in range(n)]
    for i, p in enumerate(pay):
        p.gen_state.fm_seq_len = hist[i]
    dispatch = B200FMDispatch(head)
    dispatch(pay)                      # first tick: bulk prefill of every history backlog
    torch.cuda.synchronize()

    def advance():
        # the engine's own per-tick appends (a patch and the next hidden row):
        # the rows are already in each buffer, so only the length moves
        for p in pay:
            p.gen_state.fm_seq_len += cfg.stride

    # host time of the dispatch's parts (wall clock, no synchronisation inside)
    parts = {"plan": 0.0, "pack": 0.0, "prepare": 0.0}

    def timed(name, fn):
        def w(*a, **kw):
            t0 = time.perf_counter()
            try:
                return fn(*a, **kw)
            finally:
                parts[name] += time.perf_counter() - t0
        return w
    dispatch.plan = timed("plan", dispatch.plan)
    dispatch.pack = timed("pack", dispatch.pack)
    head.prepare = timed("prepare", head.prepare)
    times_d, times_s, times_g = [], [], []
    for t in range(ticks - 1):
        advance()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        dispatch(pay)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        if t < max(args.warmup, 3) - 1:
            parts = dict.fromkeys(parts, 0.0)
            continue
        times_d.append(t1 - t0)
        # the same tick again (its inputs are still in the graph's buffers; it
        # rewrites the same cache rows): through dfm_step alone (the C ABI,
        # eager launches) and as the bare graph replay
        tg = dispatch._graphs[n]
        t0 = time.perf_counter()
        head.launch(out=tg.out, **tg.inputs)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        tg.replay()
        torch.cuda.synchronize()
        times_s.append(t1 - t0)
        times_g.append(time.perf_counter() - t1)
    head.check_errors()
    md = 1000 * statistics.median(times_d)
    ms_ = 1000 * statistics.median(times_s)
    mg = 1000 * statistics.median(times_g)
    if rank == 0:
        line = {"metric": ENGINE_METRIC, "value": round(n * AUDIO_S_PER_PATCH / (md / 1000), 2),
                "unit": "audio-s/s", "n_gpus": world, "steps": len(times_d),
                "warmup": max(args.warmup, 3), "ms_per_step": round(md, 4),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (engine-style bf16 FM histories of config 2's lengths on the GPU)",
                "config": {"workload": "engine", "requests_per_gpu": n,
                           "mean_history_rows": round(sum(hist) / n, 1),
                           "timing": "host wall clock per tick with a device synchronisation, "
                                     "median; the dispatch replays a captured tick per batch "
                                     "size; dfm_step_ms is the same tick launched eagerly "
                                     "through the C ABI"},
                "dfm_step_ms": round(ms_, 4),
                "graph_replay_ms": round(mg, 4),
                "host_ms_per_tick": {k: round(1000 * v / len(times_d), 4) for k, v in parts.items()},
                "dispatch_overhead_frac": round(md / ms_ - 1.0, 4),
                "dispatch_over_graph_replay_frac": round(md / mg - 1.0, 4)}
        print(json.dumps(line), flush=True)
    head.close()


# --------------------------------------------------------------------------- #
# Vocoder (``--workload voc`` streaming, ``--workload voc1`` one-shot)         #
# --------------------------------------------------------------------------- #
VOC_METRIC = "vocoder xRT (audio-s/s), strict streaming of 16-frame chunks, conc {n} per GPU"
VOC1_METRIC = "vocoder xRT (audio-s/s), one-shot 10 s utterances, conc {n} per GPU"
VOC_CHUNK, VOC_ONESHOT_FRAMES, VOC_FRAME_S = 16, 250, 0.04


def voc_conv_flops(cfg, T: int, n: int) -> list[float]:
    """Algorithmic FLOPs of each decoder convolution (execution order) for n
    requests of T latent frames: 2 x output frames x Cout x Cin x taps, with the
    unpadded channel counts and only the valid frames."""
    out = [2.0 * n * T * cfg.initial_channels * cfg.latent_dim * (2 * cfg.lookahead + 1)]
    t = T
    for i, u in enumerate(cfg.upsample_rates):
        cin, c = cfg.stage_channels(i - 1), cfg.stage_channels(i)
        out.append(2.0 * n * t * u * c * 2 * cin)
        t *= u
        for k, dil in zip(cfg.resblock_kernel_sizes, cfg.resblock_dilations):
            layers = 2 * len(dil) if cfg.resblock == "1" else 2
            out += [2.0 * n * t * c * c * k] * layers
    return out


def run_voc(args, rank, world, oneshot: bool, n: int = 64):
    from nanovllm_dots_b200 import synthetic as syn
    from nanovllm_dots_b200.vocoder import B200Vocoder

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    cfg = syn.VOC_BASE
    w = syn.make_voc_weights(cfg, seed=1)
    W = VOC_CHUNK + cfg.lookahead + _voc_left(cfg)
    F = VOC_ONESHOT_FRAMES if oneshot else VOC_CHUNK
    T = F if oneshot else W
    voc = B200Vocoder(w, cfg, max_batch=n, max_frames=T, device=dev)
    assert oneshot or voc.stream_window_size(VOC_CHUNK) == W
    g = torch.Generator(device=dev).manual_seed(99 + rank)
    Lm, Hm = cfg.latent_dim, 4 * cfg.latent_dim
    lat = torch.randn(n, F, Lm, device=dev, generator=g)
    h = torch.zeros(cfg.mi_layers, n, Hm, device=dev)
    c = torch.zeros_like(h)
    audio = torch.empty(n, T * cfg.hop, device=dev)
    if oneshot:
        b = voc.batch(n, F, 0, audio, latents=lat, h=h, c=c)
    else:
        win = torch.randn(n, W, Lm, device=dev, generator=g)        # steady state: windows full
        valid = torch.full((n,), W, dtype=torch.int32, device=dev)
        b = voc.batch(n, F, W, audio, latents=lat, h=h, c=c, windows=win, valid=valid)
    stream = torch.cuda.current_stream(dev)

    def call():
        if oneshot:
            h.zero_()
            c.zero_()
        voc.launch(b)

    call()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        call()
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    voc.check_errors()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
        e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    eager0, eager1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    eager0.record(stream)
    for _ in range(3):
        call()
    eager1.record(stream)
    eager1.synchronize()
    eager_ms = eager0.elapsed_time(eager1) / 3
    voc.check_errors()

    # each decoder convolution launched alone with the call's arguments
    flops = voc_conv_flops(cfg, F if oneshot else W, n)
    conv_us = []
    reps = 3
    for i in range(voc.num_convs):
        voc.launch(b, conv=i)
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for _ in range(reps):
            voc.launch(b, conv=i)
        c1.record(stream)
        c1.synchronize()
        conv_us.append(c0.elapsed_time(c1) * 1000 / reps)
    voc.check_errors()
    hbm, bf16, peak_kind = load_peaks()
    peaks = {}
    if peak_kind == "measured":
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    f16 = peaks.get("bf16_tflops_sustained", 1400.0)   # kind::f16 runs fp16 at the bf16 rate
    conv_total_us = sum(conv_us)
    top = max(range(len(conv_us)), key=lambda i: conv_us[i] * 1.0)
    heavy = max(range(len(flops)), key=lambda i: flops[i])
    ach = lambda fl, us: fl / (us * 1e-6) / 1e12

    # end to end through the public API: pinned host latents in, emitted audio out
    audio_s = n * F * VOC_FRAME_S
    h_lat = lat.cpu().pin_memory()
    if oneshot:
        def e2e_step():
            outs = voc.decode_batch(h_lat)
            return [o.to("cpu", non_blocking=True) for o in outs]
        d2h = n * F * cfg.hop * 4
    else:
        states = [voc.init_stream_state(1, VOC_CHUNK) for _ in range(n)]
        for st in states:
            st.window.normal_(generator=g)
            st.total, st.emitted = 10 ** 6, 10 ** 6 - cfg.lookahead

        def e2e_step():
            outs = voc.stream_step_many(states, h_lat)
            return [o.to("cpu", non_blocking=True) for o in outs]
        d2h = n * VOC_CHUNK * cfg.hop * 4
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(3, min(args.steps, 10))
    f0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    f1.record(stream)
    f1.synchronize()
    e2e_ms = f0.elapsed_time(f1) / e2e_steps
    voc.check_errors()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import voc_oracle as vo
        orc = vo.VocOracle(w, cfg, dtype=torch.float32)
        t0 = time.perf_counter()
        if oneshot:
            frames = 50
            orc.inference(lat[:1, :frames].cpu())
            sample = f"one {frames}-frame utterance (2 s) of the same workload"
        else:
            frames = 0
            for i in range(2):
                st = vo.stream_init(orc, VOC_CHUNK)
                st.window.copy_(win[i].cpu())
                st.total, st.emitted = 10 ** 6, 10 ** 6 - cfg.lookahead
                vo.stream_step(orc, st, lat[i].cpu())
                frames += VOC_CHUNK
            sample = "2 request stream steps (16-frame chunks, 51-frame windows) of the same workload"
        secs = time.perf_counter() - t0
        cpu = {"value": round(frames * VOC_FRAME_S / secs, 4), "unit": "audio-s/s",
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{sample}: this build's restatement of the reference AudioVAE "
                         f"(oracle/voc_oracle.py), fp32 torch on the host, {secs:.2f} s"}
    if rank == 0:
        line = {"metric": (VOC1_METRIC if oneshot else VOC_METRIC).format(n=n),
                "value": round(audio_s / (ms / 1000), 2), "unit": "audio-s/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "fp32 (front, activations, accumulation) + fp16 convolution operands",
                "data": "synthetic (seeded random-init vocoder of the VOC_BASE shape, N(0,1) latents)",
                "config": {"workload": args.workload, "requests_per_gpu": n,
                           "frames_per_request": F, "decoded_frames": T, "hop": cfg.hop,
                           "initial_channels": cfg.initial_channels,
                           "upsample_rates": list(cfg.upsample_rates),
                           "l2": "activations (GBs per call) larger than L2, no flush",
                           "parallelism": f"request-sharded x{world}"},
                "e2e": {"value": round(audio_s / (e2e_ms / 1000), 2), "unit": "audio-s/s",
                        "h2d_bytes_per_step": h_lat.numel() * 4, "d2h_bytes_per_step": d2h,
                        "ms_per_step": round(e2e_ms, 4), "api": "decode_batch" if oneshot else "stream_step_many"},
                "eager_ms_per_step": round(eager_ms, 4),
                "gpu_launches": voc_launches(cfg, F, oneshot, voc.num_convs) * args.steps,
                "roofline": {"kernel": f"convolution #{heavy} (the call's largest)",
                             "bound": "tensor", "achieved": round(ach(flops[heavy], conv_us[heavy]), 1),
                             "peak": round(f16, 1), "unit": "TFLOP/s",
                             "frac": round(ach(flops[heavy], conv_us[heavy]) / f16, 4), "traffic": None,
                             "algorithmic_per_launch": flops[heavy],
                             "peak_source": f"{peak_kind} sustained bf16 (fp16 operands run at the bf16 rate)",
                             "timing": "dvoc_conv_launch, CUDA events, 3 launches"},
                "kernels": {"convs": {"count": len(conv_us), "us": round(conv_total_us, 1),
                                      "achieved": round(ach(sum(flops), conv_total_us), 1),
                                      "unit": "TFLOP/s", "frac": round(ach(sum(flops), conv_total_us) / f16, 4),
                                      "share_of_call": round(conv_total_us / (ms * 1000), 4)},
                            "slowest_conv": {"index": top, "us": round(conv_us[top], 1),
                                             "achieved": round(ach(flops[top], conv_us[top]), 1)},
                            "per_conv_us": [round(x, 1) for x in conv_us]},
                "clocks": clk.summary(), "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)
    graph = None
    voc.close()


def voc_launches(cfg, F: int, oneshot: bool, convs: int) -> int:
    """Kernels of one dvoc_decode call: the front (3 linears, per LSTM layer its
    input linear, F steps and the state copy), the decoder input (and the
    window store), every convolution and activation, conv_post."""
    per = 6 if cfg.resblock == "1" else 2
    acts = len(cfg.upsample_rates) * len(cfg.resblock_kernel_sizes) * per + 1
    return 3 + cfg.mi_layers * (2 + F) + (1 if oneshot else 2) + convs + acts + 1


def _voc_left(cfg) -> int:
    import ctypes
    from nanovllm_dots_b200 import _lib
    from nanovllm_dots_b200.vocoder import dvoc_config
    c = dvoc_config(cfg, 1, 1)
    return _lib.lib().dvoc_stream_left_context(ctypes.byref(c))


def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=180))
    try:
        if args.workload == "pe":
            run_pe(args, rank, world)
        elif args.workload == "llmattn":
            run_llmattn(args, rank, world)
        elif args.workload == "llmdecode":
            run_llmdecode(args, rank, world)
        elif args.workload == "engine":
            run_engine(args, rank, world)
        elif args.workload in ("voc", "voc1"):
            run_voc(args, rank, world, oneshot=args.workload == "voc1")
        elif args.workload == "vocprof":
            run_voc(args, rank, world, oneshot=False, n=16)
        else:
            run_b200(args, rank, world)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
