"""The engine drop-in (``fm_accel="b200"``) with a real ``B200FMHead`` against
golden vectors made by the reference's own engine code
(``tests/golden/make_golden_engine.py``: ``_pack_fm_inputs`` +
``batched_meanflow``, the MeanFlow ``_full_fm`` path of ``engine.py:690-709``).

Three requests over three ticks, shaped like the reference's payloads
(``DotsSeqState.gen_state.fm_sequence`` bf16 on the device, ``fm_seq_len``,
``g_cond``): one without prompt, one whose history starts with a voice-clone
prompt (the dispatch bulk-prefills it), one with a speaker condition that joins
at the second tick; the request order changes between ticks and one request
finishes early.  Each tick's noise is the golden run's.  Both dispatch modes:
a captured tick per batch size, and eager launches.  Tolerance (bf16 path,
after 4 NFE): per-frame cosine >= 0.9999 and max-abs <= 2e-2 against the fp32
reference."""
from __future__ import annotations

import gc
from types import SimpleNamespace

import pytest
import torch

from conftest import cos_min
from nanovllm_dots_b200 import synthetic as syn
from nanovllm_dots_b200.engine_mode import B200FMDispatch, install
from nanovllm_dots_b200.fm_head import B200FMHead
from test_engine_golden import load_engine_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
COS, MAXABS = 0.9999, 2e-2


class _Payload:
    """The fields of DotsSeqState the FM dispatch reads (a plain object, so the
    dispatch can key its state on it and see it go away)."""

    def __init__(self, seq: torch.Tensor, g_cond):
        cap = seq.shape[0] + 8
        buf = torch.zeros(1, cap, seq.shape[1], dtype=torch.bfloat16, device=DEV)
        buf[0, :seq.shape[0]] = seq.to(DEV)
        self.gen_state = SimpleNamespace(fm_sequence=buf, fm_seq_len=0,
                                         fm_null_g_cond=torch.zeros(1, seq.shape[1],
                                                                    dtype=torch.bfloat16,
                                                                    device=DEV))
        self.g_cond = g_cond
        self.num_steps = syn.BASE.nfe


@pytest.mark.parametrize("use_graphs", [True, False], ids=["graph", "eager"])
def test_dispatch_matches_reference_engine(weights, use_graphs):
    man, arr = load_engine_golden()
    head = B200FMHead(weights, syn.BASE, num_pages=64, max_pages_per_req=16, max_requests=4,
                      device=DEV)
    engine = SimpleNamespace(fm_accel="none")
    noise = {}
    dispatch = install(engine, head)
    dispatch.use_graphs = use_graphs
    dispatch.noise_fn = lambda n: noise["t"]
    payloads = {}
    for name in "ABC":
        g = arr.get(f"{name}_g_cond")
        payloads[name] = _Payload(arr[f"{name}_fm_sequence"], None if g is None else g.to(DEV))
    try:
        for t, tk in enumerate(man["ticks"]):
            names = tk["requests"]
            for name, L in zip(names, tk["fm_seq_len"]):
                payloads[name].gen_state.fm_seq_len = L
            noise["t"] = arr[f"tick{t}_noise"].to(DEV)
            out = engine._batched_fm([payloads[nm] for nm in names])
            head.check_errors()
            ref = arr[f"tick{t}_z"]
            got = out.float().cpu()
            for j, name in enumerate(names):
                c = cos_min(got[j], ref[j])
                e = (got[j] - ref[j]).abs().max().item()
                assert c >= COS and e <= MAXABS, f"tick {t} {name}: cos_min={c:.6f} max_abs={e:.4g}"
            if t == 1:
                # B finishes after tick 1: its pages return to the pool
                rid = id(payloads["B"])
                assert rid in head.requests
                del payloads["B"]
                gc.collect()
                assert rid not in head.requests
        assert isinstance(dispatch, B200FMDispatch) and engine.fm_accel == "b200"
    finally:
        head.close()
