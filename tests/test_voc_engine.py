"""``vocoder.batched_step_stream`` against the reference's own
``DotsBatchEngine.step_stream`` (``engine.py:855-893``), on the CPU with a
deterministic stand-in vocoder whose batched methods are its per-request
methods in a loop: the events (order, kinds, audio) and the per-request
bookkeeping must be identical.  The script of steps covers streaming requests
with one and several pending patches, a stream that finishes without a patch
(no flush audio), one-shot requests finishing with and without latents, and
``vocode=False``.  Needs the reference checkout (DFM_REFERENCE, default a
``reference`` folder beside this repository); skipped without it."""
from __future__ import annotations

import os
import sys
import types

import pytest
import torch

from nanovllm_dots_b200.vocoder import batched_step_stream, install_vocoder

# the checkout named by DFM_REFERENCE, else a `reference` folder beside this
# repository
REF = os.environ.get("DFM_REFERENCE") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference")


def _reference():
    if not os.path.isdir(REF):
        pytest.skip("reference checkout not available")
    sys.modules.setdefault("torchdiffeq", types.SimpleNamespace(odeint=None))
    if REF not in sys.path:
        sys.path.insert(0, REF)
    from nanovllm_dots.models.dots.engine import DotsBatchEngine, DotsSeqState
    from nanovllm_dots.models.dots.native import model as nmodel
    return DotsBatchEngine, DotsSeqState, nmodel


class FakeVocoder:
    """Deterministic AudioVAE stand-in: a stream's audio depends on its own
    state and chunk; the batched methods loop over the per-request ones."""
    hop_size = 3

    def init_stream_state(self, batch_size=1, chunk_size=8):
        return types.SimpleNamespace(total=0, chunk=chunk_size, calls=0)

    def stream_step(self, latents, state):              # [1, L, chunk]
        state.calls += 1
        state.total += latents.shape[-1]
        n = 0 if state.calls == 1 else latents.shape[-1] * self.hop_size   # first call emits nothing
        return (latents.sum() + state.total + torch.arange(n, dtype=torch.float32)).view(1, 1, -1)

    def stream_flush(self, state):
        return torch.full((1, 1, 5), -float(state.total))

    def inference_from_latents(self, x, do_sample=True):   # [1, L, T]
        return x.sum(1, keepdim=True).repeat_interleave(self.hop_size, dim=-1)

    def stream_step_many(self, states, latents):          # [n, chunk, L]
        return [self.stream_step(latents[i:i + 1].transpose(1, 2), s)[0, 0] for i, s in enumerate(states)]

    def stream_flush_many(self, states):
        return [self.stream_flush(s)[0, 0] for s in states]

    def decode_batch(self, lats):                         # [T, L] each
        return [self.inference_from_latents(l.T[None])[0, 0] for l in lats]


PS, L = 4, 6
# per step: {name: (new patches, stops)}; streams A, B, D; one-shot C, E
SCRIPT = [
    {"A": (1, False), "B": (0, False), "C": (1, False)},
    {"A": (1, False), "B": (2, False), "C": (2, True), "D": (0, False)},
    {"A": (1, True), "B": (1, False), "D": (0, True), "E": (0, True)},
    {"B": (1, True)},
]
STREAM = {"A": True, "B": True, "D": True, "C": False, "E": False}


def run(DotsBatchEngine, DotsSeqState, nmodel, batched: bool, vocode_steps=(True, True, True, True)):
    g = torch.Generator().manual_seed(7)
    core = types.SimpleNamespace(latent_patch_size=PS)
    dots = nmodel.DotsModel(core, FakeVocoder(), None, patch_size=PS)
    states = {k: DotsSeqState(schedule=torch.zeros(1, 1), prefill_end=0, span_count=1, g_cond=None,
                              gen_state=None, prefill_embed=torch.zeros(1, 1), num_steps=1,
                              stream=STREAM[k]) for k in STREAM}
    seqs = {k: types.SimpleNamespace(seq_id=k, custom_payload=states[k], stoped=False) for k in STREAM}
    script = iter(SCRIPT)

    def step():
        out = []
        for k, (n, stop) in next(script).items():
            for _ in range(n):
                states[k].latents.append(torch.randn(1, PS, L, generator=g))
            seqs[k].stoped = stop
            out.append(seqs[k])
        return out

    engine = types.SimpleNamespace(dots=dots, core=core, device=torch.device("cpu"), step=step,
                                   scheduler=types.SimpleNamespace(is_finished=lambda: False))
    if not batched:
        for name in ("_vocode_stream_step", "_vocode_flush", "vocode"):
            setattr(engine, name, types.MethodType(getattr(DotsBatchEngine, name), engine))
    events = []
    for vocode in vocode_steps:
        events.append(batched_step_stream(engine, vocode=vocode) if batched
                      else DotsBatchEngine.step_stream(engine, vocode=vocode))
    return events, {k: (s.vocoded, s.vocoder_state is not None) for k, s in states.items()}


@pytest.mark.parametrize("vocode_steps", [(True,) * 4, (True, False, True, True)], ids=["vocode", "mixed"])
def test_batched_step_stream_matches_reference(vocode_steps):
    DotsBatchEngine, DotsSeqState, nmodel = _reference()
    ref, ref_st = run(DotsBatchEngine, DotsSeqState, nmodel, batched=False, vocode_steps=vocode_steps)
    got, got_st = run(DotsBatchEngine, DotsSeqState, nmodel, batched=True, vocode_steps=vocode_steps)
    assert got_st == ref_st
    assert len(got) == len(ref)
    for step, (a, b) in enumerate(zip(got, ref)):
        assert [(s, kind) for s, kind, _ in a] == [(s, kind) for s, kind, _ in b], step
        for (_, _, x), (_, _, y) in zip(a, b):
            assert (x is None) == (y is None)
            if x is not None:
                assert torch.equal(x, y), step


def test_install_vocoder_sets_step_stream():
    engine = types.SimpleNamespace(dots=types.SimpleNamespace(vocoder=None, hop_size=0))
    voc = FakeVocoder()
    install_vocoder(engine, voc)
    assert engine.dots.vocoder is voc and engine.dots.hop_size == 3 and callable(engine.step_stream)
