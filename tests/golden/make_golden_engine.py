"""Golden vectors for the engine-level FM dispatch, made by running the
REFERENCE's own engine code on the CPU.

    python tests/golden/make_golden_engine.py --reference /path/to/nanovllm_dots

Three requests shaped like the reference's ``DotsSeqState`` /
``_GenerateState`` (``nanovllm_dots/models/dots/engine.py:48-77``,
``native/model.py:18-28``) are decoded for three engine ticks.  Their FM
histories are built with the reference's own ``DotsModel._append_hidden_chunk``
and ``_append_history_chunk`` (``native/model.py:101-120``) into bf16 buffers,
as the engine allocates them (``engine.py:286-319``), and every tick runs the
reference's MeanFlow dispatch: ``DotsBatchEngine._pack_fm_inputs``
(``engine.py:635-688``, padded batch + FM mask + positions + g_cond) and
``batched_meanflow`` (``batched_fm.py:82-126``), i.e. ``_full_fm``
(``engine.py:690-709``) with the tick's noise passed in instead of drawn.
Everything runs in fp32 on the CPU with the seeded weights of
``nanovllm_dots_b200.synthetic``.

Requests:
  A  no prompt, no speaker condition: ticks 0, 1, 2
  B  a voice-clone prompt of 3 patches seeded into the history first
     (latent, hidden, latent, hidden, latent, hidden rows): ticks 0, 1
  C  joins at tick 1 with a speaker condition g_cond: ticks 1, 2
After each tick the request's decoded patch is appended to its history
(``engine.py:751``) and a new LLM hidden row before the next tick
(``engine.py:531``).  The fixture holds, per request, the final history buffer
(bf16 bits), its length before each tick, g_cond, and per tick the request
order, noise and decoded latents.
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
sys.path.insert(0, HERE)

from nanovllm_dots_b200 import synthetic as syn  # noqa: E402
from make_golden import build, load_reference  # noqa: E402

TICKS = [["A", "B"], ["A", "B", "C"], ["C", "A"]]
PROMPT_PATCHES = 3


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.bfloat16).contiguous().view(torch.int16).numpy()


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
    nmodel, batched_fm = ref[2], ref[3]
    from nanovllm_dots.models.dots.engine import DotsBatchEngine, DotsSeqState

    w = syn.make_weights(cfg, seed=0)
    dit, core = build(ref, cfg, w)
    core.mode = "meanflow"
    # the reference's own DotsModel over the synthetic core (its vocoder and
    # speaker encoder are not used on this path)
    dots = nmodel.DotsModel(core, types.SimpleNamespace(hop_size=1), None,
                            patch_size=cfg.latent_patch)
    engine = types.SimpleNamespace(core=core, dots=dots, fm_len_bucket=0,
                                   device=torch.device("cpu"), dtype=torch.float32)
    append_hidden = dots._append_hidden_chunk
    append_latent = dots._append_history_chunk

    g = torch.Generator().manual_seed(404)
    cap = 160
    states, payloads, gconds = {}, {}, {}
    for name in "ABC":
        z = lambda *s: torch.zeros(*s, dtype=torch.bfloat16)
        states[name] = nmodel._GenerateState(fm_seq_len=0, fm_capacity=cap,
                                             fm_sequence=z(1, cap, cfg.hidden),
                                             fm_cfg_sequence=z(1, cap, cfg.hidden),
                                             fm_null_g_cond=z(1, cfg.hidden))
        gc = (torch.randn(cfg.hidden, generator=g) * 0.5).to(torch.bfloat16) if name == "C" else None
        gconds[name] = gc
        payloads[name] = DotsSeqState(schedule=torch.zeros(1, 1), prefill_end=0, span_count=8,
                                      g_cond=gc, gen_state=states[name],
                                      prefill_embed=torch.zeros(1, 1), num_steps=cfg.nfe)

    def hidden():
        return torch.randn(1, 1, cfg.cond_dim, generator=g).to(torch.bfloat16)

    with torch.no_grad():
        # B's voice-clone prompt: prompt latents interleaved with prefill hiddens
        for _ in range(PROMPT_PATCHES):
            lat = torch.randn(1, cfg.latent_patch, cfg.latent_dim, generator=g).to(torch.bfloat16)
            append_latent(states["B"], lat.float())
            append_hidden(states["B"], hidden().float())
        arrays, man = {}, {"weights_sha256": syn.weights_digest(w), "ticks": []}
        for t, names in enumerate(TICKS):
            for name in names:
                if name != "B" or t > 0:           # B's first active hidden came with the prompt
                    append_hidden(states[name], hidden().float())
            plist = [payloads[nm] for nm in names]
            lens = [states[nm].fm_seq_len for nm in names]
            noise = torch.randn(len(names), cfg.latent_patch, cfg.latent_dim,
                                generator=g).to(torch.bfloat16)
            inp, _, mask, pos, gcond, p0, meanflow = DotsBatchEngine._pack_fm_inputs(engine, plist)
            assert meanflow
            z = batched_fm.batched_meanflow(core, input_sequence=inp, attn_mask=mask, pos_ids=pos,
                                            g_cond=gcond, num_steps=p0.num_steps,
                                            noise=noise.float(), vfp=dit)
            arrays[f"tick{t}_noise"] = bf16_bits(noise)
            arrays[f"tick{t}_z"] = z.float().numpy()
            man["ticks"].append({"requests": names, "fm_seq_len": lens})
            for j, name in enumerate(names):
                append_latent(states[name], z[j:j + 1])
            print(f"tick {t}: {names} lens {lens} |z|max {float(z.abs().max()):.3f}")
    for name in "ABC":
        st = states[name]
        arrays[f"{name}_fm_sequence"] = bf16_bits(st.fm_sequence[0, :st.fm_seq_len])
        if gconds[name] is not None:
            arrays[f"{name}_g_cond"] = bf16_bits(gconds[name])
    np.savez_compressed(os.path.join(args.out, "engine_golden.npz"), **arrays)
    with open(os.path.join(args.out, "engine_manifest.json"), "w") as f:
        json.dump(man, f, indent=1)
    print("wrote", os.path.join(args.out, "engine_golden.npz"))


if __name__ == "__main__":
    main()
