"""Golden vectors for the vocoder, made by running the REFERENCE's own
``AudioVAE`` (``nanovllm_dots/models/dots/native/vocoder/bigvgan.py``) on the
CPU in fp32.

    python tests/golden/make_golden_voc.py --reference /path/to/nanovllm_dots

The reference model is built from ``synthetic.VOC_SMALL.reference_dict()``
the way its loader does (``native/loader.py:94-110``: construct,
``remove_weight_norm``, load the state dict), with the seeded weights of
``synthetic.make_voc_weights(VOC_SMALL, seed=0)`` (the encoder half, unused
on this path, keeps its constructor init).  Recorded:

* one-shot ``inference_from_latents(do_sample=False)`` of two utterances of
  7 and 12 frames (``native/model.py:205-206``);
* strict streaming with chunk 8 (``init_stream_state``, ``stream_step``,
  ``stream_flush``; ``native/model.py:208-218``): stream A takes 13 chunks
  (104 frames, more than the 84-frame window, so the window slides), stream B
  3 chunks; every emitted piece of audio is stored in order.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from nanovllm_dots_b200 import synthetic as syn  # noqa: E402

ONESHOT_FRAMES = (7, 12)
CHUNK = 8
STREAM_CHUNKS = {"A": 13, "B": 3}


def build_reference(path: str, cfg: syn.VocConfig, w: dict[str, torch.Tensor]):
    sys.path.insert(0, path)
    from nanovllm_dots.models.dots.native.vocoder import AudioVAE, AudioVAEConfig
    torch.manual_seed(0)
    vae = AudioVAE(AudioVAEConfig.from_dict(cfg.reference_dict())).eval()
    vae.remove_weight_norm()
    missing, unexpected = vae.load_state_dict(w, strict=False)
    assert not unexpected, unexpected[:8]
    bad = [k for k in missing if not k.startswith(("audio_encoder.", "enc_mi_layer.", "pre_proj."))]
    assert not bad, bad[:8]
    return vae


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DFM_REFERENCE"),
                    required=os.environ.get("DFM_REFERENCE") is None,
                    help="reference checkout (or set DFM_REFERENCE)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    cfg = syn.VOC_SMALL
    w = syn.make_voc_weights(cfg, seed=0)
    vae = build_reference(args.reference, cfg, w)
    arrays, man = {}, {"config": cfg.reference_dict(), "chunk": CHUNK,
                       "oneshot_frames": list(ONESHOT_FRAMES), "streams": {}}
    with torch.no_grad():
        for i, T in enumerate(ONESHOT_FRAMES):
            lat = syn.make_voc_latents(1, T, seed=100 + i, cfg=cfg)
            wav = vae.inference_from_latents(lat.transpose(1, 2), do_sample=False)
            arrays[f"oneshot{i}_latents"] = lat[0].numpy()
            arrays[f"oneshot{i}_audio"] = wav.reshape(-1).numpy()
        for s, (name, n) in enumerate(STREAM_CHUNKS.items()):
            lat = syn.make_voc_latents(1, n * CHUNK, seed=200 + s, cfg=cfg)
            st = vae.init_stream_state(batch_size=1, chunk_size=CHUNK)
            pieces = []
            for k in range(n):
                out = vae.stream_step(lat[:, k * CHUNK:(k + 1) * CHUNK].transpose(1, 2), st)
                pieces.append(out.reshape(-1).numpy())
            pieces.append(vae.stream_flush(st).reshape(-1).numpy())
            arrays[f"stream{name}_latents"] = lat[0].numpy()
            for k, p in enumerate(pieces):
                arrays[f"stream{name}_piece{k}"] = p
            man["streams"][name] = {"chunks": n, "piece_samples": [int(p.size) for p in pieces],
                                    "window": int(st.decoder.window.shape[-1])}
            print(name, "window", st.decoder.window.shape[-1], "pieces", [p.size for p in pieces])
    man["weights_sha256"] = syn.weights_digest(w)
    np.savez_compressed(os.path.join(args.out, "voc_golden.npz"), **arrays)
    with open(os.path.join(args.out, "voc_manifest.json"), "w") as f:
        json.dump(man, f, indent=1)
    print("wrote", os.path.join(args.out, "voc_golden.npz"))


if __name__ == "__main__":
    main()
