"""Generate the golden patch-encoder fixtures by running the REFERENCE's own code.

Run in a container where the reference checkout is importable (it is not on
the GPU test box; the fixture it writes is committed):

    python tests/golden/make_golden_pe.py --reference /path/to/nanovllm_dots

The reference module used is ``nanovllm_dots/models/dots/native/patch_encoder.py``
(``VAESemanticEncoder``: ``init_decode_state``, ``decode_patch``, ``prefill``)
with its config wrapper ``native/config.py`` (``PatchEncoderModelConfig``).
Everything runs in fp32 on the CPU with the seeded bf16-valued weights of
``nanovllm_dots_b200.synthetic.make_pe_weights`` (the script checks that the
reference module built under the same seed holds exactly those values before
the LayerNorm jitter, then loads the jittered set).

Cases (outputs fp32 embeddings):
  small_decode   small config, 3 requests, 6 patches each, advanced through the
                 reference's per-request ``decode_patch`` (dense-mask SDPA over
                 the fixed cache capacity)
  small_prefill  small config, a 3-patch prompt through ``prefill``, then 2
                 ``decode_patch`` steps
  full_decode    the synthetic full-size config (PE_BASE), 2 requests x 2
                 patches
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

SMALL = syn.PEConfig(layers=2, hidden=128, heads=2, ffn=256, out_dim=192)
CAP_PATCHES = 16


def load_reference(path):
    sys.path.insert(0, path)
    from nanovllm_dots.models.dots.native.patch_encoder import VAESemanticEncoder
    from nanovllm_dots.models.dots.native.config import PatchEncoderModelConfig
    return VAESemanticEncoder, PatchEncoderModelConfig


def build(ref, cfg: syn.PEConfig):
    VAESemanticEncoder, PatchEncoderModelConfig = ref
    raw = {"patch_size": cfg.patch,
           "PatchEncoder": {"hidden_size": cfg.hidden, "num_heads": cfg.heads,
                            "ffn_hidden_size": cfg.ffn, "num_layers": cfg.layers,
                            "norm_layer": "LayerNorm", "causal": True}}
    torch.manual_seed(0)
    pe = VAESemanticEncoder(in_dim=cfg.latent_dim, out_dim=cfg.out_dim,
                            config=PatchEncoderModelConfig(raw)).eval()
    assert pe.out_ds_rate == cfg.rows
    w0 = syn.make_pe_weights(cfg, ln_jitter=0.0)
    sd = {k: v.detach().to(torch.bfloat16).float() for k, v in pe.state_dict().items()}
    assert set(sd) == set(w0), sorted(set(sd) ^ set(w0))[:8]
    for k in w0:
        assert torch.equal(sd[k], w0[k]), k
    w = syn.make_pe_weights(cfg)
    pe.load_state_dict(w)
    return pe, w


def decode_case(pe, cfg, patches):
    """patches [P, n, patch, ld] -> embeddings [P, n, out_dim] via per-request
    reference decode_patch."""
    P, n = patches.shape[:2]
    states = [pe.init_decode_state(max_audio_patch_count=CAP_PATCHES, batch_size=1,
                                   device=torch.device("cpu"), dtype=torch.float32)
              for _ in range(n)]
    out = torch.zeros(P, n, cfg.out_dim)
    with torch.no_grad():
        for p in range(P):
            for i in range(n):
                st = states[i]
                pos = torch.arange(pe.out_ds_rate, dtype=torch.long) + st.seq_len
                emb, tail = pe.decode_patch(patches[p, i:i + 1].float(), st.conv_tail,
                                            st.layer_caches, pos)
                st.conv_tail.copy_(tail)
                st.seq_len += pe.out_ds_rate
                out[p, i] = emb.reshape(-1)
    return out


def prefill_case(pe, cfg, prompt, tail_patches):
    st = pe.init_decode_state(max_audio_patch_count=CAP_PATCHES, batch_size=1,
                              device=torch.device("cpu"), dtype=torch.float32)
    with torch.no_grad():
        emb, st = pe.prefill(prompt.float().unsqueeze(0), st)
        dec = []
        for p in range(tail_patches.shape[0]):
            pos = torch.arange(pe.out_ds_rate, dtype=torch.long) + st.seq_len
            e, tail = pe.decode_patch(tail_patches[p:p + 1].float(), st.conv_tail,
                                      st.layer_caches, pos)
            st.conv_tail.copy_(tail)
            st.seq_len += pe.out_ds_rate
            dec.append(e.reshape(-1))
    return emb.reshape(-1, cfg.out_dim), torch.stack(dec)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=os.path.join(HERE, "pe_golden.npz"))
    args = ap.parse_args()
    ref = load_reference(args.reference)
    arrays, manifest = {}, {"cases": {}}

    pe, w = build(ref, SMALL)
    manifest["small_weights_sha256"] = syn.weights_digest(w)
    patches = syn.make_pe_patches(3, 6, seed=11, cfg=SMALL)
    arrays["small_decode_patches"] = patches.float().numpy()
    arrays["small_decode_out"] = decode_case(pe, SMALL, patches).numpy()
    manifest["cases"]["small_decode"] = {"n": 3, "patches": 6, "seed": 11}

    prompt = syn.make_pe_patches(1, 3, seed=12, cfg=SMALL).reshape(-1, SMALL.latent_dim)
    tailp = syn.make_pe_patches(1, 2, seed=13, cfg=SMALL)[:, 0]
    pre, dec = prefill_case(pe, SMALL, prompt, tailp)
    arrays["small_prefill_prompt"] = prompt.float().numpy()
    arrays["small_prefill_tail"] = tailp.float().numpy()
    arrays["small_prefill_out"] = pre.numpy()
    arrays["small_prefill_dec"] = dec.numpy()
    manifest["cases"]["small_prefill"] = {"prompt_patches": 3, "decode_patches": 2,
                                          "seeds": [12, 13]}

    pe, w = build(ref, syn.PE_BASE)
    manifest["full_weights_sha256"] = syn.weights_digest(w)
    patches = syn.make_pe_patches(2, 2, seed=14)
    arrays["full_decode_patches"] = patches.float().numpy()
    arrays["full_decode_out"] = decode_case(pe, syn.PE_BASE, patches).numpy()
    manifest["cases"]["full_decode"] = {"n": 2, "patches": 2, "seed": 14}

    np.savez_compressed(args.out, **arrays)
    with open(os.path.join(HERE, "pe_manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    print("wrote", args.out, {k: v.shape for k, v in arrays.items()})


if __name__ == "__main__":
    main()
