"""CPU pin of the FP8 path's numerics (config 3): the QKV and fc1 projections
on e4m3 operands with one scale per activation row and one per weight row,
every other operation as in the fp32 oracle.  After the 4 MeanFlow steps the
output latents must stay within the FP8 tolerance (per-frame cosine >= 0.999)
of the unquantised oracle."""
from __future__ import annotations

import torch

from conftest import cos_min
from nanovllm_dots_b200 import synthetic as syn
from nanovllm_dots_b200.fm_head import quantize_rows_e4m3
from oracle import dit_oracle as O

FP8_COS = 0.999


def _rowwise_fp8(x: torch.Tensor) -> torch.Tensor:
    q, s = quantize_rows_e4m3(x)
    return q.view(torch.float8_e4m3fn).float() * s.unsqueeze(-1)


def test_rowwise_fp8_qkv_fc1_stays_within_tolerance(weights, monkeypatch):
    b = syn.make_batch(2, [3, 0], seed=7, n_extend=[17, 0])
    ref = O.tick_batch(weights, b, syn.BASE)
    base = O.linear

    def linear_fp8(x, w, name, bias=True):
        if not name.endswith(("q_proj", "k_proj", "v_proj", "ffn.fc1")):
            return base(x, w, name, bias)
        y = _rowwise_fp8(x.float()) @ _rowwise_fp8(w[name + ".weight"].float()).t()
        if bias and (name + ".bias") in w:
            y = y + w[name + ".bias"].float()
        return y

    monkeypatch.setattr(O, "linear", linear_fp8)
    out = O.tick_batch(weights, b, syn.BASE)
    assert cos_min(out, ref) >= FP8_COS
