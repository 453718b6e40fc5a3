"""The B200 vocoder against the reference's own AudioVAE outputs
(``tests/golden/voc_golden.npz``, made by ``make_golden_voc.py``) and against
the oracle at the full synthetic shape.

Tolerance: the decoder's convolutions run with fp16 operands (a 10-bit
mantissa: the precision of the tf32 operands PyTorch's cuDNN convolutions use
on this GPU by default) and fp32 accumulation; the front, the activations and
conv_post run in fp32.  Audio in [-1, 1] must match the fp32 reference with max-abs <= 2e-2
and a signal-to-error ratio >= 40 dB per request (per emitted piece for
streams)."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from nanovllm_dots_b200 import synthetic as syn
from nanovllm_dots_b200.vocoder import B200Vocoder, install_vocoder
from oracle import voc_oracle as vo

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
MAXABS, SNR_DB = 2e-2, 40.0
DEV = torch.device("cuda")


def check(got: torch.Tensor, ref, what: str) -> None:
    got = got.detach().float().cpu().numpy().astype(np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    if ref.size == 0:
        return
    err = np.abs(got - ref)
    snr = 10 * np.log10((ref ** 2).sum() / max((err ** 2).sum(), 1e-30))
    assert err.max() <= MAXABS and snr >= SNR_DB, f"{what}: max_abs={err.max():.3g} snr={snr:.1f} dB"


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLDEN, "voc_manifest.json")) as f:
        man = json.load(f)
    return man, dict(np.load(os.path.join(GOLDEN, "voc_golden.npz")))


@pytest.fixture(scope="module")
def small():
    voc = B200Vocoder(syn.make_voc_weights(syn.VOC_SMALL, seed=0), syn.VOC_SMALL, max_batch=4,
                      max_frames=96, device=DEV)
    yield voc
    voc.close()


def test_oneshot_matches_reference(small, golden):
    """Two utterances of different lengths in one call."""
    man, arr = golden
    lats = [torch.from_numpy(arr[f"oneshot{i}_latents"]) for i in range(len(man["oneshot_frames"]))]
    audio = small.decode_batch(lats)
    small.check_errors()
    for i, a in enumerate(audio):
        check(a, arr[f"oneshot{i}_audio"], f"oneshot{i}")


def test_oneshot_api_shape(small, golden):
    man, arr = golden
    lat = torch.from_numpy(arr["oneshot1_latents"]).T[None].to(DEV)     # [1, L, T]
    out = small.inference_from_latents(lat, do_sample=False)
    assert out.shape == (1, 1, lat.shape[-1] * syn.VOC_SMALL.hop)
    check(out[0, 0], arr["oneshot1_audio"], "inference_from_latents")


def test_streams_match_reference(small, golden):
    """Streams A (13 chunks: the window slides) and B (3 chunks) batched in the
    same calls while both run, every emitted piece compared."""
    man, arr = golden
    chunk = man["chunk"]
    lat = {k: torch.from_numpy(arr[f"stream{k}_latents"]) for k in "AB"}
    st = {k: small.init_stream_state(1, chunk) for k in "AB"}
    assert st["A"].window.shape[0] == man["streams"]["A"]["window"]
    pieces = {k: [] for k in "AB"}
    nA, nB = man["streams"]["A"]["chunks"], man["streams"]["B"]["chunks"]
    for k in range(nA):
        names = ["A", "B"] if k < nB else ["A"]
        x = torch.stack([lat[n][k * chunk:(k + 1) * chunk] for n in names])
        for n, p in zip(names, small.stream_step_many([st[n] for n in names], x)):
            pieces[n].append(p)
        if k == nB - 1:
            pieces["B"] += small.stream_flush_many([st["B"]])
    pieces["A"].append(small.stream_flush(st["A"])[0, 0])
    small.check_errors()
    for n in "AB":
        ref = man["streams"][n]["piece_samples"]
        assert [p.numel() for p in pieces[n]] == ref
        for i, p in enumerate(pieces[n]):
            check(p, arr[f"stream{n}_piece{i}"], f"stream {n} piece {i}")


def test_stream_single_api(small, golden):
    """``stream_step`` with the reference's [1, L, chunk] layout."""
    man, arr = golden
    chunk = man["chunk"]
    lat = torch.from_numpy(arr["streamB_latents"])
    st = small.init_stream_state(1, chunk)
    for k in range(2):
        out = small.stream_step(lat[k * chunk:(k + 1) * chunk].T[None], st)
        check(out[0, 0], arr[f"streamB_piece{k}"], f"stream_step {k}")


def test_stream_errors(small):
    st = small.init_stream_state(1, 8)
    with pytest.raises(ValueError, match="chunk_size must stay fixed"):
        small.stream_step_many([st], torch.zeros(1, 4, syn.VOC_SMALL.latent_dim))
    with pytest.raises(ValueError):
        small.init_stream_state(1, 40)          # window 40 + 2 + 74 > max_frames
    with pytest.raises(ValueError):
        small.decode_batch([torch.zeros(97, syn.VOC_SMALL.latent_dim)])


def test_install_vocoder(small):
    from types import SimpleNamespace
    engine = SimpleNamespace(dots=SimpleNamespace(vocoder=None, hop_size=0))
    install_vocoder(engine, small)
    assert engine.dots.vocoder is small and engine.dots.hop_size == syn.VOC_SMALL.hop


def test_full_shape_against_oracle():
    """The synthetic full shape (1536 initial channels, six stages, hop 1920):
    one-shot of 3 utterances and a stream of two 16-frame chunks + flush for
    two requests, against the float64 oracle."""
    cfg = syn.VOC_BASE
    w = syn.make_voc_weights(cfg, seed=1)
    voc = B200Vocoder(w, cfg, max_batch=3, max_frames=64, device=DEV)
    oracle = vo.VocOracle(w, cfg)
    try:
        lats = [syn.make_voc_latents(1, T, seed=50 + T, cfg=cfg)[0] for T in (5, 3, 6)]
        audio = voc.decode_batch(lats)
        for i, lat in enumerate(lats):
            check(audio[i], oracle.inference(lat[None])[0].numpy(), f"full one-shot {i}")
        lat = syn.make_voc_latents(2, 32, seed=77, cfg=cfg)
        st = [voc.init_stream_state(1, 16) for _ in range(2)]
        ost = [vo.stream_init(oracle, 16) for _ in range(2)]
        for k in range(2):
            got = voc.stream_step_many(st, lat[:, 16 * k:16 * (k + 1)])
            for i in range(2):
                check(got[i], vo.stream_step(oracle, ost[i], lat[i, 16 * k:16 * (k + 1)]).numpy(),
                      f"full stream {i} chunk {k}")
        got = voc.stream_flush_many(st)
        for i in range(2):
            check(got[i], vo.stream_flush(oracle, ost[i]).numpy(), f"full stream {i} flush")
        voc.check_errors()
    finally:
        voc.close()


def test_batched_step_stream_with_real_vocoder(small):
    """The engine's batched ``step_stream`` (``vocoder.batched_step_stream``)
    over the real vocoder: two streams and one one-shot request, audio equal to
    the per-request AudioVAE-style calls (the same kernels, so equal to rounding
    of the batch size: same tolerance as above)."""
    from types import SimpleNamespace
    from nanovllm_dots_b200.vocoder import batched_step_stream
    cfg = syn.VOC_SMALL
    ps = 8
    lat = syn.make_voc_latents(3, 3 * ps, seed=21, cfg=cfg)
    dots = SimpleNamespace(vocoder=small, hop_size=small.hop_size,
                           _init_vocoder_stream_state=lambda: small.init_stream_state(1, ps))
    mk = lambda sid, stream: SimpleNamespace(
        seq_id=sid, stoped=False, custom_payload=SimpleNamespace(stream=stream, latents=[], vocoded=0,
                                                                 vocoder_state=None))
    seqs = [mk("s0", True), mk("s1", True), mk("o2", False)]
    steps = iter(range(3))

    def step():
        k = next(steps)
        for i, s in enumerate(seqs):
            s.custom_payload.latents.append(lat[i:i + 1, k * ps:(k + 1) * ps])
            s.stoped = k == 2
        return seqs

    engine = SimpleNamespace(dots=dots, core=SimpleNamespace(latent_patch_size=ps), step=step,
                             scheduler=SimpleNamespace(is_finished=lambda: False))
    audio = {s.seq_id: [] for s in seqs}
    for _ in range(3):
        for sid, kind, x in batched_step_stream(engine):
            if kind == "audio":
                audio[sid].append(x)
    for i in range(2):
        st = small.init_stream_state(1, ps)
        ref = [small.stream_step(lat[i:i + 1, k * ps:(k + 1) * ps].transpose(1, 2), st)[0, 0] for k in range(3)]
        ref.append(small.stream_flush(st)[0, 0])
        ref = torch.cat([r for r in ref if r.numel()])
        check(torch.cat(audio[f"s{i}"]), ref.cpu().numpy(), f"batched step_stream s{i}")
    check(torch.cat(audio["o2"]), small.decode_batch([lat[2]])[0].cpu().numpy(), "batched step_stream one-shot")
