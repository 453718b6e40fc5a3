"""The engine-side drop-in (``fm_accel="b200"``) on duck-typed payloads shaped
like the reference's DotsSeqState (``engine.py:48-77``): which history rows
graduate each tick, and the bulk prefill of a backlog (``prime_to``)."""
from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from nanovllm_dots_b200 import synthetic as syn
from nanovllm_dots_b200.engine_mode import B200FMDispatch
from nanovllm_dots_b200.fm_head import FMRequest

H = syn.BASE.hidden


class _FakeHead:
    """Records the calls the dispatch makes (no GPU)."""

    def __init__(self):
        self.cfg = syn.BASE
        self.device = torch.device("cpu")
        self.requests = {}
        self.calls = []

    def prime(self, rids, rows, g_cond=None):
        self.calls.append(("prime", list(rids), [r.shape[0] for r in rows]))
        for rid, r in zip(rids, rows):
            self.requests.setdefault(rid, FMRequest(rid)).cache_len += r.shape[0]

    def tick(self, rids, *, noise, act_row, ext_rows, n_extend, g_cond):
        self.calls.append(("tick", list(rids), list(n_extend)))
        for rid, e in zip(rids, n_extend):
            self.requests.setdefault(rid, FMRequest(rid)).cache_len += e
        return torch.zeros(len(rids), syn.BASE.latent_patch, syn.BASE.latent_dim)

    def release(self, rid):
        self.requests.pop(rid, None)


class _Payload:
    """Stands in for DotsSeqState (a plain object, so weak references work)."""

    def __init__(self, rows: int, seed: int):
        g = torch.Generator().manual_seed(seed)
        seq = torch.randn(1, 400, H, generator=g).to(torch.bfloat16)
        self.gen_state = SimpleNamespace(fm_sequence=seq, fm_seq_len=rows, fm_null_g_cond=None)
        self.g_cond = None
        self.num_steps = syn.BASE.nfe


def _payload(rows: int, seed: int):
    return _Payload(rows, seed)


def _cpu_dispatch(head):
    """The dispatch with its device gather replaced by zero rows (no GPU here)."""
    d = B200FMDispatch(head, noise_fn=lambda n: torch.zeros(n, syn.BASE.latent_patch,
                                                            syn.BASE.latent_dim))
    d.pack = lambda payloads, plans: (torch.zeros(len(plans), H),
                                      torch.zeros(len(plans), syn.BASE.stride, H),
                                      torch.zeros(len(plans), H))
    return d


def test_dispatch_graduates_history_and_primes_backlog():
    head = _FakeHead()
    d = _cpu_dispatch(head)
    a, b = _payload(1, 0), _payload(100, 1)      # a: first patch; b: 100-row prompt
    d([a, b])
    # b's backlog: rows [0, 99) pending; all but the last 17 are bulk-prefilled
    assert head.calls[0] == ("prime", [id(b)], [99 - 17])
    assert head.calls[1] == ("tick", [id(a), id(b)], [0, 17])
    assert head.requests[id(b)].cache_len == 99
    a.gen_state.fm_seq_len = 18                  # one patch later
    b.gen_state.fm_seq_len = 117
    d([a, b])
    assert head.calls[2] == ("tick", [id(a), id(b)], [17, 17])
    b.gen_state.fm_seq_len = 50
    with pytest.raises(RuntimeError, match="shrank"):
        d([b])


def test_install_patch_encoder_swaps_the_engine_encoder():
    from nanovllm_dots_b200.engine_mode import install_patch_encoder

    class _FakePE:
        max_rows = 5

        def decode_patch(self, patches, rows):
            return torch.zeros(patches.shape[0], 1, 8)

        def prefill(self, prompt_latents, row):
            return torch.zeros(1, prompt_latents.shape[1] // 16, 8)

        def reset_rows(self, rows):
            pass

    eng = SimpleNamespace(flash_pe=False)
    pe = _FakePE()
    install_patch_encoder(eng, pe)
    assert eng.flash_pe and eng._flash_pe is pe
    assert eng._pe_free == [0, 1, 2, 3, 4] and eng._pe_max_batch == 5
    with pytest.raises(TypeError, match="decode_patch"):
        install_patch_encoder(eng, SimpleNamespace(max_rows=1))


def test_patch_encoder_has_no_cpu_path():
    from nanovllm_dots_b200.patch_encoder import B200PatchEncoder
    with pytest.raises(RuntimeError, match="CUDA"):
        B200PatchEncoder({}, syn.PE_BASE, max_batch=1, max_seq_len=16, device="cpu")


def test_patch_encoder_prime_schedules_rows_in_shared_calls():
    """prime(): every row is reset, then decoded one patch per call with all
    rows that still have patches in the same call (at most max_batch)."""
    from nanovllm_dots_b200.patch_encoder import B200PatchEncoder

    calls, resets = [], []

    class _PE(B200PatchEncoder):
        def __init__(self):      # no device: only the scheduling is under test
            self.cfg = syn.PE_BASE
            self.device = torch.device("cpu")
            self.max_batch = 2
            self.out_ds_rate = self.cfg.rows
            self.cap = 64 * self.cfg.rows

        def reset_rows(self, rows):
            resets.append(list(rows))

        def decode_patch(self, latent_patches, rows):
            calls.append((list(rows), latent_patches.shape[0]))
            return torch.full((len(rows), 1, self.cfg.out_dim), float(len(calls)))

    pe = _PE()
    P = syn.PE_BASE.patch
    prompts = [torch.zeros(3 * P, 64), torch.zeros(1 * P, 64), torch.zeros(2 * P, 64)]
    outs = pe.prime([7, 3, 5], prompts)
    assert resets == [[7, 3, 5]]
    assert calls == [([7, 3], 2), ([5], 1), ([7, 5], 2), ([7], 1)]
    assert [o.shape[0] for o in outs] == [3, 1, 2]
    assert outs[0][:, 0].tolist() == [1.0, 3.0, 4.0]
    with pytest.raises(ValueError, match="divisible"):
        pe.prime([1], [torch.zeros(P + 1, 64)])


def test_install_decode_attention_routes_only_decode_steps():
    from nanovllm_dots_b200.llm_attention import install_decode_attention

    class _Mod:
        num_heads, head_dim, num_kv_heads, is_causal = 4, 8, 2, True
        k_cache = torch.zeros(2, 16, 2, 8)
        v_cache = torch.zeros(2, 16, 2, 8)

        def forward(self, q, k, v):
            return "flash"

    seen = []

    class _Dec:
        def decode(self, q, k, v, kc, vc, slot, cl, bt):
            seen.append((tuple(q.shape), tuple(k.shape), slot, cl, bt))
            return "b200"

    ctx = SimpleNamespace(is_prefill=True, slot_mapping="s", context_lens="c", block_tables="b")
    m = _Mod()
    install_decode_attention(m, lambda: ctx, _Dec())
    q, k = torch.zeros(3, 32), torch.zeros(3, 16)
    assert m.forward(q, k, k) == "flash"            # prefill keeps the original path
    ctx.is_prefill = False
    assert m.forward(q, k, k) == "b200"
    assert seen == [((3, 4, 8), (3, 2, 8), "s", "c", "b")]
    m.is_causal = False
    assert m.forward(q, k, k) == "flash"
