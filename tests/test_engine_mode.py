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


# --------------------------------------------------------------------------- #
# Post-FM with one host synchronisation per tick                               #
# --------------------------------------------------------------------------- #
class _Seq:
    def __init__(self, payload):
        self.custom_payload = payload
        self.tokens = []
        self.stoped = False

    def append_token(self, tok):
        self.tokens.append(tok)


def _engine_and_seqs(n, seed):
    """A stand-in engine with the attributes the reference's post-FM step reads
    (``engine.py:743-778``): core.eos_proj / io_helper, dots._append_history_chunk,
    the batched patch encoder and its free rows."""
    g = torch.Generator().manual_seed(seed)
    lin = torch.nn.Linear(8, 2)
    core = SimpleNamespace(eos_proj=lin,
                           io_helper=SimpleNamespace(denormalize=lambda x: x * 2.0 + 1.0))
    hist = []
    dots = SimpleNamespace(_append_history_chunk=lambda st, chunk: hist.append((id(st), chunk)))

    class _PE:
        def __init__(self):
            self.reset = []

        def reset_rows(self, rows):
            self.reset.extend(rows.tolist())

        def decode_patch(self, patches, rows):
            return patches.reshape(patches.shape[0], 1, -1)[:, :, :4] + rows.view(-1, 1, 1).float()

    eng = SimpleNamespace(core=core, dots=dots, flash_pe=True, _flash_pe=_PE(), _pe_free=[5, 6, 7],
                          _pe_max_batch=3)
    seqs = []
    for i in range(n):
        st = SimpleNamespace(llm_hiddens=torch.randn(1, 1, 8, generator=g), end_flag=(i == 2))
        p = SimpleNamespace(gen_state=st, pe_row=(1 if i == 0 else None), next_embed=None, latents=[],
                            patches_emitted=0, position=3, schedule=torch.zeros(1, 5 if i != 1 else 4),
                            span_count=10, max_patches=None, eos_threshold=0.5)
        seqs.append(_Seq(p))
    latents = torch.randn(n, syn.BASE.latent_patch, syn.BASE.latent_dim, generator=g)
    return eng, seqs, latents, hist


def test_batched_finish_matches_the_per_request_post_fm_step():
    from nanovllm_dots_b200.engine_mode import BatchedFinish
    eng, seqs, latents, hist = _engine_and_seqs(4, 3)
    fin = BatchedFinish(eng)
    stops = [fin.deferred_stop(s.custom_payload.gen_state, eos_threshold=0.5) for s in seqs]
    # the per-request reference rule (model.py:197-201): end flag, else eos prob > threshold
    want_eos = []
    for s in seqs:
        st = s.custom_payload.gen_state
        prob = eng.core.eos_proj(st.llm_hiddens).softmax(dim=-1)[:, -1, 1]
        want_eos.append(st.end_flag or bool((prob > 0.5).item()))
    assert [bool(x) for x in stops] == want_eos
    fin(seqs, latents, stops)
    assert len(hist) == 4                                   # every patch appended to its history
    assert eng._flash_pe.reset == [7, 6, 5]                # rows claimed in order, one call
    for i, s in enumerate(seqs):
        p = s.custom_payload
        want = latents[i:i + 1] * 2.0 + 1.0                 # denormalised patch (engine.py:761)
        assert torch.equal(p.latents[0], want)
        assert s.tokens == [want.reshape(-1).numpy().tobytes()]
        assert p.patches_emitted == 1 and p.position == 4
        assert p.next_embed is not None
        # stop rule (engine.py:772-774): eos/end flag, schedule exhausted (seq 1), or cap
        assert s.stoped == (want_eos[i] or i == 1)
