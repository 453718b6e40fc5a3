"""The attention entry point that allocates nothing, against the one that
takes a workspace.

``dfm_paged_attention_noalloc`` is for callers that cannot allocate device
memory where they launch work (their allocator is owned by another thread or
framework, or their memory budget is fixed).  It keeps its scratch in one
array inside the library, so these tests check that it gives the same result
as ``dfm_paged_attention`` on two calls in a row (the shared array is reused
and must be cleared properly between calls), and that a call too large for the
array is refused before anything runs.  This file sorts last so a run that
stops at the first failure has run every other test first.
"""
from __future__ import annotations

import ctypes
import math

import pytest
import torch

from conftest import cos_min
from nanovllm_dots_b200 import _lib

DEV = "cuda"


def test_noalloc_refuses_calls_beyond_its_scratch():
    L = _lib.lib()
    one = ctypes.c_void_p(1)   # never dereferenced: the size check comes first
    rc = L.dfm_paged_attention_noalloc(one, one, one, 10, 2, 16, 0, 1, one, one, one, 4000, 64,
                                       one, None)
    assert rc == 6
    assert b"scratch" in L.dfm_error_string(rc)


def test_noalloc_requires_an_error_word():
    """Device errors are reported only through the caller's error word, so a
    call without one is refused (nothing launches)."""
    L = _lib.lib()
    one = ctypes.c_void_p(1)   # never dereferenced: the argument check comes first
    rc = L.dfm_paged_attention_noalloc(one, one, one, 10, 2, 16, 0, 1, one, one, one, 4, 2,
                                       None, None)
    assert rc == 1


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point():
    heads, num_pages, max_pages, planes = 16, 1000, 330, 2
    # the long requests are split over work units and merged through the scratch
    lens = [(496, 17), (5000, 17), (2040, 17), (4110, 0), (0, 0)]
    g = torch.Generator(device=DEV).manual_seed(11)
    pool = torch.randn(planes, num_pages, heads, 16, 64, device=DEV, generator=g).to(torch.bfloat16)
    n = len(lens)
    perm = torch.randperm(num_pages, generator=torch.Generator().manual_seed(5)).tolist()
    bt = torch.full((n, max_pages), -1, dtype=torch.int32)
    cur = 0
    for i, (P, ne) in enumerate(lens):
        need = math.ceil((P + ne + 17) / 16)
        bt[i, :need] = torch.tensor(perm[cur:cur + need])
        cur += need
    q = torch.randn(n * 34, heads * 64, device=DEV, generator=g).to(torch.bfloat16)
    cl = torch.tensor([a for a, _ in lens], dtype=torch.int32, device=DEV)
    ne = torch.tensor([b for _, b in lens], dtype=torch.int32, device=DEV)
    btd = bt.to(DEV)
    L = _lib.lib()
    stream = _lib.c_void_p(torch.cuda.current_stream().cuda_stream)

    wsb = L.dfm_attention_workspace_size(n, max_pages, heads)
    assert wsb <= 8 << 20
    ws = torch.zeros(wsb, dtype=torch.uint8, device=DEV)
    ref = torch.zeros_like(q)
    _lib.check(L.dfm_paged_attention(q.data_ptr(), ref.data_ptr(), pool.data_ptr(), num_pages,
                                     planes, heads, 0, 1, cl.data_ptr(), ne.data_ptr(),
                                     btd.data_ptr(), max_pages, n, ws.data_ptr(), wsb, stream),
               "dfm_paged_attention")
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    for call in range(2):
        out = torch.full_like(q, float("nan"))
        _lib.check(L.dfm_paged_attention_noalloc(q.data_ptr(), out.data_ptr(), pool.data_ptr(),
                                                 num_pages, planes, heads, 0, 1, cl.data_ptr(),
                                                 ne.data_ptr(), btd.data_ptr(), max_pages, n,
                                                 err.data_ptr(), stream),
                   "dfm_paged_attention_noalloc")
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.isfinite(out.float()).all(), f"call {call}"
        assert (out.float() - ref.float()).abs().max().item() < 2e-2, f"call {call}"
        assert cos_min(out, ref, 64) > 0.9999, f"call {call}"


@pytest.mark.gpu
def test_noalloc_reports_a_bad_block_id_through_the_error_word():
    """A block-table entry outside the pool is reported in the caller's error
    word (the kernel skips the page and reads zeros), and the next good call
    on the shared scratch is unaffected."""
    heads, num_pages, max_pages, planes = 16, 64, 8, 2
    g = torch.Generator(device=DEV).manual_seed(3)
    pool = torch.randn(planes, num_pages, heads, 16, 64, device=DEV, generator=g).to(torch.bfloat16)
    n = 2
    bt = torch.tensor([[0, 1, 2, 3, -1, -1, -1, -1], [4, 5, 10 ** 6, 7, -1, -1, -1, -1]],
                      dtype=torch.int32, device=DEV)
    cl = torch.tensor([30, 30], dtype=torch.int32, device=DEV)
    ne = torch.tensor([17, 17], dtype=torch.int32, device=DEV)
    q = torch.randn(n * 34, heads * 64, device=DEV, generator=g).to(torch.bfloat16)
    L = _lib.lib()
    stream = _lib.c_void_p(torch.cuda.current_stream().cuda_stream)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.empty_like(q)
    _lib.check(L.dfm_paged_attention_noalloc(q.data_ptr(), out.data_ptr(), pool.data_ptr(),
                                             num_pages, planes, heads, 0, 1, cl.data_ptr(),
                                             ne.data_ptr(), bt.data_ptr(), max_pages, n,
                                             err.data_ptr(), stream),
               "dfm_paged_attention_noalloc")
    torch.cuda.synchronize()
    assert int(err.item()) & _lib.DEVERR_PAGE
    # the same call with a valid table: no error, and the result equals the
    # workspace entry point's
    bt[1, 2] = 6
    err.zero_()
    _lib.check(L.dfm_paged_attention_noalloc(q.data_ptr(), out.data_ptr(), pool.data_ptr(),
                                             num_pages, planes, heads, 0, 1, cl.data_ptr(),
                                             ne.data_ptr(), bt.data_ptr(), max_pages, n,
                                             err.data_ptr(), stream),
               "dfm_paged_attention_noalloc")
    wsb = L.dfm_attention_workspace_size(n, max_pages, heads)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=DEV)
    ref = torch.empty_like(q)
    _lib.check(L.dfm_paged_attention(q.data_ptr(), ref.data_ptr(), pool.data_ptr(), num_pages,
                                     planes, heads, 0, 1, cl.data_ptr(), ne.data_ptr(),
                                     bt.data_ptr(), max_pages, n, ws.data_ptr(), wsb, stream),
               "dfm_paged_attention")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(out, ref)
