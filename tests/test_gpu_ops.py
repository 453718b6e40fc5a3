"""Building-block kernels through the C ABI against plain fp32 torch references:
the tcgen05 GEMM (``dfm_linear``) and the paged prefix attention
(``dfm_paged_attention``)."""
from __future__ import annotations

import math

import pytest
import torch

from conftest import cos_min
from nanovllm_dots_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _linear(a, w, bias=None, out_f32=True, gelu=False):
    M, K = a.shape
    N = w.shape[0]
    out = torch.empty(M, N, device=DEV, dtype=torch.float32 if out_f32 else torch.bfloat16)
    rc = _lib.lib().dfm_linear(a.data_ptr(), a.stride(0), M, K, w.data_ptr(), w.stride(0), N,
                               None if bias is None else bias.data_ptr(), out.data_ptr(),
                               int(out_f32), int(gelu),
                               _lib.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "dfm_linear")
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("M,K,N", [(1, 64, 64), (100, 1024, 1024), (128, 64, 1024),
                                   (300, 1024, 3072), (257, 4096, 1024), (129, 1536, 1024),
                                   (2176, 1024, 4096), (1024, 1024, 64), (256, 1024, 75776)])
def test_linear_fp32_out(M, K, N):
    g = torch.Generator(device=DEV).manual_seed(M * 7 + N)
    a = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=DEV, generator=g) / math.sqrt(K)).to(torch.bfloat16)
    b = torch.randn(N, device=DEV, generator=g)
    out = _linear(a, w, b)
    ref = a.float() @ w.float().t() + b
    err = (out - ref).abs().max().item()
    assert err < 2e-3 * max(1.0, ref.abs().max().item()), err


def test_linear_bf16_gelu_and_no_bias():
    g = torch.Generator(device=DEV).manual_seed(5)
    a = torch.randn(333, 1024, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(4096, 1024, device=DEV, generator=g) / 32).to(torch.bfloat16)
    b = torch.randn(4096, device=DEV, generator=g)
    out = _linear(a, w, b, out_f32=False, gelu=True).float()
    ref = torch.nn.functional.gelu(a.float() @ w.float().t() + b, approximate="tanh")
    assert (out - ref).abs().max().item() < 3e-2
    out2 = _linear(a, w, None, out_f32=True)
    assert (out2 - a.float() @ w.float().t()).abs().max().item() < 2e-3 * 4


def test_linear_strided_operand():
    g = torch.Generator(device=DEV).manual_seed(9)
    big = torch.randn(200, 1536, device=DEV, generator=g).to(torch.bfloat16)
    a = big[:, :1024]
    w = (torch.randn(1024, 1024, device=DEV, generator=g) / 32).to(torch.bfloat16)
    out = _linear(a, w)
    assert (out - a.float() @ w.float().t()).abs().max().item() < 5e-3


def test_linear_rejects_bad_shapes():
    L = _lib.lib()
    a = torch.zeros(4, 96, device=DEV, dtype=torch.bfloat16)
    assert L.dfm_linear(a.data_ptr(), 96, 4, 96, a.data_ptr(), 96, 4, None, a.data_ptr(), 1, 0,
                        None) == 1


# ----------------------------------------------------------------------- attention
def _attn_reference(q, pool, heads, plane_k, plane_v, cache_len, n_ext, tables):
    """fp32 reference: per request, gather its pages, apply the FM prefix mask."""
    n = len(cache_len)
    out = torch.zeros(n * 34, heads * 64, device=DEV)
    for i in range(n):
        P, ne = cache_len[i], n_ext[i]
        T = P + ne + 17
        pages = tables[i][: math.ceil(T / 16)]
        K = pool[plane_k, pages].float()            # [np, heads, 16, 64]
        V = pool[plane_v, pages].float()
        K = K.permute(0, 2, 1, 3).reshape(-1, heads, 64)[:T]
        V = V.permute(0, 2, 1, 3).reshape(-1, heads, 64)[:T]
        qi = q[i * 34:(i + 1) * 34].float().view(34, heads, 64)
        s = torch.einsum("mhd,thd->hmt", qi, K) / 8.0
        lim = torch.full((34,), T, device=DEV)
        lim[:ne] = P + torch.arange(1, ne + 1, device=DEV)
        keep = torch.arange(T, device=DEV)[None] < lim[:, None]
        s = s.masked_fill(~keep[None], float("-inf"))
        o = torch.einsum("hmt,thd->mhd", torch.softmax(s, -1), V)
        out[i * 34:(i + 1) * 34] = o.reshape(34, heads * 64)
    return out


@pytest.mark.parametrize("lens,max_pages", [
    ([(0, 0), (0, 17), (5, 17), (40, 3)], 130),
    ([(496, 17), (511, 17), (1000, 0), (2040, 17), (17, 17)], 130),
    # requests longer than one 4096-key work unit: split keys + merge
    ([(5000, 17), (4110, 0), (100, 17), (4062, 17)], 330)])
def test_paged_attention_matches_reference(lens, max_pages):
    heads, num_pages, planes = 16, 1200, 4
    g = torch.Generator(device=DEV).manual_seed(len(lens))
    pool = torch.randn(planes, num_pages, heads, 16, 64, device=DEV, generator=g).to(torch.bfloat16)
    n = len(lens)
    cache_len = [a for a, _ in lens]
    n_ext = [b for _, b in lens]
    perm = torch.randperm(num_pages, generator=torch.Generator().manual_seed(3)).tolist()
    tables, cur = [], 0
    bt = torch.full((n, max_pages), -1, dtype=torch.int32)
    for i in range(n):
        need = math.ceil((cache_len[i] + n_ext[i] + 17) / 16)
        tables.append(perm[cur:cur + need])
        bt[i, :need] = torch.tensor(perm[cur:cur + need])
        cur += need
    q = torch.randn(n * 34, heads * 64, device=DEV, generator=g).to(torch.bfloat16)
    out = torch.zeros_like(q)
    L = _lib.lib()
    wsb = L.dfm_attention_workspace_size(n, max_pages, heads)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=DEV)
    cl = torch.tensor(cache_len, dtype=torch.int32, device=DEV)
    ne = torch.tensor(n_ext, dtype=torch.int32, device=DEV)
    btd = bt.to(DEV)
    for pk, pv in ((0, 1), (2, 3)):
        rc = L.dfm_paged_attention(q.data_ptr(), out.data_ptr(), pool.data_ptr(), num_pages, planes,
                                   heads, pk, pv, cl.data_ptr(), ne.data_ptr(), btd.data_ptr(),
                                   max_pages, n, ws.data_ptr(), wsb,
                                   _lib.c_void_p(torch.cuda.current_stream().cuda_stream))
        _lib.check(rc, "dfm_paged_attention")
        torch.cuda.synchronize()
        ref = _attn_reference(q, pool, heads, pk, pv, cache_len, n_ext, tables)
        assert (out.float() - ref).abs().max().item() < 2e-2
        assert cos_min(out, ref, 64) > 0.9999
    assert int(ws[:4].view(torch.int32).item()) == 0
