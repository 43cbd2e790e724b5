"""The public entry points under CUDA-graph capture: a serving loop captures a
decode step once and replays it with new inputs written into the same
buffers.  Nothing on these paths reads the device from the host, so every call
captures; a replay after new values are copied into the captured inputs must
give exactly the output of an eager call on those values (the kernels are
deterministic: no atomics in any accumulation), and match the oracle."""
import pytest
import torch

from oracle import naive as N

from attention_kernel_triton_b200 import _lib
from attention_kernel_triton_b200 import workloads as W
from attention_kernel_triton_b200.decode_flash_attention_redundant import flash_attention_decode
from attention_kernel_triton_b200.decode_flash_attention_redundant_var_len_paged import (
    flash_attention_decode_paged)
from attention_kernel_triton_b200.magicpig_sparsetoken_decode_flash_attention_redundant_var_len_paged_with_norm import (
    magicpig_sparsetoken_flash_attention_decode_paged)
from attention_kernel_triton_b200.prefill_flash_attention import flash_attention_prefill
from attention_kernel_triton_b200.sparsetoken_decode_flash_attention_redundant_var_len_paged import (
    sparsetoken_flash_attention_decode_paged)

pytestmark = pytest.mark.gpu
TOL = 2e-3
DEV = "cuda"


@pytest.fixture(autouse=True)
def device_status_clean():
    _lib.device_status(0, clear=True)
    yield
    assert _lib.device_status(0) == 0


def capture(fn):
    """Warm up on a side stream, then capture ``fn()`` into a graph; returns
    (graph, captured output)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn()
    return g, out


def check(out, ref):
    out = out.float().cpu()
    assert not torch.isnan(out).any()
    assert (out - ref).abs().max().item() <= TOL


def test_paged_decode_graph_replay_with_new_q():
    c = W.make_paged(Hq=32, Hkv=8, D=128, page_size=16, lens=[700, 33, 4096, 1], seed=61, device=DEV)
    g, out = capture(lambda: flash_attention_decode_paged(c.q, c.cache, c.indptr, c.indices, c.last_page_len))
    for step in range(3):
        c.q.copy_(torch.randn(c.q.shape, generator=torch.Generator(device=DEV).manual_seed(100 + step),
                              device=DEV, dtype=c.q.dtype))
        g.replay()
        eager = flash_attention_decode_paged(c.q, c.cache, c.indptr, c.indices, c.last_page_len)
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    check(out, N.naive_paged_attention(c.q.cpu(), c.cache.cpu(), c.indptr.cpu(), c.indices.cpu(),
                                       c.last_page_len.cpu()))


def test_dense_decode_graph_replay_with_new_kv():
    d = W.make_decode(B=2, Hq=16, Hkv=4, L=1500, D=64, seed=62, device=DEV)
    g, out = capture(lambda: flash_attention_decode(d.q, d.K, d.V, d.softmax_scale, d.group))
    d.K.mul_(-0.5)
    d.V.add_(0.25)
    g.replay()
    eager = flash_attention_decode(d.q, d.K, d.V, d.softmax_scale, d.group)
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    check(out, N.decode_reference(d.q.cpu(), d.K.cpu(), d.V.cpu(), d.softmax_scale, d.group))


def test_prefill_graph_replay_with_new_q():
    f = W.make_prefill(B=1, Hq=8, Hkv=2, S=384, D=64, causal=True, seed=63, device=DEV)
    g, out = capture(lambda: flash_attention_prefill(f.Q, f.K, f.V, True, f.softmax_scale, f.group))
    f.Q.copy_(torch.randn(f.Q.shape, generator=torch.Generator(device=DEV).manual_seed(7), device=DEV,
                          dtype=f.Q.dtype))
    g.replay()
    eager = flash_attention_prefill(f.Q, f.K, f.V, True, f.softmax_scale, f.group)
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    check(out, N.prefill_reference(f.Q.cpu(), f.K.cpu(), f.V.cpu(), True, f.softmax_scale, f.group))


@pytest.mark.parametrize("magicpig", [False, True])
def test_sparse_paged_graph_replay_with_new_lists(magicpig):
    kw = dict(B=2, Hq=8, Hkv=2, D=128, page_size=16, lens=[900, 257], keep_p=0.05, magicpig=magicpig)
    a = W.make_sparse_paged(seed=64, device=DEV, **kw)
    b = W.make_sparse_paged(seed=65, device=DEV, **kw)  # same shapes, other q, keep lists and counts
    if magicpig:
        fn = lambda: magicpig_sparsetoken_flash_attention_decode_paged(a.q, a.cache, a.indptr, a.indices,
                                                                          a.sparse_ind, a.sparse_nnz, a.K, a.L)
    else:
        fn = lambda: sparsetoken_flash_attention_decode_paged(a.q, a.cache, a.indptr, a.indices, a.sparse_ind,
                                                               a.sparse_nnz)
    g, out = capture(fn)
    assert a.sparse_ind.shape == b.sparse_ind.shape
    pairs = [(a.q, b.q), (a.sparse_ind, b.sparse_ind), (a.sparse_nnz, b.sparse_nnz)]
    if magicpig:
        pairs += [(a.K, b.K), (a.L, b.L)]
    for dst, src in pairs:
        dst.copy_(src)
    g.replay()
    eager = fn()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    args = (a.q.cpu(), a.cache.cpu(), a.indptr.cpu(), a.indices.cpu(), a.sparse_ind.cpu(), a.sparse_nnz.cpu())
    ref = (N.magicpig_sparsetoken_naive_paged_attention(*args, a.K.cpu(), a.L.cpu()) if magicpig
           else N.sparsetoken_naive_paged_attention(*args))
    check(out, ref)
