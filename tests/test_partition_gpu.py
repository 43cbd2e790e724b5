"""GPU parity of the multi-GPU partitions, with the ranks emulated one after another on
one GPU (every rank's share runs through the same kernels a rank would launch):

* paged decode split by kv head (``KVHeadPartition`` + ``decode_paged_partitioned``):
  the ranks' head slices, put together, against the fp32 oracle;
* prefill split by kv head (``prefill_partitioned``) and by LPT blocks
  (``prefill_unit_blocks`` + ``prefill_blocks``): bit-identical to the single call
  (each (batch, head) row is computed the same way in either), and against the oracle;
* sparse-token paged decode and MagicPIG split along the key axis (``PagedKeyShard``,
  ``sparse_paged_partial``, ``lse_merge_into``): against the oracle and the single call.

Tolerance: max-abs <= 2e-3 against the fp32 oracle on the same inputs, no NaNs.
"""
import pytest
import torch

from oracle import naive as N

from attention_kernel_triton_b200 import _lib
from attention_kernel_triton_b200 import workloads as W
from attention_kernel_triton_b200.decode_flash_attention_redundant_var_len_paged import flash_attention_decode_paged
from attention_kernel_triton_b200.distributed import (KVHeadPartition, PagedKeyShard, decode_paged_partitioned,
                                                      lse_merge_into, prefill_blocks, prefill_partitioned,
                                                      prefill_unit_blocks)
from attention_kernel_triton_b200.magicpig_sparsetoken_decode_flash_attention_redundant_var_len_paged_with_norm import (
    magicpig_sparsetoken_flash_attention_decode_paged)
from attention_kernel_triton_b200.prefill_flash_attention import flash_attention_prefill
from attention_kernel_triton_b200.prefill_flash_attention_var_len_padding import (
    flash_attention_prefill as flash_attention_prefill_varlen)
from attention_kernel_triton_b200.sparsetoken_decode_flash_attention_redundant_var_len_paged import (
    sparse_paged_partial, sparsetoken_flash_attention_decode_paged)

pytestmark = pytest.mark.gpu
TOL = 2e-3
DEV = "cuda"


@pytest.fixture(autouse=True)
def device_status_clean():
    _lib.device_status(0, clear=True)
    yield
    assert _lib.device_status(0) == 0, "a kernel recorded an error"


def maxerr(a, b):
    return (a.float().cpu() - b.float().cpu()).abs().max().item()


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_paged_decode_kv_head_partition(world):
    c = W.make_paged(B=6, Hq=32, Hkv=8, D=128, page_size=16, min_len=1, max_len=9000, seed=90 + world, device=DEV)
    parts = [KVHeadPartition(8, 4, world, r) for r in range(world)]
    outs = [decode_paged_partitioned(c.q, p.local_paged_cache(c.cache), c.indptr, c.indices, c.last_page_len, p)
            for p in parts]
    O = torch.cat(outs, dim=1)
    assert O.shape == (6, 32, 128) and not torch.isnan(O).any()
    ref = N.naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.last_page_len)
    assert maxerr(O, ref) <= TOL
    single = flash_attention_decode_paged(c.q, c.cache, c.indptr, c.indices, c.last_page_len)
    assert maxerr(O, single) <= TOL


def test_paged_decode_kv_head_partition_writes_into_a_slice_of_the_output():
    c = W.make_paged(B=3, Hq=32, Hkv=8, D=128, page_size=16, min_len=100, max_len=3000, seed=95, device=DEV)
    out = torch.full((3, 32, 128), float("nan"), dtype=torch.float16, device=DEV)
    for r in range(4):
        p = KVHeadPartition(8, 4, 4, r)
        decode_paged_partitioned(c.q, p.local_paged_cache(c.cache), c.indptr, c.indices, c.last_page_len, p,
                                 out=p.q_heads(out))
    ref = N.naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.last_page_len)
    assert not torch.isnan(out).any() and maxerr(out, ref) <= TOL


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("varlen", [False, True])
def test_prefill_kv_head_partition_is_bit_identical(world, varlen):
    f = W.make_prefill(B=2, Hq=32, Hkv=8, S=640, D=64, causal=True, seed=96, device=DEV, varlen=varlen)
    vl = f.varlen if varlen else None
    if varlen:
        single = flash_attention_prefill_varlen(f.Q, f.K, f.V, True, f.softmax_scale, f.group, f.varlen)
    else:
        single = flash_attention_prefill(f.Q, f.K, f.V, True, f.softmax_scale, f.group)
    outs = [prefill_partitioned(f.Q, f.K, f.V, True, f.softmax_scale, f.group, KVHeadPartition(8, f.group, world, r),
                                varlen=vl) for r in range(world)]
    O = torch.cat(outs, dim=1)
    assert torch.equal(O, single)
    # one sampled head against the oracle (the full oracle is covered by the prefill tests)
    b, h = 1, 13
    ref = N.prefill_reference(f.Q[b:b + 1, h:h + 1].cpu(), f.K[b:b + 1, h // 4:h // 4 + 1].cpu(),
                              f.V[b:b + 1, h // 4:h // 4 + 1].cpu(), True, f.softmax_scale, 1)
    n = int(f.varlen[b]) if varlen else 640
    assert maxerr(O[b:b + 1, h:h + 1, :n], ref[:, :, :n]) <= TOL


@pytest.mark.parametrize("Hkv,world", [(2, 4), (3, 2)])
def test_prefill_lpt_blocks_are_bit_identical(Hkv, world):
    f = W.make_prefill(B=4, Hq=2 * Hkv, Hkv=Hkv, S=512, D=64, causal=True, seed=97, device=DEV, varlen=True)
    single = flash_attention_prefill_varlen(f.Q, f.K, f.V, True, f.softmax_scale, f.group, f.varlen)
    O = torch.full_like(single, float("nan"))
    lens = f.varlen.tolist()
    for r in range(world):
        blocks = prefill_unit_blocks(lens, Hkv, world, r)
        for (b, h0, h1), Ob in prefill_blocks(f.Q, f.K, f.V, True, f.softmax_scale, f.group, blocks, f.varlen):
            O[b:b + 1, h0 * f.group:h1 * f.group] = Ob
    assert torch.equal(O, single)


def _paged_split(c, world, magic):
    B, Hq, _, D = c.q.shape
    rows = B * Hq
    recv = torch.empty((world, rows * D + rows), dtype=torch.float32, device=DEV)
    for r in range(world):
        sh = PagedKeyShard(c.cache, c.indptr, c.indices, world, r, compact=(r % 2 == 0))
        ind, nnz = sh.lists(c.sparse_ind, c.sparse_nnz)
        sparse_paged_partial(recv[r, : rows * D].view(B, Hq, D), recv[r, rows * D:].view(B, Hq), c.q, sh.cache,
                             sh.indptr, sh.indices, ind, nnz, K=c.K if magic else None, L=c.L if magic else None)
    out = torch.empty((B, Hq, D), dtype=c.q.dtype, device=DEV)
    lse_merge_into(out, recv, rows, D)
    return out


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("magic", [False, True])
def test_sparse_paged_key_split(world, magic):
    c = W.make_sparse_paged(B=3, Hq=32, Hkv=8, D=256, page_size=16, lens=[8192, 20000, 777], keep_p=0.02,
                            seed=98, device=DEV, magicpig=True)
    out = _paged_split(c, world, magic)
    assert not torch.isnan(out).any()
    if magic:
        ref = N.magicpig_sparsetoken_naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.sparse_ind,
                                                           c.sparse_nnz, c.K, c.L)
        single = magicpig_sparsetoken_flash_attention_decode_paged(c.q, c.cache, c.indptr, c.indices, c.sparse_ind,
                                                                   c.sparse_nnz, c.K, c.L)
    else:
        ref = N.sparsetoken_naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.sparse_ind, c.sparse_nnz)
        single = sparsetoken_flash_attention_decode_paged(c.q, c.cache, c.indptr, c.indices, c.sparse_ind,
                                                          c.sparse_nnz)
    assert maxerr(out, ref) <= TOL
    assert maxerr(out, single) <= TOL


def test_sparse_paged_partial_of_an_empty_shard_is_minus_infinity():
    c = W.make_sparse_paged(B=1, Hq=8, Hkv=2, D=128, page_size=16, lens=[256], keep_p=0.05, seed=99, device=DEV)
    ind = torch.full_like(c.sparse_ind, -1)
    nnz = torch.zeros_like(c.sparse_nnz)
    o = torch.full((1, 8, 128), float("nan"), device=DEV)
    lse = torch.zeros((1, 8), device=DEV)
    sparse_paged_partial(o, lse, c.q, c.cache, c.indptr, c.indices, ind, nnz)
    assert torch.all(o == 0) and torch.all(torch.isinf(lse) & (lse < 0))
