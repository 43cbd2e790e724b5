"""GPU parity of the sparse-token decode paths (dense KV, paged KV, MagicPIG)
against the CPU oracle and the reference's golden outputs.

Tolerance: max-abs <= 2e-3 against the fp32 oracle, no NaNs (bf16 adds half a
bf16 ulp of the reference value).  Index handling is checked bit-exactly with
known-answer cases: a head that keeps one token must output exactly that
token's V row, and with q = 0 two kept tokens give exactly their mean.
"""
import math

import pytest
import torch

from golden_io import load
from oracle import naive as N

from attention_kernel_triton_b200 import _lib
from attention_kernel_triton_b200 import workloads as W
from attention_kernel_triton_b200.magicpig_sparsetoken_decode_flash_attention_redundant_var_len_paged_with_norm import (
    magicpig_sparsetoken_flash_attention_decode_paged)
from attention_kernel_triton_b200.sparsetoken_decode_flash_attention_redundant import (
    sparsetoken_flash_attention_decode)
from attention_kernel_triton_b200.sparsetoken_decode_flash_attention_redundant_var_len_paged import (
    sparsetoken_flash_attention_decode_paged)

pytestmark = pytest.mark.gpu
TOL = 2e-3
DEV = "cuda"


def check_close(out, ref, dtype=torch.float16):
    out = out.detach().float().cpu()
    ref = ref.detach().float().cpu()
    assert out.shape == ref.shape
    assert not torch.isnan(out).any()
    err = (out - ref).abs()
    bound = TOL + (2.0 ** -8 * ref.abs() if dtype == torch.bfloat16 else 0.0)
    assert bool((err <= bound).all()), f"max err {err.max().item()}"


@pytest.fixture(autouse=True)
def device_status_clean():
    _lib.device_status(0, clear=True)
    yield
    assert _lib.device_status(0) == 0, "a kernel recorded an error"


def cuda(x):
    return x.to(DEV)


# ---------------------------------------------------------------- golden
def test_sparse_dense_matches_reference_golden():
    f = load("sparse_dense")
    O = sparsetoken_flash_attention_decode(cuda(f["q"]), cuda(f["K"]), cuda(f["V"]), cuda(f["sparse_ind"]),
                                           cuda(f["sparse_nnz"]), f["softmax_scale"], f["group"])
    assert O.shape == f["O"].shape
    check_close(O, f["O"])
    check_close(O, f["O_by_mask"])


@pytest.mark.parametrize("name", ["sparse_paged", "sparse_paged_perhead"])
def test_sparse_paged_matches_reference_golden(name):
    f = load(name)
    O = sparsetoken_flash_attention_decode_paged(cuda(f["q"]), cuda(f["cache"]), cuda(f["indptr"]),
                                                 cuda(f["indices"]), cuda(f["sparse_ind"]), cuda(f["sparse_nnz"]))
    assert O.shape == f["O"].shape
    check_close(O, f["O"])


def test_magicpig_matches_reference_golden():
    f = load("magicpig_paged")
    O = magicpig_sparsetoken_flash_attention_decode_paged(cuda(f["q"]), cuda(f["cache"]), cuda(f["indptr"]),
                                                          cuda(f["indices"]), cuda(f["sparse_ind"]),
                                                          cuda(f["sparse_nnz"]), cuda(f["K"]), cuda(f["L"]))
    assert O.shape == f["O"].shape and O.dtype == torch.float16
    check_close(O, f["O"])


# ---------------------------------------------------------------- cfg4 shapes (32000-token dense and 8K-32K paged, keep 2%)
def test_sparse_dense_cfg4():
    c = W.make_sparse_dense(seed=41)  # q [1,32,1,128], K/V [1,8,32000,128], keep 2% per kv head
    O = sparsetoken_flash_attention_decode(cuda(c.q), cuda(c.K), cuda(c.V), cuda(c.sparse_ind),
                                           cuda(c.sparse_nnz), c.softmax_scale, c.group)
    check_close(O, N.sparsetoken_naive_decode(c.q, c.K, c.V, c.sparse_ind, c.sparse_nnz, c.softmax_scale, c.group))


def test_sparse_paged_cfg4():
    c = W.make_sparse_paged(seed=42)  # B=3 Hq=32 Hkv=8 D=256 P=16 lens U[8K,32K]
    O = sparsetoken_flash_attention_decode_paged(cuda(c.q), cuda(c.cache), cuda(c.indptr), cuda(c.indices),
                                                 cuda(c.sparse_ind), cuda(c.sparse_nnz))
    check_close(O, N.sparsetoken_naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.sparse_ind,
                                                       c.sparse_nnz))


def test_magicpig_cfg4():
    c = W.make_sparse_paged(seed=43, magicpig=True)
    O = magicpig_sparsetoken_flash_attention_decode_paged(cuda(c.q), cuda(c.cache), cuda(c.indptr), cuda(c.indices),
                                                          cuda(c.sparse_ind), cuda(c.sparse_nnz), cuda(c.K),
                                                          cuda(c.L))
    check_close(O, N.magicpig_sparsetoken_naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.sparse_ind,
                                                                c.sparse_nnz, c.K, c.L))


def test_magicpig_reference_test_shape_keep_4_percent():
    # the reference driver also runs kept_ratio 0.04 (MP:401), page size 256
    c = W.make_sparse_paged(B=3, Hq=32, Hkv=8, D=256, page_size=256, lens=[2000, 3000, 1500], keep_p=0.04,
                            seed=44, magicpig=True, per_qo_head=True)
    O = magicpig_sparsetoken_flash_attention_decode_paged(cuda(c.q), cuda(c.cache), cuda(c.indptr), cuda(c.indices),
                                                          cuda(c.sparse_ind), cuda(c.sparse_nnz), cuda(c.K),
                                                          cuda(c.L))
    check_close(O, N.magicpig_sparsetoken_naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.sparse_ind,
                                                                c.sparse_nnz, c.K, c.L))


# ---------------------------------------------------------------- shapes / packing
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("D,G", [(64, 1), (64, 8), (128, 2), (128, 4), (256, 4), (128, 16)])
@pytest.mark.parametrize("per_qo_head", [False, True])
def test_sparse_paged_shapes(dtype, D, G, per_qo_head):
    Hkv = 2
    c = W.make_sparse_paged(B=3, Hq=Hkv * G, Hkv=Hkv, D=D, page_size=16, lens=[1, 200, 1500], keep_p=0.1,
                            seed=D + G, dtype=dtype, per_qo_head=per_qo_head)
    O = sparsetoken_flash_attention_decode_paged(cuda(c.q), cuda(c.cache), cuda(c.indptr), cuda(c.indices),
                                                 cuda(c.sparse_ind), cuda(c.sparse_nnz))
    ref = N.sparsetoken_naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.sparse_ind, c.sparse_nnz)
    check_close(O, ref, dtype)
    c2 = W.make_sparse_paged(B=3, Hq=Hkv * G, Hkv=Hkv, D=D, page_size=16, lens=[1, 200, 1500], keep_p=0.1,
                             seed=D + G, dtype=dtype, per_qo_head=per_qo_head, magicpig=True)
    O = magicpig_sparsetoken_flash_attention_decode_paged(cuda(c2.q), cuda(c2.cache), cuda(c2.indptr),
                                                          cuda(c2.indices), cuda(c2.sparse_ind),
                                                          cuda(c2.sparse_nnz), cuda(c2.K), cuda(c2.L))
    ref = N.magicpig_sparsetoken_naive_paged_attention(c2.q, c2.cache, c2.indptr, c2.indices, c2.sparse_ind,
                                                       c2.sparse_nnz, c2.K, c2.L)
    check_close(O, ref, dtype)


@pytest.mark.parametrize("D,G", [(64, 4), (128, 1), (256, 2)])
def test_sparse_dense_shapes(D, G):
    c = W.make_sparse_dense(B=2, Hq=2 * G, Hkv=2, L=3000, D=D, keep_p=0.05, seed=7 * D + G)
    O = sparsetoken_flash_attention_decode(cuda(c.q), cuda(c.K), cuda(c.V), cuda(c.sparse_ind),
                                           cuda(c.sparse_nnz), c.softmax_scale, c.group)
    check_close(O, N.sparsetoken_naive_decode(c.q, c.K, c.V, c.sparse_ind, c.sparse_nnz, c.softmax_scale, c.group))


def test_mixed_group_lists_partially_equal():
    # heads 0..2 of the group share a list, head 3 differs: the item falls back to per-head gathers
    c = W.make_sparse_paged(B=2, Hq=8, Hkv=2, D=128, page_size=16, lens=[500, 900], keep_p=0.1, seed=5)
    ind = c.sparse_ind.clone()
    nnz = c.sparse_nnz.clone()
    ind[:, 3, :5] = torch.tensor([0, 2, 4, 6, 8], dtype=torch.int32)
    nnz[:, 3, 0] = 5
    O = sparsetoken_flash_attention_decode_paged(cuda(c.q), cuda(c.cache), cuda(c.indptr), cuda(c.indices),
                                                 cuda(ind), cuda(nnz))
    check_close(O, N.sparsetoken_naive_paged_attention(c.q, c.cache, c.indptr, c.indices, ind, nnz))


# ---------------------------------------------------------------- edge cases and known answers
def test_nnz_zero_gives_zeros_and_full_lists():
    c = W.make_sparse_paged(B=2, Hq=8, Hkv=2, D=64, page_size=16, lens=[100, 64], keep_p=0.2, seed=9)
    ind = c.sparse_ind.clone()
    nnz = c.sparse_nnz.clone()
    nnz[0, 1, 0] = 0                      # one head empty
    nnz[1, 4:8, 0] = 0                    # a whole kv group empty
    ind[0, 0, :] = -1
    ind[0, 0, :64] = torch.arange(64, dtype=torch.int32)
    nnz[0, 0, 0] = 64                     # every token of the first 64
    O = sparsetoken_flash_attention_decode_paged(cuda(c.q), cuda(c.cache), cuda(c.indptr), cuda(c.indices),
                                                 cuda(ind), cuda(nnz))
    ref = N.sparsetoken_naive_paged_attention(c.q, c.cache, c.indptr, c.indices, ind, nnz)
    check_close(O, ref)
    assert torch.all(O[0, 1] == 0) and torch.all(O[1, 4:8] == 0)
    Om = magicpig_sparsetoken_flash_attention_decode_paged(cuda(c.q), cuda(c.cache), cuda(c.indptr),
                                                           cuda(c.indices), cuda(ind), cuda(nnz),
                                                           torch.full((2, 8), 2.0, device=DEV),
                                                           torch.full((2, 8), 3.0, device=DEV))
    assert torch.all(Om[0, 1] == 0) and not torch.isnan(Om).any()


@pytest.mark.parametrize("paged", [False, True])
def test_single_kept_token_returns_its_v_row_exactly(paged):
    g = torch.Generator().manual_seed(17)
    B, Hq, Hkv, D, P = 2, 8, 2, 128, 16
    if paged:
        c = W.make_sparse_paged(B=B, Hq=Hq, Hkv=Hkv, D=D, page_size=P, lens=[77, 300], keep_p=0.1, seed=17)
        seq = [77, 300]
    else:
        c = W.make_sparse_dense(B=B, Hq=Hq, Hkv=Hkv, L=300, D=D, keep_p=0.1, seed=17)
        seq = [300, 300]
    ind = torch.full((B, Hq, 4), -1, dtype=torch.int32)
    nnz = torch.ones((B, Hq, 1), dtype=torch.int32)
    for b in range(B):
        for h in range(Hq):
            ind[b, h, 0] = int(torch.randint(0, seq[b], (1,), generator=g))
    ind[0, 0, 0] = 0
    ind[1, 1, 0] = seq[1] - 1  # last token (the reference's -1 padding must not be read as it)
    if paged:
        O = sparsetoken_flash_attention_decode_paged(cuda(c.q), cuda(c.cache), cuda(c.indptr), cuda(c.indices),
                                                     cuda(ind), cuda(nnz))
        ref = N.sparsetoken_naive_paged_attention(c.q, c.cache, c.indptr, c.indices, ind, nnz).half()
    else:
        O = sparsetoken_flash_attention_decode(cuda(c.q), cuda(c.K), cuda(c.V), cuda(ind), cuda(nnz),
                                               c.softmax_scale, c.group)[:, :, 0]
        ref = N.sparsetoken_naive_decode(c.q, c.K, c.V, ind, nnz, c.softmax_scale, c.group)[:, :, 0].half()
    assert torch.equal(O.cpu(), ref)


def test_q_zero_two_tokens_give_exact_mean():
    c = W.make_sparse_paged(B=1, Hq=4, Hkv=1, D=64, page_size=16, lens=[200], keep_p=0.1, seed=21)
    q = torch.zeros_like(c.q)
    ind = torch.tensor([[[3, 150, -1], [0, 199, -1], [16, 17, -1], [5, 6, -1]]], dtype=torch.int32)
    nnz = torch.full((1, 4, 1), 2, dtype=torch.int32)
    O = sparsetoken_flash_attention_decode_paged(cuda(q), cuda(c.cache), cuda(c.indptr), cuda(c.indices),
                                                 cuda(ind), cuda(nnz))
    ref = N.sparsetoken_naive_paged_attention(q, c.cache, c.indptr, c.indices, ind, nnz).half()
    assert torch.equal(O.cpu(), ref)
    # MagicPIG with q = 0: cos = 0 for every token, so u and the weights are uniform too
    Om = magicpig_sparsetoken_flash_attention_decode_paged(cuda(q), cuda(c.cache), cuda(c.indptr), cuda(c.indices),
                                                           cuda(ind), cuda(nnz), torch.full((1, 4), 3.0, device=DEV),
                                                           torch.full((1, 4), 2.5, device=DEV))
    assert torch.equal(Om.cpu(), ref)


def test_out_of_range_token_is_reported_not_faulted():
    c = W.make_sparse_paged(B=2, Hq=4, Hkv=2, D=64, page_size=16, lens=[40, 40], keep_p=0.3, seed=23)
    ind = c.sparse_ind.clone()
    ind[0, 0, 0] = 48  # past sequence 0's three pages
    O = sparsetoken_flash_attention_decode_paged(cuda(c.q), cuda(c.cache), cuda(c.indptr), cuda(c.indices),
                                                 cuda(ind), cuda(c.sparse_nnz))
    torch.cuda.synchronize()
    assert _lib.device_status(0, clear=True) == 3
    ref = N.sparsetoken_naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.sparse_ind, c.sparse_nnz)
    check_close(O[1], ref[1])
    assert not torch.isnan(O).any()


def test_nnz_above_list_length_is_clamped_and_reported():
    c = W.make_sparse_dense(B=1, Hq=4, Hkv=1, L=100, D=64, keep_p=0.5, seed=25, L_max=8)
    nnz = c.sparse_nnz.clone()
    nnz[0, 2, 0] = 1000
    O = sparsetoken_flash_attention_decode(cuda(c.q), cuda(c.K), cuda(c.V), cuda(c.sparse_ind), cuda(nnz),
                                           c.softmax_scale, c.group)
    torch.cuda.synchronize()
    assert _lib.device_status(0, clear=True) == 3
    nnz[0, 2, 0] = 8
    check_close(O, N.sparsetoken_naive_decode(c.q, c.K, c.V, c.sparse_ind, nnz, c.softmax_scale, c.group))


def test_gqa_group_size_mismatch_asserts_like_the_reference():
    c = W.make_sparse_dense(B=1, Hq=8, Hkv=2, L=64, D=64, keep_p=0.5, seed=27)
    with pytest.raises(AssertionError):
        sparsetoken_flash_attention_decode(cuda(c.q), cuda(c.K), cuda(c.V), cuda(c.sparse_ind),
                                           cuda(c.sparse_nnz), c.softmax_scale, 2)
