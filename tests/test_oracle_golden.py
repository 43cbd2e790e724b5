"""Pin the CPU oracle to outputs of the reference's own naive code.

The fixtures under tests/golden/ were produced by tests/golden/make_golden.py,
which runs the reference modules' naive functions on CPU.  Each oracle
function must reproduce them: within fp32 rounding where the reference ran in
fp32, within fp16 rounding where it ran in fp16 (its prefill and dense-decode
references round P to fp16, PF:424 / DR:311).
"""
import math

import pytest
import torch

from golden_io import load
from oracle import naive as N


def maxabs(a, b):
    return (a.double() - b.double()).abs().max().item()


@pytest.mark.parametrize("name", ["prefill_causal_gqa", "prefill_noncausal", "prefill_causal_d128"])
def test_prefill_oracle_matches_reference(name):
    f = load(name)
    O = N.prefill_reference(f["Q"], f["K"], f["V"], f["causal"], f["softmax_scale"], f["group"],
                            p_round=torch.float16)
    # the reference ran fp16 matmuls; the oracle's fp32 result rounded to fp16
    assert maxabs(O.half(), f["O"]) <= 2e-3
    strict = N.prefill_reference(f["Q"], f["K"], f["V"], f["causal"], f["softmax_scale"], f["group"])
    assert maxabs(strict, f["O"]) <= 2e-3
    assert not torch.isnan(strict).any()


def test_prefill_varlen_oracle_matches_reference():
    f = load("prefill_varlen")
    O = N.prefill_varlen_reference(f["Q"], f["K"], f["V"], True, f["softmax_scale"], f["group"],
                                   f["varlen"], p_round=torch.float16)
    assert maxabs(O.half(), f["O"]) <= 2e-3
    for b, l in enumerate(f["varlen"].tolist()):
        assert torch.all(O[b, :, l:] == 0)


@pytest.mark.parametrize("name", ["decode_dense", "decode_dense_d128"])
def test_decode_oracle_matches_reference(name):
    f = load(name)
    O = N.decode_reference(f["q"], f["K"], f["V"], f["softmax_scale"], f["group"], p_round=torch.float16)
    assert O.shape == f["O"].shape
    assert maxabs(O.half(), f["O"]) <= 2e-3


@pytest.mark.parametrize("name", ["paged_ref_table", "paged_p16"])
def test_paged_oracle_matches_reference(name):
    f = load(name)
    O = N.naive_paged_attention(f["q"], f["cache"], f["indptr"], f["indices"], f["last_page_len"])
    assert O.shape == f["O"].shape
    assert maxabs(O, f["O"]) <= 1e-5


def test_paged_oracle_batch_subset():
    f = load("paged_p16")
    O = N.naive_paged_attention(f["q"], f["cache"], f["indptr"], f["indices"], f["last_page_len"],
                                batches=[1, 3])
    assert maxabs(O[[1, 3]], f["O"][[1, 3]]) <= 1e-5
    assert torch.all(O[[0, 2]] == 0)


def test_sparse_dense_oracle_matches_reference():
    f = load("sparse_dense")
    O = N.sparsetoken_naive_decode(f["q"], f["K"], f["V"], f["sparse_ind"], f["sparse_nnz"],
                                   f["softmax_scale"], f["group"])
    assert O.shape == f["O"].shape
    assert maxabs(O, f["O"]) <= 1e-5
    # the reference's own cross-check: gather oracle == mask oracle (SD:315-328)
    mask = N.sparse_mask_from_lists(f["sparse_ind"], f["sparse_nnz"], f["K"].shape[2])
    assert torch.equal(mask, f["mask"])
    Om = N.sparsetoken_naive_decode_by_mask(f["q"], f["K"], f["V"], f["sparse_ind"], f["sparse_nnz"],
                                            f["softmax_scale"], f["group"], mask)
    assert maxabs(Om, f["O_by_mask"]) <= 1e-5
    assert maxabs(Om, O) <= 1e-5


@pytest.mark.parametrize("name", ["sparse_paged", "sparse_paged_perhead"])
def test_sparse_paged_oracle_matches_reference(name):
    f = load(name)
    O = N.sparsetoken_naive_paged_attention(f["q"], f["cache"], f["indptr"], f["indices"],
                                            f["sparse_ind"], f["sparse_nnz"])
    assert O.shape == f["O"].shape
    assert maxabs(O, f["O"]) <= 1e-5


def test_magicpig_oracle_matches_reference():
    f = load("magicpig_paged")
    O = N.magicpig_sparsetoken_naive_paged_attention(f["q"], f["cache"], f["indptr"], f["indices"],
                                                     f["sparse_ind"], f["sparse_nnz"], f["K"], f["L"])
    assert O.shape == f["O"].shape
    assert maxabs(O, f["O"]) <= 1e-5


def test_lse_merge_reference_is_exact_split():
    # splitting a softmax into parts and merging by LSE reproduces the whole
    g = torch.Generator().manual_seed(7)
    s = torch.randn(3, 40, generator=g, dtype=torch.float64)
    v = torch.randn(40, 16, generator=g, dtype=torch.float64)
    full = torch.softmax(s, -1) @ v
    cuts = [0, 7, 8, 25, 40]
    os_, ls = [], []
    for a, b in zip(cuts[:-1], cuts[1:]):
        os_.append(torch.softmax(s[:, a:b], -1) @ v[a:b])
        ls.append(torch.logsumexp(s[:, a:b], -1))
    os_.append(torch.zeros(3, 16, dtype=torch.float64))
    ls.append(torch.full((3,), float("-inf"), dtype=torch.float64))
    merged = N.lse_merge_reference(torch.stack(os_), torch.stack(ls))
    assert maxabs(merged, full) <= 1e-12


def test_mask_index_oracles_match_reference_loops():
    f = load("mask_index")
    ind, nnz = N.sparse_lists_from_mask(f["kept_mask"], int(f["L_max"]))
    assert torch.equal(ind, f["sparse_ind"]) and torch.equal(nnz, f["sparse_nnz"])
    m = N.sparse_mask_from_lists(f["sparse_ind"], f["sparse_nnz"], f["kept_mask"].shape[2])
    assert torch.equal(m, f["precompute_mask"])
    # an empty row's list is [0, -1, ...]; reading it back marks token 0 only
    empty = f["kept_mask"].sum(-1) == 0
    assert empty.any() and torch.all(f["precompute_mask"][empty].sum(-1) == 1)
