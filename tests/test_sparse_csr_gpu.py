"""GPU parity of the CSR-list (inds + ptr) sparse-token decodes: the same kernels as
the padded-list entry points, so outputs must be bit-identical to them, and within
max-abs 2e-3 of the fp32 oracle run on the equivalent padded lists."""
import pytest
import torch

from golden_io import load
from oracle import naive as N

from attention_kernel_triton_b200 import _lib
from attention_kernel_triton_b200 import workloads as W
from attention_kernel_triton_b200.magicpig_sparsetoken_decode_flash_attention_redundant_var_len_paged_with_norm import (
    magicpig_sparsetoken_flash_attention_decode_paged, magicpig_sparsetoken_flash_attention_decode_paged_csr)
from attention_kernel_triton_b200.sparse_index import sparse_csr_from_lists
from attention_kernel_triton_b200.sparsetoken_decode_flash_attention_redundant import (
    sparsetoken_flash_attention_decode, sparsetoken_flash_attention_decode_csr)
from attention_kernel_triton_b200.sparsetoken_decode_flash_attention_redundant_var_len_paged import (
    sparsetoken_flash_attention_decode_paged, sparsetoken_flash_attention_decode_paged_csr)

pytestmark = pytest.mark.gpu
TOL = 2e-3
DEV = "cuda"


@pytest.fixture(autouse=True)
def device_status_clean():
    _lib.device_status(0, clear=True)
    yield


def cuda(*ts):
    return [t.to(DEV) for t in ts]


def test_csr_conversion_matches_oracle():
    f = load("sparse_dense")
    inds, ptr = sparse_csr_from_lists(*cuda(f["sparse_ind"], f["sparse_nnz"]))
    B, H, _ = f["sparse_ind"].shape
    ind, nnz = N.sparse_lists_from_csr(inds.cpu(), ptr.cpu(), B, H)
    assert torch.equal(nnz, f["sparse_nnz"].reshape(B, H, 1).clamp(min=0))
    for b in range(B):
        for h in range(H):
            n = int(nnz[b, h])
            assert torch.equal(ind[b, h, :n], f["sparse_ind"][b, h, :n])


def test_dense_csr_matches_padded_and_golden():
    f = load("sparse_dense")
    q, K, V, ind, nnz = cuda(f["q"], f["K"], f["V"], f["sparse_ind"], f["sparse_nnz"])
    inds, ptr = sparse_csr_from_lists(ind, nnz)
    O_pad = sparsetoken_flash_attention_decode(q, K, V, ind, nnz, f["softmax_scale"], f["group"])
    O_csr = sparsetoken_flash_attention_decode_csr(q, K, V, inds, ptr, f["softmax_scale"], f["group"],
                                                   max_nnz=ind.shape[2])
    assert torch.equal(O_csr, O_pad)
    assert (O_csr.float().cpu() - f["O"]).abs().max().item() <= TOL
    assert _lib.device_status(0) == 0


def test_dense_csr_cfg4_with_explicit_bound():
    c = W.make_sparse_dense(seed=41, device=DEV)  # cfg4: q [1,32,1,128], K/V [1,8,32000,128], keep 2%
    inds, ptr = sparse_csr_from_lists(c.sparse_ind, c.sparse_nnz)
    O = sparsetoken_flash_attention_decode_csr(c.q, c.K, c.V, inds, ptr, c.softmax_scale, c.group,
                                               max_nnz=c.sparse_ind.shape[2])
    ref = N.sparsetoken_naive_decode(c.q, c.K, c.V, c.sparse_ind, c.sparse_nnz, c.softmax_scale, c.group)
    assert (O.float().cpu() - ref).abs().max().item() <= TOL


@pytest.mark.parametrize("name", ["sparse_paged", "sparse_paged_perhead"])
def test_paged_csr_matches_padded_and_golden(name):
    f = load(name)
    q, cache, indptr, indices, ind, nnz = cuda(f["q"], f["cache"], f["indptr"], f["indices"], f["sparse_ind"],
                                               f["sparse_nnz"])
    inds, ptr = sparse_csr_from_lists(ind, nnz)
    O_pad = sparsetoken_flash_attention_decode_paged(q, cache, indptr, indices, ind, nnz)
    O_csr = sparsetoken_flash_attention_decode_paged_csr(q, cache, indptr, indices, inds, ptr, max_nnz=ind.shape[2])
    assert torch.equal(O_csr, O_pad)
    assert (O_csr.float().cpu() - f["O"]).abs().max().item() <= TOL


def test_magicpig_csr_matches_padded_and_golden():
    f = load("magicpig_paged")
    q, cache, indptr, indices, ind, nnz, Kp, Lp = cuda(f["q"], f["cache"], f["indptr"], f["indices"],
                                                       f["sparse_ind"], f["sparse_nnz"], f["K"], f["L"])
    inds, ptr = sparse_csr_from_lists(ind, nnz)
    O_pad = magicpig_sparsetoken_flash_attention_decode_paged(q, cache, indptr, indices, ind, nnz, Kp, Lp)
    O_csr = magicpig_sparsetoken_flash_attention_decode_paged_csr(q, cache, indptr, indices, inds, ptr, Kp, Lp,
                                                                  max_nnz=ind.shape[2])
    assert torch.equal(O_csr, O_pad)
    assert (O_csr.float().cpu() - f["O"]).abs().max().item() <= TOL


def test_csr_ragged_rows_empty_rows_and_no_padding():
    # rows of very different lengths (one empty) in one flat array of exactly sum(nnz) entries
    c = W.make_sparse_dense(B=2, Hq=8, Hkv=2, L=3000, D=128, keep_p=0.05, seed=77, device=DEV, per_qo_head=True)
    nnz = c.sparse_nnz.clone()
    nnz[0, 3] = 0
    nnz[1, 5] = 1
    inds, ptr = sparse_csr_from_lists(c.sparse_ind, nnz)
    assert inds.numel() == int(nnz.clamp(min=0).sum())
    O = sparsetoken_flash_attention_decode_csr(c.q, c.K, c.V, inds, ptr, c.softmax_scale, c.group,
                                               max_nnz=c.sparse_ind.shape[2])
    assert torch.all(O[0, 3] == 0)
    ref = N.sparsetoken_naive_decode(c.q, c.K, c.V, c.sparse_ind, nnz, c.softmax_scale, c.group)
    mask = torch.ones(2, 8, dtype=torch.bool)
    mask[0, 3] = False  # the oracle reads an empty list as the reference does (index -1); we give zeros
    assert (O.float().cpu()[mask] - ref[mask]).abs().max().item() <= TOL


def test_csr_max_nnz_is_required():
    c = W.make_sparse_dense(B=1, Hq=4, Hkv=1, L=500, D=128, keep_p=0.05, seed=79, device=DEV)
    inds, ptr = sparse_csr_from_lists(c.sparse_ind, c.sparse_nnz)
    with pytest.raises(TypeError):
        sparsetoken_flash_attention_decode_csr(c.q, c.K, c.V, inds, ptr, c.softmax_scale, c.group)
    with pytest.raises(ValueError):
        sparsetoken_flash_attention_decode_csr(c.q, c.K, c.V, inds, ptr, c.softmax_scale, c.group, max_nnz=-1)


def test_csr_malformed_offsets_and_overlong_rows_are_recorded():
    c = W.make_sparse_dense(B=1, Hq=4, Hkv=1, L=2000, D=128, keep_p=0.05, seed=78, device=DEV)
    inds, ptr = sparse_csr_from_lists(c.sparse_ind, c.sparse_nnz)
    bad = ptr.clone()
    bad[2] = bad[1] - 1  # row 1 ends before it starts: malformed
    O = sparsetoken_flash_attention_decode_csr(c.q, c.K, c.V, inds, bad, c.softmax_scale, c.group,
                                               max_nnz=c.sparse_ind.shape[2])
    assert _lib.device_status(0, clear=True) == 4
    assert torch.all(O[0, 1] == 0)
    good = sparsetoken_flash_attention_decode_csr(c.q, c.K, c.V, inds, ptr, c.softmax_scale, c.group,
                                                  max_nnz=c.sparse_ind.shape[2])
    assert torch.equal(O[0, 0], good[0, 0])
    # a bound shorter than the rows: rows are cut there and the cut is recorded
    sparsetoken_flash_attention_decode_csr(c.q, c.K, c.V, inds, ptr, c.softmax_scale, c.group, max_nnz=5)
    assert _lib.device_status(0) == 3
