"""GPU parity of the keep-mask <-> kept-index-list kernels against the reference's
own loops (golden fixture) and the CPU oracle.  Integer/byte work: bit-exact."""
import pytest
import torch

from golden_io import load
from oracle import naive as N

from attention_kernel_triton_b200 import _lib
from attention_kernel_triton_b200 import workloads as W
from attention_kernel_triton_b200.sparse_index import precompute_mask, sparse_index_from_mask
from attention_kernel_triton_b200.sparsetoken_decode_flash_attention_redundant import (
    sparsetoken_flash_attention_decode)

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def device_status_clean():
    _lib.device_status(0, clear=True)
    yield


def test_matches_reference_loops_golden():
    f = load("mask_index")
    ind, nnz = sparse_index_from_mask(f["kept_mask"].to(DEV), int(f["L_max"]))
    assert torch.equal(ind.cpu(), f["sparse_ind"]) and torch.equal(nnz.cpu(), f["sparse_nnz"])
    m = precompute_mask(f["sparse_ind"].to(DEV), f["sparse_nnz"].to(DEV), f["kept_mask"].shape[2])
    assert torch.equal(m.cpu(), f["precompute_mask"])
    assert _lib.device_status(0) == 0


@pytest.mark.parametrize("L", [1, 15, 16, 17, 300, 16384, 16385, 40000])
@pytest.mark.parametrize("p", [0.0, 0.002, 0.05, 0.5, 1.0])
def test_mask_to_lists_matches_oracle(L, p):
    g = torch.Generator().manual_seed(L * 7 + int(p * 1000))
    mask = torch.rand((2, 3, L), generator=g) < p
    L_max = L  # never overflows
    ind, nnz = sparse_index_from_mask(mask.to(DEV), L_max)
    ri, rn = N.sparse_lists_from_mask(mask, L_max)
    assert torch.equal(nnz.cpu(), rn) and torch.equal(ind.cpu(), ri)
    assert _lib.device_status(0) == 0


def test_mask_to_lists_strided_and_uint8_input():
    g = torch.Generator().manual_seed(5)
    full = (torch.rand((2, 8, 1000), generator=g) < 0.1).to(torch.uint8)
    view = full[:, 1::2]  # head stride 2000 bytes, rows not 16-byte aligned
    ind, nnz = sparse_index_from_mask(full.to(DEV)[:, 1::2], 150)
    ri, rn = N.sparse_lists_from_mask(view.bool(), 150)
    assert torch.equal(ind.cpu(), ri) and torch.equal(nnz.cpu(), rn)


def test_overflow_truncates_and_records_status():
    mask = torch.zeros((1, 2, 100), dtype=torch.bool)
    mask[0, 0, ::2] = True  # 50 kept, list holds 20
    mask[0, 1, 7] = True
    ind, nnz = sparse_index_from_mask(mask.to(DEV), 20)
    assert nnz.cpu().flatten().tolist() == [20, 1]
    assert ind[0, 0].cpu().tolist() == list(range(0, 40, 2))
    assert ind[0, 1].cpu().tolist() == [7] + [-1] * 19
    assert _lib.device_status(0) == 5


def test_empty_rows_without_keep_first():
    mask = torch.zeros((1, 2, 64), dtype=torch.bool)
    mask[0, 1, 63] = True
    ind, nnz = sparse_index_from_mask(mask.to(DEV), 8, keep_first_if_empty=False)
    assert nnz.cpu().flatten().tolist() == [0, 1]
    assert torch.all(ind[0, 0] == -1) and ind[0, 1, 0].item() == 63


@pytest.mark.parametrize("L", [1, 17, 333, 40000])
def test_lists_to_mask_matches_oracle(L):
    c_ind = torch.full((2, 4, 40), -1, dtype=torch.int32)
    nnz = torch.tensor([[[0], [1], [40], [7]], [[3], [0], [12], [40]]], dtype=torch.int32)
    g = torch.Generator().manual_seed(L)
    for b in range(2):
        for h in range(4):
            n = int(nnz[b, h])
            if n:
                c_ind[b, h, :n] = torch.sort(torch.randint(0, L, (n,), generator=g)).values.to(torch.int32)
    if L >= 2:
        c_ind[1, 2, 3] = -2  # a negative Python index counts from the end
    m = precompute_mask(c_ind.to(DEV), nnz.to(DEV), L)
    assert torch.equal(m.cpu(), N.sparse_mask_from_lists(c_ind, nnz, L))
    assert _lib.device_status(0) == 0


def test_lists_to_mask_out_of_range_is_skipped_and_recorded():
    ind = torch.tensor([[[3, 100, -101, 5]]], dtype=torch.int32)
    nnz = torch.tensor([[[4]]], dtype=torch.int32)
    m = precompute_mask(ind.to(DEV), nnz.to(DEV), 100)
    assert torch.nonzero(m[0, 0]).flatten().cpu().tolist() == [3, 5]
    assert _lib.device_status(0) == 3


def test_round_trip_and_decode_through_device_lists():
    # cfg4 shape (32000 tokens): keep mask per (kv head, token), p = 0.02, repeated over the group
    c = W.make_sparse_dense(B=1, Hq=32, Hkv=8, L=32000, D=128, keep_p=0.02, seed=41, device=DEV)
    mask = N.sparse_mask_from_lists(c.sparse_ind.cpu(), c.sparse_nnz.cpu(), 32000).to(DEV)
    ind, nnz = sparse_index_from_mask(mask, c.sparse_ind.shape[2])
    assert torch.equal(nnz, c.sparse_nnz) and torch.equal(ind, c.sparse_ind)
    assert torch.equal(precompute_mask(ind, nnz, 32000), mask)
    O = sparsetoken_flash_attention_decode(c.q, c.K, c.V, ind, nnz, c.softmax_scale, c.group)
    ref = N.sparsetoken_naive_decode_by_mask(c.q, c.K, c.V, ind, nnz, c.softmax_scale, c.group, mask.cpu())
    assert (O.float().cpu() - ref).abs().max().item() <= 2e-3
    assert _lib.device_status(0) == 0
