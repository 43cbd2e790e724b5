"""GPU parity of the paged KV append (write path): the pool after the append is
bit-identical to the CPU oracle's, and the paged decode over it equals the decode
over a pool that held those rows all along."""
import pytest
import torch

from oracle import naive as N

from attention_kernel_triton_b200 import _lib
from attention_kernel_triton_b200 import workloads as W
from attention_kernel_triton_b200.decode_flash_attention_redundant_var_len_paged import flash_attention_decode_paged
from attention_kernel_triton_b200.paged_kv_append import append_paged_kv_cache

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def device_status_clean():
    _lib.device_status(0, clear=True)
    yield


def rows_at(c, b, positions, P):
    """K and V rows [n, Hkv, D] of sequence b at the given positions (through the page table)."""
    s = int(c.indptr[b])
    ks, vs = [], []
    for pos in positions:
        page = int(c.indices[s + pos // P])
        ks.append(c.cache[page, 0, :, pos % P])
        vs.append(c.cache[page, 1, :, pos % P])
    return torch.stack(ks), torch.stack(vs)


@pytest.mark.parametrize("P,D", [(16, 128), (64, 64)])
def test_append_matches_oracle_and_decode(P, D):
    lens = [1, 16, 17, 250, 40]
    new = [1, 1, 3, 37, 40]  # one-token decode appends, a page-crossing chunk, a whole sequence
    c = W.make_paged(B=5, Hq=8, Hkv=2, D=D, page_size=P, lens=lens, seed=P + D, device=DEV)
    ks, vs, ap = [], [], [0]
    for b, n in enumerate(new):
        k, v = rows_at(c, b, range(lens[b] - n, lens[b]), P)
        ks.append(k)
        vs.append(v)
        ap.append(ap[-1] + n)
    app_k, app_v = torch.cat(ks).contiguous(), torch.cat(vs).contiguous()
    app_indptr = torch.tensor(ap, dtype=torch.int32, device=DEV)
    holed = c.cache.clone()
    for b, n in enumerate(new):  # wipe the rows the append must restore
        s = int(c.indptr[b])
        for pos in range(lens[b] - n, lens[b]):
            holed[int(c.indices[s + pos // P]), :, :, pos % P] = 0
    ref = N.append_paged_kv_reference(holed, app_k, app_v, app_indptr, c.indptr, c.indices, c.last_page_len)
    append_paged_kv_cache(holed, app_k, app_v, app_indptr, c.indptr, c.indices, c.last_page_len)
    assert torch.equal(holed.cpu(), ref)
    assert torch.equal(holed, c.cache)
    O = flash_attention_decode_paged(c.q, holed, c.indptr, c.indices, c.last_page_len)
    assert torch.equal(O, flash_attention_decode_paged(c.q, c.cache, c.indptr, c.indices, c.last_page_len))
    assert _lib.device_status(0) == 0


def test_append_strided_rows_and_empty_sequences():
    c = W.make_paged(B=3, Hq=4, Hkv=2, D=128, page_size=16, lens=[5, 33, 9], seed=3, device=DEV)
    big = torch.randn(4, 3, 128, dtype=torch.float16, device=DEV)  # head stride 128, token stride 384
    app_k, app_v = big[:, :2], big[:, 1:]
    app_indptr = torch.tensor([0, 0, 4, 4], dtype=torch.int32, device=DEV)  # only sequence 1 grows
    pool = c.cache.clone()
    ref = N.append_paged_kv_reference(pool, app_k, app_v, app_indptr, c.indptr, c.indices, c.last_page_len)
    append_paged_kv_cache(pool, app_k, app_v, app_indptr, c.indptr, c.indices, c.last_page_len)
    assert torch.equal(pool.cpu(), ref)
    assert _lib.device_status(0) == 0


def test_append_bad_page_is_skipped_and_recorded():
    c = W.make_paged(B=1, Hq=4, Hkv=2, D=128, page_size=16, lens=[20], seed=4, device=DEV)
    indices = c.indices.clone()
    indices[1] = 10_000  # the page holding positions 16..19
    app_k = torch.ones(1, 2, 128, dtype=torch.float16, device=DEV)
    pool = c.cache.clone()
    append_paged_kv_cache(pool, app_k, app_k, torch.tensor([0, 1], dtype=torch.int32, device=DEV), c.indptr,
                          indices, c.last_page_len)
    assert _lib.device_status(0) == 2
    assert torch.equal(pool, c.cache)
