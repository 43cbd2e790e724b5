"""Host logic of the multi-GPU KV split on CPU: shard ranges, list sharding
and rebasing, and the all-gather + merge orchestration across 2 gloo ranks
(the CUDA partial/merge steps are replaced by CPU stand-ins here)."""

import pytest
import torch
import torch.multiprocessing as mp

from attention_kernel_triton_b200 import workloads as W
from attention_kernel_triton_b200.distributed import (KVHeadPartition, PagedKeyShard, lpt_assign, prefill_unit_blocks,
                                                      shard_range, shard_sparse_lists)


def test_shard_range_covers_exactly():
    for n in (0, 1, 7, 131072):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1


def test_shard_sparse_lists_matches_python():
    c = W.make_sparse_dense(B=2, Hq=4, Hkv=2, L=300, D=64, keep_p=0.1, seed=1, per_qo_head=True)
    c.sparse_nnz[1, 2, 0] = 0
    for lo, hi in [(0, 100), (100, 200), (250, 300), (0, 300), (299, 300)]:
        ind, nnz = shard_sparse_lists(c.sparse_ind, c.sparse_nnz, lo, hi)
        for b in range(2):
            for h in range(4):
                full = c.sparse_ind[b, h, : int(c.sparse_nnz[b, h])].tolist()
                want = [t - lo for t in full if lo <= t < hi]
                got = ind[b, h, : int(nnz[b, h])].tolist()
                assert got == want
                assert all(x == -1 for x in ind[b, h, int(nnz[b, h]):].tolist())


def test_shard_sparse_lists_per_sequence_ranges():
    c = W.make_sparse_dense(B=3, Hq=4, Hkv=2, L=400, D=64, keep_p=0.1, seed=2)
    lo, hi = torch.tensor([0, 100, 390]), torch.tensor([50, 300, 400])
    ind, nnz = shard_sparse_lists(c.sparse_ind, c.sparse_nnz, lo, hi)
    for b in range(3):
        for h in range(4):
            full = c.sparse_ind[b, h, : int(c.sparse_nnz[b, h])].tolist()
            want = [t - int(lo[b]) for t in full if lo[b] <= t < hi[b]]
            assert ind[b, h, : int(nnz[b, h])].tolist() == want


def test_kv_head_partition_covers_every_head_once():
    for Hkv, G, world in [(8, 4, 1), (8, 4, 2), (8, 4, 8), (16, 4, 8), (5, 2, 3)]:
        parts = [KVHeadPartition(Hkv, G, world, r) for r in range(world)]
        assert [p.h0 for p in parts][0] == 0 and parts[-1].h1 == Hkv
        assert all(a.h1 == b.h0 for a, b in zip(parts, parts[1:]))
        assert all(p.q0 == p.h0 * G and p.q1 == p.h1 * G for p in parts)
        t = torch.arange(Hkv * G).view(1, Hkv * G, 1)
        assert torch.equal(torch.cat([p.q_heads(t) for p in parts], 1), t)


def test_lpt_assign_is_within_four_thirds_of_the_lower_bound():
    g = torch.Generator().manual_seed(0)
    for world in (2, 3, 4, 8):
        costs = (torch.randint(64, 1025, (40,), generator=g).float() ** 2).tolist()
        owners, loads = lpt_assign(costs, world)
        assert len(owners) == len(costs) and all(0 <= o < world for o in owners)
        assert abs(sum(loads) - sum(costs)) < 1e-6 * sum(costs)
        lower = max(sum(costs) / world, max(costs))
        assert max(loads) <= 4.0 / 3.0 * lower + 1e-6


@pytest.mark.parametrize("Hkv,world", [(16, 8), (16, 4), (4, 8), (3, 2), (2, 8)])
def test_prefill_unit_blocks_cover_every_unit_once(Hkv, world):
    lens = [1024, 468, 631, 258, 353, 599, 732, 94]
    seen = []
    for r in range(world):
        for b, h0, h1 in prefill_unit_blocks(lens, Hkv, world, r):
            assert 0 <= b < len(lens) and 0 <= h0 < h1 <= Hkv
            seen += [(b, h) for h in range(h0, h1)]
    assert sorted(seen) == [(b, h) for b in range(len(lens)) for h in range(Hkv)]


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_paged_key_shard_tables_partition_the_pages(world):
    c = W.make_sparse_paged(B=3, Hq=8, Hkv=2, D=64, page_size=16, lens=[100, 1000, 37], keep_p=0.1, seed=4)
    covered = {b: [] for b in range(3)}
    for r in range(world):
        for compact in (True, False):
            sh = PagedKeyShard(c.cache, c.indptr, c.indices, world, r, compact=compact)
            for b in range(3):
                s, e = int(sh.indptr[b]), int(sh.indptr[b + 1])
                lo, hi = int(sh.tok_lo[b]), int(sh.tok_hi[b])
                assert lo % 16 == 0 and (hi - lo) == 16 * (e - s)
                gs = int(c.indptr[b]) + lo // 16
                for j in range(e - s):  # local page j holds the same rows as global page lo/P + j
                    assert torch.equal(sh.cache[int(sh.indices[s + j])], c.cache[int(c.indices[gs + j])])
                if compact:
                    covered[b] += list(range(lo, hi))
    for b in range(3):
        n = int(c.indptr[b + 1] - c.indptr[b])
        assert sorted(covered[b]) == list(range(16 * n))



def _worker(rank, world, port_q, q):
    import torch.distributed as dist

    import dist_helpers as H
    from attention_kernel_triton_b200.distributed import sparsetoken_decode_kv_split
    from oracle import naive as N
    H.init_group("gloo", rank, world, port_q)
    try:
        c = W.make_sparse_dense(B=1, Hq=8, Hkv=2, L=1000, D=64, keep_p=0.05, seed=3)
        lo, hi = shard_range(1000, world, rank)
        ind, nnz = shard_sparse_lists(c.sparse_ind, c.sparse_nnz, lo, hi)
        out = sparsetoken_decode_kv_split(c.q, c.K[:, :, lo:hi], c.V[:, :, lo:hi], ind, nnz, c.softmax_scale,
                                          c.group, partial_fn=H.oracle_partial, merge_fn=H.oracle_merge)
        ref = N.sparsetoken_naive_decode(c.q, c.K, c.V, c.sparse_ind, c.sparse_nnz, c.softmax_scale, c.group)
        q.put((rank, float((out.float() - ref).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_kv_split_orchestration_two_gloo_ranks(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port_q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port_q, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    errs = dict(q.get(timeout=5) for _ in range(world))
    assert max(errs.values()) <= 2e-3, errs


def _paged_worker(rank, world, port_q, q, magic):
    import torch.distributed as dist

    import dist_helpers as H
    from attention_kernel_triton_b200.distributed import sparsetoken_decode_paged_kv_split
    from oracle import naive as N
    H.init_group("gloo", rank, world, port_q)
    try:
        c = W.make_sparse_paged(B=2, Hq=8, Hkv=2, D=64, page_size=16, lens=[700, 333], keep_p=0.05, seed=5,
                                magicpig=magic)
        sh = PagedKeyShard(c.cache, c.indptr, c.indices, world, rank)
        ind, nnz = sh.lists(c.sparse_ind, c.sparse_nnz)
        out = sparsetoken_decode_paged_kv_split(c.q, sh, ind, nnz, K=c.K, L=c.L, partial_fn=H.oracle_paged_partial,
                                                merge_fn=H.oracle_merge)
        if magic:
            ref = N.magicpig_sparsetoken_naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.sparse_ind,
                                                               c.sparse_nnz, c.K, c.L)
        else:
            ref = N.sparsetoken_naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.sparse_ind, c.sparse_nnz)
        q.put((rank, float((out.float() - ref).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("magic", [False, True])
def test_paged_kv_split_orchestration_two_gloo_ranks(magic):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port_q = ctx.Queue()
    procs = [ctx.Process(target=_paged_worker, args=(r, 2, port_q, q, magic)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    errs = dict(q.get(timeout=5) for _ in range(2))
    assert max(errs.values()) <= 2e-3, errs


def test_peer_exchange_layout_regions_do_not_overlap():
    from attention_kernel_triton_b200.distributed import exchange_layout
    for rows, D, world in [(32, 128, 1), (32, 128, 2), (96, 256, 8)]:
        total, part, data_off, flag_off, counter_off = exchange_layout(rows, D, world)
        assert part == rows * D + rows
        assert flag_off(0) + 4 * 8 <= flag_off(1) and flag_off(1) + 4 * 8 <= counter_off
        assert counter_off + 8 <= data_off(0)
        assert data_off(0) + world * part * 4 == data_off(1)
        assert data_off(1) + world * part * 4 == total
        assert data_off(0) % 16 == 0 and data_off(1) % 16 == 0
