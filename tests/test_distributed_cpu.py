"""Host logic of the multi-GPU KV split on CPU: shard ranges, list sharding
and rebasing, and the all-gather + merge orchestration across 2 gloo ranks
(the CUDA partial/merge steps are replaced by CPU stand-ins here)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from attention_kernel_triton_b200 import workloads as W
from attention_kernel_triton_b200.distributed import shard_range, shard_sparse_lists


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


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import torch.distributed as dist

    import dist_helpers as H
    from attention_kernel_triton_b200.distributed import sparsetoken_decode_kv_split
    from oracle import naive as N
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
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
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    errs = dict(q.get(timeout=5) for _ in range(world))
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
