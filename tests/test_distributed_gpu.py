"""GPU checks of the KV-split sparse decode: per-rank CUDA partials merged by
akt_lse_merge (ranks emulated one after another on one GPU), the merge kernel
against the oracle, and the real NCCL path on 2 GPUs when the box has them.

Tolerance: max-abs <= 2e-3 against the fp32 oracle, no NaNs.
"""
import math
import os

import pytest
import torch
import torch.multiprocessing as mp

from oracle import naive as N

from attention_kernel_triton_b200 import _lib
from attention_kernel_triton_b200 import workloads as W
from attention_kernel_triton_b200.distributed import (PeerKVSplit, lse_merge_into, shard_range, shard_sparse_lists,
                                                      sparsetoken_decode_kv_split)
from attention_kernel_triton_b200.sparsetoken_decode_flash_attention_redundant import (
    sparse_dense_partial, sparsetoken_flash_attention_decode)

pytestmark = pytest.mark.gpu
TOL = 2e-3
DEV = "cuda"


@pytest.fixture(autouse=True)
def device_status_clean():
    _lib.device_status(0, clear=True)
    yield
    assert _lib.device_status(0) == 0, "a kernel recorded an error"


def emulate_split(c, world):
    B, Hq, _, D = c.q.shape
    L = c.K.shape[2]
    rows = B * Hq
    recv = torch.empty((world, rows * D + rows), dtype=torch.float32, device=DEV)
    for r in range(world):
        lo, hi = shard_range(L, world, r)
        ind, nnz = shard_sparse_lists(c.sparse_ind, c.sparse_nnz, lo, hi)
        sparse_dense_partial(recv[r, : rows * D].view(rows, D), recv[r, rows * D:], c.q, c.K[:, :, lo:hi],
                             c.V[:, :, lo:hi], ind, nnz, c.softmax_scale, c.group)
    out = torch.empty((B, Hq, 1, D), dtype=c.q.dtype, device=DEV)
    lse_merge_into(out, recv, rows, D)
    return out


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_kv_split_emulated_matches_oracle(world):
    c = W.make_sparse_dense(B=2, Hq=8, Hkv=2, L=4000, D=128, keep_p=0.03, seed=10 + world, device=DEV)
    out = emulate_split(c, world)
    ref = N.sparsetoken_naive_decode(c.q, c.K, c.V, c.sparse_ind, c.sparse_nnz, c.softmax_scale, c.group)
    assert not torch.isnan(out).any()
    assert (out.float().cpu() - ref).abs().max().item() <= TOL
    single = sparsetoken_flash_attention_decode(c.q, c.K, c.V, c.sparse_ind, c.sparse_nnz, c.softmax_scale, c.group)
    assert (out.float() - single.float()).abs().max().item() <= TOL


def test_kv_split_128k_single_sequence_over_8_shards():
    # cfg4 long-context case: 128K-token single sequence, keep 2% per kv head, split over 8 ranks
    c = W.make_sparse_dense(B=1, Hq=32, Hkv=8, L=131072, D=128, keep_p=0.02, seed=12, device=DEV, L_max=4096)
    out = emulate_split(c, 8)
    ref = N.sparsetoken_naive_decode(c.q, c.K, c.V, c.sparse_ind, c.sparse_nnz, c.softmax_scale, c.group)
    assert (out.float().cpu() - ref).abs().max().item() <= TOL


def test_lse_merge_matches_oracle_with_empty_parts():
    g = torch.Generator().manual_seed(3)
    n, rows, D = 5, 37, 64
    o = torch.randn(n, rows, D, generator=g)
    lse = torch.randn(n, rows, generator=g) * 4
    lse[1] = -math.inf          # a part with no keys
    lse[:, 5] = -math.inf       # a row with no keys anywhere
    recv = torch.cat([o.reshape(n, -1), lse], dim=1).to(DEV)
    out = torch.empty(rows, D, dtype=torch.float16, device=DEV)
    lse_merge_into(out, recv, rows, D)
    ref = N.lse_merge_reference(o, lse)
    assert (out.float().cpu() - ref.float()).abs().max().item() <= TOL
    assert torch.all(out[5] == 0)



def _nccl_worker(rank, world, port_q, q):
    import torch.distributed as dist

    import dist_helpers as H
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    H.init_group("nccl", rank, world, port_q, device_id=dev)
    try:
        c = W.make_sparse_dense(B=1, Hq=32, Hkv=8, L=32768, D=128, keep_p=0.02, seed=21)  # CPU, same on all ranks
        lo, hi = shard_range(32768, world, rank)
        ind, nnz = shard_sparse_lists(c.sparse_ind, c.sparse_nnz, lo, hi)
        out = sparsetoken_decode_kv_split(c.q.to(dev), c.K[:, :, lo:hi].to(dev), c.V[:, :, lo:hi].to(dev),
                                          ind.to(dev), nnz.to(dev), c.softmax_scale, c.group)
        torch.cuda.synchronize(dev)
        ref = N.sparsetoken_naive_decode(c.q, c.K, c.V, c.sparse_ind, c.sparse_nnz, c.softmax_scale, c.group)
        q.put((rank, float((out.float().cpu() - ref).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_kv_split_nccl_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port_q = ctx.Queue()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port_q, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    errs = dict(q.get(timeout=5) for _ in range(2))
    assert max(errs.values()) <= TOL, errs


@pytest.mark.parametrize("fused", [True, False])
def test_peer_exchange_single_device_epochs(fused):
    # world 1: the kernel publishes into its own region and the merge waits on its own
    # flag; several epochs exercise both buffer parities and the counter reset.  fused:
    # the wait and the final merge run in the publishing merge kernel
    c = W.make_sparse_dense(B=1, Hq=32, Hkv=8, L=32768, D=128, keep_p=0.02, seed=31, device=DEV)
    ref = N.sparsetoken_naive_decode(c.q, c.K, c.V, c.sparse_ind, c.sparse_nnz, c.softmax_scale, c.group)
    x = PeerKVSplit(1, 32, 128, DEV, fused=fused)
    try:
        for _ in range(3):
            out = x(c.q, c.K, c.V, c.sparse_ind, c.sparse_nnz, c.softmax_scale, c.group)
            assert (out.float().cpu() - ref).abs().max().item() <= TOL
        x.bind(c.K, c.V, c.sparse_ind, c.sparse_nnz, c.softmax_scale, c.group)
        for _ in range(3):
            assert (x.step(c.q).float().cpu() - ref).abs().max().item() <= TOL
        x.capture()
        for _ in range(4):  # graph replays alternate the two parities
            assert (x.step_graph(c.q).float().cpu() - ref).abs().max().item() <= TOL
        assert (x.step(c.q).float().cpu() - ref).abs().max().item() <= TOL  # eager again after graphs
    finally:
        x.close()
    assert _lib.device_status(0) == 0


def test_peer_exchange_call_order_is_checked():
    c = W.make_sparse_dense(B=1, Hq=8, Hkv=2, L=2048, D=128, keep_p=0.05, seed=32, device=DEV)
    with PeerKVSplit(1, 8, 128, DEV) as x:
        with pytest.raises(RuntimeError, match="bind"):
            x.step(c.q)
        with pytest.raises(AssertionError, match="head_dim"):
            x.bind(c.K[..., :64], c.V[..., :64], c.sparse_ind, c.sparse_nnz, c.softmax_scale, c.group)
        x.bind(c.K, c.V, c.sparse_ind, c.sparse_nnz, c.softmax_scale, c.group)
        with pytest.raises(RuntimeError, match="capture"):
            x.step_graph(c.q)
        ref = N.sparsetoken_naive_decode(c.q, c.K, c.V, c.sparse_ind, c.sparse_nnz, c.softmax_scale, c.group)
        assert (x.step(c.q).float().cpu() - ref).abs().max().item() <= TOL
    with pytest.raises(RuntimeError, match="closed"):
        x.step(c.q)
    assert _lib.device_status(0) == 0


def _peer_worker(rank, world, port_q, q):
    import torch.distributed as dist

    import dist_helpers as H
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    H.init_group("nccl", rank, world, port_q, device_id=dev)
    x = None
    try:
        c = W.make_sparse_dense(B=1, Hq=32, Hkv=8, L=32768, D=128, keep_p=0.02, seed=22)  # CPU, same on all ranks
        lo, hi = shard_range(32768, world, rank)
        ind, nnz = shard_sparse_lists(c.sparse_ind, c.sparse_nnz, lo, hi)
        args = (c.q.to(dev), c.K[:, :, lo:hi].contiguous().to(dev), c.V[:, :, lo:hi].contiguous().to(dev),
                ind.to(dev), nnz.to(dev), c.softmax_scale, c.group)
        x = PeerKVSplit(1, 32, 128, dev)
        outs = [x(*args) for _ in range(3)]
        x.bind(*args[1:])
        outs += [x.step(args[0]).clone() for _ in range(3)]
        x.capture()
        outs += [x.step_graph(args[0]).clone() for _ in range(4)]
        torch.cuda.synchronize(dev)
        ref = N.sparsetoken_naive_decode(c.q, c.K, c.V, c.sparse_ind, c.sparse_nnz, c.softmax_scale, c.group)
        err = max(float((o.float().cpu() - ref).abs().max()) for o in outs)
        q.put((rank, err, _lib.device_status(rank)))
    finally:
        if x is not None:
            x.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_exchange_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port_q = ctx.Queue()
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port_q, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [q.get(timeout=5) for _ in range(2)]
    assert max(r[1] for r in res) <= TOL, res
    assert all(r[2] == 0 for r in res), res
