"""CPU stand-ins for the two compute steps of the KV-split sparse decode, used
only to exercise the host logic (sharding, all-gather, ordering) under gloo."""
import math

import torch

from oracle import naive as N


def oracle_partial(buf, rows, D, q, K, V, ind, nnz, scale, group):
    B, Hq = q.shape[0], q.shape[1]
    o = buf[: rows * D].view(B, Hq, D)
    lse = buf[rows * D:].view(B, Hq)
    qf, Kf, Vf = q.float(), K.float(), V.float()
    for b in range(B):
        for h in range(Hq):
            n = int(nnz[b, h])
            if n <= 0:
                o[b, h] = 0
                lse[b, h] = -math.inf
                continue
            idx = ind[b, h, :n].long()
            s = (Kf[b, h // group, idx] @ qf[b, h, 0]) * scale
            lse[b, h] = torch.logsumexp(s, 0)
            o[b, h] = torch.softmax(s, 0) @ Vf[b, h // group, idx]


def oracle_merge(out, recv, rows, D):
    n = recv.shape[0]
    o = recv[:, : rows * D].view(n, rows, D)
    lse = recv[:, rows * D:]
    out.view(rows, D).copy_(N.lse_merge_reference(o, lse).to(out.dtype))


def oracle_paged_partial(buf, rows, D, q, shard, ind, nnz, K=None, L=None):
    """CPU stand-in for the paged partial: softmax over the kept tokens the shard's
    page table holds (MagicPIG scores when ``K``/``L`` are given)."""
    B, Hq = q.shape[0], q.shape[1]
    o = buf[: rows * D].view(B, Hq, D)
    lse = buf[rows * D:].view(B, Hq)
    cache = shard.cache.float()
    P = cache.shape[3]
    G = Hq // cache.shape[2]
    qf = q.float()
    for b in range(B):
        for h in range(Hq):
            n = int(nnz[b, h])
            if n <= 0:
                o[b, h] = 0
                lse[b, h] = -math.inf
                continue
            toks = ind[b, h, :n].long()
            phys = shard.indices[int(shard.indptr[b]) + toks // P].long()
            k = cache[phys, 0, h // G, toks % P]
            v = cache[phys, 1, h // G, toks % P]
            if K is None:
                s = (k @ qf[b, h, 0]) / math.sqrt(D)
            else:
                s = N.magicpig_logits(qf[b, h, 0], k, float(K[b, h]), float(L[b, h]), D)
            lse[b, h] = torch.logsumexp(s, 0)
            o[b, h] = torch.softmax(s, 0) @ v


def init_group(backend, rank, world, port_q, device_id=None, timeout_s=60):
    """Join a process group whose TCPStore rank 0 binds to a port the OS picks.

    Rank 0 creates the store on port 0 (bound at once, so no other socket can
    take it in between) and hands the port to the other ranks through
    ``port_q``.  Picking a free port in the parent and binding it later in the
    child races with every other socket on the machine, NCCL's own bootstrap
    sockets included, and fails with "address already in use".
    """
    import datetime

    import torch.distributed as dist
    timeout = datetime.timedelta(seconds=timeout_s)
    if rank == 0:
        store = dist.TCPStore("127.0.0.1", 0, world, is_master=True, timeout=timeout, wait_for_workers=False)
        for _ in range(world - 1):
            port_q.put(store.port)
    else:
        store = dist.TCPStore("127.0.0.1", port_q.get(timeout=timeout_s * 2), world, is_master=False,
                              timeout=timeout)
    kw = {"device_id": device_id} if device_id is not None else {}
    dist.init_process_group(backend, store=store, rank=rank, world_size=world, timeout=timeout, **kw)
    return store
