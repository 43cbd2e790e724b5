"""Multi-GPU partitioning of the decode paths on one box.

Two layouts, following the structure of the work:

* Independent units (every path): kv heads (``KVHeadPartition``: each rank
  takes the same head range of every sequence) or, when the ranks do not
  divide the heads, (batch, kv head) units by longest-processing-time
  (``prefill_unit_blocks``); each GPU runs the single-GPU kernels on its share
  -- no communication.
* One long sequence, sparse-token decode: the key axis is split into
  contiguous token ranges, one per rank.  Each rank runs the sparse kernel in
  partial-output mode over its range (fp32 O normalised over its kept tokens
  and the natural-log sum-exp), the ``[O | LSE]`` partials are all-gathered
  over NCCL (NVLink) and merged with ``akt_lse_merge``:
  ``O = sum_r e^{lse_r - M} O_r / sum_r e^{lse_r - M}``.

Two implementations of the exchange: ``sparsetoken_decode_kv_split`` calls the
library all-gather (NCCL); ``PeerKVSplit`` fuses it into the kernels -- the
sparse kernel's last stage stores each rank's partial straight into every
peer's exchange region over NVLink (CUDA IPC mappings) and raises a flag, and
the merge kernel waits on the flags (bounded) and merges locally.

The reference has no multi-GPU code; this is the exchange step the 128K
single-sequence case needs.
"""
from __future__ import annotations

import ctypes
from ctypes import c_void_p
from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous, balanced slice ``[lo, hi)`` of ``n`` items for ``rank``."""
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_sparse_lists(sparse_ind: torch.Tensor, sparse_nnz: torch.Tensor, lo, hi):
    """Kept-token lists restricted to tokens ``[lo, hi)`` and rebased to ``lo``.

    ``lo``/``hi`` are ints (one range for every sequence) or ``[B]`` tensors (a range
    per sequence, as the paged key split uses).  Lists are sorted ascending (the
    reference builds them with ``nonzero``, SD:294).  Returns ``(ind [B, Hq, L_local]
    int32, -1 padded, nnz [B, Hq, 1])`` with ``L_local`` the longest local list (at
    least 1)."""
    B, Hq, Lmax = sparse_ind.shape
    ind = sparse_ind.to(torch.int64)
    nnz = sparse_nnz.reshape(B, Hq, 1).to(torch.int64)
    pos = torch.arange(Lmax, device=ind.device).view(1, 1, Lmax)
    big = torch.iinfo(torch.int64).max
    srt = torch.where(pos < nnz, ind, torch.full_like(ind, big)).reshape(B * Hq, Lmax).contiguous()
    lo_t = torch.as_tensor(lo, dtype=torch.int64, device=ind.device).reshape(-1).expand(B).reshape(B, 1)
    hi_t = torch.as_tensor(hi, dtype=torch.int64, device=ind.device).reshape(-1).expand(B).reshape(B, 1)
    bounds = torch.cat([lo_t, hi_t], 1).repeat_interleave(Hq, 0).contiguous()  # [B*Hq, 2]
    se = torch.searchsorted(srt, bounds)  # first index >= lo, first index >= hi
    cnt = (se[:, 1] - se[:, 0]).clamp_min(0)
    L_loc = max(int(cnt.max().item()) if cnt.numel() else 0, 1)
    j = torch.arange(L_loc, device=ind.device).view(1, L_loc)
    src = (se[:, :1] + j).clamp_max(Lmax - 1)
    vals = torch.gather(srt, 1, src) - bounds[:, :1]
    local = torch.where(j < cnt.view(-1, 1), vals, torch.full_like(vals, -1))
    return local.view(B, Hq, L_loc).to(torch.int32), cnt.view(B, Hq, 1).to(torch.int32)


# ----------------------------------------------------------------------------
# partition of one workload across ranks with no communication
# ----------------------------------------------------------------------------
class KVHeadPartition:
    """Rank ``rank``'s share of a GQA workload split by kv head: kv heads ``[h0, h1)``
    (``shard_range``) and their query heads ``[h0*G, h1*G)``.  Every sequence is
    split the same way, so the ranks' work is equal for any length distribution
    (dense, paged or var-len) whenever ``world`` divides the kv heads.  The rank's
    output is the matching head slice of the full output; nothing crosses NVLink."""

    def __init__(self, num_kv_heads: int, group: int, world: int, rank: int):
        if not (0 <= rank < world):
            raise ValueError("rank outside the world")
        self.num_kv_heads, self.group, self.world, self.rank = num_kv_heads, group, world, rank
        self.h0, self.h1 = shard_range(num_kv_heads, world, rank)
        self.q0, self.q1 = self.h0 * group, self.h1 * group

    @property
    def num_local_kv_heads(self) -> int:
        return self.h1 - self.h0

    def q_heads(self, t: torch.Tensor, dim: int = 1) -> torch.Tensor:
        """View of ``t``'s query heads on this rank (no copy)."""
        return t.narrow(dim, self.q0, self.q1 - self.q0)

    def kv_heads(self, t: torch.Tensor, dim: int = 1) -> torch.Tensor:
        """View of ``t``'s kv heads on this rank (no copy)."""
        return t.narrow(dim, self.h0, self.h1 - self.h0)

    def local_paged_cache(self, paged_kv_cache: torch.Tensor) -> torch.Tensor:
        """This rank's kv heads of a pool ``[N, 2, Hkv, P, D]`` as its own contiguous
        pool ``[N, 2, h1-h0, P, D]``: the resident cache a rank keeps (built once)."""
        return paged_kv_cache[:, :, self.h0:self.h1].contiguous()


def decode_paged_partitioned(q: torch.Tensor, local_cache: torch.Tensor, kv_page_indptr, kv_page_indices,
                             kv_last_page_len, part: KVHeadPartition, out: Optional[torch.Tensor] = None):
    """Paged decode (DP:228) of this rank's kv heads.  ``q`` is the full ``[B, Hq, 1, D]``
    (its head slice is taken as a view), ``local_cache`` the rank's pool
    (``part.local_paged_cache``); the page table is shared by all ranks.  Returns the
    output head slice ``[B, (h1-h0)*G, D]`` (written into ``out`` when given)."""
    from .decode_flash_attention_redundant_var_len_paged import decode_paged_into
    if local_cache.shape[2] != part.num_local_kv_heads:
        raise ValueError("local_cache must hold exactly this rank's kv heads")
    ql = part.q_heads(q)
    if out is None:
        out = torch.empty((q.shape[0], ql.shape[1], q.shape[3]), dtype=q.dtype, device=q.device)
    if ql.shape[1] == 0:
        return out
    return decode_paged_into(out, ql, local_cache, kv_page_indptr, kv_page_indices, kv_last_page_len)


def prefill_partitioned(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, causal: bool, softmax_scale: float,
                        GQA_group_size: int, part: KVHeadPartition, varlen: Optional[torch.Tensor] = None):
    """Prefill (PF:342, or PV:348 with ``varlen``) of this rank's heads: views of the
    rank's query and kv heads go straight to the kernel (its TMA maps take the strides),
    and the output ``[B, (h1-h0)*G, S, D]`` is the rank's head slice."""
    from ._prefill import prefill_into
    Ql = part.q_heads(Q)
    O = torch.empty(Ql.shape, dtype=Q.dtype, device=Q.device)
    if part.num_local_kv_heads == 0:
        return O
    return prefill_into(O, Ql, part.kv_heads(K), part.kv_heads(V), causal, softmax_scale, GQA_group_size, varlen)


def lpt_assign(costs, world: int):
    """Longest-processing-time assignment: items in descending cost (ties by index)
    each go to the currently least-loaded rank (ties to the lowest rank).  Returns
    ``(owners, loads)``: the rank of every item and each rank's total cost.  Its
    makespan is within 4/3 of the optimum (Graham, 1969)."""
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    loads = [0.0] * world
    owners = [0] * len(costs)
    for i in order:
        r = min(range(world), key=lambda k: (loads[k], k))
        owners[i] = r
        loads[r] += costs[i]
    return owners, loads


def prefill_unit_blocks(seq_lens, num_kv_heads: int, world: int, rank: int, causal: bool = True):
    """This rank's prefill work as blocks ``(b, h0, h1)``: batch ``b``, kv heads
    ``[h0, h1)``.  When ``world`` divides the kv heads, every rank takes the same head
    range of every sequence (``KVHeadPartition``), which balances any length mix
    exactly.  Otherwise the ``(b, kv head)`` units are spread by ``lpt_assign`` on
    their attention cost (``len_b^2`` causal, ``len_b * S_max`` not) and each rank's
    units are merged into runs of consecutive heads per batch."""
    B = len(seq_lens)
    if num_kv_heads % world == 0:
        part = KVHeadPartition(num_kv_heads, 1, world, rank)
        return [(b, part.h0, part.h1) for b in range(B)] if part.h1 > part.h0 else []
    s_max = max([int(x) for x in seq_lens] + [0])
    cost = [float(int(x)) ** 2 if causal else float(int(x)) * s_max for x in seq_lens]
    units = [(b, h) for b in range(B) for h in range(num_kv_heads)]
    owners, _ = lpt_assign([cost[b] for b, _ in units], world)
    mine = sorted(u for u, o in zip(units, owners) if o == rank)
    blocks = []
    for b, h in mine:
        if blocks and blocks[-1][0] == b and blocks[-1][2] == h:
            blocks[-1] = (b, blocks[-1][1], h + 1)
        else:
            blocks.append((b, h, h + 1))
    return blocks


def prefill_blocks(Q, K, V, causal: bool, softmax_scale: float, GQA_group_size: int, blocks,
                   varlen: Optional[torch.Tensor] = None):
    """Run the prefill on each block ``(b, h0, h1)`` (views, one launch per block) and
    return ``[(block, O_block [1, (h1-h0)*G, S, D])]``."""
    from ._prefill import prefill_into
    G = GQA_group_size
    res = []
    for b, h0, h1 in blocks:
        vl = None if varlen is None else varlen.narrow(0, b, 1)
        Qb = Q[b:b + 1, h0 * G:h1 * G]
        O = torch.empty(Qb.shape, dtype=Q.dtype, device=Q.device)
        prefill_into(O, Qb, K[b:b + 1, h0:h1], V[b:b + 1, h0:h1], causal, softmax_scale, G, vl)
        res.append(((b, h0, h1), O))
    return res


# ----------------------------------------------------------------------------
# key-axis split of paged sequences (sparse-token decode)
# ----------------------------------------------------------------------------
class PagedKeyShard:
    """One rank's share of paged sequences split along the key axis.

    Sequence ``b``'s pages ``[p_lo, p_hi)`` (``shard_range`` of its page count, so
    shard boundaries fall on page boundaries) hold its tokens ``[tok_lo[b],
    tok_hi[b])``; ``indptr``/``indices`` are the rank's own CSR page table over
    ``cache``, which with ``compact`` holds only the rank's pages (their copy,
    renumbered in order) and otherwise is the full pool with global page ids."""

    def __init__(self, paged_kv_cache, kv_page_indptr, kv_page_indices, world: int, rank: int,
                 compact: bool = True):
        dev = paged_kv_cache.device
        P = paged_kv_cache.shape[3]
        ip = kv_page_indptr.to("cpu", torch.int64).tolist()
        B = len(ip) - 1
        idx = kv_page_indices.to(dev, torch.int64)
        lo, hi, counts, pieces = [], [], [], []
        for b in range(B):
            n = ip[b + 1] - ip[b]
            p_lo, p_hi = shard_range(max(n, 0), world, rank)
            lo.append(p_lo * P)
            hi.append(p_hi * P)
            counts.append(p_hi - p_lo)
            pieces.append(idx[ip[b] + p_lo: ip[b] + p_hi])
        local = torch.cat(pieces) if pieces else idx[:0]
        self.indptr = torch.tensor([0] + list(torch.tensor(counts).cumsum(0).tolist()), dtype=torch.int32,
                                   device=dev)
        if compact:
            self.cache = paged_kv_cache.index_select(0, local).contiguous()
            self.indices = torch.arange(local.numel(), dtype=torch.int32, device=dev)
        else:
            self.cache = paged_kv_cache
            self.indices = local.to(torch.int32)
        self.tok_lo = torch.tensor(lo, dtype=torch.int64)
        self.tok_hi = torch.tensor(hi, dtype=torch.int64)
        self.world, self.rank = world, rank

    def lists(self, sparse_ind: torch.Tensor, sparse_nnz: torch.Tensor):
        """The kept-index lists of this shard, rebased to its first token per sequence."""
        dev = sparse_ind.device
        return shard_sparse_lists(sparse_ind, sparse_nnz, self.tok_lo.to(dev), self.tok_hi.to(dev))


def _cuda_paged_partial(buf, rows, D, q, shard, ind_local, nnz_local, K, L):
    from .sparsetoken_decode_flash_attention_redundant_var_len_paged import sparse_paged_partial
    B, Hq = q.shape[0], q.shape[1]
    sparse_paged_partial(buf[: rows * D].view(B, Hq, D), buf[rows * D:].view(B, Hq), q, shard.cache, shard.indptr,
                         shard.indices, ind_local, nnz_local, K=K, L=L)


def sparsetoken_decode_paged_kv_split(q: torch.Tensor, shard: PagedKeyShard, ind_local: torch.Tensor,
                                      nnz_local: torch.Tensor, K: Optional[torch.Tensor] = None,
                                      L: Optional[torch.Tensor] = None, process_group=None,
                                      partial_fn: Optional[Callable] = None,
                                      merge_fn: Optional[Callable] = None) -> torch.Tensor:
    """Sparse-token paged decode (SP:170; MagicPIG with ``K``, ``L``, MP:166) of sequences
    whose keys are split across ranks (``PagedKeyShard``).  Each rank passes the full
    ``q [B, Hq, 1, D]``, its shard and its rebased lists (``shard.lists``); every rank
    returns the full output ``[B, Hq, D]``.  The MagicPIG score of a key depends only on
    that key and q, so a shard's partial is exact and the merge is the same.  One
    all-gather of ``B*Hq*(D+1)`` fp32 per rank crosses NVLink.

    ``partial_fn``/``merge_fn`` replace the CUDA steps only in host-logic tests on CPU."""
    B, Hq, _, D = q.shape
    rows = B * Hq
    world = dist.get_world_size(process_group) if dist.is_initialized() else 1
    send = torch.empty(rows * D + rows, dtype=torch.float32, device=q.device)
    (partial_fn or _cuda_paged_partial)(send, rows, D, q, shard, ind_local, nnz_local, K, L)
    if world > 1:
        recv = torch.empty((world, send.numel()), dtype=torch.float32, device=q.device)
        if dist.get_backend(process_group) == "nccl":
            dist.all_gather_into_tensor(recv, send, group=process_group)
        else:
            dist.all_gather(list(recv.unbind(0)), send, group=process_group)
    else:
        recv = send.view(1, -1)
    out = torch.empty((B, Hq, D), dtype=q.dtype, device=q.device)
    (merge_fn or lse_merge_into)(out, recv, rows, D)
    return out


def lse_merge_into(out: torch.Tensor, parts: torch.Tensor, rows: int, head_dim: int) -> torch.Tensor:
    """Merge ``parts [n, rows*head_dim + rows]`` (each ``[O | LSE]``) into ``out``
    (``rows`` rows of ``head_dim`` contiguous elements) with ``akt_lse_merge``."""
    dev = _lib.require_cuda(out, parts)
    n = parts.shape[0]
    stride = parts.stride(0)
    base = parts.data_ptr()
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().akt_lse_merge(base, stride, base + 4 * rows * head_dim, stride, n, rows, head_dim,
                                            out.data_ptr(), head_dim, _lib.dtype_code(out), _lib.stream_ptr(dev)))
    return out


def _cuda_partial(buf: torch.Tensor, rows: int, D: int, q, K_local, V_local, ind_local, nnz_local, scale, group):
    from .sparsetoken_decode_flash_attention_redundant import sparse_dense_partial
    sparse_dense_partial(buf[: rows * D].view(rows, D), buf[rows * D:], q, K_local, V_local, ind_local, nnz_local,
                         scale, group)


def sparsetoken_decode_kv_split(q: torch.Tensor, K_local: torch.Tensor, V_local: torch.Tensor,
                                ind_local: torch.Tensor, nnz_local: torch.Tensor, softmax_scale: float,
                                GQA_group_size: int, process_group=None,
                                partial_fn: Optional[Callable] = None,
                                merge_fn: Optional[Callable] = None) -> torch.Tensor:
    """Sparse-token decode of one long sequence whose keys are split across ranks.

    Each rank passes the full ``q [B, Hq, 1, D]``, its own token range of
    ``K/V [B, Hkv, L_local, D]`` and its rebased lists (``shard_sparse_lists``).
    Every rank returns the full output ``[B, Hq, 1, D]`` in ``q.dtype``.
    One all-gather of ``B*Hq*(D+1)`` fp32 per rank crosses NVLink.

    ``partial_fn``/``merge_fn`` replace the CUDA partial and merge steps only
    in host-logic tests on CPU (gloo); the default path runs the sm_100a
    kernels."""
    B, Hq, _, D = q.shape
    rows = B * Hq
    world = dist.get_world_size(process_group) if dist.is_initialized() else 1
    send = torch.empty(rows * D + rows, dtype=torch.float32, device=q.device)
    (partial_fn or _cuda_partial)(send, rows, D, q, K_local, V_local, ind_local, nnz_local, softmax_scale,
                                  GQA_group_size)
    if world > 1:
        recv = torch.empty((world, send.numel()), dtype=torch.float32, device=q.device)
        if dist.get_backend(process_group) == "nccl":
            dist.all_gather_into_tensor(recv, send, group=process_group)
        else:
            dist.all_gather(list(recv.unbind(0)), send, group=process_group)
    else:
        recv = send.view(1, -1)
    out = torch.empty((B, Hq, 1, D), dtype=q.dtype, device=q.device)
    (merge_fn or lse_merge_into)(out, recv, rows, D)
    return out


# ----------------------------------------------------------------------------
# exchange fused into the kernels: NVLink peer stores + flags
# ----------------------------------------------------------------------------
_HEADER = 256  # flags [2 parities][AKT_MAX_PEERS] uint32 at 0 and 32, completion counters at 64 and 68


def exchange_layout(rows: int, head_dim: int, world: int):
    """Byte layout of one device's exchange region: ``(total_bytes, part_floats,
    data_offset(parity), flags_offset(parity), counter_offset)``.  Data for parity
    ``p`` is ``[world][rows*head_dim + rows]`` fp32."""
    part = rows * head_dim + rows
    total = _HEADER + 2 * world * part * 4
    return total, part, (lambda p: _HEADER + p * world * part * 4), (lambda p: 4 * _lib.AKT_MAX_PEERS * p), 64


class PeerKVSplit:
    """Sparse-token decode of one sequence split along the key axis across the ranks of
    ``process_group`` (one GPU each), with the exchange fused into the kernels.

    Built once per shape (it allocates and maps the exchange regions: CUDA IPC handles
    are all-gathered on the host); each call is one epoch.  Calls must be issued in the
    same order on every rank, on the current stream.  ``close()`` (collective) unmaps
    and frees; used as a context manager, the exchange closes on exit."""

    def __init__(self, B: int, Hq: int, head_dim: int, device, process_group=None, fused: bool = True):
        self.pg = process_group
        # fused: the wait for the peers and the final merge run in the publishing
        # merge kernel (akt_sparse_dense_split_peer), two launches a step; else a
        # separate merge kernel (akt_lse_merge_peer), three
        self.fused = fused
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        if self.world > _lib.AKT_MAX_PEERS:
            raise ValueError(f"at most {_lib.AKT_MAX_PEERS} ranks")
        self.device = torch.device(device)
        self.B, self.Hq, self.D = B, Hq, head_dim
        self.rows = B * Hq
        total, _, self._data_off, self._flag_off, self._counter_off = exchange_layout(self.rows, head_dim, self.world)
        L = _lib.lib()
        ptr, handle = c_void_p(), (ctypes.c_char * 64)()
        with torch.cuda.device(self.device):
            _lib.check(L.akt_ipc_alloc(total, ctypes.byref(ptr), handle))
        self.local = ptr.value
        handles = [bytes(handle)]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=process_group)
        self.bases = []
        with torch.cuda.device(self.device):
            for r in range(self.world):
                if r == self.rank:
                    self.bases.append(self.local)
                    continue
                h = (ctypes.c_char * 64).from_buffer_copy(handles[r])
                pp = c_void_p()
                _lib.check(L.akt_ipc_open(h, ctypes.byref(pp)))
                self.bases.append(pp.value)
        self.epoch = 0
        self._bound = None
        self._graphs = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False

    def _require(self, bound: bool = False, graphs: bool = False):
        if self.bases is None:
            raise RuntimeError("PeerKVSplit is closed")
        if bound and self._bound is None:
            raise RuntimeError("PeerKVSplit.bind() must come before step()")
        if graphs and self._graphs is None:
            raise RuntimeError("PeerKVSplit.capture() must come before step_graph()")

    def _descriptor(self, epoch: int, flag_value: Optional[int] = None):
        """Exchange descriptor of call ``epoch`` (its parity picks the buffers); the flag
        value is the epoch itself unless given (graph replays use a constant)."""
        x = _lib.PeerExchange()
        par = epoch & 1
        for r, base in enumerate(self.bases):
            x.peer_data[r] = base + self._data_off(par)
            x.peer_flags[r] = base + self._flag_off(par)
        x.counter = self.local + self._counter_off
        x.merge_counter = self.local + self._counter_off + 4
        x.world, x.rank = self.world, self.rank
        x.epoch = (flag_value if flag_value is not None else epoch) & 0xFFFFFFFF or 1
        return x

    def __call__(self, q, K_local, V_local, ind_local, nnz_local, softmax_scale: float, GQA_group_size: int):
        from .sparsetoken_decode_flash_attention_redundant import _sparse_dense_call
        self._require()
        B, Hq, _, D = q.shape
        assert (B, Hq, D) == (self.B, self.Hq, self.D), "shape differs from the one this exchange was built for"
        self.epoch += 1
        x = self._descriptor(self.epoch)
        out = torch.empty((B, Hq, 1, D), dtype=q.dtype, device=q.device)
        if self.fused:
            _sparse_dense_call("akt_sparse_dense_split_peer", out, q, K_local, V_local, ind_local, nnz_local,
                               softmax_scale, GQA_group_size, peer=x)
            return out
        _sparse_dense_call("akt_sparse_dense_partial_peer", None, q, K_local, V_local, ind_local, nnz_local,
                           softmax_scale, GQA_group_size, peer=x)
        with torch.cuda.device(q.device):
            _lib.check(_lib.lib().akt_lse_merge_peer(ctypes.byref(x), self.rows, D, out.data_ptr(), D,
                                                     _lib.dtype_code(out), _lib.stream_ptr(q.device)))
        return out

    def bind(self, K_local, V_local, ind_local, nnz_local, softmax_scale: float, GQA_group_size: int,
             dtype=torch.float16):
        """Fix this rank's key shard and lists for repeated ``step`` calls: the argument
        structs, scratch and the q / output buffers are built once, so a step is a copy
        of q and two launches."""
        self._require()
        assert K_local.dim() == 4 and K_local.shape[0] == self.B and K_local.shape[3] == self.D, \
            "K shard must be [B, Hkv, L_local, D] with this exchange's B and head_dim"
        assert V_local.shape == K_local.shape, "V shard must match the K shard"
        L = _lib.lib()
        dev = self.device
        ind = _lib.as_int32(ind_local, dev)
        nnz = _lib.as_int32(nnz_local, dev)
        q = torch.empty((self.B, self.Hq, 1, self.D), dtype=dtype, device=dev)
        out = torch.empty_like(q)
        K, V = K_local, V_local
        a = _lib.SparseDenseArgs()
        a.q = q.data_ptr()
        a.q_stride_batch, a.q_stride_head, a.q_stride_dim = q.stride(0), q.stride(1), q.stride(3)
        a.k = K.data_ptr()
        a.k_stride_batch, a.k_stride_head, a.k_stride_token, a.k_stride_dim = K.stride()
        a.v = V.data_ptr()
        a.v_stride_batch, a.v_stride_head, a.v_stride_token, a.v_stride_dim = V.stride()
        (a.ind_stride_batch, a.ind_stride_head, a.ind_stride_pos), (a.nnz_stride_batch, a.nnz_stride_head) = \
            _lib.index_strides(ind, nnz)
        a.sparse_ind, a.sparse_nnz = ind.data_ptr(), nnz.data_ptr()
        a.batch, a.num_qo_heads, a.num_kv_heads, a.seq_len, a.head_dim = self.B, self.Hq, K.shape[1], K.shape[2], self.D
        a.max_nnz = ind.shape[2]
        a.dtype = _lib.dtype_code(q)
        a.softmax_scale = float(softmax_scale)
        a.out = out.data_ptr()
        a.out_stride_batch, a.out_stride_head, a.out_stride_dim = out.stride(0), out.stride(1), out.stride(3)
        assert self.Hq // K.shape[1] == GQA_group_size
        ws = _lib.workspace(L.akt_sparse_dense_workspace_size(ctypes.byref(a)), dev)
        self._bound = {"args": a, "ws": ws, "q": q, "out": out, "keep": (K, V, ind, nnz),
                       "dtype": _lib.dtype_code(q)}

    def step(self, q):
        """One decode over the bound shard (``bind`` first); returns the output buffer,
        which the next step overwrites."""
        self._require(bound=True)
        self._bound["q"].copy_(q)
        self.epoch += 1
        self._launch(self._descriptor(self.epoch))
        return self._bound["out"]

    def _launch(self, x):
        b = self._bound
        L = _lib.lib()
        st = _lib.stream_ptr(self.device)
        if self.fused:
            _lib.check(L.akt_sparse_dense_split_peer(ctypes.byref(b["args"]), ctypes.byref(x), b["ws"].data_ptr(),
                                                     b["ws"].numel(), st))
            return
        _lib.check(L.akt_sparse_dense_partial_peer(ctypes.byref(b["args"]), ctypes.byref(x), b["ws"].data_ptr(),
                                                   b["ws"].numel(), st))
        _lib.check(L.akt_lse_merge_peer(ctypes.byref(x), self.rows, self.D, b["out"].data_ptr(), self.D,
                                        b["dtype"], st))

    def capture(self):
        """Record the bound step as two CUDA graphs, one per buffer parity (flag value 1;
        the merge clears the flags it consumed, so the same values recur).  Collective in
        the sense that every rank must then use ``step_graph`` for the same calls."""
        self._require(bound=True)
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            self._graphs = []
            for par in (0, 1):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self._launch(self._descriptor(par, flag_value=1))
                self._graphs.append(g)

    def step_graph(self, q):
        """One decode by graph replay (``bind`` and ``capture`` first)."""
        self._require(bound=True, graphs=True)
        self._bound["q"].copy_(q)
        self.epoch += 1
        self._graphs[self.epoch & 1].replay()
        return self._bound["out"]

    def close(self):
        """Collective: every rank's kernels are done before any region is unmapped."""
        if self.bases is None:
            return
        self._graphs = None
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.pg)
        L = _lib.lib()
        with torch.cuda.device(self.device):
            for r, base in enumerate(self.bases):
                if r != self.rank:
                    _lib.check(L.akt_ipc_close(c_void_p(base)))
            if self.world > 1:
                dist.barrier(group=self.pg)
            _lib.check(L.akt_ipc_free(c_void_p(self.local)))
        self.bases = None
