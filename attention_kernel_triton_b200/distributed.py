"""Multi-GPU partitioning of the decode paths on one box.

Two layouts, following the structure of the work:

* Independent units (every path): batches or kv heads are split across GPUs
  and each GPU runs the single-GPU kernels on its share -- no communication.
  ``shard_range`` gives each rank its contiguous slice.
* One long sequence, sparse-token decode: the key axis is split into
  contiguous token ranges, one per rank.  Each rank runs the sparse kernel in
  partial-output mode over its range (fp32 O normalised over its kept tokens
  and the natural-log sum-exp), the ``[O | LSE]`` partials are all-gathered
  over NCCL (NVLink) and merged with ``akt_lse_merge``:
  ``O = sum_r e^{lse_r - M} O_r / sum_r e^{lse_r - M}``.

The reference has no multi-GPU code; this is the exchange step BASELINE's
north star names for the 128K single-sequence case.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous, balanced slice ``[lo, hi)`` of ``n`` items for ``rank``."""
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_sparse_lists(sparse_ind: torch.Tensor, sparse_nnz: torch.Tensor, lo: int, hi: int):
    """Kept-token lists restricted to tokens ``[lo, hi)`` and rebased to ``lo``.

    Lists are sorted ascending (the reference builds them with ``nonzero``,
    SD:294).  Returns ``(ind [B, Hq, L_local] int32, -1 padded, nnz [B, Hq, 1])``
    with ``L_local`` the longest local list (at least 1)."""
    B, Hq, Lmax = sparse_ind.shape
    ind = sparse_ind.to(torch.int64)
    nnz = sparse_nnz.reshape(B, Hq, 1).to(torch.int64)
    pos = torch.arange(Lmax, device=ind.device).view(1, 1, Lmax)
    big = torch.iinfo(torch.int64).max
    srt = torch.where(pos < nnz, ind, torch.full_like(ind, big)).reshape(B * Hq, Lmax).contiguous()
    bounds = torch.tensor([lo, hi], dtype=torch.int64, device=ind.device).expand(B * Hq, 2).contiguous()
    se = torch.searchsorted(srt, bounds)  # first index >= lo, first index >= hi
    cnt = (se[:, 1] - se[:, 0]).clamp_min(0)
    L_loc = max(int(cnt.max().item()) if cnt.numel() else 0, 1)
    j = torch.arange(L_loc, device=ind.device).view(1, L_loc)
    src = (se[:, :1] + j).clamp_max(Lmax - 1)
    vals = torch.gather(srt, 1, src) - lo
    local = torch.where(j < cnt.view(-1, 1), vals, torch.full_like(vals, -1))
    return local.view(B, Hq, L_loc).to(torch.int32), cnt.view(B, Hq, 1).to(torch.int32)


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
