"""Keep mask <-> padded kept-index lists, on the device.

The sparse-token decodes take per-(batch, qo head) lists of kept token
positions, ``sparse_ind [B, H, L_max]`` (ascending, ``-1`` padded) with
``sparse_nnz [B, H, 1]``.  The reference builds them from a keep mask with a
Python loop that calls ``.item()`` per row
(``sparsetoken_decode_flash_attention_redundant.py:283-295``), and builds the
mask back (``precompute_mask``, same file :317-324) for its mask-based naive
check.  These two functions do the same on the GPU, asynchronously on the
current stream, with the reference's rules:

* :func:`sparse_index_from_mask` -- kept positions in ascending order, the rest
  ``-1``; an empty row keeps token 0 (``nnz = 1``).  A row with more than
  ``L_max`` kept tokens keeps the first ``L_max`` and records device status 5
  (the reference's slice assignment raises there).
* :func:`sparse_csr_from_lists` -- the padded lists as CSR (``inds`` + ``ptr``,
  the format the reference's notes propose, ``sparse_decode_flash_attention.py:13-15``),
  for the ``*_csr`` decode entry points.
* :func:`precompute_mask` -- ``nnz == 0`` reads as 1 and entries are Python
  indices, so a negative entry counts from the end (the ``-1`` padding of an
  empty list marks the last token, exactly as the reference loop does);
  entries outside ``[-L, L)`` are skipped and record device status 3 (the
  reference raises ``IndexError``).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


def sparse_index_from_mask(kept_mask: torch.Tensor, L_max: int, keep_first_if_empty: bool = True):
    """``kept_mask [B, H, L]`` (bool / uint8, CUDA) -> ``(sparse_ind [B, H, L_max] int32,
    sparse_nnz [B, H, 1] int32)``."""
    assert kept_mask.dim() == 3, "kept_mask must be [B, H, L]"
    assert L_max >= 0
    dev = _lib.require_cuda(kept_mask)
    if kept_mask.dtype not in (torch.bool, torch.uint8, torch.int8):
        kept_mask = kept_mask != 0
    if kept_mask.stride(2) != 1:
        kept_mask = kept_mask.contiguous()
    B, H, L = kept_mask.shape
    sparse_ind = torch.empty((B, H, L_max), dtype=torch.int32, device=dev)
    sparse_nnz = torch.empty((B, H, 1), dtype=torch.int32, device=dev)
    a = _lib.MaskToIndexArgs()
    a.mask = kept_mask.data_ptr()
    a.mask_stride_batch, a.mask_stride_head = kept_mask.stride(0), kept_mask.stride(1)
    a.sparse_ind = sparse_ind.data_ptr()
    a.ind_stride_batch, a.ind_stride_head = sparse_ind.stride(0), sparse_ind.stride(1)
    a.sparse_nnz = sparse_nnz.data_ptr()
    a.nnz_stride_batch, a.nnz_stride_head = sparse_nnz.stride(0), sparse_nnz.stride(1)
    a.batch, a.num_heads, a.seq_len, a.max_kept = B, H, L, L_max
    a.keep_first_if_empty = 1 if keep_first_if_empty else 0
    _lib.check(_lib.lib().akt_mask_to_sparse_index(ctypes.byref(a), _lib.stream_ptr(dev)))
    return sparse_ind, sparse_nnz


def precompute_mask(sparse_ind: torch.Tensor, sparse_nnz: torch.Tensor, SEQ_LEN: int) -> torch.Tensor:
    """``(sparse_ind [B, H, L_max], sparse_nnz [B, H(, 1)])`` -> ``mask [B, H, SEQ_LEN]`` bool."""
    dev = _lib.require_cuda(sparse_ind, sparse_nnz)
    sparse_ind = _lib.as_int32(sparse_ind, dev)
    sparse_nnz = _lib.as_int32(sparse_nnz, dev)
    if sparse_ind.dim() == 3 and sparse_ind.stride(2) != 1:
        sparse_ind = sparse_ind.contiguous()
    (isb, ish, _), (nsb, nsh) = _lib.index_strides(sparse_ind, sparse_nnz)
    B, H, L_max = sparse_ind.shape
    assert sparse_nnz.shape[0] == B and sparse_nnz.shape[1] == H
    mask = torch.empty((B, H, SEQ_LEN), dtype=torch.bool, device=dev)
    a = _lib.IndexToMaskArgs()
    a.sparse_ind = sparse_ind.data_ptr()
    a.ind_stride_batch, a.ind_stride_head = isb, ish
    a.sparse_nnz = sparse_nnz.data_ptr()
    a.nnz_stride_batch, a.nnz_stride_head = nsb, nsh
    a.mask = mask.data_ptr()
    a.mask_stride_batch, a.mask_stride_head = mask.stride(0), mask.stride(1)
    a.batch, a.num_heads, a.seq_len, a.max_kept = B, H, SEQ_LEN, L_max
    _lib.check(_lib.lib().akt_sparse_index_to_mask(ctypes.byref(a), _lib.stream_ptr(dev)))
    return mask


def sparse_csr_from_lists(sparse_ind: torch.Tensor, sparse_nnz: torch.Tensor):
    """Padded lists ``(sparse_ind [B, H, L_max], sparse_nnz [B, H(, 1)])`` -> CSR
    ``(inds [sum nnz] int32, ptr [B*H + 1] int32)``: row ``b*H + h`` is
    ``inds[ptr[b*H + h] : ptr[b*H + h + 1]]``, the first ``nnz`` entries of that list
    (``nnz`` clamped to ``[0, L_max]``).  Device-side torch ops; the boolean selection
    sizes its output, which costs one host synchronisation (a list-building step, not a
    decode launch)."""
    dev = _lib.require_cuda(sparse_ind, sparse_nnz)
    B, H, L_max = sparse_ind.shape
    n = sparse_nnz.reshape(B * H).to(torch.int64).clamp(0, L_max)
    ptr = torch.zeros(B * H + 1, dtype=torch.int64, device=dev)
    ptr[1:] = torch.cumsum(n, 0)
    keep = torch.arange(L_max, device=dev).unsqueeze(0) < n.unsqueeze(1)
    inds = sparse_ind.reshape(B * H, L_max)[keep].to(torch.int32)
    return inds, ptr.to(torch.int32)
