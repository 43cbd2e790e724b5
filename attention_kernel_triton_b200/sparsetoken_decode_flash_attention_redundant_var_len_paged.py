"""Sparse-token GQA decode over a paged KV cache -- drop-in for the reference module of the same name.

``sparsetoken_flash_attention_decode_paged`` keeps the reference launcher's
signature and return shape ``[B, Hq, D]``
(``sparsetoken_decode_flash_attention_redundant_var_len_paged.py:170-232``):
kept token ``t`` of sequence ``b`` is row ``t % page_size`` of physical page
``kv_page_indices[kv_page_indptr[b] + t // page_size]``; the scale is
``1/sqrt(D)``; ``nnz == 0`` gives zeros.  Runs the sm_100a gather kernel behind
``akt_sparse_paged``.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

redundant_len = 16  # reference module constant (SP:7)


def sparse_paged_call(entry, out, q, paged_kv_cache, kv_page_indptr, kv_page_indices, sparse_ind, sparse_nnz,
                      softmax_scale, K=None, L=None, csr=None, partial=None):
    """Shared launcher; ``csr=(sparse_ptr, max_nnz)`` selects a CSR-list entry point
    (``sparse_ind`` is then the flat index array and ``sparse_nnz`` is not used);
    ``partial=(o_part, lse_part)`` a partial-output one (``out`` is then None)."""
    dev = _lib.require_cuda(q, paged_kv_cache, *([out] if out is not None else []))
    if q.dtype != paged_kv_cache.dtype or (out is not None and out.dtype != q.dtype):
        raise TypeError("q, paged_kv_cache and the output must share one dtype")
    B, Hq, one, D = q.shape
    if paged_kv_cache.dim() != 5 or paged_kv_cache.shape[1] != 2 or paged_kv_cache.shape[4] != D:
        raise ValueError("paged_kv_cache must be [num_pages, 2, Hkv, page_size, D]")
    indptr = _lib.as_int32(kv_page_indptr, dev)
    indices = _lib.as_int32(kv_page_indices, dev)
    ind = _lib.as_int32(sparse_ind, dev)
    nnz = _lib.as_int32(sparse_nnz, dev) if csr is None else None
    ptr = _lib.as_int32(csr[0], dev) if csr is not None else None
    t = {"q": q, "cache": paged_kv_cache}
    if K is not None:
        t["K"] = K.to(device=dev, dtype=torch.float32)
        t["L"] = L.to(device=dev, dtype=torch.float32)
    lib = _lib.lib()
    fn = getattr(lib, entry)
    wsfn = getattr(lib, entry.replace("_csr", "").replace("_partial", "") + "_workspace_size")

    def call():
        a = _lib.SparsePagedArgs()
        qq, cache = t["q"], t["cache"]
        a.q = qq.data_ptr()
        a.q_stride_batch, a.q_stride_head, a.q_stride_dim = qq.stride(0), qq.stride(1), qq.stride(3)
        a.kv_cache = cache.data_ptr()
        (a.kv_stride_page, a.kv_stride_kv, a.kv_stride_head, a.kv_stride_token, a.kv_stride_dim) = cache.stride()
        a.num_pages = cache.shape[0]
        a.kv_page_indptr, a.kv_page_indices, a.num_page_entries = indptr.data_ptr(), indices.data_ptr(), indices.numel()
        if csr is None:
            (a.ind_stride_batch, a.ind_stride_head, a.ind_stride_pos), (a.nnz_stride_batch, a.nnz_stride_head) = \
                _lib.index_strides(ind, nnz)
            a.sparse_ind, a.sparse_nnz = ind.data_ptr(), nnz.data_ptr()
        else:
            a.sparse_ind = ind.data_ptr()
        if "K" in t:
            a.magicpig_k, a.magicpig_l = t["K"].data_ptr(), t["L"].data_ptr()
            if t["K"].shape != (B, Hq) or t["K"].stride() != t["L"].stride():
                t["K"], t["L"] = t["K"].reshape(B, Hq).contiguous(), t["L"].reshape(B, Hq).contiguous()
                a.magicpig_k, a.magicpig_l = t["K"].data_ptr(), t["L"].data_ptr()
            a.param_stride_batch, a.param_stride_head = t["K"].stride()
        if out is not None:
            a.out = out.data_ptr()
            a.out_stride_batch, a.out_stride_head, a.out_stride_dim = out.stride()
        a.batch, a.num_qo_heads, a.num_kv_heads = B, Hq, cache.shape[2]
        a.page_size, a.head_dim = cache.shape[3], D
        a.max_nnz = ind.shape[2] if csr is None else int(csr[1])
        a.dtype = _lib.dtype_code(qq)
        a.softmax_scale = float(softmax_scale)
        ws = _lib.workspace(wsfn(ctypes.byref(a)), dev)
        if partial is not None:
            return fn(ctypes.byref(a), partial[0].data_ptr(), partial[1].data_ptr(), ws.data_ptr(), ws.numel(),
                      _lib.stream_ptr(dev))
        if csr is not None:
            return fn(ctypes.byref(a), ptr.data_ptr(), ind.numel(), ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
        return fn(ctypes.byref(a), ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))

    def contiguous():
        t["q"], t["cache"] = t["q"].contiguous(), t["cache"].contiguous()

    with _lib.on_device(dev):
        _lib.run_with_layout_retry(call, contiguous)
    return out


def sparsetoken_flash_attention_decode_paged(q, paged_kv_cache, kv_page_indptr, kv_page_indices, sparse_ind,
                                             sparse_nnz):
    """q [B,Hq,1,D], paged_kv_cache [pages,2,Hkv,P,D], CSR page table, sparse_ind [B,Hq,L_max],
    sparse_nnz [B,Hq(,1)] -> O [B, Hq, D] in q.dtype."""
    B, Hq, _, D = q.shape
    O = torch.empty((B, Hq, D), dtype=q.dtype, device=q.device)
    return sparse_paged_call("akt_sparse_paged", O, q, paged_kv_cache, kv_page_indptr, kv_page_indices, sparse_ind,
                             sparse_nnz, 1.0 / math.sqrt(D))


def csr_max_nnz(max_nnz) -> int:
    """The caller's bound on CSR row length, checked (no device read)."""
    max_nnz = int(max_nnz)
    if max_nnz < 0:
        raise ValueError("max_nnz must be non-negative")
    return max_nnz


def sparsetoken_flash_attention_decode_paged_csr(q, paged_kv_cache, kv_page_indptr, kv_page_indices, sparse_inds,
                                                 sparse_ptr, max_nnz):
    """CSR-list variant (``inds`` + ``ptr``, the format of the reference's notes,
    ``sparse_decode_flash_attention.py:13-15``): head ``h`` of batch ``b`` keeps
    ``sparse_inds[sparse_ptr[b*Hq + h] : sparse_ptr[b*Hq + h + 1]]``.  ``max_nnz`` (required)
    bounds the row lengths and sizes the scratch, so nothing is read back from the device;
    longer rows are cut there and the cut is recorded (status 3).  -> O [B, Hq, D]."""
    B, Hq, _, D = q.shape
    assert sparse_ptr.numel() == B * Hq + 1, "sparse_ptr must hold B * Hq + 1 offsets"
    max_nnz = csr_max_nnz(max_nnz)
    O = torch.empty((B, Hq, D), dtype=q.dtype, device=q.device)
    return sparse_paged_call("akt_sparse_paged_csr", O, q, paged_kv_cache, kv_page_indptr, kv_page_indices,
                             sparse_inds.reshape(-1), None, 1.0 / math.sqrt(D),
                             csr=(sparse_ptr.reshape(-1), max_nnz))


def sparse_paged_partial(o_part, lse_part, q, paged_kv_cache, kv_page_indptr, kv_page_indices, sparse_ind,
                         sparse_nnz, K=None, L=None):
    """Partial over the kept tokens this device's page table holds: fp32 ``o_part [B, Hq, D]``
    normalised over them and natural-log ``lse_part [B, Hq]`` (-inf for none).  With MagicPIG
    parameters ``K``, ``L`` ``[B, Hq]`` the scores are the MagicPIG estimator's.  Runs
    ``akt_sparse_paged_partial`` / ``akt_magicpig_paged_partial``."""
    _lib.require_cuda(o_part, lse_part)
    if o_part.dtype != torch.float32 or lse_part.dtype != torch.float32:
        raise TypeError("partials are fp32")
    if not (o_part.is_contiguous() and lse_part.is_contiguous()):
        raise ValueError("partials must be contiguous [B, Hq, D] and [B, Hq]")
    D = q.shape[3]
    entry = "akt_magicpig_paged_partial" if K is not None else "akt_sparse_paged_partial"
    sparse_paged_call(entry, None, q, paged_kv_cache, kv_page_indptr, kv_page_indices, sparse_ind, sparse_nnz,
                      1.0 / math.sqrt(D), K=K, L=L, partial=(o_part, lse_part))
    return o_part, lse_part
