"""Append tokens' K and V rows to a paged KV cache (the write path the paged
decodes read; the reference has none -- its drivers fill the pool in Python).

``append_paged_kv_cache`` writes, on the current stream, appended row ``i`` of
sequence ``b`` (row ``append_indptr[b] + i`` of ``append_k`` / ``append_v``,
``[num_append, Hkv, D]``) into the pool ``[num_pages, 2, Hkv, P, D]`` at
position ``len_b - n_b + i``, where the page table (``kv_page_indptr``,
``kv_page_indices``, ``kv_last_page_len``, the format of
``decode_flash_attention_redundant_var_len_paged.flash_attention_decode_paged``)
already describes the sequences *after* the append and ``n_b`` is the number
of appended rows of ``b``.  Runs ``akt_append_paged_kv`` (sm_100a).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


def append_paged_kv_cache(paged_kv_cache, append_k, append_v, append_indptr, kv_page_indptr, kv_page_indices,
                          kv_last_page_len):
    dev = _lib.require_cuda(paged_kv_cache, append_k, append_v)
    if not (paged_kv_cache.dtype == append_k.dtype == append_v.dtype):
        raise TypeError("the pool and the appended rows must share one dtype")
    if paged_kv_cache.dim() != 5 or paged_kv_cache.shape[1] != 2:
        raise ValueError("paged_kv_cache must be [num_pages, 2, Hkv, page_size, D]")
    _, _, Hkv, P, D = paged_kv_cache.shape
    assert append_k.dim() == 3 and append_k.shape[1:] == (Hkv, D), "append_k must be [num_append, Hkv, D]"
    assert append_v.shape == append_k.shape
    indptr = _lib.as_int32(kv_page_indptr, dev)
    indices = _lib.as_int32(kv_page_indices, dev)
    last = _lib.as_int32(kv_last_page_len, dev)
    app = _lib.as_int32(append_indptr, dev)
    B = indptr.numel() - 1
    assert app.numel() == B + 1 and last.numel() == B
    k = append_k if append_k.stride(2) == 1 else append_k.contiguous()
    v = append_v if append_v.stride(2) == 1 else append_v.contiguous()
    a = _lib.AppendPagedArgs()
    a.kv_cache = paged_kv_cache.data_ptr()
    (a.kv_stride_page, a.kv_stride_kv, a.kv_stride_head, a.kv_stride_token, a.kv_stride_dim) = paged_kv_cache.stride()
    a.num_pages = paged_kv_cache.shape[0]
    a.kv_page_indptr, a.kv_page_indices, a.kv_last_page_len = indptr.data_ptr(), indices.data_ptr(), last.data_ptr()
    a.num_page_entries = indices.numel()
    a.append_k, (a.k_stride_token, a.k_stride_head, a.k_stride_dim) = k.data_ptr(), k.stride()
    a.append_v, (a.v_stride_token, a.v_stride_head, a.v_stride_dim) = v.data_ptr(), v.stride()
    a.append_indptr, a.num_append = app.data_ptr(), k.shape[0]
    a.batch, a.num_kv_heads, a.page_size, a.head_dim = B, Hkv, P, D
    a.dtype = _lib.dtype_code(k)
    with _lib.on_device(dev):
        _lib.check(_lib.lib().akt_append_paged_kv(ctypes.byref(a), _lib.stream_ptr(dev)))
    return paged_kv_cache
