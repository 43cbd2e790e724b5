"""Paged var-len GQA decode -- drop-in for the reference module of the same name.

``flash_attention_decode_paged`` keeps the reference launcher's signature,
argument meaning, return shape ``[B, Hq, D]`` and assertion
(``decode_flash_attention_redundant_var_len_paged.py:228-274``).  The work is
done by the sm_100a split-KV kernel behind ``akt_decode_paged`` (C ABI,
``include/akt.h``) on torch's current stream.

Page table (FlashInfer-style CSR, as in the reference): sequence ``b`` owns
pages ``kv_page_indices[kv_page_indptr[b]:kv_page_indptr[b+1]]`` of the pool
``paged_kv_cache [num_pages, 2, Hkv, page_size, D]``; its last page holds
``kv_last_page_len[b]`` tokens.  An empty sequence gives zeros (the reference
kernel leaves 0/0 there, DP:167).
"""
from __future__ import annotations

import ctypes
import math
import os

import torch

from . import _lib

redundant_len = 16  # reference module constant (DP:8); kept for drop-in imports


def _as_i32(t: torch.Tensor, device) -> torch.Tensor:
    if t.dtype != torch.int32 or t.device != device or not t.is_contiguous():
        t = t.to(device=device, dtype=torch.int32).contiguous()
    return t


def _paged_args(q, cache, indptr, indices, last, out, scale) -> _lib.DecodePagedArgs:
    B, Hq, _, D = q.shape
    a = _lib.DecodePagedArgs()
    a.q = q.data_ptr()
    a.q_stride_batch, a.q_stride_head, a.q_stride_dim = q.stride(0), q.stride(1), q.stride(3)
    a.kv_cache = cache.data_ptr()
    (a.kv_stride_page, a.kv_stride_kv, a.kv_stride_head,
     a.kv_stride_token, a.kv_stride_dim) = cache.stride()
    a.num_pages = cache.shape[0]
    a.kv_page_indptr = indptr.data_ptr()
    a.kv_page_indices = indices.data_ptr()
    a.kv_last_page_len = last.data_ptr()
    a.num_page_entries = indices.numel()
    a.out = out.data_ptr()
    a.out_stride_batch, a.out_stride_head, a.out_stride_dim = out.stride()
    a.batch, a.num_qo_heads, a.num_kv_heads = B, Hq, cache.shape[2]
    a.page_size, a.head_dim = cache.shape[3], D
    a.dtype = _lib.dtype_code(q)
    a.softmax_scale = float(scale)
    return a


def decode_paged_into(out, q, paged_kv_cache, kv_page_indptr, kv_page_indices, kv_last_page_len,
                      softmax_scale=None):
    """Write the paged decode of ``q`` into ``out [B, Hq, D]`` (no allocation of the output)."""
    dev = _lib.require_cuda(q, paged_kv_cache, out)
    if q.dtype != paged_kv_cache.dtype or out.dtype != q.dtype:
        raise TypeError("q, paged_kv_cache and the output must share one dtype")
    B, Hq, one, D = q.shape
    if one != 1:
        raise ValueError("q must be [B, Hq, 1, D]")
    if paged_kv_cache.dim() != 5 or paged_kv_cache.shape[1] != 2 or paged_kv_cache.shape[4] != D:
        raise ValueError("paged_kv_cache must be [num_pages, 2, Hkv, page_size, D]")
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    indptr = _as_i32(kv_page_indptr, dev)
    indices = _as_i32(kv_page_indices, dev)
    last = _as_i32(kv_last_page_len, dev)
    if indptr.numel() != B + 1 or last.numel() != B:
        raise ValueError("kv_page_indptr must have B+1 entries and kv_last_page_len B entries")
    qq = q if q.stride(3) == 1 else q.contiguous()
    cache = paged_kv_cache
    L = _lib.lib()
    with _lib.on_device(dev):
        for attempt in range(2):
            a = _paged_args(qq, cache, indptr, indices, last, out, scale)
            ws = _lib.workspace(L.akt_decode_paged_workspace_size(ctypes.byref(a)), dev)
            rc = L.akt_decode_paged(ctypes.byref(a), ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
            if rc == _lib.AKT_ERR_UNSUPPORTED and attempt == 0:
                qq, cache = qq.contiguous(), cache.contiguous()
                continue
            _lib.check(rc)
            break
    return out


def flash_attention_decode_paged(q, paged_kv_cache, kv_page_indptr, kv_page_indices, kv_last_page_len):
    """
    q: [B, H*GQA_group_size, 1, D]
    paged_kv_cache: [all_num_pages, 2, H, page_size, D] (2 for k and v)
    kv_page_indptr: [B+1] (int32)
    kv_page_indices: [total_num_pages] (int32)
    kv_last_page_len: [B] (int32)
    returns O: [B, H*GQA_group_size, D] in q.dtype, scale 1/sqrt(D)
    """
    page_size = paged_kv_cache.shape[3]
    # the reference's tile-size check on its env knob (DP:255-257); the CUDA
    # kernel picks its own tiles, so the knob only gates what the reference gated
    blk = int(os.environ.get("VAR_KV_SEQ_BLK_SIZE", 16))
    assert blk <= page_size and page_size % blk == 0, "page_size must be multiple of VAR_KV_SEQ_BLK_SIZE"
    B, Hq, _, D = q.shape
    O = torch.empty((B, Hq, D), dtype=q.dtype, device=q.device)
    return decode_paged_into(O, q, paged_kv_cache, kv_page_indptr, kv_page_indices, kv_last_page_len)
