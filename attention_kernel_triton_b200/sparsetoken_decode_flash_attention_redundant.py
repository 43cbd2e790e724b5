"""Sparse-token GQA decode over dense K/V -- drop-in for the reference module of the same name.

``sparsetoken_flash_attention_decode`` keeps the reference launcher's
signature and return shape ``[B, Hq, 1, D]``
(``sparsetoken_decode_flash_attention_redundant.py:127-170``).  Head ``h`` of
batch ``b`` attends only to tokens ``sparse_ind[b, h, 0:nnz]`` of kv head
``h // GQA_group_size``; ``sparse_nnz`` is ``[B, Hq]`` or ``[B, Hq, 1]``.
``nnz == 0`` gives zeros (the reference kernel would divide 0/0 there).
Runs the sm_100a gather kernel behind ``akt_sparse_dense``.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

redundant_len = 16  # reference module constant (SD:7)


def _sparse_dense_call(entry, out, q, K, V, sparse_ind, sparse_nnz, softmax_scale, GQA_group_size, partial=None,
                       csr=None, peer=None):
    """Shared launcher; ``partial=(o_part, lse_part)`` selects the partial-output entry point,
    ``csr=(sparse_ptr, max_nnz)`` the CSR-list one (``sparse_ind`` is then the flat index array)."""
    dev = _lib.require_cuda(q, K, V)
    if not (q.dtype == K.dtype == V.dtype) or (out is not None and out.dtype != q.dtype):
        raise TypeError("q, K, V and the output must share one dtype")
    B, Hq, _, D = q.shape
    Hkv = K.shape[1]
    assert Hq % Hkv == 0
    assert Hq // Hkv == GQA_group_size
    ind = _lib.as_int32(sparse_ind, dev)
    nnz = _lib.as_int32(sparse_nnz, dev) if csr is None else None
    ptr = _lib.as_int32(csr[0], dev) if csr is not None else None
    t = {"q": q, "K": K, "V": V}
    L = _lib.lib()
    fn = getattr(L, entry)

    def call():
        a = _lib.SparseDenseArgs()
        qq, KK, VV = t["q"], t["K"], t["V"]
        a.q = qq.data_ptr()
        a.q_stride_batch, a.q_stride_head, a.q_stride_dim = qq.stride(0), qq.stride(1), qq.stride(3)
        a.k = KK.data_ptr()
        a.k_stride_batch, a.k_stride_head, a.k_stride_token, a.k_stride_dim = KK.stride()
        a.v = VV.data_ptr()
        a.v_stride_batch, a.v_stride_head, a.v_stride_token, a.v_stride_dim = VV.stride()
        if csr is None:
            (a.ind_stride_batch, a.ind_stride_head, a.ind_stride_pos), (a.nnz_stride_batch, a.nnz_stride_head) = \
                _lib.index_strides(ind, nnz)
            a.sparse_ind, a.sparse_nnz = ind.data_ptr(), nnz.data_ptr()
            a.max_nnz = ind.shape[2]
        else:
            a.sparse_ind, a.max_nnz = ind.data_ptr(), int(csr[1])
        if out is not None:
            a.out = out.data_ptr()
            a.out_stride_batch, a.out_stride_head, a.out_stride_dim = out.stride(0), out.stride(1), out.stride(3)
        a.batch, a.num_qo_heads, a.num_kv_heads, a.seq_len, a.head_dim = B, Hq, Hkv, KK.shape[2], D
        a.dtype = _lib.dtype_code(qq)
        a.softmax_scale = float(softmax_scale)
        ws = _lib.workspace(L.akt_sparse_dense_workspace_size(ctypes.byref(a)), dev)
        if partial is not None:
            return fn(ctypes.byref(a), partial[0].data_ptr(), partial[1].data_ptr(), ws.data_ptr(), ws.numel(),
                      _lib.stream_ptr(dev))
        if csr is not None:
            return fn(ctypes.byref(a), ptr.data_ptr(), ind.numel(), ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
        if peer is not None:
            return fn(ctypes.byref(a), ctypes.byref(peer), ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
        return fn(ctypes.byref(a), ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))

    def contiguous():
        for k in t:
            t[k] = t[k].contiguous()

    with _lib.on_device(dev):
        _lib.run_with_layout_retry(call, contiguous)


def sparse_dense_into(out, q, K, V, sparse_ind, sparse_nnz, softmax_scale, GQA_group_size):
    """Write the sparse-token decode into ``out [B, Hq, 1, D]``."""
    _lib.require_cuda(out)
    _sparse_dense_call("akt_sparse_dense", out, q, K, V, sparse_ind, sparse_nnz, softmax_scale, GQA_group_size)
    return out


def sparse_dense_partial(o_part, lse_part, q, K, V, sparse_ind, sparse_nnz, softmax_scale, GQA_group_size):
    """Partial over this device's tokens: fp32 ``o_part [B, Hq, D]`` normalised over the
    kept tokens present in ``K``/``V``, natural-log ``lse_part [B, Hq]`` (-inf if none)."""
    _sparse_dense_call("akt_sparse_dense_partial", None, q, K, V, sparse_ind, sparse_nnz, softmax_scale,
                       GQA_group_size, partial=(o_part, lse_part))
    return o_part, lse_part


def sparsetoken_flash_attention_decode(q, K, V, sparse_ind, sparse_nnz, softmax_scale, GQA_group_size):
    """q [B,Hq,1,D], K/V [B,Hkv,S,D], sparse_ind [B,Hq,L_max] (-1 padded), sparse_nnz [B,Hq(,1)]
    -> O [B, Hq, 1, D] in q.dtype."""
    B, Hq, _, D = q.shape
    O = torch.empty((B, Hq, 1, D), dtype=q.dtype, device=q.device)
    return sparse_dense_into(O, q, K, V, sparse_ind, sparse_nnz, softmax_scale, GQA_group_size)


def sparsetoken_flash_attention_decode_csr(q, K, V, sparse_inds, sparse_ptr, softmax_scale, GQA_group_size,
                                           max_nnz):
    """CSR-list variant (the ``inds`` + ``ptr`` format of the reference's notes,
    ``sparse_decode_flash_attention.py:13-15``): head ``h`` of batch ``b`` keeps
    ``sparse_inds[sparse_ptr[b*Hq + h] : sparse_ptr[b*Hq + h + 1]]`` (ascending token positions).
    ``max_nnz`` (required) bounds the row lengths and sizes the split-KV scratch, so the
    call reads nothing back from the device; rows longer than it are cut there and the cut
    is recorded in the device status word (code 3).  -> O [B, Hq, 1, D]."""
    B, Hq, _, D = q.shape
    max_nnz = int(max_nnz)
    if max_nnz < 0:
        raise ValueError("max_nnz must be non-negative")
    O = torch.empty((B, Hq, 1, D), dtype=q.dtype, device=q.device)
    _lib.require_cuda(O, sparse_inds, sparse_ptr)
    assert sparse_ptr.numel() == B * Hq + 1, "sparse_ptr must hold B * Hq + 1 offsets"
    _sparse_dense_call("akt_sparse_dense_csr", O, q, K, V, sparse_inds.reshape(-1), None, softmax_scale,
                       GQA_group_size, csr=(sparse_ptr.reshape(-1), max_nnz))
    return O
