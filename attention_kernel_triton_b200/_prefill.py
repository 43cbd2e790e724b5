"""Shared launcher of the sm_100a prefill kernel (``akt_prefill``) for the two
prefill drop-in modules."""
from __future__ import annotations

import ctypes

import torch

from . import _lib


def prefill_into(O, Q, K, V, causal, softmax_scale, GQA_group_size, varlen=None, lse=None):
    """Write ``softmax(Q K^T * scale [causal]) V`` (GQA) into ``O [B, H, S, D]``; with
    ``lse`` (fp32 ``[B, H, S]``, token stride 1) also each row's natural-log sum-exp of the
    scaled scores over its visible keys (-inf for var-len padding rows)."""
    dev = _lib.require_cuda(Q, K, V, O)
    if lse is not None:
        _lib.require_cuda(lse)
        if lse.dtype != torch.float32 or lse.shape != O.shape[:3] or lse.stride(2) != 1:
            raise ValueError("lse must be fp32 [B, H, S] with token stride 1")
    if not (Q.dtype == K.dtype == V.dtype == O.dtype):
        raise TypeError("Q, K, V and the output must share one dtype")
    B, H, S, D = Q.shape
    lens = None
    if varlen is not None:
        lens = _lib.as_int32(torch.as_tensor(varlen), dev).contiguous()
        if lens.numel() != B:
            raise ValueError("varlen must hold one length per batch entry")
    t = {"Q": Q, "K": K, "V": V}
    L = _lib.lib()

    def call():
        a = _lib.PrefillArgs()
        qq, kk, vv = t["Q"], t["K"], t["V"]
        a.q = qq.data_ptr()
        a.q_stride_batch, a.q_stride_head, a.q_stride_token, a.q_stride_dim = qq.stride()
        a.k = kk.data_ptr()
        a.k_stride_batch, a.k_stride_head, a.k_stride_token, a.k_stride_dim = kk.stride()
        a.v = vv.data_ptr()
        a.v_stride_batch, a.v_stride_head, a.v_stride_token, a.v_stride_dim = vv.stride()
        a.out = O.data_ptr()
        a.out_stride_batch, a.out_stride_head, a.out_stride_token, a.out_stride_dim = O.stride()
        a.varlen = lens.data_ptr() if lens is not None else None
        a.batch, a.num_qo_heads, a.num_kv_heads, a.seq_len, a.head_dim = B, H, kk.shape[1], S, D
        a.causal = 1 if causal else 0
        a.dtype = _lib.dtype_code(qq)
        a.softmax_scale = float(softmax_scale)
        if lse is not None:
            return L.akt_prefill_with_lse(ctypes.byref(a), lse.data_ptr(), lse.stride(0), lse.stride(1),
                                          _lib.stream_ptr(dev))
        return L.akt_prefill(ctypes.byref(a), _lib.stream_ptr(dev))

    def contiguous():
        for k in t:
            t[k] = t[k].contiguous()

    with _lib.on_device(dev):
        _lib.run_with_layout_retry(call, contiguous)
    return O
