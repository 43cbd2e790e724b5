"""Dense ("redundant") GQA decode -- drop-in for the reference module of the same name.

``flash_attention_decode(q, K, V, softmax_scale, GQA_group_size=1)`` keeps the
reference launcher's signature, assertions and return shape ``[B, Hq, 1, D]``
(``decode_flash_attention_redundant.py:233-271``).  The reference replicates q
16 times because its tensor-core dot needs M >= 16 (DR:235); the sm_100a
split-KV kernel behind ``akt_decode_dense`` needs no replication: it reads
each K/V byte once for the whole GQA group.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

q_redundant_len = 16  # reference module constant (DR:5)


def _dense_args(q, K, V, out, scale) -> _lib.DecodeDenseArgs:
    B, Hq, _, D = q.shape
    a = _lib.DecodeDenseArgs()
    a.q = q.data_ptr()
    a.q_stride_batch, a.q_stride_head, a.q_stride_dim = q.stride(0), q.stride(1), q.stride(3)
    a.k = K.data_ptr()
    a.k_stride_batch, a.k_stride_head, a.k_stride_token, a.k_stride_dim = K.stride()
    a.v = V.data_ptr()
    a.v_stride_batch, a.v_stride_head, a.v_stride_token, a.v_stride_dim = V.stride()
    a.out = out.data_ptr()
    a.out_stride_batch, a.out_stride_head, a.out_stride_dim = out.stride(0), out.stride(1), out.stride(3)
    a.batch, a.num_qo_heads, a.num_kv_heads = B, Hq, K.shape[1]
    a.seq_len, a.head_dim = K.shape[2], D
    a.dtype = _lib.dtype_code(q)
    a.softmax_scale = float(scale)
    return a


def decode_dense_into(out, q, K, V, softmax_scale):
    """Write the decode of ``q [B,Hq,1,D]`` over ``K, V [B,Hkv,L,D]`` into ``out [B,Hq,1,D]``."""
    dev = _lib.require_cuda(q, K, V, out)
    if not (q.dtype == K.dtype == V.dtype == out.dtype):
        raise TypeError("q, K, V and the output must share one dtype")
    L = _lib.lib()
    qq, KK, VV = q, K, V
    with _lib.on_device(dev):
        for attempt in range(2):
            a = _dense_args(qq, KK, VV, out, softmax_scale)
            ws = _lib.workspace(L.akt_decode_dense_workspace_size(ctypes.byref(a)), dev)
            rc = L.akt_decode_dense(ctypes.byref(a), ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
            if rc == _lib.AKT_ERR_UNSUPPORTED and attempt == 0:
                qq, KK, VV = qq.contiguous(), KK.contiguous(), VV.contiguous()
                continue
            _lib.check(rc)
            break
    return out


def flash_attention_decode(q, K, V, softmax_scale, GQA_group_size=1):
    """q [B, H*G, 1, D], K/V [B, H, S, D] -> O [B, H*G, 1, D] in q.dtype."""
    B, H, S, D = K.shape
    assert q.shape == (B, H * GQA_group_size, 1, D)
    assert V.shape == (B, H, S, D)
    assert D % 64 == 0, "HEAD_DIM must be a multiple of 64?"
    O = torch.empty((B, H * GQA_group_size, 1, D), dtype=q.dtype, device=q.device)
    return decode_dense_into(O, q, K, V, softmax_scale)
