"""Causal / non-causal GQA prefill -- drop-in for the reference module of the same name.

``flash_attention_prefill(Q, K, V, causal, softmax_scale, GQA_group_size=1)``
keeps the reference launcher's signature, assertions and return shape
``[B, H, S, D]`` in ``Q.dtype`` (``prefill_flash_attention.py:342-383``).
Causal masking is top-left aligned (query i sees keys j <= i).  The work runs
on the tcgen05/TMEM flash-attention kernel behind ``akt_prefill``; any S is
accepted (the reference needs S to be a multiple of its tiles), head_dim 64
or 128.
"""
from __future__ import annotations

import torch

from ._prefill import prefill_into


def flash_attention_prefill(Q, K, V, causal, softmax_scale, GQA_group_size=1):
    B, H, S, D = Q.shape
    assert K.shape == (B, H // GQA_group_size, S, D)
    assert V.shape == (B, H // GQA_group_size, S, D)
    assert D % 64 == 0, "HEAD_DIM must be a multiple of 64?"
    O = torch.empty((B, H, S, D), dtype=Q.dtype, device=Q.device)
    return prefill_into(O, Q, K, V, causal, softmax_scale, GQA_group_size)


def flash_attention_prefill_with_lse(Q, K, V, causal, softmax_scale, GQA_group_size=1):
    """``flash_attention_prefill`` that also returns each row's log-sum-exp: ``(O, LSE)`` with
    LSE fp32 ``[B, H, S]`` = ``log(sum_j exp(q_i.k_j * softmax_scale))`` over the row's visible
    keys -- the value the reference computes and leaves unstored (``tmp_m_i +=
    tl.math.log(tmp_l_i)``, prefill_flash_attention.py:331-334); -inf for var-len padding rows."""
    B, H, S, D = Q.shape
    assert K.shape == (B, H // GQA_group_size, S, D)
    assert V.shape == (B, H // GQA_group_size, S, D)
    assert D % 64 == 0, "HEAD_DIM must be a multiple of 64?"
    O = torch.empty((B, H, S, D), dtype=Q.dtype, device=Q.device)
    LSE = torch.empty((B, H, S), dtype=torch.float32, device=Q.device)
    prefill_into(O, Q, K, V, causal, softmax_scale, GQA_group_size, lse=LSE)
    return O, LSE
