"""Padded var-len causal GQA prefill -- drop-in for the reference module of the same name.

``flash_attention_prefill(Q, K, V, causal, softmax_scale, GQA_group_size=1,
varlen=None)`` keeps the reference launcher's signature, assertions and return
shape (``prefill_flash_attention_var_len_padding.py:348-391``).  ``varlen``
holds each sequence's valid length; query rows past it are padding.  The
reference skips whole query blocks past the length (PV:186-187) and leaves
them unwritten; here every padding row is written as zeros (the reference's
test zeroes them on both sides before comparing, PV:447-450).  Keys are not
masked by ``varlen`` (the reference does not either: causality keeps valid rows
inside their own length).
"""
from __future__ import annotations

import torch

from ._prefill import prefill_into


def flash_attention_prefill(Q, K, V, causal, softmax_scale, GQA_group_size=1, varlen=None):
    B, H, S, D = Q.shape
    assert K.shape == (B, H // GQA_group_size, S, D)
    assert V.shape == (B, H // GQA_group_size, S, D)
    assert D % 64 == 0, "HEAD_DIM must be a multiple of 64?"
    O = torch.empty((B, H, S, D), dtype=Q.dtype, device=Q.device)
    return prefill_into(O, Q, K, V, causal, softmax_scale, GQA_group_size, varlen)


def flash_attention_prefill_with_lse(Q, K, V, causal, softmax_scale, GQA_group_size=1, varlen=None):
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
    prefill_into(O, Q, K, V, causal, softmax_scale, GQA_group_size, varlen, lse=LSE)
    return O, LSE
