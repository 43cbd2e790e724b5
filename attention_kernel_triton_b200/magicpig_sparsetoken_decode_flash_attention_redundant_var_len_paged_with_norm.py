"""MagicPIG sparse-token paged decode with norm -- drop-in for the reference module of the same name.

``magicpig_sparsetoken_flash_attention_decode_paged`` keeps the reference
launcher's signature and return shape ``[B, Hq, D]`` in ``q.dtype``
(``magicpig_sparsetoken_decode_flash_attention_redundant_var_len_paged_with_norm.py:166-209``).
Each kept token's score is ``q.k/sqrt(D) - log(u)`` with
``u = 1 - (1-p^K)^L - L p^K (1-p^K)^(L-1)`` and ``p = 1 - acos(cos(q, k))/pi``
(clamps of the reference's naive code, MP:263-278); ``K`` and ``L`` are fp32
``[B, Hq]``.  ``nnz == 0`` gives zeros (MP:51-53).  The reference targets an
Ascend NPU (``torch_npu``); this module runs the sm_100a gather kernel behind
``akt_magicpig_paged``.
"""
from __future__ import annotations

import math

import torch

from .sparsetoken_decode_flash_attention_redundant_var_len_paged import csr_max_nnz, sparse_paged_call


def magicpig_sparsetoken_flash_attention_decode_paged(q, paged_kv_cache, kv_page_indptr, kv_page_indices, sparse_ind,
                                                      sparse_nnz, K, L):
    B, H_q, _, D = q.shape
    output = torch.empty((B, H_q, D), device=q.device, dtype=q.dtype)
    return sparse_paged_call("akt_magicpig_paged", output, q, paged_kv_cache, kv_page_indptr, kv_page_indices,
                             sparse_ind, sparse_nnz, 1.0 / math.sqrt(D), K=K, L=L)


def magicpig_sparsetoken_flash_attention_decode_paged_csr(q, paged_kv_cache, kv_page_indptr, kv_page_indices,
                                                          sparse_inds, sparse_ptr, K, L, max_nnz):
    """CSR-list variant: head ``h`` of batch ``b`` keeps
    ``sparse_inds[sparse_ptr[b*Hq + h] : sparse_ptr[b*Hq + h + 1]]`` (the ``inds`` + ``ptr``
    format of ``sparse_decode_flash_attention.py:13-15``).  ``max_nnz`` (required) bounds the
    row lengths and sizes the scratch; no device read.  -> O [B, Hq, D]."""
    B, H_q, _, D = q.shape
    assert sparse_ptr.numel() == B * H_q + 1, "sparse_ptr must hold B * Hq + 1 offsets"
    max_nnz = csr_max_nnz(max_nnz)
    output = torch.empty((B, H_q, D), device=q.device, dtype=q.dtype)
    return sparse_paged_call("akt_magicpig_paged_csr", output, q, paged_kv_cache, kv_page_indptr, kv_page_indices,
                             sparse_inds.reshape(-1), None, 1.0 / math.sqrt(D), K=K, L=L,
                             csr=(sparse_ptr.reshape(-1), max_nnz))
