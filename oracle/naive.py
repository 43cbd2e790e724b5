"""CPU oracle: restatements of the reference's naive PyTorch attention code.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (the package
``attention_kernel_triton_b200``) imports this module; only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
(``--impl reference`` and the ``cpu_baseline`` object) call it, always as the
checker or as the timed CPU baseline, never as the thing measured.

Parity pinning: ``tests/golden/make_golden.py`` runs the reference's *own*
naive functions (imported from the reference sources, CPU) on seeded inputs and
stores inputs + outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks every function here against those
fixtures.  So this oracle is pinned to the reference, not only to itself.

Each function follows the cited reference lines.  The file names are the
reference's module names:

* PF ``prefill_flash_attention.py``
* PV ``prefill_flash_attention_var_len_padding.py``
* DR ``decode_flash_attention_redundant.py``
* DP ``decode_flash_attention_redundant_var_len_paged.py``
* SD ``sparsetoken_decode_flash_attention_redundant.py``
* SP ``sparsetoken_decode_flash_attention_redundant_var_len_paged.py``
* MP ``magicpig_sparsetoken_decode_flash_attention_redundant_var_len_paged_with_norm.py``

All math is done in ``dtype`` (fp32 by default, fp64 for a high-precision
reference) on CPU copies of the inputs.  Deliberate, documented differences
from the reference's naive code (the product follows these too):

* empty paged sequence (``indptr[b] == indptr[b+1]``): zeros ``[Hq, D]``
  (DP:291-294 appends a tensor of the wrong rank there);
* ``sparse_nnz == 0``: zeros (SD:193-194 would read index ``-1``, i.e. the last
  token; SP:261-264 and MP:231-233 already give zeros);
* ``kv_last_page_len`` is clamped to ``[0, page_size]`` (slicing does the same).
"""
from __future__ import annotations

import math
from typing import Optional

import torch

F32 = torch.float32


def _c(t: torch.Tensor, dtype) -> torch.Tensor:
    return t.detach().to("cpu").to(dtype)


# ----------------------------------------------------------------------------
# prefill  (PF:415-425 / PV:428-438, nested in test_op)
# ----------------------------------------------------------------------------

def prefill_reference(Q, K, V, causal: bool, softmax_scale: float, GQA_group_size: int = 1,
                      dtype=F32, p_round: Optional[torch.dtype] = None) -> torch.Tensor:
    """``softmax(Q K^T * s [causal]) V`` with GQA (PF:415-425).

    The reference rounds the probabilities to fp16 before ``P @ V`` (PF:424);
    pass ``p_round=torch.float16`` to mirror that, default keeps them in
    ``dtype`` (the stricter oracle).  Causal masking is top-left aligned
    (``tril`` of an ``S x S`` ones matrix, PF:416, 421-423).
    """
    Q, K, V = _c(Q, dtype), _c(K, dtype), _c(V, dtype)
    S = Q.shape[2]
    if GQA_group_size > 1:
        K = K.repeat_interleave(GQA_group_size, dim=1)
        V = V.repeat_interleave(GQA_group_size, dim=1)
    P = torch.matmul(Q, K.transpose(-2, -1)) * softmax_scale
    if causal:
        mask = torch.tril(torch.ones((S, S), dtype=torch.bool))
        P = P.masked_fill(~mask, float("-inf"))
    P = torch.softmax(P, dim=-1)
    if p_round is not None:
        P = P.to(p_round).to(dtype)
    return torch.matmul(P, V)


def prefill_lse_reference(Q, K, V, causal: bool, softmax_scale: float, GQA_group_size: int = 1, varlen=None,
                          dtype=F32) -> torch.Tensor:
    """Per-row log-sum-exp of the scaled scores over the visible keys, the value the
    reference computes at PF:331 (``tmp_m_i += log(tmp_l_i)``) and does not store.
    Var-len padding rows (``i >= varlen[b]``) are -inf."""
    Q, K = _c(Q, dtype), _c(K, dtype)
    K = K.repeat_interleave(GQA_group_size, dim=1)
    S = Q.shape[2]
    s = torch.matmul(Q, K.transpose(-2, -1)) * softmax_scale
    if causal:
        s = s.masked_fill(~torch.tril(torch.ones(S, S, dtype=torch.bool)), float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    if varlen is not None:
        for b, n in enumerate(_c(torch.as_tensor(varlen), torch.int64).tolist()):
            lse[b, :, int(n):] = float("-inf")
    return lse


def prefill_varlen_reference(Q, K, V, causal: bool, softmax_scale: float, GQA_group_size: int,
                             varlen, dtype=F32, p_round=None) -> torch.Tensor:
    """PV:428-438 followed by the test's zeroing of padded rows (PV:447-450).

    The reference kernel masks no keys: only whole query blocks past a
    sequence's length are skipped (PV:186-187), and causality keeps every valid
    row inside its own length.  Rows ``i >= len_b`` are padding and are zero
    here; the product writes zeros there too."""
    O = prefill_reference(Q, K, V, causal, softmax_scale, GQA_group_size, dtype, p_round)
    lens = [int(x) for x in _c(varlen, torch.int64).tolist()]
    for b, l in enumerate(lens):
        O[b, :, max(l, 0):, :] = 0.0
    return O


# ----------------------------------------------------------------------------
# dense decode  (DR:306-312, nested in test_op_decode)
# ----------------------------------------------------------------------------

def decode_reference(q, K, V, softmax_scale: float, GQA_group_size: int = 1, dtype=F32,
                     p_round=None) -> torch.Tensor:
    """One-query attention over all L keys, no mask (DR:306-312) -> [B,Hq,1,D]."""
    q, K, V = _c(q, dtype), _c(K, dtype), _c(V, dtype)
    if GQA_group_size > 1:
        K = K.repeat_interleave(GQA_group_size, dim=1)
        V = V.repeat_interleave(GQA_group_size, dim=1)
    P = torch.matmul(q, K.transpose(-2, -1)) * softmax_scale
    P = torch.softmax(P, dim=-1)
    if p_round is not None:
        P = P.to(p_round).to(dtype)
    return torch.matmul(P, V)


# ----------------------------------------------------------------------------
# paged decode  (DP:278-329)
# ----------------------------------------------------------------------------

def naive_paged_attention(q, paged_kv_cache, kv_page_indptr, kv_page_indices, kv_last_page_len,
                          dtype=F32, batches=None) -> torch.Tensor:
    """Paged decode over the CSR page table (DP:278-329) -> [B, Hq, D].

    Sequence ``b`` is the pages ``indices[indptr[b]:indptr[b+1]]`` in order;
    its last page holds ``last_page_len[b]`` tokens (DP:305-308); GQA by
    ``repeat_interleave`` over the kv heads (DP:317-320); scale ``1/sqrt(D)``
    (DP:324).  ``batches`` restricts the computation to a subset of sequences
    (rows of other sequences are left zero) so that full-size cases can be
    checked on a sample.
    """
    q = _c(q, dtype)
    cache = paged_kv_cache.detach().to("cpu")
    indptr = _c(kv_page_indptr, torch.int64)
    indices = _c(kv_page_indices, torch.int64)
    last = _c(kv_last_page_len, torch.int64)
    B, Hq, _, D = q.shape
    Hkv, P = cache.shape[2], cache.shape[3]
    out = torch.zeros((B, Hq, D), dtype=dtype)
    for b in (range(B) if batches is None else batches):
        s, e = int(indptr[b]), int(indptr[b + 1])
        if s == e:
            continue
        pages = indices[s:e]
        kc = cache[pages, 0].to(dtype)      # [n, Hkv, P, D]
        vc = cache[pages, 1].to(dtype)
        n = e - s
        valid = (n - 1) * P + min(max(int(last[b]), 0), P)
        kseq = kc.permute(1, 0, 2, 3).reshape(Hkv, n * P, D)[:, :valid]
        vseq = vc.permute(1, 0, 2, 3).reshape(Hkv, n * P, D)[:, :valid]
        if Hq != Hkv:
            kseq = kseq.repeat_interleave(Hq // Hkv, dim=0)
            vseq = vseq.repeat_interleave(Hq // Hkv, dim=0)
        if valid == 0:
            continue
        scores = torch.matmul(q[b], kseq.transpose(1, 2)) / math.sqrt(D)   # [Hq,1,valid]
        w = torch.softmax(scores, dim=-1)
        out[b] = torch.matmul(w, vseq).squeeze(1)
    return out


def append_paged_kv_reference(paged_kv_cache, append_k, append_v, append_indptr, kv_page_indptr, kv_page_indices,
                              kv_last_page_len):
    """Write appended rows into a copy of the pool, one token at a time: sequence b holds
    ``(pages_b - 1) * P + last_b`` tokens after the append, the last ``n_b`` of them new;
    new row ``i`` goes to position ``len_b - n_b + i`` (page ``indices[indptr[b] + pos // P]``,
    row ``pos % P``), the addressing of the paged decode (DP:170-174)."""
    cache = paged_kv_cache.detach().cpu().clone()
    k, v = append_k.detach().cpu(), append_v.detach().cpu()
    ip = _c(kv_page_indptr, torch.int64).tolist()
    ind = _c(kv_page_indices, torch.int64).tolist()
    last = _c(kv_last_page_len, torch.int64).tolist()
    ap = _c(append_indptr, torch.int64).tolist()
    P = cache.shape[3]
    for b in range(len(ip) - 1):
        n = ap[b + 1] - ap[b]
        length = (ip[b + 1] - ip[b] - 1) * P + last[b]
        for i in range(n):
            pos = length - n + i
            page = ind[ip[b] + pos // P]
            cache[page, 0, :, pos % P] = k[ap[b] + i]
            cache[page, 1, :, pos % P] = v[ap[b] + i]
    return cache


# ----------------------------------------------------------------------------
# sparse-token decode, dense KV  (SD:173-230)
# ----------------------------------------------------------------------------

def sparsetoken_naive_decode(q, K, V, sparse_ind, sparse_nnz, softmax_scale, GQA_group_size,
                             dtype=F32) -> torch.Tensor:
    """Softmax over the kept tokens ``sparse_ind[b,h,:nnz]`` (SD:173-202) -> [B,Hq,1,D]."""
    q, K, V = _c(q, dtype), _c(K, dtype), _c(V, dtype)
    ind = _c(sparse_ind, torch.int64)
    B, Hq, _, D = q.shape
    nnz = _c(sparse_nnz, torch.int64).reshape(B, Hq)
    out = torch.zeros((B, Hq, 1, D), dtype=dtype)
    for b in range(B):
        for h in range(Hq):
            n = int(nnz[b, h])
            if n <= 0:
                continue
            kh = h // GQA_group_size
            idx = ind[b, h, :n]
            kv = K[b, kh, idx]
            vv = V[b, kh, idx]
            s = torch.matmul(kv, q[b, h, 0]) * softmax_scale
            out[b, h, 0] = torch.matmul(torch.softmax(s, 0).unsqueeze(0), vv)[0]
    return out


def sparsetoken_naive_decode_by_mask(q, K, V, sparse_ind, sparse_nnz, softmax_scale, GQA_group_size,
                                     mask, dtype=F32) -> torch.Tensor:
    """Dense attention with a boolean keep mask [B,Hq,L] (SD:204-230)."""
    q, K, V = _c(q, dtype), _c(K, dtype), _c(V, dtype)
    K = K.repeat_interleave(GQA_group_size, dim=1)
    V = V.repeat_interleave(GQA_group_size, dim=1)
    s = torch.matmul(q, K.transpose(-2, -1)) * softmax_scale
    s = s.masked_fill(~_c(mask, torch.bool).unsqueeze(2), float("-inf"))
    return torch.matmul(torch.softmax(s, dim=-1), V)


def sparse_lists_from_mask(kept_mask, L_max: int):
    """Kept-index lists from a per-row keep mask, as the reference's driver builds
    them (SD:283-295): ascending positions, the rest -1, an empty row keeps token 0.
    Returns ``(sparse_ind [B,H,L_max] int32, sparse_nnz [B,H,1] int32)``."""
    m = _c(kept_mask, torch.bool).clone()
    B, H, _ = m.shape
    ind = torch.full((B, H, L_max), -1, dtype=torch.int32)
    nnz = torch.zeros((B, H, 1), dtype=torch.int32)
    for b in range(B):
        for h in range(H):
            n = int(m[b, h].sum())
            if n == 0:
                n = 1
                m[b, h, 0] = True
            nnz[b, h, 0] = n
            ind[b, h, :n] = torch.nonzero(m[b, h], as_tuple=False).squeeze(-1)
    return ind, nnz


def sparse_lists_from_csr(inds, ptr, B: int, H: int):
    """CSR kept-index rows (``inds`` + ``ptr``, the format of SS:13-15; row ``b*H + h`` is
    ``inds[ptr[r]:ptr[r+1]]``) as the padded ``(sparse_ind, sparse_nnz)`` the naive
    references take; the padding length is the longest row (at least 1)."""
    inds, ptr = _c(inds, torch.int64), _c(ptr, torch.int64)
    n = (ptr[1:] - ptr[:-1]).reshape(B, H)
    L_max = max(int(n.max()) if n.numel() else 0, 1)
    ind = torch.full((B, H, L_max), -1, dtype=torch.int32)
    for b in range(B):
        for h in range(H):
            r = b * H + h
            ind[b, h, : int(n[b, h])] = inds[int(ptr[r]):int(ptr[r + 1])].to(torch.int32)
    return ind, n.to(torch.int32).unsqueeze(-1)


def sparse_mask_from_lists(sparse_ind, sparse_nnz, seq_len: int) -> torch.Tensor:
    """The keep mask the reference's driver builds from the lists (SD:315-324)."""
    ind = _c(sparse_ind, torch.int64)
    B, Hq, _ = ind.shape
    nnz = _c(sparse_nnz, torch.int64).reshape(B, Hq)
    m = torch.zeros((B, Hq, seq_len), dtype=torch.bool)
    for b in range(B):
        for h in range(Hq):
            n = max(int(nnz[b, h]), 1)
            m[b, h, ind[b, h, :n]] = True
    return m


# ----------------------------------------------------------------------------
# sparse-token decode, paged KV  (SP:234-288)
# ----------------------------------------------------------------------------

def _gather_paged_rows(cache, indptr, indices, b, kvh, toks, P):
    page = toks // P
    off = toks % P
    phys = indices[int(indptr[b]) + page]
    return cache[phys, 0, kvh, off], cache[phys, 1, kvh, off]


def sparsetoken_naive_paged_attention(q, paged_kv_cache, kv_page_indptr, kv_page_indices, sparse_ind,
                                      sparse_nnz, dtype=F32) -> torch.Tensor:
    """Kept tokens mapped through the page table (SP:234-288) -> [B, Hq, D].

    Token ``t`` of sequence ``b`` lives in physical page
    ``indices[indptr[b] + t // P]`` at row ``t % P`` (SP:271-276); scale
    ``1/sqrt(D)`` (SP:282); ``nnz == 0`` gives zeros (SP:261-264)."""
    q = _c(q, dtype)
    cache = paged_kv_cache.detach().to("cpu")
    indptr = _c(kv_page_indptr, torch.int64)
    indices = _c(kv_page_indices, torch.int64)
    ind = _c(sparse_ind, torch.int64)
    B, Hq, _, D = q.shape
    Hkv, P = cache.shape[2], cache.shape[3]
    G = Hq // Hkv
    nnz = _c(sparse_nnz, torch.int64).reshape(B, Hq)
    out = torch.zeros((B, Hq, D), dtype=dtype)
    for b in range(B):
        for h in range(Hq):
            n = int(nnz[b, h])
            if n <= 0:
                continue
            k, v = _gather_paged_rows(cache, indptr, indices, b, h // G, ind[b, h, :n], P)
            s = torch.matmul(k.to(dtype), q[b, h, 0]) / math.sqrt(D)
            out[b, h] = torch.matmul(torch.softmax(s, 0).unsqueeze(0), v.to(dtype))[0]
    return out


# ----------------------------------------------------------------------------
# MagicPIG sparse-token paged decode with norm  (MP:212-291; formula TODO.md:6)
# ----------------------------------------------------------------------------

def magicpig_logits(qv: torch.Tensor, k: torch.Tensor, K_val: float, L_val: float, D: int) -> torch.Tensor:
    """MagicPIG score ``q.k/sqrt(D) - log(u)`` for one head (MP:252-283).

    ``cos = q.k / (|q||k| + 1e-8)`` clamped to ``+-(1 - 1e-7)``;
    ``p = 1 - acos(cos)/pi`` clamped to [0, 1];
    ``u = 1 - (1 - p^K)^L - L p^K (1 - p^K)^(L-1)`` clamped below at 1e-10
    (the naive's clamp, MP:278; the reference kernel's ``u <= 0 -> 1e-10`` at
    MP:142 differs only on (0, 1e-10))."""
    scores = k @ qv
    q_norm = torch.linalg.vector_norm(qv)
    k_norm = torch.linalg.vector_norm(k, dim=-1)
    cos = scores / (q_norm * k_norm + 1e-8)
    cos = torch.clamp(cos, -1.0 + 1e-7, 1.0 - 1e-7)
    p = 1.0 - (1.0 / math.pi) * torch.acos(cos)
    p = torch.clamp(p, 0.0, 1.0)
    pK = torch.pow(p, K_val)
    omp = torch.clamp(1.0 - pK, 0.0, 1.0)
    u = 1.0 - torch.pow(omp, L_val) - L_val * pK * torch.pow(omp, L_val - 1.0)
    u = torch.clamp(u, min=1e-10)
    return scores / math.sqrt(D) - torch.log(u)


def magicpig_sparsetoken_naive_paged_attention(q, paged_kv_cache, kv_page_indptr, kv_page_indices,
                                               sparse_ind, sparse_nnz, K, L, dtype=F32) -> torch.Tensor:
    """MagicPIG estimator over the kept tokens (MP:212-291) -> [B, Hq, D].

    The reference computes in fp32 on ``q.float()``/``k.float()`` (MP:252-253)
    and returns ``q.dtype`` (MP:288); this returns ``dtype``."""
    q = _c(q, dtype)
    cache = paged_kv_cache.detach().to("cpu")
    indptr = _c(kv_page_indptr, torch.int64)
    indices = _c(kv_page_indices, torch.int64)
    ind = _c(sparse_ind, torch.int64)
    Kp = _c(K, torch.float64)
    Lp = _c(L, torch.float64)
    B, Hq, _, D = q.shape
    Hkv, P = cache.shape[2], cache.shape[3]
    G = Hq // Hkv
    nnz = _c(sparse_nnz, torch.int64).reshape(B, Hq)
    out = torch.zeros((B, Hq, D), dtype=dtype)
    for b in range(B):
        for h in range(Hq):
            n = int(nnz[b, h])
            if n <= 0:
                continue
            k, v = _gather_paged_rows(cache, indptr, indices, b, h // G, ind[b, h, :n], P)
            # .item() of an fp32 tensor: the exponents are fp32 values (MP:249-250)
            Kv = float(torch.tensor(float(Kp[b, h]), dtype=F32))
            Lv = float(torch.tensor(float(Lp[b, h]), dtype=F32))
            s = magicpig_logits(q[b, h, 0], k.to(dtype), Kv, Lv, D)
            out[b, h] = torch.matmul(torch.softmax(s, 0).unsqueeze(0), v.to(dtype))[0]
    return out


# ----------------------------------------------------------------------------
# log-sum-exp merge of split-KV partials (no reference counterpart)
# ----------------------------------------------------------------------------

def lse_merge_reference(o_parts: torch.Tensor, lse_parts: torch.Tensor) -> torch.Tensor:
    """``O = sum_j e^{lse_j - lse*} O_j / sum_j e^{lse_j - lse*}`` over dim 0.

    ``o_parts [n, ..., D]`` are per-part normalised outputs, ``lse_parts
    [n, ...]`` natural-log sum-exp of each part's scores (``-inf`` for an
    empty part)."""
    o = _c(o_parts, torch.float64)
    lse = _c(lse_parts, torch.float64)
    m = lse.max(0).values
    m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    w = torch.exp(lse - m)
    den = w.sum(0)
    num = (w.unsqueeze(-1) * o).sum(0)
    return torch.where(den.unsqueeze(-1) > 0, num / den.clamp_min(1e-300).unsqueeze(-1),
                       torch.zeros_like(num))
