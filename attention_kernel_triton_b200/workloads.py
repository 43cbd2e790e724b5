"""Seeded synthetic inputs for the five attention paths.

Every generator is deterministic for a given ``seed`` and ``device``: values
come from a ``torch.Generator`` seeded with ``seed`` on that device (a CPU
generator and a CUDA generator give different streams, so a parity check always
feeds the *same* tensors to the GPU path and to the CPU oracle by copying).

Shapes and value distributions follow the benchmark configurations of the
project (Q/K/V iid N(0,1) fp16, var-len lengths from the seed, paged pools in a
seeded random physical page order, per-(kv-head, token) Bernoulli keep masks)
and the input builders of the reference's own test drivers:

* prefill inputs: ``prefill_flash_attention.py:387-407``
* var-len lengths (``Ls[0] = S``): ``prefill_flash_attention_var_len_padding.py:418-419``
* CSR page table ``(indptr, indices, last_page_len)`` and pool layout
  ``[pages, 2, Hkv, P, D]``: ``decode_flash_attention_redundant_var_len_paged.py:228-235, 337-353``
* sparse index lists (sorted ``nonzero`` of a Bernoulli mask, ``nnz >= 1`` forced
  by keeping token 0, ``-1`` padding): ``sparsetoken_decode_flash_attention_redundant.py:277-295``,
  ``sparsetoken_decode_flash_attention_redundant_var_len_paged.py:333-353``
* MagicPIG ``K, L = rand * 5 + 1``: ``magicpig_sparsetoken_decode_flash_attention_redundant_var_len_paged_with_norm.py:344-345``
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional, Sequence

import torch


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=torch.device(device))
    g.manual_seed(int(seed))
    return g


def randn(shape, g: torch.Generator, device, dtype=torch.float16, std: float = 1.0) -> torch.Tensor:
    """iid N(0, std^2) in fp32, rounded once to ``dtype``."""
    t = torch.randn(tuple(shape), generator=g, device=device, dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    return t.to(dtype)


# ----------------------------------------------------------------------------
# prefill (dense and padded var-len)
# ----------------------------------------------------------------------------

@dataclass
class PrefillCase:
    Q: torch.Tensor
    K: torch.Tensor
    V: torch.Tensor
    causal: bool
    softmax_scale: float
    group: int
    varlen: Optional[torch.Tensor] = None

    @property
    def flops(self) -> float:
        """Algorithmic FLOPs: 4*D per (query, key) pair actually attended.

        Causal counts ``S(S+1)/2`` pairs per head, var-len counts only the
        valid ``len_b (len_b + 1)/2`` pairs (padding is not counted)."""
        B, H, S, D = self.Q.shape
        if self.varlen is not None:
            lens = [int(x) for x in self.varlen.tolist()]
            if self.causal:
                pairs = sum(l * (l + 1) // 2 for l in lens)
            else:
                pairs = sum(l * S for l in lens)
            return 4.0 * H * D * pairs
        pairs = S * (S + 1) // 2 if self.causal else S * S
        return 4.0 * B * H * D * pairs


def make_prefill(B=8, Hq=64, Hkv=16, S=1024, D=64, causal=True, seed=0,
                 device="cpu", dtype=torch.float16, std=1.0, varlen=False,
                 min_len=64) -> PrefillCase:
    g = _gen(seed, device)
    Q = randn((B, Hq, S, D), g, device, dtype, std)
    K = randn((B, Hkv, S, D), g, device, dtype, std)
    V = randn((B, Hkv, S, D), g, device, dtype, std)
    lens = None
    if varlen:
        # first sequence at full length, the rest uniform in [min_len, S]
        lens = torch.randint(min_len, S + 1, (B,), generator=g, device=device, dtype=torch.int64)
        lens[0] = S
        lens = lens.to(torch.int32)
    return PrefillCase(Q, K, V, causal, 1.0 / math.sqrt(D), Hq // Hkv, lens)


# ----------------------------------------------------------------------------
# dense ("redundant") decode
# ----------------------------------------------------------------------------

@dataclass
class DecodeCase:
    q: torch.Tensor
    K: torch.Tensor
    V: torch.Tensor
    softmax_scale: float
    group: int

    @property
    def bytes(self) -> float:
        """Algorithmic HBM bytes: K + V once, q read once, O written once."""
        return float(self.K.numel() * self.K.element_size() * 2
                     + 2 * self.q.numel() * self.q.element_size())


def make_decode(B=8, Hq=64, Hkv=16, L=1024, D=64, seed=0, device="cpu",
                dtype=torch.float16, std=1.0) -> DecodeCase:
    g = _gen(seed, device)
    q = randn((B, Hq, 1, D), g, device, dtype, std)
    K = randn((B, Hkv, L, D), g, device, dtype, std)
    V = randn((B, Hkv, L, D), g, device, dtype, std)
    return DecodeCase(q, K, V, 1.0 / math.sqrt(D), Hq // Hkv)


# ----------------------------------------------------------------------------
# paged var-len decode
# ----------------------------------------------------------------------------

@dataclass
class PagedCase:
    q: torch.Tensor                 # [B, Hq, 1, D]
    cache: torch.Tensor             # [N, 2, Hkv, P, D]
    indptr: torch.Tensor            # [B+1] int32
    indices: torch.Tensor           # [N] int32
    last_page_len: torch.Tensor     # [B] int32
    seq_lens: torch.Tensor          # [B] int32 (host-side bookkeeping)
    block_table: torch.Tensor = field(default=None)  # [B, max_pages] int32, -1 padded

    @property
    def bytes(self) -> float:
        """Algorithmic HBM bytes: every valid token's K and V once per kv head,
        q and O once, plus the page-table metadata."""
        B, Hq, _, D = self.q.shape
        Hkv = self.cache.shape[2]
        es = self.cache.element_size()
        toks = int(self.seq_lens.sum())
        meta = 4 * (self.indices.numel() + self.indptr.numel() + self.last_page_len.numel())
        return float(toks * Hkv * D * es * 2 + 2 * B * Hq * D * self.q.element_size() + meta)


def paged_layout_from_lens(lens: Sequence[int], page_size: int, g: torch.Generator,
                           device="cpu", permute=True):
    """CSR page table for the given sequence lengths.

    Pages are numbered ``0..N-1`` with ``N = sum(ceil(len/P))`` and placed in a
    seeded random physical order (``randperm``), as the reference's paged test
    drivers do (``sparsetoken_decode_flash_attention_redundant_var_len_paged.py:322-327``).
    A zero-length sequence owns no pages; its ``last_page_len`` is 0.
    """
    lens = [int(l) for l in lens]
    pages = [(l + page_size - 1) // page_size for l in lens]
    N = sum(pages)
    perm = torch.randperm(N, generator=g, device=device) if permute else torch.arange(N, device=device)
    indices = perm.to(torch.int32)
    indptr = torch.zeros(len(lens) + 1, dtype=torch.int32)
    indptr[1:] = torch.cumsum(torch.tensor(pages, dtype=torch.int64), 0).to(torch.int32)
    last = torch.tensor([l - page_size * (p - 1) if p > 0 else 0 for l, p in zip(lens, pages)],
                        dtype=torch.int32)
    maxp = max(pages) if pages else 0
    bt = torch.full((len(lens), max(maxp, 1)), -1, dtype=torch.int32)
    ind_cpu = indices.cpu()
    for b in range(len(lens)):
        s, e = int(indptr[b]), int(indptr[b + 1])
        bt[b, : e - s] = ind_cpu[s:e]
    return (indptr.to(device), indices, last.to(device), torch.tensor(lens, dtype=torch.int32),
            bt.to(device), N)


def make_paged(B=64, Hq=32, Hkv=8, D=128, page_size=16, min_len=512, max_len=32768,
               lens: Optional[Sequence[int]] = None, seed=0, device="cpu",
               dtype=torch.float16, std=1.0, extra_pages=0) -> PagedCase:
    g = _gen(seed, device)
    if lens is None:
        lens = torch.randint(min_len, max_len + 1, (B,), generator=_gen(seed + 7919, "cpu")).tolist()
    indptr, indices, last, seq_lens, bt, N = paged_layout_from_lens(lens, page_size, g, device)
    cache = randn((N + extra_pages, 2, Hkv, page_size, D), g, device, dtype, std)
    q = randn((len(lens), Hq, 1, D), g, device, dtype, std)
    return PagedCase(q, cache, indptr, indices, last, seq_lens, bt)


# ----------------------------------------------------------------------------
# sparse-token decode (dense KV, paged KV, MagicPIG)
# ----------------------------------------------------------------------------

def sparse_lists(seq_lens: Sequence[int], Hkv: int, group: int, keep_p: float, L_max: int,
                 g: torch.Generator, device="cpu", per_qo_head=False):
    """Sorted kept-token index lists, ``-1`` padded to ``L_max``.

    One Bernoulli(keep_p) mask per (batch, kv-head) over that sequence's
    tokens, repeated over the ``group`` qo-heads of the kv head (set
    ``per_qo_head`` to draw an independent mask per qo head instead, as the
    reference's own drivers do).  An empty mask keeps token 0 (the reference
    forces ``nnz >= 1`` the same way).  Returns ``(sparse_ind [B,Hq,L_max]
    int32, sparse_nnz [B,Hq,1] int32)``.
    """
    B = len(seq_lens)
    Hq = Hkv * group
    ind = torch.full((B, Hq, L_max), -1, dtype=torch.int32, device=device)
    nnz = torch.zeros((B, Hq, 1), dtype=torch.int32, device=device)
    heads = Hq if per_qo_head else Hkv
    for b in range(B):
        n = int(seq_lens[b])
        if n == 0:
            continue
        u = torch.rand((heads, n), generator=g, device=device)
        keep = u < keep_p
        keep[keep.sum(1) == 0, 0] = True
        for h in range(heads):
            idx = torch.nonzero(keep[h], as_tuple=False).squeeze(-1).to(torch.int32)
            k = min(idx.numel(), L_max)
            targets = [h] if per_qo_head else range(h * group, (h + 1) * group)
            for hq in targets:
                ind[b, hq, :k] = idx[:k]
                nnz[b, hq, 0] = k
    return ind, nnz


@dataclass
class SparseDenseCase:
    q: torch.Tensor
    K: torch.Tensor
    V: torch.Tensor
    sparse_ind: torch.Tensor
    sparse_nnz: torch.Tensor
    softmax_scale: float
    group: int

    @property
    def bytes(self) -> float:
        """Gathered K+V rows once per kv head (the group shares one list),
        the index lists read, q and O once."""
        B, Hq, _, D = self.q.shape
        es = self.K.element_size()
        nnz = self.sparse_nnz.reshape(B, Hq)
        kv_rows = int(nnz[:, :: self.group].sum())
        return float(kv_rows * D * es * 2 + int(nnz.sum()) * 4 + 2 * B * Hq * D * es)


def make_sparse_dense(B=1, Hq=32, Hkv=8, L=32000, D=128, keep_p=0.02, seed=0, device="cpu",
                      dtype=torch.float16, std=1.0, L_max=None, per_qo_head=False) -> SparseDenseCase:
    g = _gen(seed, device)
    q = randn((B, Hq, 1, D), g, device, dtype, std)
    K = randn((B, Hkv, L, D), g, device, dtype, std)
    V = randn((B, Hkv, L, D), g, device, dtype, std)
    if L_max is None:
        L_max = int(L * (keep_p + 0.1))
    ind, nnz = sparse_lists([L] * B, Hkv, Hq // Hkv, keep_p, L_max, g, device, per_qo_head)
    return SparseDenseCase(q, K, V, ind, nnz, 1.0 / math.sqrt(D), Hq // Hkv)


@dataclass
class SparsePagedCase:
    q: torch.Tensor
    cache: torch.Tensor
    indptr: torch.Tensor
    indices: torch.Tensor
    sparse_ind: torch.Tensor
    sparse_nnz: torch.Tensor
    seq_lens: torch.Tensor
    K: Optional[torch.Tensor] = None   # MagicPIG per-(b, qo-head) parameters
    L: Optional[torch.Tensor] = None

    @property
    def bytes(self) -> float:
        B, Hq, _, D = self.q.shape
        Hkv = self.cache.shape[2]
        group = Hq // Hkv
        es = self.cache.element_size()
        nnz = self.sparse_nnz.reshape(B, Hq)
        kv_rows = int(nnz[:, ::group].sum())
        # index lists + the page-table entries each kept row goes through
        return float(kv_rows * D * es * 2 + int(nnz.sum()) * 8 + 2 * B * Hq * D * es)


def make_sparse_paged(B=3, Hq=32, Hkv=8, D=256, page_size=16, min_len=8192, max_len=32768,
                      lens: Optional[Sequence[int]] = None, keep_p=0.02, seed=0, device="cpu",
                      dtype=torch.float16, std=1.0, magicpig=False, per_qo_head=False,
                      L_max=None) -> SparsePagedCase:
    g = _gen(seed, device)
    if lens is None:
        lens = torch.randint(min_len, max_len + 1, (B,), generator=_gen(seed + 7919, "cpu")).tolist()
    indptr, indices, last, seq_lens, bt, N = paged_layout_from_lens(lens, page_size, g, device)
    cache = randn((N, 2, Hkv, page_size, D), g, device, dtype, std)
    q = randn((len(lens), Hq, 1, D), g, device, dtype, std)
    if L_max is None:
        L_max = max(1, max(int(x) for x in bt.shape[1:]) * page_size)
    ind, nnz = sparse_lists(lens, Hkv, Hq // Hkv, keep_p, L_max, g, device, per_qo_head)
    Kp = Lp = None
    if magicpig:
        Kp = torch.rand((len(lens), Hq), generator=g, device=device, dtype=torch.float32) * 5 + 1
        Lp = torch.rand((len(lens), Hq), generator=g, device=device, dtype=torch.float32) * 5 + 1
    return SparsePagedCase(q, cache, indptr, indices, ind, nnz, seq_lens, Kp, Lp)
