"""Generate the golden fixtures under tests/golden/ from the reference itself.

Usage::

    python tests/golden/make_golden.py --reference-dir <checkout of KiritoHugh/attention_kernel_triton>

The reference's naive PyTorch functions are imported from its own modules and
run on CPU on seeded inputs (``attention_kernel_triton_b200.workloads``).  The
prefill and dense-decode references are closures nested inside the reference's
``test_op*`` drivers; they are lifted out of the source with ``ast`` and run
unchanged except for the one ``device="cuda"`` literal of the causal mask
(PF:416, PV:429), which becomes ``device=Q.device``.  The MagicPIG module
imports ``torch_npu`` at the top (MP:2); a stand-in empty module is registered
so the import succeeds (its kernel is never launched here).

Every fixture stores the inputs (as used) and the reference output.  Only this
script reads the reference; the tests read the ``.npz`` files.
"""
from __future__ import annotations

import argparse
import ast
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from attention_kernel_triton_b200 import workloads as W  # noqa: E402


def nested_function(path: str, outer: str, inner: str, env: dict):
    src = open(path).read()
    tree = ast.parse(src)
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name == outer:
            for sub in node.body:
                if isinstance(sub, ast.FunctionDef) and sub.name == inner:
                    seg = ast.get_source_segment(src, sub)
                    seg = "\n".join(l[4:] if l.startswith("    ") else l for l in seg.splitlines())
                    seg = seg.replace('device="cuda"', "device=Q.device")
                    ns = dict(env)
                    exec(compile(seg, f"{path}:{outer}.{inner}", "exec"), ns)
                    return ns[inner]
    raise KeyError(f"{outer}.{inner} not found in {path}")


def loop_in(path: str, outer: str, target: str, must_contain: str) -> str:
    """Source of the top-level-in-body ``for <target> in ...`` loop of function ``outer``
    whose text contains ``must_contain`` (dedented to column 0)."""
    src = open(path).read()
    for node in ast.parse(src).body:
        if isinstance(node, ast.FunctionDef) and node.name == outer:
            for sub in ast.walk(node):
                if isinstance(sub, ast.For) and ast.unparse(sub.target) == target:
                    seg = ast.get_source_segment(src, sub)
                    if must_contain in seg:
                        pad = " " * sub.col_offset
                        return "\n".join(l[len(pad):] if l.startswith(pad) else l for l in seg.splitlines())
    raise KeyError(f"{outer}: for {target} ... {must_contain}")


class _SeededTorch(types.ModuleType):
    """``torch`` for an exec'd reference loop: ``torch.rand`` draws from a seeded
    CPU generator and records every draw; everything else is torch."""

    def __init__(self, seed: int):
        super().__init__("torch")
        self._g = torch.Generator().manual_seed(seed)
        self.draws = []

    def rand(self, size, device=None, **kw):
        r = torch.rand(size, generator=self._g)
        self.draws.append(r)
        return r

    def __getattr__(self, name):
        return getattr(torch, name)


def f32(t):
    return t.float()


def save(name, **arrays):
    out = {}
    for k, v in arrays.items():
        if isinstance(v, torch.Tensor):
            v = v.detach().cpu()
            out[k] = v.numpy()
        else:
            out[k] = np.asarray(v)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
    print(f"wrote {name}.npz", {k: (a.shape, str(a.dtype)) for k, a in out.items()})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-dir", required=True)
    args = ap.parse_args()
    ref = os.path.abspath(args.reference_dir)
    sys.path.insert(0, ref)
    sys.modules.setdefault("torch_npu", types.ModuleType("torch_npu"))
    torch.manual_seed(0)

    import decode_flash_attention_redundant_var_len_paged as DP
    import sparsetoken_decode_flash_attention_redundant as SD
    import sparsetoken_decode_flash_attention_redundant_var_len_paged as SP
    import magicpig_sparsetoken_decode_flash_attention_redundant_var_len_paged_with_norm as MP

    # ---------------- prefill (PF:415-425), fp16 end to end as the reference runs it
    for name, kw in [
        ("prefill_causal_gqa", dict(B=1, Hq=4, Hkv=1, S=128, D=64, causal=True, seed=101)),
        ("prefill_noncausal", dict(B=1, Hq=2, Hkv=2, S=128, D=64, causal=False, seed=102)),
        ("prefill_causal_d128", dict(B=1, Hq=2, Hkv=1, S=64, D=128, causal=True, seed=103)),
    ]:
        c = W.make_prefill(**kw)
        fn = nested_function(os.path.join(ref, "prefill_flash_attention.py"), "test_op",
                             "reference_implementation", {"torch": torch, "SEQ_LEN": kw["S"]})
        O = fn(c.Q, c.K, c.V, c.causal, c.softmax_scale, c.group)
        save(name, Q=c.Q, K=c.K, V=c.V, causal=c.causal, softmax_scale=c.softmax_scale,
             group=c.group, O=O)

    # ---------------- var-len prefill (PV:428-438 then PV:447-450)
    c = W.make_prefill(B=3, Hq=4, Hkv=2, S=128, D=64, causal=True, seed=104)
    lens = torch.tensor([128, 37, 90], dtype=torch.int32)
    fn = nested_function(os.path.join(ref, "prefill_flash_attention_var_len_padding.py"),
                         "test_op_var_len_padding", "reference_implementation",
                         {"torch": torch, "SEQ_LEN": 128})
    O = fn(c.Q, c.K, c.V, True, c.softmax_scale, c.group)
    for i in range(3):
        O[i, :, int(lens[i]):, :] = 0.0
    save("prefill_varlen", Q=c.Q, K=c.K, V=c.V, causal=True, softmax_scale=c.softmax_scale,
         group=c.group, varlen=lens, O=O)

    # ---------------- dense decode (DR:306-312)
    for name, kw in [
        ("decode_dense", dict(B=2, Hq=8, Hkv=2, L=192, D=64, seed=201)),
        ("decode_dense_d128", dict(B=1, Hq=4, Hkv=1, L=100, D=128, seed=202)),
    ]:
        c = W.make_decode(**kw)
        fn = nested_function(os.path.join(ref, "decode_flash_attention_redundant.py"),
                             "test_op_decode", "reference_implementation", {"torch": torch})
        O = fn(c.q, c.K, c.V, c.softmax_scale, c.group)
        save(name, q=c.q, K=c.K, V=c.V, softmax_scale=c.softmax_scale, group=c.group, O=O)

    # ---------------- paged decode (DP:278-329), fp32 on fp16-valued inputs
    # (a) the reference's own hand-written page table (DP:337-353)
    g = torch.Generator().manual_seed(301)
    cache = W.randn((8, 2, 2, 64, 64), g, "cpu")
    q = W.randn((3, 4, 1, 64), g, "cpu")
    indptr = torch.tensor([0, 4, 5, 8], dtype=torch.int32)
    indices = torch.tensor([0, 1, 3, 5, 2, 6, 7, 4], dtype=torch.int32)
    last = torch.tensor([2, 22, 3], dtype=torch.int32)
    O = DP.naive_paged_attention(f32(q), f32(cache), indptr, indices, last)
    save("paged_ref_table", q=q, cache=cache, indptr=indptr, indices=indices, last_page_len=last, O=O)
    # (b) page size 16, D=128, ragged lengths incl. a 1-token sequence and a full page
    c = W.make_paged(B=4, Hq=8, Hkv=2, D=128, page_size=16, lens=[1, 16, 17, 250], seed=302)
    O = DP.naive_paged_attention(f32(c.q), f32(c.cache), c.indptr, c.indices, c.last_page_len)
    save("paged_p16", q=c.q, cache=c.cache, indptr=c.indptr, indices=c.indices,
         last_page_len=c.last_page_len, O=O)

    # ---------------- sparse-token decode, dense KV (SD:173-230)
    c = W.make_sparse_dense(B=2, Hq=8, Hkv=2, L=512, D=128, keep_p=0.05, seed=401, per_qo_head=True)
    O = SD.sparsetoken_naive_decode(f32(c.q), f32(c.K), f32(c.V), c.sparse_ind, c.sparse_nnz,
                                    c.softmax_scale, c.group)
    mask = torch.zeros((2, 8, 512), dtype=torch.bool)
    for b in range(2):
        for h in range(8):
            n = max(int(c.sparse_nnz[b, h]), 1)
            mask[b, h, c.sparse_ind[b, h, :n].long()] = True
    O_mask = SD.sparsetoken_naive_decode_by_mask(f32(c.q), f32(c.K), f32(c.V), c.sparse_ind,
                                                 c.sparse_nnz, c.softmax_scale, c.group, mask)
    save("sparse_dense", q=c.q, K=c.K, V=c.V, sparse_ind=c.sparse_ind, sparse_nnz=c.sparse_nnz,
         softmax_scale=c.softmax_scale, group=c.group, mask=mask, O=O, O_by_mask=O_mask)

    # ---------------- sparse-token decode, paged KV (SP:234-288)
    c = W.make_sparse_paged(B=2, Hq=8, Hkv=2, D=64, page_size=16, lens=[300, 129], keep_p=0.1,
                            seed=501)
    O = SP.sparsetoken_naive_paged_attention(f32(c.q), f32(c.cache), c.indptr, c.indices,
                                             c.sparse_ind, c.sparse_nnz)
    save("sparse_paged", q=c.q, cache=c.cache, indptr=c.indptr, indices=c.indices,
         sparse_ind=c.sparse_ind, sparse_nnz=c.sparse_nnz, O=O)
    c = W.make_sparse_paged(B=2, Hq=8, Hkv=2, D=128, page_size=16, lens=[200, 77], keep_p=0.1,
                            seed=502, per_qo_head=True)
    O = SP.sparsetoken_naive_paged_attention(f32(c.q), f32(c.cache), c.indptr, c.indices,
                                             c.sparse_ind, c.sparse_nnz)
    save("sparse_paged_perhead", q=c.q, cache=c.cache, indptr=c.indptr, indices=c.indices,
         sparse_ind=c.sparse_ind, sparse_nnz=c.sparse_nnz, O=O)

    # ---------------- MagicPIG with norm (MP:212-291)
    c = W.make_sparse_paged(B=2, Hq=8, Hkv=2, D=128, page_size=16, lens=[300, 129], keep_p=0.1,
                            seed=601, magicpig=True)
    O = MP.magicpig_sparsetoken_naive_paged_attention(f32(c.q), f32(c.cache), c.indptr, c.indices,
                                                      c.sparse_ind, c.sparse_nnz, c.K, c.L)
    save("magicpig_paged", q=c.q, cache=c.cache, indptr=c.indptr, indices=c.indices,
         sparse_ind=c.sparse_ind, sparse_nnz=c.sparse_nnz, K=c.K, L=c.L, O=O)


    # ---------------- keep mask <-> kept-index lists (SD:283-295 and SD:317-324), the
    # reference's own loops run on seeded draws; the raw keep mask is recovered from them
    sd_path = os.path.join(ref, "sparsetoken_decode_flash_attention_redundant.py")
    gen_loop = loop_in(sd_path, "test_op_decode_sparsetoken", "bh", "sparse_ind")
    mask_loop = loop_in(sd_path, "test_op_decode_sparsetoken", "b", "precompute_mask")
    B, H, SEQ_LEN, kept_ratio = 2, 6, 300, 0.006  # a few rows draw nothing and keep token 0
    L_max = int(SEQ_LEN * (kept_ratio + 0.1))
    shim = _SeededTorch(701)
    env = {"torch": shim, "BATCH_SIZE": B, "num_qo_heads": H, "kept_ratio": kept_ratio, "device": "cpu",
           "original_nzz": torch.full((B, H, 1), SEQ_LEN, dtype=torch.int32),
           "sparse_ind": torch.zeros((B, H, L_max), dtype=torch.int32) - 1}
    exec(compile(gen_loop, f"{sd_path}:mask->lists", "exec"), env)
    kept_mask = torch.stack([d < kept_ratio for d in shim.draws]).reshape(B, H, SEQ_LEN)
    sparse_ind, sparse_nnz = env["sparse_ind"], env["original_nzz"]
    env2 = {"torch": torch, "BATCH_SIZE": B, "num_qo_heads": H, "sparse_nnz": sparse_nnz,
            "sparse_ind": sparse_ind,
            "precompute_mask": torch.zeros((B, H, SEQ_LEN), dtype=torch.bool)}
    exec(compile(mask_loop, f"{sd_path}:lists->mask", "exec"), env2)
    save("mask_index", kept_mask=kept_mask, L_max=L_max, sparse_ind=sparse_ind, sparse_nnz=sparse_nnz,
         precompute_mask=env2["precompute_mask"])


if __name__ == "__main__":
    main()
