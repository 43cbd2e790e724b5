"""The CPU baseline's stand-in, checked against the reference's own code.

TEST INFRASTRUCTURE ONLY: run by hand in a container that has a checkout of the
reference (nothing in the package, the tests or ``bench.py`` runs it).

``bench.py``'s CPU arm (``--impl reference`` and ``cpu_baseline``) times
``oracle.naive.naive_paged_attention``, this repository's restatement of the
reference's ``naive_paged_attention``
(``decode_flash_attention_redundant_var_len_paged.py:278``), because the
reference cannot travel to the GPU box: it is a set of scripts, not an
installable package (``pip install`` of it stops at "Neither 'setup.py' nor
'pyproject.toml' found").  This script imports the reference's function from
its own module and runs it beside the restatement on the same bounded cfg3
sample (fp32, CPU, all host threads), reporting both times and the largest
output difference, so that the stand-in can be seen to time the same work.

Usage::

    python oracle/compare_reference_cpu.py --reference-dir <checkout> [--seqs 4] [--reps 3]
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

from attention_kernel_triton_b200 import workloads as W  # noqa: E402
from oracle import naive as N  # noqa: E402


def load_reference(ref_dir: str):
    path = os.path.join(ref_dir, "decode_flash_attention_redundant_var_len_paged.py")
    spec = importlib.util.spec_from_file_location("ref_paged_decode", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.naive_paged_attention


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-dir", required=True)
    ap.add_argument("--seqs", type=int, default=4)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    ref_fn = load_reference(args.reference_dir)
    torch.set_num_threads(os.cpu_count() or 1)
    # the bench's sample: the first sequences of the cfg3 length distribution
    lens = torch.randint(512, 32768 + 1, (64,), generator=torch.Generator().manual_seed(7919)).tolist()
    c = W.make_paged(lens=lens[:args.seqs], seed=0)
    q, cache = c.q.float(), c.cache.float()

    def timed(fn):
        fn()
        ts = []
        for _ in range(args.reps):
            t0 = time.perf_counter()
            out = fn()
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts), out

    t_ref, o_ref = timed(lambda: ref_fn(q, cache, c.indptr, c.indices, c.last_page_len))
    t_port, o_port = timed(lambda: N.naive_paged_attention(q, cache, c.indptr, c.indices, c.last_page_len))
    o_ref = o_ref.reshape(o_port.shape).float()
    print(json.dumps({
        "sample": f"first {args.seqs} cfg3 sequences ({sum(lens[:args.seqs])} tokens), fp32, "
                  f"{torch.get_num_threads()} threads, median of {args.reps}",
        "reference_s": t_ref, "port_s": t_port, "port_over_reference": t_port / t_ref,
        "reference_gbs": c.bytes / t_ref / 1e9, "port_gbs": c.bytes / t_port / 1e9,
        "max_abs_diff": float((o_ref - o_port).abs().max())}))


if __name__ == "__main__":
    main()
