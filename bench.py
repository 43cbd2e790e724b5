"""Benchmark of the headline path: paged var-len GQA decode (workload cfg3: B=64, Hq=32, Hkv=8, D=128, P=16).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one call of ``flash_attention_decode_paged`` over the whole cfg3
batch (B=64, Hq=32, Hkv=8, D=128, fp16, page size 16, lengths U[512, 32768],
pages in seeded random physical order), inputs resident in HBM.  The pool is
4.4 GB, far larger than the 126 MB L2, so no flush is needed between steps.

Multi-GPU (torchrun, one rank per GPU): every rank decodes its own cfg3 batch
(seed + rank): weak scaling, no data-path collective.  ``value`` is the
algorithmic bytes of all ranks divided by the max-over-ranks device time.
``strong_scaling`` splits ONE cfg3 / cfg0 / cfg1 workload over the ranks by kv
head (no communication) and gives its throughput and efficiency at this N;
``parity`` checks sampled outputs of every timed run against the CPU oracle
(max over ranks), outside the timed regions.

``--impl reference`` times the reference's naive paged decode (the CPU oracle's
restatement of ``naive_paged_attention``, fp32 torch on all host cores) on a
bounded sample of cfg3 sequences, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from attention_kernel_triton_b200 import workloads as W  # noqa: E402

METRIC = "paged decode HBM GB/s"
GRAPH_STEPS = 16  # e2e steps per captured CUDA graph
# DRAM bytes of one split-KV launch on cfg3.  Tensor-core kernel: ncu on the
# 8-sequence case (--batch 8: read 437.694 MB + write 3.844 MB for 437.439 MB of
# algorithmic bytes) scaled to cfg3's 4513.9 MB by the algorithmic bytes (reads
# grow with the tokens; the partials' writes grow more slowly, so this bounds
# them from above).  CUDA-core kernel: ncu on cfg3 itself (4.51 GB + 7.19 MB).
CFG3_TRAFFIC_BYTES = (437.694e6 + 3.844e6) / 437.439e6 * 4513.900124e6
CFG3_TRAFFIC_BYTES_CUDA_CORES = 4.51e9 + 7.19e6
WORKLOAD = ("cfg3 paged var-len GQA decode: B=64 Hq=32 Hkv=8 D=128 fp16 page_size=16 "
            "lens U[512,32768] seeded, random physical page order")


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle sampling while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.3)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_reference_step(sample, threads):
    from oracle import naive as N  # CPU baseline leg only
    torch.set_num_threads(threads)
    t0 = time.perf_counter()
    N.naive_paged_attention(sample["q"], sample["cache"], sample["indptr"], sample["indices"],
                            sample["last"])
    return time.perf_counter() - t0


def make_cpu_sample(n_seqs: int, seed: int = 0):
    """A bounded cfg3 sample: the first ``n_seqs`` sequences of the cfg3
    length distribution, fp32 copies (the CPU oracle computes in fp32)."""
    lens = torch.randint(512, 32768 + 1, (64,), generator=torch.Generator().manual_seed(seed + 7919)).tolist()
    c = W.make_paged(lens=lens[:n_seqs], seed=seed)
    sample = {"q": c.q.float(), "cache": c.cache.float(), "indptr": c.indptr, "indices": c.indices,
              "last": c.last_page_len}
    return sample, c.bytes


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    sample, nbytes = make_cpu_sample(args.cpu_seqs)
    for _ in range(args.warmup):
        cpu_reference_step(sample, threads)
    times = [cpu_reference_step(sample, threads) for _ in range(args.steps)]
    t = statistics.mean(times)
    val = nbytes / t / 1e9
    desc = (f"naive_paged_attention restated (oracle port), fp32 torch CPU, first {args.cpu_seqs} "
            f"cfg3 sequences per step")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": val, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": desc},
        "cpu_baseline": {"value": val, "unit": "GB/s", "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": val, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def measured_tflops():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def time_kernels(fn, iters, dev, flush=None):
    """``(kernel_ms, call_ms)`` over ``iters`` calls: the mean device time of the
    library's main kernel, from CUDA events the library records around that kernel
    on its stream, and the mean device time of the whole call (every kernel it
    launches), from events around the call.  ``flush`` (a buffer larger than L2)
    is overwritten before every call, outside both; a device sleep ahead of each
    call keeps the host's dispatch time out of the call's events."""
    from attention_kernel_triton_b200 import _lib
    for _ in range(3):
        fn()
    torch.cuda.synchronize(dev)
    with _lib.profile_kernels() as prof:
        for _ in range(iters):
            if flush is not None:
                flush.zero_()
            fn()
        torch.cuda.synchronize(dev)
    # whole calls, without the library's profiling events between their kernels
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    for a, b in ev:
        if flush is not None:
            flush.zero_()
        torch.cuda._sleep(200_000)  # ~0.1 ms
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize(dev)
    call_ms = sum(a.elapsed_time(b) for a, b in ev) / iters
    return prof.total_ms / max(prof.launches, 1), call_ms


# ----------------------------------------------------------------------------
# parity of the timed runs against the CPU oracle (outside every timed region)
# ----------------------------------------------------------------------------
TOL = 2e-3


def _paged_sample(c, batches, heads=None):
    """The sampled sequences of a paged case as a small CPU case (their pages only),
    for the oracle: ``(q, cache, indptr, indices, last)``, kv heads ``heads`` of the
    pool when given."""
    ip = c.indptr.cpu().tolist()
    idx = c.indices.cpu()
    pages, counts = [], []
    for b in batches:
        pages.append(idx[ip[b]:ip[b + 1]])
        counts.append(ip[b + 1] - ip[b])
    sel = torch.cat(pages).to(c.cache.device, torch.int64)
    cache = c.cache.index_select(0, sel)
    if heads is not None:
        cache = cache[:, :, heads[0]:heads[1]]
    indptr = torch.tensor([0] + torch.tensor(counts).cumsum(0).tolist(), dtype=torch.int32)
    indices = torch.arange(sel.numel(), dtype=torch.int32)
    q = c.q[list(batches)].cpu()
    last = c.last_page_len[list(batches)].cpu()
    return q, cache.cpu(), indptr, indices, last


def paged_parity(out, c, batches, kv_heads=None, group=None):
    """Max-abs error of ``out`` (the decode of case ``c``, or of kv heads ``kv_heads``
    of it) against the oracle on the sampled sequences; NaN counts as infinite."""
    from oracle import naive as N  # checker only, outside the timed regions
    q, cache, indptr, indices, last = _paged_sample(c, batches, kv_heads)
    if kv_heads is not None:
        q = q[:, kv_heads[0] * group:kv_heads[1] * group]
    ref = N.naive_paged_attention(q, cache, indptr, indices, last)
    got = out[list(batches)].float().cpu()
    if torch.isnan(got).any():
        return float("inf")
    return float((got - ref).abs().max())


def prefill_parity(O, f, samples, q_off=0):
    """Max-abs error of the prefill output ``O`` (query heads ``q_off ..`` of case ``f``)
    against the oracle on sampled (batch, local query head) pairs, valid rows only."""
    from oracle import naive as N  # checker only
    err = 0.0
    for b, hl in samples:
        h = q_off + hl
        kvh = h // f.group
        ref = N.prefill_reference(f.Q[b:b + 1, h:h + 1].cpu(), f.K[b:b + 1, kvh:kvh + 1].cpu(),
                                  f.V[b:b + 1, kvh:kvh + 1].cpu(), True, f.softmax_scale, 1)
        n = int(f.varlen[b]) if f.varlen is not None else f.Q.shape[2]
        got = O[b:b + 1, hl:hl + 1, :n].float().cpu()
        if torch.isnan(O[b:b + 1, hl:hl + 1]).any():
            return float("inf")
        err = max(err, float((got - ref[:, :, :n]).abs().max()))
    return err


def _max_over_ranks(pg, dev, values):
    t = torch.tensor(values, dtype=torch.float64, device=dev)
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


def _timed(fn, steps, dev, pg, flush=None):
    """Mean device ms per call of ``fn`` over ``steps`` calls, max over ranks (barrier
    and synchronize on both sides; ``flush`` is overwritten before each call)."""
    for _ in range(3):
        fn()
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize(dev)
    if flush is None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / steps
    else:
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for a, b in ev:
            flush.zero_()
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize(dev)
        ms = sum(a.elapsed_time(b) for a, b in ev) / steps
    return _max_over_ranks(pg, dev, [ms])[0]


def strong_scaling_measurements(dev, pg, world, rank, steps=100):
    """One BASELINE workload partitioned over all ranks by kv head (no communication):
    cfg3 paged decode (8 kv heads: 8/N per GPU, each rank's pool slice built before
    timing), cfg0 causal prefill and cfg1 var-len prefill (16 kv heads: 16/N per GPU).
    Time is the max over ranks; ``single_gpu_ms`` is the whole workload on rank 0's GPU
    in the same run, and ``efficiency`` = single_gpu_ms / (N * ms).  Returns
    ``(results, parity)``; parity samples each rank's output slice against the oracle."""
    from attention_kernel_triton_b200.decode_flash_attention_redundant_var_len_paged import decode_paged_into
    from attention_kernel_triton_b200.distributed import KVHeadPartition, decode_paged_partitioned, prefill_partitioned
    from attention_kernel_triton_b200.prefill_flash_attention import flash_attention_prefill
    from attention_kernel_triton_b200.prefill_flash_attention_var_len_padding import (
        flash_attention_prefill as flash_attention_prefill_varlen)
    res, par = {}, {}

    # cfg3 paged decode by kv head (the full case on every rank, same seed; each rank keeps its slice)
    c = W.make_paged(seed=0, device=dev)
    part = KVHeadPartition(8, 4, world, rank)
    local = part.local_paged_cache(c.cache)
    out_l = torch.empty((64, part.q1 - part.q0, 128), dtype=torch.float16, device=dev)
    ms = _timed(lambda: decode_paged_partitioned(c.q, local, c.indptr, c.indices, c.last_page_len, part, out=out_l),
                steps, dev, pg)
    out_full = torch.empty((64, 32, 128), dtype=torch.float16, device=dev)
    single = _timed(lambda: decode_paged_into(out_full, c.q, c.cache, c.indptr, c.indices, c.last_page_len),
                    steps, dev, None) if rank == 0 else 0.0
    single = _max_over_ranks(pg, dev, [single])[0]
    res["cfg3_paged_decode_kv_head"] = {
        "gbs": c.bytes / ms / 1e6, "ms": ms, "kv_heads_per_gpu": part.num_local_kv_heads,
        "single_gpu_ms": single, "efficiency": single / (world * ms), "l2": "inputs larger than L2"}
    longest = int(torch.argmax(c.seq_lens))
    par["cfg3_kv_head_sampled"] = paged_parity(out_l, c, [rank % 64, longest], (part.h0, part.h1), 4)
    del c, local, out_full
    torch.cuda.empty_cache()

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for name, varlen in (("prefill_cfg0_causal_kv_head", False), ("prefill_cfg1_varlen_kv_head", True)):
        f = W.make_prefill(seed=1 if varlen else 0, device=dev, varlen=varlen)
        part = KVHeadPartition(16, f.group, world, rank)
        vl = f.varlen if varlen else None
        holder = {}

        def run_part():
            holder["O"] = prefill_partitioned(f.Q, f.K, f.V, True, f.softmax_scale, f.group, part, varlen=vl)
        ms = _timed(run_part, 20, dev, pg, flush)
        if rank == 0:
            fn = (lambda: flash_attention_prefill_varlen(f.Q, f.K, f.V, True, f.softmax_scale, f.group, f.varlen)) \
                if varlen else (lambda: flash_attention_prefill(f.Q, f.K, f.V, True, f.softmax_scale, f.group))
            single = _timed(fn, 20, dev, None, flush)
        else:
            single = 0.0
        single = _max_over_ranks(pg, dev, [single])[0]
        res[name] = {"tflops": f.flops / ms / 1e9, "ms": ms, "kv_heads_per_gpu": part.num_local_kv_heads,
                     "single_gpu_ms": single, "efficiency": single / (world * ms), "l2": "flushed"}
        par[name + "_sampled"] = prefill_parity(holder["O"], f, [(rank % 8, 0), (0, part.q1 - part.q0 - 1)],
                                                q_off=part.q0)
        del f, holder
        torch.cuda.empty_cache()
    return res, par


def secondary_measurements(dev, iters=20, only=None):
    """The other benchmark workloads (prefill cfg0/cfg1, decode cfg2 and the long-context
    sweep, the sparse cfg4 family) and the added paths, one kernel each (single GPU).
    ``only`` restricts the run to one configuration (profiler captures)."""
    from attention_kernel_triton_b200.decode_flash_attention_redundant import flash_attention_decode
    from attention_kernel_triton_b200.magicpig_sparsetoken_decode_flash_attention_redundant_var_len_paged_with_norm import (
        magicpig_sparsetoken_flash_attention_decode_paged)
    from attention_kernel_triton_b200.prefill_flash_attention import flash_attention_prefill
    from attention_kernel_triton_b200.prefill_flash_attention_var_len_padding import (
        flash_attention_prefill as flash_attention_prefill_varlen)
    from attention_kernel_triton_b200.sparsetoken_decode_flash_attention_redundant import (
        sparsetoken_flash_attention_decode, sparsetoken_flash_attention_decode_csr)
    from attention_kernel_triton_b200.sparsetoken_decode_flash_attention_redundant_var_len_paged import (
        sparsetoken_flash_attention_decode_paged)
    hbm, _ = measured_peaks()
    tf, _ = measured_tflops()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # 256 MB > 126 MB L2

    def prefill_cfg0():
        c = W.make_prefill(seed=0, device=dev)
        ms, call_ms = time_kernels(lambda: flash_attention_prefill(c.Q, c.K, c.V, True, c.softmax_scale, c.group),
                          iters, dev, flush)
        return {"tflops": c.flops / ms / 1e9, "ms": ms, "call_ms": call_ms, "frac_of_bf16_peak": c.flops / ms / 1e9 / tf,
                "gflop": c.flops / 1e9, "l2": "flushed"}

    def prefill_cfg1():
        c = W.make_prefill(seed=1, device=dev, varlen=True)
        ms, call_ms = time_kernels(lambda: flash_attention_prefill_varlen(c.Q, c.K, c.V, True, c.softmax_scale, c.group,
                                                                 c.varlen), iters, dev, flush)
        return {"tflops": c.flops / ms / 1e9, "ms": ms, "call_ms": call_ms, "frac_of_bf16_peak": c.flops / ms / 1e9 / tf,
                "gflop_valid": c.flops / 1e9, "lens": c.varlen.tolist(), "l2": "flushed"}

    def decode(kw, fl):
        def run():
            d = W.make_decode(seed=2, device=dev, **kw)
            ms, call_ms = time_kernels(lambda: flash_attention_decode(d.q, d.K, d.V, d.softmax_scale, d.group), iters, dev,
                              flush if fl else None)
            return {"gbs": d.bytes / ms / 1e6, "ms": ms, "call_ms": call_ms, "call_gbs": d.bytes / call_ms / 1e6,
                    "frac_of_hbm": d.bytes / ms / 1e6 / hbm,
                    "mb": d.bytes / 1e6, "l2": "flushed" if fl else "inputs larger than L2"}
        return run

    def sparse_dense():
        sd = W.make_sparse_dense(seed=41, device=dev)
        ms, call_ms = time_kernels(lambda: sparsetoken_flash_attention_decode(sd.q, sd.K, sd.V, sd.sparse_ind, sd.sparse_nnz,
                                                                     sd.softmax_scale, sd.group), iters, dev, flush)
        return {"gbs": sd.bytes / ms / 1e6, "ms": ms, "call_ms": call_ms, "mb": sd.bytes / 1e6, "l2": "flushed"}

    def sparse_paged(magic):
        def run():
            sp = W.make_sparse_paged(seed=42, device=dev, magicpig=True)
            if magic:
                fn = lambda: magicpig_sparsetoken_flash_attention_decode_paged(  # noqa: E731
                    sp.q, sp.cache, sp.indptr, sp.indices, sp.sparse_ind, sp.sparse_nnz, sp.K, sp.L)
            else:
                fn = lambda: sparsetoken_flash_attention_decode_paged(  # noqa: E731
                    sp.q, sp.cache, sp.indptr, sp.indices, sp.sparse_ind, sp.sparse_nnz)
            ms, call_ms = time_kernels(fn, iters, dev, flush)
            return {"gbs": sp.bytes / ms / 1e6, "ms": ms, "call_ms": call_ms, "mb": sp.bytes / 1e6, "l2": "flushed"}
        return run

    def sparse_128k():
        sd = W.make_sparse_dense(B=1, Hq=32, Hkv=8, L=131072, D=128, keep_p=0.02, seed=12, device=dev, L_max=4096)
        ms, call_ms = time_kernels(lambda: sparsetoken_flash_attention_decode(sd.q, sd.K, sd.V, sd.sparse_ind, sd.sparse_nnz,
                                                                     sd.softmax_scale, sd.group), iters, dev, flush)
        return {"gbs": sd.bytes / ms / 1e6, "ms": ms, "call_ms": call_ms, "mb": sd.bytes / 1e6, "l2": "flushed"}

    def sparse_128k_csr():
        from attention_kernel_triton_b200.sparse_index import sparse_csr_from_lists
        sd = W.make_sparse_dense(B=1, Hq=32, Hkv=8, L=131072, D=128, keep_p=0.02, seed=12, device=dev, L_max=4096)
        inds, ptr = sparse_csr_from_lists(sd.sparse_ind, sd.sparse_nnz)
        ms, call_ms = time_kernels(lambda: sparsetoken_flash_attention_decode_csr(sd.q, sd.K, sd.V, inds, ptr,
                                                                         sd.softmax_scale, sd.group, max_nnz=4096),
                          iters, dev, flush)
        return {"gbs": sd.bytes / ms / 1e6, "ms": ms, "call_ms": call_ms, "mb": sd.bytes / 1e6, "l2": "flushed",
                "index_bytes_csr": (inds.numel() + ptr.numel()) * 4,
                "index_bytes_padded": sd.sparse_ind.numel() * 4 + sd.sparse_nnz.numel() * 4}

    def append_cfg0():
        # write path ahead of paged decode: cfg0's K/V (8 x 1024 tokens, 16 kv heads, D=64) into a P=16 pool
        from attention_kernel_triton_b200.paged_kv_append import append_paged_kv_cache
        c = W.make_paged(B=8, Hq=64, Hkv=16, D=64, page_size=16, lens=[1024] * 8, seed=44, device=dev)
        g = torch.Generator(device=dev).manual_seed(44)
        k = torch.randn((8 * 1024, 16, 64), generator=g, device=dev, dtype=torch.float16)
        v = torch.randn((8 * 1024, 16, 64), generator=g, device=dev, dtype=torch.float16)
        app = torch.arange(0, 8 * 1024 + 1, 1024, dtype=torch.int32, device=dev)
        ms, call_ms = time_kernels(lambda: append_paged_kv_cache(c.cache, k, v, app, c.indptr, c.indices, c.last_page_len),
                          iters, dev, flush)
        nbytes = 2 * 2 * k.numel() * 2  # K and V rows read and written
        return {"gbs": nbytes / ms / 1e6, "ms": ms, "call_ms": call_ms, "frac_of_hbm": nbytes / ms / 1e6 / hbm,
                "mb": nbytes / 1e6, "l2": "flushed"}

    def mask_to_index(L, L_max):
        def run():
            from attention_kernel_triton_b200.sparse_index import sparse_index_from_mask
            g = torch.Generator(device=dev).manual_seed(43)
            mask = torch.rand((1, 32, L), generator=g, device=dev) < 0.02
            ms, call_ms = time_kernels(lambda: sparse_index_from_mask(mask, L_max), iters, dev, flush)
            nbytes = mask.numel() + 32 * L_max * 4 + 32 * 4  # mask read, lists and nnz written
            return {"gbs": nbytes / ms / 1e6, "ms": ms, "call_ms": call_ms, "mb": nbytes / 1e6, "l2": "flushed"}
        return run

    def torch_sdpa_cfg0(backend):
        """Context, not the product: torch's own scaled_dot_product_attention on
        the cfg0 inputs through one library backend (K/V expanded to the 64
        query heads outside the timed region), timed with CUDA events around
        the call; a 1 ms device sleep ahead of each call keeps the host's
        dispatch time out of the events.  Null when the backend refuses the
        inputs."""
        def run():
            import torch.nn.functional as F
            from torch.nn.attention import SDPBackend, sdpa_kernel
            c = W.make_prefill(seed=0, device=dev)
            Ke = c.K.repeat_interleave(c.group, dim=1)
            Ve = c.V.repeat_interleave(c.group, dim=1)
            be = {"cudnn": SDPBackend.CUDNN_ATTENTION, "flash": SDPBackend.FLASH_ATTENTION}[backend]

            def fn():
                with sdpa_kernel([be]):
                    return F.scaled_dot_product_attention(c.Q, Ke, Ve, is_causal=True, scale=c.softmax_scale)
            try:
                fn()
            except RuntimeError as e:
                return {"tflops": None, "error": str(e).splitlines()[0][:160]}
            for _ in range(3):
                fn()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
            for a, b in ev:
                flush.zero_()
                torch.cuda._sleep(2_000_000)  # ~1 ms at 1.9 GHz
                a.record()
                fn()
                b.record()
            torch.cuda.synchronize(dev)
            ms = sum(a.elapsed_time(b) for a, b in ev) / iters
            return {"tflops": c.flops / ms / 1e9, "ms": ms, "frac_of_bf16_peak": c.flops / ms / 1e9 / tf,
                    "backend": backend, "l2": "flushed", "note": "library reference for context; not this repo's kernel"}
        return run

    table = [
        ("prefill_cfg0_causal", prefill_cfg0),
        ("prefill_cfg1_varlen", prefill_cfg1),
        ("decode_cfg2", decode(dict(B=8, Hq=64, Hkv=16, L=1024, D=64), True)),
        ("decode_L4K", decode(dict(B=1, Hq=32, Hkv=8, L=4096, D=128), True)),
        ("decode_L32K", decode(dict(B=1, Hq=32, Hkv=8, L=32768, D=128), True)),
        ("decode_L128K", decode(dict(B=1, Hq=32, Hkv=8, L=131072, D=128), False)),
        ("sparse_cfg4_dense", sparse_dense),
        ("sparse_cfg4_paged", sparse_paged(False)),
        ("magicpig_cfg4_paged", sparse_paged(True)),
        ("sparse_128k_single_sequence", sparse_128k),
        ("sparse_128k_csr", sparse_128k_csr),
        ("append_paged_cfg0_kv", append_cfg0),
        ("mask_to_index_cfg4", mask_to_index(32000, 3840)),
        ("mask_to_index_128k", mask_to_index(131072, 4096)),
        ("context_torch_sdpa_cudnn_cfg0", torch_sdpa_cfg0("cudnn")),
        ("context_torch_sdpa_flash_cfg0", torch_sdpa_cfg0("flash")),
    ]
    out = {}
    for name, fn in table:
        if only is None or only == name:
            out[name] = fn()
            torch.cuda.empty_cache()
    return out


def kv_split_measurement(dev, pg, world, rank, steps=50, L=131072):
    """L-token single-sequence sparse decode (2 % kept per kv head) split along the
    key axis over all ranks: partial on each GPU, NCCL all-gather of [O | LSE], LSE
    merge; and the same with the exchange fused into the kernels (peer stores and
    flags, eager and as CUDA graphs).  ``single_gpu_ms`` is the whole sequence on
    rank 0's GPU in the same run (whole calls).  Every rank takes the same
    collective steps; times are the max over ranks."""
    from attention_kernel_triton_b200.distributed import shard_range, shard_sparse_lists, sparsetoken_decode_kv_split
    from attention_kernel_triton_b200.sparsetoken_decode_flash_attention_redundant import (
        sparsetoken_flash_attention_decode)
    L_max = 4096 if L == 131072 else int(L * 0.02 * 1.25) + 64
    c = W.make_sparse_dense(B=1, Hq=32, Hkv=8, L=L, D=128, keep_p=0.02, seed=12, device=dev, L_max=L_max)
    single = 0.0
    if rank == 0:
        single = _timed(lambda: sparsetoken_flash_attention_decode(c.q, c.K, c.V, c.sparse_ind, c.sparse_nnz,
                                                                   1.0 / math.sqrt(128), 4), steps, dev, None)
    single = _max_over_ranks(pg, dev, [single])[0]
    lo, hi = shard_range(L, world, rank)
    ind, nnz = shard_sparse_lists(c.sparse_ind, c.sparse_nnz, lo, hi)
    K, V = c.K[:, :, lo:hi].contiguous(), c.V[:, :, lo:hi].contiguous()
    total_bytes = c.bytes
    # the oracle's output on rank 0 (CPU, fp32), sent to every rank for its check
    ref = torch.zeros((1, 32, 1, 128), dtype=torch.float32, device=dev)
    if rank == 0:
        from oracle import naive as N  # checker only, outside the timed regions
        ref.copy_(N.sparsetoken_naive_decode(c.q.cpu(), c.K.cpu(), c.V.cpu(), c.sparse_ind.cpu(), c.sparse_nnz.cpu(),
                                             1.0 / math.sqrt(128), 4))
    if pg is not None:
        pg.broadcast(ref, 0)
    q_full = c.q.clone()
    del c

    def err_of(o):
        o = o.float()
        return float("inf") if bool(torch.isnan(o).any()) else float((o.reshape(ref.shape) - ref).abs().max())

    def step():
        return sparsetoken_decode_kv_split(q, K, V, ind, nnz, scale, 4)
    q = q_full
    scale = 1.0 / math.sqrt(128)
    for _ in range(3):
        step()
    pg.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize(dev)
    t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    ms = float(t[0])
    err_nccl = err_of(step())
    # the same split with the exchange fused into the kernels (NVLink peer stores + flags)
    from attention_kernel_triton_b200.distributed import PeerKVSplit
    x = PeerKVSplit(1, 32, 128, dev)
    try:
        x.bind(K, V, ind, nnz, scale, 4)
        for _ in range(3):
            x.step(q)
        pg.barrier()
        torch.cuda.synchronize(dev)
        e0.record()
        for _ in range(steps):
            x.step(q)
        e1.record()
        torch.cuda.synchronize(dev)
        tp = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
        pg.all_reduce(tp, op=pg.ReduceOp.MAX)
        err_peer = err_of(x.step(q))
        # and replayed as CUDA graphs (no per-step host launches)
        x.capture()
        for _ in range(3):
            x.step_graph(q)
        pg.barrier()
        torch.cuda.synchronize(dev)
        e0.record()
        for _ in range(steps):
            x.step_graph(q)
        e1.record()
        torch.cuda.synchronize(dev)
        tg = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
        pg.all_reduce(tg, op=pg.ReduceOp.MAX)
        err_graph = err_of(x.step_graph(q))
        torch.cuda.synchronize(dev)
    finally:
        x.close()
    ms_graph = float(tg[0])
    ms_peer = float(tp[0])
    errs = _max_over_ranks(pg, dev, [err_nccl, err_peer, err_graph])
    parity = {"kv_split_128k_nccl": errs[0], "kv_split_128k_peer": errs[1], "kv_split_128k_peer_graph": errs[2]}
    return {"seq_len": L, "gbs": total_bytes / ms / 1e6, "ms": ms, "n_gpus": world, "mb": total_bytes / 1e6,
            "single_gpu_ms": single, "allgather_bytes_per_rank": 32 * (128 + 1) * 4, "steps": steps,
            "peer_exchange": {"gbs": total_bytes / ms_peer / 1e6, "ms": ms_peer},
            "peer_exchange_graph": {"gbs": total_bytes / ms_graph / 1e6, "ms": ms_graph}}, parity


def run_ours(args):
    from attention_kernel_triton_b200 import _lib
    from attention_kernel_triton_b200.decode_flash_attention_redundant_var_len_paged import (
        decode_paged_into, flash_attention_decode_paged)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
        pg = dist

    c = W.make_paged(B=args.batch, seed=1000 + rank, device=dev)
    nbytes = c.bytes
    out = torch.empty((args.batch, 32, 128), dtype=torch.float16, device=dev)

    def step():
        decode_paged_into(out, c.q, c.cache, c.indptr, c.indices, c.last_page_len)

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()

    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with _lib.profile_kernels() as prof:
        ev0.record()
        for _ in range(args.steps):
            step()
        ev1.record()
        torch.cuda.synchronize(dev)
    barrier()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    kern_ms = prof.total_ms / max(prof.launches, 1)
    t = torch.tensor([ms, kern_ms], dtype=torch.float64, device=dev)
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    ms, kern_ms = float(t[0]), float(t[1])
    ms_step = ms / args.steps
    value = world * nbytes / (ms_step * 1e-3) / 1e9
    # parity of the timed output (the last step's) on two sampled sequences of this rank's batch
    parity = {"cfg3_weak_sampled": paged_parity(out, c, [rank % args.batch, int(torch.argmax(c.seq_lens))])}

    # e2e through the public API: per step, the step's inputs (q and the page
    # table) come from pinned host memory and the output goes back to host.
    # The KV pool is the resident cache state of the serving loop.  As a
    # serving loop does, the copies run on a side stream: step i+1's inputs
    # are uploaded (into the other of two device buffer sets) and step i's
    # output is read back while step i's or i+1's kernels run.  Every step's
    # copies are inside the timed region, which ends when the last output is
    # on the host.  Measured twice: issued eagerly from Python every step, and
    # with GRAPH_STEPS steps (their copies and public-API calls) captured once in
    # a CUDA graph and replayed, as a serving loop with fixed shapes does; the
    # graph takes the per-step host work (about 0.3 ms of Python and driver calls)
    # off the critical path when several ranks share the host's cores.
    h_q = c.q.cpu().pin_memory()
    h_indptr = c.indptr.cpu().pin_memory()
    h_indices = c.indices.cpu().pin_memory()
    h_last = c.last_page_len.cpu().pin_memory()
    h_out = torch.empty((args.batch, 32, 128), dtype=torch.float16).pin_memory()
    h2d = sum(x.numel() * x.element_size() for x in (h_q, h_indptr, h_indices, h_last))
    d2h = h_out.numel() * h_out.element_size()
    e2e_steps = max(3, args.steps)  # as many steps as the device-timed loop
    compute = torch.cuda.current_stream(dev)
    copier = torch.cuda.Stream(dev)
    hosts = (h_q, h_indptr, h_indices, h_last)
    bufs = [[torch.empty_like(x, device=dev) for x in hosts] for _ in range(2)]

    def run_steps(n, cs):
        """Issue n e2e steps on compute stream cs (the copier joins it first)."""
        copier.wait_stream(cs)
        uploaded = [torch.cuda.Event() for _ in range(2)]
        consumed = [None, None]  # event after the kernel that last read buffer set k
        outs = []

        def upload(i):
            k = i & 1
            with torch.cuda.stream(copier):
                if consumed[k] is not None:
                    copier.wait_event(consumed[k])
                for d, h in zip(bufs[k], hosts):
                    d.copy_(h, non_blocking=True)
                uploaded[k].record(copier)

        upload(0)
        for i in range(n):
            k = i & 1
            cs.wait_event(uploaded[k])
            O = flash_attention_decode_paged(*bufs[k][:1], c.cache, *bufs[k][1:])
            done = torch.cuda.Event()
            done.record(cs)
            consumed[k] = done
            if i + 1 < n:
                upload(i + 1)
            with torch.cuda.stream(copier):
                copier.wait_event(done)
                h_out.copy_(O, non_blocking=True)
            outs.append(O)  # kept alive until the copier has read it
        cs.wait_stream(copier)
        return outs

    def timed_e2e(issue, n):
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(compute)
        h0 = time.perf_counter()
        issue()
        e1.record(compute)
        host = (time.perf_counter() - h0) * 1e3 / n  # host time to issue one step (no waits inside)
        torch.cuda.synchronize(dev)
        return _max_over_ranks(pg, dev, [e0.elapsed_time(e1) / n, host])

    run_steps(3, compute)
    eager_ms, eager_host_ms = timed_e2e(lambda: run_steps(e2e_steps, compute), e2e_steps)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        graph_outs = run_steps(GRAPH_STEPS, torch.cuda.current_stream(dev))
    graph_reps = max(1, -(-e2e_steps // GRAPH_STEPS))
    for _ in range(2):
        graph.replay()

    def replay_all():
        for _ in range(graph_reps):
            graph.replay()
    e2e_ms, host_ms = timed_e2e(replay_all, graph_reps * GRAPH_STEPS)
    # the graph's last output equals the eager decode of the same inputs
    parity["cfg3_weak_e2e_graph_vs_eager"] = float((graph_outs[-1].float() - out.float()).abs().max())
    e2e_val = world * nbytes / (e2e_ms * 1e-3) / 1e9
    e2e_eager_val = world * nbytes / (eager_ms * 1e-3) / 1e9
    del graph, graph_outs

    peak, peak_kind = measured_peaks()
    achieved = nbytes / (kern_ms * 1e-3) / 1e9
    result = None
    secondary = None
    del c
    torch.cuda.empty_cache()
    strong = None
    if not args.no_strong:
        strong, p_strong = strong_scaling_measurements(dev, pg, world, rank)
        parity.update(p_strong)
    if world == 1 and not args.no_secondary:
        secondary = secondary_measurements(dev)
    elif world > 1 and not args.no_secondary:
        split, p_split = kv_split_measurement(dev, pg, world, rank)
        secondary = {"kv_split_128k": split}
        parity.update(p_split)
        # longer sequences: where the split starts to beat one GPU
        sweep = []
        for L in (524288, 2097152):
            torch.cuda.empty_cache()
            m, p_m = kv_split_measurement(dev, pg, world, rank, steps=30, L=L)
            sweep.append(m)
            parity.update({f"{k}_L{L}": v for k, v in p_m.items()})
        secondary["kv_split_sweep"] = sweep
    names = sorted(parity)
    vals = _max_over_ranks(pg, dev, [parity[k] for k in names])
    checks = dict(zip(names, vals))
    parity = {"tol": TOL, "max_abs": max(vals), "nan": any(v == float("inf") for v in vals),
              "pass": all(v <= TOL for v in vals), "checks": checks,
              "against": "CPU oracle (fp32 restatement of the reference's naive functions), sampled outputs of "
                         "the timed runs, max over ranks"}
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            sample, sbytes = make_cpu_sample(args.cpu_seqs)
            cpu_reference_step(sample, threads)
            reps = [cpu_reference_step(sample, threads) for _ in range(2)]
            cpu_t = statistics.mean(reps)
            cpu = {"value": sbytes / cpu_t / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
                   "sample": f"naive_paged_attention restated (oracle port), fp32 torch CPU, first "
                             f"{args.cpu_seqs} cfg3 sequences, mean of 2 runs"}
        cfg3_traffic = (CFG3_TRAFFIC_BYTES_CUDA_CORES
                        if os.environ.get("AKT_DECODE_TENSOR_CORES", "1").startswith("0") else CFG3_TRAFFIC_BYTES)
        result = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": WORKLOAD if args.batch == 64 else WORKLOAD.replace("B=64", f"B={args.batch}"),
                       "bytes_per_step_per_gpu": nbytes,
                       "l2": "inputs larger than L2 (4.4 GB pool per GPU), no flush",
                       "parallelism": f"independent batch per GPU x{world}"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": peak_kind,
                         # cfg3's pages (16 keys) take the tensor-core split-KV kernel unless it is
                         # switched off for the call's process
                         "kernel": ("decode_splitkv_kernel<half,128,4,paged>"
                                    if os.environ.get("AKT_DECODE_TENSOR_CORES", "1").startswith("0")
                                    else "decode_mma_kernel<half,128,4,paged>"),
                         "kernel_ms": kern_ms,
                         # dram__bytes_read.sum + dram__bytes_write.sum of one launch of this
                         # kernel on this workload (ncu; see CFG3_TRAFFIC_BYTES)
                         "traffic": cfg3_traffic if args.batch == 64 else None,
                         "traffic_over_algorithmic": cfg3_traffic / nbytes if args.batch == 64 else None},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms, "host_issue_ms_per_step": host_ms,
                    "method": f"public API calls and each step's copies captured in a CUDA graph of {GRAPH_STEPS} "
                              f"steps, replayed {graph_reps} times",
                    "eager": {"value": e2e_eager_val, "ms_per_step": eager_ms, "host_issue_ms_per_step": eager_host_ms,
                              "method": "the same steps issued from Python every step"}},
            "parity": parity,
            "gpu_launches": 3 * args.steps,  # planner, split-KV kernel and merge per step
            "clocks": clk,
        }
        if strong is not None:
            result["strong_scaling"] = strong
        if secondary is not None:
            result["secondary"] = secondary
        print(json.dumps(result), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seqs", type=int, default=4)
    ap.add_argument("--batch", type=int, default=64,
                    help="sequences per GPU (64 = cfg3; smaller only for profiler captures)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the other configurations (prefill, dense decode, sparse)")
    ap.add_argument("--no-strong", action="store_true",
                    help="skip the strong-scaling partitions of one cfg3 / cfg0 / cfg1 workload")
    ap.add_argument("--only", default=None,
                    help="run just one secondary configuration by name and print it (profiler captures)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.only:
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        print(json.dumps({args.only: secondary_measurements(dev, iters=args.steps, only=args.only)[args.only]}))
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
