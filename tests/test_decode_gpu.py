"""GPU parity of the dense and paged decode paths against the CPU oracle and
the reference's golden outputs.

Tolerance (the parity bar for fp16/bf16 outputs): max-abs <= 2e-3 against the fp32 oracle on
the same inputs, no NaNs.  For bf16 outputs the output rounding alone is up to
half a bf16 ulp (2^-9 relative), so bf16 cases allow ``2e-3 + 2^-8 * |ref|``.
"""
import math
import os

import pytest
import torch

from golden_io import load
from oracle import naive as N

from attention_kernel_triton_b200 import _lib
from attention_kernel_triton_b200 import workloads as W
from attention_kernel_triton_b200.decode_flash_attention_redundant import flash_attention_decode
from attention_kernel_triton_b200.decode_flash_attention_redundant_var_len_paged import (
    decode_paged_into, flash_attention_decode_paged)

pytestmark = pytest.mark.gpu
TOL = 2e-3
DEV = "cuda"


def check_close(out, ref, dtype=torch.float16):
    out = out.detach().float().cpu()
    ref = ref.detach().float().cpu()
    assert out.shape == ref.shape
    assert not torch.isnan(out).any()
    err = (out - ref).abs()
    if dtype == torch.bfloat16:
        bound = TOL + 2.0 ** -8 * ref.abs()
        assert bool((err <= bound).all()), f"max err {err.max().item()}"
    else:
        assert err.max().item() <= TOL, f"max err {err.max().item()}"


@pytest.fixture(autouse=True)
def device_status_clean():
    _lib.device_status(0, clear=True)
    yield
    assert _lib.device_status(0) == 0, "a kernel recorded an error"


def cuda(x):
    return x.to(DEV)


# ---------------------------------------------------------------- golden
@pytest.mark.parametrize("name", ["decode_dense", "decode_dense_d128"])
def test_dense_decode_matches_reference_golden(name):
    f = load(name)
    O = flash_attention_decode(cuda(f["q"]), cuda(f["K"]), cuda(f["V"]), f["softmax_scale"], f["group"])
    assert O.shape == f["O"].shape and O.dtype == torch.float16
    check_close(O, f["O"])
    check_close(O, N.decode_reference(f["q"], f["K"], f["V"], f["softmax_scale"], f["group"]))


@pytest.mark.parametrize("name", ["paged_ref_table", "paged_p16"])
def test_paged_decode_matches_reference_golden(name):
    f = load(name)
    O = flash_attention_decode_paged(cuda(f["q"]), cuda(f["cache"]), cuda(f["indptr"]), cuda(f["indices"]),
                                     cuda(f["last_page_len"]))
    assert O.shape == f["O"].shape
    check_close(O, f["O"])


# ---------------------------------------------------------------- dense decode, shapes
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("G", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("L", [1, 17, 1000])
def test_dense_decode_shapes(dtype, D, G, L):
    Hkv = 2
    c = W.make_decode(B=2, Hq=Hkv * G, Hkv=Hkv, L=L, D=D, seed=1000 + D + G + L, dtype=dtype)
    O = flash_attention_decode(cuda(c.q), cuda(c.K), cuda(c.V), c.softmax_scale, c.group)
    assert O.shape == (2, Hkv * G, 1, D) and O.dtype == dtype
    check_close(O, N.decode_reference(c.q, c.K, c.V, c.softmax_scale, c.group), dtype)


def test_dense_decode_cfg2_baseline_shape():
    c = W.make_decode(B=8, Hq=64, Hkv=16, L=1024, D=64, seed=2, device=DEV)
    O = flash_attention_decode(c.q, c.K, c.V, c.softmax_scale, c.group)
    check_close(O, N.decode_reference(c.q, c.K, c.V, c.softmax_scale, c.group))


@pytest.mark.parametrize("L", [4096, 32768, 131072])
def test_dense_decode_long_context_sweep(L):
    c = W.make_decode(B=1, Hq=32, Hkv=8, L=L, D=128, seed=3, device=DEV)
    O = flash_attention_decode(c.q, c.K, c.V, c.softmax_scale, c.group)
    check_close(O, N.decode_reference(c.q, c.K, c.V, c.softmax_scale, c.group))


def test_dense_decode_strided_inputs():
    c = W.make_decode(B=2, Hq=8, Hkv=2, L=300, D=128, seed=4)
    big_q = torch.randn(2, 8, 3, 128, dtype=torch.float16)
    big_q[:, :, 1:2] = c.q
    Kt = c.K.transpose(1, 2).contiguous().transpose(1, 2)  # [B,H,L,D] view with token-major storage
    O = flash_attention_decode(cuda(big_q)[:, :, 1:2], cuda(Kt), cuda(c.V), c.softmax_scale, c.group)
    check_close(O, N.decode_reference(c.q, c.K, c.V, c.softmax_scale, c.group))


def test_dense_decode_reference_asserts():
    q = torch.zeros(1, 4, 1, 96, dtype=torch.float16, device=DEV)
    K = torch.zeros(1, 2, 8, 96, dtype=torch.float16, device=DEV)
    with pytest.raises(AssertionError):
        flash_attention_decode(q, K, K, 0.1, 2)
    with pytest.raises(AssertionError):
        flash_attention_decode(q[:, :, :, :64], K[..., :64], K[..., :64], 0.1, 4)


# ---------------------------------------------------------------- paged decode
PAGED_LENS = [0, 1, 15, 16, 17, 33, 300, 2000]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("D,G", [(64, 1), (64, 4), (128, 2), (128, 4), (128, 8), (256, 4), (128, 16)])
@pytest.mark.parametrize("P", [16, 64])
def test_paged_decode_shapes(dtype, D, G, P):
    Hkv = 2
    c = W.make_paged(Hq=Hkv * G, Hkv=Hkv, D=D, page_size=P, lens=PAGED_LENS, seed=D * 7 + G + P, dtype=dtype)
    O = flash_attention_decode_paged(cuda(c.q), cuda(c.cache), cuda(c.indptr), cuda(c.indices),
                                     cuda(c.last_page_len))
    assert O.shape == (len(PAGED_LENS), Hkv * G, D) and O.dtype == dtype
    ref = N.naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.last_page_len)
    check_close(O, ref, dtype)
    assert torch.all(O[0] == 0)  # empty sequence -> zeros


def test_paged_decode_small_pages(monkeypatch):
    # page sizes below the reference's default tile need its env knob lowered (DP:255-257)
    monkeypatch.setenv("VAR_KV_SEQ_BLK_SIZE", "1")
    for P in (1, 3, 8):
        c = W.make_paged(Hq=8, Hkv=2, D=128, page_size=P, lens=[1, 5, 40, 77], seed=P)
        O = flash_attention_decode_paged(cuda(c.q), cuda(c.cache), cuda(c.indptr), cuda(c.indices),
                                         cuda(c.last_page_len))
        check_close(O, N.naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.last_page_len))


def test_paged_decode_reference_assert(monkeypatch):
    c = W.make_paged(Hq=4, Hkv=2, D=64, page_size=8, lens=[5], seed=1)
    with pytest.raises(AssertionError):
        flash_attention_decode_paged(cuda(c.q), cuda(c.cache), cuda(c.indptr), cuda(c.indices),
                                     cuda(c.last_page_len))


@pytest.mark.parametrize("D,P", [(128, 16), (64, 64), (256, 32)])
def test_paged_decode_nan_past_last_token(D, P):
    # The tensor-core kernel moves whole 16-key tiles of a page; the pool slots
    # past a sequence's last token are not the sequence's data and may hold
    # anything (here NaN, in K and V).  They must not reach the output.
    c = W.make_paged(Hq=8, Hkv=2, D=D, page_size=P, lens=[1, 17, P + 3, 5 * P - 1], seed=D + P)
    cache = c.cache.clone()
    for b in range(len(c.last_page_len)):
        s, e = int(c.indptr[b]), int(c.indptr[b + 1])
        last = int(c.last_page_len[b])
        if e > s and last < P:
            cache[int(c.indices[e - 1]), :, :, last:, :] = float("nan")
    O = flash_attention_decode_paged(cuda(c.q), cuda(cache), cuda(c.indptr), cuda(c.indices),
                                     cuda(c.last_page_len))
    check_close(O, N.naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.last_page_len))


def test_paged_decode_last_page_len_clamped():
    c = W.make_paged(Hq=4, Hkv=2, D=64, page_size=16, lens=[40, 16], seed=5)
    last = c.last_page_len.clone()
    last[0] = 99  # past the page: slicing semantics clamp to the page size
    O = flash_attention_decode_paged(cuda(c.q), cuda(c.cache), cuda(c.indptr), cuda(c.indices), cuda(last))
    check_close(O, N.naive_paged_attention(c.q, c.cache, c.indptr, c.indices, last))


def test_paged_decode_strided_pool_and_q():
    c = W.make_paged(Hq=8, Hkv=2, D=128, page_size=16, lens=[100, 7], seed=6)
    wide = torch.zeros(c.cache.shape[:-1] + (256,), dtype=torch.float16)
    wide[..., :128] = c.cache
    O = flash_attention_decode_paged(cuda(c.q).transpose(0, 1).contiguous().transpose(0, 1),
                                     cuda(wide)[..., :128], cuda(c.indptr), cuda(c.indices),
                                     cuda(c.last_page_len))
    check_close(O, N.naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.last_page_len))


def test_paged_decode_int64_metadata():
    c = W.make_paged(Hq=8, Hkv=2, D=64, page_size=16, lens=[50, 3], seed=7)
    O = flash_attention_decode_paged(cuda(c.q), cuda(c.cache), cuda(c.indptr).long(), cuda(c.indices).long(),
                                     cuda(c.last_page_len).long())
    check_close(O, N.naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.last_page_len))


def test_paged_decode_side_stream():
    c = W.make_paged(Hq=8, Hkv=2, D=128, page_size=16, lens=[500, 20, 1], seed=8, device=DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        O = flash_attention_decode_paged(c.q, c.cache, c.indptr, c.indices, c.last_page_len)
    s.synchronize()
    check_close(O, N.naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.last_page_len))


def test_paged_decode_out_of_pool_page_is_reported_not_faulted():
    c = W.make_paged(Hq=8, Hkv=2, D=128, page_size=16, lens=[64, 64], seed=9)
    bad = c.indices.clone()
    bad[1] = c.cache.shape[0] + 5  # sequence 0, second page: outside the pool
    O = flash_attention_decode_paged(cuda(c.q), cuda(c.cache), cuda(c.indptr), cuda(bad), cuda(c.last_page_len))
    torch.cuda.synchronize()
    assert _lib.device_status(0, clear=True) == 2
    ref = N.naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.last_page_len)
    check_close(O[1], ref[1])  # the other sequence is unaffected


def test_paged_decode_malformed_indptr_is_reported():
    c = W.make_paged(Hq=4, Hkv=2, D=64, page_size=16, lens=[40, 40], seed=10)
    ip = c.indptr.clone()
    ip[1] = ip[2] + 1  # sequence 1 would have a negative page count; sequence 0 runs past it
    O = flash_attention_decode_paged(cuda(c.q), cuda(c.cache), cuda(ip), cuda(c.indices), cuda(c.last_page_len))
    torch.cuda.synchronize()
    assert _lib.device_status(0, clear=True) == 4
    assert not torch.isnan(O).any()


@pytest.mark.parametrize("B", [300, 1100])
def test_paged_decode_many_sequences_both_chunk_orders(B):
    # up to 1024 sequences the planner puts every partial last chunk after all full
    # chunks (longest first); beyond that it keeps each sequence's chunks in place
    g = torch.Generator().manual_seed(B)
    lens = torch.randint(0, 3000, (B,), generator=g).tolist()
    lens[5] = 0
    c = W.make_paged(Hq=8, Hkv=2, D=128, page_size=16, lens=lens, seed=B, device=DEV)
    O = flash_attention_decode_paged(c.q, c.cache, c.indptr, c.indices, c.last_page_len)
    sample = [0, 5, 17, B // 2, B - 1]
    ref = N.naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.last_page_len, batches=sample)
    check_close(O[sample], ref[sample])
    assert not torch.isnan(O).any()


def test_paged_decode_overlapping_indptr_stays_inside_the_workspace():
    # indptr [0, n, 0, n]: sequence 1 runs backwards (malformed) and sequences 0 and 2 both
    # cover all n pages, so together they ask for about twice the chunks the workspace is
    # sized for (num_page_entries * P / chunk + B).  The planner drops the excess and records
    # the malformed indptr; nothing past the workspace is read (a NaN-filled guard follows it).
    import ctypes

    from attention_kernel_triton_b200.decode_flash_attention_redundant_var_len_paged import _paged_args
    one = W.make_paged(B=1, Hq=32, Hkv=8, D=128, page_size=16, lens=[16000], seed=12)
    n = one.indices.numel()
    q = torch.randn((3, 32, 1, 128), generator=torch.Generator().manual_seed(5)).half()
    indptr = torch.tensor([0, n, 0, n], dtype=torch.int32)
    last = torch.tensor([16, 16, 16], dtype=torch.int32)
    dq, dcache, dip, didx, dlast = cuda(q), cuda(one.cache), cuda(indptr), cuda(one.indices), cuda(last)
    out = torch.empty((3, 32, 128), dtype=torch.float16, device=DEV)
    a = _paged_args(dq, dcache, dip, didx, dlast, out, 1.0 / math.sqrt(128))
    L = _lib.lib()
    need = L.akt_decode_paged_workspace_size(ctypes.byref(a))
    ws = torch.full((2 * need // 4 + 64,), float("nan"), dtype=torch.float32, device=DEV)
    _lib.check(L.akt_decode_paged(ctypes.byref(a), ws.data_ptr(), need, _lib.stream_ptr(out.device)))
    torch.cuda.synchronize()
    assert _lib.device_status(0, clear=True) == 4
    assert not torch.isnan(out).any()
    assert torch.isnan(ws[(need + 3) // 4:]).all()  # the guard past the workspace is untouched
    assert torch.all(out[1] == 0)


# ---------------------------------------------------------------- cfg3 (B=64, lens U[512, 32768]), full size
@pytest.fixture(scope="module")
def cfg3():
    return W.make_paged(seed=0, device=DEV)


def test_paged_decode_cfg3_full_size_sampled(cfg3):
    c = cfg3
    O = flash_attention_decode_paged(c.q, c.cache, c.indptr, c.indices, c.last_page_len)
    assert O.shape == (64, 32, 128)
    assert not torch.isnan(O).any()
    lens = c.seq_lens.tolist()
    sample = sorted({int(torch.tensor(lens).argmin()), int(torch.tensor(lens).argmax()), 5, 37})
    ref = N.naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.last_page_len, batches=sample)
    check_close(O[sample], ref[sample])


def test_paged_decode_cfg3_page_permutation_invariance(cfg3):
    # moving pages to other physical slots (and the table with them) must give
    # bit-identical output: same tiles, same order, only addresses change
    c = cfg3
    O = flash_attention_decode_paged(c.q, c.cache, c.indptr, c.indices, c.last_page_len)
    g = torch.Generator(device=DEV).manual_seed(123)
    perm = torch.randperm(c.cache.shape[0], generator=g, device=DEV)
    cache2 = torch.empty_like(c.cache)
    cache2[perm] = c.cache
    idx2 = perm[c.indices.long()].to(torch.int32)
    O2 = flash_attention_decode_paged(c.q, cache2, c.indptr, idx2, c.last_page_len)
    assert torch.equal(O, O2)
    del cache2


def test_paged_decode_into_preallocated(cfg3):
    c = cfg3
    out = torch.empty((64, 32, 128), dtype=torch.float16, device=DEV)
    decode_paged_into(out, c.q, c.cache, c.indptr, c.indices, c.last_page_len)
    O = flash_attention_decode_paged(c.q, c.cache, c.indptr, c.indices, c.last_page_len)
    assert torch.equal(out, O)


_CUDA_CORE_SCRIPT = r"""
import sys, torch
sys.path.insert(0, ".")
sys.path.insert(0, "tests")
from oracle import naive as N
from attention_kernel_triton_b200 import _lib
from attention_kernel_triton_b200 import workloads as W
from attention_kernel_triton_b200.decode_flash_attention_redundant import flash_attention_decode
from attention_kernel_triton_b200.decode_flash_attention_redundant_var_len_paged import flash_attention_decode_paged
worst = 0.0
for D, G, L in [(64, 4, 1000), (128, 4, 4096), (128, 1, 17)]:
    c = W.make_decode(B=2, Hq=2 * G, Hkv=2, L=L, D=D, seed=D + G + L)
    O = flash_attention_decode(c.q.cuda(), c.K.cuda(), c.V.cuda(), c.softmax_scale, c.group)
    ref = N.decode_reference(c.q, c.K, c.V, c.softmax_scale, c.group)
    worst = max(worst, float((O.float().cpu() - ref.float()).abs().max()))
for D, G, P in [(128, 4, 16), (64, 2, 64)]:
    c = W.make_paged(Hq=2 * G, Hkv=2, D=D, page_size=P, lens=[0, 1, 17, 300, 2000], seed=D + P)
    O = flash_attention_decode_paged(c.q.cuda(), c.cache.cuda(), c.indptr.cuda(), c.indices.cuda(),
                                     c.last_page_len.cuda())
    ref = N.naive_paged_attention(c.q, c.cache, c.indptr, c.indices, c.last_page_len)
    worst = max(worst, float((O.float().cpu() - ref.float()).abs().max()))
torch.cuda.synchronize()
print("max_err", worst, "status", _lib.device_status(0))
sys.exit(0 if worst <= 2e-3 and _lib.device_status(0) == 0 else 1)
"""


def test_cuda_core_kernel_forced():
    # Dense calls and paged calls with 16-key-multiple pages take the
    # tensor-core kernel; AKT_DECODE_TENSOR_CORES=0 (read once per process)
    # forces the CUDA-core kernel, which otherwise serves only other page
    # sizes.  Run it in a child process against the oracle.
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, AKT_DECODE_TENSOR_CORES="0")
    r = subprocess.run([sys.executable, "-c", _CUDA_CORE_SCRIPT], cwd=root, env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
